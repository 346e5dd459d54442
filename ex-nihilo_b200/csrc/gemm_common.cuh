// gemm_common.cuh -- pieces shared by the tcgen05 GEMM kernels (gemm.cu, gemm_q8.cu): tile
// constants, the tile order, and the fused epilogues that drain a TMEM accumulator.
//
// The epilogues replace the reference's separate elementwise launches
// (src/cuda/dit.cu: x_gate_add :34-41, x_qk_norm_rope :43-58, x_swiglu2
// :186-192, x_gelu_tanh :194-199) and the host Euler update
// (src/generate.lisp:135) that followed illatio's GEMMs (src/cuda-dit.lisp
// :115-130).
#pragma once

#include "exn_device.cuh"
#include "exn_internal.h"

namespace exn {

int make_tmap(CUtensorMap* m, CUtensorMapDataType type, const void* base, int rank, const uint64_t* dims,
              const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle);
int make_tmap_bf16(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                   const uint32_t* box);

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int GEMM_THREADS = 192;

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr uint32_t IDESC = idesc_bf16(BM, BN);
};

__device__ __forceinline__ long long map_row(const GemmEpi& e, int r) {
  const int b = r / e.seg_in, t = r - b * e.seg_in;
  return static_cast<long long>(b) * e.seg_out + e.off + t + (t >= e.split_at ? e.split_gap : 0);
}

// Tiles run in groups of GM row blocks, all columns of a group before the
// next: a weight tile is read from HBM once per group while the group's
// activation rows stay in L2.
__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int GM, int& mb, int& nb) {
  const int group = tile / (GM * num_n);
  const int first = group * GM;
  const int gm = min(GM, num_m - first);
  const int in_g = tile - group * GM * num_n;
  mb = first + in_g % gm;
  nb = in_g / gm;
}

__device__ __forceinline__ float gelu_tanh(float v) {
  return 0.5f * v * (1.f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
}

__device__ __forceinline__ float silu(float g) { return g / (1.f + expf(-g)); }

__device__ __forceinline__ void store_bf16x32(bf16* dst, const float* v) {
  uint4* o = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    o[i] = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                      pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
}

// ----------------------------------------------------------------------------- epilogues
// TADDR: TMEM address of this warp's 32 lanes at the accumulator's column 0.
// ROW: this thread's GEMM row; VALID: row < M; COL0: the tile's first column.

template <int BN, int EPI>
__device__ __forceinline__ void epilogue(uint32_t taddr, int row, bool valid, int col0, const GemmEpi& e) {
  if constexpr (EPI == EPI_F32 || EPI == EPI_BF16 || EPI == EPI_GELU_BF16) {
    const long long orow = valid ? map_row(e, row) : 0;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + c, r);
      if (!valid) continue;
      float f[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(r[i]);
      if constexpr (EPI == EPI_F32) {
        float4* o = reinterpret_cast<float4*>(static_cast<float*>(e.out) + orow * e.ld_out + col0 + c);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = make_float4(f[4 * i], f[4 * i + 1], f[4 * i + 2], f[4 * i + 3]);
      } else {
        if constexpr (EPI == EPI_GELU_BF16) {
#pragma unroll
          for (int i = 0; i < 32; ++i) f[i] = gelu_tanh(f[i]);
        }
        store_bf16x32(static_cast<bf16*>(e.out) + orow * e.ld_out + col0 + c, f);
      }
    }
  } else if constexpr (EPI == EPI_I8_F32) {
    // s32 accumulators of an int8 product, scaled by A's row scale (e.mod) and B's row scales (e.norm_q)
    const float sr = valid ? __ldg(e.mod + row) : 0.f;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + c, r);
      if (!valid) continue;
      float4* o = reinterpret_cast<float4*>(static_cast<float*>(e.out) + static_cast<long long>(row) * e.ld_out + col0 + c);
      const float4* sc = reinterpret_cast<const float4*>(e.norm_q + col0 + c);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 s4 = __ldg(sc + i);
        o[i] = make_float4(__int2float_rn(static_cast<int>(r[4 * i])) * sr * s4.x,
                           __int2float_rn(static_cast<int>(r[4 * i + 1])) * sr * s4.y,
                           __int2float_rn(static_cast<int>(r[4 * i + 2])) * sr * s4.z,
                           __int2float_rn(static_cast<int>(r[4 * i + 3])) * sr * s4.w);
      }
    }
  } else if constexpr (EPI == EPI_GATE_RESID) {
    const int t = row % e.seg_in;
    const float* g = e.mod + (e.n0 + t < e.p ? e.mod_stride : 0) + col0;
    float* x = static_cast<float*>(e.out) + static_cast<long long>(row) * e.ld_out + col0;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + c, r);
      if (!valid) continue;
      float4* xp = reinterpret_cast<float4*>(x + c);
      const float4* gp = reinterpret_cast<const float4*>(g + c);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float4 xv = xp[i];
        const float4 gv = __ldg(gp + i);
        xv.x += gv.x * __uint_as_float(r[4 * i]);
        xv.y += gv.y * __uint_as_float(r[4 * i + 1]);
        xv.z += gv.z * __uint_as_float(r[4 * i + 2]);
        xv.w += gv.w * __uint_as_float(r[4 * i + 3]);
        xp[i] = xv;
      }
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    static_assert(BN == 256, "SwiGLU tiles hold 128 gate and 128 up columns");
    bf16* o = static_cast<bf16*>(e.out) + static_cast<long long>(row) * e.ld_out + col0 / 2;
#pragma unroll 1
    for (int c = 0; c < 128; c += 32) {
      uint32_t rg[32], ru[32];
      tmem_ld32(taddr + c, rg);
      tmem_ld32(taddr + 128 + c, ru);
      if (!valid) continue;
      float f[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) f[i] = silu(__uint_as_float(rg[i])) * __uint_as_float(ru[i]);
      store_bf16x32(o + c, f);
    }
  } else if constexpr (EPI == EPI_QKV) {
    static_assert(BN == 256, "QKV tiles hold two whole heads");
    const int kvw = e.kv_width > 0 ? e.kv_width : e.width;
    const int sec = col0 < e.width ? 0 : 1 + (col0 - e.width) / kvw;        // 0 q, 1 k, 2 v
    const int hc0 = sec == 0 ? col0 : col0 - e.width - (sec - 1) * kvw;     // first column within q / k / v
    const int t = row % e.seg_in, b = row / e.seg_in;
    bf16* dst;
    if (e.group_w > 0) {  // sequence-parallel: straight into the rank that keeps this head group
      const int g = hc0 / e.group_w, cg = hc0 % e.group_w;
      long long qrow, kvrow;
      if (row < e.sp_pl_loc) {
        qrow = kvrow = static_cast<long long>(e.sp_rank) * e.sp_pl + row;
      } else {
        const long long i = static_cast<long long>(e.sp_rank) * e.sp_nl + (row - e.sp_pl_loc);
        qrow = e.sp_img0 + i;
        kvrow = e.sp_p + i;
      }
      dst = sec == 0 ? e.sp_q[g] + qrow * e.group_w + cg : (sec == 1 ? e.sp_k[g] : e.sp_v[g]) + kvrow * e.group_w + cg;
    } else if (sec == 0)
      dst = e.q + static_cast<long long>(row) * e.width + hc0;
    else
      dst = (sec == 1 ? e.k : e.v) + b * e.kv_sample_stride + static_cast<long long>(e.n0 + t) * kvw + hc0;
    const float* nw = sec == 0 ? e.norm_q : e.norm_k;
    const float2* cs = e.rope + static_cast<long long>(e.n0 + t) * 64;
#pragma unroll 1
    for (int hh = 0; hh < 2; ++hh) {
      float v[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(taddr + hh * 128 + c * 32, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[c * 32 + i] = __uint_as_float(r[i]);
      }
      if (!valid) continue;
      if (sec < 2) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 128; ++i) ss += v[i] * v[i];
        const float inv = rsqrtf(ss / 128.f + 1e-6f);
        if (e.rope_halves) {  // dims j and j + 64 turn together (rotate-half form)
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const float a = v[j] * inv * __ldg(nw + j);
            const float bq = v[j + 64] * inv * __ldg(nw + j + 64);
            const float2 r = __ldg(cs + j);
            v[j] = a * r.x - bq * r.y;
            v[j + 64] = a * r.y + bq * r.x;
          }
        } else {              // dims 2j and 2j + 1 turn together (complex-pair form)
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const float a = v[2 * j] * inv * __ldg(nw + 2 * j);
            const float bq = v[2 * j + 1] * inv * __ldg(nw + 2 * j + 1);
            const float2 r = __ldg(cs + j);
            v[2 * j] = a * r.x - bq * r.y;
            v[2 * j + 1] = a * r.y + bq * r.x;
          }
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) store_bf16x32(dst + hh * 128 + c * 32, v + c * 32);
    }
    if (e.group_w > 0) __threadfence_system();  // peer stores performed before the pass's barrier
  } else if constexpr (EPI == EPI_PROJ) {
    static_assert(BN == 64, "proj_out has the latent's 64 channels");
    const int b = row / e.nimg, i = row - (row / e.nimg) * e.nimg;
    const int zs = e.zstride > 0 ? e.zstride : e.nimg;
    const long long base = static_cast<long long>(b) * 64 * zs + i;
#pragma unroll 1
    for (int c = 0; c < 64; c += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + c, r);
      if (!valid) continue;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const long long idx = base + static_cast<long long>(c + j) * zs;
        const float val = __uint_as_float(r[j]);
        if (e.vout) e.vout[idx] = val;
        if (e.z) e.z[idx] += e.dsigma * val;
      }
    }
  }
}

}  // namespace exn
