// attention.cu -- the DiT's masked attention on the 5th-generation tensor
// cores, head dim 128.
//
// Semantics of src/cuda/dit.cu:60-66 (xa_lim) and :208-336 (x_attend_mma):
// query row g of the sequence sees keys 0 .. lim(g), with lim(g) = L-1 for
// image rows (g >= p), b1-1 for a reference picture's rows (b0 <= g < b1)
// and g otherwise (the prompt is causal); softmax(q k^T / sqrt(128)) v.
// Queries of one pass are sequence rows q0 .. q0+nq-1 (q0 = the cached
// prefix length on steps 2-8), keys rows 0 .. L-1 of the layer's K/V, whose
// prefix rows persist from the first step (no copy, unlike
// src/cuda-dit.lisp:207-218).
//
// One CTA = one (sample, head) and two tiles of 128 queries (a, b) that
// share every K/V tile:
//   warp 0      TMA: Q_a, Q_b once; K_j, V_j (128 keys x 128 dims, bf16)
//   warp 1      tcgen05.mma: S_x = Q_x K_j^T into TMEM, O_x += P_x V_j
//   warps 2..5  softmax of tile a, warps 6..9 of tile b: one query row per
//               thread straight from TMEM (32x32b loads); P_x (bf16, two per
//               column) written back into TMEM over the first 64 columns of
//               S_x and fed to the PV MMA from there (A operand in TMEM); O_x
//               rescaled in TMEM only when the row maximum grows by more
//               than 2^8
// The MMA order PV_a(j), S_a(j+1), PV_b(j), S_b(j+1) lets one tile's softmax
// run while the tensor core serves the other.
#include <stdlib.h>

#include "exn_device.cuh"
#include "exn_internal.h"

namespace exn {

int make_tmap_bf16(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                   const uint32_t* box);

namespace {

constexpr int ATT_THREADS = 320;
constexpr int TILE = 128;                 // queries per tile, keys per K/V tile
constexpr int HALF = TILE * 128;          // bytes of one 64-column swizzled half of a 128 x 128 bf16 tile
constexpr int TILE_BYTES = 2 * HALF;      // 32 KB
// K_0 V_0 K_1 V_1 ... stream through a ring of 4 tile slots, so each load has
// a slot free well before its MMA needs it.
constexpr int SLOTS = 4;
constexpr int OFF_QA = 0, OFF_QB = TILE_BYTES, OFF_SLOT = 2 * TILE_BYTES, OFF_BAR = (2 + SLOTS) * TILE_BYTES;
constexpr int ATT_SMEM = OFF_BAR + 256 + 1024;
constexpr uint32_t IDESC_S = idesc_bf16(128, 128);
constexpr uint32_t IDESC_PV = idesc_bf16(128, 128, false, true);  // V is MN-major (dims contiguous)
constexpr float RESCALE_THRESHOLD = 8.0f;                          // log2 units

// 2^x on the FMA and integer pipes, for x <= 8: Cody-Waite split x = n + f,
// n = round(x) by the 1.5 * 2^23 magic add, f in [-1/2, 1/2]; 2^f by a
// degree-3 polynomial fitted to 2^f on that interval (Lawson-weighted least
// squares, max relative error 7.5e-5, far under bf16's 2^-9 rounding of P);
// 2^n added into the exponent field; below 2^-126 (masked keys) exactly 0.
// The MUFU pipe gives 16 ex2 a clock per SM; computing a share of each row
// here lets the FMA pipes carry part of the softmax's exponentials.
__device__ __forceinline__ float exp2_fma(float x) {
  const float xc = fmaxf(x, -126.f);
  const float t = __fadd_rn(xc, 12582912.f);
  const float f = __fsub_rn(xc, __fsub_rn(t, 12582912.f));
  const float p = fmaf(fmaf(fmaf(0.0551716685f, f, 0.24261114f), f, 0.69326097f), f, 0.99992806f);
  return x > -126.f ? __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23)) : 0.f;
}

__device__ __forceinline__ int xa_lim(int g, int p, int l, int b0, int b1) {
  return g >= p ? l - 1 : (g >= b0 && g < b1 ? b1 - 1 : g);
}

struct Bars {
  uint64_t q_full, slot_full[SLOTS], slot_empty[SLOTS];
  uint64_t s_full[2], p_full[2], o_full[2];
  uint64_t done;
  uint32_t tmem_slot;
  int abort_flag;
};

}  // namespace

template <int POLY>  // of each 8 exponentials of a row, POLY are computed by exp2_fma
__global__ void __launch_bounds__(ATT_THREADS, 1)
    k_attention(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, bf16* __restrict__ out, int nq, int q0, int p, int l,
                int b0, int b1, int width, float scale_log2, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + OFF_BAR);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, head = blockIdx.y, sample = blockIdx.z;
  const int qlast = min(nq, (qt + 1) * 2 * TILE) - 1;
  const int last_key = xa_lim(q0 + qlast, p, l, b0, b1);
  const int nkv = last_key / TILE + 1;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int i = 0; i < SLOTS; ++i) {
      mbar_init(&bars->slot_full[i], 1);
      mbar_init(&bars->slot_empty[i], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars->s_full[x], 1);
      mbar_init(&bars->p_full[x], 4);
      mbar_init(&bars->o_full[x], 1);
    }
    mbar_init(&bars->done, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;
  // TMEM columns: S_a [0,128), S_b [128,256), O_a [256,384), O_b [384,512)

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch(&tmQ);
      tma_prefetch(&tmK);
      tma_prefetch(&tmV);
      const int hx = head * 128;
      mbar_arrive_expect_tx(&bars->q_full, 2 * TILE_BYTES);
      for (int x = 0; x < 2; ++x)
        for (int hf = 0; hf < 2; ++hf)
          tma_load_3d(smem + (x ? OFF_QB : OFF_QA) + hf * HALF, &tmQ, &bars->q_full, hx + hf * 64,
                      qt * 2 * TILE + x * TILE, sample);
      // load number t: K_{t/2} for even t, V_{t/2} for odd t; slot t % 3, its (t / 3)-th use
      int issued = 0;
      for (int t = 0; t < 2 * nkv; ++t) {
        const int slot = t % SLOTS;
        const uint32_t use = static_cast<uint32_t>(t / SLOTS);
        if (!mbar_wait(&bars->slot_empty[slot], (use & 1) ^ 1, abort_flag, status, STATUS_TIMEOUT_ATTN)) break;
        mbar_arrive_expect_tx(&bars->slot_full[slot], TILE_BYTES);
        const CUtensorMap* map = (t & 1) ? &tmV : &tmK;
        for (int hf = 0; hf < 2; ++hf)
          tma_load_3d(smem + OFF_SLOT + slot * TILE_BYTES + hf * HALF, map, &bars->slot_full[slot], hx + hf * 64,
                      (t >> 1) * TILE, sample);
        issued = t + 1;
      }
      if (*abort_flag) {  // the copies in flight land before the CTA leaves
        volatile int no_abort = 0;
        mbar_wait(&bars->q_full, 0, &no_abort, nullptr, 0);
        for (int t = issued - SLOTS < 0 ? 0 : issued - SLOTS; t < issued; ++t)
          mbar_wait(&bars->slot_full[t % SLOTS], static_cast<uint32_t>(t / SLOTS) & 1, &no_abort, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // descriptors formed once; start addresses then advance in 16-byte units
      const uint64_t dq_a = sdesc_sw128(smem_u32(smem + OFF_QA), 16, 1024);
      const uint64_t dq_b = sdesc_sw128(smem_u32(smem + OFF_QB), 16, 1024);
      const uint64_t dk0 = sdesc_sw128(smem_u32(smem + OFF_SLOT), 16, 1024);     // keys x dims, K-major
      const uint64_t dv0 = sdesc_sw128(smem_u32(smem + OFF_SLOT), HALF, 1024);   // keys x dims read MN-major
      const uint32_t slot0 = smem_u32(smem + OFF_SLOT);
      auto issue_s = [&](uint64_t dq, uint32_t k_addr, uint32_t d) {
        const uint64_t dk = dk0 + static_cast<uint64_t>((k_addr - slot0) >> 4);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t o = static_cast<uint64_t>(((kk >> 2) * HALF + (kk & 3) * 32) >> 4);
          umma_ss(d, dq + o, dk + o, IDESC_S, kk ? 1u : 0u);
        }
      };
      // O_x += P_x V: P_x in TMEM at S_x's columns (8 columns = 16 keys per instruction)
      auto issue_pv = [&](uint32_t p_tmem, uint32_t v_addr, uint32_t d, bool acc) {
        const uint64_t dv = dv0 + static_cast<uint64_t>((v_addr - slot0) >> 4);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts(d, p_tmem + kk * 8, dv + static_cast<uint64_t>((kk * 2048) >> 4), IDESC_PV, (acc || kk) ? 1u : 0u);
      };
      // wait for load T (K_{T/2} or V_{T/2}); its slot's address
      auto wait_load = [&](int t, uint32_t& addr) -> bool {
        const int slot = t % SLOTS;
        addr = slot0 + slot * TILE_BYTES;
        return mbar_wait(&bars->slot_full[slot], static_cast<uint32_t>(t / SLOTS) & 1, abort_flag, status,
                         STATUS_TIMEOUT_ATTN);
      };
      uint32_t k_addr = 0, v_addr = 0;
      bool ok = mbar_wait(&bars->q_full, 0, abort_flag, status, STATUS_TIMEOUT_ATTN) && wait_load(0, k_addr);
      if (ok) {
        tc_fence_after();
        issue_s(dq_a, k_addr, tmem + 0);
        umma_commit(&bars->s_full[0]);
        issue_s(dq_b, k_addr, tmem + 128);
        umma_commit(&bars->s_full[1]);
        umma_commit(&bars->slot_empty[0]);
      }
      for (int j = 0; j < nkv && ok; ++j) {
        const uint32_t par = j & 1;
        const bool more = j + 1 < nkv;
        if (!(ok = wait_load(2 * j + 1, v_addr))) break;
        if (!(ok = mbar_wait(&bars->p_full[0], par, abort_flag, status, STATUS_TIMEOUT_ATTN))) break;
        tc_fence_after();
        issue_pv(tmem + 0, v_addr, tmem + 256, j > 0);
        if (!more) umma_commit(&bars->o_full[0]);
        if (more) {
          if (!(ok = wait_load(2 * j + 2, k_addr))) break;
          tc_fence_after();
          issue_s(dq_a, k_addr, tmem + 0);
          umma_commit(&bars->s_full[0]);
        }
        if (!(ok = mbar_wait(&bars->p_full[1], par, abort_flag, status, STATUS_TIMEOUT_ATTN))) break;
        tc_fence_after();
        issue_pv(tmem + 128, v_addr, tmem + 384, j > 0);
        umma_commit(&bars->slot_empty[(2 * j + 1) % SLOTS]);
        if (!more) umma_commit(&bars->o_full[1]);
        if (more) {
          issue_s(dq_b, k_addr, tmem + 128);
          umma_commit(&bars->s_full[1]);
          umma_commit(&bars->slot_empty[(2 * j + 2) % SLOTS]);
        }
      }
      umma_commit(&bars->done);
      volatile int no_abort = 0;
      mbar_wait(&bars->done, 0, &no_abort, nullptr, 0);
    }
  } else {
    // ---- softmax: tile x, TMEM lane quarter wq, query row r of the tile
    const int x = (warp - 2) >> 2;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const int qi = qt * 2 * TILE + x * TILE + r;  // query index within the pass
    const int lim = xa_lim(q0 + qi, p, l, b0, b1);
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + x * 128;
    const uint32_t o_addr = tmem + lane_off + 256 + x * 128;
    float m = -INFINITY, lsum = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      if (!mbar_wait_warp(&bars->s_full[x], j & 1, abort_flag, status, STATUS_TIMEOUT_ATTN)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[128];
      {
        uint32_t rr[128];
        tmem_ld128(s_addr, rr);
#pragma unroll
        for (int i = 0; i < 128; ++i) s[i] = __uint_as_float(rr[i]);
      }
      const int key0 = j * TILE;
      if (key0 + TILE - 1 > lim) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (key0 + c > lim) s[c] = -INFINITY;
      }
      // row maximum as an 8-way tree (a serial chain of 128 would cost its latency every tile)
      float m8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) m8[i] = s[i];
#pragma unroll
      for (int c = 8; c < 128; c += 8)
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = fmaxf(m8[i], s[c + i]);
      const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
      const float m_new = fmaxf(m, mx * scale_log2);
      const bool need = m_new > m + RESCALE_THRESHOLD;
      float alpha = 1.f;
      if (need) {
        alpha = fast_exp2(m - m_new);
        lsum *= alpha;
        m = m_new;
      }
      if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t rr[32];
          tmem_ld32(o_addr + c * 32, rr);
#pragma unroll
          for (int i = 0; i < 32; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * alpha);
          tmem_st32(o_addr + c * 32, rr);
        }
        tmem_st_wait();
      }
      float ps8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint32_t pk[64];  // P as bf16 pairs: key 2c and 2c+1 in column c
#pragma unroll
      for (int c16 = 0; c16 < 16; ++c16) {
        float e[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float xv = fmaf(s[c16 * 8 + i], scale_log2, -m);
          e[i] = i >= 8 - POLY ? exp2_fma(xv) : fast_exp2(xv);
          ps8[i] += e[i];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) pk[c16 * 4 + i] = pack_bf16x2(e[2 * i], e[2 * i + 1]);
      }
      lsum += ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
      {
        uint32_t half0[32], half1[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          half0[i] = pk[i];
          half1[i] = pk[32 + i];
        }
        tmem_st32(s_addr, half0);
        tmem_st32(s_addr + 32, half1);
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[x]);
    }
    if (ok && mbar_wait_warp(&bars->o_full[x], 0, abort_flag, status, STATUS_TIMEOUT_ATTN)) {
      tc_fence_after();
      const float inv = 1.f / lsum;
      bf16* dst = out + (static_cast<long long>(sample) * nq + qi) * width + head * 128;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t rr[32];
        tmem_ld32(o_addr + c * 32, rr);
        if (qi < nq) {
          uint4* o = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            o[i] = make_uint4(pack_bf16x2(__uint_as_float(rr[8 * i]) * inv, __uint_as_float(rr[8 * i + 1]) * inv),
                              pack_bf16x2(__uint_as_float(rr[8 * i + 2]) * inv, __uint_as_float(rr[8 * i + 3]) * inv),
                              pack_bf16x2(__uint_as_float(rr[8 * i + 4]) * inv, __uint_as_float(rr[8 * i + 5]) * inv),
                              pack_bf16x2(__uint_as_float(rr[8 * i + 6]) * inv, __uint_as_float(rr[8 * i + 7]) * inv));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int attention_launch(const AttnArgs& a, int* d_status, cudaStream_t st) {
  if (a.nq <= 0 || a.l <= 0 || a.width % 128 || a.heads * 128 != a.width || a.kv_rows < a.l) return -1;
  if (a.q0 + a.nq > a.l) return -1;
  static int poly = -1;  // EXN_ATTN_POLY: exponentials of each 8 on the FMA pipes (0, 1, 2 or 3)
  if (poly < 0) {
    const char* e = getenv("EXN_ATTN_POLY");
    const int v = e ? atoi(e) : 0;
    if (cudaFuncSetAttribute(k_attention<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(k_attention<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(k_attention<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(k_attention<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM) != cudaSuccess)
      return -3;
    poly = v < 0 || v > 3 ? 0 : v;
  }
  CUtensorMap tq, tk, tv;
  const uint32_t box[3] = {64, TILE, 1};
  const uint64_t dq[3] = {static_cast<uint64_t>(a.width), static_cast<uint64_t>(a.nq),
                          static_cast<uint64_t>(a.batch)};
  const uint64_t sq[2] = {static_cast<uint64_t>(a.width) * 2, static_cast<uint64_t>(a.nq) * a.width * 2};
  const uint64_t dk[3] = {static_cast<uint64_t>(a.width), static_cast<uint64_t>(a.l), static_cast<uint64_t>(a.batch)};
  const uint64_t sk[2] = {static_cast<uint64_t>(a.width) * 2, static_cast<uint64_t>(a.kv_rows) * a.width * 2};
  if (make_tmap_bf16(&tq, a.q, 3, dq, sq, box) || make_tmap_bf16(&tk, a.k, 3, dk, sk, box) ||
      make_tmap_bf16(&tv, a.v, 3, dk, sk, box))
    return -4;
  dim3 grid((a.nq + 2 * TILE - 1) / (2 * TILE), a.heads, a.batch);
  auto kern = poly == 0 ? k_attention<0> : poly == 1 ? k_attention<1> : poly == 2 ? k_attention<2> : k_attention<3>;
  kern<<<grid, ATT_THREADS, ATT_SMEM, st>>>(tq, tk, tv, a.out, a.nq, a.q0, a.p, a.l, a.b0, a.b1, a.width,
                                            a.scale_log2, d_status);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace exn
