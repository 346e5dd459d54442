// conv.cu -- the VAE decoder's convolutions on the 5th-generation tensor cores:
// implicit GEMM over channels-last (NHWC) bf16 pictures, fp32 accumulation in
// TMEM.  The reference runs them as fp32 SIMT kernels (src/cuda/vae.cu: x_conv3
// :23-69 for 3 x 3, illatio's d41_mm_f32 for 1 x 1; src/cuda-vae.lisp:37-60).
//
// C[pixel][o] = bias[o] + sum over taps (dy, dx) and channels c of
//   X[y + dy - 1][x + dx - 1][c] W[o][dy][dx][c]
// (zero outside the picture: "same" padding, stride 1).  One persistent CTA per
// SM walks tiles of 128 pixels x BN output channels.  For a 3 x 3 convolution
// the k loop runs over (tap, 64-channel block); the TMA producer loads each
// block as a box of the picture shifted by the tap, so the A tile is the
// im2col rows without materialising them, and the tensor map's zero fill is
// the padding.  A tile is a block of 128 pixels, bw columns by 128 / bw rows,
// bw the largest divisor of the width that divides 128 (a row segment of 128
// pixels when the width is a multiple of 128).  Channels are
// padded to a multiple of 64 (the activations' and the weights' padding is
// zero), output channels come in tiles of BN (144 divides every width of the
// decoder: 144, 288, 576, 1152).  The 144-channel tiles run on CTA pairs
// (k_conv2, M = 256: two pixel tiles, each CTA half the weight block); the
// latent's 64 channels and the RGBA head on one CTA (k_conv).
//
//   warp 0      TMA producer (A shifted picture boxes, B weight blocks)
//   warp 1      MMA issuer: tcgen05.mma kind::f16, M = 128 (pairs: 256), N = BN, K = 16
//   warps 2..5  epilogue: bias, the residual, fp32 or bf16 out, or the RGBA head
#include "gemm_common.cuh"

namespace exn {

template <int BN>
struct ConvCfg {
  static constexpr int A_BYTES = BM * BK * 2;  // 128 pixels x 64 channels
  static constexpr int B_BYTES = BN * BK * 2;  // BN output channels x 64 channels
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 8 ? 8 : (200 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN <= 32 ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr uint32_t IDESC = idesc_bf16(BM, BN);
};

// TMEM -> the output of tile (pixel ROW, columns COL0 ..): 16 columns at a time
template <int BN, int EPI>
__device__ __forceinline__ void conv_epilogue(uint32_t taddr, int row, bool valid, int col0, const ConvEpi& e) {
#pragma unroll 1
  for (int c = 0; c < BN; c += 16) {
    uint32_t r[16];
    tmem_ld16(taddr + c, r);
    if (!valid) continue;
    const int col = col0 + c;
    if (col >= e.cout) continue;
    float v[16];
    const float4* bp = reinterpret_cast<const float4*>(e.bias + col);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 b = __ldg(bp + i);
      v[4 * i] = __uint_as_float(r[4 * i]) + b.x;
      v[4 * i + 1] = __uint_as_float(r[4 * i + 1]) + b.y;
      v[4 * i + 2] = __uint_as_float(r[4 * i + 2]) + b.z;
      v[4 * i + 3] = __uint_as_float(r[4 * i + 3]) + b.w;
    }
    if constexpr (EPI == CONV_F32) {
      if (e.res) {
        const float4* rp = reinterpret_cast<const float4*>(e.res + static_cast<long long>(row) * e.ld_res + col);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 x = rp[i];
          v[4 * i] += x.x;
          v[4 * i + 1] += x.y;
          v[4 * i + 2] += x.z;
          v[4 * i + 3] += x.w;
        }
      }
      if (e.dup) {  // DupUp3D (ref_vae.py:77-83): output channel o of sub-pixel (sy, sx) repeats
                    // input channel f / rep, f = ((o ft + ft - 1) 2 + sy) 2 + sx, rep = 4 cout ft / ci
        const int y = row / e.out_w, x = row - y * e.out_w, sy = y & 1, sx = x & 1;
        const int rep = 4 * e.cout * e.dup_ft / e.dup_ci;
        const float* src = e.dup + (static_cast<long long>(y >> 1) * (e.out_w >> 1) + (x >> 1)) * e.dup_ci;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int f = (((col + i) * e.dup_ft + e.dup_ft - 1) * 2 + sy) * 2 + sx;
          v[i] += __ldg(src + f / rep);
        }
      }
      float4* o = reinterpret_cast<float4*>(static_cast<float*>(e.out) + static_cast<long long>(row) * e.ld_out + col);
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else if constexpr (EPI == CONV_BF16) {
      uint4* o = reinterpret_cast<uint4*>(static_cast<bf16*>(e.out) + static_cast<long long>(row) * e.ld_out + col);
      o[0] = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                        pack_bf16x2(v[6], v[7]));
      o[1] = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]), pack_bf16x2(v[12], v[13]),
                        pack_bf16x2(v[14], v[15]));
    } else {  // CONV_RGBA: the head's first 4 channels, clamped to -1 .. 1
      float* o = static_cast<float*>(e.out) + static_cast<long long>(row) * 4;
      *reinterpret_cast<float4*>(o) = make_float4(fminf(fmaxf(v[0], -1.f), 1.f), fminf(fmaxf(v[1], -1.f), 1.f),
                                                  fminf(fmaxf(v[2], -1.f), 1.f), fminf(fmaxf(v[3], -1.f), 1.f));
    }
  }
}

// TAPS 9: A is the picture [h][w][cp] (3-D map, box {64, wt, ht}); TAPS 1: A is [pixels][cp]
template <int BN, int EPI, int TAPS>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_conv(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int h, int w, int bw,
           int cp, int cout_tiles, const ConvEpi ep, int* status) {
  using C = ConvCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // pixel tiles: blocks of bw columns x 128 / bw rows of the h x w picture, row-major over the picture
  const int bh = BM / bw, tiles_x = (w + bw - 1) / bw;
  const int num_m = tiles_x * ((h + bh - 1) / bh);
  const int num_tiles = num_m * cout_tiles;
  const int cblocks = cp / BK;
  const int num_kb = TAPS * cblocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      griddep_wait();
      int stage = 0;
      uint32_t phase = 0;
      int last_phase[C::STAGES];
#pragma unroll
      for (int s = 0; s < C::STAGES; ++s) last_phase[s] = -1;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mb = tile % num_m, nb = tile / num_m;  // pixel tiles fastest: a weight block stays in L2
        const int y0 = (mb / tiles_x) * bh, x0 = (mb % tiles_x) * bw;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, status, STATUS_TIMEOUT_GEMM)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          const int tap = kb / cblocks, cb = kb - tap * cblocks;
          if constexpr (TAPS == 9)
            tma_load_3d(sA + stage * C::A_BYTES, &tmA, &full[stage], cb * BK, x0 + tap % 3 - 1, y0 + tap / 3 - 1);
          else
            tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], cb * BK, x0);
          tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * BK, nb * BN);
          last_phase[stage] = static_cast<int>(phase);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {  // the copies already issued land before the CTA leaves (bounded waits)
        volatile int no_abort = 0;
        for (int s = 0; s < C::STAGES; ++s)
          if (last_phase[s] >= 0) mbar_wait(&full[s], static_cast<uint32_t>(last_phase[s]), &no_abort, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      const uint64_t a_desc0 = sdesc_sw128(smem_u32(sA), 16, 1024);
      const uint64_t b_desc0 = sdesc_sw128(smem_u32(sB), 16, 1024);
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, status, STATUS_TIMEOUT_GEMM)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, status, STATUS_TIMEOUT_GEMM)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = a_desc0 + static_cast<uint64_t>((stage * C::A_BYTES) >> 4);
          const uint64_t bd = b_desc0 + static_cast<uint64_t>((stage * C::B_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) umma_ss(d_tmem, ad + 2 * k, bd + 2 * k, C::IDESC, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
      umma_commit(done);
      volatile int no_abort = 0;
      mbar_wait(done, 0, &no_abort, nullptr, 0);
    }
  } else {
    const int quarter = warp & 3;
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int mb = tile % num_m, nb = tile / num_m;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag, status, STATUS_TIMEOUT_GEMM)) break;
      tc_fence_after();
      const int r = quarter * 32 + lane, y = (mb / tiles_x) * bh + r / bw, x = (mb % tiles_x) * bw + r % bw;
      const int row = y * w + x;  // this thread's pixel
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      conv_epilogue<BN, EPI>(taddr, row, y < h && x < w, nb * BN, ep);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---- the same convolution on CTA pairs (tcgen05.mma.cta_group::2, M = 256): a pair takes two pixel
// tiles (the leader tile 2 u, the peer 2 u + 1) and all 144 output channels, each CTA loading its own
// shifted picture box and HALF of the weight block (72 rows), so a stage carries 25 instead of 34 KB
// for the same MMA work -- the 144-channel convolutions are bound by what reaches shared memory.
// Roles and barriers as the pair GEMM (gemm.cu): the leader's full barrier counts both CTAs' bytes,
// its MMA commits arrive on both CTAs' empty barriers, both CTAs' epilogue warps on its tempty.
struct Conv2Cfg {
  static constexpr int BN = 144;                        // output channels of a pair tile
  static constexpr int A_BYTES = BM * BK * 2;           // this CTA's 128 pixels x 64 channels
  static constexpr int B_BYTES = (BN / 2) * BK * 2;     // this CTA's 72 weight rows
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 8;
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr uint32_t IDESC = idesc_bf16(256, BN);
};

template <int EPI, int TAPS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM_THREADS, 1)
    k_conv2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int h, int w, int bw,
            int cp, int cout_tiles, const ConvEpi ep, int* status) {
  using C = Conv2Cfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int bh = BM / bw, tiles_x = (w + bw - 1) / bw;
  const int num_m = tiles_x * ((h + bh - 1) / bh);
  const int num_mp = (num_m + 1) / 2;  // pixel-tile pairs (the last peer tile may lie past the picture)
  const int num_units = num_mp * cout_tiles;
  const int cblocks = cp / BK;
  const int num_kb = TAPS * cblocks;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // 4 epilogue warps x 2 CTAs (the leader's instance)
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      griddep_wait();
      int stage = 0;
      uint32_t phase = 0;
      int last_phase[C::STAGES];
#pragma unroll
      for (int s = 0; s < C::STAGES; ++s) last_phase[s] = -1;
      bool ok = true;
      for (int u = cluster; u < num_units && ok; u += nclusters) {
        const int mp = u % num_mp, nb = u / num_mp;  // pixel tiles fastest: a weight block stays in L2
        const int mb = 2 * mp + static_cast<int>(rank);
        const int y0 = (mb / tiles_x) * bh, x0 = (mb % tiles_x) * bw;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, status, STATUS_TIMEOUT_GEMM)) {
            ok = false;
            break;
          }
          const uint32_t lfull = mapa_shared(&full[stage], 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
          const int tap = kb / cblocks, cb = kb - tap * cblocks;
          if constexpr (TAPS == 9)
            tma_load_3d_pair(sA + stage * C::A_BYTES, &tmA, lfull, cb * BK, x0 + tap % 3 - 1, y0 + tap / 3 - 1);
          else
            tma_load_2d_pair(sA + stage * C::A_BYTES, &tmA, lfull, cb * BK, x0);
          tma_load_2d_pair(sB + stage * C::B_BYTES, &tmB, lfull, kb * BK, nb * C::BN + static_cast<int>(rank) * 72);
          last_phase[stage] = static_cast<int>(phase);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok && rank == 0) {
        // the copies already issued land before the pair leaves (bounded waits on the leader's full
        // barriers, which count both CTAs' bytes)
        volatile int no_abort = 0;
        for (int s = 0; s < C::STAGES; ++s)
          if (last_phase[s] >= 0) mbar_wait(&full[s], static_cast<uint32_t>(last_phase[s]), &no_abort, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint64_t a_desc0 = sdesc_sw128(smem_u32(sA), 16, 1024);
      const uint64_t b_desc0 = sdesc_sw128(smem_u32(sB), 16, 1024);
      int it = 0;
      for (int u = cluster; u < num_units && ok; u += nclusters, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, status, STATUS_TIMEOUT_GEMM)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 256;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, status, STATUS_TIMEOUT_GEMM)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = a_desc0 + static_cast<uint64_t>((stage * C::A_BYTES) >> 4);
          const uint64_t bd = b_desc0 + static_cast<uint64_t>((stage * C::B_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) umma_pair(d_tmem, ad + 2 * k, bd + 2 * k, C::IDESC, (kb | k) != 0 ? 1u : 0u);
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit_pair(&tfull[acc], 0x3);
      }
      umma_commit_pair(done, 0x3);
      volatile int no_abort = 0;
      mbar_wait(done, 0, &no_abort, nullptr, 0);
    } else if (lane == 0 && rank == 1) {
      volatile int no_abort = 0;
      mbar_wait(done, 0, &no_abort, nullptr, 0);
    }
  } else {
    const int quarter = warp & 3;
    int it = 0;
    for (int u = cluster; u < num_units; u += nclusters, ++it) {
      const int mp = u % num_mp, nb = u / num_mp;
      const int mb = 2 * mp + static_cast<int>(rank);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag, status, STATUS_TIMEOUT_GEMM)) break;
      tc_fence_after();
      const int r = quarter * 32 + lane, y = (mb / tiles_x) * bh + r / bw, x = (mb % tiles_x) * bw + r % bw;
      const int row = y * w + x;  // this thread's pixel
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * 256;
      conv_epilogue<C::BN, EPI>(taddr, row, mb < num_m && y < h && x < w, nb * C::BN, ep);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(&tempty[acc], 0));
    }
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

template <int EPI, int TAPS>
static cudaError_t allow_smem_conv2() {
  return cudaFuncSetAttribute(k_conv2<EPI, TAPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, Conv2Cfg::SMEM);
}

template <int BN, int EPI, int TAPS>
static cudaError_t allow_smem_conv() {
  return cudaFuncSetAttribute(k_conv<BN, EPI, TAPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, ConvCfg<BN>::SMEM);
}

int conv_prepare() {
  const cudaError_t e[] = {allow_smem_conv<64, CONV_F32, 9>(),
                           allow_smem_conv<64, CONV_F32, 1>(), allow_smem_conv<64, CONV_BF16, 1>(),
                           allow_smem_conv<16, CONV_RGBA, 9>(), allow_smem_conv2<CONV_F32, 9>(),
                           allow_smem_conv2<CONV_F32, 1>(), allow_smem_conv2<CONV_BF16, 1>()};
  for (cudaError_t x : e)
    if (x != cudaSuccess) return static_cast<int>(x);
  return 0;
}

// the width of a 3 x 3 convolution's pixel tile: the largest divisor of W that divides 128, so a tile
// is bw columns x 128 / bw rows and one TMA box of the shifted picture
static int tile_width(int w) {
  int g = 128;
  while (w % g) g >>= 1;
  return g;
}

template <int BN, int EPI, int TAPS>
static int conv_run(const ConvArgs& a, int* d_status, int num_sms, cudaStream_t st) {
  using C = ConvCfg<BN>;
  CUtensorMap ta, tb;
  const int npix = a.h * a.w;
  if (TAPS == 9) {
    const int wt = tile_width(a.w), ht = 128 / wt;
    const uint64_t d[3] = {static_cast<uint64_t>(a.cp), static_cast<uint64_t>(a.w), static_cast<uint64_t>(a.h)};
    const uint64_t s[2] = {static_cast<uint64_t>(a.cp) * 2, static_cast<uint64_t>(a.w) * a.cp * 2};
    const uint32_t b[3] = {BK, static_cast<uint32_t>(wt), static_cast<uint32_t>(ht)};
    if (make_tmap_bf16(&ta, a.x, 3, d, s, b)) return -4;
  } else {
    const uint64_t d[2] = {static_cast<uint64_t>(a.cp), static_cast<uint64_t>(npix)};
    const uint64_t s[1] = {static_cast<uint64_t>(a.cp) * 2};
    const uint32_t b[2] = {BK, BM};
    if (make_tmap_bf16(&ta, a.x, 2, d, s, b)) return -4;
  }
  const int cout_tiles = (a.cout + BN - 1) / BN;
  {
    const uint64_t d[2] = {static_cast<uint64_t>(TAPS) * a.cp, static_cast<uint64_t>(cout_tiles) * BN};
    const uint64_t s[1] = {static_cast<uint64_t>(TAPS) * a.cp * 2};
    const uint32_t b[2] = {BK, BN};
    if (make_tmap_bf16(&tb, a.wt, 2, d, s, b)) return -4;
  }
  // a 1 x 1 convolution sees the picture as one row of pixels, tiles of 128 consecutive ones
  const int th = TAPS == 9 ? a.h : 1, tw = TAPS == 9 ? a.w : npix;
  const int bw = TAPS == 9 ? tile_width(a.w) : BM;
  const int tiles = ((tw + bw - 1) / bw) * ((th + BM / bw - 1) / (BM / bw)) * cout_tiles;
  const int grid = tiles < num_sms ? tiles : num_sms;
  ConvEpi ep = a.ep;
  ep.cout = a.cout;
  return static_cast<int>(launch_pdl(k_conv<BN, EPI, TAPS>, dim3(grid), dim3(GEMM_THREADS), C::SMEM, st, ta, tb, th,
                                     tw, bw, a.cp, cout_tiles, ep, d_status));
}

// BN = 144 on CTA pairs (k_conv2): the same tensor maps but weight boxes of 72 rows
template <int EPI, int TAPS>
static int conv2_run(const ConvArgs& a, int* d_status, int num_sms, cudaStream_t st) {
  using C = Conv2Cfg;
  CUtensorMap ta, tb;
  const int npix = a.h * a.w;
  if (TAPS == 9) {
    const int wt = tile_width(a.w), ht = 128 / wt;
    const uint64_t d[3] = {static_cast<uint64_t>(a.cp), static_cast<uint64_t>(a.w), static_cast<uint64_t>(a.h)};
    const uint64_t s[2] = {static_cast<uint64_t>(a.cp) * 2, static_cast<uint64_t>(a.w) * a.cp * 2};
    const uint32_t b[3] = {BK, static_cast<uint32_t>(wt), static_cast<uint32_t>(ht)};
    if (make_tmap_bf16(&ta, a.x, 3, d, s, b)) return -4;
  } else {
    const uint64_t d[2] = {static_cast<uint64_t>(a.cp), static_cast<uint64_t>(npix)};
    const uint64_t s[1] = {static_cast<uint64_t>(a.cp) * 2};
    const uint32_t b[2] = {BK, BM};
    if (make_tmap_bf16(&ta, a.x, 2, d, s, b)) return -4;
  }
  const int cout_tiles = (a.cout + C::BN - 1) / C::BN;
  {
    const uint64_t d[2] = {static_cast<uint64_t>(TAPS) * a.cp, static_cast<uint64_t>(cout_tiles) * C::BN};
    const uint64_t s[1] = {static_cast<uint64_t>(TAPS) * a.cp * 2};
    const uint32_t b[2] = {BK, C::BN / 2};
    if (make_tmap_bf16(&tb, a.wt, 2, d, s, b)) return -4;
  }
  const int th = TAPS == 9 ? a.h : 1, tw = TAPS == 9 ? a.w : npix;
  const int bw = TAPS == 9 ? tile_width(a.w) : BM;
  const int num_m = ((tw + bw - 1) / bw) * ((th + BM / bw - 1) / (BM / bw));
  const int units = ((num_m + 1) / 2) * cout_tiles;
  int clusters = num_sms / 2;
  clusters = units < clusters ? units : clusters;
  ConvEpi ep = a.ep;
  ep.cout = a.cout;
  return static_cast<int>(launch_pdl(k_conv2<EPI, TAPS>, dim3(clusters * 2), dim3(GEMM_THREADS), C::SMEM, st, ta, tb,
                                     th, tw, bw, a.cp, cout_tiles, ep, d_status));
}

int conv_launch(const ConvArgs& a, int* d_status, int num_sms, cudaStream_t st) {
  if (a.h <= 0 || a.w <= 0 || a.cp <= 0 || a.cp % BK || a.cout <= 0) return -1;
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.wt)) & 15) return -1;
  const int epi = a.ep.kind;
  if (a.ep.dup && (epi != CONV_F32 || a.ep.out_w != a.w || (a.w | a.h) & 1 || a.ep.dup_ci <= 0 || a.ep.dup_ft < 1 ||
                   (4 * a.cout * a.ep.dup_ft) % a.ep.dup_ci))
    return -1;
  if (epi == CONV_RGBA) {
    if (a.taps != 9 || a.cout > 16) return -1;
    return conv_run<16, CONV_RGBA, 9>(a, d_status, num_sms, st);
  }
  if (a.cout % 144 == 0 && num_sms >= 2) {
    if (a.taps == 9 && epi == CONV_F32) return conv2_run<CONV_F32, 9>(a, d_status, num_sms, st);
    if (a.taps == 1 && epi == CONV_F32) return conv2_run<CONV_F32, 1>(a, d_status, num_sms, st);
    if (a.taps == 1 && epi == CONV_BF16) return conv2_run<CONV_BF16, 1>(a, d_status, num_sms, st);
  } else if (a.cout % 64 == 0) {
    if (a.taps == 9 && epi == CONV_F32) return conv_run<64, CONV_F32, 9>(a, d_status, num_sms, st);
    if (a.taps == 1 && epi == CONV_F32) return conv_run<64, CONV_F32, 1>(a, d_status, num_sms, st);
    if (a.taps == 1 && epi == CONV_BF16) return conv_run<64, CONV_BF16, 1>(a, d_status, num_sms, st);
  }
  return -1;
}

}  // namespace exn
