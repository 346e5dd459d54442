// gemm_q8.cu -- the pair GEMM of gemm.cu with the weights kept as Q8_0: int8
// values with an fp16 scale per 32 along K, as ex-nihilo's upload-dit keeps them
// on the device (repack_q8 into qs + d, src/cuda-dit.lisp:71-76) and feeds them
// to its GEMMs (d4_mm_q8_0, src/cuda-dit.lisp:115-130).
//
// C[M x N] = A[M x K] . B[N x K]^T, A bf16 activations, B = q * d.  A CTA pair
// computes 256 x 256 tiles with tcgen05.mma.cta_group::2 exactly as k_gemm2
// does; what changes is where B comes from.  Per 64-deep k-block each CTA's TMA
// producer brings its 128 rows of A (bf16, 128B swizzle) and its half of B as
// int8 (128 rows x 64 bytes) with the two fp16 scales of each row; eight
// converter warps then write B as bf16 into the 128B-swizzled operand layout a
// TMA load would have produced (row r's 16-byte chunk j at chunk j ^ (r % 8)),
// computing each value as round-to-nearest bf16 of (float) q * (float) d: the
// same bits as the load-time conversion of the bf16 weight slab, so the products
// are bit-identical to k_gemm2's on that slab.
//
//   warp 0      TMA: A (counted on the leader's full barrier), int8 + scales
//               (on this CTA's qfull barrier)
//   warp 1      MMA issue (leader only)
//   warps 2..5  epilogue (as k_gemm2)
//   warps 6..13 int8 -> bf16 conversion into the stage's B buffer, a pair of
//               warps per k-block, four k-blocks at once
// The leader's full barrier of a stage completes when both CTAs' A bytes have
// landed and both CTAs' two converter warps have arrived.  No multicast loads.
#include "gemm_common.cuh"

namespace exn {

struct Gemm2QCfg {
  static constexpr int BN = 256;
  static constexpr int STAGES = 5;
  static constexpr int A_BYTES = 128 * BK * 2;  // this CTA's 128 rows of A
  static constexpr int B_BYTES = 128 * BK * 2;  // this CTA's half of B, converted to bf16
  static constexpr int Q_BYTES = 128 * BK;      // the same half as int8
  static constexpr int D_BYTES = 128 * 2 * 2;   // its fp16 scales: two 32-blocks per row
  static constexpr int CONV = 8;                // converter warps: 4 pairs, a pair per k-block in flight
  static constexpr int THREADS = 32 * (6 + CONV);
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM = STAGES * (A_BYTES + B_BYTES + Q_BYTES + D_BYTES) + 1024 + 256;
  static constexpr uint32_t IDESC = idesc_bf16(256, 256);
};

// 16 int8 (Q) times the fp16 scale D as 8 bf16 pairs, each value rounded once from the exact fp32
// product.  int8 -> float exactly: with its sign bit flipped a byte is q + 128; placed as the low
// mantissa byte of 2^23 it reads as 2^23 + q + 128, and subtracting 2^23 + 128 leaves q.
__device__ __forceinline__ void q8_to_bf16x16(const int4 q, float d, uint32_t (&out)[8]) {
  const uint64_t bias = f2(-8388736.f, -8388736.f), dd = f2(d, d);
  const uint32_t w[4] = {static_cast<uint32_t>(q.x) ^ 0x80808080u, static_cast<uint32_t>(q.y) ^ 0x80808080u,
                         static_cast<uint32_t>(q.z) ^ 0x80808080u, static_cast<uint32_t>(q.w) ^ 0x80808080u};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float lo = __uint_as_float(__byte_perm(w[k], 0x4B000000u, 0x7650 + 2 * h));
      const float hi = __uint_as_float(__byte_perm(w[k], 0x4B000000u, 0x7651 + 2 * h));
      uint64_t v;
      asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(v) : "l"(fadd2(f2(lo, hi), bias)), "l"(dd));
      float a, b;
      f2_split(v, a, b);
      out[2 * k + h] = pack_bf16x2(a, b);
    }
  }
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Gemm2QCfg::THREADS, 1)
    k_gemm2_q8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmQ,
               const __grid_constant__ CUtensorMap tmD, int M, int N, int K, int group_m, const GemmEpi ep,
               int* status) {
  using C = Gemm2QCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + C::STAGES * C::A_BYTES;
  uint8_t* sQ = sB + C::STAGES * C::B_BYTES;
  uint8_t* sD = sQ + C::STAGES * C::Q_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sD + C::STAGES * C::D_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* qfull = empty + C::STAGES;
  uint64_t* tfull = qfull + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int num_m = (M + 255) / 256, num_n = N / C::BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = K / BK;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 5);   // the leader's producer (A bytes of both CTAs) + two converter warps per CTA
      mbar_init(&empty[s], 1);  // the leader's multicast commit
      mbar_init(&qfull[s], 1);  // this CTA's producer (int8 and scale bytes)
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tmA);
    tma_prefetch(&tmQ);
    tma_prefetch(&tmD);
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
      for (int tile = cluster; tile < num_tiles && ok; tile += nclusters) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, group_m, mb, nb);
        const int brow = nb * C::BN + static_cast<int>(rank) * 128;  // this CTA's half of B
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, status, STATUS_TIMEOUT_GEMM)) {
            ok = false;
            break;
          }
          const uint32_t lfull = mapa_shared(&full[stage], 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * C::A_BYTES);
          tma_load_2d_pair(sA + stage * C::A_BYTES, &tmA, lfull, kb * BK, mb * 256 + static_cast<int>(rank) * 128);
          mbar_arrive_expect_tx(&qfull[stage], C::Q_BYTES + C::D_BYTES);
          tma_load_2d(sQ + stage * C::Q_BYTES, &tmQ, &qfull[stage], kb * BK, brow);
          tma_load_2d(sD + stage * C::D_BYTES, &tmD, &qfull[stage], brow * 2, kb);
          last_phase[stage] = static_cast<int>(phase);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {  // the copies already issued land before the CTA moves on (bounded waits)
        volatile int no_abort = 0;
        for (int s = 0; s < C::STAGES; ++s)
          if (last_phase[s] >= 0) {
            mbar_wait(&qfull[s], static_cast<uint32_t>(last_phase[s]), &no_abort, nullptr, 0);
            if (rank == 0) mbar_wait(&full[s], static_cast<uint32_t>(last_phase[s]), &no_abort, nullptr, 0);
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      const uint64_t a_desc0 = sdesc_sw128(smem_u32(sA), 16, 1024);
      const uint64_t b_desc0 = sdesc_sw128(smem_u32(sB), 16, 1024);
      for (int tile = cluster; tile < num_tiles && ok; tile += nclusters, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, status, STATUS_TIMEOUT_GEMM)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::BN;
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
  } else if (warp < 6) {
    // ---- epilogue warps 2..5 of each CTA: TMEM lane quarter = warp % 4
    const int quarter = warp & 3;
    int it = 0;
    for (int tile = cluster; tile < num_tiles; tile += nclusters, ++it) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, group_m, mb, nb);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag, status, STATUS_TIMEOUT_GEMM)) break;
      tc_fence_after();
      const int row = mb * 256 + static_cast<int>(rank) * 128 + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * C::BN;
      epilogue<256, EPI>(taddr, row, row < M, nb * C::BN, ep);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(&tempty[acc], 0));
    }
  } else {
    // ---- converter warps 6..13: pair p = (w - 6) / 2 converts the k-blocks i with i % 4 == p, its two
    // warps half the rows each, so four k-blocks convert at once and each warp's chain (wait, convert,
    // fence, arrive) overlaps the others'.  Lane l takes the 16-byte pieces c = l + 32 j (j < 8) of its
    // 64 rows, row 64 h + c / 4, k 16 (c % 4) .. +15: each int8 load of the warp covers 512 contiguous
    // bytes, each bf16 store 32 bank-spread chunks of the 128-byte-swizzled layout.
    const int cw = warp - 6, pair = cw >> 1, half = cw & 1;
    bool ok = true;
    int it = 0;
    for (int tile = cluster; tile < num_tiles && ok; tile += nclusters) {
      for (int kb = 0; kb < num_kb; ++kb, ++it) {
        if ((it & 3) != pair) continue;
        const int stage = it % C::STAGES;
        const uint32_t phase = static_cast<uint32_t>(it / C::STAGES) & 1;
        if (!(ok = mbar_wait_uniform(&qfull[stage], phase, abort_flag, status, STATUS_TIMEOUT_GEMM))) break;
        const uint8_t* q = sQ + stage * C::Q_BYTES;
        const __half* d = reinterpret_cast<const __half*>(sD + stage * C::D_BYTES);
        uint8_t* b = sB + stage * C::B_BYTES;
#pragma unroll 4
        for (int j = 0; j < 8; ++j) {
          const int c = lane + 32 * j;
          const int row = 64 * half + (c >> 2), seg = c & 3;
          const int4 qv = *reinterpret_cast<const int4*>(q + row * 64 + seg * 16);
          const float dv = __half2float(d[row * 2 + (seg >> 1)]);
          uint32_t o[8];
          q8_to_bf16x16(qv, dv, o);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int chunk = (2 * seg + hh) ^ (row & 7);
            *reinterpret_cast<uint4*>(b + row * 128 + chunk * 16) =
                make_uint4(o[4 * hh], o[4 * hh + 1], o[4 * hh + 2], o[4 * hh + 3]);
          }
        }
        // the generic-proxy stores reach the tensor core's (async proxy) view before the arrival
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(&full[stage], 0));
      }
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

// Q8_0 scales [N][K/32] (GGUF order) -> [K/64][N][2]: one k-block's scales of 128 rows are 512
// contiguous bytes, a single TMA box.
__global__ void k_q8_scales_by_kblock(const __half* __restrict__ d, __half* __restrict__ out, int n, int k) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long nb = static_cast<long long>(n) * (k / 32);
  if (i >= nb) return;
  const long long r = i / (k / 32);
  const int b = static_cast<int>(i - r * (k / 32));
  out[(static_cast<long long>(b >> 1) * n + r) * 2 + (b & 1)] = d[i];
}

int q8_scales_by_kblock_launch(const __half* d, __half* out, int n, int k, cudaStream_t st) {
  if (n <= 0 || k <= 0 || k % 64) return -1;
  const long long nb = static_cast<long long>(n) * (k / 32);
  k_q8_scales_by_kblock<<<static_cast<unsigned>((nb + 255) / 256), 256, 0, st>>>(d, out, n, k);
  return static_cast<int>(cudaGetLastError());
}

template <int EPI>
static cudaError_t allow_smem_q8() {
  return cudaFuncSetAttribute(k_gemm2_q8<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, Gemm2QCfg::SMEM);
}

int gemm_q8_prepare() {
  cudaError_t e = allow_smem_q8<EPI_F32>();
  if (e == cudaSuccess) e = allow_smem_q8<EPI_SWIGLU>();
  return static_cast<int>(e);
}

// C = A . (q d)^T on CTA pairs.  QS int8 [N][K], DK the scales by k-block ([K/64][N][2] fp16).
int gemm_q8_launch(const GemmArgs& g, const int8_t* qs, const __half* dk, int* d_status, int num_sms,
                   cudaStream_t st) {
  using C = Gemm2QCfg;
  if (g.M <= 0 || g.N <= 0 || g.K <= 0 || g.K % BK || g.N % C::BN || num_sms < 2) return -1;
  if ((reinterpret_cast<uintptr_t>(g.a) | reinterpret_cast<uintptr_t>(qs) | reinterpret_cast<uintptr_t>(dk)) & 15)
    return -1;
  if ((g.lda * 2) % 16) return -1;
  CUtensorMap ta, tq, td;
  const uint64_t da[2] = {static_cast<uint64_t>(g.K), static_cast<uint64_t>(g.M)};
  const uint64_t sa[1] = {static_cast<uint64_t>(g.lda) * 2};
  const uint32_t ba[2] = {BK, 128};
  const uint64_t dq[2] = {static_cast<uint64_t>(g.K), static_cast<uint64_t>(g.N)};
  const uint64_t sq[1] = {static_cast<uint64_t>(g.K)};
  const uint32_t bq[2] = {BK, 128};
  const uint64_t dd[2] = {static_cast<uint64_t>(g.N) * 2, static_cast<uint64_t>(g.K / BK)};
  const uint64_t sd[1] = {static_cast<uint64_t>(g.N) * 4};
  const uint32_t bd[2] = {256, 1};
  if (make_tmap_bf16(&ta, g.a, 2, da, sa, ba) ||
      make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, qs, 2, dq, sq, bq, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      make_tmap(&td, CU_TENSOR_MAP_DATA_TYPE_UINT16, dk, 2, dd, sd, bd, CU_TENSOR_MAP_SWIZZLE_NONE))
    return -4;
  const int num_m = (g.M + 255) / 256;
  const int tiles = num_m * (g.N / C::BN);
  int clusters = num_sms / 2;
  clusters = tiles < clusters ? tiles : clusters;
  int group_m = static_cast<int>((48ll << 20) / (256ll * g.K * 2));
  group_m = group_m < 4 ? 4 : group_m;
  group_m = group_m > num_m ? num_m : group_m;
  switch (g.epi) {
    case EPI_F32:
      return static_cast<int>(launch_pdl(k_gemm2_q8<EPI_F32>, dim3(clusters * 2), dim3(C::THREADS), C::SMEM, st, ta,
                                         tq, td, g.M, g.N, g.K, group_m, g.ep, d_status));
    case EPI_SWIGLU:
      return static_cast<int>(launch_pdl(k_gemm2_q8<EPI_SWIGLU>, dim3(clusters * 2), dim3(C::THREADS), C::SMEM, st,
                                         ta, tq, td, g.M, g.N, g.K, group_m, g.ep, d_status));
    default:
      return -1;
  }
}

}  // namespace exn
