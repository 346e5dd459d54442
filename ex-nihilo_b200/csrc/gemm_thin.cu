// gemm_thin.cu -- the product of a thin activation block with a weight
// matrix, for the prompt encoder's GEMMs (a prompt is ~100-250 tokens):
// part[s] = (X W^T) over the s-th part of K, fp32, with the WEIGHTS as the
// 256-row MMA operand and the tokens as N (a multiple of 16 up to 256).
//
// The pair GEMM (gemm.cu) puts the tokens on the 256-row side, where 141
// tokens leave 115 rows of every MMA empty and a k-block costs as many tensor
// clocks as streaming its weights.  Here the weights fill the rows, the MMA is
// 256 x NT x 16 (NT = tokens rounded up to 16), and each stage holds 16 KB of
// weights and NT/2 token rows a CTA, so more stages (and weight bytes) are in
// flight.  The accumulator is D^T: TMEM lane = output column, TMEM column =
// token; the epilogue stores each token's 32 columns of a warp as one
// 128-byte row segment of part [s][n][N].
//
// Roles as in the pair GEMM: warp 0 TMA producer (both CTAs), warp 1 the
// leader's MMA issuer (tcgen05.mma.cta_group::2, accumulators double-buffered
// in TMEM), warps 2..5 the epilogue.  Work units: (256-column block of the
// output, part of K), round-robin over the pairs.
#include "gemm_common.cuh"

namespace exn {

namespace {

template <int NTM>
struct ThinCfg {
  static constexpr int A_BYTES = 128 * BK * 2;            // this CTA's 128 weight rows
  static constexpr int B_BYTES = (NTM / 2) * BK * 2;      // this CTA's half of the token rows
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 8 ? 8 : (200 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * NTM <= 256 ? 256 : 512;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

template <int NTM>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_thin(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, int n, int nt,
                int N, int K, int splits, float* __restrict__ part, int* status) {
  using C = ThinCfg<NTM>;
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
  const int num_mb = N / 256, num_kb = K / BK;
  const int num_units = num_mb * splits;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int b_bytes = (nt / 2) * BK * 2;  // this CTA's token rows of a stage (the box, zero-filled past n)

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
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
    tma_prefetch(&tmW);
    tma_prefetch(&tmX);
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
      // ---- TMA producer: the token rows are the previous kernel's output
      griddep_wait();
      int stage = 0;
      uint32_t phase = 0;
      int last_phase[C::STAGES];
#pragma unroll
      for (int s = 0; s < C::STAGES; ++s) last_phase[s] = -1;
      bool ok = true;
      for (int u = cluster; u < num_units && ok; u += nclusters) {
        const int sp = u / num_mb, mb = u - sp * num_mb;
        const int kb1 = (sp + 1) * num_kb / splits;
        for (int kb = sp * num_kb / splits; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, status, STATUS_TIMEOUT_GEMM)) {
            ok = false;
            break;
          }
          const uint32_t lfull = mapa_shared(&full[stage], 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (C::A_BYTES + b_bytes));
          tma_load_2d_pair(sA + stage * C::A_BYTES, &tmW, lfull, kb * BK, mb * 256 + rank * 128);
          tma_load_2d_pair(sB + stage * C::B_BYTES, &tmX, lfull, kb * BK, rank * (nt / 2));
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
      // ---- MMA issuer (leader only): D^T (256 output columns x nt tokens) += W X^T
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint32_t idesc = idesc_bf16(256, nt);
      const uint64_t a_desc0 = sdesc_sw128(smem_u32(sA), 16, 1024);
      const uint64_t b_desc0 = sdesc_sw128(smem_u32(sB), 16, 1024);
      int it = 0;
      for (int u = cluster; u < num_units && ok; u += nclusters, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, status, STATUS_TIMEOUT_GEMM)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * NTM;
        const int sp = u / num_mb;
        const int kbn = (sp + 1) * num_kb / splits - sp * num_kb / splits;
        for (int kb = 0; kb < kbn; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, status, STATUS_TIMEOUT_GEMM)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = a_desc0 + static_cast<uint64_t>((stage * C::A_BYTES) >> 4);
          const uint64_t bd = b_desc0 + static_cast<uint64_t>((stage * C::B_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_pair(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
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
    // ---- epilogue warps 2..5: TMEM lane quarter = warp % 4; lane = output column, column = token
    const int quarter = warp & 3;
    int it = 0;
    for (int u = cluster; u < num_units; u += nclusters, ++it) {
      const int sp = u / num_mb, mb = u - sp * num_mb;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag, status, STATUS_TIMEOUT_GEMM)) break;
      tc_fence_after();
      const int col = mb * 256 + static_cast<int>(rank) * 128 + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * NTM;
      float* dst = part + static_cast<long long>(sp) * n * N + col;
#pragma unroll 1
      for (int j0 = 0; j0 < nt; j0 += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + j0, r);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (j0 + i < n) dst[static_cast<long long>(j0 + i) * N] = __uint_as_float(r[i]);
      }
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

template <int NTM>
int thin_run(const bf16* x, int n, const bf16* w, int N, int K, int splits, float* part, int* d_status, int num_sms,
             cudaStream_t st) {
  using C = ThinCfg<NTM>;
  const int nt = (n + 15) / 16 * 16;
  CUtensorMap tw, tx;
  const uint64_t dw[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
  const uint64_t sw[1] = {static_cast<uint64_t>(K) * 2};
  const uint32_t bw[2] = {BK, 128};
  const uint64_t dx[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(n)};
  const uint64_t sx[1] = {static_cast<uint64_t>(K) * 2};
  const uint32_t bx[2] = {BK, static_cast<uint32_t>(nt / 2)};
  if (make_tmap_bf16(&tw, w, 2, dw, sw, bw) || make_tmap_bf16(&tx, x, 2, dx, sx, bx)) return -4;
  const int units = (N / 256) * splits;
  int clusters = num_sms / 2;
  clusters = units < clusters ? units : clusters;
  return static_cast<int>(launch_pdl(k_gemm_thin<NTM>, dim3(clusters * 2), dim3(GEMM_THREADS), C::SMEM, st, tw, tx, n,
                                     nt, N, K, splits, part, d_status));
}

}  // namespace

int gemm_thin_prepare() {
  cudaError_t e = cudaFuncSetAttribute(k_gemm_thin<160>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       ThinCfg<160>::SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_gemm_thin<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, ThinCfg<256>::SMEM);
  return static_cast<int>(e);
}

int gemm_thin_launch(const bf16* x, int n, const bf16* w, int N, int K, int splits, float* part, int* d_status,
                     int num_sms, cudaStream_t st) {
  if (n < 1 || n > 256 || N < 256 || N % 256 || K < BK || K % BK || splits < 1 || splits > K / BK || num_sms < 2)
    return -1;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) return -1;
  if (n <= 160) return thin_run<160>(x, n, w, N, K, splits, part, d_status, num_sms, st);
  return thin_run<256>(x, n, w, N, K, splits, part, d_status, num_sms, st);
}

}  // namespace exn
