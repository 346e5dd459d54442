// gemm.cu -- the DiT's weight products on the 5th-generation tensor cores.
//
// C[M x N] = A[M x K] . B[N x K]^T with A the bf16 activations and B a bf16
// weight (out x in, both K-contiguous: the "TN" case).  One persistent CTA
// per SM walks output tiles of 128 x BN:
//
//   warp 0      TMA producer: A and B k-blocks of 64 into a STAGES-deep ring
//               of 128-byte-swizzled shared memory tiles
//   warp 1      MMA issuer: tcgen05.mma kind::f16 (M=128, N=BN, K=16) into
//               one of two TMEM accumulators (2 x BN fp32 columns)
//   warps 2..5  epilogue: tcgen05.ld of the finished accumulator (one row per
//               thread) and the fused per-layer arithmetic of the DiT, while
//               the MMA already fills the other accumulator
//
// The fused epilogues are in gemm_common.cuh.
#include <stdlib.h>

#include <mutex>

#include "gemm_common.cuh"

namespace exn {

// ----------------------------------------------------------------------------- the kernel

template <int BN, int EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N, int K,
           int group_m, const GemmEpi ep, int* status) {
  using C = GemmCfg<BN>;
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
  const int num_m = (M + BM - 1) / BM, num_n = N / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = K / BK;

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
      // ---- TMA producer: the previous kernel's outputs (A, and the epilogue's rows) are ready
      griddep_wait();
      int stage = 0;
      uint32_t phase = 0;
      int last_phase[C::STAGES];
#pragma unroll
      for (int s = 0; s < C::STAGES; ++s) last_phase[s] = -1;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, group_m, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, status, STATUS_TIMEOUT_GEMM)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * BK, mb * BM);
          tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * BK, nb * BN);
          last_phase[stage] = static_cast<int>(phase);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {  // let the copies already issued land before the CTA leaves
        volatile int no_abort = 0;
        for (int s = 0; s < C::STAGES; ++s)
          if (last_phase[s] >= 0) mbar_wait(&full[s], static_cast<uint32_t>(last_phase[s]), &no_abort, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      // descriptors formed once; start addresses then advance in 16-byte units
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
      // every MMA issued has finished before TMEM is released
      umma_commit(done);
      volatile int no_abort = 0;
      mbar_wait(done, 0, &no_abort, nullptr, 0);
    }
  } else {
    // ---- epilogue warps 2..5: TMEM lane quarter = warp % 4
    const int quarter = warp & 3;
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, group_m, mb, nb);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag, status, STATUS_TIMEOUT_GEMM)) break;
      tc_fence_after();
      const int row = mb * BM + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      epilogue<BN, EPI>(taddr, row, row < M, nb * BN, ep);
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


// ----------------------------------------------------------------------------- CTA-pair kernel
// A cluster of two CTAs computes a 256 x 256 tile with tcgen05.mma.cta_group::2
// (M = 256): each CTA loads its own 128 rows of A and its half (128 rows) of
// B per k-block, so per SM the tensor cores read 64 bytes of operands a clock
// from shared memory and the TMA pulls half the B traffic of a 128 x 256 tile.
// The leader (rank 0) issues the MMAs; each CTA's TMEM holds the fp32
// accumulator of its 128 rows over all 256 columns and its own epilogue warps
// drain it.  Barriers: full[] of the leader counts both CTAs' bytes; empty[]
// and tfull[] are armed in both CTAs by multicast commits; tempty[] of the
// leader counts the 8 epilogue warps of the pair.  No multicast loads.

struct Gemm2Cfg {
  static constexpr int BN = 256;
  static constexpr int STAGES = 6;
  static constexpr int A_BYTES = 128 * BK * 2;   // this CTA's 128 rows of A
  static constexpr int B_BYTES = 128 * BK * 2;   // this CTA's half of B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 512;           // two accumulators of 256 columns
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr uint32_t IDESC = idesc_bf16(256, 256);
};

// I8: A and B int8 (tcgen05.mma kind::i8, s32 accumulators): the same 128-byte k-blocks hold 128
// elements, so the tile geometry, swizzle and descriptors are the bf16 ones; K counts elements.
template <int EPI, bool I8 = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM_THREADS, 1)
    k_gemm2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N, int K,
            int group_m, const GemmEpi ep, int* status) {
  using C = Gemm2Cfg;
  constexpr int KB = I8 ? 2 * BK : BK;  // elements of a 128-byte k-block
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
  const int num_m = (M + 255) / 256, num_n = N / C::BN;
  // split-K (EPI_F32 only): tile t + s * num_mn sums k-blocks [s * num_kb / splits, (s + 1) *
  // num_kb / splits) of output tile t into rows s * M .. of the output (fp32 partials)
  const int splits = ep.splits > 1 ? ep.splits : 1;
  const int num_mn = num_m * num_n;
  const int num_tiles = num_mn * splits;
  const int num_kb = K / KB;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);     // the leader's producer, armed with both CTAs' bytes
      mbar_init(&empty[s], 1);    // the leader's multicast commit
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);    // multicast commit
      mbar_init(&tempty[a], 8);   // 4 epilogue warps x 2 CTAs (leader's instance used)
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
      // ---- TMA producer (both CTAs): the previous kernel's outputs (A, and the epilogue's rows) are ready
      griddep_wait();
      int stage = 0;
      uint32_t phase = 0;
      int last_phase[C::STAGES];  // the last phase of each stage whose copies this CTA issued
#pragma unroll
      for (int s = 0; s < C::STAGES; ++s) last_phase[s] = -1;
      bool ok = true;
      for (int tile = cluster; tile < num_tiles && ok; tile += nclusters) {
        int mb, nb;
        const int sp = tile / num_mn;
        tile_coords(tile - sp * num_mn, num_m, num_n, group_m, mb, nb);
        const int kb1 = (sp + 1) * num_kb / splits;
        for (int kb = sp * num_kb / splits; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, status, STATUS_TIMEOUT_GEMM)) {
            ok = false;
            break;
          }
          const uint32_t lfull = mapa_shared(&full[stage], 0);
          // the leader counts both CTAs' bytes; the peer's copies may land first (the phase
          // cannot complete before the leader's arrival)
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
          tma_load_2d_pair(sA + stage * C::A_BYTES, &tmA, lfull, kb * KB, mb * 256 + rank * 128);
          tma_load_2d_pair(sB + stage * C::B_BYTES, &tmB, lfull, kb * KB, nb * C::BN + rank * 128);
          last_phase[stage] = static_cast<int>(phase);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok && rank == 0) {
        // the copies already issued land before the pair moves on: each stage's full barrier (the
        // leader's) counts both CTAs' bytes of a phase, so waiting, bounded, for the last phase
        // armed here covers the peer's copies of that phase too; the peer cannot leave before this
        // wait ends (both CTAs meet at the cluster barrier at the end of the kernel)
        volatile int no_abort = 0;
        for (int s = 0; s < C::STAGES; ++s)
          if (last_phase[s] >= 0) mbar_wait(&full[s], static_cast<uint32_t>(last_phase[s]), &no_abort, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---- MMA issuer (leader only)
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
        const int sp = tile / num_mn;
        const int kbn = (sp + 1) * num_kb / splits - sp * num_kb / splits;  // k-blocks of this tile
        for (int kb = 0; kb < kbn; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, status, STATUS_TIMEOUT_GEMM)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = a_desc0 + static_cast<uint64_t>((stage * C::A_BYTES) >> 4);
          const uint64_t bd = b_desc0 + static_cast<uint64_t>((stage * C::B_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // 32 bytes of k a step: 16 bf16 or 32 int8
            if constexpr (I8)
              umma_pair_i8(d_tmem, ad + 2 * k, bd + 2 * k, idesc_i8(256, 256), (kb | k) != 0 ? 1u : 0u);
            else
              umma_pair(d_tmem, ad + 2 * k, bd + 2 * k, C::IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit_pair(&tfull[acc], 0x3);
      }
      // every MMA issued has finished before either CTA releases its TMEM
      umma_commit_pair(done, 0x3);
      volatile int no_abort = 0;
      mbar_wait(done, 0, &no_abort, nullptr, 0);
    } else if (lane == 0 && rank == 1) {
      volatile int no_abort = 0;  // the peer's copy of DONE is armed by the leader's commit
      mbar_wait(done, 0, &no_abort, nullptr, 0);
    }
  } else {
    // ---- epilogue warps 2..5 of each CTA: TMEM lane quarter = warp % 4
    const int quarter = warp & 3;
    int it = 0;
    for (int tile = cluster; tile < num_tiles; tile += nclusters, ++it) {
      int mb, nb;
      const int sp = tile / num_mn;
      tile_coords(tile - sp * num_mn, num_m, num_n, group_m, mb, nb);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag, status, STATUS_TIMEOUT_GEMM)) break;
      tc_fence_after();
      const int row = mb * 256 + static_cast<int>(rank) * 128 + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * C::BN;
      epilogue<256, EPI>(taddr, row + sp * M, row < M, nb * C::BN, ep);
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

// ----------------------------------------------------------------------------- host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// A tensor map of element type TYPE, zero fill out of bounds.  dims[0] is the contiguous axis;
// strides (bytes) for dims 1..rank-1.
int make_tmap(CUtensorMap* m, CUtensorMapDataType type, const void* base, int rank, const uint64_t* dims,
              const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i < rank - 1) s[i] = strides[i];
  }
  CUresult r = fn(m, type, rank, const_cast<void*>(base), d, s, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// bf16 tensor map, 128-byte swizzle (the tcgen05 operand layout)
int make_tmap_bf16(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                   const uint32_t* box) {
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, rank, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int BN, int EPI>
static int launch_bn(const GemmArgs& g, int* d_status, int num_sms, cudaStream_t st) {
  using C = GemmCfg<BN>;
  CUtensorMap ta, tb;
  const uint64_t da[2] = {static_cast<uint64_t>(g.K), static_cast<uint64_t>(g.M)};
  const uint64_t sa[1] = {static_cast<uint64_t>(g.lda) * 2};
  const uint32_t ba[2] = {BK, BM};
  const uint64_t db[2] = {static_cast<uint64_t>(g.K), static_cast<uint64_t>(g.N)};
  const uint64_t sb[1] = {static_cast<uint64_t>(g.ldb) * 2};
  const uint32_t bb[2] = {BK, BN};
  if (make_tmap_bf16(&ta, g.a, 2, da, sa, ba) || make_tmap_bf16(&tb, g.b, 2, db, sb, bb)) return -4;
  const int num_m = (g.M + BM - 1) / BM;
  const int tiles = num_m * (g.N / BN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  // as many row blocks per group as keep ~48 MB of activations in L2
  int group_m = static_cast<int>((48ll << 20) / (static_cast<long long>(BM) * g.K * 2));
  group_m = group_m < 8 ? 8 : group_m;
  group_m = group_m > num_m ? num_m : group_m;
  return static_cast<int>(launch_pdl(k_gemm<BN, EPI>, dim3(grid), dim3(GEMM_THREADS), C::SMEM, st, ta, tb, g.M, g.N,
                                     g.K, group_m, g.ep, d_status));
}

template <int EPI>
static int launch_pair(const GemmArgs& g, int* d_status, int num_sms, cudaStream_t st) {
  using C = Gemm2Cfg;
  CUtensorMap ta, tb;
  const uint64_t da[2] = {static_cast<uint64_t>(g.K), static_cast<uint64_t>(g.M)};
  const uint64_t sa[1] = {static_cast<uint64_t>(g.lda) * 2};
  const uint32_t ba[2] = {BK, 128};
  const uint64_t db[2] = {static_cast<uint64_t>(g.K), static_cast<uint64_t>(g.N)};
  const uint64_t sb[1] = {static_cast<uint64_t>(g.ldb) * 2};
  const uint32_t bb[2] = {BK, 128};
  if (make_tmap_bf16(&ta, g.a, 2, da, sa, ba) || make_tmap_bf16(&tb, g.b, 2, db, sb, bb)) return -4;
  const int num_m = (g.M + 255) / 256;
  const int tiles = num_m * (g.N / C::BN) * (g.ep.splits > 1 ? g.ep.splits : 1);
  int clusters = num_sms / 2;
  clusters = tiles < clusters ? tiles : clusters;
  int group_m = static_cast<int>((48ll << 20) / (256ll * g.K * 2));
  group_m = group_m < 4 ? 4 : group_m;
  group_m = group_m > num_m ? num_m : group_m;
  return static_cast<int>(launch_pdl(k_gemm2<EPI>, dim3(clusters * 2), dim3(GEMM_THREADS), C::SMEM, st, ta, tb,
                                     g.M, g.N, g.K, group_m, g.ep, d_status));
}

static cudaError_t allow_smem_i8() {
  return cudaFuncSetAttribute(k_gemm2<EPI_I8_F32, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, Gemm2Cfg::SMEM);
}
template <int BN, int EPI>
static cudaError_t allow_smem_bn() {
  return cudaFuncSetAttribute(k_gemm<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN>::SMEM);
}
template <int EPI>
static cudaError_t allow_smem_pair() {
  return cudaFuncSetAttribute(k_gemm2<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, Gemm2Cfg::SMEM);
}

// The dynamic shared-memory limit of every GEMM instantiation, raised on the CURRENT device (the
// attribute belongs to one device's context, so each handle's device gets it at exn_open).
int gemm_prepare() {
  const cudaError_t e[] = {
      allow_smem_pair<EPI_QKV>(),        allow_smem_pair<EPI_SWIGLU>(),   allow_smem_pair<EPI_GATE_RESID>(),
      allow_smem_pair<EPI_F32>(),        allow_smem_pair<EPI_BF16>(),     allow_smem_pair<EPI_GELU_BF16>(),
      allow_smem_bn<256, EPI_QKV>(),     allow_smem_bn<256, EPI_SWIGLU>(), allow_smem_bn<64, EPI_PROJ>(),
      allow_smem_bn<256, EPI_GATE_RESID>(), allow_smem_bn<128, EPI_GATE_RESID>(), allow_smem_bn<256, EPI_F32>(),
      allow_smem_bn<64, EPI_F32>(),      allow_smem_bn<256, EPI_BF16>(),  allow_smem_bn<64, EPI_BF16>(),
      allow_smem_bn<256, EPI_GELU_BF16>(), allow_smem_i8()};
  for (cudaError_t x : e)
    if (x != cudaSuccess) return static_cast<int>(x);
  return 0;
}

// C[M x N] f32 = (A . B^T) * sa[row] * sb[col] with A [M][K] and B [N][K] int8 (tcgen05 kind::i8 on
// CTA pairs); the scales are g.ep.mod (A's rows) and g.ep.norm_q (B's rows)
int gemm_i8_launch(const GemmArgs& g, const int8_t* a, const int8_t* b, int* d_status, int num_sms, cudaStream_t st) {
  using C = Gemm2Cfg;
  if (g.M <= 0 || g.N % 256 || g.K % 128 || g.K <= 0 || num_sms < 2) return -1;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) return -1;
  CUtensorMap ta, tb;
  const uint64_t da[2] = {static_cast<uint64_t>(g.K), static_cast<uint64_t>(g.M)};
  const uint64_t sa[1] = {static_cast<uint64_t>(g.K)};
  const uint32_t ba[2] = {128, 128};
  const uint64_t db[2] = {static_cast<uint64_t>(g.K), static_cast<uint64_t>(g.N)};
  const uint64_t sb[1] = {static_cast<uint64_t>(g.K)};
  if (make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, 2, da, sa, ba, CU_TENSOR_MAP_SWIZZLE_128B) ||
      make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, 2, db, sb, ba, CU_TENSOR_MAP_SWIZZLE_128B))
    return -4;
  const int num_m = (g.M + 255) / 256;
  const int tiles = num_m * (g.N / C::BN);
  int clusters = num_sms / 2;
  clusters = tiles < clusters ? tiles : clusters;
  int group_m = static_cast<int>((48ll << 20) / (256ll * g.K));
  group_m = group_m < 4 ? 4 : group_m;
  group_m = group_m > num_m ? num_m : group_m;
  return static_cast<int>(launch_pdl(k_gemm2<EPI_I8_F32, true>, dim3(clusters * 2), dim3(GEMM_THREADS), C::SMEM, st,
                                     ta, tb, g.M, g.N, g.K, group_m, g.ep, d_status));
}

int gemm_launch(const GemmArgs& g, int* d_status, int num_sms, cudaStream_t st) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0 || g.K % BK) return -1;
  if ((reinterpret_cast<uintptr_t>(g.a) | reinterpret_cast<uintptr_t>(g.b)) & 15) return -1;
  if ((g.lda * 2) % 16 || (g.ldb * 2) % 16) return -1;
  if (g.ep.splits > 1) {  // split-K: fp32 partials from the pair kernel only
    if (g.epi != EPI_F32 || !g.pairs || g.N % 256 || num_sms < 2 || g.ep.splits > g.K / BK) return -1;
    return launch_pair<EPI_F32>(g, d_status, num_sms, st);
  }
  if (g.epi == EPI_QKV) {  // whole heads a tile: q, k and v widths multiples of 256, N their sum
    const int kvw = g.ep.kv_width > 0 ? g.ep.kv_width : g.ep.width;
    if (g.ep.width <= 0 || g.ep.width % 256 || kvw % 256 || g.N != g.ep.width + 2 * kvw) return -1;
  }
  // CTA pairs for 256 x 256 tiles where N allows -- unless (pairs 1) those tiles would not fill one
  // round of the SM pairs and the epilogue has a narrower one-CTA tile that does: then 128-row tiles
  // of 64 (F32, BF16) or 128 (GATE_RESID) columns (every tile shape gives the same bits)
  const bool narrow = g.pairs == 1 && (g.epi == EPI_F32 || g.epi == EPI_BF16 || g.epi == EPI_GATE_RESID) &&
                      ((g.M + 255) / 256) * (g.N / 256) < num_sms / 2;
  if (g.pairs && !narrow && g.N % 256 == 0 && num_sms >= 2) {
    switch (g.epi) {
      case EPI_QKV:
        if (g.ep.width % 256) return -1;
        return launch_pair<EPI_QKV>(g, d_status, num_sms, st);
      case EPI_SWIGLU: return launch_pair<EPI_SWIGLU>(g, d_status, num_sms, st);
      case EPI_GATE_RESID: return launch_pair<EPI_GATE_RESID>(g, d_status, num_sms, st);
      case EPI_F32: return launch_pair<EPI_F32>(g, d_status, num_sms, st);
      case EPI_BF16: return launch_pair<EPI_BF16>(g, d_status, num_sms, st);
      case EPI_GELU_BF16: return launch_pair<EPI_GELU_BF16>(g, d_status, num_sms, st);
      default: break;
    }
  }
  switch (g.epi) {
    case EPI_QKV:
      if (g.N % 256 || g.ep.width % 256) return -1;
      return launch_bn<256, EPI_QKV>(g, d_status, num_sms, st);
    case EPI_SWIGLU:
      if (g.N % 256) return -1;
      return launch_bn<256, EPI_SWIGLU>(g, d_status, num_sms, st);
    case EPI_PROJ:
      if (g.N != 64) return -1;
      return launch_bn<64, EPI_PROJ>(g, d_status, num_sms, st);
    case EPI_GATE_RESID:
      if (g.N % 256 == 0 && !narrow) return launch_bn<256, EPI_GATE_RESID>(g, d_status, num_sms, st);
      if (g.N % 128 == 0) return launch_bn<128, EPI_GATE_RESID>(g, d_status, num_sms, st);
      return -1;
    case EPI_F32:
      if (g.N % 256 == 0 && !narrow) return launch_bn<256, EPI_F32>(g, d_status, num_sms, st);
      if (g.N % 64 == 0) return launch_bn<64, EPI_F32>(g, d_status, num_sms, st);
      return -1;
    case EPI_BF16:
      if (g.N % 256 == 0 && !narrow) return launch_bn<256, EPI_BF16>(g, d_status, num_sms, st);
      if (g.N % 64 == 0) return launch_bn<64, EPI_BF16>(g, d_status, num_sms, st);
      return -1;
    case EPI_GELU_BF16:
      if (g.N % 256 == 0) return launch_bn<256, EPI_GELU_BF16>(g, d_status, num_sms, st);
      return -1;
  }
  return -1;
}

}  // namespace exn
