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
// share every K/V tile; when the last round of such pair items would fill at
// most half the SMs, each of its items runs as two CTAs of one tile (no
// ping-pong partner; the same per-row arithmetic).  Keys are taken 64 at a time ("units"; K and V are
// loaded 128 keys at a time, two units a load):
//   warp 0      TMA: Q_a, Q_b once; K_t, V_t (128 keys x 128 dims, bf16)
//               through a ring of 4 slots
//   warp 1, 2   tcgen05.mma for tile a, b: S_x(u) = Q_x K(u)^T (128 x 64,
//               fp32) into one of two TMEM buffers of tile x; O_x += P_x(u)
//               V(u) with P_x read from TMEM (A operand in TMEM)
//   warps 3..6  softmax of tile a, warps 7..10 of tile b: one query row per
//               thread straight from TMEM (32x32b loads); P_x(u) (bf16, two
//               per column) written over the first 32 columns of S_x(u)'s
//               buffer; O_x rescaled in TMEM only when the row maximum grows
//               by more than 2^8
// With two S buffers a tile, S_x(u+1) is already in TMEM when the softmax of
// unit u ends, and the MMA thread computes S_x(u+2) while the softmax of u+1
// runs: the tensor core is off the softmax's critical path.  The MMA thread
// issues S_x(u+2) right after PV_x(u) into the buffer P_x(u) occupies; the
// tensor core runs one thread's MMAs in order, so PV_x(u) reads P_x(u) before
// S_x(u+2) overwrites it.
// Each scheduler of the SM also runs two softmax warps (TMEM lane quarter q
// is reachable only from warps w with w % 4 == q), which leave an issuing
// thread few issue slots; one MMA thread per tile, on two schedulers, halves
// the instructions each must get through.
#include "exn_device.cuh"
#include "exn_internal.h"

namespace exn {

int make_tmap_bf16(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                   const uint32_t* box);

namespace {

constexpr int ATT_THREADS = 352;
constexpr int TILE = 128;                 // queries per tile, keys per K/V load
constexpr int UNIT = 64;                  // keys per S tile
constexpr int HALF = TILE * 128;          // bytes of one 64-column swizzled half of a 128 x 128 bf16 tile
constexpr int TILE_BYTES = 2 * HALF;      // 32 KB
constexpr int SLOTS = 4;                  // K_0 V_0 K_1 V_1 ... stream through 4 slots
constexpr int OFF_QA = 0, OFF_QB = TILE_BYTES, OFF_SLOT = 2 * TILE_BYTES, OFF_BAR = (2 + SLOTS) * TILE_BYTES;
constexpr int ATT_SMEM = OFF_BAR + 256 + 1024;
constexpr uint32_t IDESC_S = idesc_bf16(128, UNIT);
constexpr uint32_t IDESC_PV = idesc_bf16(128, 128, false, true);  // V is MN-major (dims contiguous)
constexpr float RESCALE_THRESHOLD = 8.0f;                          // log2 units

__device__ __forceinline__ int xa_lim(int g, int p, int l, int b0, int b1) {
  return g >= p ? l - 1 : (g >= b0 && g < b1 ? b1 - 1 : g);
}

// Sequence-parallel output: each query row goes to the rank that keeps it (peer memory)
struct SpOut {
  bf16* out[kMaxSp];
  int ld, col0, pl, pl_loc, nl, img0;
};

struct Bars {
  uint64_t q_full, slot_full[SLOTS], slot_empty[SLOTS];
  uint64_t s_full[2][2], p_full[2][2];  // [tile][S buffer]
  uint64_t pv_done[2];                  // one phase per PV_x(u); waited only with at most one PV in flight
  uint64_t o_full[2];                   // after the last PV_x
  uint64_t done[2];
  uint32_t tmem_slot;
  int abort_flag;
};

}  // namespace

__global__ void __launch_bounds__(ATT_THREADS, 1)
    k_attention(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, bf16* __restrict__ out, int nq, int q0, int p, int l,
                int b0, int b1, int width, float scale_log2, int qpairs, int heads, int kv_group, int n_pairs,
                const SpOut spo, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + OFF_BAR);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // work item: blocks below N_PAIRS take a pair of query tiles (a, b); each later block takes one
  // tile of a pair item (the last round of pair items split in two when that fills the SMs better)
  int item = blockIdx.x, tiles = 2, tile0 = 0;
  if (item >= n_pairs) {
    const int sgl = item - n_pairs;
    item = n_pairs + (sgl >> 1);
    tiles = 1;
    tile0 = sgl & 1;
  }
  const int qt = item % qpairs, head = (item / qpairs) % heads, sample = item / (qpairs * heads);
  const int qbase = qt * 2 * TILE + tile0 * TILE;  // first query row (within the pass) of tile a
  const int qlast = min(nq, qbase + tiles * TILE) - 1;
  const int last_key = xa_lim(q0 + qlast, p, l, b0, b1);
  const int nunits = last_key / UNIT + 1;   // 64-key units any row of the CTA sees
  const int nloads = (nunits + 1) / 2;      // 128-key K/V loads

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int i = 0; i < SLOTS; ++i) {
      mbar_init(&bars->slot_full[i], 1);
      mbar_init(&bars->slot_empty[i], tiles);  // a K or V tile is free once every tile's MMAs are done with it
    }
    for (int x = 0; x < 2; ++x) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(&bars->s_full[x][b], 1);
        mbar_init(&bars->p_full[x][b], 4);  // one arrival per softmax warp
      }
      mbar_init(&bars->pv_done[x], 1);
      mbar_init(&bars->o_full[x], 1);
      mbar_init(&bars->done[x], 1);
    }
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
  griddep_launch();
  // TMEM columns: S_a buffers [0,64) [64,128), S_b [128,192) [192,256), O_a [256,384), O_b [384,512)

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch(&tmQ);
      tma_prefetch(&tmK);
      tma_prefetch(&tmV);
      griddep_wait();  // Q, K and V are the previous kernel's output
      const int hx = head * 128, kx = (head / kv_group) * 128;  // this head's Q columns, its K/V head's
      mbar_arrive_expect_tx(&bars->q_full, tiles * TILE_BYTES);
      for (int x = 0; x < tiles; ++x)
        for (int hf = 0; hf < 2; ++hf)
          tma_load_3d(smem + (x ? OFF_QB : OFF_QA) + hf * HALF, &tmQ, &bars->q_full, hx + hf * 64, qbase + x * TILE,
                      sample);
      // load number t: K_{t/2} for even t, V_{t/2} for odd t; slot t % SLOTS, its (t / SLOTS)-th use
      int issued = 0;
      for (int t = 0; t < 2 * nloads; ++t) {
        const int slot = t % SLOTS;
        const uint32_t use = static_cast<uint32_t>(t / SLOTS);
        if (!mbar_wait(&bars->slot_empty[slot], (use & 1) ^ 1, abort_flag, status, STATUS_TIMEOUT_ATTN)) break;
        mbar_arrive_expect_tx(&bars->slot_full[slot], TILE_BYTES);
        const CUtensorMap* map = (t & 1) ? &tmV : &tmK;
        for (int hf = 0; hf < 2; ++hf)
          tma_load_3d(smem + OFF_SLOT + slot * TILE_BYTES + hf * HALF, map, &bars->slot_full[slot], kx + hf * 64,
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
  } else if (warp <= 2) {
    if (lane == 0 && warp - 1 < tiles) {
      // ---- the MMAs of tile x.  This thread shares its scheduler with two busy softmax warps, so
      // its instruction stream is kept short: descriptors are formed once, as 32-bit low words
      // over a common high word (every operand here is 128B-swizzled with 1024-byte 8-row
      // groups), and each MMA then costs a constant add per operand.
      const int x = warp - 1;
      const uint32_t dhi = static_cast<uint32_t>(sdesc_sw128(0, 16, 1024) >> 32);
      const uint32_t qlo = static_cast<uint32_t>(sdesc_sw128(smem_u32(smem + (x ? OFF_QB : OFF_QA)), 16, 1024));
      const uint32_t klo = static_cast<uint32_t>(sdesc_sw128(smem_u32(smem + OFF_SLOT), 16, 1024));    // K-major
      const uint32_t vlo = static_cast<uint32_t>(sdesc_sw128(smem_u32(smem + OFF_SLOT), HALF, 1024));  // MN-major
      const uint32_t s_tm = tmem + x * 128, o_tm = tmem + 256 + x * 128;
      // S_x(u) = Q_x K(u)^T: keys (u % 2) * 64 .. +63 of load 2 * (u / 2), into S buffer u % 2
      auto issue_s = [&](int u) {
        const uint32_t k = klo + ((((u >> 1) * 2) % SLOTS) * TILE_BYTES + (u & 1) * UNIT * 128) / 16;
        const uint32_t d = s_tm + (u & 1) * UNIT;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t o = ((kk >> 2) * HALF + (kk & 3) * 32) / 16;
          umma_ss_lo(d, qlo + o, k + o, dhi, IDESC_S, kk ? 1u : 0u);
        }
      };
      // O_x += P_x(u) V(u): P_x in TMEM at S buffer u % 2 (8 columns = 16 keys per instruction)
      auto issue_pv = [&](int u) {
        const uint32_t v = vlo + ((((u >> 1) * 2 + 1) % SLOTS) * TILE_BYTES + (u & 1) * UNIT * 128) / 16;
        const uint32_t a = s_tm + (u & 1) * UNIT;
#pragma unroll
        for (int kk = 0; kk < UNIT / 16; ++kk)
          umma_ts_lo(o_tm, a + kk * 8, v + kk * 2048 / 16, dhi, IDESC_PV, (u > 0 || kk) ? 1u : 0u);
      };
      auto wait_load = [&](int t) {
        return mbar_wait(&bars->slot_full[t % SLOTS], static_cast<uint32_t>(t / SLOTS) & 1, abort_flag, status,
                         STATUS_TIMEOUT_ATTN);
      };
      bool ok = mbar_wait(&bars->q_full, 0, abort_flag, status, STATUS_TIMEOUT_ATTN) && wait_load(0);
      if (ok) {
        tc_fence_after();
        for (int u = 0; u < 2 && u < nunits; ++u) {
          issue_s(u);
          umma_commit(&bars->s_full[x][u]);
        }
        umma_commit(&bars->slot_empty[0]);  // K_0: both its units issued
      }
      for (int u = 0; u < nunits && ok; ++u) {
        const int b = u & 1;
        const bool more = u + 2 < nunits;
        if (b == 0 && !(ok = wait_load(2 * (u >> 1) + 1))) break;  // V(u)
        if (!(ok = mbar_wait(&bars->p_full[x][b], static_cast<uint32_t>(u >> 1) & 1, abort_flag, status,
                             STATUS_TIMEOUT_ATTN)))
          break;
        tc_fence_after();
        issue_pv(u);
        umma_commit(&bars->pv_done[x]);
        if (u + 1 == nunits) umma_commit(&bars->o_full[x]);
        if (more) {
          if (b == 0 && !(ok = wait_load(2 * ((u + 2) >> 1)))) break;  // K(u + 2)
          issue_s(u + 2);
          umma_commit(&bars->s_full[x][b]);
        }
        // this tile's share of freeing the slots whose last reader was just issued
        if (b == 1 || u + 1 == nunits) umma_commit(&bars->slot_empty[(2 * (u >> 1) + 1) % SLOTS]);   // V(u)
        if (more && (b == 1 || u + 3 == nunits)) umma_commit(&bars->slot_empty[(2 * ((u + 2) >> 1)) % SLOTS]);
      }
      umma_commit(&bars->done[x]);  // every MMA queued above has finished before TMEM is released
      volatile int no_abort = 0;
      mbar_wait(&bars->done[x], 0, &no_abort, nullptr, 0);
    }
  } else if ((warp - 3) >> 2 < tiles) {
    // ---- softmax: tile x, TMEM lane quarter wq, query row r of the tile
    const int x = (warp - 3) >> 2;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const int qi = qbase + x * TILE + r;  // query index within the pass
    const int lim = xa_lim(q0 + qi, p, l, b0, b1);
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + x * 128;
    const uint32_t o_addr = tmem + lane_off + 256 + x * 128;
    float m = -INFINITY, lsum = 0.f;
    bool ok = true;
    const uint64_t sc2 = f2(scale_log2, scale_log2);
    // Ping-pong: this warp and the other tile's warp on the same scheduler (same lane quarter)
    // take turns with their exponentials, a then b, through two 64-thread named barriers.  Each
    // exp phase then has the scheduler's MUFU pipe to itself, and the two tiles stay half a unit
    // apart, so one tile's MMAs run during the other's softmax.  Every warp takes every
    // iteration and every turn, also after a failed wait (then with the work skipped), so no
    // partner is left waiting at a barrier.
    const uint32_t my_turn = (x ? 5u : 1u) + static_cast<uint32_t>(wq);
    const uint32_t other_turn = (x ? 1u : 5u) + static_cast<uint32_t>(wq);
    const bool pingpong = tiles == 2;  // a lone tile has the schedulers' MUFU pipes to itself
    if (pingpong && x == 1) asm volatile("bar.arrive %0, 64;" ::"r"(other_turn) : "memory");  // tile a goes first
    for (int u = 0; u < nunits; ++u) {
      const int b = u & 1;
      // the warp stays converged through the whole loop (warp-uniform waits and branches), so
      // the TMEM loads and stores need no __syncwarp
      ok = ok && mbar_wait_uniform(&bars->s_full[x][b], static_cast<uint32_t>(u >> 1) & 1, abort_flag, status,
                                   STATUS_TIMEOUT_ATTN);
      float s[UNIT];
      if (ok) {
        tc_fence_after();
        {
          uint32_t rr[UNIT];
          tmem_ld64_conv(s_addr + b * UNIT, rr);
#pragma unroll
          for (int i = 0; i < UNIT; ++i) s[i] = __uint_as_float(rr[i]);
        }
        const int key0 = u * UNIT;
        if (__any_sync(0xffffffffu, key0 + UNIT - 1 > lim)) {
#pragma unroll
          for (int c = 0; c < UNIT; ++c)
            if (key0 + c > lim) s[c] = -INFINITY;
        }
        // row maximum: 8 independent chains of 3-input maxima, then a tree
        float m8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = fmax3(s[i], s[8 + i], s[16 + i]);
#pragma unroll
        for (int c = 24; c < UNIT - 8; c += 16)
#pragma unroll
          for (int i = 0; i < 8; ++i) m8[i] = fmax3(m8[i], s[c + i], s[c + 8 + i]);
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = fmaxf(m8[i], s[UNIT - 8 + i]);
        const float mx = fmaxf(fmax3(m8[0], m8[1], m8[2]), fmax3(fmax3(m8[3], m8[4], m8[5]), m8[6], m8[7]));
        const float m_new = fmaxf(m, mx * scale_log2);
        const bool need = m_new > m + RESCALE_THRESHOLD;
        const float alpha = need ? fast_exp2(m - m_new) : 1.f;
        lsum *= alpha;
        m = need ? m_new : m;
        if (u > 0 && __any_sync(0xffffffffu, need)) {
          // O_x holds the sum through PV_x(u-1): wait for it, then scale in place.  PV_x(u-2)
          // has finished (it was queued before S_x(u), whose commit this softmax waited for), so
          // the parity of u-1 is unambiguous.
          ok = mbar_wait_uniform(&bars->pv_done[x], static_cast<uint32_t>(u - 1) & 1, abort_flag, status,
                                 STATUS_TIMEOUT_ATTN);
          if (ok) {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              uint32_t ov[32];
              tmem_ld32(o_addr + c * 32, ov);
#pragma unroll
              for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
              tmem_st32(o_addr + c * 32, ov);
            }
            tmem_st_wait();
          }
        }
      }
      if (pingpong) asm volatile("bar.sync %0, 64;" ::"r"(my_turn) : "memory");
      uint32_t pk[UNIT / 2];  // P as bf16 pairs: key 2c and 2c+1 in column c
      if (ok) {
        // x = s * scale - m and the row sums on paired f32 instructions (two keys per issue)
        const uint64_t nm2 = f2(-m, -m);
        uint64_t ps2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int c8 = 0; c8 < UNIT / 8; ++c8) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float x0, x1;
            f2_split(ffma2(f2(s[c8 * 8 + 2 * i], s[c8 * 8 + 2 * i + 1]), sc2, nm2), x0, x1);
            const float e0 = fast_exp2(x0), e1 = fast_exp2(x1);
            ps2[i] = fadd2(ps2[i], f2(e0, e1));
            pk[c8 * 4 + i] = pack_bf16x2(e0, e1);
          }
        }
        float a0, a1;
        f2_split(fadd2(fadd2(ps2[0], ps2[1]), fadd2(ps2[2], ps2[3])), a0, a1);
        lsum += a0 + a1;
      }
      if (pingpong && (x == 0 || u + 1 < nunits)) asm volatile("bar.arrive %0, 64;" ::"r"(other_turn) : "memory");
      if (ok) {
        tmem_st32_conv(s_addr + b * UNIT, pk);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full[x][b]);
      }
    }
    if (ok && mbar_wait_uniform(&bars->o_full[x], 0, abort_flag, status, STATUS_TIMEOUT_ATTN)) {
      tc_fence_after();
      const float inv = 1.f / lsum;
      bf16* dst;
      if (spo.out[0] != nullptr) {  // sequence-parallel: the row's owner, at this rank's head columns
        int owner, local;
        if (qi < spo.img0) {
          owner = qi / spo.pl;
          local = qi - owner * spo.pl;
        } else {
          const int i = qi - spo.img0;
          owner = i / spo.nl;
          local = spo.pl_loc + (i - owner * spo.nl);
        }
        dst = spo.out[owner < kMaxSp ? owner : 0] + static_cast<long long>(local) * spo.ld + spo.col0 + head * 128;
      } else {
        dst = out + (static_cast<long long>(sample) * nq + qi) * width + head * 128;
      }
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
      if (spo.out[0] != nullptr) __threadfence_system();  // peer stores performed before the pass's barrier
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

// The attention kernel's dynamic shared-memory limit, raised on the CURRENT device (a per-device
// attribute: each handle's device gets it at exn_open).
int attention_prepare() {
  return static_cast<int>(
      cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM));
}

int attention_launch(const AttnArgs& a, int* d_status, cudaStream_t st) {
  if (a.nq <= 0 || a.l <= 0 || a.width % 128 || a.heads * 128 != a.width || a.kv_rows < a.l) return -1;
  if (a.q0 + a.nq > a.l) return -1;
  const int kv_heads = a.kv_heads > 0 ? a.kv_heads : a.heads;
  if (a.heads % kv_heads) return -1;
  const int kvw = kv_heads * 128;
  CUtensorMap tq, tk, tv;
  const uint32_t box[3] = {64, TILE, 1};
  const uint64_t dq[3] = {static_cast<uint64_t>(a.width), static_cast<uint64_t>(a.nq),
                          static_cast<uint64_t>(a.batch)};
  const uint64_t sq[2] = {static_cast<uint64_t>(a.width) * 2, static_cast<uint64_t>(a.nq) * a.width * 2};
  const uint64_t dk[3] = {static_cast<uint64_t>(kvw), static_cast<uint64_t>(a.l), static_cast<uint64_t>(a.batch)};
  const uint64_t sk[2] = {static_cast<uint64_t>(kvw) * 2, static_cast<uint64_t>(a.kv_rows) * kvw * 2};
  if (make_tmap_bf16(&tq, a.q, 3, dq, sq, box) || make_tmap_bf16(&tk, a.k, 3, dk, sk, box) ||
      make_tmap_bf16(&tv, a.v, 3, dk, sk, box))
    return -4;
  // pair items (two query tiles a CTA); when the last round of them fills at most half the SMs,
  // its items run as two one-tile CTAs each (split_mode 0: pairs only, 1: every item split)
  const int qpairs = (a.nq + 2 * TILE - 1) / (2 * TILE);
  const int items = qpairs * a.heads * a.batch;
  int n_pairs = items;
  if (a.split_mode == 1) {
    n_pairs = 0;
  } else if (a.split_mode == 2 && a.sms > 0) {
    const int last = items % a.sms;
    if (last > 0 && 2 * last <= a.sms) n_pairs = items - last;
  }
  const dim3 grid(static_cast<unsigned>(n_pairs + 2 * (items - n_pairs)));
  SpOut spo;
  for (int i = 0; i < kMaxSp; ++i) spo.out[i] = a.sp_out[i];
  spo.ld = a.sp_ld;
  spo.col0 = a.sp_col0;
  spo.pl = a.sp_pl;
  spo.pl_loc = a.sp_pl_loc;
  spo.nl = a.sp_nl;
  spo.img0 = a.sp_img0;
  if (spo.out[0] != nullptr && (a.batch != 1 || spo.nl <= 0 || (spo.img0 > 0 && spo.pl <= 0))) return -1;
  return static_cast<int>(launch_pdl(k_attention, grid, dim3(ATT_THREADS), ATT_SMEM, st, tq, tk, tv, a.out, a.nq, a.q0,
                                     a.p, a.l, a.b0, a.b1, a.width, a.scale_log2, qpairs, a.heads, a.heads / kv_heads,
                                     n_pairs, spo, d_status));
}

}  // namespace exn
