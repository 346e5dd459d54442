// elementwise.cu -- the DiT's memory-bound kernels: LayerNorm x (1 + scale),
// txt_in's RMSNorm, the latent's channel-major -> row transpose, the RoPE
// table, the timestep embedding, the small M=2 products of the timestep MLP
// and modulation, and the weight conversions done once at load.
//
// Rows are read and written with 16-byte vector accesses; reductions are warp
// shuffles plus one shared-memory step.
#include <math.h>

#include "exn_device.cuh"
#include "exn_internal.h"

namespace exn {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// sum over a block of NW warps
template <int NW>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NW; ++i) t += red[i];
  return t;
}

constexpr int LN_THREADS = 128;
constexpr int LN_MAXV = 8;  // float4 per thread: width <= 4096

__global__ void __launch_bounds__(LN_THREADS) k_ln_mod(const float* __restrict__ x, bf16* __restrict__ y,
                                                      const float* __restrict__ scale, int mod_stride, int rows,
                                                      int width, int seg_in, int seg_out, int off, int n0, int p,
                                                      int single) {
  __shared__ float red[LN_THREADS / 32];
  griddep_launch();
  griddep_wait();  // x is the previous kernel's output, y its input
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int b = r / seg_in, t = r - b * seg_in;
  const long long xr = static_cast<long long>(b) * seg_out + off + t;
  const float4* xp = reinterpret_cast<const float4*>(x + xr * width);
  const float* sc = scale + (single ? 0 : (n0 + t < p ? mod_stride : 0));
  const int nv = width >> 2;
  float4 v[LN_MAXV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int idx = threadIdx.x + i * LN_THREADS;
    v[i] = idx < nv ? __ldg(xp + idx) : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  const float mean = block_sum<LN_THREADS / 32>(s, red) / static_cast<float>(width);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int idx = threadIdx.x + i * LN_THREADS;
    if (idx < nv) {
      const float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
      ss += (a * a + bb * bb) + (c * c + d * d);
    }
  }
  const float inv = rsqrtf(block_sum<LN_THREADS / 32>(ss, red) / static_cast<float>(width) + 1e-6f);
  uint2* yp = reinterpret_cast<uint2*>(y + static_cast<long long>(r) * width);
  const float4* sp = reinterpret_cast<const float4*>(sc);
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int idx = threadIdx.x + i * LN_THREADS;
    if (idx < nv) {
      const float4 m = __ldg(sp + idx);
      yp[idx] = make_uint2(pack_bf16x2((v[i].x - mean) * inv * (1.f + m.x), (v[i].y - mean) * inv * (1.f + m.y)),
                           pack_bf16x2((v[i].z - mean) * inv * (1.f + m.z), (v[i].w - mean) * inv * (1.f + m.w)));
    }
  }
}

__global__ void __launch_bounds__(LN_THREADS) k_rms(const float* __restrict__ x, const float* __restrict__ w,
                                                   bf16* __restrict__ y, int rows, int width) {
  __shared__ float red[LN_THREADS / 32];
  const int r = blockIdx.x;
  if (r >= rows) return;
  const float4* xp = reinterpret_cast<const float4*>(x + static_cast<long long>(r) * width);
  const int nv = width >> 2;
  float4 v[LN_MAXV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int idx = threadIdx.x + i * LN_THREADS;
    v[i] = idx < nv ? __ldg(xp + idx) : make_float4(0.f, 0.f, 0.f, 0.f);
    ss += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
  }
  const float inv = rsqrtf(block_sum<LN_THREADS / 32>(ss, red) / static_cast<float>(width) + 1e-6f);
  uint2* yp = reinterpret_cast<uint2*>(y + static_cast<long long>(r) * width);
  const float4* wp = reinterpret_cast<const float4*>(w);
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int idx = threadIdx.x + i * LN_THREADS;
    if (idx < nv) {
      const float4 m = __ldg(wp + idx);
      yp[idx] = make_uint2(pack_bf16x2(v[i].x * inv * m.x, v[i].y * inv * m.y),
                           pack_bf16x2(v[i].z * inv * m.z, v[i].w * inv * m.w));
    }
  }
}

// lat [B][C][ld], columns col0.. -> rows [B*n][C], 32 x 32 tiles through shared memory
__global__ void k_latent_rows(const float* __restrict__ lat, bf16* __restrict__ rows, int channels, int n, int ld,
                              int col0) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z, i0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const float* src = lat + static_cast<long long>(b) * channels * ld + col0;
  for (int k = threadIdx.y; k < 32; k += 8) {
    const int c = c0 + k, i = i0 + threadIdx.x;
    tile[k][threadIdx.x] = (c < channels && i < n) ? src[static_cast<long long>(c) * ld + i] : 0.f;
  }
  __syncthreads();
  bf16* dst = rows + static_cast<long long>(b) * n * channels;
  for (int k = threadIdx.y; k < 32; k += 8) {
    const int i = i0 + k, c = c0 + threadIdx.x;
    if (i < n && c < channels) dst[static_cast<long long>(i) * channels + c] = __float2bfloat16_rn(tile[threadIdx.x][k]);
  }
}

// host.lisp:32-50 (image-positions, dit-positions) and :19-30 (rope-table):
// one thread per (row, pair); pairs 0..7 axis 0 (16 dims), 8..35 axis 1,
// 36..63 axis 2 (56 each); theta 10000, angles in double.
__global__ void k_rope_table(float2* __restrict__ table, int r0, int count, int p, int h, int w, int ra, int rh,
                             int rw, int split, int r1) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= count * 64) return;
  const int i = idx >> 6, j = idx & 63;
  const int g = split > 0 ? (i < split ? r0 + i : r1 + (i - split)) : r0 + i;
  int pos[3];
  auto image = [&](int frame, int k, int hh, int ww) {
    const int rr = k / ww, cc = k - (k / ww) * ww;
    pos[0] = frame;
    pos[1] = rr - (hh - hh / 2);
    pos[2] = cc - (ww - ww / 2);
  };
  if (rh > 0) {  // edit: A text rows, the reference picture, the rest of the text, the target
    const int after = p - ra - rh * rw, start = ra + (rh > rw ? rh : rw);
    if (g < ra) {
      pos[0] = pos[1] = pos[2] = g;
    } else if (g < ra + rh * rw) {
      image(ra, g - ra, rh, rw);
    } else if (g < p) {
      pos[0] = pos[1] = pos[2] = start + (g - ra - rh * rw);
    } else {
      image(start + after, g - p, h, w);
    }
  } else if (g < p) {
    pos[0] = pos[1] = pos[2] = g;
  } else {
    image(p, g - p, h, w);
  }
  int axis, k, d;
  if (j < 8) {
    axis = 0; k = j; d = 16;
  } else if (j < 36) {
    axis = 1; k = j - 8; d = 56;
  } else {
    axis = 2; k = j - 36; d = 56;
  }
  const double omega = 1.0 / pow(10000.0, static_cast<double>(2 * k) / static_cast<double>(d));
  const double ang = static_cast<double>(pos[axis]) * omega;
  table[static_cast<long long>(i) * 64 + j] = make_float2(static_cast<float>(cos(ang)), static_cast<float>(sin(ang)));
}

// host.lisp:9-15: cos then sin of t times exp(-ln(10000) j / half); row 0 t = 1000 sigma, row 1 t = 0
__global__ void k_temb(float* emb, double t, int freq) {
  const int half = freq / 2;
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const double a = t * exp(-log(10000.0) * static_cast<double>(j) / static_cast<double>(half));
    emb[j] = static_cast<float>(cos(a));
    emb[half + j] = static_cast<float>(sin(a));
    emb[freq + j] = 1.f;
    emb[freq + half + j] = 0.f;
  }
}

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_MAXM = 2;
constexpr int GEMV_CHUNKS = 8;  // 16-byte weight loads a lane keeps in flight

// y[m][o] = act(sum_k x[m][k] W[o][k]), M <= 2: HBM-bound on W.  A warp owns
// ROWS consecutive output rows; each lane reads 16 contiguous weight bytes a
// chunk (Q8_0: half a block, the block scale shared by a lane pair; or 8
// bf16 / 4+4 f32) and issues GEMV_CHUNKS of them before using any, so a warp
// keeps 4 KB of the row in flight (the HBM latency is hidden by bytes in
// flight, not by arithmetic).  x (M x in floats) is staged in shared memory
// once per block, permuted so that the float4 j of a lane's chunk sits at
// ((chunk * J + j) * 32 + lane), J = EPC / 4: the 32 lanes of a warp then
// read 512 contiguous bytes per instruction (in x's own order a lane's 64
// contiguous bytes would put 16 lanes on the same 4 banks).  A lane adds its
// chunks in column order and the warp sum follows, so the result does not
// depend on ROWS.
template <int KIND, int RB>
__global__ void __launch_bounds__(GEMV_WARPS * 32, 2)
    k_gemv(const void* __restrict__ wv, const __half* __restrict__ wd, const float* __restrict__ x,
           float* __restrict__ y, int m, int in, int out, int act, int piece, int rows) {
  extern __shared__ float4 xs4[];
  constexpr int EPC = KIND == W_Q8 ? 16 : 8;  // weights a lane takes per chunk
  constexpr int J = EPC / 4;                  // float4 of x per lane per chunk
  const int row4 = (in + 32 * EPC - 1) / (32 * EPC) * 8 * EPC;  // float4 per row of x, whole chunks
  {
    // x into shared memory (permuted, above): consecutive threads fill consecutive float4 of
    // the permuted layout (conflict-free stores) and gather x from L2, 8 loads in flight each
    const int in4 = in / 4, n4 = m * row4;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int i0 = threadIdx.x; i0 < n4; i0 += 8 * blockDim.x) {
      float4 t[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = i0 + j * blockDim.x;
        const int mm = i / row4, p = i - mm * row4;
        const int ln = p & 31, cj = p >> 5, chunk = cj / J, jj = cj - chunk * J;
        const int k4 = (chunk * 32 * EPC + ln * EPC) / 4 + jj;  // float4 index of x's row
        t[j] = i < n4 && k4 < in4 ? __ldg(x4 + mm * in4 + k4) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = i0 + j * blockDim.x;
        if (i < n4) xs4[i] = t[j];
      }
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if constexpr (KIND == W_Q8) {
    // RB rows at a time share each chunk of x read from shared memory; RB x CH = 8 16-byte
    // loads per lane in flight
    constexpr int CH = GEMV_CHUNKS / RB;
    const int8_t* qbase = static_cast<const int8_t*>(wv);
    for (int r0 = 0; r0 < rows; r0 += RB) {
      const int o0 = (blockIdx.x * GEMV_WARPS + warp) * rows + r0;
      if (o0 >= out) return;
      float acc[RB][GEMV_MAXM];
#pragma unroll
      for (int r = 0; r < RB; ++r)
#pragma unroll
        for (int mm = 0; mm < GEMV_MAXM; ++mm) acc[r][mm] = 0.f;
      for (int kb = 0; kb < in; kb += 32 * EPC * CH) {
        int4 qv[RB][CH];
        float sc[RB][CH];
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          const bool rv = r0 + r < rows && o0 + r < out;
          const long long o = o0 + r;
#pragma unroll
          for (int c = 0; c < CH; ++c) {
            const int k0 = kb + c * 32 * EPC + lane * EPC;
            const bool v = rv && k0 < in;
            qv[r][c] = v ? __ldg(reinterpret_cast<const int4*>(qbase + o * in + k0)) : make_int4(0, 0, 0, 0);
            sc[r][c] = v ? __half2float(wd[o * (in / 32) + (k0 >> 5)]) : 0.f;
          }
        }
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int k0 = kb + c * 32 * EPC + lane * EPC;
          if (k0 >= in) break;
          const float4* xc = xs4 + ((kb / (32 * EPC) + c) * J) * 32 + lane;  // this lane's chunk of x row 0
          float4 xv[GEMV_MAXM][4];
#pragma unroll
          for (int mm = 0; mm < GEMV_MAXM; ++mm)
#pragma unroll
            for (int k = 0; k < 4; ++k) xv[mm][k] = mm < m ? xc[mm * row4 + k * 32] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int r = 0; r < RB; ++r) {
            const int qw[4] = {qv[r][c].x, qv[r][c].y, qv[r][c].z, qv[r][c].w};
            // int8 -> float exactly without the conversion unit: with its sign bit flipped a byte
            // is q + 128 in 0..255; placed as the low mantissa byte of 2^23 (0x4B000000) it reads
            // as the float 2^23 + q + 128, and subtracting 2^23 + 128 leaves q
            float wf[16];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t u = static_cast<uint32_t>(qw[k]) ^ 0x80808080u;
              wf[4 * k] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.f;
              wf[4 * k + 1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.f;
              wf[4 * k + 2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.f;
              wf[4 * k + 3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.f;
            }
#pragma unroll
            for (int mm = 0; mm < GEMV_MAXM; ++mm) {
              if (mm < m) {
                float s = 0.f;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  s += wf[4 * k] * xv[mm][k].x;
                  s += wf[4 * k + 1] * xv[mm][k].y;
                  s += wf[4 * k + 2] * xv[mm][k].z;
                  s += wf[4 * k + 3] * xv[mm][k].w;
                }
                acc[r][mm] += sc[r][c] * s;
              }
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        if (r0 + r >= rows || o0 + r >= out) break;
        const int o = o0 + r;
#pragma unroll
        for (int mm = 0; mm < GEMV_MAXM; ++mm) {
          if (mm >= m) break;
          float v = warp_sum(acc[r][mm]);
          if (lane == 0) {
            if (act == 1) v = v / (1.f + expf(-v));
            if (act == 2) {
              const int pc = o / piece;
              if (pc == 1 || pc == 3) v = tanhf(v);
            }
            y[static_cast<long long>(mm) * out + o] = v;
          }
        }
      }
    }
  } else {
  for (int rr = 0; rr < rows; ++rr) {
    const int o = (blockIdx.x * GEMV_WARPS + warp) * rows + rr;
    if (o >= out) return;
    float acc[GEMV_MAXM] = {0.f, 0.f};
    for (int kb = 0; kb < in; kb += 32 * EPC * GEMV_CHUNKS) {
      {
        uint4 raw[GEMV_CHUNKS][KIND == W_F32 ? 2 : 1];
#pragma unroll
        for (int c = 0; c < GEMV_CHUNKS; ++c) {
          const int k0 = kb + c * 32 * EPC + lane * EPC;
          if constexpr (KIND == W_BF16) {
            raw[c][0] = k0 < in ? __ldg(reinterpret_cast<const uint4*>(static_cast<const bf16*>(wv) +
                                                                      static_cast<long long>(o) * in + k0))
                                : make_uint4(0, 0, 0, 0);
          } else {
            const uint4* fp =
                reinterpret_cast<const uint4*>(static_cast<const float*>(wv) + static_cast<long long>(o) * in + k0);
            raw[c][0] = k0 < in ? __ldg(fp) : make_uint4(0, 0, 0, 0);
            raw[c][KIND == W_F32 ? 1 : 0] = k0 < in ? __ldg(fp + 1) : make_uint4(0, 0, 0, 0);
          }
        }
#pragma unroll
        for (int c = 0; c < GEMV_CHUNKS; ++c) {
          const int k0 = kb + c * 32 * EPC + lane * EPC;
          if (k0 >= in) break;
          float wf[8];
          if constexpr (KIND == W_BF16) {
            const bf16* bp = reinterpret_cast<const bf16*>(&raw[c][0]);
#pragma unroll
            for (int e = 0; e < 8; ++e) wf[e] = __bfloat162float(bp[e]);
          } else {
            const float* f0 = reinterpret_cast<const float*>(&raw[c][0]);
            const float* f1 = reinterpret_cast<const float*>(&raw[c][KIND == W_F32 ? 1 : 0]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              wf[e] = f0[e];
              wf[4 + e] = f1[e];
            }
          }
          const float4* xc = xs4 + ((kb / (32 * EPC) + c) * J) * 32 + lane;
          for (int mm = 0; mm < m; ++mm) {
            const float4 xa = xc[mm * row4], xb = xc[mm * row4 + 32];
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            float s = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) s += wf[e] * xv[e];
            acc[mm] += s;
          }
        }
      }
    }
    for (int mm = 0; mm < m; ++mm) {
      float v = warp_sum(acc[mm]);
      if (lane == 0) {
        if (act == 1) v = v / (1.f + expf(-v));
        if (act == 2) {
          const int pc = o / piece;
          if (pc == 1 || pc == 3) v = tanhf(v);
        }
        y[static_cast<long long>(mm) * out + o] = v;
      }
    }
  }
  }
}

// One CTA waits, through the pipelines' own bounded wait, on an mbarrier that nothing arrives
// on: after LIMIT_NS the wait gives up, sets STATUS_TIMEOUT_PROBE and the kernel returns.  It
// shows on a GPU that a stalled pipeline ends in a status the host reads, not in a hang.
__global__ void k_wait_probe(int* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, status, STATUS_TIMEOUT_PROBE, limit_ns);
}

// One thread per rank g: store EPOCH into rank g's slot for this rank, then wait until rank g's
// arrival here shows EPOCH (epochs only grow).  Bounded: after LIMIT_NS the thread records
// STATUS_TIMEOUT_COMM and stops waiting, so a rank that died ends the pass with an error.
__global__ void k_sp_flag_barrier(const SpFlags f, int world, int epoch, int* status, unsigned long long limit_ns) {
  const int g = threadIdx.x;
  if (g < world) {
    __threadfence_system();
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(f.peer[g]), "r"(epoch) : "memory");
    const uint64_t t0 = globaltimer();
    while (true) {
      int v;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(f.mine + g) : "memory");
      if (v >= epoch) break;
      if (globaltimer() - t0 > limit_ns) {
        atomicOr(status, STATUS_TIMEOUT_COMM);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  __threadfence_system();
}

// destination row of weight row r: gate_up interleaved by 128 when ilv (= FFN) > 0
__device__ __forceinline__ long long dst_row(long long r, long long row0, int ilv) {
  if (ilv <= 0) return row0 + r;
  const long long g = r < ilv ? r : r - ilv;
  return row0 + (g / 128) * 256 + (r < ilv ? 0 : 128) + (g % 128);
}

__global__ void k_q8_raw_to_bf16(const uint8_t* __restrict__ raw, bf16* __restrict__ dst, long long rows, int cols,
                                 long long row0, int ilv) {
  const long long blk = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long nb = rows * (cols / 32);
  if (blk >= nb) return;
  const long long r = blk / (cols / 32);
  const int cb = static_cast<int>(blk - r * (cols / 32));
  const uint8_t* b = raw + blk * 34;
  const __half d = __ushort_as_half(static_cast<unsigned short>(b[0] | (b[1] << 8)));
  const float df = __half2float(d);
  uint32_t pk[16];
#pragma unroll
  for (int i = 0; i < 16; ++i)
    pk[i] = pack_bf16x2(static_cast<float>(static_cast<int8_t>(b[2 + 2 * i])) * df,
                        static_cast<float>(static_cast<int8_t>(b[3 + 2 * i])) * df);
  uint4* o = reinterpret_cast<uint4*>(dst + dst_row(r, row0, ilv) * cols + cb * 32);
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
}

__global__ void k_q8_raw_split(const uint8_t* __restrict__ raw, int8_t* __restrict__ qs, __half* __restrict__ d,
                               long long nblocks) {
  const long long blk = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (blk >= nblocks) return;
  const uint8_t* b = raw + blk * 34;
  d[blk] = __ushort_as_half(static_cast<unsigned short>(b[0] | (b[1] << 8)));
  for (int i = 0; i < 32; ++i) qs[blk * 32 + i] = static_cast<int8_t>(b[2 + i]);
}

__global__ void k_q8_to_bf16(const int8_t* __restrict__ qs, const __half* __restrict__ d, bf16* __restrict__ dst,
                             long long rows, int cols, long long row0, int ilv) {
  const long long blk = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long nb = rows * (cols / 32);
  if (blk >= nb) return;
  const long long r = blk / (cols / 32);
  const int cb = static_cast<int>(blk - r * (cols / 32));
  const float df = __half2float(d[blk]);
  const int8_t* q = qs + blk * 32;
  uint32_t pk[16];
#pragma unroll
  for (int i = 0; i < 16; ++i)
    pk[i] = pack_bf16x2(static_cast<float>(q[2 * i]) * df, static_cast<float>(q[2 * i + 1]) * df);
  uint4* o = reinterpret_cast<uint4*>(dst + dst_row(r, row0, ilv) * cols + cb * 32);
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
}

template <typename T>
__global__ void k_rows_to_bf16(const T* __restrict__ src, bf16* __restrict__ dst, long long rows, int cols,
                               long long row0, int ilv) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const long long r = i / cols;
  const int c = static_cast<int>(i - r * cols);
  float v;
  if constexpr (sizeof(T) == 4)
    v = src[i];
  else
    v = __bfloat162float(src[i]);
  dst[dst_row(r, row0, ilv) * cols + c] = __float2bfloat16_rn(v);
}

__global__ void k_f16_to_f32(const __half* __restrict__ s, float* __restrict__ d, long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) d[i] = __half2float(s[i]);
}

__global__ void k_bf16_to_f32(const bf16* __restrict__ s, float* __restrict__ d, long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) d[i] = __bfloat162float(s[i]);
}

__global__ void k_add_scalar(float* v, long long n, float a) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) v[i] = __fadd_rn(a, v[i]);
}

// The oracle's generator (oracle/dit_oracle.py synth_unit): splitmix64's
// finaliser of (stream << 32 | index) + seed * golden, four 16-bit fields
// summed, centred at 131070.
__device__ __forceinline__ int synth_offset(uint64_t seed, uint32_t stream, uint64_t idx) {
  uint64_t z = ((static_cast<uint64_t>(stream) << 32) | idx) + seed * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z = z ^ (z >> 31);
  const int s = static_cast<int>(z & 0xFFFF) + static_cast<int>((z >> 16) & 0xFFFF) +
                static_cast<int>((z >> 32) & 0xFFFF) + static_cast<int>(z >> 48);
  return s - 131070;
}

// gguf-py's Q8_0 (quantize_blocks) on the generated values, one thread per block of 32
__global__ void k_synth_q8(int8_t* __restrict__ qs, __half* __restrict__ d, long long n, uint64_t seed,
                           uint32_t stream, float scale) {
  const long long blk = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (blk * 32 >= n) return;
  float v[32];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = __fmul_rn(static_cast<float>(synth_offset(seed, stream, blk * 32 + i)), scale);
    amax = fmaxf(amax, fabsf(v[i]));
  }
  const float dd = __fdiv_rn(amax, 127.f);
  const float inv = dd == 0.f ? 0.f : __fdiv_rn(1.f, dd);
  uint32_t w[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    uint32_t acc = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int q = static_cast<int>(roundf(__fmul_rn(v[4 * k + e], inv)));
      acc |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * e);
    }
    w[k] = acc;
  }
  int4* o = reinterpret_cast<int4*>(qs + blk * 32);
  o[0] = make_int4(w[0], w[1], w[2], w[3]);
  o[1] = make_int4(w[4], w[5], w[6], w[7]);
  d[blk] = __float2half_rn(dd);
}

__global__ void k_synth_f32(float* __restrict__ v, long long n, uint64_t seed, uint32_t stream, float scale,
                            float base) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) v[i] = __fadd_rn(base, __fmul_rn(static_cast<float>(synth_offset(seed, stream, i)), scale));
}

// An order-independent digest of N 8-byte words: the sum of a mix of each word with its index.
__global__ void k_digest(const uint64_t* __restrict__ p, long long n, unsigned long long* out) {
  unsigned long long acc = 0;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    uint64_t z = p[i] ^ (static_cast<uint64_t>(i) * 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    acc += z ^ (z >> 31);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(out, acc);
}

inline unsigned blocks_for(long long n, int t) { return static_cast<unsigned>((n + t - 1) / t); }

}  // namespace

void ln_mod_launch(const float* x, bf16* y, const float* scale, int mod_stride, int rows, int width, int seg_in,
                   int seg_out, int off, int n0, int p, int single, cudaStream_t st) {
  if (rows <= 0) return;
  launch_pdl(k_ln_mod, dim3(rows), dim3(LN_THREADS), 0, st, x, y, scale, mod_stride, rows, width, seg_in, seg_out, off,
             n0, p, single);
}

void rms_launch(const float* x, const float* w, bf16* y, int rows, int width, cudaStream_t st) {
  if (rows <= 0) return;
  k_rms<<<rows, LN_THREADS, 0, st>>>(x, w, y, rows, width);
}

void latent_rows_launch(const float* lat, bf16* rows, int batch, int channels, int n, cudaStream_t st, int ld,
                        int i0) {
  dim3 grid((n + 31) / 32, (channels + 31) / 32, batch);
  k_latent_rows<<<grid, dim3(32, 8), 0, st>>>(lat, rows, channels, n, ld > 0 ? ld : n, i0);
}

void rope_table_launch(float2* table, int r0, int count, int p, int h, int w, int ref_a, int ref_h, int ref_w,
                       cudaStream_t st, int split, int r1) {
  if (count <= 0) return;
  k_rope_table<<<blocks_for(static_cast<long long>(count) * 64, 256), 256, 0, st>>>(table, r0, count, p, h, w, ref_a,
                                                                                    ref_h, ref_w, split, r1);
}

void temb_launch(float* emb, double sigma, int freq, cudaStream_t st) {
  k_temb<<<1, 128, 0, st>>>(emb, 1000.0 * sigma, freq);
}

int gemv_launch(int kind, const void* w, const __half* wd, const float* x, float* y, int m, int in, int out, int act,
                int piece, cudaStream_t st) {
  // rows a warp owns: 4 (a group of rows sharing each x read) when that still leaves >= 2 blocks
  // per SM of a 148-SM part, else 1 (x is staged once a block)
  const int rows = blocks_for(out, GEMV_WARPS * 4) >= 2 * 148 ? 4 : 1;
  const unsigned grid = blocks_for(out, GEMV_WARPS * rows);
  const int epc = kind == W_Q8 ? 16 : 8;  // x is staged in whole chunks of 32 lanes x epc floats
  const size_t sm = static_cast<size_t>(m) * ((in + 32 * epc - 1) / (32 * epc)) * (32 * epc) * sizeof(float);
  if (m < 1 || m > GEMV_MAXM || sm > 48 * 1024) return -1;  // x is staged whole in the default 48 KB
  if (kind == W_Q8 && rows == 4)
    k_gemv<W_Q8, 4><<<grid, GEMV_WARPS * 32, sm, st>>>(w, wd, x, y, m, in, out, act, piece, rows);
  else if (kind == W_Q8)
    k_gemv<W_Q8, 1><<<grid, GEMV_WARPS * 32, sm, st>>>(w, wd, x, y, m, in, out, act, piece, rows);
  else if (kind == W_BF16)
    k_gemv<W_BF16, 1><<<grid, GEMV_WARPS * 32, sm, st>>>(w, wd, x, y, m, in, out, act, piece, rows);
  else
    k_gemv<W_F32, 1><<<grid, GEMV_WARPS * 32, sm, st>>>(w, wd, x, y, m, in, out, act, piece, rows);
  return static_cast<int>(cudaGetLastError());
}

void q8_raw_to_bf16_launch(const uint8_t* raw, bf16* dst, long long rows, int cols, long long row0, int ilv,
                           cudaStream_t st) {
  const long long nb = rows * (cols / 32);
  k_q8_raw_to_bf16<<<blocks_for(nb, 256), 256, 0, st>>>(raw, dst, rows, cols, row0, ilv);
}

void q8_raw_split_launch(const uint8_t* raw, int8_t* qs, __half* d, long long nblocks, cudaStream_t st) {
  k_q8_raw_split<<<blocks_for(nblocks, 256), 256, 0, st>>>(raw, qs, d, nblocks);
}

void q8_to_bf16_launch(const int8_t* qs, const __half* d, bf16* dst, long long rows, int cols, long long row0,
                       int ilv, cudaStream_t st) {
  const long long nb = rows * (cols / 32);
  k_q8_to_bf16<<<blocks_for(nb, 256), 256, 0, st>>>(qs, d, dst, rows, cols, row0, ilv);
}

void f32_to_bf16_rows_launch(const float* src, bf16* dst, long long rows, int cols, long long row0, int ilv,
                             cudaStream_t st) {
  k_rows_to_bf16<float><<<blocks_for(rows * cols, 256), 256, 0, st>>>(src, dst, rows, cols, row0, ilv);
}

void bf16_rows_launch(const bf16* src, bf16* dst, long long rows, int cols, long long row0, int ilv,
                      cudaStream_t st) {
  k_rows_to_bf16<bf16><<<blocks_for(rows * cols, 256), 256, 0, st>>>(src, dst, rows, cols, row0, ilv);
}

void f16_to_f32_launch(const __half* src, float* dst, long long n, cudaStream_t st) {
  k_f16_to_f32<<<blocks_for(n, 256), 256, 0, st>>>(src, dst, n);
}

void bf16_to_f32_launch(const bf16* src, float* dst, long long n, cudaStream_t st) {
  k_bf16_to_f32<<<blocks_for(n, 256), 256, 0, st>>>(src, dst, n);
}

void digest_launch(const void* p, size_t bytes, unsigned long long* out, cudaStream_t st) {
  const long long n = static_cast<long long>(bytes / 8);
  if (n <= 0) return;
  k_digest<<<static_cast<unsigned>(n < 148LL * 2048 ? blocks_for(n, 256) : 148 * 8), 256, 0, st>>>(
      static_cast<const uint64_t*>(p), n, out);
}

int sp_flag_barrier_launch(const SpFlags& f, int world, int epoch, int* status, cudaStream_t st) {
  if (world < 1 || world > kMaxSp) return -1;
  k_sp_flag_barrier<<<1, 32, 0, st>>>(f, world, epoch, status, 4000000000ull);
  return static_cast<int>(cudaGetLastError());
}

void wait_probe_launch(int* status, unsigned long long limit_ns, cudaStream_t st) {
  k_wait_probe<<<1, 32, 0, st>>>(status, limit_ns);
}

void add_scalar_launch(float* v, long long n, float a, cudaStream_t st) {
  k_add_scalar<<<blocks_for(n, 256), 256, 0, st>>>(v, n, a);
}

void synth_q8_launch(int8_t* qs, __half* d, long long n, uint64_t seed, uint32_t stream, float scale,
                     cudaStream_t st) {
  k_synth_q8<<<blocks_for(n / 32, 128), 128, 0, st>>>(qs, d, n, seed, stream, scale);
}

void synth_f32_launch(float* v, long long n, uint64_t seed, uint32_t stream, float scale, float base,
                      cudaStream_t st) {
  k_synth_f32<<<blocks_for(n, 256), 256, 0, st>>>(v, n, seed, stream, scale, base);
}

}  // namespace exn
