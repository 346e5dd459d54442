// vae.cu -- the VAE decoder's memory-bound kernels, channels last: the
// RMS norm (with SiLU) that feeds each convolution, the nearest 2x upsample,
// the attention's row softmax and transpose, and the weights' reorder at
// load.  They replace the reference's v_rms + x_silu, x_up2, x_softmax_rows,
// x_transpose (src/cuda/vae.cu:143-214, illatio's v_rms; called from
// src/cuda-vae.lisp:37-136) with the shapes of inspect/ref_vae.py:42-88.
// Wan's DupUp3D shortcut (x_dupup_add) is added in the upsampling
// convolution's epilogue (conv.cu).
#include <math.h>

#include "exn_device.cuh"
#include "exn_internal.h"

namespace exn {

namespace {

__device__ __forceinline__ float warp_sum32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// one warp per pixel: y = x / max(|x|, 1e-12) * sqrt(c) * gamma (ref_vae.py:47-49), SiLU on request
__global__ void k_vae_norm(const float* __restrict__ x, const float* __restrict__ gamma, bf16* __restrict__ y, int n,
                           int c, int cp, int silu) {
  const int pix = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (pix >= n) return;
  const float4* xp = reinterpret_cast<const float4*>(x + static_cast<long long>(pix) * c);
  const int c4 = c >> 2;
  float ss = 0.f;
  for (int i = lane; i < c4; i += 32) {
    const float4 v = __ldg(xp + i);
    ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
  }
  ss = warp_sum32(ss);
  const float scale = sqrtf(static_cast<float>(c)) / fmaxf(sqrtf(ss), 1e-12f);
  uint2* yp = reinterpret_cast<uint2*>(y + static_cast<long long>(pix) * cp);
  const float4* gp = reinterpret_cast<const float4*>(gamma);
  for (int i = lane; i < (cp >> 2); i += 32) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < c4) {
      const float4 a = __ldg(xp + i), g = __ldg(gp + i);
      v = make_float4(a.x * scale * g.x, a.y * scale * g.y, a.z * scale * g.z, a.w * scale * g.w);
      if (silu) {
        v.x = v.x / (1.f + expf(-v.x));
        v.y = v.y / (1.f + expf(-v.y));
        v.z = v.z / (1.f + expf(-v.z));
        v.w = v.w / (1.f + expf(-v.w));
      }
    }
    yp[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

// y bf16 [n][cp] = x f32 [n][c] (channels c .. cp-1 zero), 4 channels a thread
__global__ void k_vae_to_bf16(const float* __restrict__ x, bf16* __restrict__ y, long long n, int c, int cp) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int cp4 = cp >> 2;
  if (i >= n * cp4) return;
  const int ch = static_cast<int>(i % cp4) * 4;
  const long long pix = i / cp4;
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (ch < c) v = __ldg(reinterpret_cast<const float4*>(x + pix * c + ch));
  reinterpret_cast<uint2*>(y)[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
}

// u [2h][2w][cp] = x [h][w][c] repeated 2 x 2 (ref_vae.py:99), 4 channels a thread
__global__ void k_vae_up2(const float* __restrict__ x, bf16* __restrict__ u, int h, int w, int c, int cp) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int cp4 = cp >> 2;
  const long long total = 4LL * h * w * cp4;
  if (i >= total) return;
  const int ch = static_cast<int>(i % cp4) * 4;
  const long long op = i / cp4;
  const int ox = static_cast<int>(op % (2 * w)), oy = static_cast<int>(op / (2 * w));
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (ch < c) v = __ldg(reinterpret_cast<const float4*>(x + (static_cast<long long>(oy >> 1) * w + (ox >> 1)) * c + ch));
  reinterpret_cast<uint2*>(u)[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
}

// one block of 256 threads per row: p = softmax(s * scale) (ref_vae.py:70-71), bf16 out
__global__ void __launch_bounds__(256) k_vae_softmax(const float* __restrict__ s, bf16* __restrict__ p, int n,
                                                     float scale) {
  __shared__ float red[8];
  const float* row = s + static_cast<long long>(blockIdx.x) * n;
  float m = -INFINITY;
  for (int j = threadIdx.x; j < n; j += 256) m = fmaxf(m, row[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int k = 1; k < 8; ++k) m = fmaxf(m, red[k]);
  __syncthreads();
  float sum = 0.f;
  for (int j = threadIdx.x; j < n; j += 256) sum += expf((row[j] - m) * scale);
  sum = warp_sum32(sum);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) t += red[k];
  const float inv = 1.f / t;
  bf16* out = p + static_cast<long long>(blockIdx.x) * n;
  for (int j = threadIdx.x; j < n; j += 256) out[j] = __float2bfloat16_rn(expf((row[j] - m) * scale) * inv);
}

// out [c][n] = in [n][c] (row stride ld_in), 32 x 32 tiles through shared memory
__global__ void k_vae_transpose(const bf16* __restrict__ in, long long ld_in, bf16* __restrict__ out, int n, int c) {
  __shared__ bf16 tile[32][34];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int k = threadIdx.y; k < 32; k += 8) {
    const int r = r0 + k, cc = c0 + threadIdx.x;
    tile[k][threadIdx.x] = (r < n && cc < c) ? in[static_cast<long long>(r) * ld_in + cc] : __float2bfloat16_rn(0.f);
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += 8) {
    const int cc = c0 + k, r = r0 + threadIdx.x;
    if (cc < c && r < n) out[static_cast<long long>(cc) * n + r] = tile[threadIdx.x][k];
  }
}

// w [o][i][taps] f32 -> out [rows][taps][cp] bf16 (round to nearest); padding rows and channels zero
__global__ void k_vae_weight(const float* __restrict__ w, bf16* __restrict__ out, int o, int i, int taps, int rows,
                             int cp) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(rows) * taps * cp;
  if (idx >= total) return;
  const int ci = static_cast<int>(idx % cp);
  const long long rt = idx / cp;
  const int t = static_cast<int>(rt % taps), r = static_cast<int>(rt / taps);
  const float v = (r < o && ci < i) ? w[(static_cast<long long>(r) * i + ci) * taps + t] : 0.f;
  out[idx] = __float2bfloat16_rn(v);
}

// v = (float) bf16 (v), round to nearest even, in place
__global__ void k_round_bf16(float* v, long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) v[i] = __bfloat162float(__float2bfloat16_rn(v[i]));
}

inline unsigned nblocks(long long n, int t) { return static_cast<unsigned>((n + t - 1) / t); }

}  // namespace

void vae_norm_launch(const float* x, const float* gamma, bf16* y, int n, int c, int cp, int silu, cudaStream_t st) {
  if (n <= 0) return;
  k_vae_norm<<<nblocks(n, 8), 256, 0, st>>>(x, gamma, y, n, c, cp, silu);
}

void round_bf16_launch(float* v, long long n, cudaStream_t st) {
  if (n > 0) k_round_bf16<<<nblocks(n, 256), 256, 0, st>>>(v, n);
}

void vae_to_bf16_launch(const float* x, bf16* y, long long n, int c, int cp, cudaStream_t st) {
  const long long total = n * (cp / 4);
  k_vae_to_bf16<<<nblocks(total, 256), 256, 0, st>>>(x, y, n, c, cp);
}

void vae_up2_launch(const float* x, bf16* u, int h, int w, int c, int cp, cudaStream_t st) {
  const long long total = 4LL * h * w * (cp / 4);
  k_vae_up2<<<nblocks(total, 256), 256, 0, st>>>(x, u, h, w, c, cp);
}

void vae_softmax_launch(const float* s, bf16* p, int n, float scale, cudaStream_t st) {
  k_vae_softmax<<<n, 256, 0, st>>>(s, p, n, scale);
}

void vae_transpose_launch(const bf16* in, long long ld_in, bf16* out, int n, int c, cudaStream_t st) {
  k_vae_transpose<<<dim3(nblocks(c, 32), nblocks(n, 32)), dim3(32, 8), 0, st>>>(in, ld_in, out, n, c);
}

void vae_weight_launch(const float* w, bf16* out, int o, int i, int taps, int rows, int cp, cudaStream_t st) {
  const long long total = static_cast<long long>(rows) * taps * cp;
  k_vae_weight<<<nblocks(total, 256), 256, 0, st>>>(w, out, o, i, taps, rows, cp);
}

}  // namespace exn
