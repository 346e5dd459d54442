// encoder.cu -- the prompt encoder's memory-bound kernels (Qwen3-VL-8B's text
// model, src/encoder.lisp:143-183): the token embedding gather, the M-RoPE
// table, and the conversions of the fp32 embedding table.  The matrices run
// through the tcgen05 GEMM (gemm.cu) and the causal attention through
// attention.cu.
#include "exn_device.cuh"
#include "exn_internal.h"

namespace exn {

namespace {

// x f32 [n][width] = table f32 [vocab][width] at row ids[r]; one block a row
__global__ void k_enc_embed(const float* __restrict__ table, const int* __restrict__ ids, float* __restrict__ x,
                            int width) {
  const int r = blockIdx.x;
  const float4* src = reinterpret_cast<const float4*>(table + static_cast<long long>(__ldg(ids + r)) * width);
  float4* dst = reinterpret_cast<float4*>(x + static_cast<long long>(r) * width);
  for (int i = threadIdx.x; i < width / 4; i += blockDim.x) dst[i] = __ldg(src + i);
}

// table [n][64] float2 (cos, sin) of the angle pos[i][axis(j)] * theta^(-2j/128): Qwen3-VL's
// interleaved M-RoPE (src/encoder.lisp:26-39), axis(j) = j % 3 (t, h, w) below 60, t above; the
// angle in double precision
__global__ void k_enc_rope(const int* __restrict__ pos, float2* __restrict__ table, int n, double log_theta) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * 64) return;
  const int i = idx >> 6, j = idx & 63;
  const int axis = j < 60 ? j % 3 : 0;
  const double a = static_cast<double>(__ldg(pos + 3 * i + axis)) * exp(-(2.0 * j / 128.0) * log_theta);
  double s, c;
  sincos(a, &s, &c);
  table[idx] = make_float2(static_cast<float>(c), static_cast<float>(s));
}

// f32 out = qs * d: the Q8_0 value exactly (an int8 times an fp16 fits a float's mantissa)
__global__ void k_q8_to_f32(const int8_t* __restrict__ qs, const __half* __restrict__ d, float* __restrict__ out,
                            long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = static_cast<float>(qs[i]) * __half2float(d[i >> 5]);
}

// the same from GGUF's Q8_0 blocks (34 bytes: fp16 d, then 32 int8)
__global__ void k_q8_raw_to_f32(const uint8_t* __restrict__ raw, float* __restrict__ out, long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t* blk = raw + (i >> 5) * 34;
  const __half d = __ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8)));
  out[i] = static_cast<float>(static_cast<int8_t>(blk[2 + (i & 31)])) * __half2float(d);
}

// ---- the epilogues of a split-K GEMM: PART [splits][n][N] fp32 partials summed in split order.
// Every part's load is issued before the first sum (the loop bound is the largest split count, the
// parts beyond SPLITS predicated off), so a thread waits for memory once, not once a part.

// q / k / v: one warp a (row, head of 128 columns); q and k heads RMS-normed (eps 1e-6) times
// their weight and turned by RoPE on halves (dims j and j + 64 by angle j of ROPE [row][64]);
// lane l holds dims l, l + 32, l + 64, l + 96
__global__ void k_enc_qkv_sum(const float* __restrict__ part, int splits, int n, int qw, int kvw,
                              const float* __restrict__ norm_q, const float* __restrict__ norm_k,
                              const float2* __restrict__ rope, bf16* __restrict__ q, bf16* __restrict__ k,
                              bf16* __restrict__ v) {
  const int heads = (qw + 2 * kvw) / 128;
  const long long wid = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= static_cast<long long>(n) * heads) return;
  const int r = static_cast<int>(wid / heads), h = static_cast<int>(wid - static_cast<long long>(r) * heads);
  const int N = qw + 2 * kvw;
  const long long stride = static_cast<long long>(n) * N;
  const float* p = part + static_cast<long long>(r) * N + h * 128 + lane;
  float pv[kEncMaxSplits][4];
#pragma unroll
  for (int sp = 0; sp < kEncMaxSplits; ++sp)
    if (sp < splits)
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[sp][i] = p[sp * stride + 32 * i];
  float x[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = pv[0][i];
#pragma unroll
  for (int sp = 1; sp < kEncMaxSplits; ++sp)
    if (sp < splits)
#pragma unroll
      for (int i = 0; i < 4; ++i) x[i] += pv[sp][i];
  const int col = h * 128;
  const int sec = col < qw ? 0 : (col < qw + kvw ? 1 : 2);
  if (sec < 2) {
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / 128.f + 1e-6f);
    const float* w = sec == 0 ? norm_q : norm_k;
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = x[i] * inv * __ldg(w + lane + 32 * i);
    const float2 c0 = __ldg(rope + static_cast<long long>(r) * 64 + lane);
    const float2 c1 = __ldg(rope + static_cast<long long>(r) * 64 + lane + 32);
    const float a0 = x[0], b0 = x[2], a1 = x[1], b1 = x[3];
    x[0] = a0 * c0.x - b0 * c0.y;
    x[2] = a0 * c0.y + b0 * c0.x;
    x[1] = a1 * c1.x - b1 * c1.y;
    x[3] = a1 * c1.y + b1 * c1.x;
  }
  bf16* dst = sec == 0 ? q + static_cast<long long>(r) * qw + col
                       : (sec == 1 ? k + static_cast<long long>(r) * kvw + (col - qw)
                                   : v + static_cast<long long>(r) * kvw + (col - qw - kvw));
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = __float2bfloat16_rn(x[i]);
}

// one block of 1024 threads a row, a float4 of the row a thread: x [n][w] += the sum of the partials,
// then (NORM given) xn bf16 = x / sqrt(mean(x^2) + 1e-6) * norm, the next GEMM's operand; w <= 4096,
// a multiple of 4
__global__ void __launch_bounds__(1024) k_enc_resid_rms(const float* __restrict__ part, int splits, int n, int w,
                                                        float* __restrict__ x, const float* __restrict__ norm,
                                                        bf16* __restrict__ xn) {
  __shared__ float red[32];
  const int r = blockIdx.x, c = threadIdx.x;
  const int w4 = w / 4;
  const long long stride4 = static_cast<long long>(n) * w4;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  float ss = 0.f;
  if (c < w4) {
    const float4* p = reinterpret_cast<const float4*>(part) + static_cast<long long>(r) * w4 + c;
    float4* xr = reinterpret_cast<float4*>(x) + static_cast<long long>(r) * w4 + c;
    float4 pv[kEncMaxSplits];
#pragma unroll
    for (int sp = 0; sp < kEncMaxSplits; ++sp)
      if (sp < splits) pv[sp] = p[sp * stride4];
    o = *xr;
    float4 a = pv[0];
#pragma unroll
    for (int sp = 1; sp < kEncMaxSplits; ++sp)
      if (sp < splits) {
        a.x += pv[sp].x;
        a.y += pv[sp].y;
        a.z += pv[sp].z;
        a.w += pv[sp].w;
      }
    o.x += a.x;
    o.y += a.y;
    o.z += a.z;
    o.w += a.w;
    *xr = o;
    ss = (o.x * o.x + o.y * o.y) + (o.z * o.z + o.w * o.w);
  }
  if (norm == nullptr) return;
#pragma unroll
  for (int k = 16; k > 0; k >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, k);
  if ((c & 31) == 0) red[c >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) t += red[i];
  const float inv = rsqrtf(t / static_cast<float>(w) + 1e-6f);
  if (c < w4) {
    const float4 m = __ldg(reinterpret_cast<const float4*>(norm) + c);
    reinterpret_cast<uint2*>(xn + static_cast<long long>(r) * w)[c] =
        make_uint2(pack_bf16x2(o.x * inv * m.x, o.y * inv * m.y), pack_bf16x2(o.z * inv * m.z, o.w * inv * m.w));
  }
}

// h [n][ffn] bf16 = silu(gate) * up, the partials' columns gate and up interleaved by 128
__global__ void k_enc_swiglu_sum(const float* __restrict__ part, int splits, int n, int ffn, bf16* __restrict__ h) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(n) * ffn) return;
  const int r = static_cast<int>(i / ffn), j = static_cast<int>(i - static_cast<long long>(r) * ffn);
  const long long stride = static_cast<long long>(n) * 2 * ffn;
  const float* p = part + static_cast<long long>(r) * 2 * ffn + (j >> 7) * 256 + (j & 127);
  float pg[kEncMaxSplits], pu[kEncMaxSplits];
#pragma unroll
  for (int sp = 0; sp < kEncMaxSplits; ++sp)
    if (sp < splits) {
      pg[sp] = p[sp * stride];
      pu[sp] = p[sp * stride + 128];
    }
  float g = pg[0], u = pu[0];
#pragma unroll
  for (int sp = 1; sp < kEncMaxSplits; ++sp)
    if (sp < splits) {
      g += pg[sp];
      u += pu[sp];
    }
  h[i] = __float2bfloat16_rn(g / (1.f + expf(-g)) * u);
}

unsigned blocks(long long n, int t) { return static_cast<unsigned>((n + t - 1) / t); }

}  // namespace

void enc_embed_launch(const float* table, const int* ids, float* x, int n, int width, cudaStream_t st) {
  k_enc_embed<<<n, 256, 0, st>>>(table, ids, x, width);
}

void enc_rope_launch(const int* pos, float2* table, int n, double theta, cudaStream_t st) {
  k_enc_rope<<<blocks(static_cast<long long>(n) * 64, 256), 256, 0, st>>>(pos, table, n, log(theta));
}

void q8_to_f32_launch(const int8_t* qs, const __half* d, float* out, long long n, cudaStream_t st) {
  k_q8_to_f32<<<blocks(n, 256), 256, 0, st>>>(qs, d, out, n);
}

void q8_raw_to_f32_launch(const uint8_t* raw, float* out, long long n, cudaStream_t st) {
  k_q8_raw_to_f32<<<blocks(n, 256), 256, 0, st>>>(raw, out, n);
}

void enc_qkv_sum_launch(const float* part, int splits, int n, int qw, int kvw, const float* norm_q,
                        const float* norm_k, const float2* rope, bf16* q, bf16* k, bf16* v, cudaStream_t st) {
  const long long warps = static_cast<long long>(n) * ((qw + 2 * kvw) / 128);
  k_enc_qkv_sum<<<blocks(warps * 32, 256), 256, 0, st>>>(part, splits, n, qw, kvw, norm_q, norm_k, rope, q, k, v);
}

void enc_resid_rms_launch(const float* part, int splits, int n, int w, float* x, const float* norm, bf16* xn,
                          cudaStream_t st) {
  k_enc_resid_rms<<<n, 1024, 0, st>>>(part, splits, n, w, x, norm, xn);
}

void enc_swiglu_sum_launch(const float* part, int splits, int n, int ffn, bf16* h, cudaStream_t st) {
  k_enc_swiglu_sum<<<blocks(static_cast<long long>(n) * ffn, 256), 256, 0, st>>>(part, splits, n, ffn, h);
}

}  // namespace exn
