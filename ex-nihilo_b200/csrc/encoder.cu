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

}  // namespace exn
