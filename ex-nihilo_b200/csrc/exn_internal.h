// exn_internal.h -- declarations shared by the kernels (.cu) and the host
// driver (dit.cpp).  Not part of the public C ABI (include/exn_b200.h).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace exn {

typedef __nv_bfloat16 bf16;

// What a GEMM's epilogue does with the fp32 accumulator tile.
enum EpiKind : int {
  EPI_F32 = 0,         // out f32 at the mapped row
  EPI_BF16 = 1,        // out bf16 at the mapped row
  EPI_GELU_BF16 = 2,   // out bf16 = gelu_tanh(acc)                          (txt_in.in_layer)
  EPI_QKV = 3,         // q/k: per-head RMSNorm * w, RoPE; v: as is -> bf16  (fused to_q/to_k/to_v)
  EPI_GATE_RESID = 4,  // x[row] += tanh(gate)[mod row] * acc, f32           (to_out.0, img_mlp.out)
  EPI_SWIGLU = 5,      // out bf16 = silu(gate) * up, gate/up interleaved by 128 columns (img_mlp.gate_up)
  EPI_PROJ = 6,        // v channel-major and/or z += dsigma * v              (proj_out)
  EPI_I8_F32 = 7,      // int8 product: f32 out = acc * mod[row] * norm_q[col] (a measured experiment)
};

// ranks of a sequence-parallel group that kernels address directly (peer pointers)
constexpr int kMaxSp = 16;

// Launch KERNEL with programmatic dependent launch allowed: it may begin while the previous kernel
// on ST finishes; the kernel itself must call griddep_wait (exn_device.cuh) before touching
// anything the previous kernel reads or writes.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// GEMM row r maps to output row
//   (r / seg_in) * seg_out + off + t + (t >= split_at ? split_gap : 0),  t = r % seg_in
struct GemmEpi {
  void* out = nullptr;
  long long ld_out = 0;
  int seg_in = 1 << 30, seg_out = 0, off = 0, split_at = 1 << 30, split_gap = 0;
  // modulation rows [2][mod_stride]: row 0 (from t) for image rows, row 1 (from 0) for prompt rows;
  // a row t of a sample is a prompt row when n0 + t < p
  const float* mod = nullptr;
  int mod_stride = 0, n0 = 0, p = 0;
  // EPI_QKV
  int width = 0;
  const float* norm_q = nullptr;
  const float* norm_k = nullptr;
  const float2* rope = nullptr;  // [sequence row][64] (cos, sin)
  bf16* q = nullptr;
  bf16* k = nullptr;
  bf16* v = nullptr;
  long long kv_sample_stride = 0;  // elements from one sample's K (V) rows to the next
  // grouped K/V (the prompt encoder): columns [0, width) are q, then kv_width of k and of v, each
  // stored with row stride kv_width (0: kv_width = width)
  int kv_width = 0;
  int rope_halves = 0;             // 0: dims (2j, 2j+1) turn by angle j; 1: dims (j, j+64)
  // split-K (EPI_F32 on CTA pairs): part s of the k-blocks of every tile into output rows s * M ..,
  // fp32 partials the caller sums (1: no split)
  int splits = 1;
  // EPI_QKV, sequence-parallel (group_w > 0): the tile's columns belong to head group
  // g = column / group_w, kept by rank g; each row is stored straight into rank g's buffers
  // (peer memory over NVLink): q at sp_q[g] + qrow * group_w, k and v at sp_k[g] / sp_v[g] +
  // kvrow * group_w.  This rank's local row t is prefix row sp_rank * sp_pl + t when t <
  // sp_pl_loc, else image row i = t - sp_pl_loc at qrow sp_img0 + sp_rank * sp_nl + i and
  // kvrow sp_p + sp_rank * sp_nl + i (qrow = kvrow for prefix rows).
  int group_w = 0;
  bf16* sp_q[kMaxSp] = {};
  bf16* sp_k[kMaxSp] = {};
  bf16* sp_v[kMaxSp] = {};
  int sp_rank = 0, sp_pl = 0, sp_pl_loc = 0, sp_nl = 0, sp_img0 = 0, sp_p = 0;
  // EPI_PROJ
  float* z = nullptr;
  float* vout = nullptr;
  float dsigma = 0.f;
  int nimg = 0;        // image rows of a sample in this GEMM
  int zstride = 0;     // floats between channels of v / z (0: nimg)
};

struct GemmArgs {
  const bf16* a = nullptr;  // [M][K], row stride lda elements
  long long lda = 0;
  const bf16* b = nullptr;  // [N][K], row stride ldb elements (a weight, out x in)
  long long ldb = 0;
  int M = 0, N = 0, K = 0;
  int epi = EPI_F32;
  GemmEpi ep;
  // tile shape: 1 (default) 256 x 256 tiles on CTA pairs where N allows, one-CTA tiles of fewer
  // columns where pair tiles would not fill one round; 2 pairs where N allows; 0 128-row tiles of
  // one CTA
  int pairs = 1;
};

// C = A B^T through the tcgen05 kernel.  0, or a cudaError_t / -1 (bad shape).
int gemm_launch(const GemmArgs& g, int* d_status, int num_sms, cudaStream_t st);

struct AttnArgs {
  const bf16* q = nullptr;   // [B][nq][width]
  const bf16* k = nullptr;   // [B][kv_rows][kv_heads * 128]: this layer's keys
  const bf16* v = nullptr;
  bf16* out = nullptr;       // [B][nq][width]
  int batch = 1, nq = 0, q0 = 0, p = 0, l = 0, b0 = 0, b1 = 0;
  int heads = 0, width = 0;
  int kv_heads = 0;          // K/V heads (0: heads); query head i reads K/V head i / (heads / kv_heads)
  int kv_rows = 0;           // row capacity of one sample's K/V
  float scale_log2 = 0.f;    // log2(e) / sqrt(128)
  // work split: CTAs of two query tiles, except (split_mode 2) a last round that would fill at most
  // half of the SMS multiprocessors runs as one-tile CTAs; split_mode 0: two-tile CTAs only, 1:
  // one-tile CTAs only.  Each query row's arithmetic is the same in every mode.
  int sms = 0, split_mode = 2;
  // sequence-parallel (sp_out[0] != null): query row qi of the pass is stored into the rank that
  // keeps it, at sp_out[owner] + local * sp_ld + sp_col0 + head * 128: prefix rows qi < sp_img0
  // (first pass) belong to rank qi / sp_pl at local qi % sp_pl; image row i = qi - sp_img0 to
  // rank i / sp_nl at local sp_pl_loc + i % sp_nl
  bf16* sp_out[kMaxSp] = {};
  int sp_ld = 0, sp_col0 = 0, sp_pl = 0, sp_pl_loc = 0, sp_nl = 0, sp_img0 = 0;
};
int attention_launch(const AttnArgs& a, int* d_status, cudaStream_t st);
// kernel attributes (dynamic shared memory) on the current device: 0 or a cudaError_t
int attention_prepare();
int gemm_prepare();
int gemm_q8_prepare();

// C = A . (q d)^T with the weights as Q8_0 (gemm_q8.cu): QS int8 [N][K], DK the fp16 scales laid out
// by k-block ([K/64][N][2], q8_scales_by_kblock_launch from GGUF's [N][K/32]).  Epilogues EPI_F32
// and EPI_SWIGLU.  0, -1 (bad shape), -4 (tensor map) or a cudaError_t.
// C = (A . B^T) * sa[row] * sb[col], A and B int8 (kind::i8), sa = g.ep.mod, sb = g.ep.norm_q, out f32
int gemm_i8_launch(const GemmArgs& g, const int8_t* a, const int8_t* b, int* d_status, int num_sms, cudaStream_t st);
int gemm_q8_launch(const GemmArgs& g, const int8_t* qs, const __half* dk, int* d_status, int num_sms,
                   cudaStream_t st);
int q8_scales_by_kblock_launch(const __half* d, __half* out, int n, int k, cudaStream_t st);

// Thin activations (gemm_thin.cu): part [s][n][N] fp32 = X [n][K] W^T over part s of the k-blocks
// (SPLITS parts), with the weights W [N][K] as the 256-row MMA operand; n <= 256, N a multiple of
// 256.  0, -1 (bad shape), -4 (tensor map) or a cudaError_t.
int gemm_thin_launch(const bf16* x, int n, const bf16* w, int N, int K, int splits, float* part, int* d_status,
                     int num_sms, cudaStream_t st);
int gemm_thin_prepare();

// Scratch that needs no allocation (noalloc.cu): a RoPE table of at most kNoAllocMaxRows sequence
// rows in a fixed device array.  Its address on DEVICE, which must be the current device: looked up
// on the first call for that device, then cached.  0, -1 (bad argument) or a cudaError_t.
constexpr int kNoAllocMaxRows = 8704;
int noalloc_rope_scratch(int device, float2** table);

// A barrier of the sequence-parallel group on the device (elementwise.cu): PEER[g] is rank g's
// arrival slot for this rank (peer memory), MINE this rank's slots [WORLD].  The kernel stores EPOCH
// into every PEER[g] and waits (bounded, 4 s; then STATUS_TIMEOUT_COMM into *status) until every
// MINE[g] >= EPOCH.  0 or a cudaError_t.
struct SpFlags {
  int* peer[kMaxSp];
  int* mine;
};
int sp_flag_barrier_launch(const SpFlags& f, int world, int epoch, int* status, cudaStream_t st);

// --- the VAE decoder's convolutions (conv.cu): implicit GEMM over channels-last bf16 pictures ---
enum ConvKind : int {
  CONV_F32 = 0,   // out f32 [pixel][ld_out] = acc + bias (+ res [pixel][ld_res])
  CONV_BF16 = 1,  // out bf16 [pixel][ld_out] = acc + bias
  CONV_RGBA = 2,  // out f32 [pixel][4] = clamp(acc + bias, -1, 1) of the first 4 channels
};
struct ConvEpi {
  int kind = CONV_F32;
  void* out = nullptr;
  long long ld_out = 0;
  const float* bias = nullptr;  // [cout rounded up to 16]
  const float* res = nullptr;
  long long ld_res = 0;
  // CONV_F32 of an upsampling convolution: + Wan's DupUp3D of the stage's input DUP f32
  // [h/2][w/2][dup_ci] (the channel repeat and 2 x 2 pixel shuffle of the last of dup_ft frames),
  // pixel (y, x) of the w-wide output reading input pixel (y/2, x/2)
  const float* dup = nullptr;
  int dup_ci = 0, dup_ft = 1, out_w = 0;
  int cout = 0;                 // set by conv_launch
};
struct ConvArgs {
  const bf16* x = nullptr;   // [h][w][cp]: channels padded to a multiple of 64 with zeros
  const bf16* wt = nullptr;  // [cout tiles x BN][taps][cp]: tap-major rows of weights, zero padding
  int h = 0, w = 0, cp = 0, cout = 0, taps = 9;
  ConvEpi ep;
};
int conv_launch(const ConvArgs& a, int* d_status, int num_sms, cudaStream_t st);
int conv_prepare();
// rows of the weight matrix conv_launch wants for COUT output channels (a multiple of its tile)
inline int conv_rows(int cout) { return cout % 144 == 0 ? cout : (cout % 64 == 0 ? cout : (cout + 15) / 16 * 16); }

// --- the VAE decoder's memory-bound kernels (vae.cu) ---
// y bf16 [n][cp] = (silu)(x / max(|x|, 1e-12) * sqrt(c) * gamma) of x f32 [n][c]; channels c.. cp-1 zero
void vae_norm_launch(const float* x, const float* gamma, bf16* y, int n, int c, int cp, int silu, cudaStream_t st);
// v = bf16-rounded v (round to nearest even), in place
void round_bf16_launch(float* v, long long n, cudaStream_t st);
// y bf16 [n][cp] = x f32 [n][c]; channels c.. cp-1 zero
void vae_to_bf16_launch(const float* x, bf16* y, long long n, int c, int cp, cudaStream_t st);
// u bf16 [2h][2w][cp]: x f32 [h][w][c] repeated 2 x 2 (nearest), channels c.. cp-1 zero
void vae_up2_launch(const float* x, bf16* u, int h, int w, int c, int cp, cudaStream_t st);
// p bf16 [n][n] = softmax(s * scale) by rows of s f32 [n][n]
void vae_softmax_launch(const float* s, bf16* p, int n, float scale, cudaStream_t st);
// out bf16 [c][n] = in bf16 [n][c] (row stride ld_in)
void vae_transpose_launch(const bf16* in, long long ld_in, bf16* out, int n, int c, cudaStream_t st);
// a conv weight [o][i][taps] (f32) -> bf16 [rows][taps][cp], rows >= o and channels >= i zero
void vae_weight_launch(const float* w, bf16* out, int o, int i, int taps, int rows, int cp, cudaStream_t st);

// --- the prompt encoder's memory-bound kernels (encoder.cu) ---
// x f32 [n][width] = table f32 [vocab][width] at rows ids[0..n)
void enc_embed_launch(const float* table, const int* ids, float* x, int n, int width, cudaStream_t st);
// table [n][64] (cos, sin): Qwen3-VL's interleaved M-RoPE of positions pos [n][3] (t, h, w)
void enc_rope_launch(const int* pos, float2* table, int n, double theta, cudaStream_t st);
// Q8_0 to f32, exactly: from split (qs, d) or from GGUF's 34-byte blocks
void q8_to_f32_launch(const int8_t* qs, const __half* d, float* out, long long n, cudaStream_t st);
void q8_raw_to_f32_launch(const uint8_t* raw, float* out, long long n, cudaStream_t st);
// the most parts an encoder GEMM is split into along K (the epilogues below take at most this many)
constexpr int kEncMaxSplits = 8;
// the epilogues of split-K GEMMs (PART [splits][n][N] fp32, summed in split order): q / k / v with
// the per-head norms and RoPE on halves; h = silu(gate) * up (interleaved by 128)
void enc_qkv_sum_launch(const float* part, int splits, int n, int qw, int kvw, const float* norm_q,
                        const float* norm_k, const float2* rope, bf16* q, bf16* k, bf16* v, cudaStream_t st);
// x += the sum, then (NORM not null) xn = RMSNorm(x) * NORM in bf16 (the next GEMM's operand); w <= 4096
void enc_resid_rms_launch(const float* part, int splits, int n, int w, float* x, const float* norm, bf16* xn,
                          cudaStream_t st);
void enc_swiglu_sum_launch(const float* part, int splits, int n, int ffn, bf16* h, cudaStream_t st);

// --- memory-bound kernels (elementwise.cu) ---
// y[r] = LayerNorm(x[map(r)]) * (1 + scale[row kind]), bf16 out.  Row map as GemmEpi's.
// single: one modulation row for every row (norm_out's scale).
void ln_mod_launch(const float* x, bf16* y, const float* scale, int mod_stride, int rows, int width, int seg_in,
                   int seg_out, int off, int n0, int p, int single, cudaStream_t st);
// y = RMSNorm(x) * w (w already 1 + text_norm), bf16 out
void rms_launch(const float* x, const float* w, bf16* y, int rows, int width, cudaStream_t st);
// latent [B][C][ld] f32 channel-major, columns i0 .. i0+n -> rows [B*n][C] bf16
void latent_rows_launch(const float* lat, bf16* rows, int batch, int channels, int n, cudaStream_t st, int ld = 0,
                        int i0 = 0);
// RoPE (cos, sin) of rows r0 .. r0+count of the sequence (host.lisp's positions), [count][64].
// With split > 0 the table's rows are a rank's shard instead: local row t < split is sequence row
// r0 + t (prefix), t >= split is sequence row r1 + (t - split) (image).
void rope_table_launch(float2* table, int r0, int count, int p, int h, int w, int ref_a, int ref_h, int ref_w,
                       cudaStream_t st, int split = 0, int r1 = 0);
// emb[2][freq]: timestep embedding of 1000*sigma and of 0
void temb_launch(float* emb, double sigma, int freq, cudaStream_t st);
// Weight kinds for the small GEMVs
enum WKind : int { W_Q8 = 0, W_BF16 = 1, W_F32 = 2 };
// y[m][out] = act(x[m][in] . W[out][in]); act 0 none, 1 silu, 2 tanh on columns of pieces 1 and 3 (of 4).
// 0, -1 (m > 2 or m x in floats beyond 48 KB of shared memory) or the launch's cudaError_t.
int gemv_launch(int kind, const void* w, const __half* wd, const float* x, float* y, int m, int in, int out,
                int act, int piece, cudaStream_t st);
// GGUF Q8_0 blocks (34 B) -> bf16 rows, row r written at dst_row(r) (gate_up interleave when ilv > 0)
void q8_raw_to_bf16_launch(const uint8_t* raw, bf16* dst, long long rows, int cols, long long row0, int ilv,
                           cudaStream_t st);
// GGUF Q8_0 blocks -> separate int8 qs and fp16 d
void q8_raw_split_launch(const uint8_t* raw, int8_t* qs, __half* d, long long nblocks, cudaStream_t st);
// f32 / bf16 / f16 rows -> bf16 rows (same permutation rules)
void f32_to_bf16_rows_launch(const float* src, bf16* dst, long long rows, int cols, long long row0, int ilv,
                             cudaStream_t st);
void bf16_rows_launch(const bf16* src, bf16* dst, long long rows, int cols, long long row0, int ilv,
                      cudaStream_t st);
void f16_to_f32_launch(const __half* src, float* dst, long long n, cudaStream_t st);
void bf16_to_f32_launch(const bf16* src, float* dst, long long n, cudaStream_t st);
// synthetic Q8_0 tensor (the oracle's generator): qs int8 [n], d fp16 [n/32]
void synth_q8_launch(int8_t* qs, __half* d, long long n, uint64_t seed, uint32_t stream, float scale,
                     cudaStream_t st);
// synthetic f32 vector: base + offset * scale
void synth_f32_launch(float* v, long long n, uint64_t seed, uint32_t stream, float scale, float base,
                      cudaStream_t st);
// Q8 (qs, d) -> bf16 rows with the same permutation rules
void q8_to_bf16_launch(const int8_t* qs, const __half* d, bf16* dst, long long rows, int cols, long long row0,
                       int ilv, cudaStream_t st);
void add_scalar_launch(float* v, long long n, float a, cudaStream_t st);
// *out += an order-independent digest of BYTES (a multiple of 8) at P
void digest_launch(const void* p, size_t bytes, unsigned long long* out, cudaStream_t st);
// one CTA whose bounded wait on an mbarrier nothing arrives on runs out after LIMIT_NS
void wait_probe_launch(int* status, unsigned long long limit_ns, cudaStream_t st);

}  // namespace exn
