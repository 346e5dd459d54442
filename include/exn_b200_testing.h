/* exn_b200_testing.h -- entry points for kernel-level parity tests and
 * benchmarks.  They expose single kernels of libexn_b200.so on device
 * pointers; none of them has a counterpart in ex-nihilo, whose kernels are
 * reached only through dit-velocity (src/cuda-dit.lisp:137-243).  The
 * reference's own kernel tests (inspect/metal-kernels-test.lisp:91-146) check
 * LayerNorm-mod, QK-norm + RoPE and the attention mask; these entry points
 * let the same cases run against the sm_100a kernels. */
#ifndef EXN_B200_TESTING_H
#define EXN_B200_TESTING_H

#include "exn_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* C[M x N] (f32, row stride N) = A[M x K] (bf16) . B[N x K]^T (bf16) through
 * the tcgen05 GEMM; all device pointers. */
int exn_test_gemm(exn_handle* h, const void* a, const void* b, float* c, int m, int n, int k);

/* The same product with B as Q8_0 weights, converted to bf16 inside the GEMM (gemm_q8.cu): QS
 * int8 [n][k], D fp16 scales [n][k/32] (GGUF's order), device pointers; n a multiple of 256.  The
 * reference keeps its weights this way on the device (src/cuda-dit.lisp:71-76).  With REPS > 0
 * the GEMM then runs REPS more times back to back and *MS receives the mean time of one (CUDA
 * events on the handle's stream). */
int exn_test_gemm_q8(exn_handle* h, const void* a, const void* qs, const void* d, float* c, int m, int n, int k,
                     int reps, double* ms);

/* C[m x n] f32 = (A . B^T) * SA[row] * SB[col] with A [m][k] and B [n][k] int8 (tcgen05 kind::i8,
 * s32 accumulation, CTA pairs): the W8A8 form of the reference's *int8* path (src/cuda-dit.lisp
 * :110-126) with one scale per activation row and per weight row; n a multiple of 256, k of 128.
 * REPS and MS as exn_test_gemm_q8. */
int exn_test_gemm_i8(exn_handle* h, const void* a, const void* b, const float* sa, const float* sb, float* c, int m,
                     int n, int k, int reps, double* ms);

/* exn_test_gemm run REPS times back to back; *MS the mean time of one (CUDA events). */
int exn_test_gemm_timed(exn_handle* h, const void* a, const void* b, float* c, int m, int n, int k, int reps,
                        double* ms);

/* Masked attention (xa_lim, src/cuda/dit.cu:60-66) on bf16 device tensors:
 * q [batch][nq][heads*128], k/v [batch][kv_rows][heads*128], out like q. */
int exn_test_attention(exn_handle* h, const void* q, const void* k, const void* v, void* out, int batch, int nq,
                       int q0, int p, int l, int b0, int b1, int heads, int kv_rows);

/* The DiT's small-M matrix-vector product (timestep MLP, modulation, norm_out; src/cuda-dit.lisp:157-167)
 * on device tensors: y [m][out] fp32 = act(x [m][in] fp32 . W^T), m 1 or 2.  KIND 0: W int8 [out][in]
 * with fp16 scales D [out][in / 32] (Q8_0 split), 1: bf16 [out][in], 2: f32 [out][in].  ACT 0 none,
 * 1 SiLU, 2 tanh on the second and fourth PIECE-row pieces (the modulation's gates).  Run REPS times
 * back to back; *MS the mean time of one. */
int exn_test_gemv(exn_handle* h, int kind, const void* w, const void* d, const float* x, float* y, int m, int in,
                  int out, int act, int piece, int reps, double* ms);

/* exn_test_attention run REPS times back to back; *MS the mean time of one launch (CUDA events on
 * the handle's stream, the launches queued without a host wait between them). */
int exn_test_attention_timed(exn_handle* h, const void* q, const void* k, const void* v, void* out, int batch, int nq,
                             int q0, int p, int l, int b0, int b1, int heads, int kv_rows, int reps, double* ms);

/* Host side of the communicator waits since the handle was opened: how many times the library
 * waited for an NCCL call to be queued (every barrier of a sequence-parallel pass does), how many
 * 50 us sleeps those waits took, and their total wall time in seconds. */
int exn_test_comm_stats(exn_handle* h, long long* settles, long long* sleeps, double* seconds);

/* The GEMM tiles of this handle's later calls: PAIRS 1 (the default) 256 x 256 tiles on CTA pairs
 * wherever N is a multiple of 256, except where those would not fill one round of the SM pairs and
 * a narrower one-CTA tile does (epilogues F32, BF16, gated residual); 2 pairs wherever N allows;
 * 0 128-row tiles of one CTA everywhere. */
int exn_test_gemm_pairs(exn_handle* h, int pairs);

/* How the attention kernel splits its work, for this handle's later calls: MODE 2 (the default)
 * runs CTAs of two 128-query tiles except that a last round filling at most half of SMS
 * multiprocessors runs as one-tile CTAs; MODE 0 two-tile CTAs only; MODE 1 one-tile CTAs only.
 * SMS 0 is the device's count.  Every mode gives each query row the same arithmetic. */
int exn_test_attention_split(exn_handle* h, int mode, int sms);

/* LayerNorm(x) * (1 + mod[row kind]) -> bf16 (x_ln_mod, src/cuda/dit.cu:17-32):
 * rows n, mod [2][width] (row 1 for prompt rows, n0 + t < p). */
int exn_test_ln_mod(exn_handle* h, const float* x, void* y, const float* mod, int n, int width, int n0, int p);

/* The fused QKV epilogue alone: y [n][width] bf16, the handle's layer LAYER
 * weights; q out [n][width], k/v out [kv_rows][width] at rows n0.., bf16;
 * RoPE of the plain layout (p text rows, hh x ww picture). */
int exn_test_qkv(exn_handle* h, int layer, const void* y, void* q, void* k, void* v, int n, int n0, int p, int hh,
                 int ww, int kv_rows);

/* exn_test_qkv without any device allocation, for callers that cannot call cudaMalloc: for
 * instance a host that runs the DiT on a GPU lent to it by another server (ex-nihilo's tenant
 * mode borrows its GPUs from illatio's chat server), whose memory that server's allocator already
 * accounts for, so a new cudaMalloc would fail or take memory the owner counts on.  No counterpart
 * in the reference.  The caller passes y, q, k and v as for exn_test_qkv; the RoPE table the
 * GEMM's epilogue reads goes into a fixed 4.25 MiB device array of this library (every GPU that
 * loads the library holds it until the process exits) instead of step buffers grown with
 * cudaMalloc, so the sequence, p + hh x ww rows, may have at most 8704 rows (EXN_EINVAL beyond).
 * The first call on a device looks up that array's address there; make that first call before any
 * stream capture.  All calls on a device share the array: calls that overlap on the GPU (two
 * handles of one device on different streams) race.  Each call rewrites every table row it reads. */
int exn_qkv_noalloc(exn_handle* h, int layer, const void* y, void* q, void* k, void* v, int n, int n0, int p,
                    int hh, int ww, int kv_rows);

/* The residual stream x after every block (and txt_in's output first) of
 * the next exn_velocity call, copied into HOST (layers + 1 blocks of
 * rows x width floats, rows = the rows that call computes).  NULL disables. */
int exn_test_trace(exn_handle* h, float* host, size_t floats);

/* A Q8_0 tensor as the handle holds it (GEMV matrices only), or the bf16
 * copy of a GEMM matrix: for comparing exn_load_synthetic with the oracle. */
int exn_test_weight_bf16(exn_handle* h, const char* name, void* host_bf16, size_t elems);

/* N floats offset * scale from the synthetic generator (stream, seed) into
 * device memory: the oracle's synth_normal. */
int exn_test_synth_normal(exn_handle* h, float* d, int64_t n, uint64_t seed, uint32_t stream, double std);

/* N values of the synthetic generator (stream, seed, N(0, std) before quantisation) as Q8_0, the
 * way exn_load_synthetic makes each matrix: int8 D_QS [n] and fp16 D_D [n / 32], device pointers.
 * The same bits as the test oracle's SynthWeights, made in milliseconds instead of minutes for the
 * full-size checks. */
int exn_test_synth_q8(exn_handle* h, void* d_qs, void* d_d, int64_t n, uint64_t seed, uint32_t stream,
                      double std_dev);

/* An order-independent 64-bit digest of every weight the handle holds on the device (the bf16 slab
 * with the norm vectors, and the GEMV matrices in their stored form): two handles loaded with the
 * same weights the same way have the same digest. */
int exn_test_weights_digest(exn_handle* h, uint64_t* out);

/* Turn per-category kernel timing on or off (also on when EXN_PROFILE is set
 * at open): CUDA events recorded on the handle's stream between the GEMM,
 * attention and other kernels of every step. */
int exn_test_profile(exn_handle* h, int on);

/* Kernels of this library the handle has queued since it was opened. */
long long exn_test_launch_count(const exn_handle* h);

/* Failure detection on the GPU without a fault: one CTA waits, through the
 * kernels' own bounded mbarrier wait, on a barrier nothing arrives on, with a
 * limit of SECONDS (0 < SECONDS <= 1).  The wait runs out, the kernel records
 * it in the handle's status word and returns; the call returns EXN_ETIMEOUT
 * as a stalled pipeline would, and the handle stays usable. */
int exn_test_wait_probe(exn_handle* h, double seconds);

/* Device time in ms (CUDA events on the handle's stream) of the last
 * successful exn_velocity / exn_generate: from the end of the inputs' upload
 * to the start of the result's download, so the DiT forwards (and, across
 * GPUs, the gather of the latent) with the inputs already in HBM. */
int exn_test_last_call_ms(const exn_handle* h, double* ms);

/* Kernel time of the last exn_generate* / exn_velocity call in ms per
 * category when timing is on, else zeros: every GEMM, attention, the rest,
 * and of the GEMMs the gate_up + SwiGLU ones alone. */
int exn_test_last_profile(exn_handle* h, double* gemm_ms, double* attn_ms, double* other_ms, double* gateup_ms);

/* With profiling on, the device time of the last call's sequence-parallel barriers (from the end of
 * the kernel before each barrier to the start of the one after it: the wait for the slowest rank and
 * for the peers' stores), in ms; 0 on one GPU. */
int exn_test_last_barrier_ms(exn_handle* h, double* ms);

/* Device time in ms (CUDA events on the decoder's stream) of the last exn_vae_decode, from the
 * latent's upload to the start of the pixels' download. */
int exn_test_vae_last_ms(const exn_vae* v, double* ms);

/* Device time in ms (CUDA events on the encoder's stream) of the last exn_enc_states, from the ids'
 * upload to the states' download. */
int exn_test_enc_last_ms(const exn_enc* e, double* ms);

/* An order-independent digest of every byte of the encoder's weights on the device (the bf16
 * matrices, the fp32 vectors and embedding table), to compare two loads. */
int exn_test_enc_weights_digest(exn_enc* e, uint64_t* out);

#ifdef __cplusplus
}
#endif

#endif
