/* exn_b200.h -- C ABI of libexn_b200.so, the B200 (sm_100a) DiT of
 * Qwen-Image-2.1-Turbo behind ex-nihilo's calling conventions.
 *
 * Each entry point replaces one function of ex-nihilo's CUDA driver
 * (paths relative to that project):
 *
 *   exn_load_gguf      (upload-dit path :device d)        src/cuda-dit.lisp:52-86
 *                      with open-dit's checks              src/weights.lisp:47-61
 *   exn_velocity       (dit-velocity d context p latent h w sigma
 *                                    :prefix-key :ref)   src/cuda-dit.lisp:137-243
 *   exn_release        (dit-release d)                    src/cuda-dit.lisp:99-108
 *   exn_generate       the step loop of generate / edit   src/generate.lisp:133-135, 95-97
 *                      (z += (s' - s) v, each v a dit-velocity call)
 *   exn_generate_batch / exn_generate_device
 *                      the same loop for B independent pictures (no counterpart:
 *                      the reference runs one picture at a time)
 *
 * Conventions: every function returns an int status (EXN_OK = 0); the text
 * of the last failure is exn_last_error(h).  Nothing aborts or throws across
 * the ABI.  Host pointers belong to the caller, are read or written only
 * during the call and need not be pinned.  A handle owns one CUDA device
 * and is used by one thread at a time (the reference serialises callers with
 * *gpu-lock*, src/server.lisp:24-28).  Floats are IEEE binary32; latents are
 * channel-major 64 x H x W as in the reference.
 */
#ifndef EXN_B200_H
#define EXN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EXN_ABI_VERSION 1

enum {
  EXN_OK = 0,
  EXN_EINVAL = 1,      /* bad argument: null pointer, size, shape */
  EXN_ECUDA = 2,       /* a CUDA call failed */
  EXN_ESHAPE = 3,      /* weights that are not the DiT's (open-dit's error) */
  EXN_ENOWEIGHTS = 4,  /* a step before every tensor was loaded */
  EXN_EIO = 5,         /* file could not be read */
  EXN_ETIMEOUT = 6,    /* a kernel gave up waiting on its own pipeline */
  EXN_ENOMEM = 7,      /* device memory exhausted */
  EXN_EUNSUPPORTED = 8 /* no sm_100 device, or a tensor type not handled */
};

/* ggml tensor types accepted by exn_load_tensor */
enum { EXN_GGML_F32 = 0, EXN_GGML_F16 = 1, EXN_GGML_Q8_0 = 8, EXN_GGML_BF16 = 30 };

/* The model's shape: dit-shape of src/weights.lisp:19-20.  width must be a
 * multiple of 256 and of head_dim (128), ffn of 128, context of 64. */
typedef struct exn_config {
  int width;    /* 4096 */
  int layers;   /* 32 */
  int ffn;      /* 12288 */
  int latent;   /* 64 */
  int context;  /* 4096: the encoder's state width */
  int freq;     /* 256: timestep embedding size */
  int head_dim; /* 128 */
  int device;   /* CUDA ordinal */
} exn_config;

/* An edit's reference picture, the REF argument of dit-velocity
 * (src/cuda-dit.lisp:142-147): its latent (64 x rh x rw, channel-major,
 * normalised) goes into the prefix after the first A text rows. */
typedef struct exn_ref {
  int a;
  const float* latent;
  int rh, rw;
} exn_ref;

typedef struct exn_handle exn_handle;

int exn_abi_version(void);
void exn_default_config(exn_config* cfg);

/* Open the device cfg->device.  *out is NULL on failure; the message is then
 * exn_last_error(NULL) (per thread). */
int exn_open(const exn_config* cfg, exn_handle** out);
void exn_close(exn_handle* h);
const char* exn_last_error(const exn_handle* h);

/* upload-dit: read, check (architecture qwen_image, every tensor's name and
 * dims, nothing extra; src/weights.lisp:47-61) and upload a DiT GGUF. */
int exn_load_gguf(exn_handle* h, const char* path);

/* open-dit alone: check the GGUF at PATH against the shape CFG (architecture,
 * names, dims, no extra tensors) without a device.  EXN_OK, or EXN_ESHAPE /
 * EXN_EIO with open-dit's message (one line per problem) copied into MSG. */
int exn_check_gguf(const exn_config* cfg, const char* path, char* msg, size_t msg_len);

/* One tensor from host memory, in its GGUF encoding: name without the
 * "model.diffusion_model." prefix, ggml dims (contiguous axis first). */
int exn_load_tensor(exn_handle* h, const char* name, int ggml_type, int n_dims, const int64_t* dims,
                    const void* data, size_t nbytes);

/* Every tensor from the deterministic synthetic generator (Q8_0 matrices,
 * N(0, 0.02 sqrt(4096/width)) before quantisation; norms 1 + N(0, .)), the
 * same bits as the test oracle's generator for SEED. */
int exn_load_synthetic(exn_handle* h, uint64_t seed);

/* EXN_OK when every tensor of the shape has been loaded. */
int exn_weights_ready(const exn_handle* h);

/* dit-velocity: v (64 x h x w) at noise level SIGMA.  CONTEXT is P x context
 * floats (text rows only; with REF the picture's rows are added).  With a
 * nonzero PREFIX_KEY the prompt's keys and values are kept after the call
 * and reused by the next call with the same key and prefix length. */
int exn_velocity(exn_handle* h, const float* context, int p, const float* latent, int hh, int ww, double sigma,
                 uint64_t prefix_key, const exn_ref* ref, float* v_out);

/* The Euler loop of generate/edit: for each pair (s, s') of SIGMAS,
 * z += (s' - s) * dit-velocity(z, s), z (64 x h x w) updated in place on
 * the device and copied back once.  PREFIX_KEY as exn_velocity. */
int exn_generate(exn_handle* h, const float* context, int p, float* z, int hh, int ww, const double* sigmas,
                 int nsig, uint64_t prefix_key, const exn_ref* ref);

/* The same loop for BATCH independent pictures of the same size and prompt
 * length: contexts B x P x context, z B x 64 x h x w (host memory).  The
 * prompt K/V cache lives for the call only. */
int exn_generate_batch(exn_handle* h, int batch, const float* contexts, int p, float* z, int hh, int ww,
                       const double* sigmas, int nsig);

/* exn_generate_batch on device memory (d_contexts, d_z are CUDA device
 * pointers of the handle's device), ordered on STREAM (a cudaStream_t; NULL
 * is CUDA's default stream): the work starts after what STREAM already holds
 * and what is queued on STREAM later waits for it.  Returns once queued. */
int exn_generate_device(exn_handle* h, int batch, const float* d_contexts, int p, float* d_z, int hh, int ww,
                        const double* sigmas, int nsig, void* stream);

/* Wait for the handle's queued work and report any kernel failure. */
int exn_sync(exn_handle* h);

/* dit-release: free the step buffers and the kept prompt keys and values. */
int exn_release(exn_handle* h);

/* Sequence parallelism over GPUs for one long picture (an edit, a large
 * canvas): WORLD handles, one per GPU and process, join one NCCL
 * communicator; afterwards exn_velocity and exn_generate, called with the
 * same arguments on every rank, split the rows of the pass across the ranks
 * (prefix and image rows in equal shares), exchange Q/K/V and the attention
 * output by all-to-all (Ulysses: attention on heads/WORLD heads per rank),
 * keep the prompt's K/V per head shard, and return the full result on every
 * rank.  Needs heads, prefix rows and image rows divisible by WORLD and
 * width/WORLD a multiple of 256.  No counterpart in the reference (one GPU;
 * src/server.lisp:24-28).  Every wait on the communicator is bounded by
 * EXN_COMM_TIMEOUT_S (default 60 s), after which it is aborted and the call
 * returns EXN_ETIMEOUT. */
int exn_comm_unique_id(void* id128);  /* 128 bytes: rank 0 makes it, every rank passes the same */
int exn_comm_init(exn_handle* h, const void* id128, int rank, int world);
int exn_comm_destroy(exn_handle* h);

/* ---- The VAE decoder: a latent to RGBA pixels (Wan 2.2's decoder, one frame, 2-D), the step
 * after the DiT.  Each entry point replaces one function of src/cuda-vae.lisp:
 *
 *   exn_vae_open + exn_vae_load_safetensors
 *                      (upload-vae path :device d)   src/cuda-vae.lisp:15-27, with open-vae's
 *                      checks of the decoder's tensors (src/weights.lisp:67-100, 116-127)
 *   exn_vae_decode     (vae-decode v latent h w)      src/cuda-vae.lisp:94-136
 *   exn_vae_release    (vae-release v)                src/cuda-vae.lisp:29-33
 *
 * Same conventions as the DiT's handle (int status, exn_vae_last_error).  Convolutions run on the
 * tensor cores with bf16 operands and fp32 accumulation; the weights are the checkpoint's bf16. */
typedef struct exn_vae exn_vae;

int exn_vae_open(int device, exn_vae** out);
void exn_vae_close(exn_vae* v);
const char* exn_vae_last_error(const exn_vae* v);

/* The decoder's tensors from a safetensors file (BF16 or F32), each checked by name and shape;
 * tensors the decoder does not use (the encoder's) are ignored. */
int exn_vae_load_safetensors(exn_vae* v, const char* path);

/* Every decoder tensor from the deterministic synthetic generator (weights N(0, 1/fan_in), biases
 * N(0, 0.02), gains 1 + N(0, 0.1), all rounded to bf16), the same bits as the test oracle's. */
int exn_vae_load_synthetic(exn_vae* v, uint64_t seed);
int exn_vae_weights_ready(const exn_vae* v);

/* vae-decode: LATENT (64 x h x w floats, channel-major, denormalised) to RGBA (16h x 16w x 4
 * floats, -1 .. 1, row-major, channels last).  h x w must be a multiple of 64 (1024 x 1024: a
 * 64 x 64 latent; 1536 x 1024: 64 x 96). */
int exn_vae_decode(exn_vae* v, const float* latent, int h, int w, float* rgba);

/* vae-release: the decoder's scratch freed (the weights stay). */
int exn_vae_release(exn_vae* v);

/* ---- The prompt encoder: Qwen3-VL-8B's text model on the same GPU as the DiT, token ids to the
 * states the DiT reads.  Each entry point replaces one function of src/encoder.lisp:
 *
 *   exn_enc_open + exn_enc_load_gguf
 *                      (load-encoder path :device d)      src/encoder.lisp:41-48 (the qwen3vl GGUF)
 *   exn_enc_states     (encoder-states model ids :rope r)  src/encoder.lisp:143-183
 *   exn_enc_release    (free-context ctx)                  src/encoder.lisp:180
 *
 * Tokenising (il::tokenize) and cutting the system turn's rows (encode-prompt,
 * src/encoder.lisp:55-67) stay with the caller.  Matrices run on the tensor cores with bf16
 * operands and fp32 accumulation; the residual stream and the embedding rows are fp32. */
typedef struct exn_enc exn_enc;

typedef struct exn_enc_config {
  int width;     /* 4096 */
  int layers;    /* 36 */
  int heads;     /* 32 query heads of 128 */
  int kv_heads;  /* 8 key/value heads of 128 */
  int ffn;       /* 12288 */
  int vocab;     /* 151936 */
  double theta;  /* 5e6, the M-RoPE base */
  int device;
} exn_enc_config;

void exn_enc_default_config(exn_enc_config* cfg);
int exn_enc_open(const exn_enc_config* cfg, exn_enc** out);
void exn_enc_close(exn_enc* e);
const char* exn_enc_last_error(const exn_enc* e);

/* The text model's tensors from a qwen3vl (or qwen3) GGUF, llama.cpp's names (token_embd,
 * blk.N.attn_q / attn_k / attn_v / attn_output / attn_q_norm / attn_k_norm / attn_norm /
 * ffn_gate / ffn_up / ffn_down / ffn_norm); each checked against the configuration's dims; Q8_0,
 * BF16, F16 or F32.  The final norm and the LM head are not read. */
int exn_enc_load_gguf(exn_enc* e, const char* path);

/* Every tensor from the deterministic synthetic generator (matrices N(0, std) as Q8_0, vectors
 * 1 + N(0, std)), the same bits as the test oracle's. */
int exn_enc_load_synthetic(exn_enc* e, uint64_t seed);
int exn_enc_weights_ready(const exn_enc* e);

/* encoder-states: every token's state after the last block, before the final norm.  IDS: N token
 * ids (0 <= id < vocab).  POSITIONS: N x 3 ints (t, h, w) per token, Qwen3-VL's interleaved M-RoPE
 * as src/encoder.lisp:26-39 builds it, or NULL for a text prompt's (i, i, i).  STATES: N x width
 * floats, row-major. */
int exn_enc_states(exn_enc* e, const int32_t* ids, int n, const int32_t* positions, float* states);

/* encode-prompt's states without the host (src/encoder.lisp:55-67, whose states cross the host on
 * their way to the DiT): rows SKIP .. N-1 (the system turn's SKIP rows cut) into D_STATES, device
 * memory of the encoder's device, (N - SKIP) x width floats -- the context exn_generate_device
 * takes.  Ordered after what STREAM (a cudaStream_t, NULL = CUDA's default stream) holds; the
 * states are in place when the call returns. */
int exn_enc_states_device(exn_enc* e, const int32_t* ids, int n, const int32_t* positions, int skip,
                          float* d_states, void* stream);

/* The encoder's scratch freed (the weights stay). */
int exn_enc_release(exn_enc* e);

#ifdef __cplusplus
}
#endif

#endif /* EXN_B200_H */
