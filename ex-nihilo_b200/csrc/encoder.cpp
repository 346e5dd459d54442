// encoder.cpp -- the host side of the prompt encoder in libexn_b200.so:
// exn_enc_* of include/exn_b200.h.  It does what ex-nihilo's
// src/encoder.lisp does through illatio's qwen3 forward -- the text model of
// Qwen3-VL-8B loaded from its qwen3vl GGUF (load-encoder :41-48) and run over a
// prompt's token ids, every token's state after the last block and before the
// final norm read back (encoder-states :143-183), with Qwen3-VL's interleaved
// M-RoPE positions (mrope-table :26-39) -- on the B200, next to the DiT:
//   * the matrices are bf16 slabs in HBM, converted once at load (Q8_0, BF16,
//     F16 or F32 in the file); every projection is the tcgen05 GEMM with its
//     work fused into the epilogue: q / k per-head RMS norm and RoPE on halves
//     (EPI_QKV), the residual add (EPI_GATE_RESID with a gate of ones), SwiGLU
//     (EPI_SWIGLU over gate and up rows interleaved by 128);
//   * attention is the DiT's tcgen05 kernel with every row causal and query
//     head i reading key/value head i / 4;
//   * the residual stream and the embedding table are fp32; the embedding rows
//     are the file's values exactly.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/exn_b200.h"
#include "../../include/exn_b200_testing.h"
#include "exn_internal.h"
#include "gguf.h"

using namespace exn;

namespace {

thread_local std::string g_enc_open_error;
constexpr uint32_t kStream0 = 30000;  // synthetic stream of tensor i: kStream0 + i
constexpr int kHeadDim = 128;
constexpr int kMaxTokens = 32768;
// prompts of at most this many tokens run their GEMMs split along K (their tile grids cover a
// fraction of the SMs), in at most kMaxSplits parts
constexpr int kSplitRows = 512;
constexpr int kMaxSplits = kEncMaxSplits;

struct Spec {
  std::string name;
  std::vector<int64_t> dims;  // GGUF order: contiguous axis first
};

inline size_t al256(size_t n) { return (n + 255) & ~size_t(255); }

std::string dims_str(const std::vector<int64_t>& d) {
  std::string r = "(";
  for (size_t i = 0; i < d.size(); ++i) r += (i ? " " : "") + std::to_string(d[i]);
  return r + ")";
}

}  // namespace

struct EncLayer {
  bf16* qkv = nullptr;   // [q + 2 kv][width]: q, k, v rows
  bf16* o = nullptr;     // [width][q]
  bf16* gu = nullptr;    // [2 ffn][width]: gate and up interleaved by 128 rows
  bf16* down = nullptr;  // [width][ffn]
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  float* q_norm = nullptr;
  float* k_norm = nullptr;
};

struct exn_enc {
  exn_enc_config cfg{};
  int sms = 0;
  cudaStream_t st = nullptr;
  int* d_status = nullptr;
  std::string err;
  std::vector<Spec> spec;
  std::map<std::string, int> index;
  std::vector<char> loaded;
  size_t n_loaded = 0;
  float* embed = nullptr;  // [vocab][width]
  std::vector<EncLayer> layers;
  void* slab = nullptr;
  float* vecs = nullptr;
  float* ones = nullptr;   // [width]: the residual epilogues' gate
  // scratch for up to cap tokens
  int cap = 0;
  void* scratch = nullptr;
  cudaEvent_t ev[2] = {nullptr, nullptr};
  double last_ms = 0;
};

namespace {

int efail(exn_enc* e, int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (e)
    e->err = buf;
  else
    g_enc_open_error = buf;
  return code;
}

#define ECK(call)                                                                                       \
  do {                                                                                                  \
    cudaError_t e_ = (call);                                                                            \
    if (e_ != cudaSuccess)                                                                              \
      return efail(e, e_ == cudaErrorMemoryAllocation ? EXN_ENOMEM : EXN_ECUDA, "%s: %s (%s:%d)", #call, \
                   cudaGetErrorString(e_), __FILE__, __LINE__);                                         \
  } while (0)

int q_width(const exn_enc_config& c) { return c.heads * kHeadDim; }
int kv_width(const exn_enc_config& c) { return c.kv_heads * kHeadDim; }

// the tensors the encoder reads, llama.cpp's qwen3vl names, in the synthetic generator's order
std::vector<Spec> encoder_tensors(const exn_enc_config& c) {
  const int64_t w = c.width, q = q_width(c), kv = kv_width(c), f = c.ffn;
  std::vector<Spec> r;
  r.push_back({"token_embd.weight", {w, c.vocab}});
  for (int i = 0; i < c.layers; ++i) {
    const std::string b = "blk." + std::to_string(i) + ".";
    r.push_back({b + "attn_norm.weight", {w}});
    r.push_back({b + "attn_q.weight", {w, q}});
    r.push_back({b + "attn_k.weight", {w, kv}});
    r.push_back({b + "attn_v.weight", {w, kv}});
    r.push_back({b + "attn_q_norm.weight", {kHeadDim}});
    r.push_back({b + "attn_k_norm.weight", {kHeadDim}});
    r.push_back({b + "attn_output.weight", {q, w}});
    r.push_back({b + "ffn_norm.weight", {w}});
    r.push_back({b + "ffn_gate.weight", {w, f}});
    r.push_back({b + "ffn_up.weight", {w, f}});
    r.push_back({b + "ffn_down.weight", {f, w}});
  }
  return r;
}

// Where a tensor goes: a bf16 slab (rows from row0, gate/up interleave ilv), an fp32 vector, or
// the fp32 embedding table.
struct Route {
  bf16* dst = nullptr;
  long long row0 = 0;
  int ilv = 0;
  float* vec = nullptr;
  bool embed = false;
};

Route route(exn_enc* e, const std::string& name) {
  Route r;
  if (name == "token_embd.weight") {
    r.embed = true;
    return r;
  }
  const int li = std::atoi(name.c_str() + 4);
  EncLayer& L = e->layers[li];
  const std::string leaf = name.substr(name.find('.', 4) + 1);
  const int q = q_width(e->cfg), kv = kv_width(e->cfg);
  if (leaf == "attn_q.weight") r.dst = L.qkv;
  else if (leaf == "attn_k.weight") r.dst = L.qkv, r.row0 = q;
  else if (leaf == "attn_v.weight") r.dst = L.qkv, r.row0 = q + kv;
  else if (leaf == "attn_output.weight") r.dst = L.o;
  else if (leaf == "ffn_gate.weight") r.dst = L.gu, r.ilv = e->cfg.ffn;
  else if (leaf == "ffn_up.weight") r.dst = L.gu, r.row0 = 128, r.ilv = e->cfg.ffn;  // the up half of each 256
  else if (leaf == "ffn_down.weight") r.dst = L.down;
  else if (leaf == "attn_norm.weight") r.vec = L.attn_norm;
  else if (leaf == "ffn_norm.weight") r.vec = L.ffn_norm;
  else if (leaf == "attn_q_norm.weight") r.vec = L.q_norm;
  else if (leaf == "attn_k_norm.weight") r.vec = L.k_norm;
  return r;
}

void mark(exn_enc* e, int idx) {
  if (!e->loaded[idx]) {
    e->loaded[idx] = 1;
    ++e->n_loaded;
  }
}

// tensor IDX from RAW (device memory holding the file's bytes of TYPE) to its place; SCRATCH holds
// n floats
int place(exn_enc* e, int idx, int type, const void* raw, float* scratch) {
  const Spec& s = e->spec[idx];
  const Route r = route(e, s.name);
  const long long cols = s.dims[0], rows = s.dims.size() > 1 ? s.dims[1] : 1, n = rows * cols;
  float* f32 = r.embed ? e->embed : (r.vec ? r.vec : scratch);
  if (r.embed || r.vec) {
    if (type == GGML_F32) ECK(cudaMemcpyAsync(f32, raw, n * 4, cudaMemcpyDeviceToDevice, e->st));
    else if (type == GGML_F16) f16_to_f32_launch(static_cast<const __half*>(raw), f32, n, e->st);
    else if (type == GGML_BF16) bf16_to_f32_launch(static_cast<const bf16*>(raw), f32, n, e->st);
    else if (type == GGML_Q8_0 && r.embed) q8_raw_to_f32_launch(static_cast<const uint8_t*>(raw), f32, n, e->st);
    else return efail(e, EXN_EUNSUPPORTED, "%s: ggml type %d for a vector", s.name.c_str(), type);
  } else if (r.dst) {
    if (type == GGML_Q8_0) {
      q8_raw_to_bf16_launch(static_cast<const uint8_t*>(raw), r.dst, rows, static_cast<int>(cols), r.row0, r.ilv, e->st);
    } else if (type == GGML_BF16) {
      bf16_rows_launch(static_cast<const bf16*>(raw), r.dst, rows, static_cast<int>(cols), r.row0, r.ilv, e->st);
    } else if (type == GGML_F32) {
      f32_to_bf16_rows_launch(static_cast<const float*>(raw), r.dst, rows, static_cast<int>(cols), r.row0, r.ilv, e->st);
    } else if (type == GGML_F16) {
      f16_to_f32_launch(static_cast<const __half*>(raw), scratch, n, e->st);
      f32_to_bf16_rows_launch(scratch, r.dst, rows, static_cast<int>(cols), r.row0, r.ilv, e->st);
    } else {
      return efail(e, EXN_EUNSUPPORTED, "%s: ggml type %d", s.name.c_str(), type);
    }
  } else {
    return efail(e, EXN_EINVAL, "no place for encoder tensor %s", s.name.c_str());
  }
  ECK(cudaGetLastError());
  mark(e, idx);
  return EXN_OK;
}

int enc_status(exn_enc* e) {
  ECK(cudaStreamSynchronize(e->st));
  int s = 0;
  ECK(cudaMemcpy(&s, e->d_status, sizeof s, cudaMemcpyDeviceToHost));
  if (s) {
    cudaMemset(e->d_status, 0, sizeof(int));
    return efail(e, EXN_ETIMEOUT, "a kernel gave up waiting on its pipeline (status 0x%x)", s);
  }
  return EXN_OK;
}

// scratch for N tokens: x f32 [n][w]; xn bf16 [n][max(w, q)]; q bf16 [n][q]; k, v bf16 [n][kv];
// h bf16 [n][ffn]; rope float2 [n][64]; ids and positions int32
struct Scratch {
  float* x;
  bf16 *xn, *q, *k, *v, *h;
  float2* rope;
  int* ids;
  int* pos;
  float* part;  // split-K partials: [splits][n][N] for prompts of at most kSplitRows tokens
};

// the split of a GEMM with TILES 256 x 256 output tiles and NUM_KB k-blocks over CLUSTERS CTA
// pairs: the count of parts (1 .. kMaxSplits) whose work items fill their last wave best
int split_for(int tiles, int num_kb, int clusters) {
  int best = 1;
  double best_eff = 0;
  for (int s = 1; s <= kMaxSplits && s <= num_kb; ++s) {
    const double w = static_cast<double>(tiles) * s / clusters;
    const double eff = w / std::ceil(w);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = s;
    }
  }
  return best;
}

size_t scratch_bytes(const exn_enc_config& c, int n, Scratch* s, char* base) {
  const int q = q_width(c), kv = kv_width(c);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    off += al256(bytes);
    return p;
  };
  Scratch t;
  t.x = reinterpret_cast<float*>(take(static_cast<size_t>(n) * c.width * 4));
  t.xn = reinterpret_cast<bf16*>(take(static_cast<size_t>(n) * std::max(c.width, q) * 2));
  t.q = reinterpret_cast<bf16*>(take(static_cast<size_t>(n) * q * 2));
  t.k = reinterpret_cast<bf16*>(take(static_cast<size_t>(n) * kv * 2));
  t.v = reinterpret_cast<bf16*>(take(static_cast<size_t>(n) * kv * 2));
  t.h = reinterpret_cast<bf16*>(take(static_cast<size_t>(n) * c.ffn * 2));
  t.rope = reinterpret_cast<float2*>(take(static_cast<size_t>(n) * 64 * 8));
  t.ids = reinterpret_cast<int*>(take(static_cast<size_t>(n) * 4));
  t.pos = reinterpret_cast<int*>(take(static_cast<size_t>(n) * 12));
  const size_t widest = std::max({static_cast<size_t>(q + 2 * kv), static_cast<size_t>(2 * c.ffn),
                                  static_cast<size_t>(c.width)});
  t.part = reinterpret_cast<float*>(take(kMaxSplits * static_cast<size_t>(std::min(n, kSplitRows)) * widest * 4));
  if (s) *s = t;
  return off;
}

int ensure_scratch(exn_enc* e, int n, Scratch* s) {
  if (n > e->cap) {
    if (e->scratch) cudaFree(e->scratch);
    e->scratch = nullptr;
    e->cap = 0;
    ECK(cudaMalloc(&e->scratch, scratch_bytes(e->cfg, n, nullptr, nullptr)));
    e->cap = n;
  }
  scratch_bytes(e->cfg, e->cap, s, static_cast<char*>(e->scratch));
  return EXN_OK;
}

int gemm(exn_enc* e, const GemmArgs& g, const char* what, int layer) {
  const int r = gemm_launch(g, e->d_status, e->sms, e->st);
  if (r) return efail(e, EXN_ECUDA, "encoder block %d: %s GEMM (%d x %d x %d) launch failed: %d", layer, what, g.M, g.N,
                      g.K, r);
  return EXN_OK;
}

// parts of a thin prompt's GEMM with N output columns and K deep (1: no split)
int splits(const exn_enc* e, int n, int N, int K) {
  if (n > kSplitRows) return 1;
  return split_for(((n + 255) / 256) * (N / 256), K / 64, e->sms / 2);
}

// a split-K GEMM of A [n][K] and B [N][K] into the partials of S: up to 256 tokens with the weights
// as the 256-row MMA operand (gemm_thin.cu), longer prompts on the pair GEMM
int gemm_split(exn_enc* e, const bf16* a, const bf16* b, int n, int N, int K, int parts, const Scratch& s,
               const char* what, int layer) {
  if (n <= 256) {
    const int r = gemm_thin_launch(a, n, b, N, K, parts, s.part, e->d_status, e->sms, e->st);
    if (r) return efail(e, EXN_ECUDA, "encoder block %d: %s GEMM (%d x %d x %d, thin) launch failed: %d", layer, what,
                        n, N, K, r);
    return EXN_OK;
  }
  GemmArgs g;
  g.a = a;
  g.lda = K;
  g.b = b;
  g.ldb = K;
  g.M = n;
  g.N = N;
  g.K = K;
  g.epi = EPI_F32;
  g.ep.out = s.part;
  g.ep.ld_out = N;
  g.ep.splits = parts;
  return gemm(e, g, what, layer);
}

// one block of the text model over the N rows of S (x updated in place).  A thin prompt's GEMMs
// run split along K into fp32 partials, summed (in split order) by the kernel that applies the
// epilogue; a longer prompt's have the epilogue fused.  After a split residual GEMM the summing
// kernel also writes the next RMS norm's output.  *NORMED: on entry, whether s.xn already holds
// this block's attn_norm output; on return, whether it holds the next block's.
int block(exn_enc* e, int li, int n, const Scratch& s, bool* normed) {
  const exn_enc_config& c = e->cfg;
  const EncLayer& L = e->layers[li];
  const float* next_norm = li + 1 < c.layers ? e->layers[li + 1].attn_norm : nullptr;
  const int q = q_width(c), kv = kv_width(c);
  int rc, sp;
  if (!*normed) rms_launch(s.x, L.attn_norm, s.xn, n, c.width, e->st);
  *normed = false;
  bool ffn_normed = false;
  if ((sp = splits(e, n, q + 2 * kv, c.width)) > 1) {
    if ((rc = gemm_split(e, s.xn, L.qkv, n, q + 2 * kv, c.width, sp, s, "q/k/v", li))) return rc;
    enc_qkv_sum_launch(s.part, sp, n, q, kv, L.q_norm, L.k_norm, s.rope, s.q, s.k, s.v, e->st);
  } else {  // q, k, v: per-head RMS norm and RoPE on halves in the epilogue
    GemmArgs g;
    g.a = s.xn;
    g.lda = c.width;
    g.b = L.qkv;
    g.ldb = c.width;
    g.M = n;
    g.N = q + 2 * kv;
    g.K = c.width;
    g.epi = EPI_QKV;
    g.ep.width = q;
    g.ep.kv_width = kv;
    g.ep.rope_halves = 1;
    g.ep.norm_q = L.q_norm;
    g.ep.norm_k = L.k_norm;
    g.ep.rope = s.rope;
    g.ep.q = s.q;
    g.ep.k = s.k;
    g.ep.v = s.v;
    if ((rc = gemm(e, g, "q/k/v", li))) return rc;
  }
  {  // causal attention, query head i on key/value head i / (heads / kv_heads)
    AttnArgs a;
    a.q = s.q;
    a.k = s.k;
    a.v = s.v;
    a.out = s.xn;
    a.batch = 1;
    a.nq = n;
    a.q0 = 0;
    a.p = n;  // every row a prompt row: key j visible to row i when j <= i
    a.l = n;
    a.heads = c.heads;
    a.kv_heads = c.kv_heads;
    a.width = q;
    a.kv_rows = n;
    a.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(kHeadDim)));
    a.sms = e->sms;
    const int r = attention_launch(a, e->d_status, e->st);
    if (r) return efail(e, EXN_ECUDA, "encoder block %d: attention (%d rows) launch failed: %d", li, n, r);
  }
  if ((sp = splits(e, n, c.width, q)) > 1) {
    if ((rc = gemm_split(e, s.xn, L.o, n, c.width, q, sp, s, "attn_output", li))) return rc;
    enc_resid_rms_launch(s.part, sp, n, c.width, s.x, L.ffn_norm, s.xn, e->st);
    ffn_normed = true;
  } else {  // x += attn Wo^T
    GemmArgs g;
    g.a = s.xn;
    g.lda = q;
    g.b = L.o;
    g.ldb = q;
    g.M = n;
    g.N = c.width;
    g.K = q;
    g.epi = EPI_GATE_RESID;
    g.ep.out = s.x;
    g.ep.ld_out = c.width;
    g.ep.mod = e->ones;
    if ((rc = gemm(e, g, "attn_output", li))) return rc;
  }
  if (!ffn_normed) rms_launch(s.x, L.ffn_norm, s.xn, n, c.width, e->st);
  if ((sp = splits(e, n, 2 * c.ffn, c.width)) > 1) {
    if ((rc = gemm_split(e, s.xn, L.gu, n, 2 * c.ffn, c.width, sp, s, "ffn_gate/up", li))) return rc;
    enc_swiglu_sum_launch(s.part, sp, n, c.ffn, s.h, e->st);
  } else {  // h = silu(x Wg^T) * (x Wu^T)
    GemmArgs g;
    g.a = s.xn;
    g.lda = c.width;
    g.b = L.gu;
    g.ldb = c.width;
    g.M = n;
    g.N = 2 * c.ffn;
    g.K = c.width;
    g.epi = EPI_SWIGLU;
    g.ep.out = s.h;
    g.ep.ld_out = c.ffn;
    if ((rc = gemm(e, g, "ffn_gate/up", li))) return rc;
  }
  if ((sp = splits(e, n, c.width, c.ffn)) > 1) {
    if ((rc = gemm_split(e, s.h, L.down, n, c.width, c.ffn, sp, s, "ffn_down", li))) return rc;
    enc_resid_rms_launch(s.part, sp, n, c.width, s.x, next_norm, s.xn, e->st);
    *normed = next_norm != nullptr;
  } else {  // x += h Wd^T
    GemmArgs g;
    g.a = s.h;
    g.lda = c.ffn;
    g.b = L.down;
    g.ldb = c.ffn;
    g.M = n;
    g.N = c.width;
    g.K = c.ffn;
    g.epi = EPI_GATE_RESID;
    g.ep.out = s.x;
    g.ep.ld_out = c.width;
    g.ep.mod = e->ones;
    if ((rc = gemm(e, g, "ffn_down", li))) return rc;
  }
  return EXN_OK;
}

}  // namespace

// ============================================================================ C ABI

extern "C" {

void exn_enc_default_config(exn_enc_config* c) {
  if (!c) return;
  c->width = 4096;
  c->layers = 36;
  c->heads = 32;
  c->kv_heads = 8;
  c->ffn = 12288;
  c->vocab = 151936;
  c->theta = 5000000.0;
  c->device = 0;
}

int exn_enc_open(const exn_enc_config* cfg, exn_enc** out) {
  exn_enc* e = nullptr;
  if (!cfg || !out) return efail(nullptr, EXN_EINVAL, "exn_enc_open: null argument");
  *out = nullptr;
  const exn_enc_config& c = *cfg;
  // the kernels' shapes: whole 256-column tiles of q, k and v, 4096 at most for the row norms,
  // FFN halves in 128-row groups, head dim 128
  if (c.width <= 0 || c.width > 4096 || c.width % 256 || c.heads <= 0 || c.kv_heads <= 0 || c.heads % c.kv_heads ||
      (c.heads * kHeadDim) % 256 || (c.kv_heads * kHeadDim) % 256 || c.ffn <= 0 || c.ffn % 128 || c.layers <= 0 ||
      c.vocab <= 0 || !(c.theta > 1.0))
    return efail(nullptr, EXN_EINVAL,
                 "exn_enc_open: unsupported shape (width %d, heads %d / %d, ffn %d, layers %d, vocab %d, theta %g)",
                 c.width, c.heads, c.kv_heads, c.ffn, c.layers, c.vocab, c.theta);
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || c.device < 0 || c.device >= ndev)
    return efail(nullptr, EXN_ECUDA, "exn_enc_open: no CUDA device %d", c.device);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, c.device) != cudaSuccess)
    return efail(nullptr, EXN_ECUDA, "exn_enc_open: cannot query device %d", c.device);
  if (prop.major != 10)
    return efail(nullptr, EXN_EUNSUPPORTED, "exn_enc_open: device %d is sm_%d%d; this library is built for sm_100a",
                 c.device, prop.major, prop.minor);
  e = new exn_enc();
  e->cfg = c;
  e->sms = prop.multiProcessorCount;
  const int rc = [&]() -> int {
    ECK(cudaSetDevice(c.device));
    ECK(cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking));
    ECK(cudaMalloc(&e->d_status, sizeof(int)));
    ECK(cudaMemset(e->d_status, 0, sizeof(int)));
    ECK(static_cast<cudaError_t>(gemm_prepare()));
    ECK(static_cast<cudaError_t>(attention_prepare()));
    ECK(static_cast<cudaError_t>(gemm_thin_prepare()));
    ECK(cudaEventCreate(&e->ev[0]));
    ECK(cudaEventCreate(&e->ev[1]));
    // weights: one bf16 slab for every block's matrices, one fp32 array for the vectors
    const size_t w = c.width, q = q_width(c), kv = kv_width(c), f = c.ffn;
    const size_t per = al256((q + 2 * kv) * w * 2) + al256(w * q * 2) + al256(2 * f * w * 2) + al256(w * f * 2);
    ECK(cudaMalloc(&e->slab, per * c.layers));
    const size_t vper = 2 * w + 2 * kHeadDim;
    ECK(cudaMalloc(&e->vecs, (vper * c.layers + w) * 4));
    ECK(cudaMalloc(&e->embed, static_cast<size_t>(c.vocab) * w * 4));
    e->layers.resize(c.layers);
    char* p = static_cast<char*>(e->slab);
    for (int i = 0; i < c.layers; ++i) {
      EncLayer& L = e->layers[i];
      L.qkv = reinterpret_cast<bf16*>(p);
      p += al256((q + 2 * kv) * w * 2);
      L.o = reinterpret_cast<bf16*>(p);
      p += al256(w * q * 2);
      L.gu = reinterpret_cast<bf16*>(p);
      p += al256(2 * f * w * 2);
      L.down = reinterpret_cast<bf16*>(p);
      p += al256(w * f * 2);
      float* v = e->vecs + vper * i;
      L.attn_norm = v;
      L.ffn_norm = v + w;
      L.q_norm = v + 2 * w;
      L.k_norm = v + 2 * w + kHeadDim;
    }
    e->ones = e->vecs + vper * c.layers;
    std::vector<float> one(w, 1.f);
    ECK(cudaMemcpy(e->ones, one.data(), w * 4, cudaMemcpyHostToDevice));
    return EXN_OK;
  }();
  if (rc) {
    g_enc_open_error = e->err;
    exn_enc_close(e);
    return rc;
  }
  e->spec = encoder_tensors(c);
  for (size_t i = 0; i < e->spec.size(); ++i) e->index[e->spec[i].name] = static_cast<int>(i);
  e->loaded.assign(e->spec.size(), 0);
  *out = e;
  return EXN_OK;
}

void exn_enc_close(exn_enc* e) {
  if (!e) return;
  cudaSetDevice(e->cfg.device);
  if (e->st) cudaStreamSynchronize(e->st);
  if (e->scratch) cudaFree(e->scratch);
  if (e->slab) cudaFree(e->slab);
  if (e->vecs) cudaFree(e->vecs);
  if (e->embed) cudaFree(e->embed);
  if (e->d_status) cudaFree(e->d_status);
  for (cudaEvent_t ev : e->ev)
    if (ev) cudaEventDestroy(ev);
  if (e->st) cudaStreamDestroy(e->st);
  delete e;
}

const char* exn_enc_last_error(const exn_enc* e) { return e ? e->err.c_str() : g_enc_open_error.c_str(); }

int exn_enc_weights_ready(const exn_enc* e) { return e && e->n_loaded == e->spec.size() ? 1 : 0; }

int exn_enc_load_synthetic(exn_enc* e, uint64_t seed) {
  if (!e) return efail(e, EXN_EINVAL, "exn_enc_load_synthetic: null handle");
  ECK(cudaSetDevice(e->cfg.device));
  const double ih_std = std::sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0);
  const float scale = static_cast<float>(0.02 * std::sqrt(4096.0 / e->cfg.width) / ih_std);
  size_t maxn = 0;
  for (const Spec& s : e->spec) maxn = std::max(maxn, static_cast<size_t>(s.dims[0] * (s.dims.size() > 1 ? s.dims[1] : 1)));
  int8_t* qs = nullptr;
  __half* d = nullptr;
  ECK(cudaMalloc(&qs, maxn));
  if (cudaMalloc(&d, maxn / 32 * 2 + 256) != cudaSuccess) {
    cudaFree(qs);
    return efail(e, EXN_ENOMEM, "exn_enc_load_synthetic: staging");
  }
  int rc = EXN_OK;
  for (size_t i = 0; i < e->spec.size() && !rc; ++i) {
    const Spec& s = e->spec[i];
    const long long cols = s.dims[0], rows = s.dims.size() > 1 ? s.dims[1] : 1, n = rows * cols;
    const uint32_t stream = kStream0 + static_cast<uint32_t>(i);
    const Route r = route(e, s.name);
    if (r.vec) {
      synth_f32_launch(r.vec, n, seed, stream, scale, 1.f, e->st);
    } else {
      synth_q8_launch(qs, d, n, seed, stream, scale, e->st);
      if (r.embed)
        q8_to_f32_launch(qs, d, e->embed, n, e->st);
      else
        q8_to_bf16_launch(qs, d, r.dst, rows, static_cast<int>(cols), r.row0, r.ilv, e->st);
    }
    if (cudaGetLastError() != cudaSuccess) rc = efail(e, EXN_ECUDA, "exn_enc_load_synthetic: %s", s.name.c_str());
    else mark(e, static_cast<int>(i));
  }
  cudaStreamSynchronize(e->st);
  cudaFree(qs);
  cudaFree(d);
  return rc;
}

int exn_enc_load_gguf(exn_enc* e, const char* path) {
  if (!e || !path) return efail(e, EXN_EINVAL, "exn_enc_load_gguf: null argument");
  ECK(cudaSetDevice(e->cfg.device));
  GgufFile g;
  std::string err;
  if (!g.open(path, err)) return efail(e, EXN_EIO, "%s", err.c_str());
  // load-encoder's model: a qwen3vl text model; every tensor the encoder reads present with the
  // configuration's dims (the final norm, the LM head and anything else are left unread)
  if (g.arch != "qwen3vl" && g.arch != "qwen3")
    return efail(e, EXN_ESHAPE, "%s: architecture %s, not qwen3vl", path, g.arch.c_str());
  std::map<std::string, const GgufTensor*> by;
  for (const auto& t : g.tensors) by[t.name] = &t;
  std::string problems;
  size_t maxb = 0, maxn = 0;
  for (const Spec& s : e->spec) {
    auto it = by.find(s.name);
    if (it == by.end()) {
      problems += "\n  missing " + s.name;
      continue;
    }
    const GgufTensor& t = *it->second;
    if (t.dims != s.dims) problems += "\n  " + s.name + " is " + dims_str(t.dims) + ", not " + dims_str(s.dims);
    else if (!t.nbytes || (t.type != GGML_Q8_0 && t.type != GGML_BF16 && t.type != GGML_F16 && t.type != GGML_F32) ||
             (t.type == GGML_Q8_0 && s.dims.size() == 1))
      problems += "\n  " + s.name + ": ggml type " + std::to_string(t.type) + " not handled";
    maxb = std::max(maxb, t.nbytes);
    maxn = std::max(maxn, static_cast<size_t>(s.dims[0] * (s.dims.size() > 1 ? s.dims[1] : 1)));
  }
  if (!problems.empty()) return efail(e, EXN_ESHAPE, "%s:%s", path, problems.c_str());
  void* raw = nullptr;
  float* scratch = nullptr;
  void* pinned = nullptr;
  const size_t chunk = 64ull << 20;
  ECK(cudaMalloc(&raw, maxb));
  if (cudaMalloc(&scratch, maxn * 4) != cudaSuccess || cudaMallocHost(&pinned, 2 * chunk) != cudaSuccess) {
    cudaFree(raw);
    if (scratch) cudaFree(scratch);
    return efail(e, EXN_ENOMEM, "exn_enc_load_gguf: staging buffers");
  }
  cudaEvent_t ev[2];
  cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming);
  cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming);
  int rc = EXN_OK, slot = 0;
  for (size_t i = 0; i < e->spec.size() && !rc; ++i) {
    const GgufTensor& t = *by[e->spec[i].name];
    const uint8_t* src = g.data(t);
    // through two pinned halves: the copy of one overlaps the fill of the other
    for (size_t o = 0; o < t.nbytes && !rc; o += chunk) {
      const size_t nb = std::min(chunk, t.nbytes - o);
      char* pb = static_cast<char*>(pinned) + slot * chunk;
      cudaEventSynchronize(ev[slot]);
      std::memcpy(pb, src + o, nb);
      if (cudaMemcpyAsync(static_cast<char*>(raw) + o, pb, nb, cudaMemcpyHostToDevice, e->st) != cudaSuccess)
        rc = efail(e, EXN_ECUDA, "upload of %s failed", t.name.c_str());
      cudaEventRecord(ev[slot], e->st);
      slot ^= 1;
    }
    if (!rc) rc = place(e, static_cast<int>(i), t.type, raw, scratch);
  }
  cudaStreamSynchronize(e->st);
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  cudaFreeHost(pinned);
  cudaFree(scratch);
  cudaFree(raw);
  return rc;
}

}  // extern "C"

namespace {

// The pass of exn_enc_states: rows SKIP .. N-1 of the states into OUT, host memory or (DEVICE)
// device memory of the encoder's device, the pass ordered after what USER's stream holds
int run_states(exn_enc* e, const int32_t* ids, int n, const int32_t* positions, int skip, float* out, bool device,
               cudaStream_t user) {
  if (!e || !ids || !out) return efail(e, EXN_EINVAL, "exn_enc_states: null argument");
  if (n < 1 || n > kMaxTokens) return efail(e, EXN_EINVAL, "exn_enc_states: %d tokens (1 .. %d)", n, kMaxTokens);
  if (!exn_enc_weights_ready(e)) return efail(e, EXN_ENOWEIGHTS, "exn_enc_states: the encoder's weights are not loaded");
  for (int i = 0; i < n; ++i)
    if (ids[i] < 0 || ids[i] >= e->cfg.vocab)
      return efail(e, EXN_EINVAL, "exn_enc_states: token %d is id %d, outside 0 .. %d", i, ids[i], e->cfg.vocab - 1);
  std::vector<int32_t> pos(static_cast<size_t>(n) * 3);
  for (int i = 0; i < n; ++i)
    for (int a = 0; a < 3; ++a) pos[3 * i + a] = positions ? positions[3 * i + a] : i;
  ECK(cudaSetDevice(e->cfg.device));
  if (skip < 0 || skip >= n) return efail(e, EXN_EINVAL, "exn_enc_states: skip %d of %d tokens", skip, n);
  Scratch s;
  int rc;
  if ((rc = ensure_scratch(e, n, &s))) return rc;
  if (device) {  // after the caller's queued work (NULL: CUDA's default stream)
    cudaEvent_t ue;
    ECK(cudaEventCreateWithFlags(&ue, cudaEventDisableTiming));
    const cudaError_t r1 = cudaEventRecord(ue, user);
    const cudaError_t r2 = r1 == cudaSuccess ? cudaStreamWaitEvent(e->st, ue, 0) : r1;
    cudaEventDestroy(ue);
    ECK(r2);
  }
  ECK(cudaEventRecord(e->ev[0], e->st));
  ECK(cudaMemcpyAsync(s.ids, ids, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, e->st));
  ECK(cudaMemcpyAsync(s.pos, pos.data(), pos.size() * 4, cudaMemcpyHostToDevice, e->st));
  enc_embed_launch(e->embed, s.ids, s.x, n, e->cfg.width, e->st);
  enc_rope_launch(s.pos, s.rope, n, e->cfg.theta, e->st);
  ECK(cudaGetLastError());
  bool normed = false;
  for (int li = 0; li < e->cfg.layers; ++li)
    if ((rc = block(e, li, n, s, &normed))) return rc;
  const size_t w = e->cfg.width;
  ECK(cudaMemcpyAsync(out, s.x + static_cast<size_t>(skip) * w, static_cast<size_t>(n - skip) * w * 4,
                      device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, e->st));
  ECK(cudaEventRecord(e->ev[1], e->st));
  if ((rc = enc_status(e))) return rc;
  float ms = 0;
  ECK(cudaEventElapsedTime(&ms, e->ev[0], e->ev[1]));
  e->last_ms = ms;
  return EXN_OK;
}

}  // namespace

extern "C" {

int exn_enc_states(exn_enc* e, const int32_t* ids, int n, const int32_t* positions, float* states) {
  return run_states(e, ids, n, positions, 0, states, false, nullptr);
}

int exn_enc_states_device(exn_enc* e, const int32_t* ids, int n, const int32_t* positions, int skip,
                          float* d_states, void* stream) {
  return run_states(e, ids, n, positions, skip, d_states, true, static_cast<cudaStream_t>(stream));
}

int exn_enc_release(exn_enc* e) {
  if (!e) return efail(e, EXN_EINVAL, "exn_enc_release: null handle");
  ECK(cudaSetDevice(e->cfg.device));
  ECK(cudaStreamSynchronize(e->st));
  if (e->scratch) ECK(cudaFree(e->scratch));
  e->scratch = nullptr;
  e->cap = 0;
  return EXN_OK;
}

int exn_test_enc_last_ms(const exn_enc* e, double* ms) {
  if (!e || !ms) return EXN_EINVAL;
  *ms = e->last_ms;
  return EXN_OK;
}

int exn_test_enc_weights_digest(exn_enc* e, uint64_t* out) {
  if (!e || !out) return EXN_EINVAL;
  ECK(cudaSetDevice(e->cfg.device));
  const exn_enc_config& c = e->cfg;
  const size_t w = c.width, q = q_width(c), kv = kv_width(c), f = c.ffn;
  const size_t per = al256((q + 2 * kv) * w * 2) + al256(w * q * 2) + al256(2 * f * w * 2) + al256(w * f * 2);
  const size_t vbytes = ((2 * w + 2 * kHeadDim) * c.layers + w) * 4;
  unsigned long long* d = nullptr;
  ECK(cudaMalloc(&d, sizeof *d));
  cudaMemsetAsync(d, 0, sizeof *d, e->st);
  digest_launch(e->slab, per * c.layers, d, e->st);
  digest_launch(e->vecs, vbytes & ~size_t(7), d, e->st);
  digest_launch(e->embed, static_cast<size_t>(c.vocab) * w * 4, d, e->st);
  unsigned long long h = 0;
  const cudaError_t r = cudaMemcpyAsync(&h, d, sizeof h, cudaMemcpyDeviceToHost, e->st);
  cudaStreamSynchronize(e->st);
  cudaFree(d);
  ECK(r);
  *out = h;
  return EXN_OK;
}

}  // extern "C"
