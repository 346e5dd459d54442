// dit.cpp -- the host side of libexn_b200.so: the C ABI of include/exn_b200.h.
//
// It does what ex-nihilo's src/cuda-dit.lisp does around its kernels --
// weights checked and uploaded (upload-dit :52-86, open-dit
// src/weights.lisp:47-61), one step's schedule (dit-velocity :137-243), the
// prompt K/V kept under a key (:44-50, 148, 207-218, 232-233), buffers freed
// (dit-release :99-108) -- and the step loop of src/generate.lisp:133-135,
// with these B200-first differences:
//   * weights live in HBM as bf16, dequantised once from Q8_0 (the values a
//     dequantising GEMM would feed the tensor cores); to_q/to_k/to_v are one
//     [3W x W] matrix and gate_up is interleaved by 128 rows so one 256-wide
//     tile holds matching gate and up columns;
//   * the latent, context, RoPE table and timestep embedding stay on the
//     device; the Euler update is fused into proj_out's epilogue;
//   * each layer's K/V buffer holds the whole sequence, so the prompt rows
//     persist across steps without the reference's copies;
//   * B independent pictures run as one batch of rows.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <thread>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/exn_b200.h"
#include "../../include/exn_b200_testing.h"
#include "exn_internal.h"
#include "gguf.h"

using namespace exn;

namespace {

thread_local std::string g_open_error;
const char* kPrefix = "model.diffusion_model.";

struct TensorSpec {
  std::string name;
  std::vector<int64_t> dims;  // ggml order
};

// dit-expected, src/weights.lisp:22-45
std::vector<TensorSpec> expected_tensors(const exn_config& c) {
  const int64_t w = c.width, f = c.ffn;
  std::vector<TensorSpec> v = {
      {"img_in.weight", {c.latent, w}},
      {"txt_in.text_norm.weight", {c.context}},
      {"txt_in.in_layer.weight", {c.context, w}},
      {"txt_in.out_layer.weight", {w, w}},
      {"time_text_embed.timestep_embedder.linear_1.weight", {c.freq, w}},
      {"time_text_embed.timestep_embedder.linear_2.weight", {w, w}},
      {"modulation.1.weight", {w, 4 * w}},
      {"norm_out.linear.weight", {w, w}},
      {"proj_out.weight", {w, c.latent}},
  };
  for (int i = 0; i < c.layers; ++i) {
    const std::string b = "transformer_blocks." + std::to_string(i) + ".";
    v.push_back({b + "attn.norm_q.weight", {c.head_dim}});
    v.push_back({b + "attn.norm_k.weight", {c.head_dim}});
    v.push_back({b + "attn.to_q.weight", {w, w}});
    v.push_back({b + "attn.to_k.weight", {w, w}});
    v.push_back({b + "attn.to_v.weight", {w, w}});
    v.push_back({b + "attn.to_out.0.weight", {w, w}});
    v.push_back({b + "img_mlp.gate_up.weight", {w, 2 * f}});
    v.push_back({b + "img_mlp.out.weight", {f, w}});
  }
  return v;
}

std::string dims_str(const std::vector<int64_t>& d) {
  std::string s = "(";
  for (size_t i = 0; i < d.size(); ++i) s += (i ? " " : "") + std::to_string(d[i]);
  return s + ")";
}

struct GemvW {
  int kind = W_Q8;
  void* w = nullptr;   // int8 qs / bf16 / f32 [out][in]
  __half* d = nullptr; // Q8 scales [out][in/32]
};

struct Profile {
  bool on = false;
  std::vector<std::pair<cudaEvent_t, int>> marks;  // event, category of the work after it
};

// NCCL, bound at run time to whichever libnccl.so.2 the process has (torch's,
// or the system's); only its stable C API is used.
struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) {
      api.why = "libnccl.so.2 not found";
      return;
    }
    bool ok = true;
    auto sym = [&](const char* n) {
      void* f = dlsym(lib, n);
      if (!f) ok = false;
      return f;
    };
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
    api.CommInitRankConfig = reinterpret_cast<decltype(api.CommInitRankConfig)>(sym("ncclCommInitRankConfig"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
    api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(sym("ncclCommAbort"));
    api.CommGetAsyncError = reinterpret_cast<decltype(api.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
    api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(sym("ncclGroupStart"));
    api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(sym("ncclGroupEnd"));
    api.Send = reinterpret_cast<decltype(api.Send)>(sym("ncclSend"));
    api.Recv = reinterpret_cast<decltype(api.Recv)>(sym("ncclRecv"));
    api.AllGather = reinterpret_cast<decltype(api.AllGather)>(sym("ncclAllGather"));
    api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(sym("ncclAllReduce"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
    api.ok = ok;
    if (!ok) api.why = "libnccl.so.2 lacks a symbol this library uses";
  });
  return api;
}

// buffers of a sequence-parallel (Ulysses) pass on one rank
struct SpBufs {
  void* mem = nullptr;       // one allocation, the same layout on every rank (peers address it by offset)
  int cap_nloc = 0, cap_ntot = 0, cap_p = 0, cap_n = 0, cap_wg = 0;
  bf16* qf = nullptr;        // this rank's heads, every row of the pass [n_tot][Wg]: every rank's QKV stores here
  bf16* att_in = nullptr;    // attention out of this rank's rows, all heads [n_loc][W]: every rank's attention
                             // stores its heads' columns here
  float2* rope = nullptr;    // RoPE of this rank's rows [n_loc][64]
  float* zslice = nullptr;   // [64][N/G]
  float* zall = nullptr;     // [G][64][N/G]
  int* bar = nullptr;        // one int the set-up barriers all-reduce
  int* flags = nullptr;      // [kMaxSp]: slot g holds the last barrier epoch rank g arrived at (peers write it)
  int epoch = 0;             // barriers of the passes taken since the buffers were made (the same on every rank)
  size_t off_qf = 0, off_att = 0, off_flags = 0;
  bf16* kv = nullptr;        // [layer][K or V][L][Wg]: this rank's heads of the whole sequence
  int kv_l = 0;
  // every rank's mem and kv mapped into this process (CUDA IPC; this rank's own at its index)
  char* peer_mem[kMaxSp] = {};
  bf16* peer_kv[kMaxSp] = {};
  bool mapped = false;
};

}  // namespace

struct exn_handle {
  exn_config cfg{};
  int sms = 0;
  // attention work split (AttnArgs::split_mode, EXN_ATT_SINGLE at open) and the SM count it plans
  // for (0: the device's); a testing entry point may change both
  int att_mode = 2, att_sms = 0;
  // GEMM tiles (GemmArgs::pairs; EXN_GEMM_PAIRS at open): 1 256 x 256 on CTA pairs, narrower
  // one-CTA tiles where pair tiles would not fill one round; 2 pairs only; 0 one-CTA tiles
  int gemm_pairs = 1;
  cudaStream_t st = nullptr;
  std::string err;
  int* d_status = nullptr;
  std::vector<TensorSpec> spec;
  std::map<std::string, int> index;
  std::vector<char> loaded;
  size_t n_loaded = 0;

  // weights (one slab)
  void* slab = nullptr;
  size_t slab_bytes = 0;
  bf16 *w_qkv = nullptr, *w_out = nullptr, *w_gu = nullptr, *w_down = nullptr;
  bf16 *w_txt_in = nullptr, *w_txt_out = nullptr, *w_img_in = nullptr, *w_proj = nullptr;
  float *norm_q = nullptr, *norm_k = nullptr, *txt_norm = nullptr;
  GemvW lin1, lin2, mod, nout;
  std::vector<void*> extra_allocs;

  // step buffers
  void* act = nullptr;
  size_t act_bytes = 0;
  int cap_batch = 0, cap_rows = 0, cap_l = 0, cap_p = 0, cap_nimg = 0, cap_nref = 0;
  float* x = nullptr;
  bf16 *y = nullptr, *q = nullptr, *att = nullptr, *ff = nullptr, *ctxn = nullptr, *tin = nullptr;
  bf16 *lat_rows = nullptr, *ref_rows = nullptr;
  float *ctx_dev = nullptr, *lat_dev = nullptr, *ref_dev = nullptr, *vout = nullptr;
  float2* rope = nullptr;
  float *emb = nullptr, *e1 = nullptr, *e2 = nullptr, *modv = nullptr, *sc = nullptr;
  bf16* kv = nullptr;          // [layers][2][batch][cap_l][width]
  size_t kv_bytes = 0;
  int kv_batch = 0, kv_l = 0;

  // the kept prompt
  uint64_t prefix_key = 0;
  int prefix_len = 0;
  bool prefix_valid = false;

  // debugging
  float* trace_host = nullptr;
  size_t trace_floats = 0;
  Profile prof;
  // GEMM (other than gate_up), attention, other, gate_up GEMM, sequence-parallel barriers
  double last_ms[5] = {0, 0, 0, 0, 0};
  // device time of the last exn_velocity / exn_generate: inputs uploaded .. result ready to copy back
  cudaEvent_t call_ev[2] = {nullptr, nullptr};
  double last_call_ms = 0;
  long long launches = 0;  // kernels of this library queued by the step code since open

  // sequence parallelism over `world` handles (one per GPU)
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  double comm_timeout_s = 60.0;
  SpBufs sp;
  // host cost of waiting for the communicator: calls of nccl_settle, their 50 us sleeps, seconds
  long long settles = 0, settle_sleeps = 0;
  double settle_s = 0.0;
};

namespace {

int fail(exn_handle* h, int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (h)
    h->err = buf;
  else
    g_open_error = buf;
  return code;
}

#define CK(call)                                                                                    \
  do {                                                                                              \
    cudaError_t e_ = (call);                                                                        \
    if (e_ != cudaSuccess)                                                                          \
      return fail(h, e_ == cudaErrorMemoryAllocation ? EXN_ENOMEM : EXN_ECUDA, "%s: %s (%s:%d)", #call, \
                  cudaGetErrorString(e_), __FILE__, __LINE__);                                      \
  } while (0)

#define CKL(call)                                                                      \
  do {                                                                                 \
    int r_ = (call);                                                                   \
    if (r_ != 0) return fail(h, EXN_ECUDA, "%s failed (%d) at %s:%d", #call, r_, __FILE__, __LINE__); \
  } while (0)

int use_device(exn_handle* h) {
  CK(cudaSetDevice(h->cfg.device));
  return EXN_OK;
}

inline size_t al(size_t n) { return (n + 255) & ~size_t(255); }

// ---------------------------------------------------------------------------- weights

int alloc_weights(exn_handle* h) {
  const exn_config& c = h->cfg;
  const size_t W = c.width, F = c.ffn, L = c.layers;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += al(bytes);
    return o;
  };
  const size_t o_qkv = take(L * 3 * W * W * 2), o_out = take(L * W * W * 2), o_gu = take(L * 2 * F * W * 2),
               o_down = take(L * W * F * 2), o_tin = take(W * c.context * 2), o_tout = take(W * W * 2),
               o_img = take(W * c.latent * 2), o_proj = take(size_t(c.latent) * W * 2),
               o_nq = take(L * c.head_dim * 4), o_nk = take(L * c.head_dim * 4), o_tn = take(size_t(c.context) * 4);
  h->slab_bytes = off;
  CK(cudaMalloc(&h->slab, off));
  char* b = static_cast<char*>(h->slab);
  h->w_qkv = reinterpret_cast<bf16*>(b + o_qkv);
  h->w_out = reinterpret_cast<bf16*>(b + o_out);
  h->w_gu = reinterpret_cast<bf16*>(b + o_gu);
  h->w_down = reinterpret_cast<bf16*>(b + o_down);
  h->w_txt_in = reinterpret_cast<bf16*>(b + o_tin);
  h->w_txt_out = reinterpret_cast<bf16*>(b + o_tout);
  h->w_img_in = reinterpret_cast<bf16*>(b + o_img);
  h->w_proj = reinterpret_cast<bf16*>(b + o_proj);
  h->norm_q = reinterpret_cast<float*>(b + o_nq);
  h->norm_k = reinterpret_cast<float*>(b + o_nk);
  h->txt_norm = reinterpret_cast<float*>(b + o_tn);
  return EXN_OK;
}

// where a 2-D tensor goes: a bf16 GEMM slot (dst, row0, interleave) or a GEMV
struct Route {
  bf16* dst = nullptr;
  long long row0 = 0;
  int ilv = 0;
  GemvW* gemv = nullptr;
  float* vec = nullptr;  // 1-D
  bool plus_one = false; // txt_in.text_norm: used as 1 + w
};

Route route(exn_handle* h, const std::string& name) {
  const exn_config& c = h->cfg;
  const long long W = c.width, F = c.ffn;
  Route r;
  if (name == "img_in.weight") r.dst = h->w_img_in;
  else if (name == "txt_in.text_norm.weight") { r.vec = h->txt_norm; r.plus_one = true; }
  else if (name == "txt_in.in_layer.weight") r.dst = h->w_txt_in;
  else if (name == "txt_in.out_layer.weight") r.dst = h->w_txt_out;
  else if (name == "time_text_embed.timestep_embedder.linear_1.weight") r.gemv = &h->lin1;
  else if (name == "time_text_embed.timestep_embedder.linear_2.weight") r.gemv = &h->lin2;
  else if (name == "modulation.1.weight") r.gemv = &h->mod;
  else if (name == "norm_out.linear.weight") r.gemv = &h->nout;
  else if (name == "proj_out.weight") r.dst = h->w_proj;
  else {
    int il = -1;
    char part[128] = {0};
    if (sscanf(name.c_str(), "transformer_blocks.%d.%127s", &il, part) == 2 && il >= 0 && il < c.layers) {
      const std::string p = part;
      if (p == "attn.norm_q.weight") r.vec = h->norm_q + il * c.head_dim;
      else if (p == "attn.norm_k.weight") r.vec = h->norm_k + il * c.head_dim;
      else if (p == "attn.to_q.weight") { r.dst = h->w_qkv; r.row0 = il * 3 * W; }
      else if (p == "attn.to_k.weight") { r.dst = h->w_qkv; r.row0 = il * 3 * W + W; }
      else if (p == "attn.to_v.weight") { r.dst = h->w_qkv; r.row0 = il * 3 * W + 2 * W; }
      else if (p == "attn.to_out.0.weight") { r.dst = h->w_out; r.row0 = il * W; }
      else if (p == "img_mlp.gate_up.weight") { r.dst = h->w_gu; r.row0 = il * 2 * F; r.ilv = static_cast<int>(F); }
      else if (p == "img_mlp.out.weight") { r.dst = h->w_down; r.row0 = il * W; }
    }
  }
  return r;
}

// Place one tensor whose GGUF bytes are on the device (RAW).  Q8_0 matrices
// become bf16 (GEMM) or stay Q8_0 (GEMV); f32/f16/bf16 are converted.
int place(exn_handle* h, int idx, int type, const void* raw, void* scratch) {
  const TensorSpec& s = h->spec[idx];
  Route r = route(h, s.name);
  const long long cols = s.dims[0];
  const long long rows = s.dims.size() > 1 ? s.dims[1] : 1;
  const long long n = rows * cols;
  if (r.vec) {
    if (type == GGML_F32) CK(cudaMemcpyAsync(r.vec, raw, n * 4, cudaMemcpyDeviceToDevice, h->st));
    else if (type == GGML_F16) f16_to_f32_launch(static_cast<const __half*>(raw), r.vec, n, h->st);
    else if (type == GGML_BF16) bf16_to_f32_launch(static_cast<const bf16*>(raw), r.vec, n, h->st);
    else return fail(h, EXN_EUNSUPPORTED, "%s: ggml type %d for a vector", s.name.c_str(), type);
    if (r.plus_one) add_scalar_launch(r.vec, n, 1.f, h->st);
  } else if (r.gemv) {
    GemvW& g = *r.gemv;
    if (type == GGML_Q8_0) {
      void* qs = nullptr;
      void* d = nullptr;
      CK(cudaMalloc(&qs, n));
      h->extra_allocs.push_back(qs);
      CK(cudaMalloc(&d, (n / 32) * 2));
      h->extra_allocs.push_back(d);
      q8_raw_split_launch(static_cast<const uint8_t*>(raw), static_cast<int8_t*>(qs), static_cast<__half*>(d), n / 32,
                          h->st);
      g.kind = W_Q8;
      g.w = qs;
      g.d = static_cast<__half*>(d);
    } else if (type == GGML_BF16) {
      void* w = nullptr;
      CK(cudaMalloc(&w, n * 2));
      h->extra_allocs.push_back(w);
      CK(cudaMemcpyAsync(w, raw, n * 2, cudaMemcpyDeviceToDevice, h->st));
      g.kind = W_BF16;
      g.w = w;
    } else if (type == GGML_F32 || type == GGML_F16) {
      void* w = nullptr;
      CK(cudaMalloc(&w, n * 4));
      h->extra_allocs.push_back(w);
      if (type == GGML_F32) CK(cudaMemcpyAsync(w, raw, n * 4, cudaMemcpyDeviceToDevice, h->st));
      else f16_to_f32_launch(static_cast<const __half*>(raw), static_cast<float*>(w), n, h->st);
      g.kind = W_F32;
      g.w = w;
    } else {
      return fail(h, EXN_EUNSUPPORTED, "%s: ggml type %d", s.name.c_str(), type);
    }
  } else if (r.dst) {
    if (type == GGML_Q8_0) {
      q8_raw_to_bf16_launch(static_cast<const uint8_t*>(raw), r.dst, rows, static_cast<int>(cols), r.row0, r.ilv, h->st);
    } else if (type == GGML_BF16) {
      bf16_rows_launch(static_cast<const bf16*>(raw), r.dst, rows, static_cast<int>(cols), r.row0, r.ilv, h->st);
    } else if (type == GGML_F32) {
      f32_to_bf16_rows_launch(static_cast<const float*>(raw), r.dst, rows, static_cast<int>(cols), r.row0, r.ilv, h->st);
    } else if (type == GGML_F16) {
      float* f = static_cast<float*>(scratch);
      f16_to_f32_launch(static_cast<const __half*>(raw), f, n, h->st);
      f32_to_bf16_rows_launch(f, r.dst, rows, static_cast<int>(cols), r.row0, r.ilv, h->st);
    } else {
      return fail(h, EXN_EUNSUPPORTED, "%s: ggml type %d", s.name.c_str(), type);
    }
  } else {
    return fail(h, EXN_EINVAL, "no place for tensor %s", s.name.c_str());
  }
  CK(cudaGetLastError());
  if (!h->loaded[idx]) {
    h->loaded[idx] = 1;
    ++h->n_loaded;
  }
  return EXN_OK;
}

int check_tensor(exn_handle* h, const std::string& name, int type, const std::vector<int64_t>& dims, int* idx) {
  auto it = h->index.find(name);
  if (it == h->index.end()) return fail(h, EXN_ESHAPE, "%s: not a tensor of the DiT", name.c_str());
  const TensorSpec& s = h->spec[it->second];
  if (s.dims != dims)
    return fail(h, EXN_ESHAPE, "%s is %s, not %s", name.c_str(), dims_str(dims).c_str(), dims_str(s.dims).c_str());
  if (type != GGML_F32 && type != GGML_F16 && type != GGML_BF16 && type != GGML_Q8_0)
    return fail(h, EXN_EUNSUPPORTED, "%s: ggml type %d not handled", name.c_str(), type);
  if (type == GGML_Q8_0 && dims.size() == 1)
    return fail(h, EXN_EUNSUPPORTED, "%s: a Q8_0 vector", name.c_str());
  *idx = it->second;
  return EXN_OK;
}

// ---------------------------------------------------------------------------- step buffers

int ensure_buffers(exn_handle* h, int batch, int n, int l, int ptext, int nimg, int nref, bool with_kv = true) {
  const exn_config& c = h->cfg;
  const size_t W = c.width;
  // per-step activations
  if (batch > h->cap_batch || n > h->cap_rows || l > h->cap_l || ptext > h->cap_p || nimg > h->cap_nimg ||
      nref > h->cap_nref) {
    const int B = std::max(batch, h->cap_batch), R = std::max(n, h->cap_rows), Lc = std::max(l, h->cap_l);
    const int P = std::max(ptext, h->cap_p), NI = std::max(nimg, h->cap_nimg), NR = std::max(nref, h->cap_nref);
    const size_t rows = static_cast<size_t>(B) * R;
    size_t off = 0;
    auto take = [&](size_t bytes) {
      size_t o = off;
      off += al(bytes);
      return o;
    };
    const size_t ox = take(rows * W * 4), oy = take(rows * W * 2), oq = take(rows * W * 2), oa = take(rows * W * 2),
                 of = take(rows * c.ffn * 2), ocn = take(size_t(B) * P * c.context * 2),
                 oti = take(size_t(B) * P * W * 2), olr = take(size_t(B) * NI * c.latent * 2),
                 orr = take(size_t(B) * std::max(NR, 1) * c.latent * 2), ocd = take(size_t(B) * P * c.context * 4),
                 old = take(size_t(B) * NI * c.latent * 4), ord = take(size_t(B) * std::max(NR, 1) * c.latent * 4),
                 ov = take(size_t(B) * NI * c.latent * 4), orp = take(size_t(Lc) * 64 * 8),
                 oe = take(2 * c.freq * 4), oe1 = take(2 * W * 4), oe2 = take(2 * W * 4), om = take(8 * W * 4),
                 osc = take(W * 4);
    if (h->act) cudaFree(h->act);
    h->act = nullptr;
    CK(cudaMalloc(&h->act, off));
    h->act_bytes = off;
    char* b = static_cast<char*>(h->act);
    h->x = reinterpret_cast<float*>(b + ox);
    h->y = reinterpret_cast<bf16*>(b + oy);
    h->q = reinterpret_cast<bf16*>(b + oq);
    h->att = reinterpret_cast<bf16*>(b + oa);
    h->ff = reinterpret_cast<bf16*>(b + of);
    h->ctxn = reinterpret_cast<bf16*>(b + ocn);
    h->tin = reinterpret_cast<bf16*>(b + oti);
    h->lat_rows = reinterpret_cast<bf16*>(b + olr);
    h->ref_rows = reinterpret_cast<bf16*>(b + orr);
    h->ctx_dev = reinterpret_cast<float*>(b + ocd);
    h->lat_dev = reinterpret_cast<float*>(b + old);
    h->ref_dev = reinterpret_cast<float*>(b + ord);
    h->vout = reinterpret_cast<float*>(b + ov);
    h->rope = reinterpret_cast<float2*>(b + orp);
    h->emb = reinterpret_cast<float*>(b + oe);
    h->e1 = reinterpret_cast<float*>(b + oe1);
    h->e2 = reinterpret_cast<float*>(b + oe2);
    h->modv = reinterpret_cast<float*>(b + om);
    h->sc = reinterpret_cast<float*>(b + osc);
    h->cap_batch = B;
    h->cap_rows = R;
    h->cap_l = Lc;
    h->cap_p = P;
    h->cap_nimg = NI;
    h->cap_nref = NR;
  }
  // K/V: [layers][2][batch][kv_l][W]; grown keeping the kept prompt rows
  if (with_kv && (batch != h->kv_batch || l > h->kv_l)) {
    const int Lk = std::max(l, h->kv_l);
    const size_t bytes = static_cast<size_t>(c.layers) * 2 * batch * Lk * W * 2;
    bf16* nk = nullptr;
    CK(cudaMalloc(&nk, bytes));
    if (h->kv && h->prefix_valid && batch == h->kv_batch && h->prefix_len > 0) {
      for (int i = 0; i < c.layers * 2 * batch; ++i)
        CK(cudaMemcpyAsync(nk + static_cast<size_t>(i) * Lk * W, h->kv + static_cast<size_t>(i) * h->kv_l * W,
                           static_cast<size_t>(h->prefix_len) * W * 2, cudaMemcpyDeviceToDevice, h->st));
    } else {
      h->prefix_valid = false;
      h->prefix_key = 0;
    }
    CK(cudaStreamSynchronize(h->st));
    if (h->kv) cudaFree(h->kv);
    h->kv = nk;
    h->kv_bytes = bytes;
    h->kv_batch = batch;
    h->kv_l = Lk;
  }
  return EXN_OK;
}

void free_buffers(exn_handle* h) {
  if (h->act) cudaFree(h->act);
  if (h->kv) cudaFree(h->kv);
  h->act = nullptr;
  h->kv = nullptr;
  h->act_bytes = h->kv_bytes = 0;
  h->cap_batch = h->cap_rows = h->cap_l = h->cap_p = h->cap_nimg = h->cap_nref = 0;
  h->kv_batch = h->kv_l = 0;
  h->prefix_valid = false;
  h->prefix_key = 0;
  h->prefix_len = 0;
}

// ---------------------------------------------------------------------------- profiling

void prof_mark(exn_handle* h, int cat) {
  if (!h->prof.on) return;
  cudaEvent_t e;
  cudaEventCreate(&e);
  cudaEventRecord(e, h->st);
  h->prof.marks.push_back({e, cat});
}

void prof_collect(exn_handle* h) {
  if (!h->prof.on || h->prof.marks.size() < 2) return;
  cudaEventSynchronize(h->prof.marks.back().first);
  double acc[5] = {0, 0, 0, 0, 0};
  for (size_t i = 0; i + 1 < h->prof.marks.size(); ++i) {
    float ms = 0;
    cudaEventElapsedTime(&ms, h->prof.marks[i].first, h->prof.marks[i + 1].first);
    acc[h->prof.marks[i].second] += ms;
  }
  for (auto& m : h->prof.marks) cudaEventDestroy(m.first);
  h->prof.marks.clear();
  for (int i = 0; i < 5; ++i) h->last_ms[i] = acc[i];
}

// ---------------------------------------------------------------------------- one step

struct StepIn {
  int batch = 1, ptext = 0, nref = 0, a = 0, rh = 0, rw = 0, hh = 0, ww = 0;
  double sigma = 0;
  bool cached = false;
  const float* ctx = nullptr;   // device [B][ptext][context]
  const float* ref = nullptr;   // device [B][64][nref]
  const float* lat = nullptr;   // device [B][64][nimg]
  float* z = nullptr;           // device: z += dsigma * v
  float dsigma = 0.f;
  float* v = nullptr;           // device: v out
};

int gemm(exn_handle* h, const bf16* a, long long lda, const bf16* b, long long ldb, int M, int N, int K, int epi,
         const GemmEpi& ep) {
  GemmArgs g;
  g.a = a;
  g.lda = lda;
  g.b = b;
  g.ldb = ldb;
  g.M = M;
  g.N = N;
  g.K = K;
  g.epi = epi;
  g.ep = ep;
  g.pairs = h->gemm_pairs;
  const int r = gemm_launch(g, h->d_status, h->sms, h->st);
  if (r) return fail(h, EXN_ECUDA, "GEMM %dx%dx%d (epilogue %d) launch failed: %d", M, N, K, epi, r);
  return EXN_OK;
}

// emb(1000 sigma), emb(0) -> linear_1, SiLU -> linear_2, SiLU -> modulation (gates tanh'd) and
// norm_out (row 0 only): src/cuda-dit.lisp:157-167
int timestep_chain(exn_handle* h, double sigma) {
  const exn_config& c = h->cfg;
  const int W = c.width;
  temb_launch(h->emb, sigma, c.freq, h->st);
  int r = gemv_launch(h->lin1.kind, h->lin1.w, h->lin1.d, h->emb, h->e1, 2, c.freq, W, 1, 0, h->st);
  if (!r) r = gemv_launch(h->lin2.kind, h->lin2.w, h->lin2.d, h->e1, h->e2, 2, W, W, 1, 0, h->st);
  if (!r) r = gemv_launch(h->mod.kind, h->mod.w, h->mod.d, h->e2, h->modv, 2, W, 4 * W, 2, W, h->st);
  if (!r) r = gemv_launch(h->nout.kind, h->nout.w, h->nout.d, h->e2, h->sc, 1, W, W, 0, 0, h->st);
  if (r) return fail(h, EXN_ECUDA, "timestep GEMV launch failed: %d", r);
  return EXN_OK;
}

int run_step(exn_handle* h, const StepIn& in) {
  const exn_config& c = h->cfg;
  // kernels this step queues (timestep 5, inputs 2 or 5 (+2 with a reference), RoPE 1, 7 a block, final 2)
  h->launches += 5 + 2 + 1 + 7LL * c.layers + 2 + (in.cached ? 0 : (in.ptext > 0 ? 3 : 0) + (in.nref ? 2 : 0));
  const int W = c.width, B = in.batch;
  const int p = in.ptext + in.nref, nimg = in.hh * in.ww;
  const int n0 = in.cached ? p : 0, n = in.cached ? nimg : p + nimg, L = p + nimg;
  const int b0 = in.nref ? in.a : 0, b1 = in.nref ? in.a + in.nref : 0;
  int rc;
  if ((rc = ensure_buffers(h, B, n, L, in.ptext, nimg, in.nref))) return rc;
  const size_t kv_layer = static_cast<size_t>(2) * B * h->kv_l * W;
  const long long kv_sample = static_cast<long long>(h->kv_l) * W;

  prof_mark(h, 2);
  // timestep: emb(t), emb(0) -> linear_1, SiLU -> linear_2, SiLU -> modulation (gates tanh'd), norm_out (row 0)
  if ((rc = timestep_chain(h, in.sigma))) return rc;
  // the prompt (and an edit's picture) through txt_in / img_in, first pass only
  if (!in.cached && in.ptext > 0) {
    rms_launch(in.ctx, h->txt_norm, h->ctxn, B * in.ptext, c.context, h->st);
    prof_mark(h, 0);
    GemmEpi e1;
    e1.out = h->tin;
    e1.ld_out = W;
    if ((rc = gemm(h, h->ctxn, c.context, h->w_txt_in, c.context, B * in.ptext, W, c.context, EPI_GELU_BF16, e1)))
      return rc;
    GemmEpi e2;
    e2.out = h->x;
    e2.ld_out = W;
    e2.seg_in = in.ptext;
    e2.seg_out = n;
    e2.off = 0;
    e2.split_at = in.nref ? in.a : (1 << 30);
    e2.split_gap = in.nref;
    if ((rc = gemm(h, h->tin, W, h->w_txt_out, W, B * in.ptext, W, W, EPI_F32, e2))) return rc;
  }
  if (!in.cached) {
    if (in.nref) {
      prof_mark(h, 2);
      latent_rows_launch(in.ref, h->ref_rows, B, c.latent, in.nref, h->st);
      prof_mark(h, 0);
      GemmEpi er;
      er.out = h->x;
      er.ld_out = W;
      er.seg_in = in.nref;
      er.seg_out = n;
      er.off = in.a;
      if ((rc = gemm(h, h->ref_rows, c.latent, h->w_img_in, c.latent, B * in.nref, W, c.latent, EPI_F32, er))) return rc;
    }
    prof_mark(h, 2);
  }
  latent_rows_launch(in.lat, h->lat_rows, B, c.latent, nimg, h->st);
  prof_mark(h, 0);
  {
    GemmEpi ei;
    ei.out = h->x;
    ei.ld_out = W;
    ei.seg_in = nimg;
    ei.seg_out = n;
    ei.off = p - n0;
    if ((rc = gemm(h, h->lat_rows, c.latent, h->w_img_in, c.latent, B * nimg, W, c.latent, EPI_F32, ei))) return rc;
  }
  prof_mark(h, 2);
  rope_table_launch(h->rope, 0, L, p, in.hh, in.ww, in.nref ? in.a : 0, in.nref ? in.rh : 0, in.nref ? in.rw : 0,
                    h->st);
  if (h->trace_host && !in.cached) {
    CK(cudaStreamSynchronize(h->st));
  }
  size_t traced = 0;
  auto trace = [&](const float* src, int rows) -> int {
    if (!h->trace_host) return EXN_OK;
    const size_t nf = static_cast<size_t>(rows) * W;
    if (traced + nf > h->trace_floats) return EXN_OK;
    CK(cudaMemcpyAsync(h->trace_host + traced, src, nf * 4, cudaMemcpyDeviceToHost, h->st));
    CK(cudaStreamSynchronize(h->st));
    traced += nf;
    return EXN_OK;
  };
  if (h->trace_host && (rc = trace(h->x, B * n))) return rc;

  const int rows = B * n;
  for (int il = 0; il < c.layers; ++il) {
    bf16* kl = h->kv + il * kv_layer;
    bf16* vl = kl + static_cast<size_t>(B) * h->kv_l * W;
    ln_mod_launch(h->x, h->y, h->modv + 0 * W, 4 * W, rows, W, n, n, 0, n0, p, 0, h->st);
    prof_mark(h, 0);
    GemmEpi eq;
    eq.seg_in = n;
    eq.n0 = n0;
    eq.width = W;
    eq.norm_q = h->norm_q + il * c.head_dim;
    eq.norm_k = h->norm_k + il * c.head_dim;
    eq.rope = h->rope;
    eq.q = h->q;
    eq.k = kl;
    eq.v = vl;
    eq.kv_sample_stride = kv_sample;
    if ((rc = gemm(h, h->y, W, h->w_qkv + static_cast<size_t>(il) * 3 * W * W, W, rows, 3 * W, W, EPI_QKV, eq)))
      return rc;
    prof_mark(h, 1);
    AttnArgs aa;
    aa.q = h->q;
    aa.k = kl;
    aa.v = vl;
    aa.out = h->att;
    aa.batch = B;
    aa.nq = n;
    aa.q0 = n0;
    aa.p = p;
    aa.l = L;
    aa.b0 = b0;
    aa.b1 = b1;
    aa.heads = W / 128;
    aa.width = W;
    aa.kv_rows = h->kv_l;
    aa.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(c.head_dim)));
    aa.sms = h->att_sms ? h->att_sms : h->sms;
    aa.split_mode = h->att_mode;
    if ((rc = attention_launch(aa, h->d_status, h->st))) return fail(h, EXN_ECUDA, "attention launch failed: %d", rc);
    prof_mark(h, 0);
    GemmEpi eo;
    eo.out = h->x;
    eo.ld_out = W;
    eo.seg_in = n;
    eo.mod = h->modv + 1 * W;
    eo.mod_stride = 4 * W;
    eo.n0 = n0;
    eo.p = p;
    if ((rc = gemm(h, h->att, W, h->w_out + static_cast<size_t>(il) * W * W, W, rows, W, W, EPI_GATE_RESID, eo)))
      return rc;
    prof_mark(h, 2);
    ln_mod_launch(h->x, h->y, h->modv + 2 * W, 4 * W, rows, W, n, n, 0, n0, p, 0, h->st);
    prof_mark(h, 3);
    GemmEpi eg;
    eg.out = h->ff;
    eg.ld_out = c.ffn;
    if ((rc = gemm(h, h->y, W, h->w_gu + static_cast<size_t>(il) * 2 * c.ffn * W, W, rows, 2 * c.ffn, W, EPI_SWIGLU,
                   eg)))
      return rc;
    prof_mark(h, 0);
    GemmEpi ed = eo;
    ed.mod = h->modv + 3 * W;
    if ((rc = gemm(h, h->ff, c.ffn, h->w_down + static_cast<size_t>(il) * W * c.ffn, c.ffn, rows, W, c.ffn,
                   EPI_GATE_RESID, ed)))
      return rc;
    prof_mark(h, 2);
    if (h->trace_host && (rc = trace(h->x, rows))) return rc;
  }
  // the image rows: LayerNorm * (1 + sc), proj_out (+ the Euler update)
  ln_mod_launch(h->x, h->y, h->sc, 0, B * nimg, W, nimg, n, p - n0, n0, p, 1, h->st);
  prof_mark(h, 0);
  GemmEpi ep;
  ep.z = in.z;
  ep.vout = in.v;
  ep.dsigma = in.dsigma;
  ep.nimg = nimg;
  if ((rc = gemm(h, h->y, W, h->w_proj, W, B * nimg, c.latent, W, EPI_PROJ, ep))) return rc;
  prof_mark(h, 2);
  CK(cudaGetLastError());
  return EXN_OK;
}


// ---------------------------------------------------------------------------- sequence parallelism

int nccl_fail(exn_handle* h, ncclResult_t r, const char* what) {
  return fail(h, EXN_ECUDA, "%s: %s", what, nccl().GetErrorString ? nccl().GetErrorString(r) : "nccl error");
}

// a non-blocking communicator's queued work, or its init, settled (bounded by comm_timeout_s)
int nccl_settle(exn_handle* h, ncclComm_t comm, const char* what) {
  const auto t0 = std::chrono::steady_clock::now();
  ++h->settles;
  while (true) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = nccl().CommGetAsyncError(comm, &st);
    if (r != ncclSuccess) return nccl_fail(h, r, what);
    if (st == ncclSuccess) {
      h->settle_s += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      return EXN_OK;
    }
    ++h->settle_sleeps;
    if (st != ncclInProgress) return nccl_fail(h, st, what);
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > h->comm_timeout_s) {
      nccl().CommAbort(comm);
      if (comm == h->comm) h->comm = nullptr;
      return fail(h, EXN_ETIMEOUT, "%s: no progress in %.0f s, communicator aborted", what, h->comm_timeout_s);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// A barrier of the sequence-parallel group on the handle's stream: a one-int all-reduce.  What a
// rank's kernels stored into peers' memory before it (each writer fences at system scope) is
// visible to every rank's kernels after it.
int check_status(exn_handle* h);

int sp_barrier(exn_handle* h, const char* what) {
  const ncclResult_t nr = nccl().AllReduce(h->sp.bar, h->sp.bar, 1, ncclInt32, ncclSum, h->comm, h->st);
  if (nr != ncclSuccess && nr != ncclInProgress) return nccl_fail(h, nr, what);
  return nccl_settle(h, h->comm, what);
}

// A barrier of the pass on the device: a one-block kernel stores this barrier's epoch into every
// rank's arrival slot for this rank (peer memory over NVLink, release at system scope) and waits,
// bounded, until every rank's slot here holds it.  What a rank's kernels stored into peers before it
// (each writer fences at system scope) is then visible to every rank's kernels after it.  The host
// only queues it: unlike a collective of a non-blocking communicator it never waits for the enqueue.
int sp_flag_barrier(exn_handle* h) {
  SpBufs& b = h->sp;
  SpFlags f;
  for (int g = 0; g < kMaxSp; ++g)
    f.peer[g] = g < h->world ? reinterpret_cast<int*>(b.peer_mem[g] + b.off_flags) + h->rank : nullptr;
  f.mine = b.flags;
  ++b.epoch;
  ++h->launches;
  const int r = sp_flag_barrier_launch(f, h->world, b.epoch, h->d_status, h->st);
  if (r) return fail(h, EXN_ECUDA, "pass barrier launch failed: %d", r);
  return EXN_OK;
}

// Unmap the peers' buffers (after this rank's queued work is done).
void sp_unmap(exn_handle* h) {
  SpBufs& b = h->sp;
  if (b.mapped) {
    cudaStreamSynchronize(h->st);
    for (int g = 0; g < h->world && g < kMaxSp; ++g) {
      if (g == h->rank) continue;
      if (b.peer_mem[g]) cudaIpcCloseMemHandle(b.peer_mem[g]);
      if (b.peer_kv[g]) cudaIpcCloseMemHandle(b.peer_kv[g]);
    }
  }
  for (int g = 0; g < kMaxSp; ++g) {
    b.peer_mem[g] = nullptr;
    b.peer_kv[g] = nullptr;
  }
  b.mapped = false;
}

// Export this rank's mem and kv (CUDA IPC handles), all-gather every rank's over the communicator
// and map the peers', so kernels can store straight into any rank's buffers over NVLink.
int sp_map(exn_handle* h) {
  SpBufs& b = h->sp;
  const int G = h->world, r = h->rank;
  cudaIpcMemHandle_t mine[2];
  CK(cudaIpcGetMemHandle(&mine[0], b.mem));
  CK(cudaIpcGetMemHandle(&mine[1], b.kv));
  const size_t hb = sizeof mine;
  std::vector<char> all(hb * G);
  char* d = nullptr;
  CK(cudaMalloc(&d, hb * G));
  CK(cudaMemcpyAsync(d + hb * r, mine, hb, cudaMemcpyHostToDevice, h->st));
  const ncclResult_t nr = nccl().AllGather(d + hb * r, d, hb, ncclUint8, h->comm, h->st);
  int rc = EXN_OK;
  if (nr != ncclSuccess && nr != ncclInProgress) rc = nccl_fail(h, nr, "exchange of the peer buffers");
  if (!rc) rc = nccl_settle(h, h->comm, "exchange of the peer buffers");
  if (!rc) rc = check_status(h);
  if (!rc && cudaMemcpy(all.data(), d, hb * G, cudaMemcpyDeviceToHost) != cudaSuccess)
    rc = fail(h, EXN_ECUDA, "exchange of the peer buffers: copy failed");
  cudaFree(d);
  if (rc) return rc;
  for (int g = 0; g < G; ++g) {
    if (g == r) {
      b.peer_mem[g] = static_cast<char*>(b.mem);
      b.peer_kv[g] = b.kv;
      continue;
    }
    cudaIpcMemHandle_t th[2];
    std::memcpy(th, all.data() + hb * g, hb);
    void* pm = nullptr;
    void* pk = nullptr;
    CK(cudaIpcOpenMemHandle(&pm, th[0], cudaIpcMemLazyEnablePeerAccess));
    b.peer_mem[g] = static_cast<char*>(pm);
    CK(cudaIpcOpenMemHandle(&pk, th[1], cudaIpcMemLazyEnablePeerAccess));
    b.peer_kv[g] = static_cast<bf16*>(pk);
  }
  b.mapped = true;
  return EXN_OK;
}

int ensure_sp(exn_handle* h, int n_loc, int n_tot, int P, int N, int L) {
  const exn_config& c = h->cfg;
  const int G = h->world, W = c.width, Wg = W / G;
  SpBufs& b = h->sp;
  const bool grow_mem = n_loc > b.cap_nloc || n_tot > b.cap_ntot || P > b.cap_p || N > b.cap_n || Wg != b.cap_wg;
  const bool grow_kv = L > b.kv_l;
  int rc;
  // every rank takes the same decisions here (same arguments on every rank); before anyone frees
  // a buffer, every peer has unmapped it
  if ((grow_mem || grow_kv) && b.mapped) {
    sp_unmap(h);
    if ((rc = sp_barrier(h, "unmapping the peer buffers")) || (rc = check_status(h))) return rc;
  }
  if (grow_mem) {
    const int NL = std::max(n_loc, b.cap_nloc), NT = std::max(n_tot, b.cap_ntot), PP = std::max(P, b.cap_p),
              NN = std::max(N, b.cap_n);
    size_t off = 0;
    auto take = [&](size_t bytes) {
      size_t o = off;
      off += al(bytes);
      return o;
    };
    const size_t oqf = take(size_t(NT) * Wg * 2),
                 oat = take(size_t(NL) * W * 2), orp = take(size_t(NL) * 64 * 8),
                 ozs = take(size_t(64) * (NN / G) * 4), oza = take(size_t(64) * NN * 4), obar = take(sizeof(int)),
                 oflg = take(kMaxSp * sizeof(int));
    if (b.mem) cudaFree(b.mem);
    b.mem = nullptr;
    CK(cudaMalloc(&b.mem, off));
    char* m = static_cast<char*>(b.mem);
    b.qf = reinterpret_cast<bf16*>(m + oqf);
    b.att_in = reinterpret_cast<bf16*>(m + oat);
    b.rope = reinterpret_cast<float2*>(m + orp);
    b.zslice = reinterpret_cast<float*>(m + ozs);
    b.zall = reinterpret_cast<float*>(m + oza);
    b.bar = reinterpret_cast<int*>(m + obar);
    b.flags = reinterpret_cast<int*>(m + oflg);
    CK(cudaMemsetAsync(b.flags, 0, kMaxSp * sizeof(int), h->st));  // before the exchange that lets peers write
    b.epoch = 0;
    b.off_qf = oqf;
    b.off_att = oat;
    b.off_flags = oflg;
    b.cap_nloc = NL;
    b.cap_ntot = NT;
    b.cap_p = PP;
    b.cap_n = NN;
    b.cap_wg = Wg;
  }
  if (L > b.kv_l) {  // [layer][2][L][Wg], the kept prompt rows carried over
    bf16* nk = nullptr;
    CK(cudaMalloc(&nk, size_t(c.layers) * 2 * L * Wg * 2));
    if (b.kv && h->prefix_valid && h->prefix_len > 0)
      for (int i = 0; i < c.layers * 2; ++i)
        CK(cudaMemcpyAsync(nk + size_t(i) * L * Wg, b.kv + size_t(i) * b.kv_l * Wg, size_t(h->prefix_len) * Wg * 2,
                           cudaMemcpyDeviceToDevice, h->st));
    else {
      h->prefix_valid = false;
      h->prefix_key = 0;
    }
    CK(cudaStreamSynchronize(h->st));
    if (b.kv) cudaFree(b.kv);
    b.kv = nk;
    b.kv_l = L;
  }
  if (!b.mapped && (rc = sp_map(h))) return rc;
  return EXN_OK;
}

void free_sp(exn_handle* h) {
  sp_unmap(h);
  if (h->sp.mem) cudaFree(h->sp.mem);
  if (h->sp.kv) cudaFree(h->sp.kv);
  h->sp = SpBufs();
}

// One DiT pass with this rank's share of the rows (Ulysses): every GEMM and
// elementwise kernel on the rank's rows; before attention an all-to-all turns
// [rows of this rank x all heads] into [all rows x this rank's heads]; after
// it, back.  A rank holds prefix rows [r P/G, (r+1) P/G) (first pass only) and
// image rows [r N/G, (r+1) N/G).  Its K/V cache holds its heads for every row,
// so the prompt's K/V kept from the first pass stay sharded by head.
int run_step_sp(exn_handle* h, const StepIn& in) {
  const exn_config& c = h->cfg;
  const int G = h->world, r = h->rank, W = c.width, Wg = W / G, heads = W / 128;
  const int P = in.ptext + in.nref, N = in.hh * in.ww, L = P + N;
  if (in.batch != 1) return fail(h, EXN_EINVAL, "sequence parallelism runs one picture at a time");
  if (heads % G || Wg % 256 || P % G || N % G)
    return fail(h, EXN_EINVAL,
                "sequence parallelism over %d GPUs needs heads (%d), prefix rows (%d) and image rows (%d) divisible by "
                "it and width / GPUs (%d) a multiple of 256",
                G, heads, P, N, Wg);
  const int pl = P / G, Nl = N / G;
  const int pl_loc = in.cached ? 0 : pl;
  const int n_loc = pl_loc + Nl, n_tot = in.cached ? N : L, q0 = in.cached ? P : 0;
  const int img0 = in.cached ? 0 : P;  // first image row in qf / af
  int rc;
  if ((rc = ensure_buffers(h, 1, std::max(n_loc, 1), L, std::max(in.ptext, 1), N, in.nref, false))) return rc;
  if ((rc = ensure_sp(h, n_loc, n_tot, P, N, L))) return rc;
  SpBufs& b = h->sp;
  const size_t kv_layer = size_t(2) * b.kv_l * Wg;
  h->launches += 5 + 3 + 7LL * c.layers + 2 + (in.cached ? 0 : (in.ptext > 0 ? 3 : 0) + (in.nref ? 2 : 0));

  // timestep
  prof_mark(h, 2);
  if ((rc = timestep_chain(h, in.sigma))) return rc;
  prof_mark(h, 0);
  // first pass: this rank's prefix rows [lo, hi) through txt_in (the text rows among them) and
  // img_in (an edit picture's rows among them), straight into its x.  Prefix row of text row t: t
  // before the picture's A rows, t + nref after them; the picture holds prefix rows [a, a + nref).
  if (!in.cached) {
    const int lo = r * pl, hi = lo + pl, a = in.nref ? in.a : in.ptext, nref = in.nref;
    const int t0 = lo <= a ? lo : std::max(lo - nref, a), t1 = hi <= a ? hi : std::max(hi - nref, a);
    if (t1 > t0) {
      rms_launch(in.ctx + size_t(t0) * c.context, h->txt_norm, h->ctxn, t1 - t0, c.context, h->st);
      GemmEpi e1;
      e1.out = h->tin;
      e1.ld_out = W;
      if ((rc = gemm(h, h->ctxn, c.context, h->w_txt_in, c.context, t1 - t0, W, c.context, EPI_GELU_BF16, e1)))
        return rc;
      GemmEpi e2;
      e2.out = h->x;
      e2.ld_out = W;
      e2.off = (t0 < a ? t0 : t0 + nref) - lo;
      e2.split_at = t0 < a ? a - t0 : (1 << 30);
      e2.split_gap = nref;
      if ((rc = gemm(h, h->tin, W, h->w_txt_out, W, t1 - t0, W, W, EPI_F32, e2))) return rc;
    }
    const int r0 = std::max(lo, a), r1 = std::min(hi, a + nref);
    if (nref && r1 > r0) {
      latent_rows_launch(in.ref, h->ref_rows, 1, c.latent, r1 - r0, h->st, nref, r0 - a);
      GemmEpi er;
      er.out = h->x;
      er.ld_out = W;
      er.off = r0 - lo;
      if ((rc = gemm(h, h->ref_rows, c.latent, h->w_img_in, c.latent, r1 - r0, W, c.latent, EPI_F32, er))) return rc;
    }
  }
  // this rank's image rows: latent columns [r N/G, (r+1) N/G)
  latent_rows_launch(in.lat, h->lat_rows, 1, c.latent, Nl, h->st, N, r * Nl);
  {
    GemmEpi ei;
    ei.out = h->x;
    ei.ld_out = W;
    ei.off = pl_loc;
    if ((rc = gemm(h, h->lat_rows, c.latent, h->w_img_in, c.latent, Nl, W, c.latent, EPI_F32, ei))) return rc;
  }
  if (pl_loc > 0)
    rope_table_launch(b.rope, r * pl, n_loc, P, in.hh, in.ww, in.nref ? in.a : 0, in.nref ? in.rh : 0,
                      in.nref ? in.rw : 0, h->st, pl_loc, P + r * Nl);
  else
    rope_table_launch(b.rope, P + r * Nl, n_loc, P, in.hh, in.ww, in.nref ? in.a : 0, in.nref ? in.rh : 0,
                      in.nref ? in.rw : 0, h->st);

  for (int il = 0; il < c.layers; ++il) {
    const size_t kl_off = il * kv_layer;
    prof_mark(h, 2);
    ln_mod_launch(h->x, h->y, h->modv + 0 * W, 4 * W, n_loc, W, n_loc, n_loc, 0, 0, pl_loc, 0, h->st);
    prof_mark(h, 0);
    // QKV: every row's head group g stored by the epilogue straight into rank g's Q and K/V (over
    // NVLink for g != r), at the row's place in the sequence; the all-to-all is the GEMM's stores
    GemmEpi eq;
    eq.seg_in = n_loc;
    eq.width = W;
    eq.norm_q = h->norm_q + il * c.head_dim;
    eq.norm_k = h->norm_k + il * c.head_dim;
    eq.rope = b.rope;
    eq.group_w = Wg;
    for (int g = 0; g < G; ++g) {
      eq.sp_q[g] = reinterpret_cast<bf16*>(b.peer_mem[g] + b.off_qf);
      eq.sp_k[g] = b.peer_kv[g] + kl_off;
      eq.sp_v[g] = b.peer_kv[g] + kl_off + size_t(b.kv_l) * Wg;
    }
    eq.sp_rank = r;
    eq.sp_pl = pl;
    eq.sp_pl_loc = pl_loc;
    eq.sp_nl = Nl;
    eq.sp_img0 = img0;
    eq.sp_p = P;
    if ((rc = gemm(h, h->y, W, h->w_qkv + static_cast<size_t>(il) * 3 * W * W, W, n_loc, 3 * W, W, EPI_QKV, eq)))
      return rc;
    prof_mark(h, 4);
    if ((rc = sp_flag_barrier(h))) return rc;
    prof_mark(h, 1);
    AttnArgs aa;
    aa.q = b.qf;
    aa.k = b.kv + kl_off;
    aa.v = b.kv + kl_off + size_t(b.kv_l) * Wg;
    aa.out = b.att_in;
    aa.nq = n_tot;
    aa.q0 = q0;
    aa.p = P;
    aa.l = L;
    aa.b0 = in.nref ? in.a : 0;
    aa.b1 = in.nref ? in.a + in.nref : 0;
    aa.heads = heads / G;
    aa.width = Wg;
    aa.kv_rows = b.kv_l;
    aa.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(c.head_dim)));
    aa.sms = h->att_sms ? h->att_sms : h->sms;
    aa.split_mode = h->att_mode;
    // each output row stored into the rank that keeps it, at this rank's head columns
    for (int g = 0; g < G; ++g) aa.sp_out[g] = reinterpret_cast<bf16*>(b.peer_mem[g] + b.off_att);
    aa.sp_ld = W;
    aa.sp_col0 = r * Wg;
    aa.sp_pl = pl;
    aa.sp_pl_loc = pl_loc;
    aa.sp_nl = Nl;
    aa.sp_img0 = img0;
    if ((rc = attention_launch(aa, h->d_status, h->st))) return fail(h, EXN_ECUDA, "attention launch failed: %d", rc);
    prof_mark(h, 4);
    if ((rc = sp_flag_barrier(h))) return rc;
    prof_mark(h, 0);
    GemmEpi eo;
    eo.out = h->x;
    eo.ld_out = W;
    eo.seg_in = n_loc;
    eo.mod = h->modv + 1 * W;
    eo.mod_stride = 4 * W;
    eo.n0 = 0;
    eo.p = pl_loc;
    if ((rc = gemm(h, b.att_in, W, h->w_out + static_cast<size_t>(il) * W * W, W, n_loc, W, W, EPI_GATE_RESID, eo)))
      return rc;
    prof_mark(h, 2);
    ln_mod_launch(h->x, h->y, h->modv + 2 * W, 4 * W, n_loc, W, n_loc, n_loc, 0, 0, pl_loc, 0, h->st);
    prof_mark(h, 3);
    GemmEpi eg;
    eg.out = h->ff;
    eg.ld_out = c.ffn;
    if ((rc = gemm(h, h->y, W, h->w_gu + static_cast<size_t>(il) * 2 * c.ffn * W, W, n_loc, 2 * c.ffn, W, EPI_SWIGLU,
                   eg)))
      return rc;
    prof_mark(h, 0);
    GemmEpi ed = eo;
    ed.mod = h->modv + 3 * W;
    if ((rc = gemm(h, h->ff, c.ffn, h->w_down + static_cast<size_t>(il) * W * c.ffn, c.ffn, n_loc, W, c.ffn,
                   EPI_GATE_RESID, ed)))
      return rc;
  }
  // this rank's image rows: LayerNorm * (1 + sc), proj_out into its latent columns
  prof_mark(h, 2);
  ln_mod_launch(h->x, h->y, h->sc, 0, Nl, W, Nl, n_loc, pl_loc, 0, 0, 1, h->st);
  prof_mark(h, 0);
  GemmEpi ep;
  ep.z = in.z ? in.z + size_t(r) * Nl : nullptr;
  ep.vout = in.v ? in.v + size_t(r) * Nl : nullptr;
  ep.dsigma = in.dsigma;
  ep.nimg = Nl;
  ep.zstride = N;
  if ((rc = gemm(h, h->y, W, h->w_proj, W, Nl, c.latent, W, EPI_PROJ, ep))) return rc;
  prof_mark(h, 2);
  CK(cudaGetLastError());
  return EXN_OK;
}

// every rank's latent columns [s N/G, (s+1) N/G) of Z (64 x N) gathered into every rank's Z
int sp_gather_columns(exn_handle* h, float* z, int N) {
  const int G = h->world, r = h->rank, Nl = N / G;
  SpBufs& b = h->sp;
  CK(cudaMemcpy2DAsync(b.zslice, size_t(Nl) * 4, z + size_t(r) * Nl, size_t(N) * 4, size_t(Nl) * 4, 64,
                       cudaMemcpyDeviceToDevice, h->st));
  ncclResult_t nr = nccl().AllGather(b.zslice, b.zall, size_t(64) * Nl, ncclFloat32, h->comm, h->st);
  if (nr != ncclSuccess && nr != ncclInProgress) return nccl_fail(h, nr, "all-gather of the latent");
  int rc;
  if ((rc = nccl_settle(h, h->comm, "all-gather of the latent"))) return rc;
  for (int s = 0; s < G; ++s)
    CK(cudaMemcpy2DAsync(z + size_t(s) * Nl, size_t(N) * 4, b.zall + size_t(s) * 64 * Nl, size_t(Nl) * 4,
                         size_t(Nl) * 4, 64, cudaMemcpyDeviceToDevice, h->st));
  return EXN_OK;
}

int run_pass(exn_handle* h, const StepIn& in) {
  return (h->comm && h->world > 1) ? run_step_sp(h, in) : run_step(h, in);
}

int check_status(exn_handle* h) {
  if (h->comm) {  // a peer that stopped answering must not hang this rank: poll with a deadline
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
      const cudaError_t q = cudaStreamQuery(h->st);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) CK(q);
      ncclResult_t st = ncclSuccess;
      nccl().CommGetAsyncError(h->comm, &st);
      if (st != ncclSuccess && st != ncclInProgress) {
        nccl().CommAbort(h->comm);
        h->comm = nullptr;
        return nccl_fail(h, st, "communicator failed");
      }
      if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > h->comm_timeout_s) {
        nccl().CommAbort(h->comm);
        h->comm = nullptr;
        return fail(h, EXN_ETIMEOUT, "no progress in %.0f s; communicator aborted", h->comm_timeout_s);
      }
      std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
  }
  CK(cudaStreamSynchronize(h->st));
  int s = 0;
  CK(cudaMemcpy(&s, h->d_status, sizeof s, cudaMemcpyDeviceToHost));
  if (s) {
    cudaMemset(h->d_status, 0, sizeof(int));
    return fail(h, EXN_ETIMEOUT, "a kernel gave up waiting on its pipeline (status 0x%x)", s);
  }
  prof_collect(h);
  return EXN_OK;
}

int check_step_args(exn_handle* h, int batch, int p, int hh, int ww, const exn_ref* ref) {
  if (batch < 1) return fail(h, EXN_EINVAL, "batch %d", batch);
  if (p < 0 || hh < 1 || ww < 1) return fail(h, EXN_EINVAL, "p %d, h %d, w %d", p, hh, ww);
  if (ref && (ref->a < 0 || ref->a > p || ref->rh < 1 || ref->rw < 1 || !ref->latent))
    return fail(h, EXN_EINVAL, "bad reference picture (a %d, %d x %d)", ref ? ref->a : 0, ref ? ref->rh : 0,
                ref ? ref->rw : 0);
  if (h->n_loaded != h->spec.size())
    return fail(h, EXN_ENOWEIGHTS, "%zu of %zu tensors loaded", h->n_loaded, h->spec.size());
  return EXN_OK;
}

// upload host inputs for a batch-1 call
int upload_inputs(exn_handle* h, const float* context, int p, const float* latent, int hh, int ww, const exn_ref* ref,
                  bool need_ctx) {
  const exn_config& c = h->cfg;
  const int nimg = hh * ww, nref = ref ? ref->rh * ref->rw : 0;
  int rc;
  if ((rc = ensure_buffers(h, 1, (p + nref + nimg), p + nref + nimg, p, nimg, nref, h->comm == nullptr))) return rc;
  if (need_ctx && p) CK(cudaMemcpyAsync(h->ctx_dev, context, size_t(p) * c.context * 4, cudaMemcpyHostToDevice, h->st));
  if (need_ctx && nref)
    CK(cudaMemcpyAsync(h->ref_dev, ref->latent, size_t(nref) * c.latent * 4, cudaMemcpyHostToDevice, h->st));
  if (latent) CK(cudaMemcpyAsync(h->lat_dev, latent, size_t(nimg) * c.latent * 4, cudaMemcpyHostToDevice, h->st));
  return EXN_OK;
}

// Events on the handle's stream around the device part of a host-buffer call (I = 0 after the
// inputs' upload, 1 before the result's download).
int mark_call(exn_handle* h, int i) {
  if (!h->call_ev[i]) CK(cudaEventCreate(&h->call_ev[i]));
  CK(cudaEventRecord(h->call_ev[i], h->st));
  return EXN_OK;
}

// After the call's stream has drained: the device time between the two marks.
void read_call_time(exn_handle* h) {
  float ms = 0.f;
  h->last_call_ms = cudaEventElapsedTime(&ms, h->call_ev[0], h->call_ev[1]) == cudaSuccess ? ms : 0.0;
}

}  // namespace

// ============================================================================ C ABI

extern "C" {

int exn_abi_version(void) { return EXN_ABI_VERSION; }

void exn_default_config(exn_config* cfg) {
  if (!cfg) return;
  cfg->width = 4096;
  cfg->layers = 32;
  cfg->ffn = 12288;
  cfg->latent = 64;
  cfg->context = 4096;
  cfg->freq = 256;
  cfg->head_dim = 128;
  cfg->device = 0;
}

int exn_open(const exn_config* cfg, exn_handle** out) {
  exn_handle* h = nullptr;
  if (!out) return fail(nullptr, EXN_EINVAL, "exn_open: null handle pointer");
  *out = nullptr;
  if (!cfg) return fail(nullptr, EXN_EINVAL, "exn_open: null config");
  const exn_config& c = *cfg;
  if (c.head_dim != 128 || c.width <= 0 || c.width % 256 || c.ffn <= 0 || c.ffn % 128 || c.layers <= 0 ||
      c.latent != 64 || c.context <= 0 || c.context % 64 || c.context > 4096 || c.width > 4096 || c.freq <= 0 ||
      c.freq % 64 || c.freq > 4096)
    return fail(nullptr, EXN_EINVAL,
                "exn_open: unsupported shape (width %d, ffn %d, layers %d, latent %d, context %d, freq %d, head_dim %d)",
                c.width, c.ffn, c.layers, c.latent, c.context, c.freq, c.head_dim);
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || c.device < 0 || c.device >= ndev)
    return fail(nullptr, EXN_ECUDA, "exn_open: no CUDA device %d", c.device);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, c.device) != cudaSuccess)
    return fail(nullptr, EXN_ECUDA, "exn_open: cannot query device %d", c.device);
  if (prop.major != 10)
    return fail(nullptr, EXN_EUNSUPPORTED, "exn_open: device %d is sm_%d%d; this library is built for sm_100a",
                c.device, prop.major, prop.minor);
  h = new exn_handle();
  h->cfg = c;
  h->sms = prop.multiProcessorCount;
  int rc;
  if ((rc = use_device(h)) || (rc = [&]() -> int {
        CK(cudaStreamCreateWithFlags(&h->st, cudaStreamNonBlocking));
        CK(cudaMalloc(&h->d_status, sizeof(int)));
        CK(cudaMemset(h->d_status, 0, sizeof(int)));
        // the kernels' shared-memory limits are attributes of this device's context
        CK(static_cast<cudaError_t>(gemm_prepare()));
        CK(static_cast<cudaError_t>(attention_prepare()));
        CK(static_cast<cudaError_t>(gemm_q8_prepare()));
        return EXN_OK;
      }()) ||
      (rc = alloc_weights(h))) {
    g_open_error = h->err;
    exn_close(h);
    return rc;
  }
  h->spec = expected_tensors(c);
  for (size_t i = 0; i < h->spec.size(); ++i) h->index[h->spec[i].name] = static_cast<int>(i);
  h->loaded.assign(h->spec.size(), 0);
  h->prof.on = std::getenv("EXN_PROFILE") != nullptr;
  if (const char* e = std::getenv("EXN_GEMM_PAIRS")) h->gemm_pairs = std::atoi(e);
  if (const char* e = std::getenv("EXN_ATT_SINGLE")) h->att_mode = std::atoi(e) == 1 ? 1 : (std::atoi(e) == 0 ? 0 : 2);
  *out = h;
  return EXN_OK;
}

void exn_close(exn_handle* h) {
  if (!h) return;
  cudaSetDevice(h->cfg.device);
  if (h->st) cudaStreamSynchronize(h->st);
  free_buffers(h);
  free_sp(h);
  if (h->comm) nccl().CommDestroy(h->comm);
  for (void* p : h->extra_allocs) cudaFree(p);
  if (h->slab) cudaFree(h->slab);
  if (h->d_status) cudaFree(h->d_status);
  for (auto& m : h->prof.marks) cudaEventDestroy(m.first);
  for (cudaEvent_t e : h->call_ev)
    if (e) cudaEventDestroy(e);
  if (h->st) cudaStreamDestroy(h->st);
  delete h;
}

const char* exn_last_error(const exn_handle* h) { return h ? h->err.c_str() : g_open_error.c_str(); }

static int check_gguf(const exn_config& cfg, const std::vector<TensorSpec>& spec, const GgufFile& g,
                      const char* path, std::string& msg) {
  std::vector<std::string> problems;
  if (g.arch != "qwen_image") problems.push_back("architecture \"" + g.arch + "\", not \"qwen_image\"");
  std::map<std::string, const GgufTensor*> byname;
  for (const auto& t : g.tensors) byname[t.name] = &t;
  for (const auto& s : spec) {
    auto it = byname.find(kPrefix + s.name);
    if (it == byname.end())
      problems.push_back("missing " + s.name);
    else if (it->second->dims != s.dims)
      problems.push_back(s.name + " is " + dims_str(it->second->dims) + ", not " + dims_str(s.dims));
  }
  const long extra = static_cast<long>(g.tensors.size()) - static_cast<long>(spec.size());
  if (extra != 0) problems.push_back(std::to_string(extra) + " tensors more than the model has");
  if (problems.empty()) return EXN_OK;
  msg = std::string(path) + ":";
  for (const auto& p : problems) msg += "\n  " + p;
  (void)cfg;
  return EXN_ESHAPE;
}

int exn_check_gguf(const exn_config* cfg, const char* path, char* msg, size_t msg_len) {
  std::string m;
  int rc = EXN_OK;
  if (!cfg || !path) {
    m = "exn_check_gguf: null argument";
    rc = EXN_EINVAL;
  } else {
    GgufFile g;
    if (!g.open(path, m))
      rc = EXN_EIO;
    else
      rc = check_gguf(*cfg, expected_tensors(*cfg), g, path, m);
  }
  if (msg && msg_len) {
    std::strncpy(msg, m.c_str(), msg_len - 1);
    msg[msg_len - 1] = 0;
  }
  return rc;
}

int exn_load_gguf(exn_handle* h, const char* path) {
  if (!h || !path) return fail(h, EXN_EINVAL, "exn_load_gguf: null argument");
  int rc;
  if ((rc = use_device(h))) return rc;
  GgufFile g;
  std::string err;
  if (!g.open(path, err)) return fail(h, EXN_EIO, "%s", err.c_str());
  // open-dit: architecture, every expected tensor's presence and dims, nothing extra
  if ((rc = check_gguf(h->cfg, h->spec, g, path, err))) return fail(h, rc, "%s", err.c_str());
  // upload: a pinned staging buffer, the raw bytes to the device, converted in place
  size_t maxb = 0;
  for (const auto& t : g.tensors) {
    if (!t.nbytes) return fail(h, EXN_EUNSUPPORTED, "%s: ggml type %d not handled", t.name.c_str(), t.type);
    maxb = std::max(maxb, t.nbytes);
  }
  void* raw = nullptr;
  void* scratch = nullptr;
  void* pinned = nullptr;
  const size_t chunk = 64ull << 20;
  CK(cudaMalloc(&raw, maxb));
  if (cudaMalloc(&scratch, maxb * 2) != cudaSuccess || cudaMallocHost(&pinned, 2 * chunk) != cudaSuccess) {
    cudaFree(raw);
    if (scratch) cudaFree(scratch);
    return fail(h, EXN_ENOMEM, "exn_load_gguf: staging buffers");
  }
  cudaEvent_t ev[2];
  cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming);
  cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming);
  rc = EXN_OK;
  int slot = 0;
  for (const auto& t : g.tensors) {
    int idx = -1;
    if ((rc = check_tensor(h, t.name.substr(strlen(kPrefix)), t.type, t.dims, &idx))) break;
    const uint8_t* src = g.data(t);
    for (size_t o = 0; o < t.nbytes && rc == EXN_OK; o += chunk) {
      const size_t nb = std::min(chunk, t.nbytes - o);
      char* pb = static_cast<char*>(pinned) + slot * chunk;
      cudaEventSynchronize(ev[slot]);
      std::memcpy(pb, src + o, nb);
      if (cudaMemcpyAsync(static_cast<char*>(raw) + o, pb, nb, cudaMemcpyHostToDevice, h->st) != cudaSuccess)
        rc = fail(h, EXN_ECUDA, "upload of %s failed", t.name.c_str());
      cudaEventRecord(ev[slot], h->st);
      slot ^= 1;
    }
    if (rc) break;
    if ((rc = place(h, idx, t.type, raw, scratch))) break;
  }
  cudaStreamSynchronize(h->st);
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  cudaFreeHost(pinned);
  cudaFree(scratch);
  cudaFree(raw);
  if (rc) return rc;
  CK(cudaGetLastError());
  return EXN_OK;
}

int exn_load_tensor(exn_handle* h, const char* name, int ggml_type, int n_dims, const int64_t* dims, const void* data,
                    size_t nbytes) {
  if (!h || !name || !dims || !data || n_dims < 1 || n_dims > 4) return fail(h, EXN_EINVAL, "exn_load_tensor: bad argument");
  int rc;
  if ((rc = use_device(h))) return rc;
  std::vector<int64_t> d(dims, dims + n_dims);
  int idx = -1;
  if ((rc = check_tensor(h, name, ggml_type, d, &idx))) return rc;
  const size_t need = ggml_nbytes(ggml_type, d);
  if (need != nbytes) return fail(h, EXN_EINVAL, "%s: %zu bytes, expected %zu", name, nbytes, need);
  void* raw = nullptr;
  void* scratch = nullptr;
  CK(cudaMalloc(&raw, nbytes));
  if (cudaMalloc(&scratch, nbytes * 2 + 256) != cudaSuccess) {
    cudaFree(raw);
    return fail(h, EXN_ENOMEM, "exn_load_tensor: scratch");
  }
  rc = EXN_OK;
  if (cudaMemcpyAsync(raw, data, nbytes, cudaMemcpyHostToDevice, h->st) != cudaSuccess)
    rc = fail(h, EXN_ECUDA, "exn_load_tensor: upload failed");
  if (!rc) rc = place(h, idx, ggml_type, raw, scratch);
  cudaStreamSynchronize(h->st);
  cudaFree(raw);
  cudaFree(scratch);
  return rc;
}

int exn_load_synthetic(exn_handle* h, uint64_t seed) {
  if (!h) return fail(h, EXN_EINVAL, "exn_load_synthetic: null handle");
  int rc;
  if ((rc = use_device(h))) return rc;
  const double ih_std = std::sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0);
  const double std_dev = 0.02 * std::sqrt(4096.0 / h->cfg.width);
  const float scale = static_cast<float>(std_dev / ih_std);
  size_t maxn = 0;
  for (const auto& s : h->spec) {
    size_t n = 1;
    for (auto d : s.dims) n *= d;
    maxn = std::max(maxn, n);
  }
  int8_t* qs = nullptr;
  __half* d = nullptr;
  float* f = nullptr;
  CK(cudaMalloc(&qs, maxn));
  CK(cudaMalloc(&d, maxn / 32 * 2 + 256));
  CK(cudaMalloc(&f, maxn * 4));
  rc = EXN_OK;
  for (size_t i = 0; i < h->spec.size() && !rc; ++i) {
    const TensorSpec& s = h->spec[i];
    const long long cols = s.dims[0], rows = s.dims.size() > 1 ? s.dims[1] : 1, n = rows * cols;
    if (s.dims.size() == 1) {
      const bool tn = s.name == "txt_in.text_norm.weight";
      synth_f32_launch(f, n, seed, static_cast<uint32_t>(i), scale, tn ? 0.f : 1.f, h->st);
      rc = place(h, static_cast<int>(i), GGML_F32, f, nullptr);
    } else {
      synth_q8_launch(qs, d, n, seed, static_cast<uint32_t>(i), scale, h->st);
      Route r = route(h, s.name);
      if (r.gemv) {
        void* wq = nullptr;
        void* wd = nullptr;
        if (cudaMalloc(&wq, n) != cudaSuccess || cudaMalloc(&wd, n / 32 * 2) != cudaSuccess) {
          rc = fail(h, EXN_ENOMEM, "exn_load_synthetic: %s", s.name.c_str());
          break;
        }
        h->extra_allocs.push_back(wq);
        h->extra_allocs.push_back(wd);
        cudaMemcpyAsync(wq, qs, n, cudaMemcpyDeviceToDevice, h->st);
        cudaMemcpyAsync(wd, d, n / 32 * 2, cudaMemcpyDeviceToDevice, h->st);
        r.gemv->kind = W_Q8;
        r.gemv->w = wq;
        r.gemv->d = static_cast<__half*>(wd);
      } else {
        q8_to_bf16_launch(qs, d, r.dst, rows, static_cast<int>(cols), r.row0, r.ilv, h->st);
      }
      if (!h->loaded[i]) {
        h->loaded[i] = 1;
        ++h->n_loaded;
      }
    }
    if (cudaGetLastError() != cudaSuccess) rc = fail(h, EXN_ECUDA, "exn_load_synthetic: %s", s.name.c_str());
  }
  cudaStreamSynchronize(h->st);
  cudaFree(qs);
  cudaFree(d);
  cudaFree(f);
  return rc;
}

int exn_weights_ready(const exn_handle* h) {
  if (!h) return EXN_EINVAL;
  return h->n_loaded == h->spec.size() ? EXN_OK : EXN_ENOWEIGHTS;
}

int exn_velocity(exn_handle* h, const float* context, int p, const float* latent, int hh, int ww, double sigma,
                 uint64_t prefix_key, const exn_ref* ref, float* v_out) {
  if (!h || !latent || !v_out || (p > 0 && !context)) return fail(h, EXN_EINVAL, "exn_velocity: null argument");
  int rc;
  if ((rc = use_device(h)) || (rc = check_step_args(h, 1, p, hh, ww, ref))) return rc;
  const int nref = ref ? ref->rh * ref->rw : 0, pfx = p + nref;
  const bool cached = prefix_key && h->prefix_valid && prefix_key == h->prefix_key && pfx == h->prefix_len &&
                      (h->comm ? true : h->kv_batch == 1);
  if ((rc = upload_inputs(h, context, p, latent, hh, ww, ref, !cached)) || (rc = mark_call(h, 0))) return rc;
  if (!cached) {
    h->prefix_valid = false;
    h->prefix_key = 0;
  }
  StepIn in;
  in.ptext = p;
  in.nref = nref;
  in.a = ref ? ref->a : 0;
  in.rh = ref ? ref->rh : 0;
  in.rw = ref ? ref->rw : 0;
  in.hh = hh;
  in.ww = ww;
  in.sigma = sigma;
  in.cached = cached;
  in.ctx = h->ctx_dev;
  in.ref = h->ref_dev;
  in.lat = h->lat_dev;
  in.v = h->vout;
  if ((rc = run_pass(h, in))) return rc;
  if (h->comm && h->world > 1 && (rc = sp_gather_columns(h, h->vout, hh * ww))) return rc;
  if ((rc = mark_call(h, 1))) return rc;
  CK(cudaMemcpyAsync(v_out, h->vout, size_t(hh) * ww * h->cfg.latent * 4, cudaMemcpyDeviceToHost, h->st));
  if ((rc = check_status(h))) return rc;
  read_call_time(h);
  if (prefix_key && !cached) {
    h->prefix_key = prefix_key;
    h->prefix_len = pfx;
    h->prefix_valid = true;
  }
  return EXN_OK;
}

int exn_generate(exn_handle* h, const float* context, int p, float* z, int hh, int ww, const double* sigmas, int nsig,
                 uint64_t prefix_key, const exn_ref* ref) {
  if (!h || !z || !sigmas || (p > 0 && !context)) return fail(h, EXN_EINVAL, "exn_generate: null argument");
  if (nsig < 2) return fail(h, EXN_EINVAL, "exn_generate: %d sigmas", nsig);
  int rc;
  if ((rc = use_device(h)) || (rc = check_step_args(h, 1, p, hh, ww, ref))) return rc;
  const int nref = ref ? ref->rh * ref->rw : 0, pfx = p + nref;
  bool cached = prefix_key && h->prefix_valid && prefix_key == h->prefix_key && pfx == h->prefix_len &&
                (h->comm ? true : h->kv_batch == 1);
  if ((rc = upload_inputs(h, context, p, z, hh, ww, ref, true)) || (rc = mark_call(h, 0))) return rc;
  for (int s = 0; s + 1 < nsig; ++s) {
    if (!cached) {
      h->prefix_valid = false;
      h->prefix_key = 0;
    }
    StepIn in;
    in.ptext = p;
    in.nref = nref;
    in.a = ref ? ref->a : 0;
    in.rh = ref ? ref->rh : 0;
    in.rw = ref ? ref->rw : 0;
    in.hh = hh;
    in.ww = ww;
    in.sigma = sigmas[s];
    in.cached = cached;
    in.ctx = h->ctx_dev;
    in.ref = h->ref_dev;
    in.lat = h->lat_dev;
    in.z = h->lat_dev;
    in.dsigma = static_cast<float>(sigmas[s + 1] - sigmas[s]);
    if ((rc = run_pass(h, in))) return rc;
    if (!cached && prefix_key) {
      h->prefix_key = prefix_key;
      h->prefix_len = pfx;
      h->prefix_valid = true;
      cached = true;
    }
  }
  if (h->comm && h->world > 1 && (rc = sp_gather_columns(h, h->lat_dev, hh * ww))) return rc;
  if ((rc = mark_call(h, 1))) return rc;
  CK(cudaMemcpyAsync(z, h->lat_dev, size_t(hh) * ww * h->cfg.latent * 4, cudaMemcpyDeviceToHost, h->st));
  if ((rc = check_status(h))) {
    h->prefix_valid = false;
    h->prefix_key = 0;
    return rc;
  }
  read_call_time(h);
  return EXN_OK;
}

static int generate_dev(exn_handle* h, int batch, const float* d_ctx, int p, float* d_z, int hh, int ww,
                        const double* sigmas, int nsig) {
  int rc;
  if (h->comm) return fail(h, EXN_EINVAL, "batched pictures run one per handle; this handle shares its rows over %d GPUs",
                           h->world);
  h->prefix_valid = false;
  h->prefix_key = 0;
  for (int s = 0; s + 1 < nsig; ++s) {
    StepIn in;
    in.batch = batch;
    in.ptext = p;
    in.hh = hh;
    in.ww = ww;
    in.sigma = sigmas[s];
    in.cached = s > 0;
    in.ctx = d_ctx;
    in.lat = d_z;
    in.z = d_z;
    in.dsigma = static_cast<float>(sigmas[s + 1] - sigmas[s]);
    if ((rc = run_step(h, in))) return rc;
  }
  return EXN_OK;
}

int exn_generate_batch(exn_handle* h, int batch, const float* contexts, int p, float* z, int hh, int ww,
                       const double* sigmas, int nsig) {
  if (!h || !z || !sigmas || (p > 0 && !contexts)) return fail(h, EXN_EINVAL, "exn_generate_batch: null argument");
  if (nsig < 2) return fail(h, EXN_EINVAL, "exn_generate_batch: %d sigmas", nsig);
  int rc;
  if ((rc = use_device(h)) || (rc = check_step_args(h, batch, p, hh, ww, nullptr))) return rc;
  const exn_config& c = h->cfg;
  const int nimg = hh * ww;
  if ((rc = ensure_buffers(h, batch, p + nimg, p + nimg, p, nimg, 0))) return rc;
  CK(cudaMemcpyAsync(h->ctx_dev, contexts, size_t(batch) * p * c.context * 4, cudaMemcpyHostToDevice, h->st));
  CK(cudaMemcpyAsync(h->lat_dev, z, size_t(batch) * nimg * c.latent * 4, cudaMemcpyHostToDevice, h->st));
  if ((rc = generate_dev(h, batch, h->ctx_dev, p, h->lat_dev, hh, ww, sigmas, nsig))) return rc;
  CK(cudaMemcpyAsync(z, h->lat_dev, size_t(batch) * nimg * c.latent * 4, cudaMemcpyDeviceToHost, h->st));
  return check_status(h);
}

int exn_generate_device(exn_handle* h, int batch, const float* d_contexts, int p, float* d_z, int hh, int ww,
                        const double* sigmas, int nsig, void* stream) {
  if (!h || !d_z || !sigmas || (p > 0 && !d_contexts)) return fail(h, EXN_EINVAL, "exn_generate_device: null argument");
  if (nsig < 2) return fail(h, EXN_EINVAL, "exn_generate_device: %d sigmas", nsig);
  int rc;
  if ((rc = use_device(h)) || (rc = check_step_args(h, batch, p, hh, ww, nullptr))) return rc;
  const int nimg = hh * ww;
  if ((rc = ensure_buffers(h, batch, p + nimg, p + nimg, p, nimg, 0))) return rc;
  // ordered after the caller's stream (NULL is CUDA's default stream), and the caller's stream after the work
  cudaStream_t user = static_cast<cudaStream_t>(stream);
  cudaEvent_t e;
  CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  CK(cudaEventRecord(e, user));
  CK(cudaStreamWaitEvent(h->st, e, 0));
  cudaEventDestroy(e);
  if ((rc = generate_dev(h, batch, d_contexts, p, d_z, hh, ww, sigmas, nsig))) return rc;
  CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  CK(cudaEventRecord(e, h->st));
  CK(cudaStreamWaitEvent(user, e, 0));
  cudaEventDestroy(e);
  return EXN_OK;
}

int exn_sync(exn_handle* h) {
  if (!h) return fail(h, EXN_EINVAL, "exn_sync: null handle");
  int rc;
  if ((rc = use_device(h))) return rc;
  return check_status(h);
}

int exn_release(exn_handle* h) {
  if (!h) return fail(h, EXN_EINVAL, "exn_release: null handle");
  int rc;
  if ((rc = use_device(h))) return rc;
  CK(cudaStreamSynchronize(h->st));
  free_buffers(h);
  free_sp(h);
  return EXN_OK;
}

int exn_comm_unique_id(void* id) {
  if (!id) return fail(nullptr, EXN_EINVAL, "exn_comm_unique_id: null buffer");
  NcclApi& nc = nccl();
  if (!nc.ok) return fail(nullptr, EXN_EUNSUPPORTED, "NCCL: %s", nc.why.c_str());
  ncclUniqueId u;
  const ncclResult_t r = nc.GetUniqueId(&u);
  if (r != ncclSuccess) return fail(nullptr, EXN_ECUDA, "ncclGetUniqueId: %s", nc.GetErrorString(r));
  std::memcpy(id, &u, sizeof u);
  return EXN_OK;
}

int exn_comm_init(exn_handle* h, const void* id, int rank, int world) {
  if (!h || !id || world < 1 || rank < 0 || rank >= world) return fail(h, EXN_EINVAL, "exn_comm_init: bad argument");
  int rc;
  if ((rc = use_device(h))) return rc;
  NcclApi& nc = nccl();
  if (!nc.ok) return fail(h, EXN_EUNSUPPORTED, "NCCL: %s", nc.why.c_str());
  if (h->comm) return fail(h, EXN_EINVAL, "exn_comm_init: the handle already has a communicator");
  if (const char* t = std::getenv("EXN_COMM_TIMEOUT_S")) h->comm_timeout_s = std::max(1.0, std::atof(t));
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof u);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // every wait on it is bounded (nccl_settle, check_status)
  ncclComm_t comm = nullptr;
  const ncclResult_t r = nc.CommInitRankConfig(&comm, world, u, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) return fail(h, EXN_ECUDA, "ncclCommInitRankConfig: %s", nc.GetErrorString(r));
  if ((rc = nccl_settle(h, comm, "communicator init"))) return rc;
  h->comm = comm;
  h->rank = rank;
  h->world = world;
  h->prefix_valid = false;  // the kept prompt K/V now live per head shard
  h->prefix_key = 0;
  return EXN_OK;
}

int exn_comm_destroy(exn_handle* h) {
  if (!h) return fail(h, EXN_EINVAL, "exn_comm_destroy: null handle");
  int rc;
  if ((rc = use_device(h))) return rc;
  CK(cudaStreamSynchronize(h->st));
  if (h->comm) nccl().CommDestroy(h->comm);
  h->comm = nullptr;
  h->rank = 0;
  h->world = 1;
  free_sp(h);
  h->prefix_valid = false;
  h->prefix_key = 0;
  return EXN_OK;
}

// ---------------------------------------------------------------------------- testing entry points

int exn_test_gemm(exn_handle* h, const void* a, const void* b, float* c, int m, int n, int k) {
  if (!h || !a || !b || !c) return fail(h, EXN_EINVAL, "exn_test_gemm: null argument");
  int rc;
  if ((rc = use_device(h))) return rc;
  GemmEpi e;
  e.out = c;
  e.ld_out = n;
  if ((rc = gemm(h, static_cast<const bf16*>(a), k, static_cast<const bf16*>(b), k, m, n, k, EPI_F32, e))) return rc;
  return check_status(h);
}

int exn_test_attention(exn_handle* h, const void* q, const void* k, const void* v, void* out, int batch, int nq,
                       int q0, int p, int l, int b0, int b1, int heads, int kv_rows) {
  if (!h || !q || !k || !v || !out) return fail(h, EXN_EINVAL, "exn_test_attention: null argument");
  int rc;
  if ((rc = use_device(h))) return rc;
  AttnArgs aa;
  aa.q = static_cast<const bf16*>(q);
  aa.k = static_cast<const bf16*>(k);
  aa.v = static_cast<const bf16*>(v);
  aa.out = static_cast<bf16*>(out);
  aa.batch = batch;
  aa.nq = nq;
  aa.q0 = q0;
  aa.p = p;
  aa.l = l;
  aa.b0 = b0;
  aa.b1 = b1;
  aa.heads = heads;
  aa.width = heads * 128;
  aa.kv_rows = kv_rows;
  aa.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(128.0));
  aa.sms = h->att_sms ? h->att_sms : h->sms;
  aa.split_mode = h->att_mode;
  if ((rc = attention_launch(aa, h->d_status, h->st))) return fail(h, EXN_EINVAL, "attention launch failed: %d", rc);
  return check_status(h);
}

int exn_test_gemv(exn_handle* h, int kind, const void* w, const void* d, const float* x, float* y, int m, int in,
                  int out, int act, int piece, int reps, double* ms) {
  if (!h || !w || !x || !y || (kind == W_Q8 && !d) || kind < W_Q8 || kind > W_F32 || reps < 1 || !ms)
    return fail(h, EXN_EINVAL, "exn_test_gemv: bad argument");
  if (m < 1 || m > 2 || in <= 0 || out <= 0 || (act == 2 && piece <= 0))
    return fail(h, EXN_EINVAL, "exn_test_gemv: bad shape");
  int rc;
  if ((rc = use_device(h))) return rc;
  cudaEvent_t ev[2];
  CK(cudaEventCreate(&ev[0]));
  CK(cudaEventCreate(&ev[1]));
  CK(cudaEventRecord(ev[0], h->st));
  for (int i = 0; i < reps && !rc; ++i)
    if (gemv_launch(kind, w, static_cast<const __half*>(d), x, y, m, in, out, act, piece, h->st))
      rc = fail(h, EXN_EINVAL, "exn_test_gemv: launch failed (shape out of the kernel's range)");
  CK(cudaEventRecord(ev[1], h->st));
  if (!rc) rc = check_status(h);
  if (!rc) {
    float t = 0.f;
    cudaEventElapsedTime(&t, ev[0], ev[1]);
    *ms = t / reps;
  }
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  return rc;
}

int exn_test_attention_timed(exn_handle* h, const void* q, const void* k, const void* v, void* out, int batch, int nq,
                             int q0, int p, int l, int b0, int b1, int heads, int kv_rows, int reps, double* ms) {
  if (!h || !q || !k || !v || !out || reps < 1 || !ms) return fail(h, EXN_EINVAL, "exn_test_attention_timed: bad argument");
  int rc;
  if ((rc = use_device(h))) return rc;
  AttnArgs aa;
  aa.q = static_cast<const bf16*>(q);
  aa.k = static_cast<const bf16*>(k);
  aa.v = static_cast<const bf16*>(v);
  aa.out = static_cast<bf16*>(out);
  aa.batch = batch;
  aa.nq = nq;
  aa.q0 = q0;
  aa.p = p;
  aa.l = l;
  aa.b0 = b0;
  aa.b1 = b1;
  aa.heads = heads;
  aa.width = heads * 128;
  aa.kv_rows = kv_rows;
  aa.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(128.0));
  aa.sms = h->att_sms ? h->att_sms : h->sms;
  aa.split_mode = h->att_mode;
  cudaEvent_t ev[2];
  CK(cudaEventCreate(&ev[0]));
  CK(cudaEventCreate(&ev[1]));
  CK(cudaEventRecord(ev[0], h->st));
  for (int i = 0; i < reps && !rc; ++i)
    if (attention_launch(aa, h->d_status, h->st)) rc = fail(h, EXN_EINVAL, "attention launch failed");
  CK(cudaEventRecord(ev[1], h->st));
  if (!rc) rc = check_status(h);
  if (!rc) {
    float t = 0.f;
    cudaEventElapsedTime(&t, ev[0], ev[1]);
    *ms = t / reps;
  }
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  return rc;
}

int exn_test_comm_stats(exn_handle* h, long long* settles, long long* sleeps, double* seconds) {
  if (!h) return fail(h, EXN_EINVAL, "exn_test_comm_stats: null handle");
  if (settles) *settles = h->settles;
  if (sleeps) *sleeps = h->settle_sleeps;
  if (seconds) *seconds = h->settle_s;
  return EXN_OK;
}

int exn_test_gemm_pairs(exn_handle* h, int pairs) {
  if (!h) return fail(h, EXN_EINVAL, "exn_test_gemm_pairs: null handle");
  if (pairs < 0 || pairs > 2) return fail(h, EXN_EINVAL, "exn_test_gemm_pairs: mode %d", pairs);
  h->gemm_pairs = pairs;
  return EXN_OK;
}

int exn_test_attention_split(exn_handle* h, int mode, int sms) {
  if (!h) return fail(h, EXN_EINVAL, "exn_test_attention_split: null handle");
  if (mode < 0 || mode > 2 || sms < 0) return fail(h, EXN_EINVAL, "exn_test_attention_split: mode %d, sms %d", mode, sms);
  h->att_mode = mode;
  h->att_sms = sms;
  return EXN_OK;
}

int exn_test_ln_mod(exn_handle* h, const float* x, void* y, const float* mod, int n, int width, int n0, int p) {
  if (!h || !x || !y || !mod) return fail(h, EXN_EINVAL, "exn_test_ln_mod: null argument");
  if (width % 4 || width > 4096) return fail(h, EXN_EINVAL, "exn_test_ln_mod: width %d", width);
  int rc;
  if ((rc = use_device(h))) return rc;
  ln_mod_launch(x, static_cast<bf16*>(y), mod, width, n, width, n, n, 0, n0, p, 0, h->st);
  CK(cudaGetLastError());
  return check_status(h);
}

int exn_test_qkv(exn_handle* h, int layer, const void* y, void* q, void* k, void* v, int n, int n0, int p, int hh,
                 int ww, int kv_rows) {
  if (!h || !y || !q || !k || !v) return fail(h, EXN_EINVAL, "exn_test_qkv: null argument");
  if (layer < 0 || layer >= h->cfg.layers || n < 1 || n0 < 0 || p < 0 || hh < 1 || ww < 1 || n0 + n > kv_rows ||
      n0 + n > p + hh * ww)  // the rows' RoPE comes from the table of the p + hh x ww sequence rows
    return fail(h, EXN_EINVAL, "exn_test_qkv: bad sizes");
  int rc;
  if ((rc = use_device(h))) return rc;
  const int W = h->cfg.width, L = p + hh * ww;
  if ((rc = ensure_buffers(h, 1, 1, L, 1, 1, 0))) return rc;
  rope_table_launch(h->rope, 0, L, p, hh, ww, 0, 0, 0, h->st);
  GemmEpi eq;
  eq.seg_in = n;
  eq.n0 = n0;
  eq.width = W;
  eq.norm_q = h->norm_q + layer * 128;
  eq.norm_k = h->norm_k + layer * 128;
  eq.rope = h->rope;
  eq.q = static_cast<bf16*>(q);
  eq.k = static_cast<bf16*>(k);
  eq.v = static_cast<bf16*>(v);
  eq.kv_sample_stride = static_cast<long long>(kv_rows) * W;
  if ((rc = gemm(h, static_cast<const bf16*>(y), W, h->w_qkv + static_cast<size_t>(layer) * 3 * W * W, W, n, 3 * W, W,
                 EPI_QKV, eq)))
    return rc;
  return check_status(h);
}

int exn_qkv_noalloc(exn_handle* h, int layer, const void* y, void* q, void* k, void* v, int n, int n0, int p, int hh,
                    int ww, int kv_rows) {
  if (!h || !y || !q || !k || !v) return fail(h, EXN_EINVAL, "exn_qkv_noalloc: null argument");
  if (layer < 0 || layer >= h->cfg.layers || n < 1 || n0 < 0 || p < 0 || hh < 1 || ww < 1 || n0 + n > kv_rows ||
      n0 + n > p + hh * ww)
    return fail(h, EXN_EINVAL, "exn_qkv_noalloc: bad sizes");
  const int W = h->cfg.width, L = p + hh * ww;
  if (L > kNoAllocMaxRows)
    return fail(h, EXN_EINVAL,
                "exn_qkv_noalloc: a sequence of %d rows (p %d + %d x %d); its fixed RoPE scratch holds at most %d",
                L, p, hh, ww, kNoAllocMaxRows);
  int rc;
  if ((rc = use_device(h))) return rc;
  float2* rope = nullptr;
  if ((rc = noalloc_rope_scratch(h->cfg.device, &rope)))
    return fail(h, EXN_ECUDA, "exn_qkv_noalloc: address of the RoPE scratch on device %d: %s", h->cfg.device,
                rc > 0 ? cudaGetErrorString(static_cast<cudaError_t>(rc)) : "bad device");
  // every row the GEMM reads (0 .. L-1) is written here first, so the previous call's table needs no clearing
  rope_table_launch(rope, 0, L, p, hh, ww, 0, 0, 0, h->st);
  GemmEpi eq;
  eq.seg_in = n;
  eq.n0 = n0;
  eq.width = W;
  eq.norm_q = h->norm_q + layer * 128;
  eq.norm_k = h->norm_k + layer * 128;
  eq.rope = rope;
  eq.q = static_cast<bf16*>(q);
  eq.k = static_cast<bf16*>(k);
  eq.v = static_cast<bf16*>(v);
  eq.kv_sample_stride = static_cast<long long>(kv_rows) * W;
  if ((rc = gemm(h, static_cast<const bf16*>(y), W, h->w_qkv + static_cast<size_t>(layer) * 3 * W * W, W, n, 3 * W, W,
                 EPI_QKV, eq)))
    return rc;
  return check_status(h);
}

int exn_test_trace(exn_handle* h, float* host, size_t floats) {
  if (!h) return fail(h, EXN_EINVAL, "exn_test_trace: null handle");
  h->trace_host = host;
  h->trace_floats = host ? floats : 0;
  return EXN_OK;
}

int exn_test_weight_bf16(exn_handle* h, const char* name, void* host_bf16, size_t elems) {
  if (!h || !name || !host_bf16) return fail(h, EXN_EINVAL, "exn_test_weight_bf16: null argument");
  int rc;
  if ((rc = use_device(h))) return rc;
  auto it = h->index.find(name);
  if (it == h->index.end()) return fail(h, EXN_EINVAL, "no tensor %s", name);
  const TensorSpec& s = h->spec[it->second];
  if (s.dims.size() != 2) return fail(h, EXN_EINVAL, "%s is not a matrix", name);
  const long long cols = s.dims[0], rows = s.dims[1];
  if (elems != static_cast<size_t>(rows * cols)) return fail(h, EXN_EINVAL, "%s: %zu elements asked", name, elems);
  Route r = route(h, s.name);
  bf16* tmp = nullptr;
  CK(cudaMalloc(&tmp, elems * 2));
  if (r.gemv) {
    if (r.gemv->kind == W_Q8)
      q8_to_bf16_launch(static_cast<const int8_t*>(r.gemv->w), r.gemv->d, tmp, rows, static_cast<int>(cols), 0, 0, h->st);
    else if (r.gemv->kind == W_BF16)
      cudaMemcpyAsync(tmp, r.gemv->w, elems * 2, cudaMemcpyDeviceToDevice, h->st);
    else
      f32_to_bf16_rows_launch(static_cast<const float*>(r.gemv->w), tmp, rows, static_cast<int>(cols), 0, 0, h->st);
    cudaMemcpyAsync(host_bf16, tmp, elems * 2, cudaMemcpyDeviceToHost, h->st);
  } else {
    // undo the interleave / fusion: copy row by row from the placed position
    std::vector<uint16_t> all(elems);
    for (long long rr = 0; rr < rows; ++rr) {
      long long dr;
      if (r.ilv > 0) {
        const long long g = rr < r.ilv ? rr : rr - r.ilv;
        dr = r.row0 + (g / 128) * 256 + (rr < r.ilv ? 0 : 128) + (g % 128);
      } else {
        dr = r.row0 + rr;
      }
      cudaMemcpyAsync(all.data() + rr * cols, r.dst + dr * cols, cols * 2, cudaMemcpyDeviceToHost, h->st);
    }
    cudaStreamSynchronize(h->st);
    std::memcpy(host_bf16, all.data(), elems * 2);
  }
  cudaStreamSynchronize(h->st);
  cudaFree(tmp);
  CK(cudaGetLastError());
  return EXN_OK;
}

int exn_test_synth_normal(exn_handle* h, float* d, int64_t n, uint64_t seed, uint32_t stream, double std_dev) {
  if (!h || !d || n < 0) return fail(h, EXN_EINVAL, "exn_test_synth_normal: bad argument");
  int rc;
  if ((rc = use_device(h))) return rc;
  const double ih_std = std::sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0);
  synth_f32_launch(d, n, seed, stream, static_cast<float>(std_dev / ih_std), 0.f, h->st);
  CK(cudaGetLastError());
  return check_status(h);
}

int exn_test_synth_q8(exn_handle* h, void* d_qs, void* d_d, int64_t n, uint64_t seed, uint32_t stream,
                      double std_dev) {
  if (!h || !d_qs || !d_d || n <= 0 || n % 32) return fail(h, EXN_EINVAL, "exn_test_synth_q8: bad argument");
  int rc;
  if ((rc = use_device(h))) return rc;
  const double ih_std = std::sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0);
  synth_q8_launch(static_cast<int8_t*>(d_qs), static_cast<__half*>(d_d), n, seed, stream,
                  static_cast<float>(std_dev / ih_std), h->st);
  CK(cudaGetLastError());
  return check_status(h);
}

int exn_test_gemm_q8(exn_handle* h, const void* a, const void* qs, const void* d, float* c, int m, int n, int k,
                     int reps, double* ms) {
  if (!h || !a || !qs || !d || !c || reps < 0) return fail(h, EXN_EINVAL, "exn_test_gemm_q8: bad argument");
  if (n % 256 || k % 64) return fail(h, EXN_EINVAL, "exn_test_gemm_q8: n %d (multiple of 256), k %d (of 64)", n, k);
  int rc;
  if ((rc = use_device(h))) return rc;
  __half* dk = nullptr;
  CK(cudaMalloc(&dk, static_cast<size_t>(n) * (k / 32) * 2));
  GemmArgs g;
  g.a = static_cast<const bf16*>(a);
  g.lda = k;
  g.M = m;
  g.N = n;
  g.K = k;
  g.epi = EPI_F32;
  g.ep.out = c;
  g.ep.ld_out = n;
  int r = q8_scales_by_kblock_launch(static_cast<const __half*>(d), dk, n, k, h->st);
  if (!r) r = gemm_q8_launch(g, static_cast<const int8_t*>(qs), dk, h->d_status, h->sms, h->st);
  cudaEvent_t ev[2] = {nullptr, nullptr};
  if (!r && reps > 0) {
    cudaEventCreate(&ev[0]);
    cudaEventCreate(&ev[1]);
    cudaEventRecord(ev[0], h->st);
    for (int i = 0; i < reps && !r; ++i) r = gemm_q8_launch(g, static_cast<const int8_t*>(qs), dk, h->d_status, h->sms, h->st);
    cudaEventRecord(ev[1], h->st);
  }
  if (r) {
    cudaStreamSynchronize(h->st);
    cudaFree(dk);
    return fail(h, EXN_ECUDA, "Q8_0 GEMM %dx%dx%d launch failed: %d", m, n, k, r);
  }
  rc = check_status(h);
  if (!rc && reps > 0 && ms) {
    float t = 0.f;
    cudaEventElapsedTime(&t, ev[0], ev[1]);
    *ms = t / reps;
  }
  for (cudaEvent_t e : ev)
    if (e) cudaEventDestroy(e);
  cudaFree(dk);
  return rc;
}

int exn_test_gemm_i8(exn_handle* h, const void* a, const void* b, const float* sa, const float* sb, float* c, int m,
                     int n, int k, int reps, double* ms) {
  if (!h || !a || !b || !sa || !sb || !c || reps < 0) return fail(h, EXN_EINVAL, "exn_test_gemm_i8: bad argument");
  int rc;
  if ((rc = use_device(h))) return rc;
  GemmArgs g;
  g.M = m;
  g.N = n;
  g.K = k;
  g.epi = EPI_I8_F32;
  g.ep.out = c;
  g.ep.ld_out = n;
  g.ep.mod = sa;
  g.ep.norm_q = sb;
  const int8_t* a8 = static_cast<const int8_t*>(a);
  const int8_t* b8 = static_cast<const int8_t*>(b);
  int r = gemm_i8_launch(g, a8, b8, h->d_status, h->sms, h->st);
  cudaEvent_t ev[2] = {nullptr, nullptr};
  if (!r && reps > 0) {
    cudaEventCreate(&ev[0]);
    cudaEventCreate(&ev[1]);
    cudaEventRecord(ev[0], h->st);
    for (int i = 0; i < reps && !r; ++i) r = gemm_i8_launch(g, a8, b8, h->d_status, h->sms, h->st);
    cudaEventRecord(ev[1], h->st);
  }
  if (r) {
    cudaStreamSynchronize(h->st);
    for (cudaEvent_t e : ev)
      if (e) cudaEventDestroy(e);
    return fail(h, r == -1 ? EXN_EINVAL : EXN_ECUDA, "int8 GEMM %dx%dx%d launch failed: %d", m, n, k, r);
  }
  rc = check_status(h);
  if (!rc && reps > 0 && ms) {
    float t = 0.f;
    cudaEventElapsedTime(&t, ev[0], ev[1]);
    *ms = t / reps;
  }
  for (cudaEvent_t e : ev)
    if (e) cudaEventDestroy(e);
  return rc;
}

int exn_test_gemm_timed(exn_handle* h, const void* a, const void* b, float* c, int m, int n, int k, int reps,
                        double* ms) {
  if (!h || !a || !b || !c || reps < 1 || !ms) return fail(h, EXN_EINVAL, "exn_test_gemm_timed: bad argument");
  int rc;
  if ((rc = use_device(h))) return rc;
  GemmEpi e;
  e.out = c;
  e.ld_out = n;
  cudaEvent_t ev[2];
  CK(cudaEventCreate(&ev[0]));
  CK(cudaEventCreate(&ev[1]));
  CK(cudaEventRecord(ev[0], h->st));
  for (int i = 0; i < reps && !rc; ++i)
    rc = gemm(h, static_cast<const bf16*>(a), k, static_cast<const bf16*>(b), k, m, n, k, EPI_F32, e);
  CK(cudaEventRecord(ev[1], h->st));
  if (!rc) rc = check_status(h);
  if (!rc) {
    float t = 0.f;
    cudaEventElapsedTime(&t, ev[0], ev[1]);
    *ms = t / reps;
  }
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  return rc;
}

int exn_test_weights_digest(exn_handle* h, uint64_t* out) {
  if (!h || !out) return fail(h, EXN_EINVAL, "exn_test_weights_digest: null argument");
  int rc;
  if ((rc = use_device(h))) return rc;
  unsigned long long* acc = nullptr;
  CK(cudaMalloc(&acc, sizeof(unsigned long long)));
  cudaMemsetAsync(acc, 0, sizeof(unsigned long long), h->st);
  digest_launch(h->slab, h->slab_bytes & ~size_t(7), acc, h->st);
  const exn_config& c = h->cfg;
  const size_t W = c.width;
  const struct {
    const GemvW* g;
    size_t n;
  } gv[4] = {{&h->lin1, W * c.freq}, {&h->lin2, W * W}, {&h->mod, 4 * W * W}, {&h->nout, W * W}};
  for (const auto& x : gv) {
    if (!x.g->w) continue;
    const size_t wb = x.g->kind == W_Q8 ? x.n : (x.g->kind == W_BF16 ? 2 * x.n : 4 * x.n);
    digest_launch(x.g->w, wb & ~size_t(7), acc, h->st);
    if (x.g->kind == W_Q8) digest_launch(x.g->d, (x.n / 32 * 2) & ~size_t(7), acc, h->st);
  }
  unsigned long long v = 0;
  rc = cudaGetLastError() == cudaSuccess ? EXN_OK : fail(h, EXN_ECUDA, "exn_test_weights_digest: launch failed");
  if (!rc && cudaMemcpyAsync(&v, acc, sizeof v, cudaMemcpyDeviceToHost, h->st) != cudaSuccess)
    rc = fail(h, EXN_ECUDA, "exn_test_weights_digest: copy failed");
  if (!rc) rc = check_status(h);
  cudaFree(acc);
  *out = v;
  return rc;
}

int exn_test_profile(exn_handle* h, int on) {
  if (!h) return fail(h, EXN_EINVAL, "exn_test_profile: null handle");
  h->prof.on = on != 0;
  return EXN_OK;
}

long long exn_test_launch_count(const exn_handle* h) { return h ? h->launches : -1; }

int exn_test_wait_probe(exn_handle* h, double seconds) {
  if (!h) return fail(h, EXN_EINVAL, "exn_test_wait_probe: null handle");
  if (!(seconds > 0.0) || seconds > 1.0) return fail(h, EXN_EINVAL, "exn_test_wait_probe: %g s (0 < s <= 1)", seconds);
  int rc;
  if ((rc = use_device(h))) return rc;
  wait_probe_launch(h->d_status, static_cast<unsigned long long>(seconds * 1e9), h->st);
  CK(cudaGetLastError());
  return check_status(h);
}

int exn_test_last_call_ms(const exn_handle* h, double* ms) {
  if (!h || !ms) return EXN_EINVAL;
  *ms = h->last_call_ms;
  return EXN_OK;
}

int exn_test_last_barrier_ms(exn_handle* h, double* ms) {
  if (!h || !ms) return fail(h, EXN_EINVAL, "exn_test_last_barrier_ms: null argument");
  *ms = h->last_ms[4];
  return EXN_OK;
}

int exn_test_last_profile(exn_handle* h, double* gemm_ms, double* attn_ms, double* other_ms, double* gateup_ms) {
  if (!h) return fail(h, EXN_EINVAL, "exn_test_last_profile: null handle");
  if (gemm_ms) *gemm_ms = h->last_ms[0] + h->last_ms[3];
  if (attn_ms) *attn_ms = h->last_ms[1];
  if (other_ms) *other_ms = h->last_ms[2];
  if (gateup_ms) *gateup_ms = h->last_ms[3];
  return EXN_OK;
}

}  // extern "C"
