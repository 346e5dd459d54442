// vae.cpp -- the host side of the VAE decoder in libexn_b200.so: exn_vae_* of
// include/exn_b200.h.  It does what ex-nihilo's src/cuda-vae.lisp does for the
// decoder -- the weights checked (open-vae, src/weights.lisp:116-127, with the
// decoder's schema vae-expected :67-100) and uploaded (upload-vae
// src/cuda-vae.lisp:15-27), a latent decoded to RGBA (vae-decode :94-136),
// scratch freed (vae-release :29-33) -- on the B200's tensor cores:
//   * every convolution is an implicit GEMM of bf16 operands with fp32
//     accumulation (conv.cu); the bf16 weights of the safetensors are used as
//     they are, reordered to tap-major rows once at load;
//   * the stream between convolutions (a residual block's input, its sum) stays
//     fp32, as in the reference; the norms write the next convolution's bf16
//     operand with the channels padded to a multiple of 64;
//   * the middle attention (one head of 1152 over the latent's pixels) is two
//     GEMMs around a row softmax.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

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

using namespace exn;

namespace {

thread_local std::string g_vae_open_error;

// (in out spatial-up temporal-up) of the decoder's stages, deepest first: src/weights.lisp:63-65
struct Stage {
  int in, out;
  bool up, tup;
};
const Stage kStages[5] = {{1152, 1152, true, true}, {1152, 1152, true, true}, {1152, 576, true, true},
                          {576, 288, true, false}, {288, 144, false, false}};
constexpr int kZ = 64, kOut = 4;

struct Spec {
  std::string name;
  std::vector<int64_t> shape;  // row-major, as the safetensors header lists it
};

// vae-expected, src/weights.lisp:67-100
std::vector<Spec> vae_expected() {
  std::vector<Spec> r;
  auto add = [&](const std::string& n, std::vector<int64_t> s) { r.push_back({n, std::move(s)}); };
  auto conv = [&](const std::string& n, int64_t o, int64_t i, int64_t k, bool frames) {
    if (frames)
      add(n + ".weight", {o, i, 1, k, k});
    else
      add(n + ".weight", {o, i, k, k});
    add(n + ".bias", {o});
  };
  auto res = [&](const std::string& p, int64_t i, int64_t o) {
    add(p + ".residual.0.gamma", {i, 1, 1, 1});
    conv(p + ".residual.2", o, i, 3, true);
    add(p + ".residual.3.gamma", {o, 1, 1, 1});
    conv(p + ".residual.6", o, o, 3, true);
    if (i != o) conv(p + ".shortcut", o, i, 1, true);
  };
  const int top = kStages[0].in;
  conv("conv2", kZ, kZ, 1, true);
  conv("decoder.conv1", top, kZ, 3, true);
  res("decoder.middle.0", top, top);
  add("decoder.middle.1.norm.gamma", {top, 1, 1});
  conv("decoder.middle.1.to_qkv", 3 * top, top, 1, false);
  conv("decoder.middle.1.proj", top, top, 1, false);
  res("decoder.middle.2", top, top);
  for (int s = 0; s < 5; ++s) {
    const Stage& st = kStages[s];
    for (int j = 0; j < 3; ++j)
      res("decoder.upsamples." + std::to_string(s) + ".upsamples." + std::to_string(j), j == 0 ? st.in : st.out, st.out);
    if (st.up) {
      conv("decoder.upsamples." + std::to_string(s) + ".upsamples.3.resample.1", st.out, st.out, 3, false);
      if (st.tup) conv("decoder.upsamples." + std::to_string(s) + ".upsamples.3.time_conv", 2 * st.out, st.out, 1, true);
    }
  }
  add("decoder.head.0.gamma", {kStages[4].out, 1, 1, 1});
  conv("decoder.head.2", kOut, kStages[4].out, 3, true);
  return r;
}

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "(";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? " " : "") + std::to_string(s[i]);
  return r + ")";
}

inline int pad64(int c) { return (c + 63) / 64 * 64; }
inline size_t al256(size_t n) { return (n + 255) & ~size_t(255); }

// ---------------------------------------------------------------------------- safetensors

// The header of a safetensors file (read-safetensors, src/safetensors.lisp:13-59): 8 bytes of
// length, then a JSON object {name: {"dtype": ..., "shape": [...], "data_offsets": [a, b]}, ...}.
struct StEntry {
  std::string dtype;
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;
};

struct Json {
  const char* p;
  const char* e;
  bool ok = true;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool eat(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  std::string str() {
    ws();
    std::string s;
    if (p >= e || *p != '"') {
      ok = false;
      return s;
    }
    ++p;
    while (p < e && *p != '"') {
      if (*p == '\\' && p + 1 < e) ++p;
      s += *p++;
    }
    if (p < e) ++p;
    return s;
  }
  int64_t num() {
    ws();
    char* end = nullptr;
    const long long v = std::strtoll(p, &end, 10);
    if (end == p) ok = false;
    p = end;
    return v;
  }
  void skip() {  // any value
    ws();
    if (p >= e) {
      ok = false;
      return;
    }
    if (*p == '"') {
      str();
    } else if (*p == '{' || *p == '[') {
      const char open = *p, close = open == '{' ? '}' : ']';
      ++p;
      if (eat(close)) return;
      do {
        if (open == '{') {
          str();
          if (!eat(':')) ok = false;
        }
        skip();
      } while (ok && eat(','));
      if (!eat(close)) ok = false;
    } else {
      while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
    }
  }
};

bool parse_header(const char* text, size_t n, std::map<std::string, StEntry>& out, std::string& err) {
  Json j{text, text + n};
  if (!j.eat('{')) {
    err = "the header is not a JSON object";
    return false;
  }
  if (j.eat('}')) return true;
  do {
    const std::string name = j.str();
    if (!j.eat(':')) j.ok = false;
    if (name == "__metadata__") {
      j.skip();
      continue;
    }
    StEntry t;
    if (!j.eat('{')) j.ok = false;
    do {
      const std::string key = j.str();
      if (!j.eat(':')) j.ok = false;
      if (key == "dtype") {
        t.dtype = j.str();
      } else if (key == "shape") {
        if (!j.eat('[')) j.ok = false;
        if (!j.eat(']')) {
          do t.shape.push_back(j.num());
          while (j.ok && j.eat(','));
          if (!j.eat(']')) j.ok = false;
        }
      } else if (key == "data_offsets") {
        if (!j.eat('[')) j.ok = false;
        t.begin = static_cast<uint64_t>(j.num());
        if (!j.eat(',')) j.ok = false;
        t.end = static_cast<uint64_t>(j.num());
        if (!j.eat(']')) j.ok = false;
      } else {
        j.skip();
      }
    } while (j.ok && j.eat(','));
    if (!j.eat('}')) j.ok = false;
    out[name] = t;
  } while (j.ok && j.eat(','));
  if (!j.ok || !j.eat('}')) {
    err = "malformed safetensors header";
    return false;
  }
  return true;
}

// ---------------------------------------------------------------------------- weights on the device

struct ConvW {
  bf16* w = nullptr;   // [rows][taps][cp]
  float* b = nullptr;  // [rows]
  int o = 0, i = 0, taps = 1, rows = 0, cp = 0;
};

}  // namespace

struct exn_vae {
  int device = 0, sms = 0;
  cudaStream_t st = nullptr;
  int* d_status = nullptr;
  std::string err;
  std::vector<Spec> spec;
  std::map<std::string, int> index;
  std::vector<char> loaded;
  size_t n_loaded = 0;
  std::map<std::string, ConvW> convs;      // by prefix ("decoder.conv1")
  std::map<std::string, float*> vecs;      // gammas
  std::vector<void*> allocs;
  // scratch, grown to the largest picture decoded
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  cudaEvent_t ev[2] = {nullptr, nullptr};
  double last_ms = 0;
};

namespace {

int vfail(exn_vae* v, int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (v)
    v->err = buf;
  else
    g_vae_open_error = buf;
  return code;
}

#define VCK(call)                                                                                       \
  do {                                                                                                  \
    cudaError_t e_ = (call);                                                                            \
    if (e_ != cudaSuccess)                                                                              \
      return vfail(v, e_ == cudaErrorMemoryAllocation ? EXN_ENOMEM : EXN_ECUDA, "%s: %s (%s:%d)", #call, \
                   cudaGetErrorString(e_), __FILE__, __LINE__);                                         \
  } while (0)

int vae_status(exn_vae* v) {
  VCK(cudaStreamSynchronize(v->st));
  int s = 0;
  VCK(cudaMemcpy(&s, v->d_status, sizeof s, cudaMemcpyDeviceToHost));
  if (s) {
    cudaMemset(v->d_status, 0, sizeof(int));
    return vfail(v, EXN_ETIMEOUT, "a kernel gave up waiting on its pipeline (status 0x%x)", s);
  }
  return EXN_OK;
}

// Place tensor IDX from fp32 values on the device (SRC, the row-major shape of the schema).
int place(exn_vae* v, int idx, const float* src) {
  const Spec& s = v->spec[idx];
  const std::string& n = s.name;
  const size_t dot = n.rfind('.');
  const std::string prefix = n.substr(0, dot), leaf = n.substr(dot + 1);
  int64_t count = 1;
  for (auto d : s.shape) count *= d;
  if (leaf == "gamma") {
    float* g = nullptr;
    VCK(cudaMalloc(&g, al256(count * 4)));
    v->allocs.push_back(g);
    VCK(cudaMemcpyAsync(g, src, count * 4, cudaMemcpyDeviceToDevice, v->st));
    v->vecs[n] = g;
  } else if (leaf == "weight") {
    ConvW& c = v->convs[prefix];
    c.o = static_cast<int>(s.shape[0]);
    c.i = static_cast<int>(s.shape[1]);
    c.taps = static_cast<int>(s.shape.back() * s.shape[s.shape.size() - 2]);
    c.rows = conv_rows(c.o);
    c.cp = pad64(c.i);
    VCK(cudaMalloc(&c.w, al256(static_cast<size_t>(c.rows) * c.taps * c.cp * 2)));
    v->allocs.push_back(c.w);
    vae_weight_launch(src, c.w, c.o, c.i, c.taps, c.rows, c.cp, v->st);
  } else if (leaf == "bias") {
    ConvW& c = v->convs[prefix];
    const int rows = conv_rows(static_cast<int>(count));
    VCK(cudaMalloc(&c.b, al256(static_cast<size_t>(rows) * 4)));
    v->allocs.push_back(c.b);
    VCK(cudaMemsetAsync(c.b, 0, static_cast<size_t>(rows) * 4, v->st));
    VCK(cudaMemcpyAsync(c.b, src, count * 4, cudaMemcpyDeviceToDevice, v->st));
  } else {
    return vfail(v, EXN_EINVAL, "no place for VAE tensor %s", n.c_str());
  }
  VCK(cudaGetLastError());
  if (!v->loaded[idx]) {
    v->loaded[idx] = 1;
    ++v->n_loaded;
  }
  return EXN_OK;
}

// ---------------------------------------------------------------------------- the decoder

struct Scratch {
  float *x, *y, *t, *keep, *rgba;
  bf16 *a, *b;
  float* s;   // attention scores [n][n]
  bf16* p;    // probabilities [n][n]
  bf16 *qkv, *vt, *att;
};

int ensure_scratch(exn_vae* v, int h, int w, Scratch& sc) {
  const size_t n0 = static_cast<size_t>(h) * w;
  // the largest pixels x channels of the stream anywhere in the decoder
  size_t maxf = n0 * kStages[0].in, maxb = n0 * 128;
  size_t hh = h, ww = w;
  for (int s = 0; s < 5; ++s) {
    const size_t n = hh * ww;
    maxf = std::max(maxf, n * std::max(kStages[s].in, kStages[s].out));
    maxb = std::max(maxb, n * pad64(std::max(kStages[s].in, kStages[s].out)));
    if (kStages[s].up) {
      hh *= 2;
      ww *= 2;
      maxf = std::max(maxf, hh * ww * kStages[s].out);
      maxb = std::max(maxb, hh * ww * pad64(kStages[s].out));
    }
  }
  const size_t top = kStages[0].in;
  const size_t need = 4 * al256(maxf * 4) + al256(hh * ww * 4 * 4) + 2 * al256(maxb * 2) + al256(n0 * n0 * 4) +
                      al256(n0 * n0 * 2) + al256(n0 * 3 * top * 2) + al256(top * n0 * 2) + al256(n0 * top * 2);
  if (need > v->scratch_bytes) {
    if (v->scratch) cudaFree(v->scratch);
    v->scratch = nullptr;
    v->scratch_bytes = 0;
    VCK(cudaMalloc(&v->scratch, need));
    v->scratch_bytes = need;
  }
  char* m = static_cast<char*>(v->scratch);
  auto take = [&](size_t bytes) {
    char* r = m;
    m += al256(bytes);
    return r;
  };
  sc.x = reinterpret_cast<float*>(take(maxf * 4));
  sc.y = reinterpret_cast<float*>(take(maxf * 4));
  sc.t = reinterpret_cast<float*>(take(maxf * 4));
  sc.keep = reinterpret_cast<float*>(take(maxf * 4));
  sc.rgba = reinterpret_cast<float*>(take(hh * ww * 4 * 4));
  sc.a = reinterpret_cast<bf16*>(take(maxb * 2));
  sc.b = reinterpret_cast<bf16*>(take(maxb * 2));
  sc.s = reinterpret_cast<float*>(take(n0 * n0 * 4));
  sc.p = reinterpret_cast<bf16*>(take(n0 * n0 * 2));
  sc.qkv = reinterpret_cast<bf16*>(take(n0 * 3 * top * 2));
  sc.vt = reinterpret_cast<bf16*>(take(top * n0 * 2));
  sc.att = reinterpret_cast<bf16*>(take(n0 * top * 2));
  return EXN_OK;
}

const ConvW* cw(exn_vae* v, const std::string& prefix) {
  auto it = v->convs.find(prefix);
  return it == v->convs.end() ? nullptr : &it->second;
}

// out f32 [h w][o] = conv(x bf16 [h w][cp]) + bias (+ res); or bf16 / RGBA by KIND
int conv(exn_vae* v, const std::string& prefix, const bf16* x, int h, int w, void* out, int kind,
         const float* res = nullptr, const float* dup = nullptr, int dup_ci = 0, int dup_ft = 1) {
  const ConvW* c = cw(v, prefix);
  if (!c || !c->w || !c->b) return vfail(v, EXN_ENOWEIGHTS, "VAE tensor %s not loaded", prefix.c_str());
  ConvArgs a;
  a.x = x;
  a.wt = c->w;
  a.h = h;
  a.w = w;
  a.cp = c->cp;
  a.cout = c->o;
  a.taps = c->taps;
  a.ep.kind = kind;
  a.ep.out = out;
  a.ep.ld_out = c->o;
  a.ep.bias = c->b;
  a.ep.res = res;
  a.ep.ld_res = c->o;
  a.ep.dup = dup;
  a.ep.dup_ci = dup_ci;
  a.ep.dup_ft = dup_ft;
  a.ep.out_w = w;
  const int r = conv_launch(a, v->d_status, v->sms, v->st);
  if (r) return vfail(v, EXN_ECUDA, "convolution %s (%d x %d, %d -> %d) launch failed: %d", prefix.c_str(), h, w, c->i,
                      c->o, r);
  return EXN_OK;
}

int norm(exn_vae* v, const std::string& gamma, const float* x, bf16* y, int n, int c, int silu) {
  auto it = v->vecs.find(gamma);
  if (it == v->vecs.end()) return vfail(v, EXN_ENOWEIGHTS, "VAE tensor %s not loaded", gamma.c_str());
  vae_norm_launch(x, it->second, y, n, c, pad64(c), silu, v->st);
  return EXN_OK;
}

// OUT = conv(silu(norm(conv(silu(norm(X)))))) + (X, or its 1 x 1 shortcut): ref_vae.py:56-62
int resblock(exn_vae* v, const std::string& p, const float* x, float* out, int i, int o, int h, int w, Scratch& sc) {
  const int n = h * w;
  int rc;
  if ((rc = norm(v, p + ".residual.0.gamma", x, sc.a, n, i, 1))) return rc;
  if ((rc = conv(v, p + ".residual.2", sc.a, h, w, sc.t, CONV_F32))) return rc;
  if ((rc = norm(v, p + ".residual.3.gamma", sc.t, sc.a, n, o, 1))) return rc;
  if (i == o) return conv(v, p + ".residual.6", sc.a, h, w, out, CONV_F32, x);
  if ((rc = conv(v, p + ".residual.6", sc.a, h, w, sc.t, CONV_F32))) return rc;
  vae_to_bf16_launch(x, sc.b, n, i, pad64(i), v->st);
  return conv(v, p + ".shortcut", sc.b, h, w, out, CONV_F32, sc.t);
}

// one head over the N pixels: OUT = proj(softmax(q k^T / sqrt(c)) v) + X (ref_vae.py:65-74)
int attention(exn_vae* v, const std::string& p, const float* x, float* out, int c, int h, int w, Scratch& sc) {
  const int n = h * w;
  int rc;
  if ((rc = norm(v, p + ".norm.gamma", x, sc.a, n, c, 0))) return rc;
  if ((rc = conv(v, p + ".to_qkv", sc.a, h, w, sc.qkv, CONV_BF16))) return rc;
  GemmArgs g;
  g.a = sc.qkv;
  g.lda = 3 * c;
  g.b = sc.qkv + c;
  g.ldb = 3 * c;
  g.M = n;
  g.N = n;
  g.K = c;
  g.epi = EPI_F32;
  g.ep.out = sc.s;
  g.ep.ld_out = n;
  int r = gemm_launch(g, v->d_status, v->sms, v->st);
  if (r) return vfail(v, EXN_ECUDA, "attention scores GEMM (%d pixels) launch failed: %d", n, r);
  vae_softmax_launch(sc.s, sc.p, n, static_cast<float>(1.0 / std::sqrt(static_cast<double>(c))), v->st);
  vae_transpose_launch(sc.qkv + 2 * c, 3 * c, sc.vt, n, c, v->st);
  GemmArgs o;
  o.a = sc.p;
  o.lda = n;
  o.b = sc.vt;
  o.ldb = n;
  o.M = n;
  o.N = c;
  o.K = n;
  o.epi = EPI_BF16;
  o.ep.out = sc.att;
  o.ep.ld_out = c;
  r = gemm_launch(o, v->d_status, v->sms, v->st);
  if (r) return vfail(v, EXN_ECUDA, "attention value GEMM (%d pixels) launch failed: %d", n, r);
  return conv(v, p + ".proj", sc.att, h, w, out, CONV_F32, x);
}

// vae-decode, src/cuda-vae.lisp:94-136 (ref_vae.py:86-104): latent on the device (64 x h x w,
// channel-major) -> RGBA f32 [16h][16w][4] in sc.rgba
int decode(exn_vae* v, const float* d_latent, int h, int w, Scratch& sc) {
  int rc;
  const int top = kStages[0].in;
  int hh = h, ww = w;
  int n = hh * ww;
  latent_rows_launch(d_latent, sc.a, 1, kZ, n, v->st);
  if ((rc = conv(v, "conv2", sc.a, hh, ww, sc.b, CONV_BF16))) return rc;
  if ((rc = conv(v, "decoder.conv1", sc.b, hh, ww, sc.x, CONV_F32))) return rc;
  float* x = sc.x;
  float* y = sc.y;
  if ((rc = resblock(v, "decoder.middle.0", x, y, top, top, hh, ww, sc))) return rc;
  std::swap(x, y);
  if ((rc = attention(v, "decoder.middle.1", x, y, top, hh, ww, sc))) return rc;
  std::swap(x, y);
  if ((rc = resblock(v, "decoder.middle.2", x, y, top, top, hh, ww, sc))) return rc;
  std::swap(x, y);
  for (int s = 0; s < 5; ++s) {
    const Stage& st = kStages[s];
    n = hh * ww;
    VCK(cudaMemcpyAsync(sc.keep, x, static_cast<size_t>(n) * st.in * 4, cudaMemcpyDeviceToDevice, v->st));
    for (int j = 0; j < 3; ++j) {
      const std::string p = "decoder.upsamples." + std::to_string(s) + ".upsamples." + std::to_string(j);
      if ((rc = resblock(v, p, x, y, j == 0 ? st.in : st.out, st.out, hh, ww, sc))) return rc;
      std::swap(x, y);
    }
    if (st.up) {
      vae_up2_launch(x, sc.a, hh, ww, st.out, pad64(st.out), v->st);
      const std::string p = "decoder.upsamples." + std::to_string(s) + ".upsamples.3.resample.1";
      // the DupUp3D shortcut of the stage's input added in the convolution's epilogue
      if ((rc = conv(v, p, sc.a, 2 * hh, 2 * ww, y, CONV_F32, nullptr, sc.keep, st.in, st.tup ? 2 : 1))) return rc;
      std::swap(x, y);
      hh *= 2;
      ww *= 2;
    }
  }
  n = hh * ww;
  if ((rc = norm(v, "decoder.head.0.gamma", x, sc.a, n, kStages[4].out, 1))) return rc;
  if ((rc = conv(v, "decoder.head.2", sc.a, hh, ww, sc.rgba, CONV_RGBA))) return rc;
  VCK(cudaGetLastError());
  return EXN_OK;
}

}  // namespace

// ============================================================================ C ABI

extern "C" {

int exn_vae_open(int device, exn_vae** out) {
  if (!out) return vfail(nullptr, EXN_EINVAL, "exn_vae_open: null handle pointer");
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
    return vfail(nullptr, EXN_ECUDA, "exn_vae_open: no CUDA device %d", device);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess)
    return vfail(nullptr, EXN_ECUDA, "exn_vae_open: cannot query device %d", device);
  if (prop.major != 10)
    return vfail(nullptr, EXN_EUNSUPPORTED, "exn_vae_open: device %d is sm_%d%d; this library is built for sm_100a",
                 device, prop.major, prop.minor);
  exn_vae* v = new exn_vae();
  v->device = device;
  v->sms = prop.multiProcessorCount;
  const int rc = [&]() -> int {
    VCK(cudaSetDevice(device));
    VCK(cudaStreamCreateWithFlags(&v->st, cudaStreamNonBlocking));
    VCK(cudaMalloc(&v->d_status, sizeof(int)));
    VCK(cudaMemset(v->d_status, 0, sizeof(int)));
    VCK(static_cast<cudaError_t>(conv_prepare()));
    VCK(static_cast<cudaError_t>(gemm_prepare()));
    VCK(cudaEventCreate(&v->ev[0]));
    VCK(cudaEventCreate(&v->ev[1]));
    return EXN_OK;
  }();
  if (rc) {
    g_vae_open_error = v->err;
    exn_vae_close(v);
    return rc;
  }
  v->spec = vae_expected();
  for (size_t i = 0; i < v->spec.size(); ++i) v->index[v->spec[i].name] = static_cast<int>(i);
  v->loaded.assign(v->spec.size(), 0);
  *out = v;
  return EXN_OK;
}

void exn_vae_close(exn_vae* v) {
  if (!v) return;
  cudaSetDevice(v->device);
  if (v->st) cudaStreamSynchronize(v->st);
  for (void* p : v->allocs) cudaFree(p);
  if (v->scratch) cudaFree(v->scratch);
  if (v->d_status) cudaFree(v->d_status);
  for (cudaEvent_t e : v->ev)
    if (e) cudaEventDestroy(e);
  if (v->st) cudaStreamDestroy(v->st);
  delete v;
}

const char* exn_vae_last_error(const exn_vae* v) { return v ? v->err.c_str() : g_vae_open_error.c_str(); }

int exn_vae_load_safetensors(exn_vae* v, const char* path) {
  if (!v || !path) return vfail(v, EXN_EINVAL, "exn_vae_load_safetensors: null argument");
  VCK(cudaSetDevice(v->device));
  const int fd = ::open(path, O_RDONLY);
  if (fd < 0) return vfail(v, EXN_EIO, "%s: cannot open", path);
  struct stat sb;
  if (fstat(fd, &sb) != 0 || sb.st_size < 8) {
    ::close(fd);
    return vfail(v, EXN_EIO, "%s: not a safetensors file", path);
  }
  const size_t size = static_cast<size_t>(sb.st_size);
  void* map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map == MAP_FAILED) return vfail(v, EXN_EIO, "%s: cannot map", path);
  const uint8_t* base = static_cast<const uint8_t*>(map);
  uint64_t hlen = 0;
  std::memcpy(&hlen, base, 8);
  std::map<std::string, StEntry> ents;
  std::string err;
  int rc = EXN_OK;
  if (hlen > size - 8 || !parse_header(reinterpret_cast<const char*>(base + 8), hlen, ents, err))
    rc = vfail(v, EXN_EIO, "%s: %s", path, err.empty() ? "header past the end of the file" : err.c_str());
  // open-vae (src/weights.lisp:116-127): every decoder tensor present with its shape
  if (!rc) {
    std::string problems;
    for (const Spec& s : v->spec) {
      auto it = ents.find(s.name);
      if (it == ents.end())
        problems += "\n  missing " + s.name;
      else if (it->second.shape != s.shape)
        problems += "\n  " + s.name + " is " + shape_str(it->second.shape) + ", not " + shape_str(s.shape);
      else if (it->second.dtype != "BF16" && it->second.dtype != "F32")
        problems += "\n  " + s.name + " is " + it->second.dtype + ", not BF16 or F32";
      else if (8 + hlen + it->second.end > size || it->second.end < it->second.begin)
        problems += "\n  " + s.name + " lies past the end of the file";
    }
    if (!problems.empty()) rc = vfail(v, EXN_ESHAPE, "%s:%s", path, problems.c_str());
  }
  float* dev = nullptr;
  if (!rc) {
    size_t maxn = 0;
    for (const Spec& s : v->spec) {
      size_t c = 1;
      for (auto d : s.shape) c *= static_cast<size_t>(d);
      maxn = std::max(maxn, c);
    }
    std::vector<float> host(maxn);
    if (cudaMalloc(&dev, maxn * 4) != cudaSuccess) rc = vfail(v, EXN_ENOMEM, "exn_vae_load_safetensors: staging");
    for (size_t i = 0; i < v->spec.size() && !rc; ++i) {
      const Spec& s = v->spec[i];
      const StEntry& e = ents[s.name];
      size_t c = 1;
      for (auto d : s.shape) c *= static_cast<size_t>(d);
      const uint8_t* src = base + 8 + hlen + e.begin;
      if (e.dtype == "BF16") {
        const uint16_t* b = reinterpret_cast<const uint16_t*>(src);
        for (size_t k = 0; k < c; ++k) {
          const uint32_t u = static_cast<uint32_t>(b[k]) << 16;
          std::memcpy(&host[k], &u, 4);
        }
      } else {
        std::memcpy(host.data(), src, c * 4);
      }
      if (cudaMemcpy(dev, host.data(), c * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        rc = vfail(v, EXN_ECUDA, "upload of %s failed", s.name.c_str());
      if (!rc) rc = place(v, static_cast<int>(i), dev);
      if (!rc && cudaStreamSynchronize(v->st) != cudaSuccess) rc = vfail(v, EXN_ECUDA, "placing %s", s.name.c_str());
    }
  }
  if (dev) cudaFree(dev);
  munmap(map, size);
  return rc;
}

int exn_vae_load_synthetic(exn_vae* v, uint64_t seed) {
  if (!v) return vfail(v, EXN_EINVAL, "exn_vae_load_synthetic: null handle");
  VCK(cudaSetDevice(v->device));
  const double ih_std = std::sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0);
  size_t maxn = 0;
  for (const Spec& s : v->spec) {
    size_t c = 1;
    for (auto d : s.shape) c *= static_cast<size_t>(d);
    maxn = std::max(maxn, c);
  }
  float* f = nullptr;
  VCK(cudaMalloc(&f, maxn * 4));
  int rc = EXN_OK;
  for (size_t i = 0; i < v->spec.size() && !rc; ++i) {
    const Spec& s = v->spec[i];
    size_t c = 1;
    for (auto d : s.shape) c *= static_cast<size_t>(d);
    const std::string leaf = s.name.substr(s.name.rfind('.') + 1);
    // the stream's statistics stay those of a trained decoder: weights N(0, 1 / fan_in), biases
    // N(0, 0.02), gains 1 + N(0, 0.1); every value then rounded to bf16, the checkpoints' type
    double std_dev = 0.02, base = 0.0;
    if (leaf == "weight") {
      double fan_in = 1;
      for (size_t k = 1; k < s.shape.size(); ++k) fan_in *= static_cast<double>(s.shape[k]);
      std_dev = 1.0 / std::sqrt(fan_in);
    } else if (leaf == "gamma") {
      std_dev = 0.1;
      base = 1.0;
    }
    synth_f32_launch(f, static_cast<long long>(c), seed, static_cast<uint32_t>(20000 + i),
                     static_cast<float>(std_dev / ih_std), static_cast<float>(base), v->st);
    round_bf16_launch(f, static_cast<long long>(c), v->st);
    rc = place(v, static_cast<int>(i), f);
    if (!rc && cudaStreamSynchronize(v->st) != cudaSuccess) rc = vfail(v, EXN_ECUDA, "placing %s", s.name.c_str());
  }
  cudaFree(f);
  return rc;
}

int exn_vae_weights_ready(const exn_vae* v) {
  if (!v) return EXN_EINVAL;
  return v->n_loaded == v->spec.size() ? EXN_OK : EXN_ENOWEIGHTS;
}

int exn_vae_decode(exn_vae* v, const float* latent, int h, int w, float* rgba) {
  if (!v || !latent || !rgba) return vfail(v, EXN_EINVAL, "exn_vae_decode: null argument");
  if (h < 1 || w < 1 || (h * w) % 64)
    return vfail(v, EXN_EINVAL, "exn_vae_decode: a %d x %d latent; h x w must be a multiple of 64 (the middle "
                 "attention's products take the latent's pixels 64 at a time)", h, w);
  if (v->n_loaded != v->spec.size())
    return vfail(v, EXN_ENOWEIGHTS, "%zu of %zu VAE tensors loaded", v->n_loaded, v->spec.size());
  VCK(cudaSetDevice(v->device));
  Scratch sc;
  int rc;
  if ((rc = ensure_scratch(v, h, w, sc))) return rc;
  // the latent goes to the last buffer the decoder reads only at its end (the RGBA output)
  const size_t lat = static_cast<size_t>(kZ) * h * w;
  VCK(cudaMemcpyAsync(sc.rgba, latent, lat * 4, cudaMemcpyHostToDevice, v->st));
  VCK(cudaEventRecord(v->ev[0], v->st));
  if ((rc = decode(v, sc.rgba, h, w, sc))) return rc;
  VCK(cudaEventRecord(v->ev[1], v->st));
  const size_t px = static_cast<size_t>(16 * h) * (16 * w) * 4;
  VCK(cudaMemcpyAsync(rgba, sc.rgba, px * 4, cudaMemcpyDeviceToHost, v->st));
  if ((rc = vae_status(v))) return rc;
  float ms = 0.f;
  v->last_ms = cudaEventElapsedTime(&ms, v->ev[0], v->ev[1]) == cudaSuccess ? ms : 0.0;
  return EXN_OK;
}

int exn_vae_release(exn_vae* v) {
  if (!v) return vfail(v, EXN_EINVAL, "exn_vae_release: null handle");
  VCK(cudaSetDevice(v->device));
  VCK(cudaStreamSynchronize(v->st));
  if (v->scratch) cudaFree(v->scratch);
  v->scratch = nullptr;
  v->scratch_bytes = 0;
  return EXN_OK;
}

int exn_test_vae_last_ms(const exn_vae* v, double* ms) {
  if (!v || !ms) return EXN_EINVAL;
  *ms = v->last_ms;
  return EXN_OK;
}

}  // extern "C"
