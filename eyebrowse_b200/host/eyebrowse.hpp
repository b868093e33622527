// eyebrowse.hpp -- C++ host side of the attention path, mirroring the
// reference's Rust interface on top of the C ABI (include/eyebrowse_attn.h).
//
// The reference host code is Rust; no Rust toolchain exists here, so this
// header restates the interface a Rust caller uses, with the same names,
// argument meanings and order:
//   eyebrowse::kernels::{attn_prefill, attn_decode, rope, kv_write, rmsnorm}
//     (crates/eyebrowse-kernels/src/lib.rs:15-19; attention.rs:94-162,
//      rope.rs:38-69, ops.rs:150-179, rmsnorm.rs:42-64)
//   eyebrowse::nn::{Rope, KvCache, Attention}
//     (crates/eyebrowse-nn/src/rope.rs:18-75, kv_cache.rs:9-49,
//      attention.rs:10-185 -- the body after the q/k/v projections)
// Tensor is a device buffer with a shape (Tensor::from_f32 / empty /
// to_f32, as eyebrowse-gpu's). Recorder owns a CUDA stream and the scratch
// workspaces the C ABI asks for; kernels are enqueued at once, and submit()
// waits for them (the reference records, then submits). Errors the reference
// would meet as a panic (bad shapes, missing device) throw eyebrowse::Error
// carrying the C ABI's status string.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "../../include/eyebrowse_attn.h"

namespace eyebrowse {

struct Error : std::runtime_error {
  int status;
  Error(const std::string& what, int st) : std::runtime_error(what), status(st) {}
};

inline void check(int st, const char* call) {
  if (st != EB_OK) throw Error(std::string(call) + ": " + eb_status_string(st), st);
}
inline void check_cuda(cudaError_t e, const char* call) {
  if (e != cudaSuccess) throw Error(std::string(call) + ": " + cudaGetErrorString(e), EB_ERR_CUDA);
}

enum class DType : int32_t { F32 = EB_F32, F16 = EB_F16, BF16 = EB_BF16 };

inline size_t dtype_bytes(DType d) { return d == DType::F32 ? 4 : 2; }

// A device buffer with a shape (row-major) and an element type.
class Tensor {
 public:
  Tensor() = default;
  static Tensor empty(std::vector<size_t> shape, DType dt = DType::F32) {
    Tensor t;
    t.shape_ = std::move(shape);
    t.dtype_ = dt;
    void* p = nullptr;
    const size_t n = std::max<size_t>(t.bytes(), 16);
    check_cuda(cudaMalloc(&p, n), "cudaMalloc");
    t.buf_ = std::shared_ptr<void>(p, [](void* q) { cudaFree(q); });
    return t;
  }
  static Tensor from_f32(std::vector<size_t> shape, const std::vector<float>& host) {
    Tensor t = empty(std::move(shape), DType::F32);
    if (host.size() != t.numel()) throw Error("Tensor::from_f32: size mismatch", EB_ERR_INVALID_ARGUMENT);
    check_cuda(cudaMemcpy(t.ptr(), host.data(), t.bytes(), cudaMemcpyHostToDevice), "cudaMemcpy");
    return t;
  }
  // f16 weights from f32 host values (round to nearest even), as the
  // reference's pack_f16 stores them (testutil.rs:45-60)
  static Tensor from_f16(std::vector<size_t> shape, const std::vector<float>& host) {
    Tensor t = empty(std::move(shape), DType::F16);
    if (host.size() != t.numel()) throw Error("Tensor::from_f16: size mismatch", EB_ERR_INVALID_ARGUMENT);
    std::vector<__half> h(host.size());
    for (size_t i = 0; i < host.size(); i++) h[i] = __float2half_rn(host[i]);
    check_cuda(cudaMemcpy(t.ptr(), h.data(), t.bytes(), cudaMemcpyHostToDevice), "cudaMemcpy");
    return t;
  }
  static Tensor zeros(std::vector<size_t> shape, DType dt = DType::F32) {
    Tensor t = empty(std::move(shape), dt);
    check_cuda(cudaMemset(t.ptr(), 0, t.bytes()), "cudaMemset");
    return t;
  }
  std::vector<float> to_f32() const {
    if (dtype_ != DType::F32) throw Error("Tensor::to_f32: not an f32 tensor", EB_ERR_INVALID_ARGUMENT);
    std::vector<float> h(numel());
    check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    check_cuda(cudaMemcpy(h.data(), ptr(), bytes(), cudaMemcpyDeviceToHost), "cudaMemcpy");
    return h;
  }
  size_t numel() const {
    size_t n = 1;
    for (size_t s : shape_) n *= s;
    return n;
  }
  size_t bytes() const { return numel() * dtype_bytes(dtype_); }
  void* ptr() const { return buf_.get(); }
  DType dtype() const { return dtype_; }
  const std::vector<size_t>& shape() const { return shape_; }

 private:
  std::shared_ptr<void> buf_;
  std::vector<size_t> shape_;
  DType dtype_ = DType::F32;
};

// A CUDA stream plus grow-only scratch workspaces (one per call kind, so a
// decode workspace's split-K tickets stay zeroed between calls).
class Recorder {
 public:
  Recorder() { check_cuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate"); }
  ~Recorder() {
    if (stream_) cudaStreamDestroy(stream_);
  }
  Recorder(const Recorder&) = delete;
  Recorder& operator=(const Recorder&) = delete;
  eb_stream_t stream() const { return reinterpret_cast<eb_stream_t>(stream_); }
  // Scratch of at least `bytes` for call kind `kind` (zeroed when grown).
  std::pair<void*, size_t> workspace(int kind, size_t bytes) {
    if (kind >= (int)ws_.size()) ws_.resize(kind + 1);
    Tensor& w = ws_[kind];
    if (bytes > 0 && w.bytes() < bytes) {
      submit();
      w = Tensor::zeros({bytes}, DType::F16);  // bytes/2 halves >= bytes bytes
    }
    return {bytes ? w.ptr() : nullptr, bytes ? w.bytes() : 0};
  }
  void submit() { check_cuda(cudaStreamSynchronize(stream_), "cudaStreamSynchronize"); }

 private:
  cudaStream_t stream_ = nullptr;
  std::vector<Tensor> ws_;
};

enum WorkspaceKind {
  kWsPrefill = 0,
  kWsDecode = 1,
  kWsKernelPrefill = 2,
  kWsKernelDecode = 3,
  kWsLinear = 4
};

// ------------------------------------------------------------ eyebrowse-kernels
namespace kernels {

// attention.rs:94-120: causal GQA over q [s,h,hd], k/v [s,hkv,hd] -> o [s,h,hd], f32.
inline void attn_prefill(Recorder& rec, const Tensor& q, const Tensor& k, const Tensor& v,
                         const Tensor& o, size_t h, size_t hkv, size_t s, size_t hd,
                         float scale) {
  auto ws = rec.workspace(kWsKernelPrefill, eb_attn_prefill_workspace_bytes(h, hkv, s, hd));
  check(eb_attn_prefill(static_cast<const float*>(q.ptr()), static_cast<const float*>(k.ptr()),
                        static_cast<const float*>(v.ptr()), static_cast<float*>(o.ptr()), h, hkv,
                        s, hd, scale, ws.first, ws.second, rec.stream()),
        "attn_prefill");
}

// attention.rs:124-162: one query [h,hd] over cache rows 0..=pos of [max_seq,hkv,hd].
inline void attn_decode(Recorder& rec, const Tensor& q, const Tensor& kcache,
                        const Tensor& vcache, const Tensor& o, size_t h, size_t hkv, size_t pos,
                        size_t hd, size_t max_seq, float scale) {
  auto ws = rec.workspace(kWsKernelDecode, eb_attn_decode_workspace_bytes(h, hkv, pos, hd));
  check(eb_attn_decode(static_cast<const float*>(q.ptr()), static_cast<const float*>(kcache.ptr()),
                       static_cast<const float*>(vcache.ptr()), static_cast<float*>(o.ptr()), h,
                       hkv, pos, hd, max_seq, scale, ws.first, ws.second, rec.stream()),
        "attn_decode");
}

// rope.rs:38-69: half-split rotation of x [seq,n_heads,hd] with table rows base_pos + s.
inline void rope(Recorder& rec, const Tensor& x, const Tensor& cos, const Tensor& sin,
                 const Tensor& out, size_t seq, size_t n_heads, size_t head_dim,
                 size_t base_pos) {
  check(eb_rope(static_cast<const float*>(x.ptr()), static_cast<const float*>(cos.ptr()),
                static_cast<const float*>(sin.ptr()), static_cast<float*>(out.ptr()), seq,
                n_heads, head_dim, base_pos, rec.stream()),
        "rope");
}

// ops.rs:150-179: src [count,hkv,hd] -> cache rows [dst_start, dst_start + count).
inline void kv_write(Recorder& rec, const Tensor& cache, const Tensor& src, size_t hkv,
                     size_t count, size_t hd, size_t max_seq, size_t dst_start) {
  check(eb_kv_write(static_cast<float*>(cache.ptr()), static_cast<const float*>(src.ptr()), hkv,
                    count, hd, max_seq, dst_start, rec.stream()),
        "kv_write");
}

// rmsnorm.rs:42-64: out = x * 1/sqrt(mean(x^2) + eps) * weight, per row.
inline void rmsnorm(Recorder& rec, const Tensor& x, const Tensor& weight, const Tensor& out,
                    size_t rows, size_t dim, float eps) {
  check(eb_rmsnorm(static_cast<const float*>(x.ptr()), static_cast<const float*>(weight.ptr()),
                   static_cast<float*>(out.ptr()), rows, dim, eps, rec.stream()),
        "rmsnorm");
}

// matmul.rs:128-149: c [m, out_f] = a [m, in_f] (f32) * w [out_f, in_f]^T (f16 HF layout).
inline void linear_f16w(Recorder& rec, const Tensor& a, const Tensor& w, const Tensor& c,
                        size_t m, size_t in_f, size_t out_f) {
  auto ws = rec.workspace(kWsLinear, eb_linear_f16w_workspace_bytes(m, in_f, out_f));
  check(eb_linear_f16w(static_cast<const float*>(a.ptr()), w.ptr(), static_cast<float*>(c.ptr()),
                       m, in_f, out_f, ws.first, ws.second, rec.stream()),
        "linear_f16w");
}

}  // namespace kernels

// ------------------------------------------------------------ eyebrowse-nn
namespace nn {

// rope.rs:18-50: cos/sin tables [max_seq, head_dim/2] built in f64 on the
// host; pairs k >= rope_angles pass through (cos 1, sin 0).
struct Rope {
  Tensor cos, sin;
  size_t max_seq = 0, head_dim = 0;
  static Rope build_partial(size_t max_seq, size_t head_dim, float theta, size_t rope_angles) {
    std::vector<float> c(max_seq * (head_dim / 2)), s(c.size());
    check(eb_rope_tables(c.data(), s.data(), max_seq, head_dim, rope_angles, theta),
          "Rope::build");
    Rope r;
    r.cos = Tensor::from_f32({max_seq, head_dim / 2}, c);
    r.sin = Tensor::from_f32({max_seq, head_dim / 2}, s);
    r.max_seq = max_seq;
    r.head_dim = head_dim;
    return r;
  }
  static Rope build(size_t max_seq, size_t head_dim, float theta) {
    return build_partial(max_seq, head_dim, theta, head_dim / 2);
  }
};

// kv_cache.rs:9-49: per-layer k[l], v[l] of [max_seq, n_kv_heads, head_dim].
struct KvCache {
  std::vector<Tensor> k, v;
  size_t max_seq = 0, n_kv_heads = 0, head_dim = 0;
  DType dtype = DType::F32;
  static KvCache create(size_t n_layers, size_t max_seq, size_t n_kv_heads, size_t head_dim,
                        DType dtype = DType::F32) {
    KvCache c;
    c.max_seq = max_seq;
    c.n_kv_heads = n_kv_heads;
    c.head_dim = head_dim;
    c.dtype = dtype;
    for (size_t l = 0; l < n_layers; l++) {
      c.k.push_back(Tensor::zeros({max_seq, n_kv_heads, head_dim}, dtype));
      c.v.push_back(Tensor::zeros({max_seq, n_kv_heads, head_dim}, dtype));
    }
    return c;
  }
};

// linear.rs:5-23: a bias-free linear layer, f16 weights [out_f, in_f].
struct Linear {
  Tensor w;
  size_t in_f = 0, out_f = 0;
  // x [rows, in_f] f32 -> [rows, out_f] f32
  Tensor forward(Recorder& rec, const Tensor& x, size_t rows) const {
    Tensor out = Tensor::empty({rows, out_f});
    kernels::linear_f16w(rec, x, w, out, rows, in_f, out_f);
    return out;
  }
};

// attention.rs:10-185 after the projections: the fields that shape the path
// (GQA heads, optional per-head q/k/v RMSNorm weights, scale), prefill over
// positions 0..seq and decode at pos, both writing the layer's cache.
struct Attention {
  // attention.rs:11-14 (projections; needed by forward() only)
  std::optional<Linear> q_proj, k_proj, v_proj, o_proj;
  std::optional<Tensor> q_norm, k_norm, v_norm;  // [head_dim] weights
  size_t n_heads = 0, n_kv_heads = 0, head_dim = 0;
  float scale = 0.f, eps = 1e-6f;
  DType dtype_qkv = DType::F32, dtype_out = DType::F32;
  // Sliding-window layers (Gemma local attention; the reference defers them):
  // row i sees keys i - window < j <= i. 0 = the whole causal context.
  size_t window = 0;

  eb_attn_desc desc(const KvCache& kv) const {
    eb_attn_desc d{};
    d.n_heads = (int32_t)n_heads;
    d.n_kv_heads = (int32_t)n_kv_heads;
    d.head_dim = (int32_t)head_dim;
    d.max_seq = (int32_t)kv.max_seq;
    d.dtype_qkv = (int32_t)dtype_qkv;
    d.dtype_cache = (int32_t)kv.dtype;
    d.dtype_out = (int32_t)dtype_out;
    d.eps = eps;
    d.scale = scale;
    d.window = (int32_t)window;
    return d;
  }
  eb_attn_layer layer(const Rope& rope) const {
    eb_attn_layer l{};
    l.q_norm_w = q_norm ? static_cast<const float*>(q_norm->ptr()) : nullptr;
    l.k_norm_w = k_norm ? static_cast<const float*>(k_norm->ptr()) : nullptr;
    l.v_norm_w = v_norm ? static_cast<const float*>(v_norm->ptr()) : nullptr;
    l.rope_cos = static_cast<const float*>(rope.cos.ptr());
    l.rope_sin = static_cast<const float*>(rope.sin.ptr());
    return l;
  }
  // attention.rs:30-45: x [rows, hidden] at positions base_pos.. A fresh
  // multi-row prompt (base_pos 0, rows > 1) takes the prefill path and
  // returns [rows, hidden]; anything else is one decode step at base_pos,
  // which, as the reference's decode (attention.rs:120-130) does, projects
  // only the first row of x and returns [1, hidden].
  Tensor forward(Recorder& rec, const Tensor& x, const Rope& rope, KvCache& kv, size_t layer_idx,
                 size_t rows, size_t base_pos) const {
    if (!q_proj || !k_proj || !v_proj || !o_proj)
      throw Error("Attention::forward: projections not set", EB_ERR_INVALID_ARGUMENT);
    const bool is_prefill = base_pos == 0 && rows > 1;
    const size_t n = is_prefill ? rows : 1;
    const Tensor q = q_proj->forward(rec, x, n);
    const Tensor k = k_proj->forward(rec, x, n);
    const Tensor v = v_proj->forward(rec, x, n);
    const Tensor o = is_prefill ? prefill(rec, q, k, v, rope, kv, layer_idx, rows)
                                : decode(rec, q, k, v, rope, kv, layer_idx, base_pos);
    return o_proj->forward(rec, o, n);
  }
  // q [seq, n_heads*hd], k/v [seq, n_kv_heads*hd] -> o [seq, n_heads*hd]
  Tensor prefill(Recorder& rec, const Tensor& q, const Tensor& k, const Tensor& v,
                 const Rope& rope, KvCache& kv, size_t layer_idx, size_t seq) const {
    const eb_attn_desc d = desc(kv);
    const eb_attn_layer l = layer(rope);
    Tensor o = Tensor::empty({seq, n_heads * head_dim}, dtype_out);
    auto ws = rec.workspace(kWsPrefill, eb_attention_prefill_workspace_bytes(&d, (int64_t)seq));
    check(eb_attention_prefill(&d, &l, (int64_t)seq, q.ptr(), k.ptr(), v.ptr(),
                               kv.k[layer_idx].ptr(), kv.v[layer_idx].ptr(), o.ptr(), ws.first,
                               ws.second, rec.stream()),
          "Attention::prefill");
    return o;
  }
  // q [1, n_heads*hd], k/v [1, n_kv_heads*hd] at position pos -> o [1, n_heads*hd]
  Tensor decode(Recorder& rec, const Tensor& q, const Tensor& k, const Tensor& v,
                const Rope& rope, KvCache& kv, size_t layer_idx, size_t pos) const {
    const eb_attn_desc d = desc(kv);
    const eb_attn_layer l = layer(rope);
    Tensor o = Tensor::empty({1, n_heads * head_dim}, dtype_out);
    // sized once for the whole cache, so the ticket counters stay zeroed
    auto ws = rec.workspace(kWsDecode,
                            eb_attention_decode_workspace_bytes(&d, 1, (int64_t)kv.max_seq - 1));
    check(eb_attention_decode(&d, &l, (int64_t)pos, q.ptr(), k.ptr(), v.ptr(),
                              kv.k[layer_idx].ptr(), kv.v[layer_idx].ptr(), o.ptr(), ws.first,
                              ws.second, rec.stream()),
          "Attention::decode");
    return o;
  }
};

}  // namespace nn
}  // namespace eyebrowse
