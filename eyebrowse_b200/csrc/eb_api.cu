// eb_api.cu -- the C ABI (include/eyebrowse_attn.h): host-side argument
// checks, workspace sizing and kernel selection. No call allocates memory.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "../../include/eyebrowse_attn.h"
#include "eb_common.cuh"
#include "eb_kernels.cuh"

static_assert(eb::kErrTimeoutTma == EB_DEVICE_ERROR_TMA && eb::kErrTimeoutMma == EB_DEVICE_ERROR_MMA &&
                  eb::kErrTimeoutSoftmax == EB_DEVICE_ERROR_SOFTMAX &&
                  eb::kErrTimeoutEpilogue == EB_DEVICE_ERROR_EPILOGUE &&
                  eb::kErrTimeoutSelftest == EB_DEVICE_ERROR_SELFTEST,
              "device error bits");

namespace eb {

// Device error word: bounded waits that give up set bits here.
__device__ unsigned g_eb_error_word;

static unsigned* error_word_ptr() {
  static unsigned* ptrs[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_eb_error_word) != cudaSuccess) {
      cudaGetLastError();  // clear the failed lookup so the next CUDA call does not report it
      return nullptr;
    }
    ptrs[dev] = static_cast<unsigned*>(p);
  }
  return ptrs[dev];
}

int device_ok() {
  static int ok_dev[64] = {};  // 0 unknown, 1 sm_100, 2 other
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (!ok_dev[dev]) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return 0;
    ok_dev[dev] = major == 10 ? 1 : 2;
  }
  return ok_dev[dev] == 1;
}

int sm_count() {
  static int cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 148;
  }
  int n = __atomic_load_n(&cache[dev], __ATOMIC_RELAXED);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      return 148;
    }
    __atomic_store_n(&cache[dev], n, __ATOMIC_RELAXED);
  }
  return n;
}

static int elem_bytes(int dt) { return dt == kF32 ? 4 : 2; }
static bool dtype_ok(int dt) { return dt == kF32 || dt == kF16 || dt == kBF16; }
static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
static constexpr float kLog2e = 1.4426950408889634f;
static constexpr size_t kAlign = 256;
static size_t round_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

static int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return EB_OK;
  if (e == cudaErrorNotSupported) return EB_ERR_UNSUPPORTED;
  cudaGetLastError();  // clear a sticky launch error
  return EB_ERR_CUDA;
}

// ---------------------------------------------------------------- decode plan
struct DecodePlan {
  int chunk, cmax;
  size_t cnt_off, ml_off, acc_off, bytes;
};

#ifndef EB_DECODE_CTAS_PER_SM
#define EB_DECODE_CTAS_PER_SM 2
#endif
// The split-K plan aims at this many CTAs (a few per SM) per decode launch.
static int64_t decode_target_ctas() { return (int64_t)EB_DECODE_CTAS_PER_SM * sm_count(); }

// Split-K workspace layout for p.cmax chunks: combine tickets, then the
// per-chunk (max, sum) pairs, then the per-chunk partial outputs.
static void decode_layout(DecodePlan& p, int64_t batch, int64_t h, int64_t hd) {
  p.cnt_off = 0;
  p.ml_off = round_up((size_t)batch * h * sizeof(unsigned));
  p.acc_off = p.ml_off + round_up((size_t)batch * h * p.cmax * 2 * sizeof(float));
  p.bytes = p.acc_off + round_up((size_t)batch * h * p.cmax * hd * sizeof(float));
}

static DecodePlan plan_decode(int64_t batch, int64_t h, int64_t hkv, int64_t hd, int dtype_cache,
                              int64_t max_pos) {
  DecodePlan p{};
  const int64_t rows = max_pos + 1;
  if (hd != 64 && hd != 128 && hd != 256) {  // SIMT path: no split
    p.chunk = (int)rows;
    p.cmax = 1;
    return p;
  }
  const int rpb = decode_rows_per_batch((int)hd, dtype_cache, (int)(h / hkv));
  const int64_t target_ctas = decode_target_ctas();
  int64_t chunk = (rows * batch * hkv + target_ctas - 1) / target_ctas;
  chunk = (chunk + rpb - 1) / rpb * rpb;
  if (chunk < rpb) chunk = rpb;
  if (chunk > 8192) chunk = 8192;
  const int64_t min_chunk = (rows + 255) / 256;  // at most 256 partials per head
  if (chunk < min_chunk) chunk = (min_chunk + rpb - 1) / rpb * rpb;
  if (chunk >= rows) {
    p.chunk = (int)rows;
    p.cmax = 1;
    return p;
  }
  p.chunk = (int)chunk;
  p.cmax = (int)((rows + chunk - 1) / chunk);
  decode_layout(p, batch, h, hd);
  return p;
}

// Workspace that covers plan_decode for EVERY context of 1..max_pos+1 rows.
// The chunk count is not monotonic in the context length (rounding the chunk
// up to whole row batches can give a shorter context more chunks), so the
// size comes from a bound on it instead of the plan at max_pos: the chunk is
// at least rows*batch*hkv/target_ctas unless capped at 8192 rows, at least
// rows/256, and at least one row batch.
static size_t decode_workspace_bound(int64_t batch, int64_t h, int64_t hkv, int64_t hd,
                                     int dtype_cache, int64_t max_pos) {
  if (hd != 64 && hd != 128 && hd != 256) return 0;
  const int64_t rows = max_pos + 1;
  const int64_t rpb = decode_rows_per_batch((int)hd, dtype_cache, (int)(h / hkv));
  const int64_t bh = batch * hkv;
  const int64_t target = decode_target_ctas();
  int64_t c = (target + bh - 1) / bh;
  c = std::max<int64_t>(c, (rows + 8191) / 8192);
  c = std::min<int64_t>(c, 256);
  c = std::min<int64_t>(c, (rows + rpb - 1) / rpb);
  if (c <= 1) return 0;
  DecodePlan p{};
  p.cmax = (int)c;
  decode_layout(p, batch, h, hd);
  return p.bytes;
}

bool desc_ok(const eb_attn_desc* d) {
  if (!d) return false;
  if (d->n_heads <= 0 || d->n_kv_heads <= 0 || d->n_heads % d->n_kv_heads) return false;
  if (d->head_dim <= 0 || d->head_dim > 256 || (d->head_dim & 1)) return false;
  if (d->max_seq <= 0) return false;
  if (!dtype_ok(d->dtype_qkv) || !dtype_ok(d->dtype_cache) || !dtype_ok(d->dtype_out)) return false;
  if (d->q_stride < 0 || d->kv_stride < 0 || d->o_stride < 0) return false;
  if (d->window < 0) return false;
  return true;
}
// A decode call at max_pos attends at most this many rows minus one: a
// sliding window caps the context the split-K plan covers.
static int64_t attended_max_pos(const eb_attn_desc* d, int64_t max_pos) {
  return d->window > 0 ? std::min<int64_t>(max_pos, (int64_t)d->window - 1) : max_pos;
}
static int64_t qs_of(const eb_attn_desc* d) {
  return d->q_stride ? d->q_stride : (int64_t)d->n_heads * d->head_dim;
}
static int64_t kvs_of(const eb_attn_desc* d) {
  return d->kv_stride ? d->kv_stride : (int64_t)d->n_kv_heads * d->head_dim;
}
static int64_t os_of(const eb_attn_desc* d) {
  return d->o_stride ? d->o_stride : (int64_t)d->n_heads * d->head_dim;
}

size_t decode_plan_bytes(const eb_attn_desc* d, int64_t batch, int64_t max_pos) {
  return plan_decode(batch, d->n_heads, d->n_kv_heads, d->head_dim, d->dtype_cache,
                     attended_max_pos(d, max_pos))
      .bytes;
}

// Chunks per (sequence, KV-head group) of the cluster-combined decode, or 0
// when the workspace kernels serve the call: 16-bit f16 caches take the
// tensor-core kernel, and the cluster kernel is used only when its grid is
// one wave (one CTA per SM, every cluster resident at once) with whole-batch
// chunks -- the latency case of a single sequence or a few. At most 16 CTAs
// per cluster.
static int cl_chunks(const eb_attn_desc* d, int64_t batch, int64_t span_pos) {
  const int group = d->n_heads / d->n_kv_heads;
  if (!decode_cl_supported(d->head_dim, d->dtype_cache) ||
      decode_tc_supported(d->head_dim, d->dtype_cache, group))
    return 0;
  const int gs = group % 8 == 0 ? 8 : group % 4 == 0 ? 4 : group % 2 == 0 ? 2 : 1;
  const int64_t groups = (int64_t)d->n_kv_heads * (group / gs) * batch;
  const int64_t rpb = decode_cl_rows_per_batch(d->head_dim, d->dtype_cache, group);
  const int64_t want = std::min<int64_t>(16, (span_pos + 1 + rpb - 1) / rpb);
  const int64_t fit = sm_count() / groups;
  // every cluster resident at once (a second wave would double the latency)
  const int64_t res = decode_cl_cluster_limit(d->head_dim, d->dtype_cache, group, groups);
  const int64_t n = std::min(std::min(want, fit), res);
  if (n < 1 || (n < want && n < 4)) return 0;
  return (int)n;
}

// Shared body of single and batched decode (also used by eb_noalloc.cu).
int decode_impl(const eb_attn_desc* d, const eb_attn_layer* L, int64_t batch,
                       const int32_t* positions, int64_t pos_scalar, int64_t max_pos,
                       const void* q, const void* k, const void* v, void* kc, void* vc,
                       int64_t cache_bstride, void* o, int64_t q_bstride, int64_t kv_bstride,
                       int64_t o_bstride, void* ws, size_t ws_bytes, cudaStream_t st,
                       const GatherSpec* gather, const int32_t* seq_idx) {
  const int hd = d->head_dim;
  const float* cos_t = L ? L->rope_cos : nullptr;
  const float* sin_t = L ? L->rope_sin : nullptr;
  if ((cos_t == nullptr) != (sin_t == nullptr)) return EB_ERR_INVALID_ARGUMENT;
  const int64_t span_pos = attended_max_pos(d, max_pos);
  DecodePlan p = plan_decode(batch, d->n_heads, d->n_kv_heads, hd, d->dtype_cache, span_pos);
  const bool vec = (hd == 64 || hd == 128 || hd == 256);
  // One wave for the whole context (a single sequence or a few): the
  // cluster-combined kernel, no workspace (see cl_chunks).
  const int n_cl = vec ? cl_chunks(d, batch, span_pos) : 0;
  if (n_cl > 0) p.cmax = 1;
  if (vec && p.cmax > 1 && (ws == nullptr || ws_bytes < p.bytes)) {
    if (ws != nullptr && ws_bytes != 0) return EB_ERR_WORKSPACE;
    p.chunk = (int)(span_pos + 1);  // no workspace: one CTA walks the whole context
    p.cmax = 1;
  }
  if (vec) {
    const int es = elem_bytes(d->dtype_cache);
    if (!aligned16(kc) || !aligned16(vc) || ((cache_bstride * es) & 15)) return EB_ERR_INVALID_ARGUMENT;
    // the new rows are read with 16-byte loads
    const int eq = elem_bytes(d->dtype_qkv);
    if (!aligned16(q) || (k && !aligned16(k)) || (v && !aligned16(v)) ||
        ((q_bstride * eq) & 15) || ((kv_bstride * eq) & 15))
      return EB_ERR_INVALID_ARGUMENT;
    if (p.cmax > 1 && ((reinterpret_cast<uintptr_t>(ws) & 255) != 0)) return EB_ERR_WORKSPACE;
    DecodeArgs a{};
    a.q = q;
    a.k_new = k;
    a.v_new = v;
    a.dtype_q = d->dtype_qkv;
    a.dtype_kv = d->dtype_qkv;
    a.dtype_o = d->dtype_out;
    a.q_bstride = q_bstride;
    a.kv_bstride = kv_bstride;
    a.o_bstride = o_bstride;
    a.kcache = kc;
    a.vcache = vc;
    a.cache_bstride = cache_bstride;
    a.o = o;
    a.q_norm_w = L ? L->q_norm_w : nullptr;
    a.k_norm_w = L ? L->k_norm_w : nullptr;
    a.v_norm_w = L ? L->v_norm_w : nullptr;
    a.cos_t = cos_t;
    a.sin_t = sin_t;
    a.positions = positions;
    a.pos_scalar = (int)pos_scalar;
    a.window = d->window;
    a.H = d->n_heads;
    a.Hkv = d->n_kv_heads;
    a.hd = hd;
    a.max_seq = d->max_seq;
    a.chunk = p.chunk;
    a.cmax = p.cmax;
    a.eps = d->eps;
    a.scale_log2 = d->scale * kLog2e;
    if (p.cmax > 1) {
      char* w = static_cast<char*>(ws);
      a.ws_cnt = reinterpret_cast<unsigned*>(w + p.cnt_off);
      a.ws_ml = reinterpret_cast<float*>(w + p.ml_off);
      a.ws_acc = reinterpret_cast<float*>(w + p.acc_off);
    }
    if (gather) {
      a.n_dst = gather->n_dst;
      a.dst_h_off = gather->h_off;
      a.dst_bstride = gather->n_heads_total * hd;
      a.seq_idx = seq_idx;
      for (int i = 0; i < gather->n_dst; i++) a.dst[i] = gather->dst[i];
    }
    a.err = error_word_ptr();
    if (!a.err) return EB_ERR_CUDA;
    if (n_cl > 0) {
      a.chunk = (int)((span_pos + 1 + n_cl - 1) / n_cl);
      a.cmax = n_cl;
      return cuda_status(launch_decode_cl(a, d->dtype_cache, (int)batch, n_cl, st));
    }
    return cuda_status(launch_decode(a, d->dtype_cache, (int)batch, st));
  }
  // SIMT path: K/V prep writes the cache row, then attention over the cache.
  if (gather) return EB_ERR_INVALID_ARGUMENT;  // head gathers need head_dim 64/128/256
  if (k) {
    PrepArgs pa{};
    pa.k = k;
    pa.v = v;
    pa.dtype_kv = d->dtype_qkv;
    pa.kv_stride = kvs_of(d);
    pa.kv_bstride = kv_bstride;
    pa.kcache = kc;
    pa.vcache = vc;
    pa.dtype_cache = d->dtype_cache;
    pa.cache_bstride = cache_bstride;
    pa.rows = 1;
    pa.hkv = d->n_kv_heads;
    pa.hd = hd;
    pa.pos0 = (int)pos_scalar;
    pa.positions = positions;
    pa.k_norm_w = L ? L->k_norm_w : nullptr;
    pa.v_norm_w = L ? L->v_norm_w : nullptr;
    pa.cos_t = cos_t;
    pa.sin_t = sin_t;
    pa.eps = d->eps;
    pa.batch = (int)batch;
    cudaError_t e = launch_prep_kv(pa, st);
    if (e != cudaSuccess) return cuda_status(e);
  }
  SimtArgs s{};
  s.q = q;
  s.dtype_q = d->dtype_qkv;
  s.q_stride = 0;
  s.q_bstride = q_bstride;
  s.k = kc;
  s.v = vc;
  s.dtype_kv = d->dtype_cache;
  s.kv_stride = (int64_t)d->n_kv_heads * hd;
  s.kv_bstride = cache_bstride;
  s.o = o;
  s.dtype_o = d->dtype_out;
  s.o_stride = 0;
  s.o_bstride = o_bstride;
  s.rows = 1;
  s.H = d->n_heads;
  s.Hkv = d->n_kv_heads;
  s.hd = hd;
  s.qpos0 = (int)pos_scalar;
  s.window = d->window;
  s.positions = positions;
  s.q_norm_w = L ? L->q_norm_w : nullptr;
  s.cos_t = cos_t;
  s.sin_t = sin_t;
  s.eps = d->eps;
  s.scale = d->scale;
  s.batch = (int)batch;
  return cuda_status(launch_attn_simt(s, st));
}

}  // namespace eb

using namespace eb;

extern "C" {

const char* eb_status_string(int status) {
  switch (status) {
    case EB_OK: return "ok";
    case EB_ERR_INVALID_ARGUMENT: return "invalid argument";
    case EB_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case EB_ERR_CUDA: return "CUDA error";
    case EB_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case EB_ERR_NO_DEVICE: return "no sm_100 device";
    case EB_ERR_DEVICE_TIMEOUT: return "a kernel's bounded wait timed out";
  }
  return "unknown status";
}

const char* eb_version(void) { return "eyebrowse-b200 0.1 (sm_100a)"; }

// ---------------------------------------------------------------- kernel-level
// Tensor-core prefill workspace: [f16 hi/lo K and V planes, when the K/V
// values are f32][the prepared query rows: one 16-bit plane, or f16 hi/lo
// planes when split].
static size_t kv_split_bytes(int64_t s, int64_t hkv, int64_t hd) {
  return round_up((size_t)4 * s * hkv * hd * sizeof(__half));
}
static size_t q_prep_bytes(int64_t s, int64_t h, int64_t hd, bool split) {
  return round_up((size_t)(split ? 2 : 1) * s * h * hd * sizeof(__half));
}
// f32 K/V at head_dim 256: the attention kernel reads the raw q rows and
// normalises, rotates and splits them itself (no q pass, no q planes).
static bool q_split_in_kernel(int64_t hd) { return hd == 256; }

size_t eb_attn_prefill_workspace_bytes(int64_t h, int64_t hkv, int64_t s, int64_t hd) {
  if (!prefill_tc_supported((int)hd) || s <= 0 || hkv <= 0 || h <= 0) return 0;
  return kv_split_bytes(s, hkv, hd) + (q_split_in_kernel(hd) ? 0 : q_prep_bytes(s, h, hd, true));
}

int eb_attn_prefill(const float* q, const float* k, const float* v, float* o, int64_t h,
                    int64_t hkv, int64_t s, int64_t hd, float scale, void* workspace,
                    size_t workspace_bytes, eb_stream_t stream) {
  if (h <= 0 || hkv <= 0 || h % hkv || hd <= 0 || hd > 256 || (hd & 1) || s < 0)
    return EB_ERR_INVALID_ARGUMENT;
  if (s == 0) return EB_OK;
  if (!q || !k || !v || !o) return EB_ERR_INVALID_ARGUMENT;
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (prefill_tc_supported((int)hd)) {
    const size_t need = eb_attn_prefill_workspace_bytes(h, hkv, s, hd);
    if (!workspace || workspace_bytes < need || !aligned16(workspace)) return EB_ERR_WORKSPACE;
    if (!aligned16(q) || !aligned16(o)) return EB_ERR_INVALID_ARGUMENT;
    PrepArgs pa{};
    pa.k = k;
    pa.v = v;
    pa.dtype_kv = kF32;
    pa.kv_stride = hkv * hd;
    pa.dtype_cache = kF32;
    pa.split = workspace;
    pa.rows = (int)s;
    pa.hkv = (int)hkv;
    pa.hd = (int)hd;
    pa.batch = 1;
    cudaError_t e = launch_prep_kv(pa, st);
    if (e != cudaSuccess) return cuda_status(e);
    // q rows -> f16 hi/lo planes (k-only prep: no norm, no RoPE here), or
    // at head_dim 256 split inside the attention kernel
    const bool qk = q_split_in_kernel(hd);
    void* qplanes = qk ? const_cast<float*>(q)
                       : static_cast<void*>(static_cast<char*>(workspace) +
                                            kv_split_bytes(s, hkv, hd));
    PrepArgs qa{};
    qa.k = q;
    qa.dtype_kv = kF32;
    qa.kv_stride = h * hd;
    qa.dtype_cache = kF32;
    qa.split = qplanes;
    qa.rows = (int)s;
    qa.hkv = (int)h;
    qa.hd = (int)hd;
    qa.batch = 1;
    if (!qk) {
      e = launch_prep_kv(qa, st);
      if (e != cudaSuccess) return cuda_status(e);
    }
    PrefillArgs a{};
    a.o = o;
    a.dtype_o = kF32;
    a.o_stride = h * hd;
    a.q_stride = h * hd;
    a.q_dtype = kF32;
    a.S = (int)s;
    a.H = (int)h;
    a.Hkv = (int)hkv;
    a.scale_log2 = scale * kLog2e;
    a.err = error_word_ptr();
    if (!a.err) return EB_ERR_CUDA;
    return cuda_status(
        launch_prefill_tc(a, (int)hd, qplanes, nullptr, nullptr, false, workspace, nullptr, st));
  }
  SimtArgs sa{};
  sa.q = q;
  sa.dtype_q = kF32;
  sa.q_stride = h * hd;
  sa.k = k;
  sa.v = v;
  sa.dtype_kv = kF32;
  sa.kv_stride = hkv * hd;
  sa.o = o;
  sa.dtype_o = kF32;
  sa.o_stride = h * hd;
  sa.rows = (int)s;
  sa.H = (int)h;
  sa.Hkv = (int)hkv;
  sa.hd = (int)hd;
  sa.scale = scale;
  sa.batch = 1;
  return cuda_status(launch_attn_simt(sa, st));
}

size_t eb_attn_decode_workspace_bytes(int64_t h, int64_t hkv, int64_t pos, int64_t hd) {
  if (h <= 0 || hkv <= 0 || pos < 0) return 0;
  return decode_workspace_bound(1, h, hkv, hd, kF32, pos);
}

size_t eb_linear_f16w_workspace_bytes(int64_t m, int64_t in_f, int64_t out_f) {
  if (m <= 0 || in_f <= 0 || out_f <= 0) return 0;
  return linear_workspace_bytes(m, in_f, out_f);
}

int eb_linear_f16w(const float* x, const void* w, float* y, int64_t m, int64_t in_f,
                   int64_t out_f, void* workspace, size_t workspace_bytes, eb_stream_t stream) {
  if (m < 0 || in_f <= 0 || out_f <= 0 || in_f > INT32_MAX || out_f > INT32_MAX ||
      (m + 127) / 128 > 65535)
    return EB_ERR_INVALID_ARGUMENT;
  if (m == 0) return EB_OK;
  if (!x || !w || !y) return EB_ERR_INVALID_ARGUMENT;
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  const LinearPath path = linear_path(m, in_f, out_f, aligned16(x) && aligned16(w) && aligned16(y));
  if (path == LinearPath::kTensor &&
      (!workspace || workspace_bytes < linear_workspace_bytes(m, in_f, out_f) ||
       (reinterpret_cast<uintptr_t>(workspace) & 255)))
    return EB_ERR_WORKSPACE;
  unsigned* err = error_word_ptr();
  if (!err) return EB_ERR_CUDA;
  return cuda_status(launch_linear(x, w, y, m, in_f, out_f, workspace, path, err,
                                   reinterpret_cast<cudaStream_t>(stream)));
}

int eb_attn_decode(const float* q, const float* kcache, const float* vcache, float* o, int64_t h,
                   int64_t hkv, int64_t pos, int64_t hd, int64_t max_seq, float scale,
                   void* workspace, size_t workspace_bytes, eb_stream_t stream) {
  if (h <= 0 || hkv <= 0 || h % hkv || hd <= 0 || hd > 256 || (hd & 1) || pos < 0 ||
      pos >= max_seq)
    return EB_ERR_INVALID_ARGUMENT;
  if (!q || !kcache || !vcache || !o) return EB_ERR_INVALID_ARGUMENT;
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  eb_attn_desc d{};
  d.n_heads = (int32_t)h;
  d.n_kv_heads = (int32_t)hkv;
  d.head_dim = (int32_t)hd;
  d.max_seq = (int32_t)max_seq;
  d.dtype_qkv = EB_F32;
  d.dtype_cache = EB_F32;
  d.dtype_out = EB_F32;
  d.scale = scale;
  return decode_impl(&d, nullptr, 1, nullptr, pos, pos, q, nullptr, nullptr,
                     const_cast<float*>(kcache), const_cast<float*>(vcache), 0, o, 0, 0, 0,
                     workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int eb_rope(const float* x, const float* cos_t, const float* sin_t, float* out, int64_t seq,
            int64_t n_heads, int64_t head_dim, int64_t base_pos, eb_stream_t stream) {
  if (seq < 0 || n_heads <= 0 || head_dim <= 0 || (head_dim & 1) || base_pos < 0)
    return EB_ERR_INVALID_ARGUMENT;
  if (seq == 0) return EB_OK;
  if (!x || !cos_t || !sin_t || !out) return EB_ERR_INVALID_ARGUMENT;
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  return cuda_status(launch_rope(x, cos_t, sin_t, out, seq, n_heads, head_dim, base_pos,
                                 reinterpret_cast<cudaStream_t>(stream)));
}

int eb_kv_write(float* cache, const float* src, int64_t hkv, int64_t count, int64_t hd,
                int64_t max_seq, int64_t dst_start, eb_stream_t stream) {
  if (hkv <= 0 || count < 0 || hd <= 0 || dst_start < 0 || dst_start + count > max_seq)
    return EB_ERR_INVALID_ARGUMENT;
  if (count == 0) return EB_OK;
  if (!cache || !src) return EB_ERR_INVALID_ARGUMENT;
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  return cuda_status(launch_kv_write(cache, src, hkv, count, hd, dst_start,
                                     reinterpret_cast<cudaStream_t>(stream)));
}

int eb_rmsnorm(const float* x, const float* weight, float* out, int64_t rows, int64_t dim,
               float eps, eb_stream_t stream) {
  if (rows < 0 || dim <= 0) return EB_ERR_INVALID_ARGUMENT;
  if (rows == 0) return EB_OK;
  if (!x || !weight || !out) return EB_ERR_INVALID_ARGUMENT;
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  return cuda_status(
      launch_rmsnorm(x, weight, out, rows, dim, eps, reinterpret_cast<cudaStream_t>(stream)));
}

int eb_rope_tables(float* cos_t, float* sin_t, int64_t max_seq, int64_t head_dim,
                   int64_t rope_angles, float theta) {
  // crates/eyebrowse-nn/src/rope.rs:24-50: f64 angles, cast to f32; pairs past
  // rope_angles keep cos = 1, sin = 0.
  if (!cos_t || !sin_t || max_seq < 0 || head_dim <= 0 || (head_dim & 1) || rope_angles < 0)
    return EB_ERR_INVALID_ARGUMENT;
  const int64_t half = head_dim / 2;
  for (int64_t i = 0; i < max_seq * half; i++) {
    cos_t[i] = 1.0f;
    sin_t[i] = 0.0f;
  }
  const double th = (double)theta, hdd = (double)head_dim;
  const int64_t n = rope_angles < half ? rope_angles : half;
  for (int64_t s = 0; s < max_seq; s++)
    for (int64_t k = 0; k < n; k++) {
      const double inv_freq = pow(th, -(2.0 * (double)k) / hdd);
      const double angle = (double)s * inv_freq;
      cos_t[s * half + k] = (float)cos(angle);
      sin_t[s * half + k] = (float)sin(angle);
    }
  return EB_OK;
}

// ---------------------------------------------------------------- fused primitive
// q rows already in the 16-bit operand type are normalised and rotated
// inside the attention kernel (no staging); others go through the row-prep
// pass into the workspace.
static bool q_fused_path(const eb_attn_desc* d) {
  return d->dtype_cache != EB_F32 && d->dtype_qkv == d->dtype_cache;
}
// f32 caches at head_dim 256: the kernel reads q in any dtype and splits it.
static bool q_fused_split(const eb_attn_desc* d) {
  return d->dtype_cache == EB_F32 && q_split_in_kernel(d->head_dim);
}

size_t eb_attention_prefill_workspace_bytes(const eb_attn_desc* d, int64_t seq) {
  if (!desc_ok(d) || seq <= 0) return 0;
  if (!prefill_tc_supported(d->head_dim)) return 0;
  const bool split = d->dtype_cache == EB_F32;
  if (q_fused_path(d)) return 0;
  return (split ? kv_split_bytes(seq, d->n_kv_heads, d->head_dim) : 0) +
         (q_fused_split(d) ? 0 : q_prep_bytes(seq, d->n_heads, d->head_dim, split));
}

// Shared argument checks of the prefill entry points.
static int prefill_check(const eb_attn_desc* d, const eb_attn_layer* L, int64_t seq, void* ws,
                         size_t ws_bytes) {
  if (!desc_ok(d) || seq < 0 || seq > d->max_seq) return EB_ERR_INVALID_ARGUMENT;
  const float* cos_t = L ? L->rope_cos : nullptr;
  const float* sin_t = L ? L->rope_sin : nullptr;
  if ((cos_t == nullptr) != (sin_t == nullptr)) return EB_ERR_INVALID_ARGUMENT;
  if (seq == 0) return EB_OK;
  if (prefill_tc_supported(d->head_dim)) {
    const size_t need = eb_attention_prefill_workspace_bytes(d, seq);
    if (need > 0 && (!ws || ws_bytes < need || !aligned16(ws))) return EB_ERR_WORKSPACE;
  }
  return EB_OK;
}

int eb_attention_prefill_kv(const eb_attn_desc* d, const eb_attn_layer* L, int64_t seq,
                            const void* k, const void* v, void* kcache, void* vcache,
                            void* workspace, size_t workspace_bytes, eb_stream_t stream) {
  int rc = prefill_check(d, L, seq, workspace, workspace_bytes);
  if (rc != EB_OK || seq == 0) return rc;
  if (!k || !v || !kcache || !vcache) return EB_ERR_INVALID_ARGUMENT;
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  const bool split = prefill_tc_supported(d->head_dim) && d->dtype_cache == EB_F32;
  PrepArgs pa{};
  pa.k = k;
  pa.v = v;
  pa.dtype_kv = d->dtype_qkv;
  pa.kv_stride = kvs_of(d);
  pa.kcache = kcache;
  pa.vcache = vcache;
  pa.dtype_cache = d->dtype_cache;
  pa.split = split ? workspace : nullptr;
  pa.rows = (int)seq;
  pa.hkv = d->n_kv_heads;
  pa.hd = d->head_dim;
  pa.k_norm_w = L ? L->k_norm_w : nullptr;
  pa.v_norm_w = L ? L->v_norm_w : nullptr;
  pa.cos_t = L ? L->rope_cos : nullptr;
  pa.sin_t = L ? L->rope_sin : nullptr;
  pa.eps = d->eps;
  pa.batch = 1;
  return cuda_status(launch_prep_kv(pa, reinterpret_cast<cudaStream_t>(stream)));
}

static_assert(EB_MAX_GATHER == kMaxGather, "gather destination limit");

// The attention half of a prefill, into o or (g != nullptr) into every
// rank's gathered buffer.
static int prefill_attend(const eb_attn_desc* d, const eb_attn_layer* L, int64_t seq,
                          const void* q, const void* kcache, const void* vcache, void* o,
                          const eb_head_gather* g, void* workspace, size_t workspace_bytes,
                          eb_stream_t stream) {
  int rc = prefill_check(d, L, seq, workspace, workspace_bytes);
  if (rc != EB_OK || seq == 0) return rc;
  if (!q || !kcache || !vcache || (!o && !g)) return EB_ERR_INVALID_ARGUMENT;
  if (g) {
    if (g->n_dst < 1 || g->n_dst > kMaxGather || g->head_offset < 0 || g->n_heads_total < 1 ||
        (int64_t)g->head_offset + d->n_heads > g->n_heads_total || !g->dst ||
        !prefill_tc_supported(d->head_dim))
      return EB_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < g->n_dst; i++)
      if (!g->dst[i] || (g->dst[i] & 15)) return EB_ERR_INVALID_ARGUMENT;
  }
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int hd = d->head_dim;
  const float* cos_t = L ? L->rope_cos : nullptr;
  const float* sin_t = L ? L->rope_sin : nullptr;
  if (prefill_tc_supported(hd)) {
    const bool split = d->dtype_cache == EB_F32;
    const int eq = elem_bytes(d->dtype_qkv), eo = elem_bytes(d->dtype_out);
    if (!aligned16(q) || !aligned16(o) || !aligned16(kcache) || !aligned16(vcache) ||
        ((qs_of(d) * eq) & 15) || ((os_of(d) * eo) & 15))
      return EB_ERR_INVALID_ARGUMENT;
    const bool fused = q_fused_path(d), fused_split = q_fused_split(d);
    // q -> RMSNorm(q_norm_w) -> RoPE -> the MMA operand type (or f16 hi/lo
    // planes), the same row transform the k rows get: inside the attention
    // kernel when q already has the operand type or the cache is f32 at
    // head_dim 256, else a row pass into the workspace
    void* qprep = (fused || fused_split)
                      ? const_cast<void*>(q)
                      : static_cast<char*>(workspace) +
                            (split ? kv_split_bytes(seq, d->n_kv_heads, hd) : 0);
    if (!fused && !fused_split) {
      PrepArgs qa{};
      qa.k = q;
      qa.dtype_kv = d->dtype_qkv;
      qa.kv_stride = qs_of(d);
      qa.kcache = split ? nullptr : qprep;
      qa.dtype_cache = d->dtype_cache;
      qa.split = split ? qprep : nullptr;
      qa.rows = (int)seq;
      qa.hkv = d->n_heads;
      qa.hd = hd;
      qa.k_norm_w = L ? L->q_norm_w : nullptr;
      qa.cos_t = cos_t;
      qa.sin_t = sin_t;
      qa.eps = d->eps;
      qa.batch = 1;
      cudaError_t e = launch_prep_kv(qa, st);
      if (e != cudaSuccess) return cuda_status(e);
    }
    PrefillArgs a{};
    a.o = o;
    a.dtype_o = d->dtype_out;
    a.o_stride = os_of(d);
    a.q_fused = fused ? 1 : 0;
    a.q_stride = qs_of(d);
    a.q_dtype = d->dtype_qkv;
    a.q_norm_w = L ? L->q_norm_w : nullptr;
    a.cos_t = cos_t;
    a.sin_t = sin_t;
    a.eps = d->eps;
    GatherSpec gs{};
    if (g) {
      a.o = nullptr;
      gs.n_dst = g->n_dst;
      gs.h_off = g->head_offset;
      gs.n_heads_total = g->n_heads_total;
      gs.dst = g->dst;
    }
    a.S = (int)seq;
    a.H = d->n_heads;
    a.Hkv = d->n_kv_heads;
    a.window = d->window;
    a.scale_log2 = d->scale * kLog2e;
    a.err = error_word_ptr();
    if (!a.err) return EB_ERR_CUDA;
    return cuda_status(launch_prefill_tc(a, hd, qprep, kcache, vcache,
                                         d->dtype_cache == EB_BF16, split ? workspace : nullptr,
                                         g ? &gs : nullptr, st));
  }
  SimtArgs s{};
  s.q = q;
  s.dtype_q = d->dtype_qkv;
  s.q_stride = qs_of(d);
  s.k = kcache;
  s.v = vcache;
  s.dtype_kv = d->dtype_cache;
  s.kv_stride = (int64_t)d->n_kv_heads * hd;
  s.o = o;
  s.dtype_o = d->dtype_out;
  s.o_stride = os_of(d);
  s.rows = (int)seq;
  s.H = d->n_heads;
  s.Hkv = d->n_kv_heads;
  s.hd = hd;
  s.window = d->window;
  s.q_norm_w = L ? L->q_norm_w : nullptr;
  s.cos_t = cos_t;
  s.sin_t = sin_t;
  s.eps = d->eps;
  s.scale = d->scale;
  s.batch = 1;
  return cuda_status(launch_attn_simt(s, st));
}

int eb_attention_prefill_attend(const eb_attn_desc* d, const eb_attn_layer* L, int64_t seq,
                                const void* q, const void* kcache, const void* vcache, void* o,
                                void* workspace, size_t workspace_bytes, eb_stream_t stream) {
  return prefill_attend(d, L, seq, q, kcache, vcache, o, nullptr, workspace, workspace_bytes,
                        stream);
}

int eb_attention_prefill_attend_gather(const eb_attn_desc* d, const eb_attn_layer* L, int64_t seq,
                                       const void* q, const void* kcache, const void* vcache,
                                       const eb_head_gather* g, void* workspace,
                                       size_t workspace_bytes, eb_stream_t stream) {
  if (!g) return EB_ERR_INVALID_ARGUMENT;
  return prefill_attend(d, L, seq, q, kcache, vcache, nullptr, g, workspace, workspace_bytes,
                        stream);
}

int eb_attention_prefill_gather(const eb_attn_desc* d, const eb_attn_layer* L, int64_t seq,
                                const void* q, const void* k, const void* v, void* kcache,
                                void* vcache, const eb_head_gather* g, void* workspace,
                                size_t workspace_bytes, eb_stream_t stream) {
  int rc = prefill_check(d, L, seq, workspace, workspace_bytes);
  if (rc != EB_OK || seq == 0) return rc;
  if (!q || !g) return EB_ERR_INVALID_ARGUMENT;
  rc = eb_attention_prefill_kv(d, L, seq, k, v, kcache, vcache, workspace, workspace_bytes,
                               stream);
  if (rc != EB_OK) return rc;
  return eb_attention_prefill_attend_gather(d, L, seq, q, kcache, vcache, g, workspace,
                                            workspace_bytes, stream);
}

int eb_attention_prefill(const eb_attn_desc* d, const eb_attn_layer* L, int64_t seq,
                         const void* q, const void* k, const void* v, void* kcache,
                         void* vcache, void* o, void* workspace, size_t workspace_bytes,
                         eb_stream_t stream) {
  int rc = prefill_check(d, L, seq, workspace, workspace_bytes);
  if (rc != EB_OK || seq == 0) return rc;
  if (!q || !o) return EB_ERR_INVALID_ARGUMENT;
  rc = eb_attention_prefill_kv(d, L, seq, k, v, kcache, vcache, workspace, workspace_bytes,
                               stream);
  if (rc != EB_OK) return rc;
  return eb_attention_prefill_attend(d, L, seq, q, kcache, vcache, o, workspace, workspace_bytes,
                                     stream);
}

size_t eb_attention_decode_workspace_bytes(const eb_attn_desc* d, int64_t batch,
                                           int64_t max_pos) {
  if (!desc_ok(d) || batch <= 0 || max_pos < 0) return 0;
  return decode_workspace_bound(batch, d->n_heads, d->n_kv_heads, d->head_dim, d->dtype_cache,
                                attended_max_pos(d, max_pos));
}

int eb_attention_decode(const eb_attn_desc* d, const eb_attn_layer* L, int64_t pos,
                        const void* q, const void* k, const void* v, void* kcache, void* vcache,
                        void* o, void* workspace, size_t workspace_bytes, eb_stream_t stream) {
  if (!desc_ok(d) || pos < 0 || pos >= d->max_seq) return EB_ERR_INVALID_ARGUMENT;
  if (!q || !k || !v || !kcache || !vcache || !o) return EB_ERR_INVALID_ARGUMENT;
  // one row each of q, k, v and o: the row strides do not apply
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  return decode_impl(d, L, 1, nullptr, pos, pos, q, k, v, kcache, vcache, 0, o, 0, 0, 0,
                     workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int eb_attention_decode_batched(const eb_attn_desc* d, const eb_attn_layer* L, int64_t batch,
                                const int32_t* positions, int64_t max_pos, const void* q,
                                const void* k, const void* v, void* kcache, void* vcache,
                                int64_t cache_batch_stride, void* o, void* workspace,
                                size_t workspace_bytes, eb_stream_t stream) {
  if (!desc_ok(d) || batch < 0 || max_pos < 0 || max_pos >= d->max_seq)
    return EB_ERR_INVALID_ARGUMENT;
  if (batch == 0) return EB_OK;
  if (!positions || !q || !k || !v || !kcache || !vcache || !o) return EB_ERR_INVALID_ARGUMENT;
  if (cache_batch_stride < (int64_t)d->max_seq * d->n_kv_heads * d->head_dim)
    return EB_ERR_INVALID_ARGUMENT;
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  // sequence b's q, k, v and o rows sit b row strides from the first
  return decode_impl(d, L, batch, positions, 0, max_pos, q, k, v, kcache, vcache,
                     cache_batch_stride, o, qs_of(d), kvs_of(d), os_of(d), workspace,
                     workspace_bytes,
                     reinterpret_cast<cudaStream_t>(stream));
}

int eb_attention_decode_batched_gather(const eb_attn_desc* d, const eb_attn_layer* L,
                                       int64_t batch, const int32_t* positions, int64_t max_pos,
                                       const void* q, const void* k, const void* v, void* kcache,
                                       void* vcache, int64_t cache_batch_stride,
                                       const eb_head_gather* g, const int32_t* seq_index,
                                       void* workspace, size_t workspace_bytes,
                                       eb_stream_t stream) {
  if (!desc_ok(d) || batch < 0 || max_pos < 0 || max_pos >= d->max_seq)
    return EB_ERR_INVALID_ARGUMENT;
  if (!g || g->n_dst < 1 || g->n_dst > kMaxGather || g->head_offset < 0 ||
      g->n_heads_total < 1 || (int64_t)g->head_offset + d->n_heads > g->n_heads_total || !g->dst)
    return EB_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < g->n_dst; i++)
    if (!g->dst[i] || (g->dst[i] & 15)) return EB_ERR_INVALID_ARGUMENT;
  if (batch == 0) return EB_OK;
  if (!positions || !q || !k || !v || !kcache || !vcache) return EB_ERR_INVALID_ARGUMENT;
  if (cache_batch_stride < (int64_t)d->max_seq * d->n_kv_heads * d->head_dim)
    return EB_ERR_INVALID_ARGUMENT;
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  GatherSpec gs{g->n_dst, g->head_offset, g->n_heads_total, g->dst};
  return decode_impl(d, L, batch, positions, 0, max_pos, q, k, v, kcache, vcache,
                     cache_batch_stride, nullptr, qs_of(d), kvs_of(d), 0, workspace,
                     workspace_bytes, reinterpret_cast<cudaStream_t>(stream), &gs, seq_index);
}

int eb_workspace_init(void* workspace, size_t workspace_bytes, eb_stream_t stream) {
  if (!workspace || workspace_bytes == 0) return EB_OK;
  return cuda_status(cudaMemsetAsync(workspace, 0, workspace_bytes,
                                     reinterpret_cast<cudaStream_t>(stream)));
}

int eb_head_concat(const void* src, void* dst, int64_t shards, int64_t rows, int64_t heads_per,
                   int64_t head_dim, int32_t dtype, eb_stream_t stream) {
  if (!src || !dst || shards <= 0 || rows < 0 || heads_per <= 0 || head_dim <= 0 || !dtype_ok(dtype))
    return EB_ERR_INVALID_ARGUMENT;
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  return cuda_status(launch_head_concat(src, dst, shards, rows, heads_per, head_dim,
                                        elem_bytes(dtype), reinterpret_cast<cudaStream_t>(stream)));
}

int eb_head_broadcast(const void* local, void* multicast, int64_t rows, int64_t n_heads_total,
                      int32_t head_offset, int32_t n_heads, int64_t head_dim, int32_t dtype,
                      eb_stream_t stream) {
  if (!local || !multicast || rows < 0 || n_heads_total <= 0 || head_offset < 0 || n_heads <= 0 ||
      head_offset + n_heads > n_heads_total || head_dim <= 0 || !dtype_ok(dtype))
    return EB_ERR_INVALID_ARGUMENT;
  const int es = elem_bytes(dtype);
  if (((head_dim * es) & 15) || !aligned16(local) || !aligned16(multicast))
    return EB_ERR_INVALID_ARGUMENT;
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  return cuda_status(launch_head_broadcast(local, multicast, rows, n_heads_total, head_offset,
                                           n_heads, head_dim, es,
                                           reinterpret_cast<cudaStream_t>(stream)));
}

int eb_selftest_wait_timeout(uint32_t timeout_us, eb_stream_t stream) {
  if (timeout_us < 1 || timeout_us > 1000000) return EB_ERR_INVALID_ARGUMENT;
  if (!device_ok()) return EB_ERR_NO_DEVICE;
  unsigned* err = error_word_ptr();
  if (!err) return EB_ERR_CUDA;
  return cuda_status(launch_wait_timeout_selftest(err, 1000ull * timeout_us,
                                                  reinterpret_cast<cudaStream_t>(stream)));
}

int eb_get_device_error(uint32_t* bits) {
  if (!bits) return EB_ERR_INVALID_ARGUMENT;
  unsigned* p = error_word_ptr();
  if (!p) return EB_ERR_CUDA;
  unsigned v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return EB_ERR_CUDA;
  if (cudaMemcpy(&v, p, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return EB_ERR_CUDA;
  const unsigned zero = 0;
  if (cudaMemcpy(p, &zero, sizeof(zero), cudaMemcpyHostToDevice) != cudaSuccess) return EB_ERR_CUDA;
  // A kernel that gave up may have left split-K tickets behind in the
  // library's own no-workspace scratch; put them back to zero for its next call.
  if (v && !noalloc_clear_tickets()) return EB_ERR_CUDA;
  *bits = v;
  return v ? EB_ERR_DEVICE_TIMEOUT : EB_OK;
}

}  // extern "C"
