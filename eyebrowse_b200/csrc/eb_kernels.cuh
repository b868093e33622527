// eb_kernels.cuh -- argument blocks and launchers shared between the kernel
// translation units and the C-ABI layer (eb_api.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/eyebrowse_attn.h"

namespace eb {

// Destinations of a head gather (prefill and decode): at most this many
// buffers, this GPU's and its peers'.
constexpr int kMaxGather = 8;

// ------------------------------------------------------------- small kernels
cudaError_t launch_rope(const float* x, const float* cos_t, const float* sin_t, float* out,
                        int64_t seq, int64_t n_heads, int64_t hd, int64_t base_pos,
                        cudaStream_t st);
cudaError_t launch_kv_write(float* cache, const float* src, int64_t hkv, int64_t count, int64_t hd,
                            int64_t dst_start, cudaStream_t st);
cudaError_t launch_rmsnorm(const float* x, const float* w, float* out, int64_t rows, int64_t dim,
                           float eps, cudaStream_t st);
cudaError_t launch_head_concat(const void* src, void* dst, int64_t shards, int64_t rows,
                               int64_t heads_per, int64_t hd, int elem_bytes, cudaStream_t st);
cudaError_t launch_head_broadcast(const void* local, void* mc, int64_t rows, int64_t h_total,
                                  int64_t h0, int64_t nh, int64_t hd, int elem_bytes,
                                  cudaStream_t st);

// K/V preparation for a run of rows: k -> RMSNorm(k_norm_w) -> RoPE(row pos0+r),
// v -> RMSNorm(v_norm_w); written to the cache rows [dst0, dst0+rows) in the
// cache dtype, and (split != nullptr) as f16 hi/lo planes for the tensor-core
// path: split = [khi | klo | vhi | vlo], each rows*hkv*hd halves, of the values
// as stored (cache-rounded). batch > 1 handles `batch` sequences, each with
// its own position (positions[b]) and cache (cache + b*cache_bstride).
// v == nullptr prepares k rows only (split = [khi | klo]): the query rows of a
// prefill go through this path (q_norm_w as k_norm_w, hkv = query heads).
struct PrepArgs {
  const void* k;
  const void* v;
  int dtype_kv;
  int64_t kv_stride;   // elements between rows of k/v
  int64_t kv_bstride;  // elements between sequences of k/v
  void* kcache;
  void* vcache;
  int dtype_cache;
  int64_t cache_bstride;
  void* split;         // f16 planes or nullptr
  int rows, hkv, hd;
  int pos0;                  // position of row 0 (prefill 0)
  const int32_t* positions;  // per-sequence position (overrides pos0) or nullptr
  const float* k_norm_w;
  const float* v_norm_w;
  const float* cos_t;
  const float* sin_t;
  float eps;
  int batch;
};
cudaError_t launch_prep_kv(const PrepArgs& a, cudaStream_t st);

// Generic SIMT attention (any even head_dim <= 256): one warp per (query row,
// query head); the q row is normalised/rotated inline. Query row i of
// sequence b has position qpos0 + i (or positions[b] for decode), attends
// key rows 0..=that position of k/v.
struct SimtArgs {
  const void* q;
  int dtype_q;
  int64_t q_stride, q_bstride;
  const void* k;
  const void* v;
  int dtype_kv;
  int64_t kv_stride, kv_bstride;
  void* o;
  int dtype_o;
  int64_t o_stride, o_bstride;
  int rows, H, Hkv, hd;
  int qpos0;
  int window;  // > 0: sliding window (keys pos - window < j <= pos)
  const int32_t* positions;
  const float* q_norm_w;
  const float* cos_t;
  const float* sin_t;
  float eps, scale;
  int batch;
};
cudaError_t launch_attn_simt(const SimtArgs& a, cudaStream_t st);

// ------------------------------------------------------------- decode
struct DecodeArgs {
  const void* q;       // [B][H][hd] (row = head), dtype_q
  const void* k_new;   // [B][Hkv][hd] or nullptr (no cache write)
  const void* v_new;
  int dtype_q, dtype_kv, dtype_o;
  int64_t q_bstride, kv_bstride, o_bstride;  // elements between sequences
  void* kcache;
  void* vcache;
  int64_t cache_bstride;
  void* o;
  const float* q_norm_w;
  const float* k_norm_w;
  const float* v_norm_w;
  const float* cos_t;
  const float* sin_t;
  const int32_t* positions;  // device, per sequence; nullptr -> pos_scalar
  int pos_scalar;
  int window;          // > 0: rows pos - window < j <= pos only
  int H, Hkv, hd, chunk, cmax;
  int max_seq;         // cache rows per sequence (tensor-map extent)
  float eps, scale_log2;
  float* ws_ml;        // [B][H][cmax] x (m, l)
  float* ws_acc;       // [B][H][cmax][hd]
  unsigned* ws_cnt;    // [B][Hkv] tickets
  unsigned* err;
  // Head gather (n_dst > 0): instead of o, sequence b's rows go to row
  // seq_idx[b] (b if null), heads dst_h_off + h, of every buffer dst[i]
  // [rows][heads][hd] in dtype_o, dst_bstride elements per row
  // (eb_decode_out.cuh).
  int n_dst;
  int dst_h_off;
  int64_t dst_bstride;
  const int32_t* seq_idx;
  uint64_t dst[kMaxGather];
};
// Returns cudaErrorNotSupported when (hd, cache dtype) has no vector kernel.
cudaError_t launch_decode(const DecodeArgs& a, int dtype_cache, int batch, cudaStream_t st);
int decode_rows_per_batch(int hd, int dtype_cache, int group);
// ------------------------------------------------------------- linear_f16w (eb_linear.cu)
// y [m, out] = x [m, in] (f32) * w [out, in]^T (f16), f32 accumulation.
enum class LinearPath { kScalar, kRows, kTensor };
// kRows for m <= 8, kTensor (tcgen05, needs workspace) above; kScalar when k
// is not a multiple of 8, a pointer is not 16-byte aligned, or (kTensor) out
// is not a multiple of 4.
LinearPath linear_path(int64_t m, int64_t in_f, int64_t out_f, bool aligned);
size_t linear_workspace_bytes(int64_t m, int64_t in_f, int64_t out_f);
cudaError_t launch_linear(const float* x, const void* w, float* y, int64_t m, int64_t in_f,
                          int64_t out_f, void* ws, LinearPath path, unsigned* err,
                          cudaStream_t st);

// Latency decode for f32/bf16 caches (eb_decode_cl.cu): n_chunks (1..16)
// CTAs per (sequence, KV-head group) form a cluster and merge through
// distributed shared memory; no workspace. a.chunk = rows per CTA.
bool decode_cl_supported(int hd, int dtype_cache);
int decode_cl_rows_per_batch(int hd, int dtype_cache, int group);
// The largest cluster size (16, 8, 4, 2, 1; 0 if none) at which `clusters`
// clusters of the latency decode kernel are all resident at once.
int decode_cl_cluster_limit(int hd, int dtype_cache, int group, int64_t clusters);
cudaError_t launch_decode_cl(const DecodeArgs& a, int dtype_cache, int batch, int n_chunks,
                             cudaStream_t st);
// tcgen05 decode for 16-bit caches (eb_decode_tc.cu)
bool decode_tc_supported(int hd, int dtype_cache, int group);
cudaError_t launch_decode_tc(const DecodeArgs& a, int dtype_cache, int batch, cudaStream_t st);
// Shared body of the decode entry points, defined in eb_api.cu: validates
// the workspace against the split-K plan and launches the decode kernels.
int decode_impl(const eb_attn_desc* d, const eb_attn_layer* L, int64_t batch,
                const int32_t* positions, int64_t pos_scalar, int64_t max_pos, const void* q,
                const void* k, const void* v, void* kc, void* vc, int64_t cache_bstride, void* o,
                int64_t q_bstride, int64_t kv_bstride, int64_t o_bstride, void* ws, size_t ws_bytes,
                cudaStream_t st, const struct GatherSpec* gather = nullptr,
                const int32_t* seq_idx = nullptr);
// Workspace bytes the split-K plan of one decode call at max_pos needs (0 when
// it does not split), defined in eb_api.cu.
size_t decode_plan_bytes(const eb_attn_desc* d, int64_t batch, int64_t max_pos);
// Host-side checks shared by every entry point, defined in eb_api.cu: the
// descriptor's shape, dtype codes, strides and window are valid; the current
// device is an sm_100 part.
bool desc_ok(const eb_attn_desc* d);
int device_ok();
// Streaming multiprocessors of the current device (cached per device); 148,
// a B200's count, when no device is current (host-only calls, e.g. workspace
// sizing on a machine without a GPU). Grids and split-K plans scale with it.
int sm_count();
// Zeroes the split-K tickets of eb_attention_decode_noalloc's scratch on the
// current device (synchronously); false if a CUDA call failed. Defined in
// eb_noalloc.cu.
bool noalloc_clear_tickets();
// One-CTA kernel whose bounded wait (nothing ever arrives) gives up after
// timeout_ns and sets kErrTimeoutSelftest in *err. Defined in eb_selftest.cu.
cudaError_t launch_wait_timeout_selftest(unsigned* err, unsigned long long timeout_ns,
                                         cudaStream_t st);

// ------------------------------------------------------------- prefill (tcgen05)
struct PrefillArgs {
  void* o;
  int dtype_o;
  int64_t o_stride;  // elements between output rows
  int S, H, Hkv;
  int window;  // > 0: key j is visible to query row i iff i - window < j <= i
  float scale_log2;
  unsigned* err;
  // Head gather (n_dst > 0): o is unused; head h of row i goes to row i,
  // head h_off + h of every destination buffer [S][H_total][hd], stored by
  // TMA through the destination tensor maps passed beside the arguments.
  int n_dst;
  int h_off;
  // Query rows transformed inside the kernel (q_fused != 0): q16 is the raw
  // q [S][H][hd] in the operand type with rows q_stride elements apart; each
  // tile's rows are normalised (q_norm_w, if non-null) and rotated (cos_t /
  // sin_t [*, hd/2], if non-null) in shared memory after their TMA load,
  // with the row-prep pass's f32 arithmetic. Otherwise q16 holds rows the
  // row-prep pass already transformed.
  int q_fused;
  int64_t q_stride;
  const float* q_norm_w;
  const float* cos_t;
  const float* sin_t;
  float eps;
  // f32 caches at head_dim 256: the raw query rows [S][H][hd] (q_dtype,
  // rows q_stride elements apart), which the softmax threads normalise,
  // rotate and split into tensor memory (hi) and shared memory (lo).
  const void* q_raw;
  int q_dtype;
  // set by the launcher: the RoPE table rows come by TMA (tmCos / tmSin)
  int tab_smem;
};
// Destinations of a head gather: up to kMaxGather buffers [S][H_total][hd]
// in the output dtype (this GPU's and its peers', mapped here).
struct GatherSpec {
  int n_dst;
  int h_off;
  int64_t n_heads_total;
  const uint64_t* dst;  // host array of n_dst device addresses
};
// q16: the prepared query rows [S][H][hd] in the MMA operand type (RMSNorm +
// RoPE already applied by launch_prep_kv), or their f16 hi/lo planes when
// split. k16/v16: 16-bit K/V rows [S][Hkv][hd] (the cache when it is
// f16/bf16). split: f16 hi/lo K/V planes when the cache is f32 (k16/v16
// unused then).
cudaError_t launch_prefill_tc(const PrefillArgs& a, int hd, const void* q16, const void* k16,
                              const void* v16, bool bf16, const void* split,
                              const GatherSpec* gather, cudaStream_t st);
bool prefill_tc_supported(int hd);

}  // namespace eb
