/*
 * eyebrowse_attn.h -- C ABI of the B200 (sm_100a) attention path for eyebrowse.
 *
 * Plain C types only (bindgen-clean). Every pointer argument named as a tensor
 * is a CUDA device pointer unless stated otherwise. Every call is
 * asynchronous on `stream` (NULL = the legacy default stream) and returns an
 * eb_status; argument errors are detected on the host before any launch.
 * The caller owns all memory. The library allocates no memory in any call;
 * scratch memory comes in through `workspace` arguments.
 *
 * Layouts follow the reference (seq-major):
 *   q [seq, n_heads, head_dim]; k, v [seq, n_kv_heads, head_dim];
 *   KV cache [max_seq, n_kv_heads, head_dim]
 *   (crates/eyebrowse-nn/src/kv_cache.rs:9-49);
 *   RoPE tables cos, sin [max_seq, head_dim/2] f32 (crates/eyebrowse-nn/src/rope.rs:18-50).
 * Query head h reads KV head h / (n_heads / n_kv_heads)
 * (crates/eyebrowse-kernels/src/attention.rs:26-27).
 */
#ifndef EYEBROWSE_ATTN_H
#define EYEBROWSE_ATTN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define EB_API __attribute__((visibility("default")))
#else
#define EB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t. */
typedef struct CUstream_st* eb_stream_t;

typedef enum {
  EB_OK = 0,
  EB_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad shape, pos >= max_seq, h % hkv != 0 ... */
  EB_ERR_UNSUPPORTED = 2,      /* valid for the reference, not built here (e.g. odd head_dim) */
  EB_ERR_CUDA = 3,             /* a CUDA runtime call failed (launch, attribute, symbol) */
  EB_ERR_WORKSPACE = 4,        /* workspace missing, misaligned or smaller than required */
  EB_ERR_NO_DEVICE = 5,        /* no sm_100 device current */
  EB_ERR_DEVICE_TIMEOUT = 6    /* a kernel's bounded wait gave up (see eb_get_device_error) */
} eb_status;

typedef enum { EB_F32 = 0, EB_F16 = 1, EB_BF16 = 2 } eb_dtype;

/* Human-readable name of a status code. */
EB_API const char* eb_status_string(int status);

/* Library version string. */
EB_API const char* eb_version(void);

/* ------------------------------------------------------------------------ *
 * Kernel-level free functions: one-to-one drop-ins for eyebrowse-kernels
 * (crates/eyebrowse-kernels/src/lib.rs:15-19). All tensors f32, as in the
 * reference; sizes are the reference's usize arguments.
 * ------------------------------------------------------------------------ */

/* Causal GQA attention over full sequences, q [s,h,hd], k/v [s,hkv,hd] -> o [s,h,hd].
 * Replaces attn_prefill (crates/eyebrowse-kernels/src/attention.rs:94-120).
 * head_dim 64/128/256 runs on tcgen05 tensor cores (f32 operands split into
 * f16 hi/lo pairs, staged with the q rows in eb_attn_prefill_workspace_bytes
 * of workspace); other even head_dim up to 256 run a SIMT kernel and need no
 * workspace. */
EB_API int eb_attn_prefill(const float* q, const float* k, const float* v, float* o, int64_t h,
                    int64_t hkv, int64_t s, int64_t hd, float scale, void* workspace,
                    size_t workspace_bytes, eb_stream_t stream);
EB_API size_t eb_attn_prefill_workspace_bytes(int64_t h, int64_t hkv, int64_t s, int64_t hd);

/* Single decode step: q [h,hd] attends rows 0..=pos of kcache/vcache [max_seq,hkv,hd].
 * Replaces attn_decode (crates/eyebrowse-kernels/src/attention.rs:124-162).
 * With workspace (eb_attn_decode_workspace_bytes, zeroed once by
 * eb_workspace_init) the context is split across CTAs (split-K); with
 * workspace == NULL one CTA per KV head walks the whole context. */
EB_API int eb_attn_decode(const float* q, const float* kcache, const float* vcache, float* o,
                   int64_t h, int64_t hkv, int64_t pos, int64_t hd, int64_t max_seq, float scale,
                   void* workspace, size_t workspace_bytes, eb_stream_t stream);
EB_API size_t eb_attn_decode_workspace_bytes(int64_t h, int64_t hkv, int64_t pos, int64_t hd);

/* Half-split rotary embedding, x/out [seq, n_heads, head_dim], table row s + base_pos.
 * Replaces rope (crates/eyebrowse-kernels/src/rope.rs:38-69). out may equal x. */
EB_API int eb_rope(const float* x, const float* cos_t, const float* sin_t, float* out, int64_t seq,
            int64_t n_heads, int64_t head_dim, int64_t base_pos, eb_stream_t stream);

/* Write src [count, hkv, hd] into cache [max_seq, hkv, hd] at row dst_start.
 * Replaces kv_write (crates/eyebrowse-kernels/src/ops.rs:150-179). */
EB_API int eb_kv_write(float* cache, const float* src, int64_t hkv, int64_t count, int64_t hd,
                int64_t max_seq, int64_t dst_start, eb_stream_t stream);

/* RMSNorm over rows of [rows, dim]: out = x / sqrt(mean(x^2) + eps) * weight.
 * Replaces rmsnorm (crates/eyebrowse-kernels/src/rmsnorm.rs:42-64). */
EB_API int eb_rmsnorm(const float* x, const float* weight, float* out, int64_t rows, int64_t dim,
               float eps, eb_stream_t stream);

/* Host function (no device work): RoPE tables computed in f64 and cast to f32,
 * pairs k >= rope_angles pass through (cos 1, sin 0). cos_t/sin_t are HOST
 * arrays of max_seq*head_dim/2 floats.
 * Replaces Rope::build / Rope::build_partial (crates/eyebrowse-nn/src/rope.rs:18-50). */
EB_API int eb_rope_tables(float* cos_t, float* sin_t, int64_t max_seq, int64_t head_dim,
                   int64_t rope_angles, float theta);

/* ------------------------------------------------------------------------ *
 * The projections around the path: linear_f16w
 * (crates/eyebrowse-kernels/src/matmul.rs:128-149), the GEMM of eyebrowse-nn
 * Linear::forward (crates/eyebrowse-nn/src/linear.rs:17-22).
 * y [m, out_f] = x [m, in_f] (f32) * w [out_f, in_f]^T with w f16 in the HF
 * layout (the reference's packed-u32 f16 pairs are the same bytes) and f32
 * accumulation. m <= 8 streams w once (HBM-bound); larger m runs on the
 * tensor cores with x split into f16 hi/lo planes, which needs
 * eb_linear_f16w_workspace_bytes of workspace (256-byte aligned) and
 * |x| < 65504. A fused projection is one call over concatenated weights:
 * w = [Wq; Wk; Wv] gives rows [q | k | v] that eb_attention_* read in place
 * (q = y, k = y + n_heads*head_dim, v = k + n_kv_heads*head_dim,
 * q_stride = kv_stride = out_f).
 * ------------------------------------------------------------------------ */
EB_API size_t eb_linear_f16w_workspace_bytes(int64_t m, int64_t in_f, int64_t out_f);
EB_API int eb_linear_f16w(const float* x, const void* w, float* y, int64_t m, int64_t in_f,
                          int64_t out_f, void* workspace, size_t workspace_bytes,
                          eb_stream_t stream);

/* ------------------------------------------------------------------------ *
 * The fused attention primitive: the body of eyebrowse-nn Attention::prefill
 * and Attention::decode between the projections and o_proj
 * (crates/eyebrowse-nn/src/attention.rs:62-115 and :133-183): optional
 * per-head q/k/v RMSNorm, full or partial RoPE, the KV-cache write and the
 * attention, in one pass over q/k/v.
 * ------------------------------------------------------------------------ */
typedef struct {
  int32_t n_heads;     /* query heads (this GPU's share when heads are sharded) */
  int32_t n_kv_heads;  /* KV heads; n_heads % n_kv_heads == 0 */
  int32_t head_dim;    /* even, <= 256; 64/128/256 take the tensor-core / vector paths */
  int32_t max_seq;     /* rows of the cache and of the RoPE tables */
  int32_t dtype_qkv;   /* eb_dtype of q, k, v (projection outputs) */
  int32_t dtype_cache; /* eb_dtype of the KV cache */
  int32_t dtype_out;   /* eb_dtype of o */
  int32_t q_stride;    /* elements between consecutive rows of q; 0 = n_heads*head_dim */
  int32_t kv_stride;   /* elements between consecutive rows of k and v; 0 = n_kv_heads*head_dim */
  int32_t o_stride;    /* elements between consecutive rows of o; 0 = n_heads*head_dim */
  float eps;           /* RMSNorm epsilon (Config rms_eps) */
  float scale;         /* softmax scale (1/sqrt(head_dim), or 1.0 for Gemma 4) */
  int32_t window;      /* sliding window (Gemma local layers): query row i sees key rows
                          j with i - window < j <= i; 0 = the whole causal context */
} eb_attn_desc;

/* Optional per-layer inputs; any NULL pointer disables that step. */
typedef struct {
  const float* q_norm_w; /* [head_dim] (Attention.q_norm) */
  const float* k_norm_w; /* [head_dim] (Attention.k_norm) */
  const float* v_norm_w; /* [head_dim] (Attention.v_norm; Gemma 4 passes ones) */
  const float* rope_cos; /* [max_seq, head_dim/2] (Rope.cos), NULL = no rotation */
  const float* rope_sin; /* [max_seq, head_dim/2] (Rope.sin) */
} eb_attn_layer;

/* Prefill of `seq` rows at positions 0..seq-1 (Attention::prefill,
 * crates/eyebrowse-nn/src/attention.rs:49-117): normalises and rotates q/k,
 * normalises v, writes k/v to cache rows [0, seq) and computes causal GQA
 * attention into o [seq, n_heads, head_dim]. head_dim 64/128/256 (tensor
 * cores) stage the prepared q rows, and the f16 hi/lo planes of an f32
 * cache, in eb_attention_prefill_workspace_bytes of workspace. */
EB_API int eb_attention_prefill(const eb_attn_desc* desc, const eb_attn_layer* layer, int64_t seq,
                         const void* q, const void* k, const void* v, void* kcache,
                         void* vcache, void* o, void* workspace, size_t workspace_bytes,
                         eb_stream_t stream);
EB_API size_t eb_attention_prefill_workspace_bytes(const eb_attn_desc* desc, int64_t seq);

/* The two halves of eb_attention_prefill, for callers that schedule them
 * separately (eb_attention_prefill = _kv then _attend on one stream, same
 * workspace).
 * _kv: k -> RMSNorm -> RoPE, v -> RMSNorm, written to cache rows [0, seq)
 * (Attention::prefill's norms, rope and kv_write, attention.rs:62-97).
 * _attend: q -> RMSNorm -> RoPE (a row pass into the workspace), then the
 * causal attention over cache rows [0, seq) (attention.rs:62-76, :104-115). */
EB_API int eb_attention_prefill_kv(const eb_attn_desc* desc, const eb_attn_layer* layer,
                                   int64_t seq, const void* k, const void* v, void* kcache,
                                   void* vcache, void* workspace, size_t workspace_bytes,
                                   eb_stream_t stream);
EB_API int eb_attention_prefill_attend(const eb_attn_desc* desc, const eb_attn_layer* layer,
                                       int64_t seq, const void* q, const void* kcache,
                                       const void* vcache, void* o, void* workspace,
                                       size_t workspace_bytes, eb_stream_t stream);

/* Head-sharded prefill with the gather fused into the attention kernel: the
 * kernel of the rank that owns heads [head_offset, head_offset + n_heads)
 * stores each finished output tile straight into the gathered [seq,
 * n_heads_total, head_dim] buffer of every rank (TMA stores over NVLink, at
 * most EB_MAX_GATHER buffers), so no all-gather + eb_head_concat follows. The
 * tiles leave as they finish, while the rest of the kernel runs.
 *   dst: HOST array of n_dst device addresses, each rank's gathered buffer
 *        in desc->dtype_out as mapped in this process (peer memory),
 *        16-byte aligned.
 * Nothing else may write those buffers during the call. The caller orders
 * this call after every rank's last read of its buffer, and every rank's
 * reads after every rank's call (a cross-GPU barrier before and after).
 * Head dims other than 64/128/256 are not supported here
 * (EB_ERR_INVALID_ARGUMENT). No reference counterpart: it is the multi-GPU
 * split by KV-head group. */
#define EB_MAX_GATHER 8
typedef struct eb_head_gather {
  int32_t n_dst;
  int32_t head_offset;
  int64_t n_heads_total;
  const uint64_t* dst;
} eb_head_gather;

EB_API int eb_attention_prefill_gather(const eb_attn_desc* desc, const eb_attn_layer* layer,
                                       int64_t seq, const void* q, const void* k, const void* v,
                                       void* kcache, void* vcache, const eb_head_gather* gather,
                                       void* workspace, size_t workspace_bytes,
                                       eb_stream_t stream);
EB_API int eb_attention_prefill_attend_gather(const eb_attn_desc* desc,
                                              const eb_attn_layer* layer, int64_t seq,
                                              const void* q, const void* kcache,
                                              const void* vcache, const eb_head_gather* gather,
                                              void* workspace, size_t workspace_bytes,
                                              eb_stream_t stream);

/* One decode step at position pos (Attention::decode,
 * crates/eyebrowse-nn/src/attention.rs:120-185): q [n_heads, head_dim],
 * k/v [n_kv_heads, head_dim] are the projection outputs of the new token; the
 * processed k/v are written to cache row pos and attention runs over rows
 * 0..=pos (the last `window` of them with a sliding window) into
 * o [n_heads, head_dim]. One row each: the descriptor's row strides do not
 * apply. q, k and v start on 16-byte boundaries. */
EB_API int eb_attention_decode(const eb_attn_desc* desc, const eb_attn_layer* layer, int64_t pos,
                        const void* q, const void* k, const void* v, void* kcache, void* vcache,
                        void* o, void* workspace, size_t workspace_bytes, eb_stream_t stream);

/* Batched decode: `batch` sequences, each with its own cache at
 * kcache + b*cache_batch_stride elements (same for vcache) and its own
 * position positions[b] (DEVICE array of int32, every value < max_seq and
 * <= max_pos). q/o are [batch, n_heads, head_dim]; k/v [batch, n_kv_heads,
 * head_dim], with sequence b's rows b * q_stride / kv_stride / o_stride
 * elements from the first (16-byte multiples for q, k and v). No reference
 * counterpart: the reference decodes one sequence. */
EB_API int eb_attention_decode_batched(const eb_attn_desc* desc, const eb_attn_layer* layer,
                                int64_t batch, const int32_t* positions, int64_t max_pos,
                                const void* q, const void* k, const void* v, void* kcache,
                                void* vcache, int64_t cache_batch_stride, void* o,
                                void* workspace, size_t workspace_bytes, eb_stream_t stream);

/* Batched decode of a multi-GPU shard with the gather fused into the kernel:
 * instead of writing o, the kernel stores each finished output row (head h
 * of local sequence b) into every rank's gathered buffer [rows,
 * n_heads_total, head_dim] (dtype_out) at row seq_index[b] (b when seq_index
 * is NULL; a DEVICE array of int32 below that buffer's row count) and head
 * head_offset + h -- plain stores over NVLink into the peers' buffers, so no
 * all-gather and no concat follow. The gather's dst and head_offset mean
 * what they mean for eb_attention_prefill_gather, and the same barriers
 * apply: nothing else writes the buffers during the call, and every rank's
 * reads of a buffer are ordered around every rank's call. Head dims other
 * than 64/128/256 are not supported here (EB_ERR_INVALID_ARGUMENT). Other
 * arguments as eb_attention_decode_batched. No reference counterpart: it is
 * the multi-GPU split of batched decode by KV-head group and by sequence. */
EB_API int eb_attention_decode_batched_gather(const eb_attn_desc* desc, const eb_attn_layer* layer,
                                              int64_t batch, const int32_t* positions,
                                              int64_t max_pos, const void* q, const void* k,
                                              const void* v, void* kcache, void* vcache,
                                              int64_t cache_batch_stride,
                                              const eb_head_gather* gather,
                                              const int32_t* seq_index, void* workspace,
                                              size_t workspace_bytes, eb_stream_t stream);

/* Workspace for eb_attention_decode(_batched) with contexts up to max_pos+1
 * rows: one workspace of this size serves every call with pos (or the
 * batched max_pos) <= max_pos. 0 means no such call needs one. */
EB_API size_t eb_attention_decode_workspace_bytes(const eb_attn_desc* desc, int64_t batch,
                                           int64_t max_pos);

/* Zero a decode workspace once after allocating it: the split-K combine
 * counters it holds must start at zero (each call leaves them at zero).
 * Calls that share one workspace must not overlap on the GPU. */
EB_API int eb_workspace_init(void* workspace, size_t workspace_bytes, eb_stream_t stream);

/* Size in bytes of the device scratch eb_attention_decode_noalloc owns on
 * every GPU that loads this library. */
#define EB_NOALLOC_SCRATCH_BYTES (8u << 20)

/* eb_attention_decode without a workspace argument, for callers that cannot
 * allocate device memory: a plugin inside a host framework that owns the
 * whole device pool and hands the plugin only its inputs and outputs, or a
 * serving loop that must never call into an allocator between steps. No
 * counterpart in the reference (its kernels need no scratch).
 * The split-K scratch is a fixed EB_NOALLOC_SCRATCH_BYTES array inside this
 * library, held by every GPU that loads it until the process exits. A call
 * whose split-K plan at pos needs more is refused with EB_ERR_WORKSPACE before
 * any device work (never one with eb_attention_decode_workspace_bytes(desc,
 * 1, pos) <= EB_NOALLOC_SCRATCH_BYTES). The call allocates nothing; its first call on a device
 * looks up the array's device address (cudaGetSymbolAddress), so make that
 * first call before any stream capture. All calls on a device share the one
 * array: calls that overlap on the GPU (other streams, other threads) race
 * and corrupt each other's results; serialise them. The array keeps the last
 * call's contents; its split-K tickets, which must start at zero, are zero
 * when the library loads and every completed call leaves them at zero. A
 * call whose kernel gave up (see eb_get_device_error) can leave them set:
 * eb_get_device_error zeroes them when it reports such a failure. Same
 * arguments, argument checks and results as eb_attention_decode otherwise. */
EB_API int eb_attention_decode_noalloc(const eb_attn_desc* desc, const eb_attn_layer* layer,
                                       int64_t pos, const void* q, const void* k, const void* v,
                                       void* kcache, void* vcache, void* o, eb_stream_t stream);

/* Head-concat after a head-sharded step: src holds G shards [G][rows][heads_per][hd]
 * (as an all-gather leaves them), dst is [rows][G*heads_per][hd]. dtype is eb_dtype. */
EB_API int eb_head_concat(const void* src, void* dst, int64_t shards, int64_t rows, int64_t heads_per,
                   int64_t head_dim, int32_t dtype, eb_stream_t stream);

/* The other exchange at the head-concat boundary, for many GPUs: copies rows
 * x heads [head_offset, head_offset + n_heads) of this rank's gathered buffer
 * `local` [rows, n_heads_total, head_dim] through `multicast`, an NVLink
 * multicast address bound to every rank's gathered buffer (same offsets):
 * each 16-byte word leaves this GPU once (multimem.st) and the switch writes
 * it into every rank's buffer. A rank first writes its own heads into its
 * own buffer (eb_attention_prefill_gather with n_dst = 1), then calls this;
 * the same barriers as for eb_attention_prefill_gather apply.
 * head_dim * element size must be a multiple of 16 bytes. */
EB_API int eb_head_broadcast(const void* local, void* multicast, int64_t rows,
                             int64_t n_heads_total, int32_t head_offset, int32_t n_heads,
                             int64_t head_dim, int32_t dtype, eb_stream_t stream);

/* Returns and clears the device-side error word of the current device: a
 * non-zero value means some kernel's bounded wait gave up (the kernel then
 * returned early and its output is invalid). Synchronises the device. When
 * it reports a failure it also zeroes the split-K tickets in the scratch of
 * eb_attention_decode_noalloc. (A caller workspace shared by the failed call
 * needs eb_workspace_init again.) */
EB_API int eb_get_device_error(uint32_t* bits);
/* Bits of the device error word: the role whose bounded wait gave up. */
#define EB_DEVICE_ERROR_TMA (1u << 0)      /* a TMA producer (load ring slot or drain) */
#define EB_DEVICE_ERROR_MMA (1u << 1)      /* an MMA issuer (operands, P, its own commits) */
#define EB_DEVICE_ERROR_SOFTMAX (1u << 2)  /* a softmax / online-softmax thread */
#define EB_DEVICE_ERROR_EPILOGUE (1u << 3) /* an epilogue (final accumulator, output stores) */

/* Checks the failure path of the kernels' bounded waits on this device: a
 * one-CTA kernel waits on a barrier that nothing completes, gives up after
 * timeout_us microseconds (1 .. 1e6), sets bit EB_DEVICE_ERROR_SELFTEST in
 * the device error word and returns. No fault, no hang: the context stays
 * usable, and eb_get_device_error then reports (and clears) the bit. No
 * counterpart in the reference (its kernels have no waits). */
#define EB_DEVICE_ERROR_SELFTEST (1u << 5)
EB_API int eb_selftest_wait_timeout(uint32_t timeout_us, eb_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* EYEBROWSE_ATTN_H */
