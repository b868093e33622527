/*
 * eb_oracle.h -- CPU restatement of eyebrowse's attention-path references.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker the parity tests, the
 * smoke check and bench.py's CPU-baseline leg compare the CUDA path against.
 * The product library (eyebrowse_b200) never links, loads or calls it.
 *
 * Every function restates one reference function, cited as
 * `crate-relative path:line` inside the eyebrowse workspace, keeping its loop
 * order and its f32 arithmetic (built with -ffp-contract=off so that
 * `a*b + c` is two roundings, as in Rust).
 *
 * Deviation from the reference, for all attention functions: `scale` is an
 * argument. The reference's CPU attention hard-codes 1/sqrt(head_dim)
 * (crates/eyebrowse-kernels/src/testutil.rs:140, :188) while its kernels and
 * the `Attention` primitive take the scale as a parameter
 * (crates/eyebrowse-kernels/src/attention.rs:104, crates/eyebrowse-models/src/gemma4.rs:216).
 */
#ifndef EB_ORACLE_H
#define EB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ||a-b|| / (||b|| + 1e-12), accumulated in f64.
 * crates/eyebrowse-kernels/src/testutil.rs:16-26 */
float orc_rel_l2(const float* a, const float* b, size_t n);

/* max_i |a_i - b_i| (helper for the stated max-abs tolerance; no reference counterpart). */
float orc_max_abs(const float* a, const float* b, size_t n);

/* Round-to-nearest-even through IEEE binary16 and back, in place.
 * crates/eyebrowse-kernels/src/testutil.rs:62-64 (half::f16::from_f32 / to_f32). */
void orc_round_f16(float* x, size_t n);
/* Same through bfloat16 (round-to-nearest-even). No reference counterpart: the
 * reference is f32-only; used to model a bf16 cache. */
void orc_round_bf16(float* x, size_t n);
uint16_t orc_f32_to_f16_bits(float x);
float orc_f16_bits_to_f32(uint16_t h);

/* RMSNorm over rows of [rows, dim]: out = x * (1/sqrt(sum(x^2)/dim + eps)) * w.
 * crates/eyebrowse-kernels/src/testutil.rs:83-97 (same as eyebrowse-nn/src/tests.rs:14-28). */
void orc_rmsnorm(const float* x, const float* w, float* out, size_t rows, size_t dim, float eps);

/* Half-split RoPE on x [seq, n_heads, hd] with table rows (s + base_pos).
 * crates/eyebrowse-kernels/src/testutil.rs:101-125, with base_pos as in the
 * kernel crates/eyebrowse-kernels/src/rope.rs:25-26. out may alias x. */
void orc_rope(const float* x, const float* cos_t, const float* sin_t, float* out,
              size_t seq, size_t n_heads, size_t hd, size_t base_pos);

/* RoPE tables cos/sin [max_seq, hd/2] computed in f64 then cast to f32; pairs
 * k >= rope_angles get cos=1, sin=0.
 * crates/eyebrowse-nn/src/rope.rs:24-50 (build = build_partial with rope_angles = hd/2). */
void orc_rope_tables(float* cos_t, float* sin_t, size_t max_seq, size_t hd,
                     size_t rope_angles, float theta);

/* Scatter src [count, hkv, hd] into cache [max_seq, hkv, hd] at row dst_start.
 * crates/eyebrowse-kernels/src/ops.rs:70-87 (WGSL index arithmetic, :84-85). */
void orc_kv_write(float* cache, const float* src, size_t hkv, size_t count, size_t hd,
                  size_t max_seq, size_t dst_start);

/* Linear layer, HF layout w [out_f, in_f]: y [m, out_f] = x w^T.
 * crates/eyebrowse-kernels/src/testutil.rs:66-79 (cpu_linear), the CPU
 * reference of linear_f16w (matmul.rs:128-149) with f16-rounded w. */
void orc_linear(const float* x, const float* w, float* y, size_t m, size_t in_f, size_t out_f);

/* orc_linear spread over `nthreads` POSIX threads by output feature, with the
 * identical inner loop (bit-identical results). Used by the timed CPU
 * baseline. */
void orc_linear_threaded(const float* x, const float* w, float* y, size_t m, size_t in_f,
                         size_t out_f, int nthreads);

/* Causal GQA attention, seq-major: q [s,h,hd], k/v [s,hkv,hd] -> o [s,h,hd].
 * crates/eyebrowse-kernels/src/testutil.rs:130-172 (two-pass softmax, f32 dot
 * accumulated over d in order, then *= scale). */
void orc_attn_prefill(const float* q, const float* k, const float* v, float* o,
                      size_t h, size_t hkv, size_t s, size_t hd, float scale);

/* orc_attn_prefill with a sliding window: row i attends key rows j with
 * i - window < j <= i (HF transformers' sliding-window causal mask; no
 * counterpart in the reference, which defers sliding windows). window 0 is
 * orc_attn_prefill. */
void orc_attn_prefill_window(const float* q, const float* k, const float* v, float* o,
                             size_t h, size_t hkv, size_t s, size_t hd, float scale,
                             size_t window);

/* Same computation restricted to query rows [row_begin,row_end) and query heads
 * [head_begin,head_end), spread over `nthreads` POSIX threads (parallel over
 * (row, head) with the identical inner loop). Used by the timed CPU baseline. */
void orc_attn_prefill_part(const float* q, const float* k, const float* v, float* o,
                           size_t h, size_t hkv, size_t s, size_t hd, float scale,
                           size_t row_begin, size_t row_end, size_t head_begin,
                           size_t head_end, int nthreads, size_t window);

/* Single decode step: q [h,hd] attends rows 0..=pos of caches [max_seq,hkv,hd].
 * crates/eyebrowse-kernels/src/testutil.rs:177-218. */
void orc_attn_decode(const float* q, const float* kc, const float* vc, float* o,
                     size_t h, size_t hkv, size_t pos, size_t hd, size_t max_seq, float scale);

/* orc_attn_decode over cache rows pos - window < j <= pos (window 0: all). */
void orc_attn_decode_window(const float* q, const float* kc, const float* vc, float* o,
                            size_t h, size_t hkv, size_t pos, size_t hd, size_t max_seq,
                            float scale, size_t window);

/* Batched decode baseline: `batch` independent decode steps, sequence b using
 * q + b*h*hd, caches + b*cache_stride, position pos[b]; parallel over
 * (sequence, head) with `nthreads` threads. Same inner loop as orc_attn_decode. */
void orc_attn_decode_batched(const float* q, const float* kc, const float* vc, float* o,
                             size_t batch, const int32_t* pos, size_t h, size_t hkv,
                             size_t hd, size_t max_seq, size_t cache_stride, float scale,
                             int nthreads, size_t window);

/* Storage-rounding model for the composite functions below (no reference
 * counterpart: the reference stores f32 only). 0 = f32, 1 = f16, 2 = bf16. */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2 };

/* The attention part of Attention::prefill (crates/eyebrowse-nn/src/attention.rs:49-117)
 * from the projection outputs on: q/k/v RMSNorm when a weight is given (:62-74),
 * RoPE at base 0 (:75-76), kv_write of post-RoPE k and post-norm v at row 0
 * (:78-97), causal attention over the fresh k/v (:104-115), within `window`
 * rows when window > 0 (see orc_attn_prefill_window).
 * q [seq,h,hd], k/v [seq,hkv,hd]; caches [max_seq,hkv,hd]; o [seq,h,hd].
 * cos/sin NULL skips RoPE. cache_round rounds the stored k/v (and the k/v the
 * attention reads, which equal the stored rows); q_round rounds the post-RoPE q
 * the attention reads. */
void orc_attention_prefill(const float* q, const float* k, const float* v,
                           const float* q_norm_w, const float* k_norm_w, const float* v_norm_w,
                           float eps, const float* cos_t, const float* sin_t,
                           float* kcache, float* vcache, float* o,
                           size_t seq, size_t h, size_t hkv, size_t hd, size_t max_seq,
                           float scale, int cache_round, int q_round, size_t window);

/* The attention part of Attention::decode (crates/eyebrowse-nn/src/attention.rs:120-185):
 * norms (:133-144), RoPE at base_pos = pos (:146-147), kv_write at row pos
 * (:149-168), attention over cache rows 0..=pos (:171-183).
 * q [h,hd], k/v [hkv,hd]; caches [max_seq,hkv,hd] updated in place; o [h,hd]. */
void orc_attention_decode(const float* q, const float* k, const float* v,
                          const float* q_norm_w, const float* k_norm_w, const float* v_norm_w,
                          float eps, const float* cos_t, const float* sin_t,
                          float* kcache, float* vcache, float* o,
                          size_t pos, size_t h, size_t hkv, size_t hd, size_t max_seq,
                          float scale, int cache_round, size_t window);

#ifdef __cplusplus
}
#endif
#endif /* EB_ORACLE_H */
