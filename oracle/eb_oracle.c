/*
 * eb_oracle.c -- CPU restatement of eyebrowse's attention-path references.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path (see eb_oracle.h).
 * Build with -ffp-contract=off and without -ffast-math: the reference is Rust,
 * which neither contracts a*b+c into an FMA nor reassociates f32 sums.
 */
#include "eb_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

float orc_rel_l2(const float* a, const float* b, size_t n) {
  /* crates/eyebrowse-kernels/src/testutil.rs:16-26 */
  double num = 0.0, den = 0.0;
  for (size_t i = 0; i < n; i++) {
    double d = (double)a[i] - (double)b[i];
    num += d * d;
    den += (double)b[i] * (double)b[i];
  }
  return (float)(sqrt(num) / (sqrt(den) + 1e-12));
}

float orc_max_abs(const float* a, const float* b, size_t n) {
  float m = 0.0f;
  for (size_t i = 0; i < n; i++) {
    float d = fabsf(a[i] - b[i]);
    if (d > m || d != d) m = d;
  }
  return m;
}

/* IEEE binary16 round-to-nearest-even, the conversion the `half` crate's
 * f16::from_f32 performs (testutil.rs:62-64). */
uint16_t orc_f32_to_f16_bits(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) /* inf / nan (keep a quiet payload bit) */
    return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? (0x200u | ((ax >> 13) & 0x3ffu)) : 0u));
  if (ax >= 0x477ff000u) /* >= 65520 rounds to inf */
    return (uint16_t)(sign | 0x7c00u);
  if (ax < 0x38800000u) { /* below the smallest f16 normal 2^-14 */
    if (ax < 0x33000000u) return (uint16_t)sign; /* < 2^-25 rounds to zero */
    uint32_t e = ax >> 23;
    uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    uint32_t s = 126u - e; /* value / 2^-24 = m * 2^(e-126) */
    uint32_t q = m >> s;
    uint32_t rem = m & ((1u << s) - 1u);
    uint32_t half = 1u << (s - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t r = ax - 0x38000000u; /* rebias 127 -> 15 */
  r += 0xfffu + ((r >> 13) & 1u);
  return (uint16_t)(sign | (r >> 13));
}

float orc_f16_bits_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu;
  uint32_t x;
  if (e == 0) {
    if (m == 0) {
      x = sign;
    } else { /* subnormal: normalise */
      int sh = 0;
      while (!(m & 0x400u)) { m <<= 1; sh++; }
      m &= 0x3ffu;
      x = sign | ((uint32_t)(113 - sh) << 23) | (m << 13);
    }
  } else if (e == 31) {
    x = sign | 0x7f800000u | (m << 13);
  } else {
    x = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

void orc_round_f16(float* x, size_t n) {
  for (size_t i = 0; i < n; i++) x[i] = orc_f16_bits_to_f32(orc_f32_to_f16_bits(x[i]));
}

void orc_round_bf16(float* x, size_t n) {
  for (size_t i = 0; i < n; i++) {
    uint32_t u;
    memcpy(&u, &x[i], 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) {
      u = (u | 0x00400000u) & 0xffff0000u;
    } else {
      u += 0x7fffu + ((u >> 16) & 1u);
      u &= 0xffff0000u;
    }
    memcpy(&x[i], &u, 4);
  }
}

static void round_as(float* x, size_t n, int kind) {
  if (kind == ORC_F16) orc_round_f16(x, n);
  else if (kind == ORC_BF16) orc_round_bf16(x, n);
}

void orc_rmsnorm(const float* x, const float* w, float* out, size_t rows, size_t dim, float eps) {
  /* crates/eyebrowse-kernels/src/testutil.rs:83-97 */
  for (size_t r = 0; r < rows; r++) {
    size_t base = r * dim;
    float ss = 0.0f;
    for (size_t i = 0; i < dim; i++) ss += x[base + i] * x[base + i];
    float inv = 1.0f / sqrtf((ss / (float)dim) + eps);
    for (size_t i = 0; i < dim; i++) out[base + i] = x[base + i] * inv * w[i];
  }
}

void orc_rope(const float* x, const float* cos_t, const float* sin_t, float* out,
              size_t seq, size_t n_heads, size_t hd, size_t base_pos) {
  /* crates/eyebrowse-kernels/src/testutil.rs:101-125; table row s + base_pos as
   * in crates/eyebrowse-kernels/src/rope.rs:25-26 */
  size_t half = hd / 2;
  for (size_t s = 0; s < seq; s++) {
    for (size_t h = 0; h < n_heads; h++) {
      size_t base = (s * n_heads + h) * hd;
      size_t trow = (s + base_pos) * half;
      for (size_t p = 0; p < half; p++) {
        float c = cos_t[trow + p];
        float sn = sin_t[trow + p];
        float x1 = x[base + p];
        float x2 = x[base + half + p];
        out[base + p] = x1 * c - x2 * sn;
        out[base + half + p] = x2 * c + x1 * sn;
      }
    }
  }
}

void orc_rope_tables(float* cos_t, float* sin_t, size_t max_seq, size_t hd,
                     size_t rope_angles, float theta) {
  /* crates/eyebrowse-nn/src/rope.rs:24-50 */
  size_t half = hd / 2;
  for (size_t i = 0; i < max_seq * half; i++) { cos_t[i] = 1.0f; sin_t[i] = 0.0f; }
  double th = (double)theta;
  double hdd = (double)hd;
  size_t n = rope_angles < half ? rope_angles : half;
  for (size_t s = 0; s < max_seq; s++) {
    for (size_t k = 0; k < n; k++) {
      double inv_freq = pow(th, -(2.0 * (double)k) / hdd);
      double angle = (double)s * inv_freq;
      cos_t[s * half + k] = (float)cos(angle);
      sin_t[s * half + k] = (float)sin(angle);
    }
  }
}

void orc_kv_write(float* cache, const float* src, size_t hkv, size_t count, size_t hd,
                  size_t max_seq, size_t dst_start) {
  /* crates/eyebrowse-kernels/src/ops.rs:70-87 */
  (void)max_seq;
  for (size_t idx = 0; idx < hkv * count * hd; idx++) {
    size_t d = idx % hd;
    size_t tmp = idx / hd;
    size_t head = tmp % hkv;
    size_t c = tmp / hkv;
    cache[((dst_start + c) * hkv + head) * hd + d] = src[idx];
  }
}

/* crates/eyebrowse-kernels/src/testutil.rs:66-79 (cpu_linear): y[m, o] =
 * sum over k in order of x[m, k] * w[o, k], one f32 accumulator, multiply and
 * add rounded separately (the file is built with -ffp-contract=off). w holds
 * the f16-rounded weights as f32 (the reference rounds them with round_f16). */
void orc_linear(const float* x, const float* w, float* y, size_t m, size_t in_f, size_t out_f) {
  for (size_t i = 0; i < m; i++)
    for (size_t o = 0; o < out_f; o++) {
      float acc = 0.0f;
      for (size_t k = 0; k < in_f; k++) acc += x[i * in_f + k] * w[o * in_f + k];
      y[i * out_f + o] = acc;
    }
}

/* malloc that stops the process with a message instead of returning NULL
 * (test infrastructure: an oracle that ran out of memory has no answer). */
static void* xmalloc(size_t n) {
  void* p = malloc(n ? n : 1);
  if (!p) {
    fprintf(stderr, "eb_oracle: out of memory (%zu bytes)\n", n);
    abort();
  }
  return p;
}

/* Runs fn(arg) on the calling thread and on up to nthreads - 1 helper
 * threads. The workers share an atomic job counter, so the job completes even
 * when no helper can be started; only the helpers that started are joined. */
static void run_workers(void* (*fn)(void*), void* arg, int nthreads) {
  pthread_t* th = nthreads > 1 ? (pthread_t*)malloc(sizeof(pthread_t) * (size_t)(nthreads - 1)) : NULL;
  int started = 0;
  if (th)
    for (int t = 0; t < nthreads - 1; t++) {
      if (pthread_create(&th[started], NULL, fn, arg) != 0) break;
      started++;
    }
  fn(arg);
  for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
  free(th);
}

typedef struct {
  const float *x, *w;
  float* y;
  size_t m, in_f, out_f;
  atomic_size_t next;
} linear_job;

static void* linear_worker(void* arg) {
  linear_job* jb = (linear_job*)arg;
  for (;;) {
    /* one output row o (all m inputs) per task, same inner loop as orc_linear */
    size_t o = atomic_fetch_add(&jb->next, 1);
    if (o >= jb->out_f) break;
    for (size_t i = 0; i < jb->m; i++) {
      float acc = 0.0f;
      for (size_t k = 0; k < jb->in_f; k++) acc += jb->x[i * jb->in_f + k] * jb->w[o * jb->in_f + k];
      jb->y[i * jb->out_f + o] = acc;
    }
  }
  return NULL;
}

void orc_linear_threaded(const float* x, const float* w, float* y, size_t m, size_t in_f,
                         size_t out_f, int nthreads) {
  linear_job jb;
  jb.x = x; jb.w = w; jb.y = y; jb.m = m; jb.in_f = in_f; jb.out_f = out_f;
  atomic_init(&jb.next, 0);
  if (nthreads < 1) nthreads = 1;
  run_workers(linear_worker, &jb, nthreads);
}

/* One (query row, head) of the two-pass attention in testutil.rs:142-169.
 * `scores` has room for n_keys floats. */
static void attn_row(const float* qrow, const float* k, const float* v, float* orow,
                     size_t n_keys, size_t kv_row_stride, size_t hd, float scale,
                     float* scores) {
  float mx = -INFINITY;
  for (size_t j = 0; j < n_keys; j++) {
    const float* kr = k + j * kv_row_stride;
    float dot = 0.0f;
    for (size_t d = 0; d < hd; d++) dot += qrow[d] * kr[d];
    dot *= scale;
    scores[j] = dot;
    mx = fmaxf(mx, dot);
  }
  float sum = 0.0f;
  for (size_t j = 0; j < n_keys; j++) sum += expf(scores[j] - mx);
  for (size_t d = 0; d < hd; d++) orow[d] = 0.0f;
  for (size_t j = 0; j < n_keys; j++) {
    float w = expf(scores[j] - mx) / sum;
    const float* vr = v + j * kv_row_stride;
    for (size_t d = 0; d < hd; d++) orow[d] += w * vr[d];
  }
}

/* First key row that query row i sees. window 0: every row j <= i (the
 * reference's causal mask). window > 0: i - window < j <= i, the sliding-window
 * mask of HF transformers (masking_utils.sliding_window_causal_mask_function:
 * kv_idx > q_idx - sliding_window, and causal); the reference lists sliding
 * windows as not yet supported (README.md:25). */
static size_t window_lo(size_t i, size_t window) {
  return (window && i + 1 > window) ? i + 1 - window : 0;
}

void orc_attn_prefill_window(const float* q, const float* k, const float* v, float* o,
                             size_t h, size_t hkv, size_t s, size_t hd, float scale,
                             size_t window) {
  /* crates/eyebrowse-kernels/src/testutil.rs:130-172, keys from window_lo(i) */
  size_t group = h / hkv;
  float* scores = (float*)xmalloc(sizeof(float) * (s ? s : 1));
  for (size_t i = 0; i < s; i++) {
    size_t lo = window_lo(i, window);
    for (size_t hh = 0; hh < h; hh++) {
      size_t kvh = hh / group;
      size_t qbase = (i * h + hh) * hd;
      attn_row(q + qbase, k + (lo * hkv + kvh) * hd, v + (lo * hkv + kvh) * hd, o + qbase,
               i + 1 - lo, hkv * hd, hd, scale, scores);
    }
  }
  free(scores);
}

void orc_attn_prefill(const float* q, const float* k, const float* v, float* o,
                      size_t h, size_t hkv, size_t s, size_t hd, float scale) {
  orc_attn_prefill_window(q, k, v, o, h, hkv, s, hd, scale, 0);
}

typedef struct {
  const float *q, *k, *v;
  float* o;
  size_t h, hkv, s, hd, row_begin, row_end, head_begin, head_end, window;
  float scale;
  atomic_size_t next;
} prefill_job;

static void* prefill_worker(void* arg) {
  prefill_job* jb = (prefill_job*)arg;
  size_t group = jb->h / jb->hkv;
  float* scores = (float*)xmalloc(sizeof(float) * (jb->s ? jb->s : 1));
  for (;;) {
    /* rows handed out longest-first so the causal triangle balances */
    size_t t = atomic_fetch_add(&jb->next, 1);
    if (t >= jb->row_end - jb->row_begin) break;
    size_t i = jb->row_end - 1 - t;
    size_t lo = window_lo(i, jb->window);
    for (size_t hh = jb->head_begin; hh < jb->head_end; hh++) {
      size_t kvh = hh / group;
      size_t qbase = (i * jb->h + hh) * jb->hd;
      size_t kbase = (lo * jb->hkv + kvh) * jb->hd;
      attn_row(jb->q + qbase, jb->k + kbase, jb->v + kbase, jb->o + qbase, i + 1 - lo,
               jb->hkv * jb->hd, jb->hd, jb->scale, scores);
    }
  }
  free(scores);
  return NULL;
}

void orc_attn_prefill_part(const float* q, const float* k, const float* v, float* o,
                           size_t h, size_t hkv, size_t s, size_t hd, float scale,
                           size_t row_begin, size_t row_end, size_t head_begin,
                           size_t head_end, int nthreads, size_t window) {
  prefill_job jb;
  jb.q = q; jb.k = k; jb.v = v; jb.o = o;
  jb.h = h; jb.hkv = hkv; jb.s = s; jb.hd = hd; jb.window = window;
  jb.row_begin = row_begin; jb.row_end = row_end;
  jb.head_begin = head_begin; jb.head_end = head_end;
  jb.scale = scale;
  atomic_init(&jb.next, 0);
  if (nthreads < 1) nthreads = 1;
  run_workers(prefill_worker, &jb, nthreads);
}

void orc_attn_decode_window(const float* q, const float* kc, const float* vc, float* o,
                            size_t h, size_t hkv, size_t pos, size_t hd, size_t max_seq,
                            float scale, size_t window) {
  /* crates/eyebrowse-kernels/src/testutil.rs:177-218, cache rows from window_lo(pos) */
  (void)max_seq;
  size_t group = h / hkv;
  size_t lo = window_lo(pos, window);
  float* scores = (float*)xmalloc(sizeof(float) * (pos + 1));
  for (size_t hh = 0; hh < h; hh++) {
    size_t kvh = hh / group;
    size_t qbase = hh * hd;
    size_t kbase = (lo * hkv + kvh) * hd;
    attn_row(q + qbase, kc + kbase, vc + kbase, o + qbase, pos + 1 - lo, hkv * hd, hd, scale,
             scores);
  }
  free(scores);
}

void orc_attn_decode(const float* q, const float* kc, const float* vc, float* o,
                     size_t h, size_t hkv, size_t pos, size_t hd, size_t max_seq, float scale) {
  orc_attn_decode_window(q, kc, vc, o, h, hkv, pos, hd, max_seq, scale, 0);
}

typedef struct {
  const float *q, *kc, *vc;
  float* o;
  const int32_t* pos;
  size_t batch, h, hkv, hd, max_seq, cache_stride, window;
  float scale;
  atomic_size_t next;
} decode_job;

static void* decode_worker(void* arg) {
  decode_job* jb = (decode_job*)arg;
  size_t group = jb->h / jb->hkv;
  float* scores = (float*)xmalloc(sizeof(float) * jb->max_seq);
  for (;;) {
    size_t t = atomic_fetch_add(&jb->next, 1);
    if (t >= jb->batch * jb->h) break;
    size_t b = t / jb->h, hh = t % jb->h;
    size_t kvh = hh / group;
    size_t qbase = (b * jb->h + hh) * jb->hd;
    const size_t lo = window_lo((size_t)jb->pos[b], jb->window);
    const size_t kbase = b * jb->cache_stride + (lo * jb->hkv + kvh) * jb->hd;
    attn_row(jb->q + qbase, jb->kc + kbase, jb->vc + kbase, jb->o + qbase,
             (size_t)jb->pos[b] + 1 - lo, jb->hkv * jb->hd, jb->hd, jb->scale, scores);
  }
  free(scores);
  return NULL;
}

void orc_attn_decode_batched(const float* q, const float* kc, const float* vc, float* o,
                             size_t batch, const int32_t* pos, size_t h, size_t hkv,
                             size_t hd, size_t max_seq, size_t cache_stride, float scale,
                             int nthreads, size_t window) {
  decode_job jb;
  jb.window = window;
  jb.q = q; jb.kc = kc; jb.vc = vc; jb.o = o; jb.pos = pos;
  jb.batch = batch; jb.h = h; jb.hkv = hkv; jb.hd = hd; jb.max_seq = max_seq;
  jb.cache_stride = cache_stride; jb.scale = scale;
  atomic_init(&jb.next, 0);
  if (nthreads < 1) nthreads = 1;
  run_workers(decode_worker, &jb, nthreads);
}

static float* dup(const float* x, size_t n) {
  float* y = (float*)xmalloc(sizeof(float) * (n ? n : 1));
  memcpy(y, x, sizeof(float) * n);
  return y;
}

void orc_attention_prefill(const float* q, const float* k, const float* v,
                           const float* q_norm_w, const float* k_norm_w, const float* v_norm_w,
                           float eps, const float* cos_t, const float* sin_t,
                           float* kcache, float* vcache, float* o,
                           size_t seq, size_t h, size_t hkv, size_t hd, size_t max_seq,
                           float scale, int cache_round, int q_round, size_t window) {
  /* crates/eyebrowse-nn/src/attention.rs:49-117, after the projections (:58-60) */
  float* qn = dup(q, seq * h * hd);
  float* kn = dup(k, seq * hkv * hd);
  float* vn = dup(v, seq * hkv * hd);
  if (q_norm_w) orc_rmsnorm(qn, q_norm_w, qn, seq * h, hd, eps);   /* :62-65 */
  if (k_norm_w) orc_rmsnorm(kn, k_norm_w, kn, seq * hkv, hd, eps); /* :66-69 */
  if (v_norm_w) orc_rmsnorm(vn, v_norm_w, vn, seq * hkv, hd, eps); /* :70-73 */
  if (cos_t) {                                                     /* :75-76 */
    orc_rope(qn, cos_t, sin_t, qn, seq, h, hd, 0);
    orc_rope(kn, cos_t, sin_t, kn, seq, hkv, hd, 0);
  }
  round_as(kn, seq * hkv * hd, cache_round);
  round_as(vn, seq * hkv * hd, cache_round);
  round_as(qn, seq * h * hd, q_round);
  orc_kv_write(kcache, kn, hkv, seq, hd, max_seq, 0); /* :78-87 */
  orc_kv_write(vcache, vn, hkv, seq, hd, max_seq, 0); /* :88-97 */
  orc_attn_prefill_window(qn, kn, vn, o, h, hkv, seq, hd, scale, window); /* :104-115 */
  free(qn); free(kn); free(vn);
}

void orc_attention_decode(const float* q, const float* k, const float* v,
                          const float* q_norm_w, const float* k_norm_w, const float* v_norm_w,
                          float eps, const float* cos_t, const float* sin_t,
                          float* kcache, float* vcache, float* o,
                          size_t pos, size_t h, size_t hkv, size_t hd, size_t max_seq,
                          float scale, int cache_round, size_t window) {
  /* crates/eyebrowse-nn/src/attention.rs:120-185, after the projections (:129-131) */
  float* qn = dup(q, h * hd);
  float* kn = dup(k, hkv * hd);
  float* vn = dup(v, hkv * hd);
  if (q_norm_w) orc_rmsnorm(qn, q_norm_w, qn, h, hd, eps);   /* :133-136 */
  if (k_norm_w) orc_rmsnorm(kn, k_norm_w, kn, hkv, hd, eps); /* :137-140 */
  if (v_norm_w) orc_rmsnorm(vn, v_norm_w, vn, hkv, hd, eps); /* :141-144 */
  if (cos_t) {                                               /* :146-147 */
    orc_rope(qn, cos_t, sin_t, qn, 1, h, hd, pos);
    orc_rope(kn, cos_t, sin_t, kn, 1, hkv, hd, pos);
  }
  round_as(kn, hkv * hd, cache_round);
  round_as(vn, hkv * hd, cache_round);
  orc_kv_write(kcache, kn, hkv, 1, hd, max_seq, pos); /* :149-168 */
  orc_kv_write(vcache, vn, hkv, 1, hd, max_seq, pos);
  orc_attn_decode_window(qn, kcache, vcache, o, h, hkv, pos, hd, max_seq, scale,
                         window); /* :171-183 */
  free(qn); free(kn); free(vn);
}
