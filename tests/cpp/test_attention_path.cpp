// Parity tests of the C++ host mirror (eyebrowse_b200/host/eyebrowse.hpp),
// ported from the reference's own unit tests with their names, inputs and
// tolerances:
//   attn_prefill_matches_cpu, attn_decode_matches_cpu
//       crates/eyebrowse-kernels/src/attention.rs:175-230
//   rope_matches_cpu            crates/eyebrowse-kernels/src/rope.rs:93-111
//   rmsnorm_matches_cpu         crates/eyebrowse-kernels/src/rmsnorm.rs:73-93
//   kv_write_places_rows        crates/eyebrowse-kernels/src/ops.rs:272-292
//   rope_build_tables           crates/eyebrowse-nn/src/tests.rs:152-176
//   prefill_decode_consistency  crates/eyebrowse-nn/src/tests.rs:181-244
//   linear_f16w_matches_cpu     crates/eyebrowse-kernels/src/matmul.rs:261-279
//       (here from the projection outputs on, with the same prng seeds)
// plus tensor-core-sized cases at the north-star tolerance and the error
// behaviour. The CPU side is the C oracle (oracle/eb_oracle.c), the
// restatement of the reference's testutil.rs.
//
// Build: tests/cpp/Makefile. Run: test_attention_path [--list]. Exit status =
// number of failed tests.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <functional>
#include <string>
#include <vector>

#include "../../eyebrowse_b200/host/eyebrowse.hpp"
#include "../../oracle/eb_oracle.h"

using namespace eyebrowse;

namespace {

struct Fail : std::runtime_error {
  using std::runtime_error::runtime_error;
};
#define CHECK(cond, msg)                                                              \
  do {                                                                                \
    if (!(cond)) throw Fail(std::string(msg) + " (" #cond ", line " + std::to_string(__LINE__) + ")"); \
  } while (0)

std::vector<float> ramp(size_t n, float off, float step) {
  std::vector<float> v(n);
  for (size_t i = 0; i < n; i++) v[i] = off + (float)i * step;
  return v;
}

// crates/eyebrowse-nn/src/testutil.rs:30-41 (xorshift64, values in [-1, 1))
std::vector<float> prng(size_t n, uint64_t seed) {
  uint64_t s = seed + 0x9E3779B97F4A7C15ull;
  std::vector<float> out(n);
  for (size_t i = 0; i < n; i++) {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    const double u = (double)(s >> 11) / (double)(1ull << 53);
    out[i] = (float)(u * 2.0 - 1.0);
  }
  return out;
}

float rel_l2(const std::vector<float>& a, const std::vector<float>& b) {
  return orc_rel_l2(a.data(), b.data(), a.size());
}
float max_abs(const std::vector<float>& a, const std::vector<float>& b) {
  return orc_max_abs(a.data(), b.data(), a.size());
}

// ------------------------------------------------------------ ported tests
void attn_prefill_matches_cpu() {
  const size_t h = 2, hkv = 1, s = 5, hd = 8;
  auto q = ramp(h * s * hd, -0.5f, 0.011f);
  auto k = ramp(hkv * s * hd, -0.3f, 0.007f);
  auto v = ramp(hkv * s * hd, 0.2f, 0.013f);
  auto qt = Tensor::from_f32({s, h, hd}, q), kt = Tensor::from_f32({s, hkv, hd}, k),
       vt = Tensor::from_f32({s, hkv, hd}, v);
  auto ot = Tensor::empty({s, h, hd});
  Recorder rec;
  kernels::attn_prefill(rec, qt, kt, vt, ot, h, hkv, s, hd, 1.0f / std::sqrt((float)hd));
  rec.submit();
  auto got = ot.to_f32();
  std::vector<float> want(got.size());
  orc_attn_prefill(q.data(), k.data(), v.data(), want.data(), h, hkv, s, hd,
                   1.0f / std::sqrt((float)hd));
  CHECK(rel_l2(got, want) < 1e-4f, "rel_l2 too high");
}

void attn_decode_matches_cpu() {
  const size_t h = 4, hkv = 2, hd = 8, max_seq = 16, pos = 5;
  auto q = ramp(h * hd, -0.4f, 0.02f);
  auto kc = ramp(hkv * max_seq * hd, -0.2f, 0.005f);
  auto vc = ramp(hkv * max_seq * hd, 0.1f, 0.009f);
  auto qt = Tensor::from_f32({h, hd}, q);
  auto kt = Tensor::from_f32({max_seq, hkv, hd}, kc), vt = Tensor::from_f32({max_seq, hkv, hd}, vc);
  auto ot = Tensor::empty({h, hd});
  Recorder rec;
  kernels::attn_decode(rec, qt, kt, vt, ot, h, hkv, pos, hd, max_seq, 1.0f / std::sqrt((float)hd));
  rec.submit();
  auto got = ot.to_f32();
  std::vector<float> want(got.size());
  orc_attn_decode(q.data(), kc.data(), vc.data(), want.data(), h, hkv, pos, hd, max_seq,
                  1.0f / std::sqrt((float)hd));
  CHECK(rel_l2(got, want) < 1e-4f, "rel_l2 too high");
}

void rope_matches_cpu() {
  const size_t seq = 4, n_heads = 2, hd = 8;
  const float theta = 10000.0f;
  std::vector<float> cos(seq * hd / 2), sin(seq * hd / 2);
  orc_rope_tables(cos.data(), sin.data(), seq, hd, hd / 2, theta);
  std::vector<float> x(seq * n_heads * hd);
  for (size_t i = 0; i < x.size(); i++) x[i] = (float)i * 0.03f - 0.5f;
  auto xt = Tensor::from_f32({seq, n_heads, hd}, x);
  auto ct = Tensor::from_f32({seq, hd / 2}, cos), st = Tensor::from_f32({seq, hd / 2}, sin);
  auto ot = Tensor::empty({seq, n_heads, hd});
  Recorder rec;
  kernels::rope(rec, xt, ct, st, ot, seq, n_heads, hd, 0);
  rec.submit();
  auto got = ot.to_f32();
  std::vector<float> want(got.size());
  orc_rope(x.data(), cos.data(), sin.data(), want.data(), seq, n_heads, hd, 0);
  CHECK(rel_l2(got, want) < 1e-5f, "rel_l2 too high");
}

void rmsnorm_matches_cpu() {
  const size_t rows = 3, dim = 320;  // dim > 256 exercises a strided reduction
  const float eps = 1e-6f;
  std::vector<float> x(rows * dim), w(dim);
  for (size_t i = 0; i < x.size(); i++) x[i] = (float)(i % 17) * 0.05f - 0.4f;
  for (size_t i = 0; i < dim; i++) w[i] = 1.0f + (float)i * 0.001f;
  auto xt = Tensor::from_f32({rows, dim}, x), wt = Tensor::from_f32({dim}, w);
  auto ot = Tensor::empty({rows, dim});
  Recorder rec;
  kernels::rmsnorm(rec, xt, wt, ot, rows, dim, eps);
  rec.submit();
  auto got = ot.to_f32();
  std::vector<float> want(got.size());
  orc_rmsnorm(x.data(), w.data(), want.data(), rows, dim, eps);
  CHECK(rel_l2(got, want) < 1e-4f, "rel_l2 too high");
}

void kv_write_places_rows() {
  const size_t hkv = 2, hd = 4, max_seq = 8;
  auto ct = Tensor::from_f32({max_seq, hkv, hd}, std::vector<float>(max_seq * hkv * hd, 0.f));
  std::vector<float> src(hkv * hd);
  for (size_t i = 0; i < src.size(); i++) src[i] = (float)i + 1.0f;
  auto st = Tensor::from_f32({1, hkv, hd}, src);
  Recorder rec;
  kernels::kv_write(rec, ct, st, hkv, 1, hd, max_seq, 3);
  rec.submit();
  auto got = ct.to_f32();
  for (size_t head = 0; head < hkv; head++)
    for (size_t d = 0; d < hd; d++)
      CHECK(got[(3 * hkv + head) * hd + d] == src[head * hd + d], "row 3 holds src");
  CHECK(got[0] == 0.0f, "position 0 was never written");
}

void rope_build_tables() {
  const size_t max_seq = 8, hd = 4, half = hd / 2;
  const float theta = 10000.0f;
  auto rope = nn::Rope::build(max_seq, hd, theta);
  auto cos = rope.cos.to_f32(), sin = rope.sin.to_f32();
  for (size_t k = 0; k < half; k++) {
    CHECK(std::fabs(cos[k] - 1.0f) < 1e-6f, "row 0 cos == 1");
    CHECK(std::fabs(sin[k]) < 1e-6f, "row 0 sin == 0");
  }
  const size_t s = 3;
  for (size_t k = 0; k < half; k++) {
    const double inv_freq = std::pow((double)theta, -(2.0 * (double)k) / (double)hd);
    const double angle = (double)s * inv_freq;
    CHECK(std::fabs(cos[s * half + k] - (float)std::cos(angle)) < 1e-5f, "cos row 3");
    CHECK(std::fabs(sin[s * half + k] - (float)std::sin(angle)) < 1e-5f, "sin row 3");
  }
}

// Decode fed one token at a time agrees with prefill at the last position:
// cache layout, RoPE base_pos and the decode path match prefill. The
// reference runs the projections first; here q/k/v are the projection
// outputs, drawn with the same prng.
void prefill_decode_consistency() {
  const size_t n_heads = 4, n_kv_heads = 2, head_dim = 4, seq = 3, max_seq = 8;
  const size_t q_dim = n_heads * head_dim, kv_dim = n_kv_heads * head_dim;
  nn::Attention attn;
  attn.q_norm = Tensor::from_f32({head_dim}, prng(head_dim, 15));
  attn.k_norm = Tensor::from_f32({head_dim}, prng(head_dim, 16));
  attn.n_heads = n_heads;
  attn.n_kv_heads = n_kv_heads;
  attn.head_dim = head_dim;
  attn.scale = 1.0f / std::sqrt((float)head_dim);
  auto rope = nn::Rope::build(max_seq, head_dim, 10000.0f);
  auto q = prng(seq * q_dim, 11), k = prng(seq * kv_dim, 12), v = prng(seq * kv_dim, 13);

  auto kv_p = nn::KvCache::create(1, max_seq, n_kv_heads, head_dim);
  Recorder rec;
  auto pre = attn.prefill(rec, Tensor::from_f32({seq, q_dim}, q), Tensor::from_f32({seq, kv_dim}, k),
                          Tensor::from_f32({seq, kv_dim}, v), rope, kv_p, 0, seq);
  rec.submit();
  auto pre_out = pre.to_f32();
  std::vector<float> o_pre_last(pre_out.end() - q_dim, pre_out.end());

  auto kv_d = nn::KvCache::create(1, max_seq, n_kv_heads, head_dim);
  std::vector<float> last;
  for (size_t pos = 0; pos < seq; pos++) {
    auto row = [&](const std::vector<float>& x, size_t w) {
      return Tensor::from_f32({1, w}, std::vector<float>(x.begin() + pos * w, x.begin() + (pos + 1) * w));
    };
    auto out = attn.decode(rec, row(q, q_dim), row(k, kv_dim), row(v, kv_dim), rope, kv_d, 0, pos);
    rec.submit();
    last = out.to_f32();
  }
  CHECK(rel_l2(last, o_pre_last) < 2e-3f, "prefill/decode rel_l2");
  // the caches agree too (same rows written by either path)
  CHECK(rel_l2(kv_p.k[0].to_f32(), kv_d.k[0].to_f32()) < 1e-6f, "k cache");
  CHECK(rel_l2(kv_p.v[0].to_f32(), kv_d.v[0].to_f32()) < 1e-6f, "v cache");
}

// ------------------------------------------------------------ beyond the reference
// Tensor-core sizes (head_dim 128) at the north-star tolerance.
void attn_prefill_tensor_core_hd128() {
  const size_t h = 16, hkv = 8, s = 200, hd = 128;
  auto q = prng(h * s * hd, 21), k = prng(hkv * s * hd, 22), v = prng(hkv * s * hd, 23);
  auto ot = Tensor::empty({s, h, hd});
  Recorder rec;
  const float scale = 1.0f / std::sqrt((float)hd);
  kernels::attn_prefill(rec, Tensor::from_f32({s, h, hd}, q), Tensor::from_f32({s, hkv, hd}, k),
                        Tensor::from_f32({s, hkv, hd}, v), ot, h, hkv, s, hd, scale);
  rec.submit();
  auto got = ot.to_f32();
  std::vector<float> want(got.size());
  orc_attn_prefill(q.data(), k.data(), v.data(), want.data(), h, hkv, s, hd, scale);
  CHECK(max_abs(got, want) <= 2e-3f && rel_l2(got, want) <= 1e-3f, "north-star tolerance");
}

void attention_decode_long_context_hd128() {
  const size_t n_heads = 16, n_kv_heads = 8, hd = 128, max_seq = 3000, pos = 2999;
  nn::Attention attn;
  attn.q_norm = Tensor::from_f32({hd}, std::vector<float>(hd, 1.f));
  attn.k_norm = Tensor::from_f32({hd}, std::vector<float>(hd, 1.f));
  attn.n_heads = n_heads;
  attn.n_kv_heads = n_kv_heads;
  attn.head_dim = hd;
  attn.scale = 1.0f / std::sqrt((float)hd);
  auto rope = nn::Rope::build(max_seq, hd, 1e6f);
  auto kc = prng(max_seq * n_kv_heads * hd, 31), vc = prng(max_seq * n_kv_heads * hd, 32);
  auto kv = nn::KvCache::create(1, max_seq, n_kv_heads, hd);
  kv.k[0] = Tensor::from_f32({max_seq, n_kv_heads, hd}, kc);
  kv.v[0] = Tensor::from_f32({max_seq, n_kv_heads, hd}, vc);
  auto q = prng(n_heads * hd, 33), k = prng(n_kv_heads * hd, 34), v = prng(n_kv_heads * hd, 35);
  Recorder rec;
  auto o = attn.decode(rec, Tensor::from_f32({1, n_heads * hd}, q),
                       Tensor::from_f32({1, n_kv_heads * hd}, k),
                       Tensor::from_f32({1, n_kv_heads * hd}, v), rope, kv, 0, pos);
  rec.submit();
  auto got = o.to_f32();
  auto cos = rope.cos.to_f32(), sin = rope.sin.to_f32();
  std::vector<float> ones(hd, 1.f), want(n_heads * hd);
  orc_attention_decode(q.data(), k.data(), v.data(), ones.data(), ones.data(), nullptr, 1e-6f,
                       cos.data(), sin.data(), kc.data(), vc.data(), want.data(), pos, n_heads,
                       n_kv_heads, hd, max_seq, attn.scale, ORC_F32, 0);
  CHECK(max_abs(got, want) <= 2e-3f && rel_l2(got, want) <= 1e-3f, "north-star tolerance");
}

// Sliding-window layers (Attention::window; the reference defers them):
// prefill, then a decode step over the cache it wrote, against the oracle's
// windowed attention (row i sees keys i - window < j <= i).
void sliding_window_prefill_and_decode() {
  const size_t n_heads = 8, n_kv_heads = 2, hd = 128, seq = 300, max_seq = 320, window = 100;
  const size_t q_dim = n_heads * hd, kv_dim = n_kv_heads * hd;
  nn::Attention attn;
  attn.n_heads = n_heads;
  attn.n_kv_heads = n_kv_heads;
  attn.head_dim = hd;
  attn.scale = 1.0f / std::sqrt((float)hd);
  attn.window = window;
  auto rope = nn::Rope::build(max_seq, hd, 1e6f);
  auto q = prng(seq * q_dim, 41), k = prng(seq * kv_dim, 42), v = prng(seq * kv_dim, 43);
  auto kv = nn::KvCache::create(1, max_seq, n_kv_heads, hd);
  Recorder rec;
  auto o = attn.prefill(rec, Tensor::from_f32({seq, q_dim}, q), Tensor::from_f32({seq, kv_dim}, k),
                        Tensor::from_f32({seq, kv_dim}, v), rope, kv, 0, seq);
  rec.submit();
  auto got = o.to_f32();
  auto cos = rope.cos.to_f32(), sin = rope.sin.to_f32();
  std::vector<float> kc(max_seq * kv_dim, 0.f), vc(max_seq * kv_dim, 0.f), want(seq * q_dim);
  orc_attention_prefill(q.data(), k.data(), v.data(), nullptr, nullptr, nullptr, 1e-6f,
                        cos.data(), sin.data(), kc.data(), vc.data(), want.data(), seq, n_heads,
                        n_kv_heads, hd, max_seq, attn.scale, ORC_F32, ORC_F32, window);
  CHECK(max_abs(got, want) <= 2e-3f && rel_l2(got, want) <= 1e-3f, "prefill tolerance");
  auto qd = prng(q_dim, 44), kd = prng(kv_dim, 45), vd = prng(kv_dim, 46);
  auto od = attn.decode(rec, Tensor::from_f32({1, q_dim}, qd), Tensor::from_f32({1, kv_dim}, kd),
                        Tensor::from_f32({1, kv_dim}, vd), rope, kv, 0, seq);
  rec.submit();
  auto got_d = od.to_f32();
  std::vector<float> want_d(q_dim);
  orc_attention_decode(qd.data(), kd.data(), vd.data(), nullptr, nullptr, nullptr, 1e-6f,
                       cos.data(), sin.data(), kc.data(), vc.data(), want_d.data(), seq, n_heads,
                       n_kv_heads, hd, max_seq, attn.scale, ORC_F32, window);
  CHECK(max_abs(got_d, want_d) <= 2e-3f && rel_l2(got_d, want_d) <= 1e-3f, "decode tolerance");
}

// crates/eyebrowse-kernels/src/matmul.rs:261-279: in_f not a multiple of 16,
// f16 weights, against cpu_linear on the f16-rounded weights.
void linear_f16w_matches_cpu() {
  const size_t m = 5, in_f = 33, out_f = 7;
  auto x = ramp(m * in_f, -0.2f, 0.01f), w = ramp(out_f * in_f, -0.3f, 0.005f);
  auto ct = Tensor::empty({m, out_f});
  Recorder rec;
  kernels::linear_f16w(rec, Tensor::from_f32({m, in_f}, x), Tensor::from_f16({out_f, in_f}, w), ct,
                       m, in_f, out_f);
  rec.submit();
  auto got = ct.to_f32();
  orc_round_f16(w.data(), w.size());
  std::vector<float> want(m * out_f);
  orc_linear(x.data(), w.data(), want.data(), m, in_f, out_f);
  CHECK(rel_l2(got, want) < 2e-3f, "rel_l2");
}

// nn::Linear on both device kernels: a decode row (m = 1, streamed weights)
// and a prefill block (m = 200, tensor cores), fused q/k/v width.
void linear_forward_decode_and_prefill() {
  const size_t in_f = 1024, out_f = 4096;
  nn::Linear lin;
  auto w = prng(out_f * in_f, 51);
  for (auto& v : w) v *= 0.05f;
  lin.w = Tensor::from_f16({out_f, in_f}, w);
  lin.in_f = in_f;
  lin.out_f = out_f;
  orc_round_f16(w.data(), w.size());
  Recorder rec;
  for (size_t m : {size_t(1), size_t(200)}) {
    auto x = prng(m * in_f, 52 + m);
    auto y = lin.forward(rec, Tensor::from_f32({m, in_f}, x), m);
    rec.submit();
    auto got = y.to_f32();
    std::vector<float> want(m * out_f);
    orc_linear(x.data(), w.data(), want.data(), m, in_f, out_f);
    CHECK(rel_l2(got, want) < 1e-5f, "rel_l2 vs cpu_linear");
  }
}

// crates/eyebrowse-nn/src/attention.rs:30-185 with its projections:
// Attention::forward over a prompt (prefill), then one token (decode),
// against cpu_linear + the oracle attention on the same f16 weights.
void attention_forward_with_projections() {
  const size_t hidden = 256, n_heads = 4, n_kv_heads = 2, hd = 64, seq = 40, max_seq = 48;
  const size_t q_dim = n_heads * hd, kv_dim = n_kv_heads * hd;
  auto weight = [](size_t out_f, size_t in_f, uint64_t seed) {
    auto w = prng(out_f * in_f, seed);
    for (auto& x : w) x *= 0.05f;
    orc_round_f16(w.data(), w.size());  // the f16 values the device holds
    return w;
  };
  auto linear = [](const std::vector<float>& w, size_t in_f, size_t out_f) {
    nn::Linear l;
    l.w = Tensor::from_f16({out_f, in_f}, w);
    l.in_f = in_f;
    l.out_f = out_f;
    return l;
  };
  auto wq = weight(q_dim, hidden, 61), wk = weight(kv_dim, hidden, 62);
  auto wv = weight(kv_dim, hidden, 63), wo = weight(hidden, q_dim, 64);
  auto qn = prng(hd, 65), kn = prng(hd, 66);
  for (auto& x : qn) x = 1.f + 0.1f * x;
  for (auto& x : kn) x = 1.f + 0.1f * x;
  nn::Attention attn;
  attn.q_proj = linear(wq, hidden, q_dim);
  attn.k_proj = linear(wk, hidden, kv_dim);
  attn.v_proj = linear(wv, hidden, kv_dim);
  attn.o_proj = linear(wo, q_dim, hidden);
  attn.q_norm = Tensor::from_f32({hd}, qn);
  attn.k_norm = Tensor::from_f32({hd}, kn);
  attn.n_heads = n_heads;
  attn.n_kv_heads = n_kv_heads;
  attn.head_dim = hd;
  attn.scale = 1.0f / std::sqrt((float)hd);
  auto rope = nn::Rope::build(max_seq, hd, 1e6f);
  auto kv = nn::KvCache::create(1, max_seq, n_kv_heads, hd);
  auto cos = rope.cos.to_f32(), sin = rope.sin.to_f32();
  std::vector<float> kc(max_seq * kv_dim, 0.f), vc(max_seq * kv_dim, 0.f);
  Recorder rec;

  auto x = prng(seq * hidden, 67);
  auto y = attn.forward(rec, Tensor::from_f32({seq, hidden}, x), rope, kv, 0, seq, 0);
  rec.submit();
  auto got = y.to_f32();
  std::vector<float> q(seq * q_dim), k(seq * kv_dim), v(seq * kv_dim), o(seq * q_dim);
  std::vector<float> want(seq * hidden);
  orc_linear(x.data(), wq.data(), q.data(), seq, hidden, q_dim);
  orc_linear(x.data(), wk.data(), k.data(), seq, hidden, kv_dim);
  orc_linear(x.data(), wv.data(), v.data(), seq, hidden, kv_dim);
  orc_attention_prefill(q.data(), k.data(), v.data(), qn.data(), kn.data(), nullptr, 1e-6f,
                        cos.data(), sin.data(), kc.data(), vc.data(), o.data(), seq, n_heads,
                        n_kv_heads, hd, max_seq, attn.scale, ORC_F32, ORC_F32, 0);
  orc_linear(o.data(), wo.data(), want.data(), seq, q_dim, hidden);
  CHECK(max_abs(got, want) <= 2e-3f && rel_l2(got, want) <= 1e-3f, "prefill forward");

  auto xd = prng(hidden, 68);
  auto yd = attn.forward(rec, Tensor::from_f32({1, hidden}, xd), rope, kv, 0, 1, seq);
  rec.submit();
  auto got_d = yd.to_f32();
  std::vector<float> qd(q_dim), kd(kv_dim), vd(kv_dim), od(q_dim), want_d(hidden);
  orc_linear(xd.data(), wq.data(), qd.data(), 1, hidden, q_dim);
  orc_linear(xd.data(), wk.data(), kd.data(), 1, hidden, kv_dim);
  orc_linear(xd.data(), wv.data(), vd.data(), 1, hidden, kv_dim);
  orc_attention_decode(qd.data(), kd.data(), vd.data(), qn.data(), kn.data(), nullptr, 1e-6f,
                       cos.data(), sin.data(), kc.data(), vc.data(), od.data(), seq, n_heads,
                       n_kv_heads, hd, max_seq, attn.scale, ORC_F32, 0);
  orc_linear(od.data(), wo.data(), want_d.data(), 1, q_dim, hidden);
  CHECK(max_abs(got_d, want_d) <= 2e-3f && rel_l2(got_d, want_d) <= 1e-3f, "decode forward");

  // Two rows at base_pos > 0 are one decode step over the first row, as in the
  // reference (its decode projects one row of x): the same [1, hidden] result
  // as the one-row call above (which wrote the same cache row).
  auto x2 = prng(2 * hidden, 69);
  std::copy(xd.begin(), xd.end(), x2.begin());
  auto y2 = attn.forward(rec, Tensor::from_f32({2, hidden}, x2), rope, kv, 0, 2, seq);
  rec.submit();
  CHECK(y2.numel() == hidden, "a decode step returns one row");
  auto got_2 = y2.to_f32();
  CHECK(max_abs(got_2, got_d) == 0.0f, "two rows at base_pos > 0 decode the first row");
}

// Where the reference panics on a bad shape, the mirror throws Error.
void invalid_shapes_throw() {
  auto x = Tensor::zeros({64});
  Recorder rec;
  try {
    kernels::attn_prefill(rec, x, x, x, x, 3, 2, 1, 8, 0.3f);  // h % hkv != 0
  } catch (const Error& e) {
    CHECK(e.status == EB_ERR_INVALID_ARGUMENT, "status is EB_ERR_INVALID_ARGUMENT");
    return;
  }
  throw Fail("no exception");
}

struct Test {
  const char* name;
  std::function<void()> fn;
};

}  // namespace

int main(int argc, char** argv) {
  const std::vector<Test> tests = {
      {"attn_prefill_matches_cpu", attn_prefill_matches_cpu},
      {"attn_decode_matches_cpu", attn_decode_matches_cpu},
      {"rope_matches_cpu", rope_matches_cpu},
      {"rmsnorm_matches_cpu", rmsnorm_matches_cpu},
      {"kv_write_places_rows", kv_write_places_rows},
      {"rope_build_tables", rope_build_tables},
      {"prefill_decode_consistency", prefill_decode_consistency},
      {"attn_prefill_tensor_core_hd128", attn_prefill_tensor_core_hd128},
      {"attention_decode_long_context_hd128", attention_decode_long_context_hd128},
      {"sliding_window_prefill_and_decode", sliding_window_prefill_and_decode},
      {"linear_f16w_matches_cpu", linear_f16w_matches_cpu},
      {"linear_forward_decode_and_prefill", linear_forward_decode_and_prefill},
      {"attention_forward_with_projections", attention_forward_with_projections},
      {"invalid_shapes_throw", invalid_shapes_throw},
  };
  if (argc > 1 && std::string(argv[1]) == "--list") {
    for (const auto& t : tests) std::printf("%s\n", t.name);
    return 0;
  }
  int failed = 0;
  for (const auto& t : tests) {
    try {
      t.fn();
      std::printf("[ok] %s\n", t.name);
    } catch (const std::exception& e) {
      std::printf("[FAIL] %s: %s\n", t.name, e.what());
      failed++;
    }
  }
  std::printf("%d of %zu tests failed\n", failed, tests.size());
  return failed;
}
