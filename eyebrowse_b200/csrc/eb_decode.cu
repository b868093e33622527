// eb_decode.cu -- split-K flash-decoding over the seq-major KV cache.
//
// Replaces attn_decode (crates/eyebrowse-kernels/src/attention.rs:52-90,
// :124-162) together with the decode branch's q/k/v RMSNorm, RoPE and
// kv_write (crates/eyebrowse-nn/src/attention.rs:133-168).
//
// Grid (chunks, kv-head groups, sequences). A CTA owns one KV head, up to 8
// of its query heads (GQA: every K/V row is read once for the whole group) and
// one chunk of context rows. K and V rows stream through 16-byte loads that
// skip L1; each row's dot products reduce with xor shuffles inside the lanes
// that hold it; an online softmax runs per (warp, row slot) and the slots
// merge in shared memory. With more than one chunk the CTA writes its
// partial (m, l, acc) to the workspace, takes a ticket, and the last CTA of
// the (sequence, head group) merges all partials (no spin-wait anywhere) and
// resets the ticket counter to zero for the next call.
#include "eb_common.cuh"
#include "eb_kernels.cuh"
#include "eb_decode_out.cuh"
#include "eb_rowops.cuh"

namespace eb {

constexpr int kDecWarps = 4;
// Row steps loaded per batch, all loads issued before use: 8 for an f32 cache
// whose row a lane holds in one 16-byte load (64 registers of K/V in
// flight), else 4 (16-bit rows carry twice the elements per load, and with
// 8 query heads per CTA more steps would spill).
#ifndef EB_DECODE_U1
#define EB_DECODE_U1 8
#endif
constexpr int dec_steps(int loads, int elem_bytes) {
  return (loads == 1 && elem_bytes == 4) ? EB_DECODE_U1 : 4;
}

template <int HD, typename TC>
struct DecShape {
  static constexpr int VEC = 16 / (int)sizeof(TC);        // elements per 16-byte load
  static constexpr int LPR_RAW = HD / VEC;
  static constexpr int LPR = LPR_RAW >= 32 ? 32 : LPR_RAW;  // lanes holding one row
  static constexpr int LOADS = LPR_RAW >= 32 ? LPR_RAW / 32 : 1;
  static constexpr int RPW = 32 / LPR;                       // rows per warp step
  static constexpr int EPL = VEC * LOADS;                    // elements per lane per row
  static constexpr int NS = kDecWarps * RPW;                 // softmax state slots per CTA
  static constexpr int U = dec_steps(LOADS, (int)sizeof(TC));
  static constexpr int ROWS_PER_BATCH = kDecWarps * RPW * U;
};

template <typename TC, int N>
__device__ __forceinline__ void unpack(const uint4 (&u)[N], float (&f)[N * 16 / sizeof(TC)]) {
  constexpr int PER = 16 / (int)sizeof(TC);
#pragma unroll
  for (int w = 0; w < N; w++) {
    const TC* e = reinterpret_cast<const TC*>(&u[w]);
#pragma unroll
    for (int i = 0; i < PER; i++) f[w * PER + i] = Elem<TC>::to_f32(e[i]);
  }
}

template <int HD, typename TC, int G>
__global__ void __launch_bounds__(kDecWarps * 32) decode_kernel(DecodeArgs a, int gsubs) {
  using Sh = DecShape<HD, TC>;
  constexpr int VEC = Sh::VEC, LPR = Sh::LPR, LOADS = Sh::LOADS, RPW = Sh::RPW, EPL = Sh::EPL;
  constexpr int NS = Sh::NS;
  constexpr int MAXC = 256;  // chunk partials merged by the last CTA (host keeps cmax <= MAXC)
  constexpr int WORK = (NS * G * HD > G * MAXC) ? NS * G * HD : G * MAXC;
  __shared__ __align__(16) float qs[G][HD];
  __shared__ __align__(16) float rowbuf[2][HD];
  __shared__ __align__(16) float work[WORK];  // slot accumulators, then chunk weights
  __shared__ float sm_m[NS][G], sm_l[NS][G];
  __shared__ float sm_M[G], sm_L[G];
  __shared__ int sm_last;

  const int c = blockIdx.x;
  const int grp = blockIdx.y;  // kv head * gsubs + sub-group
  const int kvh = grp / gsubs, sub = grp % gsubs;
  const int b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pos = a.positions ? a.positions[b] : a.pos_scalar;
  // rows [row_lo, pos]: the whole context, or the last `window` rows of it
  const int row_lo = a.window > 0 ? max(0, pos - a.window + 1) : 0;
  const int n_rows = pos + 1 - row_lo;
  const int n_chunks = (n_rows + a.chunk - 1) / a.chunk;
  if (c >= n_chunks) return;
  const int head0 = kvh * (G * gsubs) + sub * G;  // first query head of this CTA

  // ---- prologue: q rows (norm, RoPE at pos), new k/v row into the cache
  for (int g = warp; g < G; g += kDecWarps) {
    float* row = qs[g];
    const int64_t qo = (int64_t)b * a.q_bstride + (int64_t)(head0 + g) * HD;
    for (int d = lane; d < HD; d += 32) row[d] = ld_any(a.q, qo + d, a.dtype_q);
    __syncwarp();
    warp_row_norm(row, HD, a.q_norm_w, a.eps, lane);
    if (a.cos_t)
      warp_row_rope(row, HD, a.cos_t + (int64_t)pos * (HD / 2), a.sin_t + (int64_t)pos * (HD / 2),
                    lane);
  }
  if (a.k_new && c == n_chunks - 1 && warp >= kDecWarps - 2) {
    // Every CTA of the last chunk writes the same bits (sub-groups of one KV
    // head compute identical rows), then reads the row back like any other.
    const int which = warp - (kDecWarps - 2);
    float* row = rowbuf[which];
    const int64_t so = (int64_t)b * a.kv_bstride + (int64_t)kvh * HD;
    const void* src = which ? a.v_new : a.k_new;
    for (int d = lane; d < HD; d += 32) row[d] = ld_any(src, so + d, a.dtype_kv);
    __syncwarp();
    warp_row_norm(row, HD, which ? a.v_norm_w : a.k_norm_w, a.eps, lane);
    if (!which && a.cos_t)
      warp_row_rope(row, HD, a.cos_t + (int64_t)pos * (HD / 2), a.sin_t + (int64_t)pos * (HD / 2),
                    lane);
    TC* cache = reinterpret_cast<TC*>(which ? a.vcache : a.kcache) + (int64_t)b * a.cache_bstride +
                ((int64_t)pos * a.Hkv + kvh) * HD;
    for (int d = lane; d < HD; d += 32) cache[d] = Elem<TC>::from_f32(row[d]);
  }
  __syncthreads();

  const int slot = lane / LPR, sl = lane % LPR;
  float qr[G][EPL];
#pragma unroll
  for (int g = 0; g < G; g++)
#pragma unroll
    for (int t = 0; t < LOADS; t++)
#pragma unroll
      for (int e = 0; e < VEC; e++)
        qr[g][t * VEC + e] = qs[g][(t * LPR + sl) * VEC + e] * a.scale_log2;

  float m[G], l[G], acc[G][EPL];
#pragma unroll
  for (int g = 0; g < G; g++) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; e++) acc[g][e] = 0.f;
  }

  const int row_begin = row_lo + c * a.chunk;
  const int row_end = min(row_begin + a.chunk, pos + 1);
  const int64_t rstride = (int64_t)a.Hkv * HD;
  const TC* kc = reinterpret_cast<const TC*>(a.kcache) + (int64_t)b * a.cache_bstride +
                 (int64_t)kvh * HD + sl * VEC;
  const TC* vc = reinterpret_cast<const TC*>(a.vcache) + (int64_t)b * a.cache_bstride +
                 (int64_t)kvh * HD + sl * VEC;

  for (int r0 = row_begin; r0 < row_end; r0 += Sh::ROWS_PER_BATCH) {
    uint4 kr[Sh::U][LOADS], vr[Sh::U][LOADS];
    bool ok[Sh::U];
#pragma unroll
    for (int u = 0; u < Sh::U; u++) {
      const int row = r0 + (u * kDecWarps + warp) * RPW + slot;
      ok[u] = row < row_end;
#pragma unroll
      for (int t = 0; t < LOADS; t++) {
        if (ok[u]) {
          kr[u][t] = ld_stream_u4(kc + (int64_t)row * rstride + t * LPR * VEC);
          vr[u][t] = ld_stream_u4(vc + (int64_t)row * rstride + t * LPR * VEC);
        } else {
          kr[u][t] = make_uint4(0, 0, 0, 0);
          vr[u][t] = make_uint4(0, 0, 0, 0);
        }
      }
    }
    float s[Sh::U][G];
#pragma unroll
    for (int u = 0; u < Sh::U; u++) {
      float kf[EPL];
      unpack<TC, LOADS>(kr[u], kf);
#pragma unroll
      for (int g = 0; g < G; g++) {
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; e++) dot = fmaf(qr[g][e], kf[e], dot);
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        s[u][g] = ok[u] ? dot : -INFINITY;
      }
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
      float mb = s[0][g];
#pragma unroll
      for (int u = 1; u < Sh::U; u++) mb = fmaxf(mb, s[u][g]);
      if (mb == -INFINITY) continue;
      const float mn = fmaxf(m[g], mb);
      const float corr = ex2(m[g] - mn);
      l[g] *= corr;
#pragma unroll
      for (int e = 0; e < EPL; e++) acc[g][e] *= corr;
      m[g] = mn;
    }
#pragma unroll
    for (int u = 0; u < Sh::U; u++) {
      float vf[EPL];
      unpack<TC, LOADS>(vr[u], vf);
#pragma unroll
      for (int g = 0; g < G; g++) {
        const float p = (s[u][g] == -INFINITY) ? 0.f : ex2(s[u][g] - m[g]);
        l[g] += p;
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[g][e] = fmaf(p, vf[e], acc[g][e]);
      }
    }
  }

  // ---- merge the NS slot states of this CTA
  const int si = warp * RPW + slot;
  float* sacc = work;  // [NS][G][HD]
  if (sl == 0) {
#pragma unroll
    for (int g = 0; g < G; g++) {
      sm_m[si][g] = m[g];
      sm_l[si][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; g++)
#pragma unroll
    for (int t = 0; t < LOADS; t++)
#pragma unroll
      for (int e = 0; e < VEC; e++)
        sacc[(si * G + g) * HD + (t * LPR + sl) * VEC + e] = acc[g][t * VEC + e];
  __syncthreads();
  if (tid < G) {
    float M = -INFINITY;
    for (int s2 = 0; s2 < NS; s2++) M = fmaxf(M, sm_m[s2][tid]);
    float L = 0.f;
    for (int s2 = 0; s2 < NS; s2++)
      if (sm_m[s2][tid] != -INFINITY) L += sm_l[s2][tid] * ex2(sm_m[s2][tid] - M);
    sm_M[tid] = M;
    sm_L[tid] = L;
  }
  __syncthreads();
  const bool split = n_chunks > 1;
  for (int idx = tid; idx < G * HD; idx += kDecWarps * 32) {
    const int g = idx / HD, d = idx % HD;
    const float M = sm_M[g];
    float O = 0.f;
    for (int s2 = 0; s2 < NS; s2++)
      if (sm_m[s2][g] != -INFINITY) O += sacc[(s2 * G + g) * HD + d] * ex2(sm_m[s2][g] - M);
    const int h = head0 + g;
    if (!split) {
      dec_store(a, b, h, HD, d, O / sm_L[g]);
    } else {
      a.ws_acc[(((int64_t)b * a.H + h) * a.cmax + c) * HD + d] = O;
    }
  }
  if (!split) return;
  if (tid < G) {
    float* ml = a.ws_ml + (((int64_t)b * a.H + head0 + tid) * a.cmax + c) * 2;
    ml[0] = sm_M[tid];
    ml[1] = sm_L[tid];
  }
  // ---- ticket: the last CTA of this (sequence, head group) merges the chunks
  __threadfence();
  __syncthreads();
  unsigned* cnt = a.ws_cnt + (int64_t)b * gridDim.y + grp;
  if (tid == 0) sm_last = (atomicAdd(cnt, 1u) == (unsigned)(n_chunks - 1));
  __syncthreads();
  if (!sm_last) return;
  __threadfence();
  float* wts = work;  // [G][MAXC], reuses the slot accumulators
  // One warp per head: lanes over the chunks for the max, the chunk weights
  // 2^(m_c - M) and the row sum (the partials are read in parallel, not by one
  // thread in a dependent loop).
  for (int g = warp; g < G; g += kDecWarps) {
    const float* ml = a.ws_ml + (((int64_t)b * a.H + head0 + g) * a.cmax) * 2;
    float M = -INFINITY;
    for (int cc = lane; cc < n_chunks; cc += 32) M = fmaxf(M, __ldcg(ml + 2 * cc));
    M = warp_max(M);
    float L = 0.f;
    for (int cc = lane; cc < n_chunks; cc += 32) {
      const float w = ex2(__ldcg(ml + 2 * cc) - M);
      wts[g * MAXC + cc] = w;
      L += __ldcg(ml + 2 * cc + 1) * w;
    }
    L = warp_sum(L);
    if (lane == 0) sm_L[g] = L;
  }
  __syncthreads();
  for (int idx = tid; idx < G * HD; idx += kDecWarps * 32) {
    const int g = idx / HD, d = idx % HD;
    const int h = head0 + g;
    const float* pa = a.ws_acc + (((int64_t)b * a.H + h) * a.cmax) * HD + d;
    const float* wg = wts + g * MAXC;
    // 8 independent sums: 8 partial loads in flight per thread
    float O8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    int cc = 0;
    for (; cc + 8 <= n_chunks; cc += 8) {
#pragma unroll
      for (int u = 0; u < 8; u++) O8[u] += __ldcg(pa + (int64_t)(cc + u) * HD) * wg[cc + u];
    }
    for (; cc < n_chunks; cc++) O8[0] += __ldcg(pa + (int64_t)cc * HD) * wg[cc];
    const float O = ((O8[0] + O8[1]) + (O8[2] + O8[3])) + ((O8[4] + O8[5]) + (O8[6] + O8[7]));
    dec_store(a, b, h, HD, d, O / sm_L[g]);
  }
  if (tid == 0) *cnt = 0u;
}

int decode_rows_per_batch(int hd, int dtype_cache, int group) {
  if (decode_tc_supported(hd, dtype_cache, group)) return 64;  // tensor-core tile rows
  const int vec = dtype_cache == kF32 ? 4 : 8;
  const int lpr_raw = hd / vec;
  const int lpr = lpr_raw > 32 ? 32 : lpr_raw;
  const int loads = lpr_raw >= 32 ? lpr_raw / 32 : 1;
  const int rpw = 32 / lpr;
  return kDecWarps * rpw * dec_steps(loads, dtype_cache == kF32 ? 4 : 2);
}

template <int HD, typename TC>
static cudaError_t launch_g(const DecodeArgs& a, int batch, cudaStream_t st) {
  const int G = a.H / a.Hkv;
  int gs;
  if (G % 8 == 0) gs = 8;
  else if (G % 4 == 0) gs = 4;
  else if (G % 2 == 0) gs = 2;
  else gs = 1;
  const int gsubs = G / gs;
  dim3 grid(a.cmax, a.Hkv * gsubs, batch);
  switch (gs) {
    case 8: decode_kernel<HD, TC, 8><<<grid, kDecWarps * 32, 0, st>>>(a, gsubs); break;
    case 4: decode_kernel<HD, TC, 4><<<grid, kDecWarps * 32, 0, st>>>(a, gsubs); break;
    case 2: decode_kernel<HD, TC, 2><<<grid, kDecWarps * 32, 0, st>>>(a, gsubs); break;
    default: decode_kernel<HD, TC, 1><<<grid, kDecWarps * 32, 0, st>>>(a, gsubs); break;
  }
  return cudaGetLastError();
}

template <int HD>
static cudaError_t launch_hd(const DecodeArgs& a, int dtype_cache, int batch, cudaStream_t st) {
  switch (dtype_cache) {
    case kF32: return launch_g<HD, float>(a, batch, st);
    case kF16: return launch_g<HD, __half>(a, batch, st);
    case kBF16: return launch_g<HD, __nv_bfloat16>(a, batch, st);
  }
  return cudaErrorNotSupported;
}

cudaError_t launch_decode(const DecodeArgs& a, int dtype_cache, int batch, cudaStream_t st) {
  if (decode_tc_supported(a.hd, dtype_cache, a.H / a.Hkv))
    return launch_decode_tc(a, dtype_cache, batch, st);
  switch (a.hd) {
    case 64: return launch_hd<64>(a, dtype_cache, batch, st);
    case 128: return launch_hd<128>(a, dtype_cache, batch, st);
    case 256: return launch_hd<256>(a, dtype_cache, batch, st);
  }
  return cudaErrorNotSupported;
}

}  // namespace eb
