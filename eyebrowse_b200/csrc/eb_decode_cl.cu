// eb_decode_cl.cu -- latency decode for f32/bf16 caches: the split-K chunks of
// one (sequence, KV-head group) form a thread-block cluster and merge their
// partials through distributed shared memory.
//
// Replaces attn_decode (crates/eyebrowse-kernels/src/attention.rs:52-90,
// :124-162) with the decode branch's q/k/v RMSNorm, RoPE and kv_write
// (crates/eyebrowse-nn/src/attention.rs:133-168), for the launches where the
// whole context fits one wave: a single sequence or a few (config 2, config
// 4's decode steps). The workspace kernel (eb_decode.cu) needs about six
// dependent trips to memory per call (q row, RoPE table, two K/V batches,
// partial write + ticket, partial read-back); here there are two:
//   - each lane issues its first batch of 16-byte K/V loads (32 of them)
//     before anything else, and the q/k/v prologue (row loads, norm, RoPE,
//     the new row's cache write) runs while they are in flight;
//   - with 8 warps per CTA and at most 16 CTAs per (sequence, group), a
//     CTA's chunk is mostly one batch;
//   - the partials never leave the cluster: every CTA stores its (m, l, O)
//     into rank 0's shared memory (distributed shared memory), and after one
//     cluster barrier rank 0 combines them locally and writes o while the
//     other CTAs exit.
// Grid (chunks, kv-head groups, sequences), cluster (chunks, 1, 1): cluster
// rank == chunk. Every CTA reaches the cluster barrier (CTAs past a short
// sequence's context contribute an empty partial).
#include <cooperative_groups.h>

#include "eb_common.cuh"
#include "eb_kernels.cuh"
#include "eb_decode_out.cuh"
#include "eb_rowops.cuh"

namespace cg = cooperative_groups;

namespace eb {

constexpr int kClWarps = 8;
constexpr int kClMaxChunks = 16;

// Row steps per batch for G query heads and EPL elements per lane: as many
// 16-byte K/V loads in flight per lane as fit beside the batch's scores
// (U x G) and the q/accumulator registers (2 x G x EPL) -- 32 loads for one
// or two query heads, 16 for four, 8 for eight 8-element (16-bit) lanes.
constexpr int cl_steps(int g, int loads, int epl) {
  return (g <= 2 ? 16 : (g <= 4 || epl < 8) ? 8 : 4) / loads;
}

template <int HD, typename TC, int G>
struct ClShape {
  static constexpr int VEC = 16 / (int)sizeof(TC);          // elements per 16-byte load
  static constexpr int LPR_RAW = HD / VEC;
  static constexpr int LPR = LPR_RAW >= 32 ? 32 : LPR_RAW;  // lanes holding one row
  static constexpr int LOADS = LPR_RAW >= 32 ? LPR_RAW / 32 : 1;
  static constexpr int RPW = 32 / LPR;                      // rows per warp step
  static constexpr int EPL = VEC * LOADS;                   // elements per lane per row
  static constexpr int NS = kClWarps * RPW;                 // softmax slots per CTA
  static constexpr int U = cl_steps(G, LOADS, EPL);
  static constexpr int RPB = kClWarps * RPW * U;            // rows per CTA batch
  // dynamic shared memory: slot accumulators, then the partials of the n
  // chunks of the cluster (every CTA pushes its own into rank 0's copy)
  static constexpr int SACC = NS * G * HD;
  static constexpr int smem(int n) { return (SACC + n * G * HD) * 4; }
};

int decode_cl_rows_per_batch(int hd, int dtype_cache, int group) {
  const int vec = dtype_cache == kF32 ? 4 : 8;
  const int lpr_raw = hd / vec;
  const int lpr = lpr_raw > 32 ? 32 : lpr_raw;
  const int loads = lpr_raw >= 32 ? lpr_raw / 32 : 1;
  const int gs = group % 8 == 0 ? 8 : group % 4 == 0 ? 4 : group % 2 == 0 ? 2 : 1;
  return kClWarps * (32 / lpr) * cl_steps(gs, loads, vec * loads);
}

// N 16-byte words of cache elements -> floats.
template <typename TC, int N>
__device__ __forceinline__ void unpack_rows(const uint4 (&u)[N], float (&f)[N * 16 / sizeof(TC)]) {
  constexpr int PER = 16 / (int)sizeof(TC);
#pragma unroll
  for (int w = 0; w < N; w++) {
    const TC* e = reinterpret_cast<const TC*>(&u[w]);
#pragma unroll
    for (int i = 0; i < PER; i++) f[w * PER + i] = Elem<TC>::to_f32(e[i]);
  }
}

template <int HD, typename TC, int G>
__global__ void __launch_bounds__(kClWarps * 32, 1) decode_cl_kernel(DecodeArgs a, int gsubs) {
  using Sh = ClShape<HD, TC, G>;
  constexpr int VEC = Sh::VEC, LPR = Sh::LPR, LOADS = Sh::LOADS, RPW = Sh::RPW, EPL = Sh::EPL;
  constexpr int NS = Sh::NS, U = Sh::U;
  extern __shared__ __align__(16) float dyn[];
  float* sacc = dyn;                 // [NS][G][HD]
  float* recv_acc = dyn + Sh::SACC;  // [n][G][HD]: rank 0's copy receives every chunk's O
  __shared__ __align__(16) float qs[G][HD];
  __shared__ float sm_m[NS][G], sm_l[NS][G];
  __shared__ float part_m[G], part_l[G];
  __shared__ float recv_m[kClMaxChunks][G], recv_l[kClMaxChunks][G];

  cg::cluster_group cluster = cg::this_cluster();
  const int c = blockIdx.x;    // chunk == cluster rank
  const int grp = blockIdx.y;  // kv head * gsubs + sub-group
  const int kvh = grp / gsubs, sub = grp % gsubs;
  const int b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pos = a.positions ? a.positions[b] : a.pos_scalar;
  const int row_lo = a.window > 0 ? max(0, pos - a.window + 1) : 0;
  const int row_begin = row_lo + c * a.chunk;
  const int row_end = min(row_begin + a.chunk, pos + 1);  // empty when row_begin > pos
  const int head0 = kvh * (G * gsubs) + sub * G;          // first query head of this CTA
  const int slot = lane / LPR, sl = lane % LPR;
  const int64_t rstride = (int64_t)a.Hkv * HD;
  const TC* kc = reinterpret_cast<const TC*>(a.kcache) + (int64_t)b * a.cache_bstride +
                 (int64_t)kvh * HD + sl * VEC;
  const TC* vc = reinterpret_cast<const TC*>(a.vcache) + (int64_t)b * a.cache_bstride +
                 (int64_t)kvh * HD + sl * VEC;

  // ---- prologue jobs: the G q rows, then (in the CTA whose chunk holds pos)
  // the new k and v rows; warp w takes jobs w, w + 8. A job's inputs -- its
  // row, norm weights and RoPE table entries (lane l holds elements
  // [l*E, l*E+E); its RoPE partner is lane l ^ 16) -- are loaded in one trip,
  // the first job's before the K/V prefetch below.
  constexpr int E = HD / 32;
  const bool has_pos = row_begin <= pos && pos < row_end;
  const int n_jobs = G + ((a.k_new && has_pos) ? 2 : 0);
  struct Job {
    float f[E], w[E], cs[E], sn[E];
  };
  auto job_load = [&](int j, Job& jb) {
    const int role = j < G ? 0 : j - G + 1;  // 0 q, 1 k, 2 v
    const float* nw = role == 0 ? a.q_norm_w : role == 1 ? a.k_norm_w : a.v_norm_w;
    const bool rope = role <= 1 && a.cos_t != nullptr;
    if (role == 0)
      ld_row<E>(a.q, (int64_t)b * a.q_bstride + (int64_t)(head0 + j) * HD + lane * E, a.dtype_q,
                jb.f);
    else
      ld_row<E>(role == 1 ? a.k_new : a.v_new,
                (int64_t)b * a.kv_bstride + (int64_t)kvh * HD + lane * E, a.dtype_kv, jb.f);
#pragma unroll
    for (int e = 0; e < E; e++) {
      jb.w[e] = nw ? nw[lane * E + e] : 1.f;
      jb.cs[e] = rope ? a.cos_t[(int64_t)pos * (HD / 2) + (lane & 15) * E + e] : 1.f;
      jb.sn[e] = rope ? a.sin_t[(int64_t)pos * (HD / 2) + (lane & 15) * E + e] : 0.f;
    }
  };
  // RMSNorm then RoPE (the reference's f32 arithmetic, crates/eyebrowse-
  // kernels/src/rmsnorm.rs:34-36, rope.rs:25-30); q rows to shared memory,
  // the new k/v row to the cache (sub-groups of one KV head write the same
  // bits).
  auto job_math = [&](int j, Job& jb) {
    const int role = j < G ? 0 : j - G + 1;
    const float* nw = role == 0 ? a.q_norm_w : role == 1 ? a.k_norm_w : a.v_norm_w;
    if (nw) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E; e++) ss = __fadd_rn(ss, __fmul_rn(jb.f[e], jb.f[e]));
      ss = warp_sum(ss);
      const float inv = 1.0f / sqrtf(ss / (float)HD + a.eps);
#pragma unroll
      for (int e = 0; e < E; e++) jb.f[e] = __fmul_rn(__fmul_rn(jb.f[e], inv), jb.w[e]);
    }
    if (role <= 1 && a.cos_t != nullptr) {
#pragma unroll
      for (int e = 0; e < E; e++) {
        const float other = __shfl_xor_sync(0xffffffffu, jb.f[e], 16);
        jb.f[e] = lane < 16 ? __fsub_rn(__fmul_rn(jb.f[e], jb.cs[e]), __fmul_rn(other, jb.sn[e]))
                            : __fadd_rn(__fmul_rn(jb.f[e], jb.cs[e]), __fmul_rn(other, jb.sn[e]));
      }
    }
    if (role == 0) {
#pragma unroll
      for (int e = 0; e < E; e++) qs[j][lane * E + e] = jb.f[e];
    } else {
      TC* cache = reinterpret_cast<TC*>(role == 2 ? a.vcache : a.kcache) +
                  (int64_t)b * a.cache_bstride + ((int64_t)pos * a.Hkv + kvh) * HD + lane * E;
#pragma unroll
      for (int e = 0; e < E; e++) cache[e] = Elem<TC>::from_f32(jb.f[e]);
    }
  };
  Job job;
  if (warp < n_jobs) job_load(warp, job);

  // ---- the first batch of K/V rows, in flight during the prologue's math
  uint4 kr[U][LOADS], vr[U][LOADS];
  auto load_batch = [&](int r0) {
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int row = r0 + (u * kClWarps + warp) * RPW + slot;
#pragma unroll
      for (int t = 0; t < LOADS; t++) {
        if (row < row_end) {
          kr[u][t] = ld_stream_u4(kc + (int64_t)row * rstride + t * LPR * VEC);
          vr[u][t] = ld_stream_u4(vc + (int64_t)row * rstride + t * LPR * VEC);
        } else {
          kr[u][t] = make_uint4(0, 0, 0, 0);
          vr[u][t] = make_uint4(0, 0, 0, 0);
        }
      }
    }
  };
  load_batch(row_begin);
  // The later batches' rows into L2 now (a hint: no registers, no waiting),
  // so each load after the first batch finds them there instead of waiting
  // on HBM behind the previous batch's compute.
  for (int r1 = row_begin + Sh::RPB; r1 < row_end; r1 += Sh::RPB) {
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int row = r1 + (u * kClWarps + warp) * RPW + slot;
      if (row < row_end) {
#pragma unroll
        for (int t = 0; t < LOADS; t++) {
          asm volatile("prefetch.global.L2 [%0];" ::"l"(kc + (int64_t)row * rstride + t * LPR * VEC));
          asm volatile("prefetch.global.L2 [%0];" ::"l"(vc + (int64_t)row * rstride + t * LPR * VEC));
        }
      }
    }
  }
  if (warp < n_jobs) job_math(warp, job);
  for (int j = warp + kClWarps; j < n_jobs; j += kClWarps) {  // G = 8 with a new row
    job_load(j, job);
    job_math(j, job);
  }
  __syncthreads();
  if (a.k_new && has_pos) {
    // the prefetched row pos predates its write above: load it again
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int row = row_begin + (u * kClWarps + warp) * RPW + slot;
      if (row == pos) {
#pragma unroll
        for (int t = 0; t < LOADS; t++) {
          kr[u][t] = __ldcg(reinterpret_cast<const uint4*>(kc + (int64_t)row * rstride + t * LPR * VEC));
          vr[u][t] = __ldcg(reinterpret_cast<const uint4*>(vc + (int64_t)row * rstride + t * LPR * VEC));
        }
      }
    }
  }

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

  for (int r0 = row_begin; r0 < row_end; r0 += Sh::RPB) {
    if (r0 != row_begin) load_batch(r0);
    float s[U][G];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const bool ok = r0 + (u * kClWarps + warp) * RPW + slot < row_end;
      float kf[EPL];
      unpack_rows<TC, LOADS>(kr[u], kf);
#pragma unroll
      for (int g = 0; g < G; g++) {
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; e++) dot = fmaf(qr[g][e], kf[e], dot);
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        s[u][g] = ok ? dot : -INFINITY;
      }
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
      float mb = s[0][g];
#pragma unroll
      for (int u = 1; u < U; u++) mb = fmaxf(mb, s[u][g]);
      if (mb == -INFINITY) continue;
      const float mn = fmaxf(m[g], mb);
      const float corr = ex2(m[g] - mn);
      l[g] *= corr;
#pragma unroll
      for (int e = 0; e < EPL; e++) acc[g][e] *= corr;
      m[g] = mn;
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      float vf[EPL];
      unpack_rows<TC, LOADS>(vr[u], vf);
#pragma unroll
      for (int g = 0; g < G; g++) {
        const float p = (s[u][g] == -INFINITY) ? 0.f : ex2(s[u][g] - m[g]);
        l[g] += p;
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[g][e] = fmaf(p, vf[e], acc[g][e]);
      }
    }
  }

  // ---- merge the NS slot states into this CTA's partial (m, l, O)
  const int si = warp * RPW + slot;
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
    if (M != -INFINITY)
      for (int s2 = 0; s2 < NS; s2++)
        if (sm_m[s2][tid] != -INFINITY) L += sm_l[s2][tid] * ex2(sm_m[s2][tid] - M);
    part_m[tid] = M;
    part_l[tid] = L;
    *cluster.map_shared_rank(&recv_m[c][tid], 0) = M;
    *cluster.map_shared_rank(&recv_l[c][tid], 0) = L;
  }
  __syncthreads();
  for (int idx = tid; idx < G * HD; idx += kClWarps * 32) {
    const int g = idx / HD, d = idx % HD;
    const float M = part_m[g];
    float O = 0.f;
    if (M != -INFINITY)
      for (int s2 = 0; s2 < NS; s2++)
        if (sm_m[s2][g] != -INFINITY) O += sacc[(s2 * G + g) * HD + d] * ex2(sm_m[s2][g] - M);
    *cluster.map_shared_rank(&recv_acc[c * G * HD + idx], 0) = O;  // into rank 0
  }

  // ---- combine across the cluster: every chunk's partial is in rank 0's
  // shared memory once the barrier completes (release/acquire); the other
  // CTAs are done and may exit, rank 0 combines from local memory.
  cluster.sync();
  if (c == 0) {
    const int n = (int)gridDim.x;
    for (int idx = tid; idx < G * HD; idx += kClWarps * 32) {
      const int g = idx / HD, d = idx % HD;
      float M = -INFINITY;
      for (int cc = 0; cc < n; cc++) M = fmaxf(M, recv_m[cc][g]);
      float L = 0.f, O = 0.f;
      for (int cc = 0; cc < n; cc++) {
        const float w = recv_m[cc][g] == -INFINITY ? 0.f : ex2(recv_m[cc][g] - M);
        L += recv_l[cc][g] * w;
        O += recv_acc[cc * G * HD + idx] * w;
      }
      dec_store(a, b, head0 + g, HD, d, O / L);
    }
  }
}

template <int HD, typename TC>
static cudaError_t launch_cl_g(const DecodeArgs& a, int batch, int n_chunks, cudaStream_t st) {
  const int group = a.H / a.Hkv;
  const int gs = group % 8 == 0 ? 8 : group % 4 == 0 ? 4 : group % 2 == 0 ? 2 : 1;
  const int gsubs = group / gs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)n_chunks, (unsigned)(a.Hkv * gsubs), (unsigned)batch);
  cfg.blockDim = dim3(kClWarps * 32);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)n_chunks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto go = [&](auto kern, int smem) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess && n_chunks > 8)
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    cfg.dynamicSmemBytes = (size_t)smem;
    return cudaLaunchKernelEx(&cfg, kern, a, gsubs);
  };
  switch (gs) {
    case 8: return go(decode_cl_kernel<HD, TC, 8>, ClShape<HD, TC, 8>::smem(n_chunks));
    case 4: return go(decode_cl_kernel<HD, TC, 4>, ClShape<HD, TC, 4>::smem(n_chunks));
    case 2: return go(decode_cl_kernel<HD, TC, 2>, ClShape<HD, TC, 2>::smem(n_chunks));
    default: return go(decode_cl_kernel<HD, TC, 1>, ClShape<HD, TC, 1>::smem(n_chunks));
  }
}

// How many clusters of n CTAs of this kernel the device runs at once
// (cached; 0 if none fits).
template <int HD, typename TC, int G>
static int active_clusters(int n) {
  static int cache[kClMaxChunks + 1] = {};  // value + 1, 0 = not asked yet
  int v = __atomic_load_n(&cache[n], __ATOMIC_RELAXED);
  if (v > 0) return v - 1;
  auto kern = decode_cl_kernel<HD, TC, G>;
  const int smem = ClShape<HD, TC, G>::smem(n);
  int num = 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)n, 1, 1);
  cfg.blockDim = dim3(kClWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)n;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
      (n > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
                    cudaSuccess) ||
      cudaOccupancyMaxActiveClusters(&num, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    num = 0;
  }
  __atomic_store_n(&cache[n], num + 1, __ATOMIC_RELAXED);
  return num;
}

template <int HD, typename TC>
static int cluster_limit_g(int group, int64_t clusters) {
  const int gs = group % 8 == 0 ? 8 : group % 4 == 0 ? 4 : group % 2 == 0 ? 2 : 1;
  for (int n = kClMaxChunks; n >= 1; n >>= 1) {
    int act = 0;
    switch (gs) {
      case 8: act = active_clusters<HD, TC, 8>(n); break;
      case 4: act = active_clusters<HD, TC, 4>(n); break;
      case 2: act = active_clusters<HD, TC, 2>(n); break;
      default: act = active_clusters<HD, TC, 1>(n); break;
    }
    if ((int64_t)act >= clusters) return n;
  }
  return 0;
}

int decode_cl_cluster_limit(int hd, int dtype_cache, int group, int64_t clusters) {
  const bool f32 = dtype_cache == kF32;
  switch (hd) {
    case 64: return f32 ? cluster_limit_g<64, float>(group, clusters)
                        : cluster_limit_g<64, __nv_bfloat16>(group, clusters);
    case 128: return f32 ? cluster_limit_g<128, float>(group, clusters)
                         : cluster_limit_g<128, __nv_bfloat16>(group, clusters);
    case 256: return f32 ? cluster_limit_g<256, float>(group, clusters)
                         : cluster_limit_g<256, __nv_bfloat16>(group, clusters);
  }
  return 0;
}

bool decode_cl_supported(int hd, int dtype_cache) {
  return (hd == 64 || hd == 128 || hd == 256) && (dtype_cache == kF32 || dtype_cache == kBF16);
}

cudaError_t launch_decode_cl(const DecodeArgs& a, int dtype_cache, int batch, int n_chunks,
                             cudaStream_t st) {
  if (n_chunks < 1 || n_chunks > kClMaxChunks) return cudaErrorInvalidValue;
  switch (a.hd) {
    case 64:
      return dtype_cache == kF32 ? launch_cl_g<64, float>(a, batch, n_chunks, st)
                                 : launch_cl_g<64, __nv_bfloat16>(a, batch, n_chunks, st);
    case 128:
      return dtype_cache == kF32 ? launch_cl_g<128, float>(a, batch, n_chunks, st)
                                 : launch_cl_g<128, __nv_bfloat16>(a, batch, n_chunks, st);
    case 256:
      return dtype_cache == kF32 ? launch_cl_g<256, float>(a, batch, n_chunks, st)
                                 : launch_cl_g<256, __nv_bfloat16>(a, batch, n_chunks, st);
  }
  return cudaErrorNotSupported;
}

}  // namespace eb
