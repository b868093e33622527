// eb_small.cu -- the reference's elementwise attention-path kernels (rope,
// rmsnorm, kv_write) as CUDA, the K/V preparation pass that feeds the cache
// and the tensor-core prefill, head-concat, and a generic SIMT attention for
// head dims the vector/tensor-core kernels do not cover.
#include "eb_common.cuh"
#include "eb_kernels.cuh"
#include "eb_rowops.cuh"

namespace eb {

// ---------------------------------------------------------------- rope
// One thread per (seq, head, pair), the reference's decomposition
// (crates/eyebrowse-kernels/src/rope.rs:13-31).
__global__ void rope_kernel(const float* __restrict__ x, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, float* out, int64_t seq,
                            int64_t n_heads, int64_t hd, int64_t base_pos) {
  const int64_t half = hd / 2;
  const int64_t total = seq * n_heads * half;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = idx % half;
    const int64_t tmp = idx / half;
    const int64_t head = tmp % n_heads;
    const int64_t s = tmp / n_heads;
    const int64_t base = (s * n_heads + head) * hd;
    const float c = cos_t[(s + base_pos) * half + p];
    const float sn = sin_t[(s + base_pos) * half + p];
    const float x1 = x[base + p];
    const float x2 = x[base + half + p];
    out[base + p] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
    out[base + half + p] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
  }
}

cudaError_t launch_rope(const float* x, const float* cos_t, const float* sin_t, float* out,
                        int64_t seq, int64_t n_heads, int64_t hd, int64_t base_pos,
                        cudaStream_t st) {
  const int64_t total = seq * n_heads * (hd / 2);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t blocks = (total + threads - 1) / threads;
  rope_kernel<<<(unsigned)(blocks < 65535 * 16 ? blocks : 65535 * 16), threads, 0, st>>>(
      x, cos_t, sin_t, out, seq, n_heads, hd, base_pos);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- kv_write
// cache[((dst + c) * hkv + head) * hd + d] = src[idx] (crates/eyebrowse-kernels/src/ops.rs:80-86).
// The source rows are contiguous and so are the destination rows, so the
// scatter is one contiguous copy of count*hkv*hd floats starting at row dst.
__global__ void kv_write_kernel(float* __restrict__ cache, const float* __restrict__ src,
                                int64_t n, int64_t dst_off) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    cache[dst_off + i] = src[i];
}
__global__ void kv_write_kernel_v4(float4* __restrict__ cache, const float4* __restrict__ src,
                                   int64_t n4) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x)
    cache[i] = src[i];
}

cudaError_t launch_kv_write(float* cache, const float* src, int64_t hkv, int64_t count, int64_t hd,
                            int64_t dst_start, cudaStream_t st) {
  const int64_t n = count * hkv * hd;
  if (n == 0) return cudaSuccess;
  const int64_t off = dst_start * hkv * hd;
  float* dst = cache + off;
  const int threads = 256;
  if ((n % 4) == 0 && (((uintptr_t)dst | (uintptr_t)src) & 15) == 0) {
    const int64_t n4 = n / 4;
    int64_t blocks = (n4 + threads - 1) / threads;
    if (blocks > 148 * 16) blocks = 148 * 16;
    kv_write_kernel_v4<<<(unsigned)blocks, threads, 0, st>>>(
        reinterpret_cast<float4*>(dst), reinterpret_cast<const float4*>(src), n4);
  } else {
    int64_t blocks = (n + threads - 1) / threads;
    if (blocks > 148 * 16) blocks = 148 * 16;
    kv_write_kernel<<<(unsigned)blocks, threads, 0, st>>>(cache, src, n, off);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- rmsnorm
// One warp per row (the reference uses a 256-thread workgroup per row,
// crates/eyebrowse-kernels/src/rmsnorm.rs:18-38, which idles most threads at
// head_dim rows). Same arithmetic per element: x * (1/sqrt(ss/dim + eps)) * w.
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                               float* __restrict__ out, int64_t rows, int64_t dim, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * (int64_t)(blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + row * dim;
  float ss = 0.f;
  for (int64_t i = lane; i < dim; i += 32) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / (float)dim + eps);
  float* orow = out + row * dim;
  for (int64_t i = lane; i < dim; i += 32) orow[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

cudaError_t launch_rmsnorm(const float* x, const float* w, float* out, int64_t rows, int64_t dim,
                           float eps, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  const int warps = 8;
  rmsnorm_kernel<<<(unsigned)((rows + warps - 1) / warps), warps * 32, 0, st>>>(x, w, out, rows,
                                                                                dim, eps);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- head concat
// dst[r][g*hp + h][:] = src[g][r][h][:], copied in `unit`-byte pieces.
template <typename U>
__global__ void head_concat_kernel(const U* __restrict__ src, U* __restrict__ dst, int64_t shards,
                                   int64_t rows, int64_t hp, int64_t row_units) {
  const int64_t total = shards * rows * hp * row_units;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t u = i % row_units;
    int64_t t = i / row_units;
    const int64_t h = t % hp;
    t /= hp;
    const int64_t r = t % rows;
    const int64_t g = t / rows;
    dst[((r * shards + g) * hp + h) * row_units + u] = src[i];
  }
}

cudaError_t launch_head_concat(const void* src, void* dst, int64_t shards, int64_t rows,
                               int64_t heads_per, int64_t hd, int elem_bytes, cudaStream_t st) {
  const int64_t row_bytes = hd * elem_bytes;
  const int64_t total_bytes = shards * rows * heads_per * row_bytes;
  if (total_bytes == 0) return cudaSuccess;
  const int threads = 256;
  auto blocks_for = [&](int64_t n) {
    int64_t b = (n + threads - 1) / threads;
    return (unsigned)(b > 148 * 32 ? 148 * 32 : b);
  };
  if (row_bytes % 16 == 0 && (((uintptr_t)src | (uintptr_t)dst) & 15) == 0) {
    const int64_t ru = row_bytes / 16;
    head_concat_kernel<uint4><<<blocks_for(total_bytes / 16), threads, 0, st>>>(
        (const uint4*)src, (uint4*)dst, shards, rows, heads_per, ru);
  } else if (row_bytes % 4 == 0 && (((uintptr_t)src | (uintptr_t)dst) & 3) == 0) {
    head_concat_kernel<uint32_t><<<blocks_for(total_bytes / 4), threads, 0, st>>>(
        (const uint32_t*)src, (uint32_t*)dst, shards, rows, heads_per, row_bytes / 4);
  } else {
    head_concat_kernel<uint16_t><<<blocks_for(total_bytes / 2), threads, 0, st>>>(
        (const uint16_t*)src, (uint16_t*)dst, shards, rows, heads_per, row_bytes / 2);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- K/V prep
// One warp per (sequence, row, kv head, k|v). The row is staged in shared
// memory, transformed with the reference's op order (norm, then RoPE for k;
// norm for v; crates/eyebrowse-nn/src/attention.rs:62-76), rounded to the cache
// dtype and written to the cache (kv_write, :78-97) and/or the split planes.
constexpr int kPrepWarps = 4;

__global__ void __launch_bounds__(kPrepWarps * 32) prep_kv_kernel(PrepArgs a) {
  __shared__ float buf[kPrepWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t per_seq = (int64_t)a.rows * a.hkv * 2;
  const int64_t task = blockIdx.x * (int64_t)kPrepWarps + warp;
  if (task >= per_seq * a.batch) return;
  const int b = (int)(task / per_seq);
  int64_t t = task % per_seq;
  const int which = (int)(t & 1);  // 0 = k, 1 = v
  t >>= 1;
  const int head = (int)(t % a.hkv);
  const int r = (int)(t / a.hkv);
  const int hd = a.hd;
  const int pos = (a.positions ? a.positions[b] : a.pos0) + r;
  const void* src = which ? a.v : a.k;
  const int64_t src_off = b * a.kv_bstride + (int64_t)r * a.kv_stride + (int64_t)head * hd;
  float* row = buf[warp];
  for (int d = lane; d < hd; d += 32) row[d] = ld_any(src, src_off + d, a.dtype_kv);
  __syncwarp();
  if (which == 0) {
    warp_row_norm(row, hd, a.k_norm_w, a.eps, lane);
    if (a.cos_t)
      warp_row_rope(row, hd, a.cos_t + (int64_t)pos * (hd / 2), a.sin_t + (int64_t)pos * (hd / 2),
                    lane);
  } else {
    warp_row_norm(row, hd, a.v_norm_w, a.eps, lane);
  }
  void* cache = which ? a.vcache : a.kcache;
  const int64_t crow = ((int64_t)pos * a.hkv + head) * hd;
  const int64_t plane = (int64_t)a.rows * a.hkv * hd;
  __half* hi = a.split ? reinterpret_cast<__half*>(a.split) + (which ? 2 * plane : 0) : nullptr;
  const int64_t srow = ((int64_t)r * a.hkv + head) * hd;
  for (int d = lane; d < hd; d += 32) {
    const float x = round_to(row[d], a.dtype_cache);
    if (cache) st_any(cache, b * a.cache_bstride + crow + d, a.dtype_cache, x);
    if (hi) {
      const __half h = __float2half_rn(x);
      const __half l = __float2half_rn(x - __half2float(h));
      hi[srow + d] = h;
      hi[plane + srow + d] = l;
    }
  }
}

// Vectorised K/V prep for head_dim = 32*E (64/128/256): RPW rows per warp,
// all loads issued before any math (row helpers in eb_rowops.cuh).
template <int E>
__global__ void __launch_bounds__(256) prep_kv_vec_kernel(PrepArgs a) {
  constexpr int HD = 32 * E;
  constexpr int RPW = 4;
  const int lane = threadIdx.x & 31;
  const int64_t warp_id = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t per_seq = (int64_t)a.rows * a.hkv * 2;
  const int64_t total = per_seq * a.batch;
  float x[RPW][E];
  int64_t task[RPW];
#pragma unroll
  for (int i = 0; i < RPW; i++) {
    task[i] = warp_id * RPW + i;
    if (task[i] < total) {
      const int64_t b = task[i] / per_seq;
      int64_t t = task[i] % per_seq;
      const int which = (int)(t & 1);
      t >>= 1;
      const int head = (int)(t % a.hkv);
      const int r = (int)(t / a.hkv);
      ld_row<E>(which ? a.v : a.k,
                b * a.kv_bstride + (int64_t)r * a.kv_stride + (int64_t)head * HD + lane * E,
                a.dtype_kv, x[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < RPW; i++) {
    if (task[i] >= total) break;
    const int64_t b = task[i] / per_seq;
    int64_t t = task[i] % per_seq;
    const int which = (int)(t & 1);
    t >>= 1;
    const int head = (int)(t % a.hkv);
    const int r = (int)(t / a.hkv);
    const int pos = (a.positions ? a.positions[b] : a.pos0) + r;
    float* v = x[i];
    warp_kv_row<E>(x[i], which ? a.v_norm_w : a.k_norm_w, a.eps,
                   (!which && a.cos_t) ? a.cos_t + (int64_t)pos * (HD / 2) : nullptr,
                   (!which && a.cos_t) ? a.sin_t + (int64_t)pos * (HD / 2) : nullptr, lane);
#pragma unroll
    for (int e = 0; e < E; e++) v[e] = round_to(v[e], a.dtype_cache);
    void* cache = which ? a.vcache : a.kcache;
    if (cache)
      st_row<E>(cache, b * a.cache_bstride + ((int64_t)pos * a.hkv + head) * HD + lane * E,
                a.dtype_cache, x[i]);
    if (a.split) {
      const int64_t plane = (int64_t)a.rows * a.hkv * HD;
      __half* hi = reinterpret_cast<__half*>(a.split) + (which ? 2 * plane : 0);
      float fh[E], fl[E];
#pragma unroll
      for (int e = 0; e < E; e++) {
        fh[e] = __half2float(__float2half_rn(v[e]));
        fl[e] = v[e] - fh[e];
      }
      const int64_t srow = ((int64_t)r * a.hkv + head) * HD + lane * E;
      st_row<E>(hi, srow, kF16, fh);
      st_row<E>(hi + plane, srow, kF16, fl);
    }
  }
}

cudaError_t launch_prep_kv(const PrepArgs& a, cudaStream_t st) {
  const int64_t tasks = (int64_t)a.rows * a.hkv * 2 * a.batch;
  if (tasks == 0) return cudaSuccess;
  const int es_in = a.dtype_kv == kF32 ? 4 : 2;
  const bool aligned = ((a.kv_stride * es_in) % 16 == 0) && ((a.kv_bstride * es_in) % 16 == 0) &&
                       ((reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v)) & 15) == 0;
  if (aligned && (a.hd == 64 || a.hd == 128 || a.hd == 256)) {
    const int64_t warps = (tasks + 3) / 4;
    const unsigned blocks = (unsigned)((warps * 32 + 255) / 256);
    if (a.hd == 64) prep_kv_vec_kernel<2><<<blocks, 256, 0, st>>>(a);
    else if (a.hd == 128) prep_kv_vec_kernel<4><<<blocks, 256, 0, st>>>(a);
    else prep_kv_vec_kernel<8><<<blocks, 256, 0, st>>>(a);
    return cudaGetLastError();
  }
  prep_kv_kernel<<<(unsigned)((tasks + kPrepWarps - 1) / kPrepWarps), kPrepWarps * 32, 0, st>>>(a);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- SIMT attention
// One warp per (sequence, query row, query head): online softmax over keys
// 0..=pos with the dot product split across lanes by dimension. Arithmetic
// order differs from the reference's two-pass loop only by the usual
// online-softmax rescaling (crates/eyebrowse-kernels/src/attention.rs:33-48
// uses the same online form).
constexpr int kSimtWarps = 4;

__global__ void __launch_bounds__(kSimtWarps * 32) attn_simt_kernel(SimtArgs a) {
  __shared__ float qbuf[kSimtWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t per_seq = (int64_t)a.rows * a.H;
  const int64_t task = blockIdx.x * (int64_t)kSimtWarps + warp;
  if (task >= per_seq * a.batch) return;
  const int b = (int)(task / per_seq);
  const int64_t t = task % per_seq;
  const int h = (int)(t % a.H);
  const int i = (int)(t / a.H);
  const int hd = a.hd;
  const int kvh = h / (a.H / a.Hkv);
  const int pos = (a.positions ? a.positions[b] : a.qpos0) + i;
  float* qr = qbuf[warp];
  const int64_t qoff = b * a.q_bstride + (int64_t)i * a.q_stride + (int64_t)h * hd;
  for (int d = lane; d < hd; d += 32) qr[d] = ld_any(a.q, qoff + d, a.dtype_q);
  __syncwarp();
  warp_row_norm(qr, hd, a.q_norm_w, a.eps, lane);
  if (a.cos_t)
    warp_row_rope(qr, hd, a.cos_t + (int64_t)pos * (hd / 2), a.sin_t + (int64_t)pos * (hd / 2),
                  lane);
  constexpr int EPL = 8;  // hd <= 256
  float qv[EPL], acc[EPL];
#pragma unroll
  for (int e = 0; e < EPL; e++) {
    const int d = lane + 32 * e;
    qv[e] = d < hd ? qr[d] : 0.f;
    acc[e] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int64_t kbase = b * a.kv_bstride + (int64_t)kvh * hd;
  for (int j = 0; j <= pos; j++) {
    const int64_t ko = kbase + (int64_t)j * a.kv_stride;
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; e++) {
      const int d = lane + 32 * e;
      if (d < hd) s = fmaf(qv[e], ld_any(a.k, ko + d, a.dtype_kv), s);
    }
    s = warp_sum(s) * a.scale;
    const float mn = fmaxf(m, s);
    const float corr = __expf(m - mn);
    const float p = __expf(s - mn);
    l = l * corr + p;
#pragma unroll
    for (int e = 0; e < EPL; e++) {
      const int d = lane + 32 * e;
      if (d < hd) acc[e] = acc[e] * corr + p * ld_any(a.v, ko + d, a.dtype_kv);
    }
    m = mn;
  }
  const float inv = 1.f / l;
  const int64_t ooff = b * a.o_bstride + (int64_t)i * a.o_stride + (int64_t)h * hd;
#pragma unroll
  for (int e = 0; e < EPL; e++) {
    const int d = lane + 32 * e;
    if (d < hd) st_any(a.o, ooff + d, a.dtype_o, acc[e] * inv);
  }
}

cudaError_t launch_attn_simt(const SimtArgs& a, cudaStream_t st) {
  const int64_t tasks = (int64_t)a.rows * a.H * a.batch;
  if (tasks == 0) return cudaSuccess;
  attn_simt_kernel<<<(unsigned)((tasks + kSimtWarps - 1) / kSimtWarps), kSimtWarps * 32, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace eb
