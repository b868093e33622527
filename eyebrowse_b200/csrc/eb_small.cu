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
    if (blocks > sm_count() * 16) blocks = sm_count() * 16;
    kv_write_kernel_v4<<<(unsigned)blocks, threads, 0, st>>>(
        reinterpret_cast<float4*>(dst), reinterpret_cast<const float4*>(src), n4);
  } else {
    int64_t blocks = (n + threads - 1) / threads;
    if (blocks > sm_count() * 16) blocks = sm_count() * 16;
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
    return (unsigned)(b > (int64_t)sm_count() * 32 ? (int64_t)sm_count() * 32 : b);
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

// ---------------------------------------------------------------- head broadcast
// Rows x heads [h0, h0 + nh) of a gathered [rows][H][hd] buffer, stored through
// an NVLink multicast address (multimem.st): the switch writes every 16-byte
// word to the same offset of each GPU's buffer bound to the multicast object,
// so each word leaves this GPU once whatever the number of GPUs.
__global__ void head_broadcast_kernel(const char* __restrict__ src, char* mc, int64_t rows,
                                      int64_t row_bytes, int64_t off_bytes, int64_t span16) {
  const int64_t total = rows * span16;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / span16, u = i - r * span16;
    const int64_t o = r * row_bytes + off_bytes + u * 16;
    const uint4 v = *reinterpret_cast<const uint4*>(src + o);
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc + o),
                 "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
                 "f"(__uint_as_float(v.w))
                 : "memory");
  }
}

cudaError_t launch_head_broadcast(const void* local, void* mc, int64_t rows, int64_t h_total,
                                  int64_t h0, int64_t nh, int64_t hd, int elem_bytes,
                                  cudaStream_t st) {
  const int64_t span16 = nh * hd * elem_bytes / 16;
  if (rows == 0 || span16 == 0) return cudaSuccess;
  const int64_t total = rows * span16;
  const int threads = 512;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > sm_count() * 4) blocks = sm_count() * 4;
  head_broadcast_kernel<<<(unsigned)blocks, threads, 0, st>>>(
      static_cast<const char*>(local), static_cast<char*>(mc), rows, h_total * hd * elem_bytes,
      h0 * hd * elem_bytes, span16);
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
  const int nk = a.v ? 2 : 1;  // k and v rows, or k rows only
  const int64_t per_seq = (int64_t)a.rows * a.hkv * nk;
  const int64_t task = blockIdx.x * (int64_t)kPrepWarps + warp;
  if (task >= per_seq * a.batch) return;
  const int b = (int)(task / per_seq);
  int64_t t = task % per_seq;
  const int which = nk == 2 ? (int)(t & 1) : 0;  // 0 = k, 1 = v
  t >>= (nk - 1);
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

// Row prep for head_dim 64/128/256 with inputs of ES bytes per element: one
// warp takes HPW consecutive heads of one token row of k (or v), which are
// contiguous in memory. A lane owns 8 consecutive elements of a head row
// (16-byte loads for 16-bit inputs), LPR = HD/8 lanes share a head row, and
// all of the warp's loads (HPW head rows, one RoPE table row, this lane's
// norm weights) are in flight together. The RMSNorm sum of squares is a
// butterfly over the row's lanes; the RoPE partner chunk (HD/2 elements
// away) is LPR/2 lanes away. Per-element arithmetic as in warp_kv_row.
template <int HD, int HPW, int ES>
__global__ void __launch_bounds__(128) prep_rows_kernel(PrepArgs a) {
  constexpr int LPR = HD / 8;            // lanes per head row
  constexpr int RPI = 32 / LPR;          // head rows per warp instruction
  constexpr int NI = (HPW + RPI - 1) / RPI;
  constexpr int NW = ES == 4 ? 2 : 1;    // 16-byte words per lane per head row
  const int lane = threadIdx.x & 31;
  const int64_t warp_id = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int nk = a.v ? 2 : 1;  // k and v rows, or k rows only
  const int n_g = a.hkv / HPW;
  const int per_seq = a.rows * n_g * nk;
  if (warp_id >= (int64_t)per_seq * a.batch) return;
  const int b = (int)(warp_id / per_seq);
  int rem = (int)(warp_id - (int64_t)b * per_seq);
  const int which = nk == 2 ? (rem & 1) : 0;
  rem >>= (nk - 1);
  const int g = rem % n_g;
  const int r = rem / n_g;
  const int pos = (a.positions ? a.positions[b] : a.pos0) + r;
  const int c8 = (lane % LPR) * 8;
  const int hsub = lane / LPR;
  const void* src = which ? a.v : a.k;
  const int64_t base = b * a.kv_bstride + (int64_t)r * a.kv_stride + (int64_t)g * HPW * HD + c8;
  uint4 raw[NI][NW];
#pragma unroll
  for (int i = 0; i < NI; i++) {
    if (i * RPI + hsub < HPW) {
      const uint4* p = reinterpret_cast<const uint4*>(static_cast<const char*>(src) +
                                                      (base + (int64_t)(i * RPI + hsub) * HD) * ES);
#pragma unroll
      for (int w = 0; w < NW; w++) raw[i][w] = p[w];
    }
  }
  const float* wn = which ? a.v_norm_w : a.k_norm_w;
  float wt[8], cs[8], sn[8];
  if (wn) {
    const float4 w0 = *reinterpret_cast<const float4*>(wn + c8);
    const float4 w1 = *reinterpret_cast<const float4*>(wn + c8 + 4);
    wt[0] = w0.x; wt[1] = w0.y; wt[2] = w0.z; wt[3] = w0.w;
    wt[4] = w1.x; wt[5] = w1.y; wt[6] = w1.z; wt[7] = w1.w;
  }
  const bool rope = !which && a.cos_t;
  if (rope) {
    const int64_t off = (int64_t)pos * (HD / 2) + (c8 % (HD / 2));
    const float4 c0 = *reinterpret_cast<const float4*>(a.cos_t + off);
    const float4 c1 = *reinterpret_cast<const float4*>(a.cos_t + off + 4);
    const float4 s0 = *reinterpret_cast<const float4*>(a.sin_t + off);
    const float4 s1 = *reinterpret_cast<const float4*>(a.sin_t + off + 4);
    cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w;
    cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
    sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
    sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
  }
  const bool first_half = c8 < HD / 2;
  void* cache = which ? a.vcache : a.kcache;
#pragma unroll
  for (int i = 0; i < NI; i++) {
    const int hl = i * RPI + hsub;  // head within the group (lanes past HPW idle)
    float x[8];
    if (ES == 4) {
      const float* f = reinterpret_cast<const float*>(&raw[i][0]);
#pragma unroll
      for (int k = 0; k < 8; k++) x[k] = f[k];
    } else {
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw[i][0]);
#pragma unroll
      for (int k = 0; k < 4; k++) {
        float2 t;
        if (a.dtype_kv == kF16) t = __half22float2(*reinterpret_cast<const __half2*>(&u[k]));
        else t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[k]));
        x[2 * k] = t.x;
        x[2 * k + 1] = t.y;
      }
    }
    if (hl >= HPW) {
#pragma unroll
      for (int k = 0; k < 8; k++) x[k] = 0.f;
    }
    if (wn) {
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < 8; k++) ss = __fadd_rn(ss, __fmul_rn(x[k], x[k]));
#pragma unroll
      for (int off = 1; off < LPR; off <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float inv = 1.0f / sqrtf(ss / (float)HD + a.eps);
#pragma unroll
      for (int k = 0; k < 8; k++) x[k] = __fmul_rn(__fmul_rn(x[k], inv), wt[k]);
    }
    if (rope) {
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const float o = __shfl_xor_sync(0xffffffffu, x[k], LPR / 2);
        x[k] = first_half ? __fsub_rn(__fmul_rn(x[k], cs[k]), __fmul_rn(o, sn[k]))
                          : __fadd_rn(__fmul_rn(x[k], cs[k]), __fmul_rn(o, sn[k]));
      }
    }
    if (hl >= HPW) continue;
    const int head = g * HPW + hl;
#pragma unroll
    for (int k = 0; k < 8; k++) x[k] = round_to(x[k], a.dtype_cache);
    if (cache)
      st_row<8>(cache, b * a.cache_bstride + ((int64_t)pos * a.hkv + head) * HD + c8,
                a.dtype_cache, x);
    if (a.split) {
      const int64_t plane = (int64_t)a.rows * a.hkv * HD;
      __half* hi = reinterpret_cast<__half*>(a.split) + (which ? 2 * plane : 0);
      float fh[8], fl[8];
#pragma unroll
      for (int k = 0; k < 8; k++) {
        fh[k] = __half2float(__float2half_rn(x[k]));
        fl[k] = x[k] - fh[k];
      }
      const int64_t srow = ((int64_t)r * a.hkv + head) * HD + c8;
      st_row<8>(hi, srow, kF16, fh);
      st_row<8>(hi + plane, srow, kF16, fl);
    }
  }
}

template <int HD, int ES>
static void launch_prep_rows(const PrepArgs& a, int hpw, cudaStream_t st) {
  const int64_t warps = (int64_t)a.rows * (a.hkv / hpw) * (a.v ? 2 : 1) * a.batch;
  const unsigned blocks = (unsigned)((warps + 3) / 4);
  switch (hpw) {
    case 16: prep_rows_kernel<HD, 16, ES><<<blocks, 128, 0, st>>>(a); break;
    case 8: prep_rows_kernel<HD, 8, ES><<<blocks, 128, 0, st>>>(a); break;
    case 4: prep_rows_kernel<HD, 4, ES><<<blocks, 128, 0, st>>>(a); break;
    case 2: prep_rows_kernel<HD, 2, ES><<<blocks, 128, 0, st>>>(a); break;
    default: prep_rows_kernel<HD, 1, ES><<<blocks, 128, 0, st>>>(a); break;
  }
}

cudaError_t launch_prep_kv(const PrepArgs& a, cudaStream_t st) {
  const int64_t tasks = (int64_t)a.rows * a.hkv * (a.v ? 2 : 1) * a.batch;
  if (tasks == 0) return cudaSuccess;
  const int es_in = a.dtype_kv == kF32 ? 4 : 2;
  const int es_c = a.dtype_cache == kF32 ? 4 : 2;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool aligned = ((a.kv_stride * es_in) % 16 == 0) && ((a.kv_bstride * es_in) % 16 == 0) &&
                       ((a.cache_bstride * es_c) % 16 == 0) && al16(a.k) && al16(a.v) &&
                       al16(a.kcache) && al16(a.vcache) && al16(a.split) &&
                       ((a.cos_t == nullptr) || (al16(a.cos_t) && al16(a.sin_t))) &&
                       al16(a.k_norm_w) && al16(a.v_norm_w);
  if (aligned && (a.hd == 64 || a.hd == 128 || a.hd == 256)) {
    // heads per warp: the largest power of two up to 16 (8 for head_dim 256)
    // that divides the head count
    int hpw = a.hd == 256 ? 8 : 16;
    while (a.hkv % hpw) hpw >>= 1;
    if (a.hd == 64) es_in == 4 ? launch_prep_rows<64, 4>(a, hpw, st) : launch_prep_rows<64, 2>(a, hpw, st);
    else if (a.hd == 128) es_in == 4 ? launch_prep_rows<128, 4>(a, hpw, st) : launch_prep_rows<128, 2>(a, hpw, st);
    else es_in == 4 ? launch_prep_rows<256, 4>(a, hpw, st) : launch_prep_rows<256, 2>(a, hpw, st);
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
  const int j_lo = a.window > 0 ? max(0, pos - a.window + 1) : 0;
  for (int j = j_lo; j <= pos; j++) {
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
