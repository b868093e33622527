// eb_rowops.cuh -- runtime-dtype element access and warp-cooperative per-head
// row transforms (RMSNorm, half-split RoPE) on a row staged in shared memory.
#pragma once

#include "eb_common.cuh"

namespace eb {

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

__device__ __forceinline__ float ld_any(const void* p, int64_t i, int dt) {
  if (dt == kF16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  if (dt == kBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void st_any(void* p, int64_t i, int dt, float x) {
  if (dt == kF16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(x);
  else if (dt == kBF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else reinterpret_cast<float*>(p)[i] = x;
}
// The value a store of x in dtype dt keeps.
__device__ __forceinline__ float round_to(float x, int dt) {
  if (dt == kF16) return __half2float(__float2half_rn(x));
  if (dt == kBF16) return __bfloat162float(__float2bfloat16_rn(x));
  return x;
}

// In-place RMSNorm of a row of `hd` floats in shared memory, reference
// arithmetic per element (crates/eyebrowse-kernels/src/rmsnorm.rs:34-36):
// inv = 1/sqrt(sum(x^2)/dim + eps); out = (x * inv) * w. The sum of squares
// is a warp tree, so it is not bit-identical to the reference's loop.
__device__ __forceinline__ void warp_row_norm(float* row, int hd, const float* w, float eps,
                                              int lane) {
  if (!w) return;
  float ss = 0.f;
  for (int d = lane; d < hd; d += 32) ss = __fadd_rn(ss, __fmul_rn(row[d], row[d]));
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / (float)hd + eps);
  for (int d = lane; d < hd; d += 32) row[d] = __fmul_rn(__fmul_rn(row[d], inv), w[d]);
  __syncwarp();
}

// In-place half-split RoPE of a row in shared memory with one table row
// (crates/eyebrowse-kernels/src/rope.rs:25-30): the lane that owns pair p
// reads and writes both p and p + hd/2, so no two lanes touch one element.
__device__ __forceinline__ void warp_row_rope(float* row, int hd, const float* cos_row,
                                              const float* sin_row, int lane) {
  const int half = hd / 2;
  for (int p = lane; p < half; p += 32) {
    const float c = cos_row[p], s = sin_row[p];
    const float x1 = row[p], x2 = row[p + half];
    row[p] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    row[p + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  }
  __syncwarp();
}

// Register rows of head_dim = 32*E (64/128/256) held across a warp: lane l
// holds elements [l*E, l*E+E), and the RoPE partner of a first-half element
// sits in lane l^16 at the same slot.
template <int E>
__device__ __forceinline__ void ld_row(const void* p, int64_t i, int dt, float (&f)[E]) {
  if (dt == kF32) {
    const float* q = reinterpret_cast<const float*>(p) + i;
    if constexpr (E % 4 == 0) {
#pragma unroll
      for (int k = 0; k < E; k += 4) {
        const float4 v = *reinterpret_cast<const float4*>(q + k);
        f[k] = v.x; f[k + 1] = v.y; f[k + 2] = v.z; f[k + 3] = v.w;
      }
    } else {
      const float2 v = *reinterpret_cast<const float2*>(q);
      f[0] = v.x; f[1] = v.y;
    }
  } else {
    const uint16_t* q = reinterpret_cast<const uint16_t*>(p) + i;
    uint32_t w[E / 2];
    if constexpr (E == 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(q);
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else if constexpr (E == 4) {
      const uint2 v = *reinterpret_cast<const uint2*>(q);
      w[0] = v.x; w[1] = v.y;
    } else {
      w[0] = *reinterpret_cast<const uint32_t*>(q);
    }
#pragma unroll
    for (int k = 0; k < E / 2; k++) {
      if (dt == kF16) {
        const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
        f[2 * k] = t.x; f[2 * k + 1] = t.y;
      } else {
        const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
        f[2 * k] = t.x; f[2 * k + 1] = t.y;
      }
    }
  }
}

template <int E>
__device__ __forceinline__ void st_row(void* p, int64_t i, int dt, const float (&f)[E]) {
  if (dt == kF32) {
    float* q = reinterpret_cast<float*>(p) + i;
    if constexpr (E % 4 == 0) {
#pragma unroll
      for (int k = 0; k < E; k += 4)
        *reinterpret_cast<float4*>(q + k) = make_float4(f[k], f[k + 1], f[k + 2], f[k + 3]);
    } else {
      *reinterpret_cast<float2*>(q) = make_float2(f[0], f[1]);
    }
  } else {
    uint32_t w[E / 2];
#pragma unroll
    for (int k = 0; k < E / 2; k++)
      w[k] = dt == kF16 ? pack_half2(f[2 * k], f[2 * k + 1]) : pack_bf162(f[2 * k], f[2 * k + 1]);
    uint16_t* q = reinterpret_cast<uint16_t*>(p) + i;
    if constexpr (E == 8) *reinterpret_cast<uint4*>(q) = make_uint4(w[0], w[1], w[2], w[3]);
    else if constexpr (E == 4) *reinterpret_cast<uint2*>(q) = make_uint2(w[0], w[1]);
    else *reinterpret_cast<uint32_t*>(q) = w[0];
  }
}


// One k or v head row held across the warp (layout above): RMSNorm with
// weight w (if non-null), then half-split RoPE with one table row (if
// non-null), both with the reference's per-element f32 arithmetic
// (crates/eyebrowse-kernels/src/rmsnorm.rs:34-36, rope.rs:25-30).
template <int E>
__device__ __forceinline__ void warp_kv_row(float (&v)[E], const float* w, float eps,
                                            const float* cos_row, const float* sin_row, int lane) {
  constexpr int HD = 32 * E;
  if (w) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; e++) ss = __fadd_rn(ss, __fmul_rn(v[e], v[e]));
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)HD + eps);
#pragma unroll
    for (int e = 0; e < E; e++) v[e] = __fmul_rn(__fmul_rn(v[e], inv), w[lane * E + e]);
  }
  if (cos_row) {
    const float* cr = cos_row + (lane & 15) * E;
    const float* sr = sin_row + (lane & 15) * E;
#pragma unroll
    for (int e = 0; e < E; e++) {
      const float other = __shfl_xor_sync(0xffffffffu, v[e], 16);
      const float c = cr[e], sn = sr[e];
      v[e] = lane < 16 ? __fsub_rn(__fmul_rn(v[e], c), __fmul_rn(other, sn))
                       : __fadd_rn(__fmul_rn(v[e], c), __fmul_rn(other, sn));
    }
  }
}

}  // namespace eb
