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

}  // namespace eb
