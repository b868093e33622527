// eb_tc.cuh -- pieces shared by the tcgen05 attention kernels (prefill and
// decode): 16-bit operand chunk stores, f32 hi/lo splitting, a bounded drain
// wait, and host-side tensor-map encoding for the KV cache.
#pragma once

#include <cudaTypedefs.h>

#include "eb_common.cuh"

namespace eb {

// Tensor-memory allocations are powers of two of at least 32 columns.
constexpr int constexpr_pow2ceil(int x) {
  int p = 32;
  while (p < x) p <<= 1;
  return p;
}

// A row's running max only moves (and O is only rescaled) when the new tile's
// max exceeds it by more than this, in log2 units: p <= 2^8 stays exact in
// f16/bf16 and in the f32 accumulators, and O/l is unaffected.
constexpr float kRescaleThreshold = 8.0f;

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ void load8_any(const void* p, int64_t idx, int dt, float (&f)[8]) {
  if (dt == kF32) {
    const float4* v = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + idx);
    const float4 a = v[0], b = v[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else if (dt == kF16) {
    const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(p) + idx);
    const __half* h = reinterpret_cast<const __half*>(&u);
#pragma unroll
    for (int i = 0; i < 8; i++) f[i] = __half2float(h[i]);
  } else {
    const uint4 u =
        *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p) + idx);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int i = 0; i < 8; i++) f[i] = __bfloat162float(h[i]);
  }
}

// 8 floats -> one 16-byte chunk of 16-bit operands at a shared address.
template <bool BF16>
__device__ __forceinline__ void st_chunk(uint32_t saddr, const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; i++)
    w[i] = BF16 ? pack_bf162(f[2 * i], f[2 * i + 1]) : pack_half2(f[2 * i], f[2 * i + 1]);
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(saddr), "r"(w[0]), "r"(w[1]),
               "r"(w[2]), "r"(w[3])
               : "memory");
}
// hi / lo split of 8 floats into two chunks.
__device__ __forceinline__ void st_chunk_split(uint32_t s_hi, uint32_t s_lo, const float (&f)[8]) {
  float hi[8], lo[8];
#pragma unroll
  for (int i = 0; i < 8; i++) {
    hi[i] = __half2float(__float2half_rn(f[i]));
    lo[i] = f[i] - hi[i];
  }
  st_chunk<false>(s_hi, hi);
  st_chunk<false>(s_lo, lo);
}

__device__ __forceinline__ bool mbar_drain(uint32_t bar, uint32_t parity, unsigned* err,
                                           unsigned bit) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (;;) {
    for (int i = 0; i < 32; i++)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      atomicOr(err, bit);
      return false;
    }
  }
}



// Host: cuTensorMapEncodeTiled from the driver, looked up once.
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();
// Host: 3-D map over a [S][Hkv][hd] 16-bit tensor, box {64, 1, BN}, 128-byte swizzle.
bool make_kv_map(CUtensorMap* m, const void* base, int S, int Hkv, int hd, int BN, bool bf16);

}  // namespace eb
