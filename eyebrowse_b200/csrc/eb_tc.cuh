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

// Packed f32x2 arithmetic (one instruction, two lanes of the FMA pipe).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x0, 2^x1 for x <= 0 on the FMA pipe instead of the MUFU unit, for the
// softmax exponentials whose MUFU throughput (16 per clock per SM, shared
// with the f32 -> f16x2 conversions) otherwise bounds the prefill loop.
// x = j + f with j = rint(x) (adding and removing 1.5 * 2^23 rounds to an
// integer and leaves j in the low mantissa bits), |f| <= 1/2, and
// 2^f ~= c0 + f (c1 + f (c2 + f c3)): a degree-3 minimax fit of 2^f on
// [-1/2, 1/2] for relative error (7.5e-5 at most, measured in f32 Horner
// form), below the 2^-11 rounding of the 16-bit P these values become.
// 2^j is applied by adding j to the exponent field: the low 9 bits of the
// rounding constant's encoding are zero, so (bits(r) << 23) == j << 23.
// Inputs are clamped to -125 first (masked -inf included), whose result
// ~2^-125 rounds to zero in 16 bits.
__device__ __forceinline__ void ex2_fma_pair(float x0, float x1, float& y0, float& y1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  constexpr float c0 = 0.99992806f, c1 = 0.69326097f, c2 = 0.24261114f, c3 = 0.05517168f;
  const uint64_t x = f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t r = f2_add(x, f2_pack(kRound, kRound));
  const uint64_t jf = f2_add(r, f2_pack(-kRound, -kRound));
  const uint64_t f = f2_fma(jf, f2_pack(-1.f, -1.f), x);  // exact: |f| <= 1/2
  uint64_t p = f2_fma(f2_pack(c3, c3), f, f2_pack(c2, c2));
  p = f2_fma(p, f, f2_pack(c1, c1));
  p = f2_fma(p, f, f2_pack(c0, c0));
  float p0, p1, r0, r1;
  f2_unpack(p, p0, p1);
  f2_unpack(r, r0, r1);
  y0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(r0) << 23));
  y1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(r1) << 23));
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
