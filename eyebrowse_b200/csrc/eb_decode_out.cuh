// eb_decode_out.cuh -- where a decode kernel's output rows go: the caller's
// o [B][H][hd], or with a head gather (a.n_dst > 0) every rank's gathered
// buffer [rows][heads][hd] (this GPU's and its peers', mapped here), at row
// seq_idx[b] (b when seq_idx is null) and head dst_h_off + h. The peer
// buffers are written with plain stores over NVLink.
#pragma once

#include "eb_common.cuh"
#include "eb_kernels.cuh"
#include "eb_rowops.cuh"

namespace eb {

__device__ __forceinline__ int64_t dec_dst_index(const DecodeArgs& a, int b, int h, int hd, int d) {
  const int64_t row = a.seq_idx ? (int64_t)a.seq_idx[b] : (int64_t)b;
  return row * a.dst_bstride + (int64_t)(a.dst_h_off + h) * hd + d;
}

// One output element (threads of a warp write consecutive d: coalesced).
__device__ __forceinline__ void dec_store(const DecodeArgs& a, int b, int h, int hd, int d,
                                          float v) {
  if (a.n_dst == 0) {
    st_any(a.o, (int64_t)b * a.o_bstride + (int64_t)h * hd + d, a.dtype_o, v);
    return;
  }
  const int64_t i = dec_dst_index(a, b, h, hd, d);
  for (int k = 0; k < a.n_dst; k++) st_any(reinterpret_cast<void*>(a.dst[k]), i, a.dtype_o, v);
}

// 32 consecutive output elements of one row held by one thread: 16-byte
// stores where the destination is aligned (one 128-byte or 64-byte run per
// destination), element stores otherwise.
__device__ __forceinline__ void dec_store32(const DecodeArgs& a, int b, int h, int hd, int d0,
                                            const float (&v)[32]) {
  const int n = a.n_dst == 0 ? 1 : a.n_dst;
  const int es = a.dtype_o == kF32 ? 4 : 2;
  for (int k = 0; k < n; k++) {
    void* base = a.n_dst == 0 ? a.o : reinterpret_cast<void*>(a.dst[k]);
    const int64_t i = a.n_dst == 0 ? (int64_t)b * a.o_bstride + (int64_t)h * hd + d0
                                   : dec_dst_index(a, b, h, hd, d0);
    char* p = static_cast<char*>(base) + i * es;
    if ((reinterpret_cast<uintptr_t>(p) & 15) != 0) {
#pragma unroll
      for (int e = 0; e < 32; e++) st_any(base, i + e, a.dtype_o, v[e]);
      continue;
    }
    uint4* q = reinterpret_cast<uint4*>(p);
    if (a.dtype_o == kF32) {
#pragma unroll
      for (int w = 0; w < 8; w++)
        q[w] = make_uint4(__float_as_uint(v[4 * w]), __float_as_uint(v[4 * w + 1]),
                          __float_as_uint(v[4 * w + 2]), __float_as_uint(v[4 * w + 3]));
    } else {
      const bool bf = a.dtype_o == kBF16;
#pragma unroll
      for (int w = 0; w < 4; w++) {
        uint32_t u[4];
#pragma unroll
        for (int k2 = 0; k2 < 4; k2++)
          u[k2] = bf ? pack_bf162(v[8 * w + 2 * k2], v[8 * w + 2 * k2 + 1])
                     : pack_half2(v[8 * w + 2 * k2], v[8 * w + 2 * k2 + 1]);
        q[w] = make_uint4(u[0], u[1], u[2], u[3]);
      }
    }
  }
}

}  // namespace eb
