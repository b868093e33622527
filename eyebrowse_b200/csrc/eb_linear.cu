// eb_linear.cu -- the projections around the attention path: linear_f16w,
// y[m, o] = sum_k x[m, k] * w[o, k], with f32 activations x [m, in], f16
// weights w [out, in] (HF Linear layout; the reference's packed-u32 f16 pairs
// are these bytes), f32 accumulation and f32 y.
// Replaces linear_f16w (crates/eyebrowse-kernels/src/matmul.rs:84-149), the
// GEMM behind eyebrowse-nn Linear (crates/eyebrowse-nn/src/linear.rs:17-22):
// the q/k/v/o projections, the MLP and the tied LM head.
//
// Three kernels, chosen by the host:
// - linear_rows_kernel (m <= 8: decode steps, the LM head). HBM-bound on w:
//   each warp owns 1 or 4 output rows and streams them once with 16-byte
//   loads, 4 per row in flight per lane; x comes through L1. f32 FMA per
//   product, a warp reduction per output.
// - linear_tc_kernel (m > 8: prefill). tcgen05 with f32 accumulation in
//   TMEM, 128 x 256 output tiles, a 3-stage TMA ring over 64-wide k chunks.
//   x is first split into f16 hi and lo planes (split_x_kernel); every tile
//   accumulates x_hi w + x_lo w. The weights are exact in f16 and the two
//   planes carry ~22 bits of each activation's mantissa, so the products
//   keep f32-level accuracy (plain f16 activations would lose ~1e-4
//   relative). The f16 hi plane limits |x| to the f16 range (65504).
// - linear_scalar_kernel: any other shape (k not a multiple of 8, unaligned
//   pointers), one warp per output element.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "eb_common.cuh"
#include "eb_kernels.cuh"
#include "eb_rowops.cuh"
#include "eb_tc.cuh"

namespace eb {

// ---------------------------------------------------------------- m <= 8
// One warp owns R output rows over the whole k range: lane l takes the
// 8-element chunks l, l+32, ..., B chunks per row in flight per pass; a warp
// reduction finishes each dot product (no shared memory, no block barrier).
constexpr int kRowsWarps = 8;
constexpr int kRowsBatch = 4;

template <int MR, int R>
__global__ void __launch_bounds__(kRowsWarps * 32) linear_rows_kernel(const float* __restrict__ x,
                                                                      const __half* __restrict__ w,
                                                                      float* __restrict__ y, int m,
                                                                      int in_f, int out_f) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o0 = (blockIdx.x * kRowsWarps + warp) * R;
  if (o0 >= out_f) return;
  const int n_chunks = in_f / 8;
  float acc[R][MR];
#pragma unroll
  for (int r = 0; r < R; r++)
#pragma unroll
    for (int i = 0; i < MR; i++) acc[r][i] = 0.f;

  for (int c0 = lane; c0 < n_chunks; c0 += 32 * kRowsBatch) {
    uint4 wv[kRowsBatch][R];
#pragma unroll
    for (int u = 0; u < kRowsBatch; u++) {
      const int c = c0 + 32 * u;
#pragma unroll
      for (int r = 0; r < R; r++)
        wv[u][r] = (c < n_chunks && o0 + r < out_f)
                       ? ld_stream_u4(w + (int64_t)(o0 + r) * in_f + (int64_t)c * 8)
                       : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kRowsBatch; u++) {
      const int c = c0 + 32 * u;
      if (c >= n_chunks) break;
      float wf[R][8];
#pragma unroll
      for (int r = 0; r < R; r++) {
        const __half2* h2 = reinterpret_cast<const __half2*>(&wv[u][r]);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float2 f = __half22float2(h2[e]);
          wf[r][2 * e] = f.x;
          wf[r][2 * e + 1] = f.y;
        }
      }
#pragma unroll
      for (int i = 0; i < MR; i++) {
        if (i >= m) break;
        const float4* xp = reinterpret_cast<const float4*>(x + (int64_t)i * in_f + (int64_t)c * 8);
        const float4 xa = __ldg(xp), xb = __ldg(xp + 1);
        const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
          for (int e = 0; e < 8; e++) acc[r][i] = fmaf(xv[e], wf[r][e], acc[r][i]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; r++)
#pragma unroll
    for (int i = 0; i < MR; i++) {
      const float v = warp_sum(acc[r][i]);
      if (lane == 0 && i < m && o0 + r < out_f) y[(int64_t)i * out_f + o0 + r] = v;
    }
}

// ---------------------------------------------------------------- any shape
__global__ void __launch_bounds__(256) linear_scalar_kernel(const float* __restrict__ x,
                                                            const __half* __restrict__ w,
                                                            float* __restrict__ y, int m,
                                                            int in_f, int out_f) {
  const int64_t task = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (task >= (int64_t)m * out_f) return;
  const int i = (int)(task / out_f), o = (int)(task % out_f);
  float acc = 0.f;
  for (int k = lane; k < in_f; k += 32)
    acc = fmaf(x[(int64_t)i * in_f + k], __half2float(w[(int64_t)o * in_f + k]), acc);
  acc = warp_sum(acc);
  if (lane == 0) y[(int64_t)i * out_f + o] = acc;
}

// ---------------------------------------------------------------- m > 8
// x (f32) -> f16 hi plane and f16 lo plane (x - hi), 8 elements per step.
__global__ void __launch_bounds__(256) split_x_kernel(const float* __restrict__ x,
                                                      __half* __restrict__ hi,
                                                      __half* __restrict__ lo, int64_t n8) {
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n8;
       g += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(x) + 2 * g);
    const float4 b = __ldg(reinterpret_cast<const float4*>(x) + 2 * g + 1);
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const __half2 hh = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
      const float2 hf = __half22float2(hh);
      h[e] = *reinterpret_cast<const uint32_t*>(&hh);
      l[e] = pack_half2(v[2 * e] - hf.x, v[2 * e + 1] - hf.y);
    }
    reinterpret_cast<uint4*>(hi)[g] = make_uint4(h[0], h[1], h[2], h[3]);
    reinterpret_cast<uint4*>(lo)[g] = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

struct LinCfg {
  static constexpr int BM = 128, BN = 256, BK = 64, ST = 3;
  static constexpr int A_BYTES = BM * BK * 2;              // one f16 plane of x: 16 KB
  static constexpr int B_BYTES = BN * BK * 2;              // w: 32 KB
  static constexpr int STAGE = 2 * A_BYTES + B_BYTES;      // 64 KB
  static constexpr int BAR_OFF = ST * STAGE;               // 192 KB
  static constexpr int SMEM = BAR_OFF + 256 + 1024;        // barriers + alignment slack
  static constexpr int THREADS = 192;                      // producer, MMA, 4 epilogue warps
  static constexpr int BOX = BM * 128;                     // epilogue staging box: 128 rows x 32 f32
  static_assert(BN / 32 * BOX <= BAR_OFF, "epilogue staging fits the stages");
};

__global__ void __launch_bounds__(LinCfg::THREADS, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tmXhi,
                     const __grid_constant__ CUtensorMap tmXlo,
                     const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmY, int in_f, int out_f,
                     unsigned* err) {
  using C = LinCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::BAR_OFF + 128);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::BAR_OFF + 136);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  constexpr int kFull0 = 0, kEmpty0 = C::ST, kDone = 2 * C::ST;
  auto s_xhi = [&](int s) { return sbase + s * C::STAGE; };
  auto s_xlo = [&](int s) { return sbase + s * C::STAGE + C::A_BYTES; };
  auto s_w = [&](int s) { return sbase + s * C::STAGE + 2 * C::A_BYTES; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * C::BN, m0 = blockIdx.y * C::BM;
  const int n_k = (in_f + C::BK - 1) / C::BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::ST; i++) {
      mbar_init(bar(kFull0 + i), 1);
      mbar_init(bar(kEmpty0 + i), 1);
    }
    mbar_init(bar(kDone), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tmXhi);
    tma_prefetch_map(&tmXlo);
    tma_prefetch_map(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued[C::ST] = {};
      for (int c = 0; c < n_k; c++) {
        const int s = c % C::ST;
        if (c >= C::ST && !mbar_wait(bar(kEmpty0 + s), (c / C::ST - 1) & 1, abort_flag, err,
                                     kErrTimeoutTma))
          break;
        const uint32_t f = bar(kFull0 + s);
        mbar_arrive_expect_tx(f, C::STAGE);
        tma_load_2d(s_xhi(s), &tmXhi, f, c * C::BK, m0);
        tma_load_2d(s_xlo(s), &tmXlo, f, c * C::BK, m0);
        tma_load_2d(s_w(s), &tmW, f, c * C::BK, n0);
        issued[s]++;
      }
      // every issued copy has landed before the CTA can exit
      for (int s = 0; s < C::ST; s++)
        if (issued[s]) mbar_drain(bar(kFull0 + s), (issued[s] - 1) & 1, err, kErrTimeoutTma);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(C::BM, C::BN, false, false);
      for (int c = 0; c < n_k; c++) {
        const int s = c % C::ST;
        if (!mbar_wait(bar(kFull0 + s), (c / C::ST) & 1, abort_flag, err, kErrTimeoutMma)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C::BK / 16; kk++) {
          const uint64_t bd = sdesc_sw128(s_w(s) + kk * 32, 16, 1024);
          umma_ss(tmem, sdesc_sw128(s_xhi(s) + kk * 32, 16, 1024), bd, idesc,
                  (c > 0 || kk > 0) ? 1u : 0u);
          umma_ss(tmem, sdesc_sw128(s_xlo(s) + kk * 32, 16, 1024), bd, idesc, 1u);
        }
        umma_commit(bar(kEmpty0 + s));  // stage s free once these MMAs have read it
      }
      // every issued MMA has completed before TMEM is read or released
      umma_commit(bar(kDone));
      mbar_drain(bar(kDone), 0, err, kErrTimeoutMma);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // warps 2..5 read TMEM lanes 32*(warp%4).. : one output row per thread
    const int g = warp & 3;
    const int r = g * 32 + lane;
    bool ok = mbar_wait(bar(kDone), 0, abort_flag, err, kErrTimeoutEpilogue);
    __syncwarp();
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
      // D columns [32c, 32c+32) of row r -> staging box c (128 rows x 128 B,
      // the 128-byte-swizzled layout the store map reads); the stages are
      // free: every MMA that read them has completed.
#pragma unroll 1
      for (int c = 0; c < C::BN / 32; c++) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(g * 32) << 16) + c * 32, v);
        tmem_ld_wait();
        const uint32_t box = sbase + c * C::BOX;
#pragma unroll
        for (int i = 0; i < 8; i++)
          asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(box + sw128_offset(r, i)),
                       "r"(v[4 * i]), "r"(v[4 * i + 1]), "r"(v[4 * i + 2]), "r"(v[4 * i + 3])
                       : "memory");
      }
    }
    fence_async_smem();
    // all 128 epilogue threads have staged (every warp arrives, stores go out
    // only if every one succeeded); rows past m and columns past out_f fall
    // outside the map and are not written
    const bool tile_ok = named_bar_and(1, 128, ok);
    if (tile_ok && warp == 2 && lane == 0) {
      for (int c = 0; c < C::BN / 32; c++)
        if (n0 + c * 32 < out_f) tma_store_2d(&tmY, sbase + c * C::BOX, n0 + c * 32, m0);
      tma_store_commit();
      tma_store_wait_read();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::BN);
  }
}

// ---------------------------------------------------------------- host side
static bool make_2d_map(CUtensorMap* m, const void* base, CUtensorMapDataType ty, int es,
                        int64_t inner, int64_t rows, int box_inner, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(inner * es)};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, ty, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

LinearPath linear_path(int64_t m, int64_t in_f, int64_t out_f, bool aligned) {
  if (!aligned || in_f % 8 != 0) return LinearPath::kScalar;
  if (m <= 8) return LinearPath::kRows;
  if (out_f % 4 != 0) return LinearPath::kScalar;
  return LinearPath::kTensor;
}

size_t linear_workspace_bytes(int64_t m, int64_t in_f, int64_t out_f) {
  // f16 hi and lo planes of x, each 256-byte aligned
  if (linear_path(m, in_f, out_f, true) != LinearPath::kTensor) return 0;
  const size_t plane = ((size_t)m * in_f * sizeof(__half) + 255) / 256 * 256;
  return 2 * plane;
}

cudaError_t launch_linear(const float* x, const void* w, float* y, int64_t m, int64_t in_f,
                          int64_t out_f, void* ws, LinearPath path, unsigned* err,
                          cudaStream_t st) {
  const __half* wh = static_cast<const __half*>(w);
  if (path == LinearPath::kScalar) {
    const int64_t tasks = m * out_f;
    linear_scalar_kernel<<<(unsigned)((tasks + 7) / 8), 256, 0, st>>>(x, wh, y, (int)m, (int)in_f,
                                                                      (int)out_f);
    return cudaGetLastError();
  }
  if (path == LinearPath::kRows) {
    // 4 rows per warp when that still gives two CTAs per SM, else 1
    const bool wide = out_f >= (int64_t)2 * sm_count() * kRowsWarps * 4;
    const int rows_per_cta = kRowsWarps * (wide ? 4 : 1);
    const unsigned grid = (unsigned)((out_f + rows_per_cta - 1) / rows_per_cta);
    const int mi = (int)m, ki = (int)in_f, ni = (int)out_f;
    constexpr int T = kRowsWarps * 32;
    if (wide) {
      if (m == 1) linear_rows_kernel<1, 4><<<grid, T, 0, st>>>(x, wh, y, mi, ki, ni);
      else if (m == 2) linear_rows_kernel<2, 4><<<grid, T, 0, st>>>(x, wh, y, mi, ki, ni);
      else if (m <= 4) linear_rows_kernel<4, 4><<<grid, T, 0, st>>>(x, wh, y, mi, ki, ni);
      else linear_rows_kernel<8, 4><<<grid, T, 0, st>>>(x, wh, y, mi, ki, ni);
    } else {
      if (m == 1) linear_rows_kernel<1, 1><<<grid, T, 0, st>>>(x, wh, y, mi, ki, ni);
      else if (m == 2) linear_rows_kernel<2, 1><<<grid, T, 0, st>>>(x, wh, y, mi, ki, ni);
      else if (m <= 4) linear_rows_kernel<4, 1><<<grid, T, 0, st>>>(x, wh, y, mi, ki, ni);
      else linear_rows_kernel<8, 1><<<grid, T, 0, st>>>(x, wh, y, mi, ki, ni);
    }
    return cudaGetLastError();
  }
  using C = LinCfg;
  const size_t plane = ((size_t)m * in_f * sizeof(__half) + 255) / 256 * 256;
  __half* hi = static_cast<__half*>(ws);
  __half* lo = reinterpret_cast<__half*>(static_cast<char*>(ws) + plane);
  const int64_t n8 = m * in_f / 8;
  split_x_kernel<<<(unsigned)std::min<int64_t>((n8 + 255) / 256, (int64_t)sm_count() * 16), 256, 0, st>>>(
      x, hi, lo, n8);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  static unsigned configured = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(__atomic_load_n(&configured, __ATOMIC_ACQUIRE) & (1u << (dev & 31)))) {
    e = cudaFuncSetAttribute(linear_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM);
    if (e != cudaSuccess) return e;
    __atomic_fetch_or(&configured, 1u << (dev & 31), __ATOMIC_RELEASE);
  }
  CUtensorMap mxh, mxl, mw, my;
  if (!make_2d_map(&mxh, hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, in_f, m, C::BK, C::BM) ||
      !make_2d_map(&mxl, lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, in_f, m, C::BK, C::BM) ||
      !make_2d_map(&mw, w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, in_f, out_f, C::BK, C::BN) ||
      !make_2d_map(&my, y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, out_f, m, 32, C::BM))
    return cudaErrorInvalidValue;
  const dim3 grid((unsigned)((out_f + C::BN - 1) / C::BN), (unsigned)((m + C::BM - 1) / C::BM));
  linear_tc_kernel<<<grid, C::THREADS, C::SMEM, st>>>(mxh, mxl, mw, my, (int)in_f, (int)out_f,
                                                      err);
  return cudaGetLastError();
}

}  // namespace eb
