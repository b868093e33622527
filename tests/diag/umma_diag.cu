// umma_diag.cu -- test-only check of the tcgen05 operand layouts the attention
// kernels rely on, one at a time, on a single 128 x 128 x K f16 product:
//   D1 = A . B^T   A, B K-major, both written by TMA (128-byte swizzle)
//   D2 = A . B^T   A written by threads with the kernel's swizzle formula
//   D3 = A . Bt    Bt [K x N] row-major read as an MN-major B operand (TMA)
//   D4 = A . Bt    A read from tensor memory (written with tcgen05.st)
// All waits are bounded; the status word reports any that gave up.
#include <cudaTypedefs.h>

#include "eb_common.cuh"

using namespace eb;

namespace {

constexpr int M = 128, N = 128;

template <int K>
__global__ void __launch_bounds__(128, 1)
    umma_diag_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmBt, const __half* A, float* D1, float* D2,
                     float* D3, float* D4, unsigned* status) {
  constexpr int KB = K / 64;             // 64-element boxes along K
  constexpr int TILE = 128 * 128;        // [128 rows x 128 B]
  constexpr int A_BYTES = KB * TILE;
  constexpr int BT_BOX = K * 128;        // [K rows x 128 B]
  extern __shared__ uint8_t raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sA = smem_u32(smem);
  const uint32_t sAm = sA + A_BYTES;
  const uint32_t sB = sAm + A_BYTES;
  const uint32_t sBt = sB + A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 3 * A_BYTES + 2 * BT_BOX);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 5);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    mbar_init(smem_u32(&bars[0]), 1);
    mbar_init(smem_u32(&bars[1]), 1);
    mbar_init(smem_u32(&bars[2]), 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_async_smem();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tslot), 512);
    tmem_relinquish();
  }
  // A written by hand: row tid, chunk c -> sw128_offset
  for (int c = 0; c < K / 8; c++) {
    float f[8];
    for (int i = 0; i < 8; i++) f[i] = __half2float(A[tid * K + c * 8 + i]);
    uint32_t w[4];
    for (int i = 0; i < 4; i++) w[i] = pack_half2(f[2 * i], f[2 * i + 1]);
    const uint32_t addr = sAm + (c >> 3) * TILE + sw128_offset(tid, c & 7);
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(w[0]), "r"(w[1]),
                 "r"(w[2]), "r"(w[3]) : "memory");
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tlane = tmem + ((uint32_t)(warp * 32) << 16);

  if (tid == 0) {
    const uint32_t full = smem_u32(&bars[0]);
    mbar_arrive_expect_tx(full, 2 * A_BYTES + 2 * BT_BOX);
    for (int kb = 0; kb < KB; kb++) {
      tma_load_3d(sA + kb * TILE, &tmA, full, kb * 64, 0, 0);
      tma_load_3d(sB + kb * TILE, &tmB, full, kb * 64, 0, 0);
    }
    for (int nb = 0; nb < 2; nb++) tma_load_3d(sBt + nb * BT_BOX, &tmBt, full, nb * 64, 0, 0);
    if (mbar_wait(full, 0, abort_flag, status, 1u)) {
      tc_fence_after();
      constexpr uint32_t id_k = idesc_f16(M, N, false, false);
      constexpr uint32_t id_mn = idesc_f16(M, N, false, true);
      for (int kk = 0; kk < K / 16; kk++) {
        const uint32_t koff = (kk >> 2) * TILE + (kk & 3) * 32;
        const uint64_t bt = sdesc_sw128(sBt + kk * 16 * 128, BT_BOX, 1024);
        umma_ss(tmem + 0, sdesc_sw128(sA + koff, 16, 1024), sdesc_sw128(sB + koff, 16, 1024), id_k, kk > 0);
        umma_ss(tmem + 128, sdesc_sw128(sAm + koff, 16, 1024), sdesc_sw128(sB + koff, 16, 1024), id_k, kk > 0);
        umma_ss(tmem + 256, sdesc_sw128(sA + koff, 16, 1024), bt, id_mn, kk > 0);
      }
      umma_commit(smem_u32(&bars[1]));
    }
  }
  __syncwarp();
  // phase 1 read-out
  const bool ok1 = mbar_wait(smem_u32(&bars[1]), 0, abort_flag, status, 2u);
  __syncwarp();
  tc_fence_after();
  if (ok1) {
    float* outs[3] = {D1, D2, D3};
    for (int d = 0; d < 3; d++)
      for (int c = 0; c < N / 32; c++) {
        uint32_t r[32];
        tmem_ld32(tlane + d * 128 + c * 32, r);
        tmem_ld_wait();
        for (int i = 0; i < 32; i++) outs[d][tid * N + c * 32 + i] = __uint_as_float(r[i]);
      }
  }
  // phase 2: A row tid into TMEM columns [384, 384 + K/2) as packed f16 pairs
  for (int c = 0; c < K / 64; c++) {
    uint32_t r[32];
    for (int i = 0; i < 32; i++)
      r[i] = pack_half2(__half2float(A[tid * K + c * 64 + 2 * i]),
                        __half2float(A[tid * K + c * 64 + 2 * i + 1]));
    tmem_st32(tlane + 384 + c * 32, r);
  }
  tmem_st_wait();
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && ok1) {
    tc_fence_after();
    constexpr uint32_t id_mn = idesc_f16(M, N, false, true);
    for (int kk = 0; kk < K / 16; kk++)
      umma_ts(tmem + 0, tmem + 384 + kk * 8, sdesc_sw128(sBt + kk * 16 * 128, BT_BOX, 1024), id_mn,
              kk > 0);
    umma_commit(smem_u32(&bars[2]));
  }
  __syncwarp();
  const bool ok2 = ok1 && mbar_wait(smem_u32(&bars[2]), 0, abort_flag, status, 4u);
  __syncwarp();
  tc_fence_after();
  if (ok2) {
    for (int c = 0; c < N / 32; c++) {
      uint32_t r[32];
      tmem_ld32(tlane + c * 32, r);
      tmem_ld_wait();
      for (int i = 0; i < 32; i++) D4[tid * N + c * 32 + i] = __uint_as_float(r[i]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

bool map2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint32_t box_rows) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess)
      return false;
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  // as a 3-D map {inner, 1, rows} so the kernel uses the same 3-D TMA load as the attention kernel
  cuuint64_t dims[3] = {inner, 1, rows};
  cuuint64_t strides[2] = {inner * 2, inner * 2};
  cuuint32_t box[3] = {64, 1, box_rows};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int K>
int run(const void* A, const void* B, const void* Bt, float* D1, float* D2, float* D3, float* D4,
        unsigned* status) {
  CUtensorMap ma, mb, mbt;
  if (!map2d(&ma, A, K, M, 128) || !map2d(&mb, B, K, N, 128) || !map2d(&mbt, Bt, N, K, K)) return -1;
  const int smem = 3 * (K / 64) * 128 * 128 + 2 * K * 128 + 1024 + 1024;
  auto kern = umma_diag_kernel<K>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return -2;
  kern<<<1, 128, smem>>>(ma, mb, mbt, reinterpret_cast<const __half*>(A), D1, D2, D3, D4, status);
  if (cudaGetLastError() != cudaSuccess) return -3;
  if (cudaDeviceSynchronize() != cudaSuccess) return -4;
  return 0;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int diag_umma(
    const void* A, const void* B, const void* Bt, float* D1, float* D2, float* D3, float* D4, int K,
    unsigned* status) {
  if (K == 64) return run<64>(A, B, Bt, D1, D2, D3, D4, status);
  if (K == 128) return run<128>(A, B, Bt, D1, D2, D3, D4, status);
  return -5;
}
