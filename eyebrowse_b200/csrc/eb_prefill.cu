// eb_prefill.cu -- causal GQA flash-attention prefill on tcgen05 tensor cores.
//
// Replaces attn_prefill (crates/eyebrowse-kernels/src/attention.rs:10-50,
// :94-120): o[i,h] = softmax_j<=i(scale * q[i,h] . k[j,kvh]) v[j,kvh], with
// kvh = h / (H/Hkv), seq-major layouts.
//
// One CTA = NQ query tiles of 128 rows (the two heads of a GQA pair when the
// group size is even, so each K/V tile feeds twice the MMA work):
//   warp 0      TMA producer: the query tiles (the raw 16-bit rows the
//               softmax warps transform in place, with the CTA's rows of the
//               RoPE tables; or rows the row-prep pass already transformed),
//               then K tiles [BN rows x 64 dims] (128-byte swizzle) into an
//               NSTK-deep ring.
//   warp 1      TMEM owner + MMA issuer (one thread): S_t = Q_t K^T into TMEM,
//               then O_t += P_t V with P read from TMEM (it overwrites S_t).
//   warp 2      TMA producer of the V ring (its own thread, so K loads never
//               queue behind a V slot).
//   warp 3      idle (softmax warps must start at a multiple of 4: a warp may
//               only address TMEM lanes 32*(warp%4)..+31).
//   warps 4..   one thread per query row of each tile: per KV tile read the S
//               row from TMEM, online softmax in f32 (exp2 on MUFU, some
//               column pairs on the FMA pipe), rescale the O row in TMEM when
//               the max moves past a threshold, write P (16-bit) back over S;
//               finally O / l to global memory. Before the first tile they
//               normalise and rotate their query rows (fused q prep).
// K/V come from the cache the K/V preparation pass has just written (the
// reference attends the same post-RoPE k / post-norm v it writes,
// crates/eyebrowse-nn/src/attention.rs:78-115).
//
// f32 caches (SPLIT): every q/k/v operand x is carried as two f16 values
// hi = f16(x), lo = f16(x - hi), and S = Qh.Kh + Qh.Kl + Ql.Kh (the standard
// error-compensated split, ~21 mantissa bits on f16 tensor cores: the
// logits need them, an f16 rounding of q or k moves a logit of a
// unit-RMS head_dim-256 row by ~1e-2). P (at most 2^8 under the lazy
// rescale) is kept at f16 only, O += P.Vh + P.Vl, and l sums those same f16
// values: o is then an exact convex combination of v rows whose weights are
// each off by at most 2^-11 relative and still sum to one, so the error is
// at most 2^-11 times the weighted spread of v about o (none when one key
// carries all the weight). At head_dim 256 Q's hi plane sits in tensor
// memory and the softmax threads build both planes from the raw q rows (see
// PfCfg::QT and q_split_transform).
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>
#include <cstring>
#include <mutex>

#include "eb_common.cuh"
#include "eb_kernels.cuh"
#include "eb_rowops.cuh"
#include "eb_tc.cuh"

namespace eb {

#ifndef EB_PREFILL_EMU_PAIRS
#define EB_PREFILL_EMU_PAIRS 2
#endif
constexpr int kEmuPairsOf8 = EB_PREFILL_EMU_PAIRS;

// Tile geometry. NQ query tiles (heads of one GQA group, same rows) share
// each K/V tile. NSB S buffers per query tile: with one query tile, two S
// buffers let QK of tile j+1 run while the softmax of tile j works; with two
// query tiles the other tile's MMAs fill that gap instead.
template <int HD, int BN, int NQ, bool SPLIT, int NSTK, int NSTV>
struct PfCfg {
  static constexpr int NQP = SPLIT ? 2 : 1;  // operand planes (hi, lo)
  // Split operands at head_dim 256: Q's hi plane lives in tensor memory (the
  // A operand of the Qh.Kh and Qh.Kl MMAs) and only its lo plane in shared
  // memory. The 64 KB this frees makes room for 64-key K/V tiles, so each
  // QK MMA covers twice the keys (the MMA thread's issue rate bounds this
  // kernel).
  static constexpr bool QT = SPLIT && HD == 256;
  static constexpr int NQP_SMEM = QT ? 1 : NQP;  // Q planes in shared memory
  static constexpr int HB = HD / 64;         // 64-element boxes along head_dim
  static constexpr int TILE128 = 128 * 128;  // one [128 rows x 128 B] box
  static constexpr int QT_BYTES = NQP_SMEM * HB * TILE128;
  static constexpr int Q_BYTES = NQ * QT_BYTES;
  static constexpr int KV_BOX = BN * 128;  // one [BN rows x 128 B] box
  static constexpr int K_BYTES = NQP * HB * KV_BOX;  // one K (or V) tile, all planes
  static constexpr int V_OFF = Q_BYTES + NSTK * K_BYTES;  // V ring follows the K ring
  static constexpr int BAR_OFF = V_OFF + NSTV * K_BYTES;
  static constexpr int SMEM = BAR_OFF + 512 + 1024;  // barriers/flags + alignment slack
  // Fused q prep with RoPE: the CTA's 128 rows of the cos / sin tables
  // (HD/2 f32 each) come by TMA with the query tiles, as [128 rows x 128 B]
  // 128-byte-swizzled boxes, into the last K slot (cos) and the last V slot
  // (sin). Those slots take their first K/V tiles once every query tile's
  // rows are transformed. (Per-thread loads of a table row each touch 32
  // cache lines per warp instruction and took ~2 us per batch at CTA start.)
  static constexpr int TAB_BYTES = 128 * (HD / 2) * 4;
  static constexpr bool TAB = !SPLIT && NSTK >= 2 && NSTV >= 2 && TAB_BYTES <= K_BYTES;
  static constexpr int TAB_COS = Q_BYTES + (NSTK - 1) * K_BYTES;  // offsets from the tile base
  static constexpr int TAB_SIN = V_OFF + (NSTV - 1) * K_BYTES;
  static constexpr int NSB = (NQ == 1 || NQ * HD + NQ * 2 * BN <= 512) ? 2 : 1;
  // TMEM columns: the O accumulators first ([t*HD, (t+1)*HD)), then Q's hi
  // plane when QT (HD/2 columns of packed f16 pairs), then the S/P buffers;
  // every MMA destination starts at a column aligned to its width.
  static constexpr int Q_TM = NQ * HD;
  static constexpr int S_COL0 = NQ * HD + (QT ? HD / 2 : 0);
  static constexpr int TMEM_COLS = constexpr_pow2ceil(S_COL0 + NQ * NSB * BN);
  static constexpr int THREADS = 128 + 128 * NQ;
  // Of every 8 column pairs of P, this many take their exp2 on the FMA pipe
  // (ex2_fma_pair) and the rest on MUFU. The hi/lo split path keeps MUFU for
  // all: its tiles are bound by the MMA issue of three QK passes, not by
  // the exponentials.
  static constexpr int EMU_PAIRS = SPLIT ? 0 : kEmuPairsOf8;
  static_assert(HD % 64 == 0 && HD <= 256, "head_dim");
  static_assert(BN % 32 == 0 && BN <= 128, "kv tile");
  static_assert(TMEM_COLS <= 512, "tensor memory budget");
  static_assert(!QT || NQ == 1, "Q in tensor memory: one query tile");
  static_assert(SMEM <= 232448, "shared memory budget");
  // Head-gather epilogue: tile t's O stages at [t*STG, (t+1)*STG) from the
  // start of shared memory (q and the K/V rings are idle by then), as
  // 128-byte-swizzled boxes of [128 rows x 128 B].
  static constexpr int STG = 128 * HD * 4;  // room for f32 output
  static_assert(NQ * STG <= BAR_OFF, "gather staging area");
};

// Barrier slots.
enum { kBarQ = 0, kBarFinal = 1, kBarS0 = 2 };

// Tensor maps of the head-gather destinations (see GatherSpec).
struct GatherMaps {
  CUtensorMap m[kMaxGather];
};




// Fused q prep: thread r of a query tile's softmax warpgroup turns its row
// of the TMA-loaded raw query tile (HD 16-bit values in 128-byte-swizzled
// boxes of 64) into the MMA operand: RMSNorm (q_norm_w), then half-split
// RoPE at position q_row, then rounding to the operand type -- the row-prep
// pass's per-element f32 arithmetic (crates/eyebrowse-kernels/src/
// rmsnorm.rs:34-36, rope.rs:25-30) on the same values, with the sum of
// squares in one thread's order. The table row is fetched (up to 32 pairs at
// a time) before the tile lands. Rows past S (zero-filled by TMA) are left
// as they are. Then the
// generic-proxy writes are made visible to the tensor core and the tile's
// ready barrier (128 arrivals) is arrived on.
// Q in tensor memory (f32 caches at head_dim 256), with the q row prep
// fused: thread r of the softmax warpgroup reads its raw query row (q_raw,
// in dtype q_dtype, rows q_stride elements apart) from global memory and
// applies the row-prep pass's per-element f32 arithmetic: RMSNorm with the
// sum of squares in one thread's order (the reference's loop order,
// crates/eyebrowse-kernels/src/rmsnorm.rs:34-36), then half-split RoPE at
// position q_row (rope.rs:25-30), then the f16 hi/lo split. The hi plane
// goes to its TMEM lane, element k at column k/2 of the given base, low
// half first -- the layout of an A operand read from tensor memory (the
// same as P's); the lo plane goes to the shared-memory tile (128-byte
// swizzled boxes of [128 rows x 64 dims]) the QlKh MMAs read. Rows past S
// store zeros. The TMEM stores are warp-collective, so every thread makes
// them. Then the tile's ready barrier (128 arrivals) tells the MMA thread.
template <int HD>
__device__ __forceinline__ void q_split_transform(const PrefillArgs& a, uint32_t taddr,
                                                  uint32_t lo_tile, int r, int q_row, int h,
                                                  bool valid, uint32_t ready_bar) {
  constexpr int HALF = HD / 2, NCH = HD / 8;  // 8-element chunks per row
  const bool rope = valid && a.cos_t != nullptr;
  const bool norm = valid && a.q_norm_w != nullptr;
  const int64_t base = (int64_t)(valid ? q_row : 0) * a.q_stride + (int64_t)h * HD;
  // N chunks starting at c0 (stride cs chunks), as f32: every load of the
  // batch is issued before any is used (the row is strided across the warp,
  // so each batch is one round trip to memory).
  auto load_chunks = [&](auto& f, int c0, int cs) {
    constexpr int N = sizeof(f) / sizeof(f[0]);
    if (!valid) {
#pragma unroll
      for (int n = 0; n < N; n++)
#pragma unroll
        for (int e = 0; e < 8; e++) f[n][e] = 0.f;
    } else if (a.q_dtype == kF32) {
      const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(a.q_raw) + base);
      float4 x[2 * N];
#pragma unroll
      for (int n = 0; n < N; n++) {
        x[2 * n] = __ldg(p + 2 * (c0 + n * cs));
        x[2 * n + 1] = __ldg(p + 2 * (c0 + n * cs) + 1);
      }
#pragma unroll
      for (int n = 0; n < N; n++) {
        f[n][0] = x[2 * n].x; f[n][1] = x[2 * n].y; f[n][2] = x[2 * n].z; f[n][3] = x[2 * n].w;
        f[n][4] = x[2 * n + 1].x; f[n][5] = x[2 * n + 1].y;
        f[n][6] = x[2 * n + 1].z; f[n][7] = x[2 * n + 1].w;
      }
    } else {
      const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.q_raw) + base);
      uint4 w[N];
#pragma unroll
      for (int n = 0; n < N; n++) w[n] = __ldg(p + c0 + n * cs);
#pragma unroll
      for (int n = 0; n < N; n++) {
        const uint32_t u[4] = {w[n].x, w[n].y, w[n].z, w[n].w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const float2 v = a.q_dtype == kBF16
                               ? __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[k]))
                               : __half22float2(*reinterpret_cast<const __half2*>(&u[k]));
          f[n][2 * k] = v.x;
          f[n][2 * k + 1] = v.y;
        }
      }
    }
  };
  // hi of chunk c -> TMEM columns [4c, 4c+4), lo -> its swizzled shared-memory slot
  auto put = [&](int c, const float (&x)[8]) {
    uint32_t hw[4];
    float lo[8];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const __half2 hh = __floats2half2_rn(x[2 * k], x[2 * k + 1]);
      const float2 hf = __half22float2(hh);
      hw[k] = *reinterpret_cast<const uint32_t*>(&hh);
      lo[2 * k] = x[2 * k] - hf.x;
      lo[2 * k + 1] = x[2 * k + 1] - hf.y;
    }
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr + 4 * c),
                 "r"(hw[0]), "r"(hw[1]), "r"(hw[2]), "r"(hw[3])
                 : "memory");
    st_chunk<false>(lo_tile + (uint32_t)(c >> 3) * (128u * 128u) +
                        sw128_offset((uint32_t)r, (uint32_t)(c & 7)),
                    lo);
  };
  float inv = 1.f;
  if (norm) {
    float ss = 0.f;
#pragma unroll 1
    for (int c0 = 0; c0 < NCH; c0 += 16) {  // elements in order: one thread's sum
      float f[16][8];
      load_chunks(f, c0, 1);
#pragma unroll
      for (int n = 0; n < 16; n++)
#pragma unroll
        for (int e = 0; e < 8; e++) ss = __fadd_rn(ss, __fmul_rn(f[n][e], f[n][e]));
    }
    inv = 1.0f / sqrtf(ss / (float)HD + a.eps);
  }
  const float* crow = rope ? a.cos_t + (int64_t)q_row * HALF : nullptr;
  const float* srow = rope ? a.sin_t + (int64_t)q_row * HALF : nullptr;
  constexpr int PB = 4;  // chunk pairs per batch
#pragma unroll 1
  for (int c0 = 0; c0 < NCH / 2; c0 += PB) {  // chunks c (first half) with partners c + NCH/2
    float x[2 * PB][8];
    load_chunks(*reinterpret_cast<float(*)[PB][8]>(&x[0]), c0, 1);
    load_chunks(*reinterpret_cast<float(*)[PB][8]>(&x[PB]), c0 + NCH / 2, 1);
    float4 tc[2 * PB], ts[2 * PB];
    if (rope) {
#pragma unroll
      for (int i = 0; i < 2 * PB; i++) {
        tc[i] = __ldg(reinterpret_cast<const float4*>(crow + 8 * c0) + i);
        ts[i] = __ldg(reinterpret_cast<const float4*>(srow + 8 * c0) + i);
      }
    }
#pragma unroll
    for (int n = 0; n < PB; n++) {
      const int c = c0 + n;
      float* x1 = x[n];
      float* x2 = x[PB + n];
      if (norm) {
#pragma unroll
        for (int e = 0; e < 8; e++) {
          x1[e] = __fmul_rn(__fmul_rn(x1[e], inv), a.q_norm_w[8 * c + e]);
          x2[e] = __fmul_rn(__fmul_rn(x2[e], inv), a.q_norm_w[HALF + 8 * c + e]);
        }
      }
      if (rope) {
        const float cs[8] = {tc[2 * n].x, tc[2 * n].y, tc[2 * n].z, tc[2 * n].w,
                             tc[2 * n + 1].x, tc[2 * n + 1].y, tc[2 * n + 1].z, tc[2 * n + 1].w};
        const float sn[8] = {ts[2 * n].x, ts[2 * n].y, ts[2 * n].z, ts[2 * n].w,
                             ts[2 * n + 1].x, ts[2 * n + 1].y, ts[2 * n + 1].z, ts[2 * n + 1].w};
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const float u = x1[e], v = x2[e];
          x1[e] = __fsub_rn(__fmul_rn(u, cs[e]), __fmul_rn(v, sn[e]));
          x2[e] = __fadd_rn(__fmul_rn(v, cs[e]), __fmul_rn(u, sn[e]));
        }
      }
      put(c, x[n]);
      put(c + NCH / 2, x[PB + n]);
    }
  }
  tmem_st_wait();
  fence_async_smem();
  tc_fence_before();
  mbar_arrive(ready_bar);
}

template <int HD, bool BF16>
__device__ __forceinline__ void q_tile_transform(uint32_t tile, int r, int q_row,
                                                 const PrefillArgs& a, uint32_t q_bar,
                                                 uint32_t ready_bar, volatile int* abort_flag,
                                                 uint32_t tab_cos, uint32_t tab_sin) {
  constexpr int HALF = HD / 2, NCH = HD / 8;  // 8-element chunks per row
  const bool valid = q_row < a.S;
  const bool rope = valid && a.cos_t != nullptr;
  const bool norm = valid && a.q_norm_w != nullptr;
  const float* crow = rope ? a.cos_t + (int64_t)q_row * HALF : nullptr;
  const float* srow = rope ? a.sin_t + (int64_t)q_row * HALF : nullptr;
  auto chunk_addr = [&](int c) {  // chunk c (elements 8c..8c+7) of row r
    return tile + (uint32_t)(c >> 3) * (128u * 128u) + sw128_offset((uint32_t)r, (uint32_t)(c & 7));
  };
  auto load8 = [&](int c, float (&f)[8]) {
    uint32_t w[4];
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                 : "r"(chunk_addr(c)));
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float2 v = BF16 ? __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]))
                            : __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
      f[2 * k] = v.x;
      f[2 * k + 1] = v.y;
    }
  };
  // The row's table entries come in passes of up to 32 pairs, all loads of a
  // pass in flight at once; the first pass's while the tile lands.
  constexpr int PP = HALF < 32 ? HALF : 32;  // pairs per pass
  constexpr int NPASS = HALF / PP;
  float cs[PP], sn[PP];
  // tab_cos != 0: the table rows are staged in shared memory (128-byte
  // swizzled boxes of 32 pairs x 128 rows, landed with the query tile)
  auto lds4 = [&](uint32_t base, int i) {  // pairs i..i+3 of row r
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(base + (uint32_t)(i >> 5) * (128u * 128u) +
                       sw128_offset((uint32_t)r, (uint32_t)((i & 31) >> 2))));
    return v;
  };
  auto fetch = [&](int pass) {
#pragma unroll
    for (int i = 0; i < PP; i += 4) {
      const float4 c4 = !rope ? make_float4(1.f, 1.f, 1.f, 1.f)
                        : tab_cos ? lds4(tab_cos, pass * PP + i)
                                  : *reinterpret_cast<const float4*>(crow + pass * PP + i);
      const float4 s4 = !rope ? make_float4(0.f, 0.f, 0.f, 0.f)
                        : tab_cos ? lds4(tab_sin, pass * PP + i)
                                  : *reinterpret_cast<const float4*>(srow + pass * PP + i);
      cs[i] = c4.x; cs[i + 1] = c4.y; cs[i + 2] = c4.z; cs[i + 3] = c4.w;
      sn[i] = s4.x; sn[i + 1] = s4.y; sn[i + 2] = s4.z; sn[i + 3] = s4.w;
    }
  };
  if (rope && !tab_cos) fetch(0);  // global rows: in flight while the tile lands
  const bool got_q = mbar_wait(q_bar, 0, abort_flag, a.err, kErrTimeoutSoftmax);
  if (rope && tab_cos && got_q) fetch(0);
  if (got_q && (rope || norm)) {
    float inv = 1.f;
    if (norm) {
      float ss = 0.f;
#pragma unroll 4
      for (int c = 0; c < NCH; c++) {
        float f[8];
        load8(c, f);
#pragma unroll
        for (int e = 0; e < 8; e++) ss = __fadd_rn(ss, __fmul_rn(f[e], f[e]));
      }
      inv = 1.0f / sqrtf(ss / (float)HD + a.eps);
    }
#pragma unroll 1
    for (int pass = 0; pass < NPASS; pass++) {
      if (rope && pass > 0) fetch(pass);
#pragma unroll
      for (int cc = 0; cc < PP / 8; cc++) {  // chunk c (first half) with its partner c + NCH/2
        const int c = pass * (PP / 8) + cc;
        float x1[8], x2[8];
        load8(c, x1);
        load8(c + NCH / 2, x2);
        if (norm) {
#pragma unroll
          for (int e = 0; e < 8; e++) {
            x1[e] = __fmul_rn(__fmul_rn(x1[e], inv), a.q_norm_w[8 * c + e]);
            x2[e] = __fmul_rn(__fmul_rn(x2[e], inv), a.q_norm_w[HALF + 8 * c + e]);
          }
        }
        if (rope) {
#pragma unroll
          for (int e = 0; e < 8; e++) {
            const float u = x1[e], v = x2[e], co = cs[8 * cc + e], si = sn[8 * cc + e];
            x1[e] = __fsub_rn(__fmul_rn(u, co), __fmul_rn(v, si));
            x2[e] = __fadd_rn(__fmul_rn(v, co), __fmul_rn(u, si));
          }
        }
        st_chunk<BF16>(chunk_addr(c), x1);
        st_chunk<BF16>(chunk_addr(c + NCH / 2), x2);
      }
    }
    fence_async_smem();
  }
  mbar_arrive(ready_bar);
}

// WIN: a sliding window narrower than the sequence (a.window). Its own
// instantiation, so the plain causal kernel carries none of the window's
// index arithmetic.
template <int HD, int BN, int NQ, bool SPLIT, bool BF16, int NSTK, int NSTV, bool WIN>
__global__ void __launch_bounds__(PfCfg<HD, BN, NQ, SPLIT, NSTK, NSTV>::THREADS, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmQlo,
                      const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV,
                      const __grid_constant__ CUtensorMap tmKlo,
                      const __grid_constant__ CUtensorMap tmVlo,
                      const __grid_constant__ CUtensorMap tmCos,
                      const __grid_constant__ CUtensorMap tmSin,
                      const __grid_constant__ GatherMaps gmaps, PrefillArgs a) {
  using C = PfCfg<HD, BN, NQ, SPLIT, NSTK, NSTV>;
  constexpr int NSB = C::NSB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK = sQ + C::Q_BYTES, sV = sQ + C::V_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::BAR_OFF + 384);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::BAR_OFF + 392);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  // barrier index map
  constexpr int kSFull0 = kBarS0;                 // [NQ][NSB]
  constexpr int kPFull0 = kSFull0 + NQ * NSB;     // [NQ][NSB]
  constexpr int kP0Full0 = kPFull0 + NQ * NSB;    // [NQ][NSB]: first half of P (BN = 128)
  constexpr int kODone0 = kP0Full0 + NQ * NSB;    // [NQ]
  constexpr int kKFull0 = kODone0 + NQ;           // [NSTK]
  constexpr int kKEmpty0 = kKFull0 + NSTK;        // [NSTK]
  constexpr int kVFull0 = kKEmpty0 + NSTK;        // [NSTV]
  constexpr int kVEmpty0 = kVFull0 + NSTV;        // [NSTV]
  constexpr int kQReady0 = kVEmpty0 + NSTV;       // [NQ]: tile t's rows transformed in smem
  constexpr int kNumBars = kQReady0 + NQ;
  static_assert(kNumBars * 8 <= 384, "barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (a.S + 127) / 128;
  const int n_grp = a.H / NQ;
  const int qt = n_qt - 1 - (int)(blockIdx.x / n_grp);  // longest causal rows first
  const int grp = (int)(blockIdx.x % n_grp);
  const int kvh = (grp * NQ) / (a.H / a.Hkv);
  const int q0 = qt * 128;
  const int kv_rows = min(q0 + 128, a.S);
  // With a sliding window the tile loop starts at the first key tile that
  // any row of this query tile sees; tile j of the loop is key tile j0 + j.
  const int j0 = WIN ? max(0, q0 - a.window + 1) / BN : 0;
  const int n_tiles = (kv_rows + BN - 1) / BN - j0;

  if (threadIdx.x == 0) {
    mbar_init(bar(kBarQ), 1);
    mbar_init(bar(kBarFinal), 1);
    for (int i = kSFull0; i < kPFull0; i++) mbar_init(bar(i), 1);
    for (int i = kPFull0; i < kODone0; i++) mbar_init(bar(i), 128);  // P and P-half-0
    for (int i = kODone0; i < kQReady0; i++) mbar_init(bar(i), 1);
    for (int i = kQReady0; i < kNumBars; i++) mbar_init(bar(i), 128);  // the tile's rows
    *abort_flag = 0;
    fence_mbar_init();
    fence_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tmQ);
    tma_prefetch_map(&tmK);
    tma_prefetch_map(&tmV);
    if (SPLIT) {
      tma_prefetch_map(&tmQlo);
      tma_prefetch_map(&tmKlo);
      tma_prefetch_map(&tmVlo);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool tab = C::TAB && a.tab_smem != 0;

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------ TMA producers
    // Warp 0 loads the query tiles and the K ring, warp 2 the V ring, each
    // from its own thread: K tile j uses K slot j % NSTK and is released when
    // its QK MMAs complete; V tile j uses V slot j % NSTV, released after its
    // PV MMAs. Separate threads let K_{j+NSTK} load as soon as QK_j is done,
    // without waiting behind V_{j+1}'s slot (with one-deep rings that wait
    // would put a load latency on every tile).
    if (lane == 0) {
      const bool is_k = warp == 0;
      if (is_k && !C::QT) {  // QT: the softmax threads build the query tile
        // The query tiles (rows past S read as zeros): NQ heads x HB boxes of
        // [128 rows x 64 dims], hi and lo planes when split. With staged RoPE
        // tables, their rows come on the same barrier.
        mbar_arrive_expect_tx(bar(kBarQ), C::Q_BYTES + (tab ? 2 * C::TAB_BYTES : 0));
        if (tab) {
#pragma unroll
          for (int bx = 0; bx < HD / 64; bx++) {  // boxes of 32 pairs
            tma_load_2d(sQ + C::TAB_COS + bx * C::TILE128, &tmCos, bar(kBarQ), bx * 32, q0);
            tma_load_2d(sQ + C::TAB_SIN + bx * C::TILE128, &tmSin, bar(kBarQ), bx * 32, q0);
          }
        }
#pragma unroll
        for (int t = 0; t < NQ; t++)
#pragma unroll
          for (int hb = 0; hb < C::HB; hb++) {
            const uint32_t dst = sQ + t * C::QT_BYTES + hb * C::TILE128;
            tma_load_3d(dst, &tmQ, bar(kBarQ), hb * 64, grp * NQ + t, q0);
            if (SPLIT)
              tma_load_3d(dst + C::HB * C::TILE128, &tmQlo, bar(kBarQ), hb * 64, grp * NQ + t, q0);
          }
      }
      const int NST = is_k ? NSTK : NSTV;
      const uint32_t ring = is_k ? sK : sV;
      const int full0 = is_k ? kKFull0 : kVFull0, empty0 = is_k ? kKEmpty0 : kVEmpty0;
      const CUtensorMap* hi = is_k ? &tmK : &tmV;
      const CUtensorMap* lo = is_k ? &tmKlo : &tmVlo;
      const uint32_t err_bit = kErrTimeoutTma;
      int iss[NSTK > NSTV ? NSTK : NSTV];
      for (int s = 0; s < NST; s++) iss[s] = 0;
      for (int j = 0; j < n_tiles; j++) {
        const int sl = j % NST;
        const uint32_t dst = ring + sl * C::K_BYTES;
        if (j >= NST && !mbar_wait(bar(empty0 + sl), (j / NST - 1) & 1, abort_flag, a.err, err_bit))
          break;
        if (tab && j == NST - 1) {  // the slot holds a staged table until the q rows are done
          bool got = true;
#pragma unroll
          for (int t = 0; t < NQ; t++)
            got = got && mbar_wait(bar(kQReady0 + t), 0, abort_flag, a.err, err_bit);
          if (!got) break;
        }
        const uint32_t fb = bar(full0 + sl);
        mbar_arrive_expect_tx(fb, C::K_BYTES);
#pragma unroll
        for (int hb = 0; hb < C::HB; hb++) {
          tma_load_3d(dst + hb * C::KV_BOX, hi, fb, hb * 64, kvh, (j0 + j) * BN);
          if (SPLIT) tma_load_3d(dst + (C::HB + hb) * C::KV_BOX, lo, fb, hb * 64, kvh, (j0 + j) * BN);
        }
        iss[sl]++;
      }
      // Every issued copy has landed before the CTA can exit.
      if (is_k && !C::QT) mbar_drain(bar(kBarQ), 0, a.err, err_bit);
      for (int s = 0; s < NST; s++)
        if (iss[s]) mbar_drain(bar(full0 + s), (iss[s] - 1) & 1, a.err, err_bit);
    }
    __syncwarp();  // reconverge before the CTA barrier below
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16(128, BN, BF16, false);
      constexpr uint32_t idesc_pv = idesc_f16(128, HD, BF16, true);
      // Base descriptors of the query tiles, the K ring and the V ring; each
      // MMA's operand is a constant offset from one of them (sdesc_add).
      const uint64_t dQ0 = sdesc_sw128(sQ, 16, 1024);
      const uint64_t dK0 = sdesc_sw128(sK, 16, 1024);
      const uint64_t dV0 = sdesc_sw128(sV, C::KV_BOX, 1024);
      // S_t(buffer b) = Q_t K^T
      auto issue_qk = [&](int t, int b, int sk) {
        const uint64_t dK = sdesc_add(dK0, sk * C::K_BYTES);
        const uint32_t tS = tmem + C::S_COL0 + (t * NSB + b) * BN;
        constexpr int NPASS = SPLIT ? 3 : 1;
#pragma unroll
        for (int pass = 0; pass < NPASS; pass++) {
          const int qa = (pass == 2) ? 1 : 0;  // Qh Kh, Qh Kl, Ql Kh
          const int kb = (pass == 1) ? 1 : 0;
#pragma unroll
          for (int kk = 0; kk < HD / 16; kk++) {
            const int hb = kk >> 2, w = kk & 3;
            const uint64_t bd = sdesc_add(dK, (kb * C::HB + hb) * C::KV_BOX + w * 32);
            const uint32_t acc = (pass > 0 || kk > 0) ? 1u : 0u;
            if (C::QT && qa == 0) {
              // Qh from tensor memory: k-step kk is columns [8kk, 8kk+8)
              umma_ts(tS, tmem + C::Q_TM + kk * 8, bd, idesc_qk, acc);
            } else {
              const int plane = C::QT ? 0 : qa;  // QT keeps only Ql in shared memory
              const uint64_t ad =
                  sdesc_add(dQ0, t * C::QT_BYTES + (plane * C::HB + hb) * C::TILE128 + w * 32);
              umma_ss(tS, ad, bd, idesc_qk, acc);
            }
          }
        }
      };
      // O_t += P_t V, P_t read from tensor memory (the S buffer it replaced)
      // keys [16*kk0, 16*kk1) of the tile
      auto issue_pv = [&](int t, int b, int sv, bool first, int kk0, int kk1) {
        const uint64_t dV = sdesc_add(dV0, sv * C::K_BYTES);
        const uint32_t tP = tmem + C::S_COL0 + (t * NSB + b) * BN;
        const uint32_t tO = tmem + t * HD;
        constexpr int NPASS = SPLIT ? 2 : 1;
#pragma unroll
        for (int vb = 0; vb < NPASS; vb++) {  // P Vh, then P Vl
#pragma unroll
          for (int kk = kk0; kk < kk1; kk++) {
            const uint64_t bd = sdesc_add(dV, vb * C::HB * C::KV_BOX + kk * 16 * 128);
            // column of P elements [16kk, 16kk+16) in the softmax's layout
            constexpr int HALF = BN >= 64 ? 64 : BN;
            const int blk = (kk * 16) / HALF, within = (kk * 16) % HALF;
            const uint32_t col = blk * (HALF / 2) + within / 2;
            umma_ts(tO, tP + col, bd, idesc_pv, (!first || vb > 0 || kk > 0) ? 1u : 0u);
          }
        }
      };
      // The query tiles: landed (TMA), or landed and then transformed in
      // shared memory by their softmax warpgroups (fused q prep).
      bool ok = (a.q_fused || C::QT) ? true
                                     : mbar_wait(bar(kBarQ), 0, abort_flag, a.err, kErrTimeoutMma);
      if (ok && mbar_wait(bar(kKFull0), 0, abort_flag, a.err, kErrTimeoutMma)) {
#pragma unroll
        for (int t = 0; t < NQ; t++) {
          if ((a.q_fused || C::QT) &&
              !mbar_wait(bar(kQReady0 + t), 0, abort_flag, a.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_qk(t, 0, 0);
          umma_commit(bar(kSFull0 + t * NSB));
        }
        if (ok) umma_commit(bar(kKEmpty0));
      } else {
        ok = false;
      }
      for (int j = 0; ok && j < n_tiles; j++) {
        const int sv = j % NSTV;
        const int nj = j + 1, nsk = nj % NSTK;
        if (NSB == 2 && nj < n_tiles) {
          // S_t(j+1) goes to the other buffer ahead of PV_t(j), so it is ready
          // when the softmax of j finishes. That buffer's P_t(j-1) was read by
          // PV_t(j-1), issued before and executed in order.
          if (!mbar_wait(bar(kKFull0 + nsk), (nj / NSTK) & 1, abort_flag, a.err, kErrTimeoutMma))
            break;
          tc_fence_after();
#pragma unroll
          for (int t = 0; t < NQ; t++) {
            issue_qk(t, nj & 1, nsk);
            umma_commit(bar(kSFull0 + t * NSB + (nj & 1)));
          }
          umma_commit(bar(kKEmpty0 + nsk));
        }
#pragma unroll
        for (int t = 0; t < NQ; t++) {
          // One P barrier per S buffer: with two buffers the softmax may finish
          // P(j+1) before this wait sees P(j), and a per-tile barrier would
          // then be two phases ahead of its parity wait. With BN = 128 this
          // first waits for P's first half only.
          if (!mbar_wait(bar((BN == 128 ? kP0Full0 : kPFull0) + t * NSB + j % NSB), (j / NSB) & 1,
                         abort_flag, a.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          if (t == 0 &&
              !mbar_wait(bar(kVFull0 + sv), (j / NSTV) & 1, abort_flag, a.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if constexpr (BN == 128) {
            // P arrives in two halves: PV over keys [0, 64) runs while the
            // softmax still computes the rest
            issue_pv(t, j % NSB, sv, j == 0, 0, BN / 32);
            if (!mbar_wait(bar(kPFull0 + t * NSB + j % NSB), (j / NSB) & 1, abort_flag, a.err,
                           kErrTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(t, j % NSB, sv, false, BN / 32, BN / 16);
          } else {
            issue_pv(t, j % NSB, sv, j == 0, 0, BN / 16);
          }
          // With one S buffer the softmax learns that PV_t(j) is done from
          // S_t(j+1), committed after it (below); two buffers need a barrier.
          if constexpr (NSB == 2) umma_commit(bar(kODone0 + t));
          if (NSB == 1 && nj < n_tiles) {
            // S_t(j+1) overwrites P_t(j): issued after PV_t(j), executed in order
            if (t == 0 &&
                !mbar_wait(bar(kKFull0 + nsk), (nj / NSTK) & 1, abort_flag, a.err, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_qk(t, 0, nsk);
            umma_commit(bar(kSFull0 + t));
          }
        }
        if (!ok) break;
        umma_commit(bar(kVEmpty0 + sv));
        if (NSB == 1 && nj < n_tiles) umma_commit(bar(kKEmpty0 + nsk));
      }
      // Every issued MMA has completed before TMEM is released.
      umma_commit(bar(kBarFinal));
      mbar_drain(bar(kBarFinal), 0, a.err, kErrTimeoutMma);
    }
    __syncwarp();  // reconverge before the CTA barrier below
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax rows
    const int t = (warp - 4) >> 2;           // query tile of this warpgroup
    const int r = threadIdx.x - 128 * (1 + t);  // tile row == TMEM lane
    const int h = grp * NQ + t;
    const int q_row = q0 + r;
    const bool valid = q_row < a.S;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const float sl2 = a.scale_log2;
    const uint32_t tO = tmem + lane_off + t * HD;
    if (a.q_fused)
      q_tile_transform<HD, BF16>(sQ + t * C::QT_BYTES, r, q_row, a, bar(kBarQ), bar(kQReady0 + t),
                                 abort_flag, tab ? sQ + C::TAB_COS : 0u, sQ + C::TAB_SIN);
    if constexpr (C::QT) q_split_transform<HD>(a, tmem + lane_off + C::Q_TM, sQ + t * C::QT_BYTES,
                                               r, q_row, h, valid, bar(kQReady0 + t));
    // With a window the running max starts finite: a row can see no key of
    // its first tiles (S row all -inf), and -inf - (-inf) would turn its P
    // into NaN. Any finite score later rescales by ex2(-1e30 - m) = 0.
    float m_run = WIN ? -1e30f : -INFINITY, l_run = 0.f;
    // lowest visible key of this row (none below it with no window)
    const int k_lo = WIN ? q_row - a.window + 1 : INT_MIN;
    bool ok = true;
    for (int j = 0; j < n_tiles; j++) {
      const int b = j % NSB;
      const uint32_t tS = tmem + lane_off + C::S_COL0 + (t * NSB + b) * BN;
      const bool got_s =
          mbar_wait(bar(kSFull0 + t * NSB + b), (j / NSB) & 1, abort_flag, a.err, kErrTimeoutSoftmax);
      __syncwarp();  // reconverge before the warp-wide tcgen05.ld
      if (!__all_sync(0xffffffffu, got_s)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = (j0 + j) * BN;
      // the tile crosses the causal diagonal or the window's lower edge
      const bool diag = k0 + BN - 1 > q_row || (WIN && k0 < k_lo);
      // pass 1: the row max (the S row is the only live data here). The first
      // (up to) 64 columns stay in registers for pass 2, which re-reads only
      // the rest from TMEM.
      constexpr int KEEP = BN < 64 ? BN : 64;
      float xk[KEEP];
      float mt;
      {
        float x[BN];
        {
          uint32_t u[BN];
#pragma unroll
          for (int c = 0; c < BN / 32; c++)
            tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&u[c * 32]));
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < BN; c++) x[c] = __uint_as_float(u[c]);
        }
        if (diag) {
#pragma unroll
          for (int c = 0; c < BN; c++)
            if (k0 + c > q_row || (WIN && k0 + c < k_lo)) x[c] = -INFINITY;
        }
        // 8 independent chains, then a short tree
        float mc[8];
#pragma unroll
        for (int i = 0; i < 8; i++) mc[i] = fmaxf(x[i], x[i + 8]);
#pragma unroll
        for (int c = 16; c < BN; c += 16)
#pragma unroll
          for (int i = 0; i < 8; i++) mc[i] = fmax3(mc[i], x[c + i], x[c + 8 + i]);
        mt = fmax3(fmax3(mc[0], mc[1], mc[2]), fmax3(mc[3], mc[4], mc[5]), fmaxf(mc[6], mc[7]));
#pragma unroll
        for (int c = 0; c < KEEP; c++) xk[c] = x[c];
      }
      const float ms = mt * sl2;
      // lazy rescale: warp-uniform, since tcgen05.ld/st of O are warp-collective
      if (__any_sync(0xffffffffu, ms > m_run + kRescaleThreshold)) {
        const float m_new = fmaxf(m_run, ms);
        const float corr = ex2(m_run - m_new);
        if (j > 0) {
          // PV(j-1) done. With one S buffer, S(j) (waited above) was committed
          // after PV(j-1), so it is. With two, a parity wait on the PV barrier
          // is sound: s_full(j) implies PV(0..j-2) completed (QK(j) is issued
          // after PV(j-2)) and PV(j) needs P(j), so at most one phase is
          // outstanding here.
          const bool got_o = NSB == 1 || mbar_wait(bar(kODone0 + t), (j - 1) & 1, abort_flag,
                                                   a.err, kErrTimeoutSoftmax);
          __syncwarp();
          if (!__all_sync(0xffffffffu, got_o)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < HD / 32; c++) {
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
            tmem_st32(tO + c * 32, o);
          }
          tmem_st_wait();
        }
        l_run *= corr;
        m_run = m_new;
      }
      // pass 2: S in halves (re-read from TMEM unless kept), P = exp2(s*scale
      // - m) -> 16-bit operand in TMEM over the columns already consumed (P
      // half h lands in S columns [h*HALF/2, (h+1)*HALF/2), read before)
      const uint64_t sl2x2 = f2_pack(sl2, sl2), negm2 = f2_pack(-m_run, -m_run);
      uint64_t rsum2[4];
#pragma unroll
      for (int i = 0; i < 4; i++) rsum2[i] = 0;
      constexpr int HALF = BN >= 64 ? 64 : BN;
      static_assert(BN <= 64 || BN == 128, "at most two halves");
      uint32_t un[BN == 128 ? 64 : 1];  // the second half's S columns, loaded ahead
#pragma unroll
      for (int hbase = 0; hbase < BN; hbase += HALF) {
        float x[HALF];
        if (hbase == 0) {  // HALF == KEEP: the first (masked) columns from pass 1
#pragma unroll
          for (int c = 0; c < HALF; c++) x[c] = xk[c];
        } else {  // BN == 128: loaded at the end of the first half
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < HALF; c++) x[c] = __uint_as_float(un[c]);
          if (diag) {
#pragma unroll
            for (int c = 0; c < HALF; c++)
              if (k0 + hbase + c > q_row || (WIN && k0 + hbase + c < k_lo)) x[c] = -INFINITY;
          }
        }
        uint32_t ph[HALF / 2];
#pragma unroll
        for (int c = 0; c < HALF; c += 2) {
          float y0, y1, p0, p1;
          f2_unpack(f2_fma(f2_pack(x[c], x[c + 1]), sl2x2, negm2), y0, y1);
          if (((c >> 1) & 7) < C::EMU_PAIRS) {
            ex2_fma_pair(y0, y1, p0, p1);
          } else {
            p0 = ex2(y0);
            p1 = ex2(y1);
          }
          ph[c / 2] = BF16 ? pack_bf162(p0, p1) : pack_half2(p0, p1);
          if constexpr (SPLIT) {
            // l sums the f16 values the PV MMAs use, so the weights p/l sum
            // to one exactly and P's rounding largely cancels (at scale 1.0
            // one key can carry nearly all the weight: o ~ v(1 + delta)).
            const float2 pr = __half22float2(*reinterpret_cast<const __half2*>(&ph[c / 2]));
            p0 = pr.x;
            p1 = pr.y;
          }
          rsum2[(c >> 1) & 3] = f2_add(rsum2[(c >> 1) & 3], f2_pack(p0, p1));
        }
        // P layout (32-bit TMEM columns, two 16-bit values each): half h
        // takes columns [h*HALF/2, (h+1)*HALF/2), S columns this pass has
        // already read.
        if constexpr (HALF == 64) {
          tmem_st32(tS + hbase / 2, ph);
        } else {  // BN == 32: one 16-column store per plane
          asm volatile(
              "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
              "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(tS),
              "r"(ph[0]), "r"(ph[1]), "r"(ph[2]), "r"(ph[3]), "r"(ph[4]), "r"(ph[5]), "r"(ph[6]),
              "r"(ph[7]), "r"(ph[8]), "r"(ph[9]), "r"(ph[10]), "r"(ph[11]), "r"(ph[12]),
              "r"(ph[13]), "r"(ph[14]), "r"(ph[15])
              : "memory");
        }
        if constexpr (BN == 128) {
          if (hbase == 0) {
            // load the second half now, then publish P's first half: the MMA
            // thread runs PV over keys [0, 64) while this thread does the rest
#pragma unroll
            for (int c = 0; c < 2; c++)
              tmem_ld32(tS + 64 + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&un[c * 32]));
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(bar(kP0Full0 + t * NSB + b));
          }
        }
      }
      {
        float rs[8];
#pragma unroll
        for (int i = 0; i < 4; i++) f2_unpack(rsum2[i], rs[2 * i], rs[2 * i + 1]);
        l_run += ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar(kPFull0 + t * NSB + b));
    }
    // ---- epilogue: O / l -> global
    // Wait on the barrier the MMA thread commits once, after its last MMA: a
    // parity wait on the per-PV barrier is only sound when at most one phase
    // is outstanding, and with two S buffers PV(n-2) can still be in flight.
    bool got_f = ok && mbar_wait(bar(kBarFinal), 0, abort_flag, a.err, kErrTimeoutEpilogue);
    __syncwarp();
    const bool warp_ok = __all_sync(0xffffffffu, got_f);
    const int esz = a.dtype_o == kF32 ? 4 : 2;
    const uint32_t stg = sQ + t * C::STG;
    if (warp_ok) {
      tc_fence_after();
      const float inv_l = 1.f / l_run;
      const int64_t obase = (int64_t)q_row * a.o_stride + (int64_t)h * HD;
#pragma unroll 1
      for (int c = 0; c < HD / 32; c++) {
        uint32_t o[32];
        __syncwarp();  // rows past S skip the stores: reconverge for the warp-wide load
        tmem_ld32(tO + c * 32, o);
        tmem_ld_wait();
        if (!valid && a.n_dst == 0) continue;
        // this row's 32 columns as 16-byte words: 8 for f32, 4 for f16/bf16
        uint4 wv[8];
        if (a.dtype_o == kF32) {
#pragma unroll
          for (int i = 0; i < 8; i++)
            wv[i] = make_uint4(__float_as_uint(__uint_as_float(o[4 * i]) * inv_l),
                               __float_as_uint(__uint_as_float(o[4 * i + 1]) * inv_l),
                               __float_as_uint(__uint_as_float(o[4 * i + 2]) * inv_l),
                               __float_as_uint(__uint_as_float(o[4 * i + 3]) * inv_l));
        } else {
#pragma unroll
          for (int i = 0; i < 4; i++) {
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
              const float lo = __uint_as_float(o[8 * i + 2 * k]) * inv_l;
              const float hi = __uint_as_float(o[8 * i + 2 * k + 1]) * inv_l;
              w[k] = a.dtype_o == kBF16 ? pack_bf162(lo, hi) : pack_half2(lo, hi);
            }
            wv[i] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        const int nw = a.dtype_o == kF32 ? 8 : 4;
        if (a.n_dst == 0) {
          uint4* d = reinterpret_cast<uint4*>(static_cast<char*>(a.o) + (obase + c * 32) * esz);
#pragma unroll
          for (int i = 0; i < 8; i++)
            if (i < nw) d[i] = wv[i];
        } else {
          // staging: 16-byte chunk j of the row's bytes sits in box j / 8
          const int j0 = c * 32 * esz / 16;
#pragma unroll
          for (int i = 0; i < 8; i++) {
            if (i >= nw) break;
            const int j = j0 + i;
            const uint32_t sa = stg + (j >> 3) * C::TILE128 + sw128_offset(r, j & 7);
            asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(sa), "r"(wv[i].x),
                         "r"(wv[i].y), "r"(wv[i].z), "r"(wv[i].w)
                         : "memory");
          }
        }
      }
    }
    if (a.n_dst > 0) {
      // The tile's 128 threads have staged it (every warp arrives here, and
      // the stores go out only if all of them completed); one thread stores
      // it to every destination by TMA and waits only until shared memory has
      // been read: the writes over NVLink drain while the next CTA starts.
      // Rows past S fall outside the maps and are not written.
      fence_async_smem();
      const bool tile_ok = named_bar_and(1 + t, 128, warp_ok);
      if (tile_ok && r == 0) {
        const int nbox = HD * esz / 128;
        for (int d = 0; d < a.n_dst; d++)
          for (int bx = 0; bx < nbox; bx++)
            tma_store_3d(&gmaps.m[d], stg + bx * C::TILE128, bx * (128 / esz), a.h_off + h, q0);
        tma_store_commit();
        tma_store_wait_read();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D map over a [S][Hkv][hd] 16-bit tensor, box {64, 1, BN}, 128-byte swizzle.
bool make_kv_map(CUtensorMap* m, const void* base, int S, int Hkv, int hd, int BN,
                        bool bf16) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)Hkv, (cuuint64_t)S};
  cuuint64_t strides[2] = {(cuuint64_t)hd * 2, (cuuint64_t)Hkv * hd * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)BN};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D map over raw query rows [S][H][hd] (16-bit) whose rows are row_stride
// elements apart (a fused q/k/v projection output is read in place), box
// {64, 1, 128}, 128-byte swizzle.
static bool make_q_map(CUtensorMap* m, const void* base, int S, int H, int hd,
                       int64_t row_stride, bool bf16) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)H, (cuuint64_t)S};
  cuuint64_t strides[2] = {(cuuint64_t)hd * 2, (cuuint64_t)row_stride * 2};
  cuuint32_t box[3] = {64, 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D map over a RoPE table [rows][half] f32, box {32, 128}, 128-byte swizzle.
static bool make_table_map(CUtensorMap* m, const float* base, int rows, int half) {
  auto fn = encode_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)half, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)half * 4};
  cuuint32_t box[2] = {32, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D map over a gathered output [S][H_total][hd] of dtype dt (16-bit or
// f32), box {128 bytes of one head row, 1 head, 128 rows}, 128-byte swizzle.
static bool make_out_map(CUtensorMap* m, uint64_t base, int S, int64_t h_total, int hd, int dt) {
  auto fn = encode_fn();
  if (!fn) return false;
  const int es = dt == kF32 ? 4 : 2;
  cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)h_total, (cuuint64_t)S};
  cuuint64_t strides[2] = {(cuuint64_t)hd * es, (cuuint64_t)(h_total * hd * es)};
  cuuint32_t box[3] = {(cuuint32_t)(128 / es), 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType ty = dt == kF32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dt == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(m, ty, 3, reinterpret_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int HD, int BN, int NQ, bool SPLIT, bool BF16, int NSTK, int NSTV, bool WIN>
static cudaError_t run_prefill_k(const PrefillArgs& a, const void* q16, const void* k16,
                                 const void* v16, const void* split, const GatherSpec* g,
                                 cudaStream_t st) {
  using C = PfCfg<HD, BN, NQ, SPLIT, NSTK, NSTV>;
  auto kern = prefill_tc_kernel<HD, BN, NQ, SPLIT, BF16, NSTK, NSTV, WIN>;
  static unsigned configured = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(__atomic_load_n(&configured, __ATOMIC_ACQUIRE) & (1u << (dev & 31)))) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    __atomic_fetch_or(&configured, 1u << (dev & 31), __ATOMIC_RELEASE);
  }
  CUtensorMap mq, mql, mk, mv, mkl, mvl;
  if (SPLIT && !PfCfg<HD, BN, NQ, SPLIT, NSTK, NSTV>::QT) {
    const __half* qp = reinterpret_cast<const __half*>(q16);
    if (!make_kv_map(&mq, qp, a.S, a.H, HD, 128, false) ||
        !make_kv_map(&mql, qp + (size_t)a.S * a.H * HD, a.S, a.H, HD, 128, false))
      return cudaErrorInvalidValue;
  } else if (C::QT) {
    // the kernel reads the raw q rows itself (q_raw): no query tensor map
  } else if (a.q_fused) {
    if (!make_q_map(&mq, q16, a.S, a.H, HD, a.q_stride, BF16)) return cudaErrorInvalidValue;
    mql = mq;
  } else {
    if (!make_kv_map(&mq, q16, a.S, a.H, HD, 128, BF16)) return cudaErrorInvalidValue;
    mql = mq;
  }
  if (SPLIT) {
    const size_t plane = (size_t)a.S * a.Hkv * HD;
    const __half* sp = reinterpret_cast<const __half*>(split);
    if (!make_kv_map(&mk, sp, a.S, a.Hkv, HD, BN, false) ||
        !make_kv_map(&mkl, sp + plane, a.S, a.Hkv, HD, BN, false) ||
        !make_kv_map(&mv, sp + 2 * plane, a.S, a.Hkv, HD, BN, false) ||
        !make_kv_map(&mvl, sp + 3 * plane, a.S, a.Hkv, HD, BN, false))
      return cudaErrorInvalidValue;
  } else {
    if (!make_kv_map(&mk, k16, a.S, a.Hkv, HD, BN, BF16) ||
        !make_kv_map(&mv, v16, a.S, a.Hkv, HD, BN, BF16))
      return cudaErrorInvalidValue;
    mkl = mk;
    mvl = mv;
  }
  GatherMaps gm;
  memset(&gm, 0, sizeof(gm));
  PrefillArgs ka = a;
  ka.n_dst = 0;
  if (C::QT) {
    // unused by this kernel; any valid map fills the parameter slots
    mq = mk;
    mql = mk;
    ka.q_raw = q16;
  }
  if (g && g->n_dst > 0) {
    if (g->n_dst > kMaxGather) return cudaErrorInvalidValue;
    for (int d = 0; d < g->n_dst; d++)
      if (!make_out_map(&gm.m[d], g->dst[d], a.S, g->n_heads_total, HD, a.dtype_o))
        return cudaErrorInvalidValue;
    ka.n_dst = g->n_dst;
    ka.h_off = g->h_off;
  }
  const int n_qt = (a.S + 127) / 128;
  // staged RoPE table rows (fused q prep): 2-D maps over cos / sin [S][HD/2]
  // f32, box {32 pairs, 128 rows}; without them the kernel reads the rows
  // from global memory
  CUtensorMap mcos = mk, msin = mk;
  ka.tab_smem = 0;
  if (C::TAB && a.q_fused && a.cos_t && a.sin_t && make_table_map(&mcos, a.cos_t, a.S, HD / 2) &&
      make_table_map(&msin, a.sin_t, a.S, HD / 2))
    ka.tab_smem = 1;
  kern<<<(unsigned)(n_qt * (a.H / NQ)), C::THREADS, C::SMEM, st>>>(mq, mql, mk, mv, mkl, mvl, mcos,
                                                                     msin, gm,
                                                                     ka);
  return cudaGetLastError();
}

// A window of at least S rows masks nothing: the causal kernel serves it.
template <int HD, int BN, int NQ, bool SPLIT, bool BF16, int NSTK, int NSTV>
static cudaError_t run_prefill(const PrefillArgs& a, const void* q16, const void* k16,
                               const void* v16, const void* split, const GatherSpec* g,
                               cudaStream_t st) {
  return (a.window > 0 && a.window < a.S)
             ? run_prefill_k<HD, BN, NQ, SPLIT, BF16, NSTK, NSTV, true>(a, q16, k16, v16, split,
                                                                        g, st)
             : run_prefill_k<HD, BN, NQ, SPLIT, BF16, NSTK, NSTV, false>(a, q16, k16, v16, split,
                                                                         g, st);
}

bool prefill_tc_supported(int hd) { return hd == 64 || hd == 128 || hd == 256; }

cudaError_t launch_prefill_tc(const PrefillArgs& a, int hd, const void* q16, const void* k16,
                              const void* v16, bool bf16, const void* split,
                              const GatherSpec* g, cudaStream_t st) {
  // Two query tiles per CTA (the heads of a GQA pair share each K/V tile)
  // when the group size is even and that is the faster grid. Causal query
  // tiles differ in length (1 to n_qt KV tiles) and one CTA runs per SM, so
  // a grid takes about max(its longest item, the average work per SM). A
  // pair's longest item is twice a single head's, which decides it when the
  // grid is small (a head-sharded rank with few heads); otherwise the pair
  // wins, its per-head rate being ~1/0.87 of the one-tile kernel's
  // (measured on config 3).
  const double n_qt = (double)((a.S + 127) / 128);
  const double per_sm = (double)a.H * n_qt * (n_qt + 1) / 2 / sm_count();
  const bool pair = ((a.H / a.Hkv) % 2) == 0 &&
                    std::max(2 * n_qt, per_sm) <= std::max(n_qt, per_sm) / 0.87;
  // A contiguous [S][H][hd] output is a one-destination gather: its tiles are
  // staged in shared memory and leave by TMA store, 1.4% faster on config 3
  // than per-thread 16-byte stores (bit-identical). Strided outputs keep the
  // per-thread stores.
  uint64_t self_dst = reinterpret_cast<uint64_t>(a.o);
  GatherSpec self_g{1, 0, a.H, &self_dst};
  if (!g && a.o && a.o_stride == (int64_t)a.H * hd && (self_dst & 15) == 0) g = &self_g;
  if (split) {
    switch (hd) {
      case 64:
        return run_prefill<64, 128, 1, true, false, 2, 2>(a, q16, k16, v16, split, g, st);
      case 128: return run_prefill<128, 64, 1, true, false, 2, 2>(a, q16, k16, v16, split, g, st);
      case 256: return run_prefill<256, 64, 1, true, false, 1, 1>(a, q16, k16, v16, split, g, st);
    }
  } else if (bf16) {
    switch (hd) {
      case 64:
        return pair ? run_prefill<64, 128, 2, false, true, 4, 3>(a, q16, k16, v16, split, g, st)
                    : run_prefill<64, 128, 1, false, true, 4, 3>(a, q16, k16, v16, split, g, st);
      case 128:
        return pair ? run_prefill<128, 128, 2, false, true, 3, 2>(a, q16, k16, v16, split, g, st)
                    : run_prefill<128, 128, 1, false, true, 3, 2>(a, q16, k16, v16, split, g, st);
      case 256: return run_prefill<256, 64, 1, false, true, 2, 2>(a, q16, k16, v16, split, g, st);
    }
  } else {
    switch (hd) {
      case 64:
        return pair ? run_prefill<64, 128, 2, false, false, 4, 3>(a, q16, k16, v16, split, g, st)
                    : run_prefill<64, 128, 1, false, false, 4, 3>(a, q16, k16, v16, split, g, st);
      case 128:
        return pair ? run_prefill<128, 128, 2, false, false, 3, 2>(a, q16, k16, v16, split, g, st)
                    : run_prefill<128, 128, 1, false, false, 3, 2>(a, q16, k16, v16, split, g, st);
      case 256: return run_prefill<256, 64, 1, false, false, 2, 2>(a, q16, k16, v16, split, g, st);
    }
  }
  return cudaErrorNotSupported;
}

}  // namespace eb
