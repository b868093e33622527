// eb_decode_tc.cu -- split-K flash-decoding on tcgen05 tensor cores for
// 16-bit (f16/bf16) KV caches.
//
// Replaces attn_decode (crates/eyebrowse-kernels/src/attention.rs:52-90,
// :124-162) with the decode branch's q/k/v RMSNorm, RoPE and kv_write
// (crates/eyebrowse-nn/src/attention.rs:133-168), like decode_kernel, but
// moves the per-byte arithmetic onto the tensor cores so that the CTA does
// nothing per cache byte except stream it: the G query heads of one KV head
// are rows 0..G-1 of a 128-row MMA operand, S = Q K^T and O += P V run as
// M=128 tcgen05 MMAs over TMA-fed [BN x 64] K/V tiles, and a single warp
// runs the online softmax of the G real rows (one TMEM lane each).
//
// One CTA = (context chunk, KV head group, sequence), 96 threads:
//   warp 0  rows: new k/v row -> cache (last chunk), Q rows -> operand,
//           softmax, partial/final output, split-K combine (last CTA)
//   warp 1  TMA producer (K/V ring, NST stages)
//   warp 2  TMEM owner + MMA issuer (two S buffers: QK of tile j+1 runs
//           while the softmax of tile j works)
// With more than one chunk the partial (m, l, O) goes to the workspace and
// the last CTA of the (sequence, head group) merges them (atomic ticket, no
// spin-wait), exactly as decode_kernel does.
#include <type_traits>

#include "eb_common.cuh"
#include "eb_decode_out.cuh"
#include "eb_kernels.cuh"
#include "eb_rowops.cuh"
#include "eb_tc.cuh"

namespace eb {

template <int HD, int BN, int NST>
struct DtcCfg {
  static constexpr int HB = HD / 64;
  static constexpr int TILE128 = 128 * 128;
  static constexpr int Q_BYTES = HB * TILE128;  // 128-row operand, rows >= 32 never written
  static constexpr int KV_BOX = BN * 128;
  static constexpr int K_BYTES = HB * KV_BOX;
  static constexpr int STAGE_BYTES = 2 * K_BYTES;
  static constexpr int BAR_OFF = Q_BYTES + NST * STAGE_BYTES;
  static constexpr int SMEM = BAR_OFF + 512 + 1024;
  static constexpr int S_COL0 = HD;  // O at [0, HD), S/P buffers at [HD, HD + 2*BN)
  static constexpr int TMEM_COLS = constexpr_pow2ceil(HD + 2 * BN);
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(TMEM_COLS <= 512, "tensor memory budget");
};

template <int HD, int BN, bool BF16, int NST>
__global__ void __launch_bounds__(96)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, DecodeArgs a, int gsubs) {
  using C = DtcCfg<HD, BN, NST>;
  using TC = std::conditional_t<BF16, __nv_bfloat16, __half>;
  constexpr int E = HD / 32;
  // KV-head group fastest: the heads of one chunk share cache rows (and DRAM
  // pages) and run side by side. Chunk index slowest: every sequence's first
  // chunk is dispatched before any second chunk, so the last waves hold only
  // the later chunks of the longest contexts, not whichever full chunks came
  // last in sequence order (an idle tail of up to one full chunk per SM).
  const int grp = blockIdx.x, b = blockIdx.y, c = blockIdx.z;
  const int G = a.H / a.Hkv / gsubs;  // query heads handled here (<= 32)
  const int kvh = grp / gsubs, sub = grp % gsubs;
  const int head0 = kvh * (G * gsubs) + sub * G;
  const int pos = a.positions ? a.positions[b] : a.pos_scalar;
  // rows [row_lo, pos]: the whole context, or the last `window` rows of it
  const int row_lo = a.window > 0 ? max(0, pos - a.window + 1) : 0;
  const int n_rows = pos + 1 - row_lo;
  const int n_chunks = (n_rows + a.chunk - 1) / a.chunk;
  if (c >= n_chunks) return;
  const int row_begin = row_lo + c * a.chunk;
  const int row_end = min(row_begin + a.chunk, pos + 1);
  const int n_tiles = (row_end - row_begin + BN - 1) / BN;
  const bool last_chunk = c == n_chunks - 1;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sKV = sQ + C::Q_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::BAR_OFF + 384);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::BAR_OFF + 392);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  // one S-full and one P-full barrier per S buffer: with two buffers the
  // softmax may finish P(j+1) before the MMA thread's wait sees P(j), and a
  // single P barrier would then be two phases ahead of that parity wait
  constexpr int kQ = 0, kFinal = 1, kSFull0 = 2, kPFull0 = 4, kODone = 6, kKFull0 = 7;
  constexpr int kKEmpty0 = kKFull0 + NST, kVFull0 = kKEmpty0 + NST, kVEmpty0 = kVFull0 + NST;
  constexpr int kNumBars = kVEmpty0 + NST;
  static_assert(kNumBars * 8 <= 384, "barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(bar(kQ), 32);
    mbar_init(bar(kFinal), 1);
    mbar_init(bar(kSFull0), 1);
    mbar_init(bar(kSFull0 + 1), 1);
    mbar_init(bar(kPFull0), 32);
    mbar_init(bar(kPFull0 + 1), 32);
    for (int i = kODone; i < kNumBars; i++) mbar_init(bar(i), 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_async_smem();
  }
  if (warp == 1 && lane == 0) {
    tma_prefetch_map(&tmK);
    tma_prefetch_map(&tmV);
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 1) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int kiss[NST], viss[NST];
      for (int s = 0; s < NST; s++) kiss[s] = viss[s] = 0;
      // Only the chunk holding row pos reads the row warp 0 writes before kQ;
      // every other chunk starts streaming at once.
      if (!(a.k_new && last_chunk) || mbar_wait(bar(kQ), 0, abort_flag, a.err, kErrTimeoutTma)) {
        for (int j = 0; j < n_tiles; j++) {
          const int st = j % NST;
          const int row = row_begin + j * BN;
          const uint32_t kst = sKV + st * C::STAGE_BYTES;
          const uint32_t vst = kst + C::K_BYTES;
          if (j >= NST && !mbar_wait(bar(kKEmpty0 + st), (j / NST - 1) & 1, abort_flag, a.err,
                                     kErrTimeoutTma))
            break;
          mbar_arrive_expect_tx(bar(kKFull0 + st), C::K_BYTES);
#pragma unroll
          for (int hb = 0; hb < C::HB; hb++)
            tma_load_4d(kst + hb * C::KV_BOX, &tmK, bar(kKFull0 + st), hb * 64, kvh, row, b);
          kiss[st]++;
          if (j >= NST && !mbar_wait(bar(kVEmpty0 + st), (j / NST - 1) & 1, abort_flag, a.err,
                                     kErrTimeoutTma))
            break;
          mbar_arrive_expect_tx(bar(kVFull0 + st), C::K_BYTES);
#pragma unroll
          for (int hb = 0; hb < C::HB; hb++)
            tma_load_4d(vst + hb * C::KV_BOX, &tmV, bar(kVFull0 + st), hb * 64, kvh, row, b);
          viss[st]++;
        }
      }
      for (int s = 0; s < NST; s++) {
        if (kiss[s]) mbar_drain(bar(kKFull0 + s), (kiss[s] - 1) & 1, a.err, kErrTimeoutTma);
        if (viss[s]) mbar_drain(bar(kVFull0 + s), (viss[s] - 1) & 1, a.err, kErrTimeoutTma);
      }
    }
    __syncwarp();  // reconverge before the CTA barrier below
  } else if (warp == 2) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16(128, BN, BF16, false);
      constexpr uint32_t idesc_pv = idesc_f16(128, HD, BF16, true);
      auto issue_qk = [&](int buf, int st) {
        const uint32_t kst = sKV + st * C::STAGE_BYTES;
        const uint32_t tS = tmem + C::S_COL0 + buf * BN;
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
          const int hb = kk >> 2, w = kk & 3;
          umma_ss(tS, sdesc_sw128(sQ + hb * C::TILE128 + w * 32, 16, 1024),
                  sdesc_sw128(kst + hb * C::KV_BOX + w * 32, 16, 1024), idesc_qk, kk > 0);
        }
      };
      auto issue_pv = [&](int buf, int st, bool first) {
        const uint32_t vst = sKV + st * C::STAGE_BYTES + C::K_BYTES;
        const uint32_t tP = tmem + C::S_COL0 + buf * BN;
#pragma unroll
        for (int kk = 0; kk < BN / 16; kk++)
          umma_ts(tmem, tP + kk * 8, sdesc_sw128(vst + kk * 16 * 128, C::KV_BOX, 1024), idesc_pv,
                  (!first || kk > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait(bar(kQ), 0, abort_flag, a.err, kErrTimeoutMma) &&
                mbar_wait(bar(kKFull0), 0, abort_flag, a.err, kErrTimeoutMma);
      if (ok) {
        tc_fence_after();
        issue_qk(0, 0);
        umma_commit(bar(kSFull0));
        umma_commit(bar(kKEmpty0));
      }
      for (int j = 0; ok && j < n_tiles; j++) {
        const int st = j % NST, nj = j + 1, nst = nj % NST;
        if (nj < n_tiles) {  // S(j+1) into the other buffer ahead of PV(j)
          if (!mbar_wait(bar(kKFull0 + nst), (nj / NST) & 1, abort_flag, a.err, kErrTimeoutMma))
            break;
          tc_fence_after();
          issue_qk(nj & 1, nst);
          umma_commit(bar(kSFull0 + (nj & 1)));
          umma_commit(bar(kKEmpty0 + nst));
        }
        if (!mbar_wait(bar(kPFull0 + (j & 1)), (j >> 1) & 1, abort_flag, a.err, kErrTimeoutMma) ||
            !mbar_wait(bar(kVFull0 + st), (j / NST) & 1, abort_flag, a.err, kErrTimeoutMma))
          break;
        tc_fence_after();
        issue_pv(j & 1, st, j == 0);
        umma_commit(bar(kODone));
        umma_commit(bar(kVEmpty0 + st));
      }
      umma_commit(bar(kFinal));
      mbar_drain(bar(kFinal), 0, a.err, kErrTimeoutMma);
    }
    __syncwarp();  // reconverge before the CTA barrier below
  } else {
    // ------------------------------------------------------------ rows (warp 0)
    const float* cos_row = a.cos_t ? a.cos_t + (int64_t)pos * (HD / 2) : nullptr;
    const float* sin_row = a.sin_t ? a.sin_t + (int64_t)pos * (HD / 2) : nullptr;
    if (a.k_new && last_chunk) {
      // the new token: k -> norm -> RoPE, v -> norm, written to cache row pos
      // (every sub-group CTA of this KV head writes the same bits)
#pragma unroll 1
      for (int which = 0; which < 2; which++) {
        float v[E];
        ld_row<E>(which ? a.v_new : a.k_new, (int64_t)b * a.kv_bstride + (int64_t)kvh * HD + lane * E,
                  a.dtype_kv, v);
        warp_kv_row<E>(v, which ? a.v_norm_w : a.k_norm_w, a.eps, which ? nullptr : cos_row,
                       which ? nullptr : sin_row, lane);
        st_row<E>(which ? a.vcache : a.kcache,
                  (int64_t)b * a.cache_bstride + ((int64_t)pos * a.Hkv + kvh) * HD + lane * E,
                  BF16 ? kBF16 : kF16, v);
      }
      // generic-proxy global writes -> visible to the TMA loads that follow
      asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    // Q rows 0..31 of the operand: lane r < G holds query head head0 + r, the
    // other lanes write zero rows (keeps their softmax lanes finite)
    {
      const int r = lane;
      const bool real = r < G;
      const int64_t qbase = (int64_t)b * a.q_bstride + (int64_t)(head0 + (real ? r : 0)) * HD;
      float inv = 1.f;
      if (real && a.q_norm_w) {
        float ss = 0.f;
        for (int d = 0; d < HD; d += 8) {
          float f[8];
          load8_any(a.q, qbase + d, a.dtype_q, f);
#pragma unroll
          for (int i = 0; i < 8; i++) ss = __fadd_rn(ss, __fmul_rn(f[i], f[i]));
        }
        inv = 1.0f / sqrtf(ss / (float)HD + a.eps);
      }
#pragma unroll 1
      for (int p0 = 0; p0 < HD / 2; p0 += 8) {
        float x1[8], x2[8];
        if (real) {
          load8_any(a.q, qbase + p0, a.dtype_q, x1);
          load8_any(a.q, qbase + HD / 2 + p0, a.dtype_q, x2);
          if (a.q_norm_w) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
              x1[i] = __fmul_rn(__fmul_rn(x1[i], inv), a.q_norm_w[p0 + i]);
              x2[i] = __fmul_rn(__fmul_rn(x2[i], inv), a.q_norm_w[HD / 2 + p0 + i]);
            }
          }
          if (cos_row) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
              const float cc = cos_row[p0 + i], sn = sin_row[p0 + i];
              const float y1 = __fsub_rn(__fmul_rn(x1[i], cc), __fmul_rn(x2[i], sn));
              const float y2 = __fadd_rn(__fmul_rn(x2[i], cc), __fmul_rn(x1[i], sn));
              x1[i] = y1;
              x2[i] = y2;
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; i++) x1[i] = x2[i] = 0.f;
        }
        const int c1 = p0 / 8, c2 = (HD / 2 + p0) / 8;
        st_chunk<BF16>(sQ + (c1 >> 3) * C::TILE128 + sw128_offset(r, c1 & 7), x1);
        st_chunk<BF16>(sQ + (c2 >> 3) * C::TILE128 + sw128_offset(r, c2 & 7), x2);
      }
      fence_async_smem();
      mbar_arrive(bar(kQ));
    }

    const float sl2 = a.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; j++) {
      const int buf = j & 1, st = j % NST;
      const uint32_t tS = tmem + C::S_COL0 + buf * BN;  // warp 0: TMEM lanes 0..31
      const bool got_s =
          mbar_wait(bar(kSFull0 + buf), (j >> 1) & 1, abort_flag, a.err, kErrTimeoutSoftmax);
      __syncwarp();
      if (!__all_sync(0xffffffffu, got_s)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float x[BN];
      {
        uint32_t u[BN];
#pragma unroll
        for (int cc = 0; cc < BN / 32; cc++)
          tmem_ld32(tS + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(&u[cc * 32]));
        tmem_ld_wait();
#pragma unroll
        for (int cc = 0; cc < BN; cc++) x[cc] = __uint_as_float(u[cc]);
      }
      const int valid = row_end - (row_begin + j * BN);  // rows of this tile <= pos
      if (valid < BN) {
#pragma unroll
        for (int cc = 0; cc < BN; cc++)
          if (cc >= valid) x[cc] = -INFINITY;
      }
      float mt;
      {
        float mc[8];
#pragma unroll
        for (int i = 0; i < 8; i++) mc[i] = fmaxf(x[i], x[i + 8]);
#pragma unroll
        for (int cc = 16; cc < BN; cc += 16)
#pragma unroll
          for (int i = 0; i < 8; i++) mc[i] = fmax3(mc[i], x[cc + i], x[cc + 8 + i]);
        mt = fmax3(fmax3(mc[0], mc[1], mc[2]), fmax3(mc[3], mc[4], mc[5]), fmaxf(mc[6], mc[7]));
      }
      const float ms = mt * sl2;
      if (__any_sync(0xffffffffu, ms > m_run + kRescaleThreshold)) {
        const float m_new = fmaxf(m_run, ms);
        const float corr = ex2(m_run - m_new);
        if (j > 0) {
          // PV(j-1) done; at most one o_done phase is outstanding here
          const bool got_o =
              mbar_wait(bar(kODone), (j - 1) & 1, abort_flag, a.err, kErrTimeoutSoftmax);
          __syncwarp();
          if (!__all_sync(0xffffffffu, got_o)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int cc = 0; cc < HD / 32; cc++) {
            uint32_t o[32];
            tmem_ld32(tmem + cc * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
            tmem_st32(tmem + cc * 32, o);
          }
          tmem_st_wait();
        }
        l_run *= corr;
        m_run = m_new;
      }
      const float neg_m = -m_run;
      float rsum[8];
#pragma unroll
      for (int i = 0; i < 8; i++) rsum[i] = 0.f;
      uint32_t ph[BN / 2];
#pragma unroll
      for (int cc = 0; cc < BN; cc += 2) {
        const float p0 = ex2(fmaf(x[cc], sl2, neg_m));
        const float p1 = ex2(fmaf(x[cc + 1], sl2, neg_m));
        rsum[(cc >> 1) & 7] += p0 + p1;
        ph[cc / 2] = BF16 ? pack_bf162(p0, p1) : pack_half2(p0, p1);
      }
      l_run += ((rsum[0] + rsum[1]) + (rsum[2] + rsum[3])) + ((rsum[4] + rsum[5]) + (rsum[6] + rsum[7]));
#pragma unroll
      for (int cc = 0; cc < BN / 64; cc++)
        tmem_st32(tS + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(&ph[cc * 32]));
      if (valid < BN) {
        // Rows past pos hold whatever the cache holds (possibly NaN): zero them
        // in the V tile so that P = 0 cannot meet them (0 * NaN = NaN).
        const bool got_v =
            mbar_wait(bar(kVFull0 + st), (j / NST) & 1, abort_flag, a.err, kErrTimeoutSoftmax);
        __syncwarp();
        if (!__all_sync(0xffffffffu, got_v)) {
          ok = false;
          break;
        }
        uint8_t* vt = smem + C::Q_BYTES + st * C::STAGE_BYTES + C::K_BYTES;
        const int nz = (BN - valid) * 8 * C::HB;  // 16-byte pieces to clear
        for (int i = lane; i < nz; i += 32) {
          const int box = i / ((BN - valid) * 8);
          const int rem = i % ((BN - valid) * 8);
          const int row = valid + rem / 8, piece = rem % 8;
          *reinterpret_cast<uint4*>(vt + box * C::KV_BOX + (row >> 3) * 1024 + (row & 7) * 128 +
                                    piece * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_async_smem();
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar(kPFull0 + buf));
    }
    // ---- partial or final output
    bool got_f = ok && mbar_wait(bar(kFinal), 0, abort_flag, a.err, kErrTimeoutEpilogue);
    __syncwarp();
    if (__all_sync(0xffffffffu, got_f)) {
      tc_fence_after();
      const bool real = lane < G;
      const int h = head0 + lane;
      const bool split = n_chunks > 1;
      const float inv_l = 1.f / l_run;
      float* pacc = split ? a.ws_acc + (((int64_t)b * a.H + h) * a.cmax + c) * HD : nullptr;
#pragma unroll 1
      for (int cc = 0; cc < HD / 32; cc++) {
        uint32_t o[32];
        tmem_ld32(tmem + cc * 32, o);
        tmem_ld_wait();
        if (real) {
          if (split) {
            float4* dst = reinterpret_cast<float4*>(pacc + cc * 32);
#pragma unroll
            for (int i = 0; i < 8; i++)
              dst[i] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                   __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3]));
          } else {
            float ov[32];
#pragma unroll
            for (int i = 0; i < 32; i++) ov[i] = __uint_as_float(o[i]) * inv_l;
            dec_store32(a, b, h, HD, cc * 32, ov);
          }
        }
      }
      if (split) {
        if (real) {
          float* ml = a.ws_ml + (((int64_t)b * a.H + h) * a.cmax + c) * 2;
          ml[0] = m_run;
          ml[1] = l_run;
        }
        __threadfence();
        __syncwarp();
        unsigned* cnt = a.ws_cnt + (int64_t)b * gridDim.x + grp;
        unsigned ticket = 0;
        if (lane == 0) ticket = atomicAdd(cnt, 1u);
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        if (ticket == (unsigned)(n_chunks - 1)) {
          // last CTA of this (sequence, head group): merge the chunk partials.
          // Per head: lanes over the chunks for the max and the weights
          // 2^(m_c - M), which go to the K/V ring (idle now: every MMA has
          // completed and every TMA load has landed); then each lane sums its
          // columns over the chunks with 8 partial loads in flight.
          __threadfence();
          float* wts = reinterpret_cast<float*>(smem + C::Q_BYTES);  // [n_chunks <= 256]
          for (int g = 0; g < G; g++) {
            const int hh = head0 + g;
            const float* mlg = a.ws_ml + (((int64_t)b * a.H + hh) * a.cmax) * 2;
            float M = -INFINITY;
            for (int k = lane; k < n_chunks; k += 32) M = fmaxf(M, __ldcg(mlg + 2 * k));
            M = warp_max(M);
            float L = 0.f;
            for (int k = lane; k < n_chunks; k += 32) {
              const float w = ex2(__ldcg(mlg + 2 * k) - M);
              wts[k] = w;
              L += __ldcg(mlg + 2 * k + 1) * w;
            }
            L = warp_sum(L);
            __syncwarp();
            const float* accg = a.ws_acc + (((int64_t)b * a.H + hh) * a.cmax) * HD;
            for (int d = lane; d < HD; d += 32) {
              float O8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
              int k = 0;
              for (; k + 8 <= n_chunks; k += 8) {
#pragma unroll
                for (int u = 0; u < 8; u++) O8[u] += __ldcg(accg + (int64_t)(k + u) * HD + d) * wts[k + u];
              }
              for (; k < n_chunks; k++) O8[0] += __ldcg(accg + (int64_t)k * HD + d) * wts[k];
              const float O = ((O8[0] + O8[1]) + (O8[2] + O8[3])) + ((O8[4] + O8[5]) + (O8[6] + O8[7]));
              dec_store(a, b, hh, HD, d, O / L);
            }
            __syncwarp();  // wts is rewritten for the next head
          }
          if (lane == 0) *cnt = 0u;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// 4-D map over B caches [max_seq][Hkv][hd] (16-bit) at a batch stride, box {64, 1, BN, 1}.
static bool make_cache_map(CUtensorMap* m, const void* base, int batch, int max_seq, int Hkv,
                           int hd, int64_t bstride_elems, int BN, bool bf16) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)hd, (cuuint64_t)Hkv, (cuuint64_t)max_seq, (cuuint64_t)batch};
  const cuuint64_t bs = (cuuint64_t)(batch > 1 ? bstride_elems : (int64_t)max_seq * Hkv * hd) * 2;
  cuuint64_t strides[3] = {(cuuint64_t)hd * 2, (cuuint64_t)Hkv * hd * 2, bs};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)BN, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
            const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int HD, int BN, bool BF16, int NST>
static cudaError_t run_decode_tc(const DecodeArgs& a, int batch, int gsubs, cudaStream_t st) {
  using C = DtcCfg<HD, BN, NST>;
  auto kern = decode_tc_kernel<HD, BN, BF16, NST>;
  static unsigned configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(__atomic_load_n(&configured, __ATOMIC_ACQUIRE) & (1u << (dev & 31)))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    __atomic_fetch_or(&configured, 1u << (dev & 31), __ATOMIC_RELEASE);
  }
  CUtensorMap mk, mv;
  if (!make_cache_map(&mk, a.kcache, batch, a.max_seq, a.Hkv, HD, a.cache_bstride, BN, BF16) ||
      !make_cache_map(&mv, a.vcache, batch, a.max_seq, a.Hkv, HD, a.cache_bstride, BN, BF16))
    return cudaErrorInvalidValue;
  dim3 grid(a.Hkv * gsubs, batch, a.cmax);
  kern<<<grid, 96, C::SMEM, st>>>(mk, mv, a, gsubs);
  return cudaGetLastError();
}

// f16 caches only: the MMA's A and B share one type, so a bf16 cache would
// force q and P to bf16 (8-bit mantissa) and cost ~2e-3 relative error;
// bf16 caches take decode_kernel, which computes in f32.
bool decode_tc_supported(int hd, int dtype_cache, int group) {
  return (hd == 64 || hd == 128 || hd == 256) && dtype_cache == kF16 && group >= 1 && group <= 32;
}

cudaError_t launch_decode_tc(const DecodeArgs& a, int dtype_cache, int batch, cudaStream_t st) {
  const bool bf16 = dtype_cache == kBF16;
  const int G = a.H / a.Hkv;
  const int gsubs = 1;  // up to 32 query heads share one CTA
  if (G > 32) return cudaErrorNotSupported;
  switch (a.hd) {
    case 64:
      return bf16 ? run_decode_tc<64, 64, true, 4>(a, batch, gsubs, st)
                  : run_decode_tc<64, 64, false, 4>(a, batch, gsubs, st);
    case 128:
      return bf16 ? run_decode_tc<128, 64, true, 2>(a, batch, gsubs, st)
                  : run_decode_tc<128, 64, false, 2>(a, batch, gsubs, st);
    case 256:
      return bf16 ? run_decode_tc<256, 64, true, 2>(a, batch, gsubs, st)
                  : run_decode_tc<256, 64, false, 2>(a, batch, gsubs, st);
  }
  return cudaErrorNotSupported;
}

}  // namespace eb
