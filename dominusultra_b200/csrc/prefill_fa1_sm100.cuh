// Causal prefill for sm_100a on pre-rotated keys, one 128-row query tile per CTA and two CTAs per
// SM (head_dim 16..64).
//
// Mathematics of the reference prefill_kernel (dominus_ultra.py:119-285): out =
// softmax(R(Q) R(K)^T * scale, causal) V and the natural-log LSE per row, query head h reading KV
// head h / (Hq / Hkv) (dominus_ultra.py:168). R(K) arrives rotated, as fp16, from the standalone
// rotary kernel (rope_sm100.cuh); Q is rotated here in fp32 by the thread that owns the row.
//
// Same pipeline as the two-tile kernel (prefill_fa_sm100.cuh) for a single tile, sized so that
// two CTAs share an SM (256 TMEM columns, under half the shared memory and registers each): the
// hardware then overlaps one CTA's start-up (query load and rotation, first Q K^T) and wind-down
// (last P V, epilogue) with the other CTA's steady state, and the two tiles on an SM never wait
// for each other's softmax. Per CTA:
//   warps 0-3  softmax: rotate the Q row, then per KV tile: wait S, load it (S is handed back at
//              once: the next Q K^T overwrites it while the exponentials run), mask the diagonal
//              tile, online softmax in the log2 domain (lazy rescale by 2^8), P to its own TMEM
//              columns after the previous P V completes, signal; finally out = O/l, lse.
//   warp 4     TMA: the query tile, then the K ring.   warp 6  TMA: the V ring.
//   warp 5     TMEM owner and MMA issuer (whole warp walks the schedule, one elected lane
//              issues; QK(j+1) as soon as the softmax has loaded S(j), PV(j) once P(j) is in).
//   warp 7     idle (setmaxnreg works on whole warpgroups).
// TMEM: S [0, 128), O [128, 128 + D), P [128 + D, 192 + D): 256 columns.
// Every mbarrier wait is bounded (du_ptx.cuh).
#pragma once

#include "du_ptx.cuh"
#include "prefill_sm100.cuh"

#ifndef DU_FA1_POLY_MASK
#define DU_FA1_POLY_MASK 0x11
#endif

namespace du {

template <int D>
struct Fa1Shape {
  static constexpr int BM = 128;
  static constexpr int BN = 128;
  static constexpr int SPAN = (2 * D >= 128) ? 128 : 2 * D;
  static constexpr int NBLK = 2 * D / SPAN;
  static constexpr int NSK = 3;
  static constexpr int NSV = 2;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + NSK * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + NSV * KV_BYTES;
  // barriers: q_full, q_rot, k_full[NSK], k_empty[NSK], v_full[NSV], v_empty[NSV], s_full,
  //           s_consumed, p_full, pv_done, o_full, drain, k_rot[NSK]
  static constexpr int N_BAR = 8 + 3 * NSK + 2 * NSV;
  static constexpr int OFF_MISC = OFF_BAR + 8 * N_BAR;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int TMEM_COLS = 256;
  static constexpr int TM_S = 0;
  static constexpr int TM_O = BN;
  static constexpr int TM_P = BN + D;
  static constexpr int NTHREADS = 256;
  // Two CTAs per SM: 128 registers per thread at launch; 128 x 200 + 128 x 56 = 256 x 128.
  static constexpr int REG_SOFTMAX = 200;
  static constexpr int REG_OTHER = 56;
  static_assert(D <= 64, "one-tile kernel: head_dim <= 64");
  static_assert(BN + D + BN / 2 <= TMEM_COLS, "TMEM budget");
  static_assert(128 * REG_SOFTMAX + 128 * REG_OTHER <= NTHREADS * 128, "register split");
  static_assert(2 * (SMEM_BYTES + 1024) <= 233472, "two CTAs per SM");
  static_assert(Q_BYTES % 1024 == 0 && KV_BYTES % 1024 == 0, "1024-byte alignment of swizzled tiles");
};

template <int D, bool BF16>
__global__ void __launch_bounds__(256, 2)
    prefill_fa1_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
  using S = Fa1Shape<D>;
  constexpr int BM = S::BM, BN = S::BN, SPAN = S::SPAN, NSK = S::NSK, NSV = S::NSV;
  constexpr uint32_t SWZ = swizzle_code(SPAN);
  constexpr uint32_t IDESC_QK = idesc_f16(128, BN, 0, 0, 0, 0);  // fp16 R(Q) x fp16 R(K)
  constexpr uint32_t IDESC_PV = idesc_f16(128, D, BF16 ? 1 : 0, BF16 ? 1 : 0, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t sbase = (raw_u32 + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - raw_u32);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int bh = blockIdx.x;                     // b * Hq + h
  const int qt = p.n_qtiles - 1 - blockIdx.y;    // longest first
  const int b = bh / p.Hq;
  const int h = bh - b * p.Hq;
  const int kv_row = b * p.Hkv + h / (p.Hq / p.Hkv);
  const int T = p.T;
  const int q0 = qt * BM;
  const int nk = (min(q0 + BM, T) - 1) / BN + 1;

  auto bar = [&](int i) -> uint32_t { return sbase + S::OFF_BAR + 8u * static_cast<uint32_t>(i); };
  const uint32_t BAR_QF = bar(0);
  const uint32_t BAR_QR = bar(1);
  auto BAR_KF = [&](int s) { return bar(2 + s); };
  auto BAR_KE = [&](int s) { return bar(2 + NSK + s); };
  auto BAR_VF = [&](int s) { return bar(2 + 2 * NSK + s); };
  auto BAR_VE = [&](int s) { return bar(2 + 2 * NSK + NSV + s); };
  constexpr int XB = 2 + 2 * NSK + 2 * NSV;
  const uint32_t BAR_SF = bar(XB);
  const uint32_t BAR_SC = bar(XB + 1);
  const uint32_t BAR_PF = bar(XB + 2);
  const uint32_t BAR_OD = bar(XB + 3);
  const uint32_t BAR_OF = bar(XB + 4);
  const uint32_t BAR_DR = bar(XB + 5);
  auto BAR_KR = [&](int s) { return bar(XB + 6 + s); };  // key tile rotated in place (krot)
  const uint32_t tmem_slot = sbase + S::OFF_MISC;
  volatile int* failed = reinterpret_cast<volatile int*>(sgen + S::OFF_MISC + 4);

#ifdef DU_TRACE
  const long long t_start = clock64();
#endif
#ifdef DU_TRACE_SM0
  const long long t_entry = clock64();
#endif
  if (warp == 5) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  // The TMA thread initialises the barriers and starts the query load before the CTA barrier.
  if (warp == 4 && lane == 0) {
    mbar_init(BAR_QF, 1);
    mbar_init(BAR_QR, 128);
    for (int s = 0; s < NSK; ++s) {
      mbar_init(BAR_KF(s), 1);
      mbar_init(BAR_KE(s), 1);
    }
    for (int s = 0; s < NSV; ++s) {
      mbar_init(BAR_VF(s), 1);
      mbar_init(BAR_VE(s), 1);
    }
    mbar_init(BAR_SF, 1);
    mbar_init(BAR_SC, 128);
    mbar_init(BAR_PF, 128);
    mbar_init(BAR_OD, 1);
    mbar_init(BAR_OF, 1);
    mbar_init(BAR_DR, 1);
    for (int s = 0; s < NSK; ++s) mbar_init(BAR_KR(s), 128);
    *failed = 0;
    mbar_fence_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    mbar_expect_tx(BAR_QF, S::Q_BYTES);
#pragma unroll
    for (int blk = 0; blk < S::NBLK; ++blk)
      tma_load_3d(sbase + S::OFF_Q + blk * BM * SPAN, &tm_q, BAR_QF, blk * (SPAN / 2), q0, bh);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sgen + S::OFF_MISC);

  if (warp < 4) {
    // ------------------------------------------------------------------ softmax
    regs_inc<S::REG_SOFTMAX>();
    const int row = tid;
    const int qrow = q0 + row;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + S::TM_S;
    const uint32_t o_addr = tmem + lane_off + S::TM_O;
    const uint32_t p_addr = tmem + lane_off + S::TM_P;
    const float sl2 = p.scale_log2;
    bool ok = true;
    {
      const uint8_t* cosb = static_cast<const uint8_t*>(p.cos);
      const uint8_t* sinb = static_cast<const uint8_t*>(p.sin);
      constexpr int NPQ = D / 16;
      uint4 cv[NPQ], sv[NPQ];
      if (qrow < T)
        load_rope_row<NPQ>(cv, sv, cosb + static_cast<size_t>(qrow) * D,
                           sinb + static_cast<size_t>(qrow) * D, 0, 1);
      ok = __all_sync(0xffffffffu, mbar_wait(BAR_QF, 0, failed, 400));
      if (ok) {
        if (qrow < T) rotate_row<D, BF16, SPAN, NPQ>(sbase + S::OFF_Q, BM, row, 0, 1, cv, sv);
        fence_proxy_async_smem();
        mbar_arrive(BAR_QR);
      }
      // Short sequences (krot: at most NSK key tiles, each in its own ring stage): the keys
      // arrive raw and thread `row` rotates row `row` of every key tile in place into fp16, as
      // the rotary pass would, before the first product reads it.
      if (p.krot) {
        for (int j = 0; ok && j < nk; ++j) {
          const int krow = j * BN + row;
          if (krow < T)
            load_rope_row<NPQ>(cv, sv, cosb + static_cast<size_t>(krow) * D,
                               sinb + static_cast<size_t>(krow) * D, 0, 1);
          ok = __all_sync(0xffffffffu, mbar_wait(BAR_KF(j), 0, failed, 404));
          if (!ok) break;
          if (krow < T)
            rotate_row<D, BF16, SPAN, NPQ>(sbase + S::OFF_K + j * S::KV_BYTES, BN, row, 0, 1, cv, sv);
          fence_proxy_async_smem();
          mbar_arrive(BAR_KR(j));
        }
      }
    }
    float m = -INFINITY;
    float l = 0.f;
    const uint64_t SL2 = f2(sl2, sl2);
#ifdef DU_TRACE_SM0
    // Debug-only timeline of the CTAs on SM 0 (softmax warp 0): [slot][tile] exp start / end.
    int t0slot = -1;
    if (tid == 0) {
      uint32_t smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      if (smid == 0) {
        t0slot = static_cast<int>(atomicAdd(reinterpret_cast<unsigned long long*>(&g_du_trace[1000]), 1ull));
        if (t0slot < 18) {
          g_du_trace[t0slot * 50 + 0] = clock64();
          g_du_trace[t0slot * 50 + 1] = nk;
          g_du_trace[t0slot * 50 + 48] = t_entry;
        } else {
          t0slot = -1;
        }
      }
    }
#endif
#ifdef DU_TRACE
    long long t_a = clock64();
    long long tr[8] = {t_a - t_start, 0, 0, 0, 0, 0, 0, 0};
#endif
    for (int j = 0; ok && j < nk; ++j) {
#ifdef DU_TRACE
      t_a = clock64();
#endif
      ok = __all_sync(0xffffffffu, mbar_wait(BAR_SF, j & 1, failed, 401));
      if (!ok) break;
#ifdef DU_TRACE
      const long long t_b = clock64();
      tr[1] += t_b - t_a;
#endif
      tc_fence_after();
      // S in two halves: the first half is masked and reduced while the second half loads.
      float s[BN];
      const int k0 = j * BN;
      const bool diag = k0 + BN - 1 > q0;
#pragma unroll
      for (int c = 0; c < BN / 2; c += 16) tmem_ld16(s_addr + c, s + c);
      tmem_wait_ld();
#pragma unroll
      for (int c = BN / 2; c < BN; c += 16) tmem_ld16(s_addr + c, s + c);
      if (diag) {
#pragma unroll
        for (int c = 0; c < BN / 2; ++c)
          if (k0 + c > qrow) s[c] = -INFINITY;
      }
      float mq[4] = {fmaxf(s[0], s[1]), fmaxf(s[2], s[3]), fmaxf(s[4], s[5]), fmaxf(s[6], s[7])};
#pragma unroll
      for (int c = 8; c < BN / 2; c += 8) {
#pragma unroll
        for (int i = 0; i < 4; ++i) mq[i] = max3(mq[i], s[c + 2 * i], s[c + 2 * i + 1]);
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(BAR_SC);  // S is in registers: the next Q K^T may overwrite it
      if (diag) {
#pragma unroll
        for (int c = BN / 2; c < BN; ++c)
          if (k0 + c > qrow) s[c] = -INFINITY;
      }
#pragma unroll
      for (int c = BN / 2; c < BN; c += 8) {
#pragma unroll
        for (int i = 0; i < 4; ++i) mq[i] = max3(mq[i], s[c + 2 * i], s[c + 2 * i + 1]);
      }
      const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * sl2;
#ifdef DU_TRACE
      const long long t_c = clock64();
      tr[2] += t_c - t_b;
#endif
      const float m_new = (mx > m + 8.0f) ? mx : m;
      const uint64_t NM = f2(-m_new, -m_new);
#ifdef DU_TRACE_SM0
      if (t0slot >= 0 && j < 16) g_du_trace[t0slot * 50 + 2 + 3 * j] = clock64();
#endif
      uint64_t acc[4] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float2 xx = f2_split(f2_fma(f2(s[c], s[c + 1]), SL2, NM));
        float2 pp;
        const int q8 = (c / 2) % 8;
        if ((DU_FA1_POLY_MASK >> q8) & 1) {
          pp = ex2_poly2(xx.x, xx.y);
        } else {
          pp = make_float2(ex2(xx.x), ex2(xx.y));
        }
        acc[(c / 2) & 3] = f2_add(acc[(c / 2) & 3], f2(pp.x, pp.y));
        pk[c / 2] = pack2<BF16>(pp.x, pp.y);
      }
      const float2 rsum = f2_split(f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3])));
#ifdef DU_TRACE_SM0
      if (t0slot >= 0 && j < 16) g_du_trace[t0slot * 50 + 3 + 3 * j] = clock64();
#endif
#ifdef DU_TRACE
      const long long t_d = clock64();
      tr[3] += t_d - t_c;
#endif
      if (j > 0) {
        // PV(j-1) must be complete before P is rewritten or O rescaled.
        ok = __all_sync(0xffffffffu, mbar_wait(BAR_OD, (j - 1) & 1, failed, 403));
        if (!ok) break;
        tc_fence_after();
        const bool need = (m_new != m);
        if (__any_sync(0xffffffffu, need)) {
          const float alpha = need ? ex2(m - m_new) : 1.0f;
          l *= alpha;
#pragma unroll
          for (int c = 0; c < D; c += 16) {
            float o[16];
            tmem_ld16(o_addr + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] *= alpha;
            tmem_st16(o_addr + c, o);
          }
        }
      }
      l += rsum.x + rsum.y;
      m = m_new;
#ifdef DU_TRACE
      const long long t_e = clock64();
      tr[4] += t_e - t_d;
#endif
#pragma unroll
      for (int c = 0; c < BN / 2; c += 16) tmem_st16u(p_addr + c, pk + c);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(BAR_PF);
#ifdef DU_TRACE_SM0
      if (t0slot >= 0 && j < 16) g_du_trace[t0slot * 50 + 4 + 3 * j] = clock64();
#endif
#ifdef DU_TRACE
      tr[5] += clock64() - t_e;
      tr[6] += 1;
#endif
    }
#ifdef DU_TRACE
    const long long t_g = clock64();
#endif
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(BAR_OF, 0, failed, 402));
    tc_fence_after();
    if (ok) {
      const float inv_l = 1.0f / l;
      const size_t orow = (static_cast<size_t>(bh) * T + qrow) * D;
#pragma unroll
      for (int c = 0; c < D; c += 16) {
        float o[16];
        tmem_ld16(o_addr + c, o);
        tmem_wait_ld();
        if (qrow < T) {
          uint32_t w[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) w[i] = pack2<BF16>(o[2 * i] * inv_l, o[2 * i + 1] * inv_l);
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.out) + (orow + c) * 2);
          dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
      if (qrow < T) p.lse[static_cast<size_t>(bh) * T + qrow] = (m + lg2(l)) * 0.69314718055994531f;
    }
#ifdef DU_TRACE_SM0
    if (t0slot >= 0) g_du_trace[t0slot * 50 + 49] = clock64();
#endif
#ifdef DU_TRACE
    if (lane == 0) {
      const long long t_h = clock64();
      tr[7] = t_h - t_g;
#pragma unroll
      for (int k = 0; k < 8; ++k) DU_STAT(k, tr[k]);
      DU_STAT(9, t_h - t_start);
      DU_STAT(10, 1);
    }
#endif
  } else if (warp == 4) {
    // ------------------------------------------------------------------ TMA: the K ring
    regs_dec<S::REG_OTHER>();
    if (lane == 0) {
      int issued = 0;
      // The rotated keys come from the preceding rotary launch (this kernel may start before
      // it completes); nothing else this CTA reads is written by it. With krot there is no such
      // launch and the wait returns at once.
      griddep_wait();
      for (int j = 0; j < nk; ++j) {
        const int s = j % NSK;
        if (j >= NSK && !mbar_wait(BAR_KE(s), (j / NSK - 1) & 1, failed, 410)) break;
        mbar_expect_tx(BAR_KF(s), S::KV_BYTES);
#pragma unroll
        for (int blk = 0; blk < S::NBLK; ++blk)
          tma_load_3d(sbase + S::OFF_K + s * S::KV_BYTES + blk * BN * SPAN, &tm_k, BAR_KF(s),
                      blk * (SPAN / 2), j * BN, kv_row);
        issued = j + 1;
      }
      mbar_wait_drain(BAR_QF, 0, 412);
      for (int j = (issued > NSK ? issued - NSK : 0); j < issued; ++j)
        mbar_wait_drain(BAR_KF(j % NSK), (j / NSK) & 1, 413);
    }
    __syncwarp();
  } else if (warp == 6) {
    // ------------------------------------------------------------------ TMA: the V ring
    regs_dec<S::REG_OTHER>();
    if (lane == 0) {
      tma_prefetch_desc(&tm_v);
      int issued = 0;
      for (int j = 0; j < nk; ++j) {
        const int s = j % NSV;
        if (j >= NSV && !mbar_wait(BAR_VE(s), (j / NSV - 1) & 1, failed, 411)) break;
        mbar_expect_tx(BAR_VF(s), S::KV_BYTES);
#pragma unroll
        for (int blk = 0; blk < S::NBLK; ++blk)
          tma_load_3d(sbase + S::OFF_V + s * S::KV_BYTES + blk * BN * SPAN, &tm_v, BAR_VF(s),
                      blk * (SPAN / 2), j * BN, kv_row);
        issued = j + 1;
      }
      for (int j = (issued > NSV ? issued - NSV : 0); j < issued; ++j)
        mbar_wait_drain(BAR_VF(j % NSV), (j / NSV) & 1, 414);
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    regs_dec<S::REG_OTHER>();
    const uint64_t dq = smem_desc(sbase + S::OFF_Q, 16, 8 * SPAN, SWZ);
    const uint64_t dk0 = smem_desc(sbase + S::OFF_K, 16, 8 * SPAN, SWZ);
    const uint64_t dv0 = smem_desc(sbase + S::OFF_V, BN * SPAN, 8 * SPAN, SWZ);
    const bool leader = elect_one();
#ifdef DU_TRACE
    long long mt[4] = {0, 0, 0, 0};
#endif
    bool ok = __all_sync(0xffffffffu, mbar_wait(BAR_QR, 0, failed, 420));
    // Step j: QK(j) (after the softmax has loaded S(j-1)), then PV(j-1) (once P(j-1) is in).
    for (int j = 0; ok && j <= nk; ++j) {
      if (j < nk) {
        const int sk = j % NSK;
#ifdef DU_TRACE
        const long long m0 = clock64();
#endif
        ok = __all_sync(0xffffffffu, mbar_wait(BAR_KF(sk), (j / NSK) & 1, failed, 421));
        if (ok && p.krot) ok = __all_sync(0xffffffffu, mbar_wait(BAR_KR(sk), 0, failed, 426));
#ifdef DU_TRACE
        const long long m1 = clock64();
#endif
        if (ok && j > 0) ok = __all_sync(0xffffffffu, mbar_wait(BAR_SC, (j - 1) & 1, failed, 424));
#ifdef DU_TRACE
        mt[0] += m1 - m0;
        mt[1] += clock64() - m1;
#endif
        if (!ok) break;
        tc_fence_after();
        if (leader) {
          const uint64_t dk = dk0 + static_cast<uint64_t>((sk * S::KV_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off_q = ((kk * 32) / SPAN) * BM * SPAN + (kk * 32) % SPAN;
            const uint32_t off_k = ((kk * 32) / SPAN) * BN * SPAN + (kk * 32) % SPAN;
            umma_f16_ss(tmem + S::TM_S, dq + (off_q >> 4), dk + (off_k >> 4), IDESC_QK,
                        kk > 0 ? 1u : 0u);
          }
          umma_commit(BAR_SF);
          umma_commit(BAR_KE(sk));
        }
        __syncwarp();
      }
      if (j > 0) {
        const int jv = j - 1;
        const int sv = jv % NSV;
#ifdef DU_TRACE
        const long long m2 = clock64();
#endif
        ok = __all_sync(0xffffffffu, mbar_wait(BAR_PF, jv & 1, failed, 422));
#ifdef DU_TRACE
        const long long m3 = clock64();
#endif
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(BAR_VF(sv), (jv / NSV) & 1, failed, 423));
#ifdef DU_TRACE
        mt[2] += m3 - m2;
        mt[3] += clock64() - m3;
#endif
        if (!ok) break;
        tc_fence_after();
        if (leader) {
          const uint64_t dv = dv0 + static_cast<uint64_t>((sv * S::KV_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk)
            umma_f16_ts(tmem + S::TM_O, tmem + S::TM_P + kk * 8,
                        dv + static_cast<uint64_t>((kk * 16 * SPAN) >> 4), IDESC_PV,
                        (jv > 0 || kk > 0) ? 1u : 0u);
          umma_commit(BAR_OD);
          umma_commit(BAR_VE(sv));
          if (jv == nk - 1) umma_commit(BAR_OF);
        }
        __syncwarp();
      }
    }
    if (leader) {
      umma_commit(BAR_DR);
      mbar_wait_drain(BAR_DR, 0, 425);
    }
#ifdef DU_TRACE
    if (lane == 0)
      for (int k = 0; k < 4; ++k) DU_STAT(11 + k, mt[k]);
#endif
    __syncwarp();
  } else {
    regs_dec<S::REG_OTHER>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

}  // namespace du
