// Fused-RoPE causal prefill for sm_100a, two query tiles per CTA (head_dim 16..128).
//
// Same mathematics as prefill_kernel (prefill_sm100.cuh; reference prefill_kernel,
// dominus_ultra.py:119-285): out = softmax(R(Q) R(K)^T / sqrt(D), causal) V and the natural-log
// LSE per row, half-split rotary rotation at each row's position, query head h reading KV head
// h / (Hq / Hkv) (dominus_ultra.py:168).
//
// Layout of the work, chosen from measurements of tcgen05 on B200: a single issuing thread
// completes one tcgen05.mma (M=128, K=16) about every 87 cycles whatever N <= 128 is, while two
// issuing threads keep the tensor pipe near its peak. So a CTA owns two consecutive 128-row
// query tiles A and B of one (b, h) -- rows [256p, 256p+128) and [256p+128, 256p+256) -- that
// share every K/V tile (loaded and rotated once), with three MMA-issuing threads and two
// softmax warpgroups ping-ponging on the tensor core.
//
// Warp roles, 512 threads (register budgets set per warpgroup with setmaxnreg: 176 for the two
// softmax warpgroups, 80 for the other two; 2*176 + 2*80 = 512 = the 128 per thread of launch):
//   warps 0-3   softmax A: thread t owns row t of tile A = TMEM lane t. Rotates its Q row at
//               the start; per KV tile loads S_A from TMEM, hands the S buffer back at once
//               (the next S_A = Q_A K^T overlaps the exponentials), masks the diagonal tile,
//               online softmax in the log2 domain (packed f32x2 arithmetic; 3 in 8 of the
//               exponentials evaluated on the FMA pipe by a cubic, the rest on MUFU), P_A stored to TMEM as 16-bit pairs (the PV MMA reads A from TMEM),
//               O_A rescaled in TMEM only when the running max grows by more than 2^8;
//               finally out = O/l and lse = (m + log2 l) ln 2.
//   warps 4-7   softmax B: the same for tile B.
//   warps 8-11  K rotation: each K tile is rotated in fp32 from shared memory (its cos/sin rows
//               staged by TMA next to it) and written back in place as fp16.
//   warp 12     TMA producer: Q_A and Q_B once; per KV tile K, its cos/sin table rows, and V
//               into NS-deep rings (no multicast).
//   warp 13     TMEM allocator; single-thread issuer of S_A = Q_A K_j^T and S_B = Q_B K_j^T
//               (fp16 x fp16 -> fp32 TMEM).
//   warps 14-15 single-thread issuers of O_A += P_A V_j and O_B += P_B V_j (input dtype, P
//               from TMEM, V MN-major from shared memory). One tcgen05.mma issuing thread
//               sustains only about one instruction per 87 cycles, so the MMAs of a KV tile
//               are spread over three issuers.
// Q/K operands are fp16 (rotated in fp32): bf16 operands would put the LSE error above 1e-3.
// TMEM columns: S_A [0, BN), S_B [BN, 2BN), O_A [2BN, 2BN + D), O_B [2BN + D, 2BN + 2D),
// P_A and P_B BN/2 columns each after them.
// Every mbarrier wait is bounded (du_ptx.cuh).
#pragma once

#include "du_ptx.cuh"
#include "prefill_sm100.cuh"

// Which of every 8 score pairs take the FMA-pipe exponential (bit i: pair i of 8).
#ifndef DU_POLY_MASK
#define DU_POLY_MASK 0x49
#endif

namespace du {

template <int D>
struct PairShape {
  static constexpr int BM = 128;                             // rows per query tile
  static constexpr int BN = (D >= 128) ? 64 : 128;            // keys per KV tile
  static constexpr int SPAN = (2 * D >= 128) ? 128 : 2 * D;   // bytes per swizzled row block
  static constexpr int NBLK = 2 * D / SPAN;                  // column blocks of a Q/K/V tile
  static constexpr int NS = 3;                               // K/V/cos/sin ring depth
  static constexpr int Q_BYTES = BM * D * 2;                 // one query tile
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int CS_BYTES = BN * D;                    // one table's rows for a KV tile
  static constexpr int OFF_QA = 0;
  static constexpr int OFF_QB = OFF_QA + Q_BYTES;
  static constexpr int OFF_K = OFF_QB + Q_BYTES;
  static constexpr int OFF_V = OFF_K + NS * KV_BYTES;
  static constexpr int OFF_CS = OFF_V + NS * KV_BYTES;        // stage s: cos at +2s*CS, sin after
  static constexpr int OFF_BAR = OFF_CS + NS * 2 * CS_BYTES;
  // barriers: q_full, q_rot[2], k_full[NS], k_rot[NS], k_empty[2][NS], v_full[NS],
  //           v_empty[2][NS], s_full[2], s_free[2], p_full[2], o_done[2], drain[3]
  static constexpr int N_BAR = 3 + 7 * NS + 11;
  static constexpr int OFF_MISC = OFF_BAR + 8 * N_BAR;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int TM_S = 0;                  // + x * BN    fp32 scores
  static constexpr int TM_O = 2 * BN;             // + x * D     fp32 output accumulator
  static constexpr int TM_P = 2 * BN + 2 * D;     // + x * BN/2  16-bit P, two per column
  static constexpr int NTHREADS = 512;
  static constexpr int REG_SOFTMAX = 176;  // setmaxnreg budgets; 2*176 + 2*80 = 4 * 128
  static constexpr int REG_OTHER = 80;
  static_assert(3 * BN + 2 * D <= TMEM_COLS, "TMEM budget");
  static_assert(2 * REG_SOFTMAX + 2 * REG_OTHER == 4 * (65536 / NTHREADS), "register split");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(Q_BYTES % 1024 == 0 && KV_BYTES % 1024 == 0 && CS_BYTES % 1024 == 0,
                "1024-byte alignment of swizzled tiles");
};

template <int D, bool BF16>
__global__ void __launch_bounds__(512, 1)
    prefill_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_cos,
                        const __grid_constant__ CUtensorMap tm_sin, const PrefillParams p) {
  using S = PairShape<D>;
  constexpr int BM = S::BM, BN = S::BN, SPAN = S::SPAN, NS = S::NS;
  constexpr uint32_t SWZ = swizzle_code(SPAN);
  constexpr uint32_t IDESC_QK = idesc_f16(128, BN, 0, 0, 0, 0);
  constexpr uint32_t IDESC_PV = idesc_f16(128, D, BF16 ? 1 : 0, BF16 ? 1 : 0, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t sbase = (raw_u32 + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - raw_u32);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int bh = blockIdx.x;                       // b * Hq + h
  const int pair = p.n_qtiles - 1 - blockIdx.y;    // longest first (p.n_qtiles = pair count)
  const int b = bh / p.Hq;
  const int h = bh - b * p.Hq;
  const int kvh = h / (p.Hq / p.Hkv);
  const int kv_row = b * p.Hkv + kvh;
  const int T = p.T;
  // Scalars, not arrays: a runtime-indexed local array would live in local memory.
  const int q0a = pair * 2 * BM, q0b = q0a + BM;
  const int nkva = (q0a < T) ? (min(q0a + BM, T) - 1) / BN + 1 : 0;
  const int nkvb = (q0b < T) ? (min(q0b + BM, T) - 1) / BN + 1 : 0;
  auto q0 = [&](int x) { return x ? q0b : q0a; };
  auto n_kv = [&](int x) { return x ? nkvb : nkva; };
  const int n_kv_all = max(nkva, nkvb);

  auto bar = [&](int i) -> uint32_t { return sbase + S::OFF_BAR + 8u * static_cast<uint32_t>(i); };
  const uint32_t BAR_QF = bar(0);
  auto BAR_QR = [&](int x) { return bar(1 + x); };
  auto BAR_KF = [&](int s) { return bar(3 + s); };
  auto BAR_KR = [&](int s) { return bar(3 + NS + s); };
  auto BAR_KE = [&](int x, int s) { return bar(3 + 2 * NS + x * NS + s); };
  auto BAR_VF = [&](int s) { return bar(3 + 4 * NS + s); };
  auto BAR_VE = [&](int x, int s) { return bar(3 + 5 * NS + x * NS + s); };
  auto BAR_SF = [&](int x) { return bar(3 + 7 * NS + x); };
  auto BAR_SR = [&](int x) { return bar(3 + 7 * NS + 2 + x); };  // S buffer released
  auto BAR_PF = [&](int x) { return bar(3 + 7 * NS + 4 + x); };
  auto BAR_OD = [&](int x) { return bar(3 + 7 * NS + 6 + x); };
  auto BAR_DR = [&](int x) { return bar(3 + 7 * NS + 8 + x); };
  const uint32_t tmem_slot = sbase + S::OFF_MISC;
  volatile int* failed = reinterpret_cast<volatile int*>(sgen + S::OFF_MISC + 4);

  if (warp == 13) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(BAR_QF, 1);
    for (int x = 0; x < 2; ++x) {
      mbar_init(BAR_QR(x), 128);
      mbar_init(BAR_SF(x), 1);
      mbar_init(BAR_SR(x), 128);
      mbar_init(BAR_PF(x), 128);
      mbar_init(BAR_OD(x), 1);
    }
    for (int i = 0; i < 3; ++i) mbar_init(BAR_DR(i), 1);  // one per MMA-issuing thread
    for (int s = 0; s < NS; ++s) {
      mbar_init(BAR_KF(s), 1);
      mbar_init(BAR_KR(s), 128);
      mbar_init(BAR_VF(s), 1);
      for (int x = 0; x < 2; ++x) {
        mbar_init(BAR_KE(x, s), 1);
        mbar_init(BAR_VE(x, s), 1);
      }
    }
    *failed = 0;
    mbar_fence_init();
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sgen + S::OFF_MISC);

  if (warp < 8) {
    // ------------------------------------------------------------------ softmax A / B
    regs_inc<S::REG_SOFTMAX>();
    const int x = warp >> 2;           // which query tile
    const int row = tid - 128 * x;     // row within the tile = TMEM lane
    const int qrow = q0(x) + row;
    const int nk = n_kv(x);
    const uint32_t q_tile = sbase + (x ? S::OFF_QB : S::OFF_QA);
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + S::TM_S + x * BN;
    const uint32_t o_addr = tmem + lane_off + S::TM_O + x * D;
    const uint32_t p_addr = tmem + lane_off + S::TM_P + x * (BN / 2);
    const float sl2 = p.scale_log2;
    bool ok = nk > 0;
    if (ok) {
      // Rotate this thread's Q row in place (cos/sin loads are issued before the TMA wait).
      const uint8_t* cosb = static_cast<const uint8_t*>(p.cos);
      const uint8_t* sinb = static_cast<const uint8_t*>(p.sin);
      constexpr int NPQ = (D / 16) < 8 ? (D / 16) : 8;
#pragma unroll 1
      for (int c0 = 0; c0 < D / 16; c0 += NPQ) {
        uint4 cv[NPQ], sv[NPQ];
        if (qrow < T)
          load_rope_row<NPQ>(cv, sv, cosb + static_cast<size_t>(qrow) * D,
                             sinb + static_cast<size_t>(qrow) * D, c0, 1);
        if (c0 == 0) {
          ok = mbar_wait(BAR_QF, 0, failed, 100);
          ok = __all_sync(0xffffffffu, ok);
        }
        if (!ok) break;
        if (qrow < T) rotate_row<D, BF16, SPAN, NPQ>(q_tile, BM, row, c0, 1, cv, sv);
      }
      if (ok) {
        fence_proxy_async_smem();
        mbar_arrive(BAR_QR(x));
      }
    }
    float m = -INFINITY;  // running max of scaled scores, log2 domain
    float l = 0.f;
    const uint64_t SL2 = f2(sl2, sl2);
    for (int j = 0; ok && j < nk; ++j) {
      ok = mbar_wait(BAR_SF(x), j & 1, failed, 101);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      if (row == 0) DU_TRACE_EV(4 * x + 0, j);
      tc_fence_after();
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN; c += 16) tmem_ld16(s_addr + c, s + c);
      tmem_wait_ld();
      if (row == 0) DU_TRACE_EV(4 * x + 1, j);
      tc_fence_before();
      mbar_arrive(BAR_SR(x));  // S is in registers: the next Q K^T may overwrite it
      const int k0 = j * BN;
      const bool diag = k0 + BN - 1 > q0(x);  // tile crosses this query tile's diagonal
      if (diag) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (k0 + c > qrow) s[c] = -INFINITY;
      }
      float mq[4] = {fmaxf(s[0], s[1]), fmaxf(s[2], s[3]), fmaxf(s[4], s[5]), fmaxf(s[6], s[7])};
#pragma unroll
      for (int c = 8; c < BN; c += 8) {
#pragma unroll
        for (int i = 0; i < 4; ++i) mq[i] = max3(mq[i], s[c + 2 * i], s[c + 2 * i + 1]);
      }
      float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * sl2;
      if (row == 0) DU_TRACE_EV(4 * x + 2, j);
      const float m_new = (mx > m + 8.0f) ? mx : m;
      const uint64_t NM = f2(-m_new, -m_new);
      uint64_t acc[4] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
      uint32_t pk[BN / 2];
      // 3 in 8 of the exponentials on the FMA pipe (masked scores give 2^-125, not 0: a
      // relative contribution below 1e-37), the rest on MUFU.
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float2 xx = f2_split(f2_fma(f2(s[c], s[c + 1]), SL2, NM));
        float2 pp;
        const int q8 = (c / 2) % 8;
        if ((DU_POLY_MASK >> q8) & 1) {
          pp = ex2_poly2(xx.x, xx.y);
        } else {
          pp = make_float2(ex2(xx.x), ex2(xx.y));
        }
        acc[(c / 2) & 3] = f2_add(acc[(c / 2) & 3], f2(pp.x, pp.y));
        pk[c / 2] = pack2<BF16>(pp.x, pp.y);
      }
      const float2 rsum = f2_split(f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3])));
      const float rs = rsum.x + rsum.y;
      if (row == 0) DU_TRACE_EV(4 * x + 3, j);
      if (j > 0) {
        ok = mbar_wait(BAR_OD(x), (j - 1) & 1, failed, 102);  // PV(j-1) done: P free, O current
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
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
      l += rs;
      m = m_new;
#pragma unroll
      for (int c = 0; c < BN / 2; c += 16) tmem_st16u(p_addr + c, pk + c);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(BAR_PF(x));
      if (row == 0) DU_TRACE_EV(14 + x, j);
    }
    if (ok) {
      ok = mbar_wait(BAR_OD(x), (nk - 1) & 1, failed, 103);
      ok = __all_sync(0xffffffffu, ok);
    }
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
  } else if (warp == 12) {
    // ------------------------------------------------------------------ TMA producer
    regs_dec<S::REG_OTHER>();
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_cos);
      tma_prefetch_desc(&tm_sin);
      const int n_q = nkvb > 0 ? 2 : 1;  // tile B is skipped when it lies past T
      mbar_expect_tx(BAR_QF, n_q * S::Q_BYTES);
      for (int x = 0; x < n_q; ++x)
#pragma unroll
        for (int blk = 0; blk < S::NBLK; ++blk)
          tma_load_3d(sbase + (x ? S::OFF_QB : S::OFF_QA) + blk * BM * SPAN, &tm_q, BAR_QF,
                      blk * (SPAN / 2), q0(x), bh);
      int issued_k = 0, issued_v = 0;
      bool ok = true;
      for (int j = 0; ok && j < n_kv_all; ++j) {
        const int s = j % NS;
        const int jp = j - NS;  // previous use of this stage
        if (jp >= 0) {
          for (int x = 0; x < 2 && ok; ++x)
            if (jp < n_kv(x)) ok = mbar_wait(BAR_KE(x, s), (jp / NS) & 1, failed, 110);
          if (!ok) break;
        }
        mbar_expect_tx(BAR_KF(s), S::KV_BYTES + 2 * S::CS_BYTES);
#pragma unroll
        for (int blk = 0; blk < S::NBLK; ++blk)
          tma_load_3d(sbase + S::OFF_K + s * S::KV_BYTES + blk * BN * SPAN, &tm_k, BAR_KF(s),
                      blk * (SPAN / 2), j * BN, kv_row);
        tma_load_2d(sbase + S::OFF_CS + s * 2 * S::CS_BYTES, &tm_cos, BAR_KF(s), 0, j * BN);
        tma_load_2d(sbase + S::OFF_CS + s * 2 * S::CS_BYTES + S::CS_BYTES, &tm_sin, BAR_KF(s), 0,
                    j * BN);
        issued_k = j + 1;
        if (jp >= 0) {
          for (int x = 0; x < 2 && ok; ++x)
            if (jp < n_kv(x)) ok = mbar_wait(BAR_VE(x, s), (jp / NS) & 1, failed, 111);
          if (!ok) break;
        }
        mbar_expect_tx(BAR_VF(s), S::KV_BYTES);
#pragma unroll
        for (int blk = 0; blk < S::NBLK; ++blk)
          tma_load_3d(sbase + S::OFF_V + s * S::KV_BYTES + blk * BN * SPAN, &tm_v, BAR_VF(s),
                      blk * (SPAN / 2), j * BN, kv_row);
        issued_v = j + 1;
      }
      // Drain: every TMA write into this CTA's shared memory lands before the CTA exits.
      mbar_wait_drain(BAR_QF, 0, 112);
      for (int j = (issued_k > NS ? issued_k - NS : 0); j < issued_k; ++j)
        mbar_wait_drain(BAR_KF(j % NS), (j / NS) & 1, 113);
      for (int j = (issued_v > NS ? issued_v - NS : 0); j < issued_v; ++j)
        mbar_wait_drain(BAR_VF(j % NS), (j / NS) & 1, 114);
    }
    __syncwarp();
  } else if (warp == 13) {
    // ------------------------------------------------------------------ QK^T issuer (A and B)
    regs_dec<S::REG_OTHER>();
    if (lane == 0) {
      bool ok = true;
      for (int x = 0; x < 2 && ok; ++x)
        if (n_kv(x) > 0) ok = mbar_wait(BAR_QR(x), 0, failed, 121);
      tc_fence_after();
      for (int j = 0; ok && j < n_kv_all; ++j) {
        const int s = j % NS;
        if (!mbar_wait(BAR_KR(s), (j / NS) & 1, failed, 120)) break;
        for (int x = 0; x < 2; ++x) {
          if (j >= n_kv(x)) continue;
          // S_x(j-1) must be in the softmax's registers before S_x(j) overwrites it.
          if (j > 0 && !mbar_wait(BAR_SR(x), (j - 1) & 1, failed, 122)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t q_tile = sbase + (x ? S::OFF_QB : S::OFF_QA);
          const uint32_t s_tmem = tmem + S::TM_S + x * BN;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int blk = (kk * 32) / SPAN;
            const int inrow = (kk * 32) % SPAN;
            const uint64_t a = smem_desc(q_tile + blk * BM * SPAN + inrow, 16, 8 * SPAN, SWZ);
            const uint64_t bd = smem_desc(sbase + S::OFF_K + s * S::KV_BYTES + blk * BN * SPAN + inrow,
                                          16, 8 * SPAN, SWZ);
            umma_f16_ss(s_tmem, a, bd, IDESC_QK, kk > 0 ? 1u : 0u);
          }
          umma_commit(BAR_SF(x));
          umma_commit(BAR_KE(x, s));
          DU_TRACE_EV(8 + 2 * x, j);
        }
      }
      // Drain: all MMAs issued by this thread complete before TMEM is released.
      umma_commit(BAR_DR(0));
      mbar_wait_drain(BAR_DR(0), 0, 125);
    }
    __syncwarp();
  } else if (warp == 14 || warp == 15) {
    // ------------------------------------------------------------------ PV issuers A / B
    regs_dec<S::REG_OTHER>();
    const int x = warp - 14;
    const int nk = n_kv(x);
    if (lane == 0) {
      const uint32_t p_tmem = tmem + S::TM_P + x * (BN / 2);
      const uint32_t o_tmem = tmem + S::TM_O + x * D;
      for (int j = 0; j < nk; ++j) {
        const int s = j % NS;
        if (!mbar_wait(BAR_PF(x), j & 1, failed, 123)) break;
        if (!mbar_wait(BAR_VF(s), (j / NS) & 1, failed, 124)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // A = P from TMEM: 16 keys per step = 8 columns of packed 16-bit pairs.
          const uint64_t bd = smem_desc(sbase + S::OFF_V + s * S::KV_BYTES + kk * 16 * SPAN,
                                        BN * SPAN, 8 * SPAN, SWZ);
          umma_f16_ts(o_tmem, p_tmem + kk * 8, bd, IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(BAR_VE(x, s));
        umma_commit(BAR_OD(x));
        DU_TRACE_EV(9 + 2 * x, j);
      }
      umma_commit(BAR_DR(1 + x));
      mbar_wait_drain(BAR_DR(1 + x), 0, 126);
    }
    __syncwarp();
  } else if (warp < 12) {
    // ------------------------------------------------------------------ K rotation (warps 8-11)
    regs_dec<S::REG_OTHER>();
    constexpr int TPR = 128 / BN;          // threads per K row
    constexpr int NP = (D / 16) / TPR;     // chunk pairs per thread
    const int rt = tid - 256;
    const int r = rt / TPR;
    const int c0 = (rt % TPR) * NP;
    for (int j = 0; j < n_kv_all; ++j) {
      const int s = j % NS;
      if (!mbar_wait(BAR_KF(s), (j / NS) & 1, failed, 130)) break;
      if (rt == 0) DU_TRACE_EV(12, j);
      if (j * BN + r < T) {
        const uint32_t ktile = sbase + S::OFF_K + s * S::KV_BYTES;
        const uint32_t cs_cos = sbase + S::OFF_CS + s * 2 * S::CS_BYTES + r * D;
        const uint32_t cs_sin = cs_cos + S::CS_BYTES;
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          const int c = c0 + i;
          const uint32_t a1 = ktile + swz_chunk_offset<SPAN>(BN, r, c);
          const uint32_t a2 = ktile + swz_chunk_offset<SPAN>(BN, r, c + D / 16);
          const uint4 x1 = ld_shared_v4(a1);
          const uint4 x2 = ld_shared_v4(a2);
          const uint4 cv = ld_shared_v4(cs_cos + c * 16);
          const uint4 sv = ld_shared_v4(cs_sin + c * 16);
          const uint32_t xa[4] = {x1.x, x1.y, x1.z, x1.w};
          const uint32_t xb[4] = {x2.x, x2.y, x2.z, x2.w};
          const uint32_t ca[4] = {cv.x, cv.y, cv.z, cv.w};
          const uint32_t sa[4] = {sv.x, sv.y, sv.z, sv.w};
          uint32_t ya[4], yb[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 lo = unpack2<BF16>(xa[e]);
            const float2 hi = unpack2<BF16>(xb[e]);
            const float2 cc = unpack2<BF16>(ca[e]);
            const float2 ss = unpack2<BF16>(sa[e]);
            ya[e] = pack2<false>(lo.x * cc.x - hi.x * ss.x, lo.y * cc.y - hi.y * ss.y);
            yb[e] = pack2<false>(hi.x * cc.x + lo.x * ss.x, hi.y * cc.y + lo.y * ss.y);
          }
          st_shared_v4(a1, make_uint4(ya[0], ya[1], ya[2], ya[3]));
          st_shared_v4(a2, make_uint4(yb[0], yb[1], yb[2], yb[3]));
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(BAR_KR(s));
      if (rt == 0) DU_TRACE_EV(13, j);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

}  // namespace du
