// Causal prefill for sm_100a on pre-rotated keys: two 128-row query tiles per CTA, one
// tcgen05.mma-issuing thread, P written over S in tensor memory (head_dim 16..128).
//
// Mathematics of the reference prefill_kernel (dominus_ultra.py:119-285): out =
// softmax(R(Q) R(K)^T * scale, causal) V and the natural-log LSE per row, query head h reading KV
// head h / (Hq / Hkv) (dominus_ultra.py:168). R(K) arrives already rotated, as fp16, from the
// standalone rotary kernel (rope_sm100.cuh) run once per (b, kv head) before this kernel; Q is
// rotated here, in fp32, by the softmax thread that owns each row.
//
// Why this shape (all measured on B200): a lone thread issuing unrolled tcgen05.mma bursts keeps
// the tensor pipe at full rate, while every hand-off between warps costs hundreds of cycles on an
// SM whose softmax warps keep the issue slots busy. So the pipeline has as few hand-offs as the
// dependencies allow:
//   * one MMA thread issues, per KV tile j and query tile x, O_x += P_x(j-1) V(j-1) and then
//     S_x = Q_x K(j)^T. Because a thread's MMAs complete in issue order, the completion of
//     S_x(j) (the only signal the softmax waits for) also means O_x holds every earlier PV:
//     the softmax may rescale O_x in place without a separate wait, and P_x(j) may be written
//     into the tensor-memory columns of S_x(j), which the next QK^T of tile x only overwrites
//     after PV_x(j) has read them. TMEM: S/P_A [0, BN), S/P_B [BN, 2BN), O_A, O_B [2BN, 2BN+2D):
//     512 columns at D = 128 with BN = 128.
//   * the two softmax warpgroups (tiles A and B) each own 128 rows, one row per thread = TMEM
//     lane, and alternate with the tensor core: while one computes exponentials the MMA thread
//     serves the other tile.
//   * K and V stream through separate TMA rings, each refilled by its own thread as soon as the
//     MMAs that read a stage have completed.
//
// Warp roles (384 threads; setmaxnreg: 224 registers for the softmax warpgroups, 56 for the rest):
//   warps 0-3   softmax A: rotate the Q row, then per KV tile: wait S_A, load it, mask the
//               diagonal tile, online softmax in the log2 domain (lazy rescale by 2^8), P_A to
//               TMEM, signal. Finally out = O/l, lse = (m + log2 l) ln 2.
//   warps 4-7   softmax B: the same for tile B.
//   warp 8      TMA: Q_A and Q_B, then the K ring.      warp 9   TMEM owner and MMA issuer.
//   warp 10     TMA: the V ring.                          warp 11  idle.
// Every mbarrier wait is bounded (du_ptx.cuh).
#pragma once

#include "du_ptx.cuh"
#include "prefill_sm100.cuh"

// Which of every 8 score pairs take the FMA-pipe exponential (bit i: pair i of 8).
#ifndef DU_FA_POLY_MASK
#define DU_FA_POLY_MASK 0x49
#endif

namespace du {

template <int D>
struct FaShape {
  static constexpr int BM = 128;                             // rows per query tile
  static constexpr int BN = 128;                             // keys per KV tile
  static constexpr int SPAN = (2 * D >= 128) ? 128 : 2 * D;   // bytes per swizzled row block
  static constexpr int NBLK = 2 * D / SPAN;                  // column blocks of a Q/K/V tile
  static constexpr int NSK = (D >= 128) ? 2 : 4;             // K ring depth
  static constexpr int NSV = (D >= 128) ? 2 : 3;             // V ring depth
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int OFF_QA = 0;
  static constexpr int OFF_QB = OFF_QA + Q_BYTES;
  static constexpr int OFF_K = OFF_QB + Q_BYTES;
  static constexpr int OFF_V = OFF_K + NSK * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + NSV * KV_BYTES;
  // P gets its own TMEM columns when they fit (head_dim <= 64): the next Q K^T of a tile can
  // then be issued as soon as the softmax has loaded S, before P is ready.
  static constexpr bool SEP_P = 2 * BN + 2 * D + BN <= 512;
  // barriers: q_full, q_rot[2], k_full[NSK], k_empty[NSK], v_full[NSV], v_empty[NSV],
  //           s_full[2], p_full[2], o_full[2], drain, s_consumed[2], pv_done[2], stagger
  static constexpr int N_BAR = 15 + 2 * NSK + 2 * NSV;
  static constexpr int OFF_MISC = OFF_BAR + 8 * N_BAR;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int TM_S = 0;        // + x * BN: fp32 scores, then 16-bit P over the first BN/2
  static constexpr int TM_O = 2 * BN;   // + x * D: fp32 output accumulator
  static constexpr int TM_P = SEP_P ? 2 * BN + 2 * D : 0;  // + x * BN/2: 16-bit P (SEP_P)
  static constexpr int NTHREADS = 384;
  static constexpr int REG_SOFTMAX = 224;
  static constexpr int REG_OTHER = 56;
  static_assert(2 * BN + 2 * D <= TMEM_COLS, "TMEM budget");
  // The split must fit the registers of the launch (384 threads x 168, the launch-bounds cap).
  static_assert(2 * 128 * REG_SOFTMAX + 128 * REG_OTHER <= NTHREADS * 168, "register split");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(Q_BYTES % 1024 == 0 && KV_BYTES % 1024 == 0, "1024-byte alignment of swizzled tiles");
};

// BLOCK: the block form of PrefillParams (query-row window, key range, causal or full, two-segment
// positions, accumulate epilogue) for context-parallel prefill; the whole-sequence causal path
// is the BLOCK = false instantiation, compiled without those generalisations.
template <int D, bool BF16, bool BLOCK>
__global__ void __launch_bounds__(384, 1)
    prefill_fa_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
  using S = FaShape<D>;
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
  // CTA order (1-D grid): KV group (b, kv head) outermost, then query-tile pairs heaviest
  // first, then the G query heads of the group. The G CTAs that read the same K/V tiles run
  // side by side, and a group's pairs (which read overlapping key prefixes) follow each other,
  // so its K/V stays in L2 while it is in flight and is read from DRAM about once.
  const int G = p.Hq / p.Hkv;
  const int per_group = p.n_qtiles * G;          // p.n_qtiles = pair count
  const int kv_row = static_cast<int>(blockIdx.x) / per_group;   // b * Hkv + kv head
  const int rem = static_cast<int>(blockIdx.x) - kv_row * per_group;
  const int pair = p.n_qtiles - 1 - rem / G;     // longest first within the group
  const int b = kv_row / p.Hkv;
  const int kvh = kv_row - b * p.Hkv;
  const int h = kvh * G + (rem - (rem / G) * G);
  const int bh = b * p.Hq + h;                   // b * Hq + h
  const int T = p.T;
  const int q_end = BLOCK ? p.q_row0 + p.Tq : T;  // query rows of this launch: [q_row0, q_end)
  const int q0a = (BLOCK ? p.q_row0 : 0) + pair * 2 * BM, q0b = q0a + BM;
  // KV tiles of a query tile: up to its diagonal (causal) or all Tk keys (block form, full).
  auto tiles_of = [&](int q0x) {
    if (q0x >= q_end) return 0;
    if (BLOCK && !p.causal) return (p.Tk + BN - 1) / BN;
    return (min(q0x + BM, q_end) - 1) / BN + 1;
  };
  const int nka = tiles_of(q0a);
  const int nkb = tiles_of(q0b);
  const int nk_all = max(nka, nkb);
  auto q0 = [&](int x) { return x ? q0b : q0a; };
  auto n_kv = [&](int x) { return x ? nkb : nka; };

  auto bar = [&](int i) -> uint32_t { return sbase + S::OFF_BAR + 8u * static_cast<uint32_t>(i); };
  const uint32_t BAR_QF = bar(0);
  auto BAR_QR = [&](int x) { return bar(1 + x); };
  auto BAR_KF = [&](int s) { return bar(3 + s); };
  auto BAR_KE = [&](int s) { return bar(3 + NSK + s); };
  auto BAR_VF = [&](int s) { return bar(3 + 2 * NSK + s); };
  auto BAR_VE = [&](int s) { return bar(3 + 2 * NSK + NSV + s); };
  auto BAR_SF = [&](int x) { return bar(3 + 2 * NSK + 2 * NSV + x); };
  auto BAR_PF = [&](int x) { return bar(5 + 2 * NSK + 2 * NSV + x); };
  auto BAR_OF = [&](int x) { return bar(7 + 2 * NSK + 2 * NSV + x); };
  const uint32_t BAR_DR = bar(9 + 2 * NSK + 2 * NSV);
  auto BAR_SC = [&](int x) { return bar(10 + 2 * NSK + 2 * NSV + x); };  // S_x loaded (SEP_P)
  auto BAR_OD = [&](int x) { return bar(12 + 2 * NSK + 2 * NSV + x); };  // PV_x done (SEP_P)
  const uint32_t BAR_STAG = bar(14 + 2 * NSK + 2 * NSV);  // tile A halfway through its first tile
  const uint32_t tmem_slot = sbase + S::OFF_MISC;
  volatile int* failed = reinterpret_cast<volatile int*>(sgen + S::OFF_MISC + 4);

  if (warp == 9) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  // The TMA thread initialises the barriers and starts the query loads before the CTA-wide
  // barrier, so their latency overlaps the TMEM allocation and the other warps' start-up.
  const bool tma_thread = (warp == 8 && lane == 0);
  if (tma_thread) {
    mbar_init(BAR_QF, 1);
    for (int x = 0; x < 2; ++x) {
      mbar_init(BAR_QR(x), 128);
      mbar_init(BAR_SF(x), 1);
      mbar_init(BAR_PF(x), 128);
      mbar_init(BAR_OF(x), 1);
    }
    for (int s = 0; s < NSK; ++s) {
      mbar_init(BAR_KF(s), 1);
      mbar_init(BAR_KE(s), 1);
    }
    for (int s = 0; s < NSV; ++s) {
      mbar_init(BAR_VF(s), 1);
      mbar_init(BAR_VE(s), 1);
    }
    mbar_init(BAR_DR, 1);
    for (int x = 0; x < 2; ++x) {
      mbar_init(BAR_SC(x), 128);
      mbar_init(BAR_OD(x), 1);
    }
    mbar_init(BAR_STAG, 128);
    *failed = 0;
    mbar_fence_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    const int n_q = nkb > 0 ? 2 : 1;  // tile B is skipped when it lies past T
    mbar_expect_tx(BAR_QF, n_q * S::Q_BYTES);
    for (int x = 0; x < n_q; ++x)
#pragma unroll
      for (int blk = 0; blk < S::NBLK; ++blk)
        tma_load_3d(sbase + (x ? S::OFF_QB : S::OFF_QA) + blk * BM * SPAN, &tm_q, BAR_QF,
                    blk * (SPAN / 2), q0(x), bh);
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
    const bool row_ok = qrow < q_end;
    const int nk = n_kv(x);
    // Keys past kmax are masked: the diagonal (causal) or the end of the keys (block form);
    // tiles whose keys all lie at or below the tile's smallest kmax need no mask.
    const int kmax = (!BLOCK || p.causal) ? qrow : p.Tk - 1;
    const int kmax_tile = (!BLOCK || p.causal) ? q0(x) : p.Tk - 1;
    const long long qpos = !BLOCK ? static_cast<long long>(qrow)
                                  : ((qrow < p.pos_split) ? p.pos_off0 + qrow : p.pos_off1 + (qrow - p.pos_split));
    const uint32_t q_tile = sbase + (x ? S::OFF_QB : S::OFF_QA);
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + S::TM_S + x * BN;
    const uint32_t o_addr = tmem + lane_off + S::TM_O + x * D;
    const uint32_t p_addr = S::SEP_P ? tmem + lane_off + S::TM_P + x * (BN / 2) : s_addr;
    const float sl2 = p.scale_log2;
    bool ok = nk > 0;
    if (ok) {
      // Rotate this thread's Q row in place (the table loads are issued before the TMA wait).
      const uint8_t* cosb = static_cast<const uint8_t*>(p.cos);
      const uint8_t* sinb = static_cast<const uint8_t*>(p.sin);
      constexpr int NPQ = (D / 16) < 8 ? (D / 16) : 8;
#pragma unroll 1
      for (int c0 = 0; c0 < D / 16; c0 += NPQ) {
        uint4 cv[NPQ], sv[NPQ];
        if (row_ok)
          load_rope_row<NPQ>(cv, sv, cosb + static_cast<size_t>(qpos) * D,
                             sinb + static_cast<size_t>(qpos) * D, c0, 1);
        if (c0 == 0) {
          ok = mbar_wait(BAR_QF, 0, failed, 300);
          ok = __all_sync(0xffffffffu, ok);
        }
        if (!ok) break;
        if (row_ok) rotate_row<D, BF16, SPAN, NPQ>(q_tile, BM, row, c0, 1, cv, sv);
      }
      if (ok) {
        fence_proxy_async_smem();
        mbar_arrive(BAR_QR(x));
      }
    }
    float m = -INFINITY;  // running max of scaled scores, log2 domain
    float l = 0.f;
    const uint64_t SL2 = f2(sl2, sl2);
    // Tile B starts half a step behind tile A: the two warpgroups share each SMSP's MUFU, so
    // their exponential phases should alternate with each other's loads, reductions and stores
    // rather than coincide. Once set, the offset persists (each tile runs back to back).
    if (S::SEP_P && x == 1 && ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(BAR_STAG, 0, failed, 304));
    }
    for (int j = 0; ok && j < nk; ++j) {
      // S_x(j) complete; without SEP_P this also means every earlier PV_x is complete.
      ok = mbar_wait(BAR_SF(x), j & 1, failed, 301);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // S in two halves: the first half is masked and reduced while the second half loads.
      float s[BN];
      const int k0 = j * BN;
      const bool diag = k0 + BN - 1 > kmax_tile;  // some key of the tile may be masked
#pragma unroll
      for (int c = 0; c < BN / 2; c += 16) tmem_ld16(s_addr + c, s + c);
      tmem_wait_ld();
#pragma unroll
      for (int c = BN / 2; c < BN; c += 16) tmem_ld16(s_addr + c, s + c);
      if (diag) {
#pragma unroll
        for (int c = 0; c < BN / 2; ++c)
          if (k0 + c > kmax) s[c] = -INFINITY;
      }
      float mq[4] = {fmaxf(s[0], s[1]), fmaxf(s[2], s[3]), fmaxf(s[4], s[5]), fmaxf(s[6], s[7])};
#pragma unroll
      for (int c = 8; c < BN / 2; c += 8) {
#pragma unroll
        for (int i = 0; i < 4; ++i) mq[i] = max3(mq[i], s[c + 2 * i], s[c + 2 * i + 1]);
      }
      tmem_wait_ld();
      if constexpr (S::SEP_P) {
        tc_fence_before();
        mbar_arrive(BAR_SC(x));  // S is in registers: the next Q K^T may overwrite it
      }
      if (diag) {
#pragma unroll
        for (int c = BN / 2; c < BN; ++c)
          if (k0 + c > kmax) s[c] = -INFINITY;
      }
#pragma unroll
      for (int c = BN / 2; c < BN; c += 8) {
#pragma unroll
        for (int i = 0; i < 4; ++i) mq[i] = max3(mq[i], s[c + 2 * i], s[c + 2 * i + 1]);
      }
      const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * sl2;
      const float m_new = (mx > m + 8.0f) ? mx : m;
      const uint64_t NM = f2(-m_new, -m_new);
      uint64_t acc[4] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
      uint32_t pk[BN / 2];
      // Some exponentials on the FMA pipe by a cubic (masked scores give 2^-125, not 0: a
      // relative contribution below 1e-37), the rest on MUFU.
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float2 xx = f2_split(f2_fma(f2(s[c], s[c + 1]), SL2, NM));
        float2 pp;
        const int q8 = (c / 2) % 8;
        if ((DU_FA_POLY_MASK >> q8) & 1) {
          pp = ex2_poly2(xx.x, xx.y);
        } else {
          pp = make_float2(ex2(xx.x), ex2(xx.y));
        }
        acc[(c / 2) & 3] = f2_add(acc[(c / 2) & 3], f2(pp.x, pp.y));
        pk[c / 2] = pack2<BF16>(pp.x, pp.y);
        if (S::SEP_P && c == BN / 2 && x == 0 && j == 0) mbar_arrive(BAR_STAG);
      }
      const float2 rsum = f2_split(f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3])));
      if (S::SEP_P && j > 0) {
        // PV_x(j-1) must be complete before O_x is rescaled or its P buffer rewritten.
        ok = mbar_wait(BAR_OD(x), (j - 1) & 1, failed, 303);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (j > 0) {
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
#pragma unroll
      for (int c = 0; c < BN / 2; c += 16) tmem_st16u(p_addr + c, pk + c);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(BAR_PF(x));
    }
    if (ok) {
      ok = mbar_wait(BAR_OF(x), 0, failed, 302);
      ok = __all_sync(0xffffffffu, ok);
    }
    tc_fence_after();
    if (ok) {
      const size_t ri = static_cast<size_t>(bh) * T + qrow;
      const size_t orow = ri * D;
      // Block weights: this block's normalised output and, with an accumulator, the running
      // one, combined by their LSEs (log2 domain).
      const float lse2 = m + lg2(l);
      float w_blk = 1.0f / l, w_acc = 0.f, lse2_out = lse2;
      if (BLOCK && p.acc_mode == 2 && row_ok) {
        const float la2 = p.acc_lse[ri] * 1.4426950408889634f;
        if (la2 > -INFINITY) {
          const float mx = fmaxf(la2, lse2);
          const float ea = ex2(la2 - mx), eb = ex2(lse2 - mx);
          const float inv = 1.0f / (ea + eb);
          w_acc = ea * inv;
          w_blk = eb * inv / l;
          lse2_out = mx + lg2(ea + eb);
        }
      }
#pragma unroll
      for (int c = 0; c < D; c += 16) {
        float o[16];
        tmem_ld16(o_addr + c, o);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] *= w_blk;
          if (BLOCK && p.acc_mode != 0) {
            float4* acc = reinterpret_cast<float4*>(p.acc_o + orow + c);
            if (w_acc > 0.f) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float4 a = acc[i];
                o[4 * i] = fmaf(a.x, w_acc, o[4 * i]);
                o[4 * i + 1] = fmaf(a.y, w_acc, o[4 * i + 1]);
                o[4 * i + 2] = fmaf(a.z, w_acc, o[4 * i + 2]);
                o[4 * i + 3] = fmaf(a.w, w_acc, o[4 * i + 3]);
              }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
          }
          uint32_t w[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) w[i] = pack2<BF16>(o[2 * i], o[2 * i + 1]);
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.out) + (orow + c) * 2);
          dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
      if (row_ok) {
        const float lse_out = lse2_out * 0.69314718055994531f;
        p.lse[ri] = lse_out;
        if (BLOCK && p.acc_mode != 0) p.acc_lse[ri] = lse_out;
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------------ TMA: Q, then the K ring
    regs_dec<S::REG_OTHER>();
    if (lane == 0) {
      int issued = 0;  // (the query tiles were issued before the CTA barrier)
      // The rotated keys come from the preceding rotary launch (this kernel may start before
      // it completes); nothing else this CTA reads is written by it.
      griddep_wait();
      for (int j = 0; j < nk_all; ++j) {
        const int s = j % NSK;
        if (j >= NSK && !mbar_wait(BAR_KE(s), (j / NSK - 1) & 1, failed, 310)) break;
        mbar_expect_tx(BAR_KF(s), S::KV_BYTES);
#pragma unroll
        for (int blk = 0; blk < S::NBLK; ++blk)
          tma_load_3d(sbase + S::OFF_K + s * S::KV_BYTES + blk * BN * SPAN, &tm_k, BAR_KF(s),
                      blk * (SPAN / 2), j * BN, kv_row);
        issued = j + 1;
      }
      // Drain: every TMA write into this CTA's shared memory lands before the CTA exits.
      mbar_wait_drain(BAR_QF, 0, 312);
      for (int j = (issued > NSK ? issued - NSK : 0); j < issued; ++j)
        mbar_wait_drain(BAR_KF(j % NSK), (j / NSK) & 1, 313);
    }
    __syncwarp();
  } else if (warp == 10) {
    // ------------------------------------------------------------------ TMA: the V ring
    regs_dec<S::REG_OTHER>();
    if (lane == 0) {
      tma_prefetch_desc(&tm_v);
      int issued = 0;
      for (int j = 0; j < nk_all; ++j) {
        const int s = j % NSV;
        if (j >= NSV && !mbar_wait(BAR_VE(s), (j / NSV - 1) & 1, failed, 311)) break;
        mbar_expect_tx(BAR_VF(s), S::KV_BYTES);
#pragma unroll
        for (int blk = 0; blk < S::NBLK; ++blk)
          tma_load_3d(sbase + S::OFF_V + s * S::KV_BYTES + blk * BN * SPAN, &tm_v, BAR_VF(s),
                      blk * (SPAN / 2), j * BN, kv_row);
        issued = j + 1;
      }
      for (int j = (issued > NSV ? issued - NSV : 0); j < issued; ++j)
        mbar_wait_drain(BAR_VF(j % NSV), (j / NSV) & 1, 314);
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp walks the schedule (every lane waits, descriptors stay warp-uniform); one
    // elected lane issues each burst of MMAs and the commits. Descriptors are built once: an
    // operand at byte offset `off` from a base has descriptor base + off / 16.
    regs_dec<S::REG_OTHER>();
    bool ok = true;
    for (int x = 0; x < 2 && ok; ++x)
      if (n_kv(x) > 0) ok = mbar_wait(BAR_QR(x), 0, failed, 320);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const uint64_t dq0 = smem_desc(sbase + S::OFF_QA, 16, 8 * SPAN, SWZ);
    const uint64_t dk0 = smem_desc(sbase + S::OFF_K, 16, 8 * SPAN, SWZ);
    const uint64_t dv0 = smem_desc(sbase + S::OFF_V, BN * SPAN, 8 * SPAN, SWZ);
    const bool leader = elect_one();
    auto issue_pv = [&](int x, int jv, uint64_t dv) {
      const uint32_t p_tmem = tmem + (S::SEP_P ? S::TM_P + x * (BN / 2) : S::TM_S + x * BN);
      const uint32_t o_tmem = tmem + S::TM_O + x * D;
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk)  // A = P from TMEM: 16 keys = 8 columns
        umma_f16_ts(o_tmem, p_tmem + kk * 8, dv + static_cast<uint64_t>((kk * 16 * SPAN) >> 4),
                    IDESC_PV, (jv > 0 || kk > 0) ? 1u : 0u);
    };
    auto issue_qk = [&](int x, uint64_t dk) {
      const uint64_t dq = dq0 + static_cast<uint64_t>((x * S::Q_BYTES) >> 4);
      const uint32_t s_tmem = tmem + S::TM_S + x * BN;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off_q = ((kk * 32) / SPAN) * BM * SPAN + (kk * 32) % SPAN;
        const uint32_t off_k = ((kk * 32) / SPAN) * BN * SPAN + (kk * 32) % SPAN;
        umma_f16_ss(s_tmem, dq + (off_q >> 4), dk + (off_k >> 4), IDESC_QK, kk > 0 ? 1u : 0u);
      }
    };
    // Step j issues QK_x(j) and PV_x(j-1) for both tiles; step nk_all only finishes the PVs.
    // With P in its own columns the QKs go first (each after the softmax has loaded S_x(j-1));
    // with P over S, PV_x(j-1) must read P_x before QK_x(j) overwrites it, so per tile PV first.
    for (int j = 0; ok && j <= nk_all; ++j) {
      const bool has_k = j < nk_all;
      const int sk = j % NSK;
      const int jv = j - 1;
      const int sv = (jv + NSV) % NSV;
      if (has_k) {
        ok = __all_sync(0xffffffffu, mbar_wait(BAR_KF(sk), (j / NSK) & 1, failed, 321));
        if (!ok) break;
      }
      const uint64_t dk = dk0 + static_cast<uint64_t>((sk * S::KV_BYTES) >> 4);
      const uint64_t dv = dv0 + static_cast<uint64_t>((sv * S::KV_BYTES) >> 4);
      bool v_ready = false;
      auto pv_step = [&](int x) -> bool {  // PV_x(jv) if tile x has that KV tile
        const int nx = n_kv(x);
        if (jv < 0 || jv >= nx) return true;
        bool w = __all_sync(0xffffffffu, mbar_wait(BAR_PF(x), jv & 1, failed, 322));
        if (w && !v_ready) {
          w = __all_sync(0xffffffffu, mbar_wait(BAR_VF(sv), (jv / NSV) & 1, failed, 323));
          v_ready = true;
        }
        if (!w) return false;
        tc_fence_after();
        if (leader) {
          issue_pv(x, jv, dv);
          if constexpr (S::SEP_P) umma_commit(BAR_OD(x));
          if (jv == nx - 1) umma_commit(BAR_OF(x));  // O_x final once this completes
        }
        __syncwarp();
        return true;
      };
      auto qk_step = [&](int x) -> bool {  // QK_x(j) if tile x has KV tile j
        if (!has_k || j >= n_kv(x)) return true;
        if (S::SEP_P && j > 0 &&
            !__all_sync(0xffffffffu, mbar_wait(BAR_SC(x), (j - 1) & 1, failed, 324)))
          return false;
        tc_fence_after();
        if (leader) {
          issue_qk(x, dk);
          umma_commit(BAR_SF(x));
        }
        __syncwarp();
        return true;
      };
      if constexpr (S::SEP_P) {
        ok = qk_step(0) && qk_step(1) && pv_step(0) && pv_step(1);
      } else {
        ok = pv_step(0) && qk_step(0) && pv_step(1) && qk_step(1);
      }
      if (!ok) break;
      if (leader) {
        if (has_k) umma_commit(BAR_KE(sk));
        if (v_ready) umma_commit(BAR_VE(sv));
      }
      __syncwarp();
    }
    // Drain: all MMAs issued by this warp complete before TMEM is released.
    if (leader) {
      umma_commit(BAR_DR);
      mbar_wait_drain(BAR_DR, 0, 325);
    }
    __syncwarp();
  } else {
    regs_dec<S::REG_OTHER>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

}  // namespace du
