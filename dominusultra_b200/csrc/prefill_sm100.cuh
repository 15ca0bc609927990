// Fused-RoPE causal prefill for sm_100a: tcgen05 tensor cores, TMEM accumulators, TMA loads.
//
// Computes, per (batch, query head), out = softmax(R(Q) R(K)^T / sqrt(D), causal) V and the
// natural-log LSE of each row, where R is the half-split rotary rotation at each row's position
// (reference: prefill_kernel, dominus_ultra.py:119-285; rotation :185-208 and :243-257, causal
// mask :260-261, online softmax :263-272, lse = m + log(l) :284-285). Query head h reads KV
// head h / (Hq / Hkv) (dominus_ultra.py:168).
//
// One CTA owns one 128-row query tile of one (b, h) and walks the KV tiles up to its diagonal
// (fully masked tiles are never visited). Warp roles, 320 threads:
//   warps 0-3  softmax: thread t owns query row t = TMEM lane t. Loads S from TMEM, applies
//              the causal mask and the online softmax in the log2 domain, writes P to shared
//              memory (16-bit, UMMA K-major layout), rescales O in TMEM only when the running
//              max grows by more than 2^8, and writes out / lse at the end.
//   warps 4-7  rotation: Q (once) and every K tile arrive from TMA in the 128B-swizzled layout
//              the tensor core reads; each thread rotates its row in fp32 registers and writes
//              it back in place as fp16 (fp16 Q/K operands keep the LSE within 1e-3 of an fp32
//              reference; bf16 operands do not).
//   warp 8     TMA producer: Q once, then K and V tiles into an NSTAGE-deep ring.
//   warp 9     TMEM allocator and single-thread tcgen05.mma issuer:
//              S[j%2] = Q K_j^T (fp16 x fp16 -> fp32 TMEM), then O += P_{j-1} V_{j-1}
//              (P and V in the input dtype, V read MN-major straight from its TMA tile).
// TMEM columns: S0 [0, BN), S1 [BN, 2BN), O [2BN, 2BN + D).
// Every mbarrier wait is bounded (du_ptx.cuh); no TMA multicast is used anywhere.
#pragma once

#include "du_ptx.cuh"


namespace du {

struct PrefillParams {
  const void* cos;  // [>= T, D/2], input dtype
  const void* sin;  // [>= T, D/2]
  void* out;        // [B, Hq, T, D], input dtype
  float* lse;       // [B, Hq, T]
  int Hq;
  int Hkv;
  int T;
  int n_qtiles;
  float scale_log2;  // softmax scale * log2(e)
  // Block form (prefill_fa_kernel only; the causal whole-sequence call sets q_row0 = 0,
  // Tq = Tk = T, causal = 1, pos_split = T, pos_off0 = 0, acc_mode = 0):
  //   query rows [q_row0, q_row0 + Tq) of the T-row tensors, keys [0, Tk) of the KV tensors;
  //   causal: key t visible to query row t' iff t <= t' (local rows; needs q_row0 = 0,
  //   Tq = Tk = T); otherwise every key is visible;
  //   query row t rotates at pos_off0 + t for t < pos_split, pos_off1 + (t - pos_split) beyond;
  //   acc_mode 1: the block's (out, lse) also overwrite the fp32 accumulators acc_o [B, Hq, T, D]
  //   and acc_lse [B, Hq, T]; 2: they are LSE-merged into them. In both, out and lse receive the
  //   merged result.
  int q_row0;
  int Tq;
  int Tk;
  int causal;
  long long pos_split;
  long long pos_off0;
  long long pos_off1;
  float* acc_o;
  float* acc_lse;
  int acc_mode;
  // prefill_fa1_kernel only: the K tensor map covers the raw keys and the kernel rotates each
  // key tile in place (T <= Fa1Shape::NSK * BN, so no ring stage is reused).
  int krot;
};

template <int D>
struct PrefillShape {
  static constexpr int BM = 128;                          // query rows per tile (UMMA M)
  static constexpr int BN = (D >= 256) ? 64 : 128;         // keys per KV tile
  static constexpr int SPAN = (2 * D >= 128) ? 128 : 2 * D;  // bytes per swizzled row block
  static constexpr int NBLK = 2 * D / SPAN;               // column blocks of a Q/K/V tile
  static constexpr int NSTAGE = (D >= 128) ? 2 : 3;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + NSTAGE * KV_BYTES;
  static constexpr int OFF_P = OFF_V + NSTAGE * KV_BYTES;
  static constexpr int OFF_BAR = OFF_P + P_BYTES;
  // barriers: q_full, q_rot, k_full[NS], k_rot[NS], k_empty[NS], v_full[NS], v_empty[NS],
  //           s_full[2], p_full, o_done, mma_drain
  static constexpr int N_BAR = 2 + 5 * NSTAGE + 5;
  static constexpr int OFF_MISC = OFF_BAR + 8 * N_BAR;  // tmem base slot (u32), failed flag
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
  static constexpr int TMEM_COLS = 512;
  static constexpr int TM_S0 = 0;
  static constexpr int TM_S1 = BN;
  static constexpr int TM_O = 2 * BN;
  static constexpr int NTHREADS = 320;
  static_assert(2 * BN + D <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(Q_BYTES % 1024 == 0 && KV_BYTES % 1024 == 0 && P_BYTES % 1024 == 0, "align");
};

// Load the cos/sin chunks a thread needs for one row: chunk c = c0 + i * cstep holds table
// entries [8c, 8c + 8) of the half-width row. All loads are issued together (they are L2 hits
// shared by every CTA) so their latency is paid once per tile, ahead of the tile's TMA wait.
template <int NP>
__device__ __forceinline__ void load_rope_row(uint4 (&cv)[NP], uint4 (&sv)[NP], const uint8_t* cos_row,
                                              const uint8_t* sin_row, int c0, int cstep) {
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    cv[i] = ldg_v4(cos_row + (c0 + i * cstep) * 16);
    sv[i] = ldg_v4(sin_row + (c0 + i * cstep) * 16);
  }
}

// Rotate NP chunk pairs of one row of a K-major swizzled tile in place: chunk c holds elements
// [8c, 8c+8) of the first half, chunk c + D/16 the matching elements of the second half.
// Input dtype -> fp32 rotation -> fp16 written back (the UMMA operand type).
template <int D, bool BF16, int SPAN, int NP>
__device__ __forceinline__ void rotate_row(uint32_t tile, int rows, int r, int c0, int cstep,
                                           const uint4 (&cv)[NP], const uint4 (&sv)[NP]) {
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int c = c0 + i * cstep;
    const uint32_t a1 = tile + swz_chunk_offset<SPAN>(rows, r, c);
    const uint32_t a2 = tile + swz_chunk_offset<SPAN>(rows, r, c + D / 16);
    const uint4 x1 = ld_shared_v4(a1);
    const uint4 x2 = ld_shared_v4(a2);
    const uint32_t xa[4] = {x1.x, x1.y, x1.z, x1.w};
    const uint32_t xb[4] = {x2.x, x2.y, x2.z, x2.w};
    const uint32_t ca[4] = {cv[i].x, cv[i].y, cv[i].z, cv[i].w};
    const uint32_t sa[4] = {sv[i].x, sv[i].y, sv[i].z, sv[i].w};
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

template <int D, bool BF16>
__global__ void __launch_bounds__(320, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
  using S = PrefillShape<D>;
  constexpr int BM = S::BM, BN = S::BN, SPAN = S::SPAN, NS = S::NSTAGE;
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
  const int bh = blockIdx.x;                      // b * Hq + h
  const int qt = p.n_qtiles - 1 - blockIdx.y;     // longest (most KV tiles) first
  const int b = bh / p.Hq;
  const int h = bh - b * p.Hq;
  const int kvh = h / (p.Hq / p.Hkv);
  const int kv_row = b * p.Hkv + kvh;
  const int q0 = qt * BM;
  const int T = p.T;
  const int q_end = min(q0 + BM, T);
  const int n_kv = (q_end - 1) / BN + 1;

  auto bar = [&](int i) -> uint32_t { return sbase + S::OFF_BAR + 8u * static_cast<uint32_t>(i); };
  const uint32_t BAR_QF = bar(0), BAR_QR = bar(1);
  auto BAR_KF = [&](int s) { return bar(2 + s); };
  auto BAR_KR = [&](int s) { return bar(2 + NS + s); };
  auto BAR_KE = [&](int s) { return bar(2 + 2 * NS + s); };
  auto BAR_VF = [&](int s) { return bar(2 + 3 * NS + s); };
  auto BAR_VE = [&](int s) { return bar(2 + 4 * NS + s); };
  auto BAR_SF = [&](int i) { return bar(2 + 5 * NS + i); };
  const uint32_t BAR_PF = bar(2 + 5 * NS + 2);
  const uint32_t BAR_OD = bar(2 + 5 * NS + 3);
  const uint32_t BAR_DRAIN = bar(2 + 5 * NS + 4);
  const uint32_t tmem_slot = sbase + S::OFF_MISC;
  volatile int* failed = reinterpret_cast<volatile int*>(sgen + S::OFF_MISC + 4);

  if (warp == 9) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(BAR_QF, 1);
    mbar_init(BAR_QR, 128);
    for (int s = 0; s < NS; ++s) {
      mbar_init(BAR_KF(s), 1);
      mbar_init(BAR_KR(s), 128);
      mbar_init(BAR_KE(s), 1);
      mbar_init(BAR_VF(s), 1);
      mbar_init(BAR_VE(s), 1);
    }
    mbar_init(BAR_SF(0), 1);
    mbar_init(BAR_SF(1), 1);
    mbar_init(BAR_PF, 128);
    mbar_init(BAR_OD, 1);
    mbar_init(BAR_DRAIN, 1);
    *failed = 0;
    mbar_fence_init();
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sgen + S::OFF_MISC);

  if (warp < 4) {
    // ------------------------------------------------------------------ softmax / epilogue
    const int row = tid;
    const int qrow = q0 + row;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t o_addr = tmem + lane_off + S::TM_O;
    const float sl2 = p.scale_log2;
    float m = -INFINITY;  // running max of scaled scores, log2 domain
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = mbar_wait(BAR_SF(j & 1), (j >> 1) & 1, failed, 10);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      if (tid == 0) DU_TRACE_EV(0, j);
      tc_fence_after();
      float s[BN];
      const uint32_t s_addr = tmem + lane_off + ((j & 1) ? S::TM_S1 : S::TM_S0);
#pragma unroll
      for (int c = 0; c < BN; c += 16) tmem_ld16(s_addr + c, s + c);
      tmem_wait_ld();
      const int k0 = j * BN;
      if (k0 + BN - 1 > q0) {  // tile crosses the diagonal of this query tile
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (k0 + c > qrow) s[c] = -INFINITY;
      }
      float mx = s[0];
#pragma unroll
      for (int c = 1; c < BN; ++c) mx = fmaxf(mx, s[c]);
      mx *= sl2;
      // Lazy rescale: keep the stale max unless the new one exceeds it by more than 8
      // (P stays <= 2^8, exact in the end because l uses the same reference point).
      const float m_new = (mx > m + 8.0f) ? mx : m;
      float rs = 0.f;
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float p0 = ex2(fmaf(s[c], sl2, -m_new));
        const float p1 = ex2(fmaf(s[c + 1], sl2, -m_new));
        rs += p0 + p1;
        pk[c / 2] = pack2<BF16>(p0, p1);
      }
      if (j > 0) {
        if (tid == 0) DU_TRACE_EV(1, j);
        ok = mbar_wait(BAR_OD, (j - 1) & 1, failed, 11);  // PV_{j-1} done: P free, O current
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        if (tid == 0) DU_TRACE_EV(2, j);
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
          tmem_wait_st();
        }
      }
      l += rs;
      m = m_new;
#pragma unroll
      for (int c = 0; c < BN / 8; ++c) {
        st_shared_v4(sbase + S::OFF_P + swz_chunk_offset<128>(BM, row, c),
                     make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]));
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(BAR_PF);
      if (tid == 0) DU_TRACE_EV(3, j);
    }
    if (ok) {
      ok = mbar_wait(BAR_OD, (n_kv - 1) & 1, failed, 12);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (tid == 0) DU_TRACE_EV(4, 0);
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
  } else if (warp < 8) {
    // ------------------------------------------------------------------ RoPE rotation
    const int rt = tid - 128;
    const uint8_t* cosb = static_cast<const uint8_t*>(p.cos);
    const uint8_t* sinb = static_cast<const uint8_t*>(p.sin);
    constexpr int ROW_TAB = D;               // bytes per cos/sin table row (D/2 16-bit values)
    constexpr int TPR = 128 / BN;            // threads per K row
    constexpr int NPQ = (D / 16) < 8 ? (D / 16) : 8;  // chunk pairs per batch of a Q row
    constexpr int NPK = (D / 16) / TPR;      // chunk pairs per thread of a K row (<= 8)
    static_assert(NPK <= 8, "K rotation batch");
    bool ok;
    {
      const int pos = q0 + rt;
      ok = true;
#pragma unroll 1
      for (int c0 = 0; c0 < D / 16; c0 += NPQ) {
        uint4 cv[NPQ], sv[NPQ];
        if (pos < T)
          load_rope_row<NPQ>(cv, sv, cosb + static_cast<size_t>(pos) * ROW_TAB,
                             sinb + static_cast<size_t>(pos) * ROW_TAB, c0, 1);
        if (c0 == 0) ok = mbar_wait(BAR_QF, 0, failed, 20);
        if (!ok) break;
        if (pos < T) rotate_row<D, BF16, SPAN, NPQ>(sbase + S::OFF_Q, BM, rt, c0, 1, cv, sv);
      }
      if (ok) {
        fence_proxy_async_smem();
        mbar_arrive(BAR_QR);
      }
    }
    const int r = rt / TPR;
    const int sub = rt % TPR;
    for (int j = 0; ok && j < n_kv; ++j) {
      const int s = j % NS;
      const int kpos = j * BN + r;
      uint4 cv[NPK], sv[NPK];
      if (kpos < T)
        load_rope_row<NPK>(cv, sv, cosb + static_cast<size_t>(kpos) * ROW_TAB,
                           sinb + static_cast<size_t>(kpos) * ROW_TAB, sub, TPR);
      if (rt == 0) DU_TRACE_EV(5, j);
      if (!mbar_wait(BAR_KF(s), (j / NS) & 1, failed, 21)) break;
      if (rt == 0) DU_TRACE_EV(6, j);
      if (kpos < T)
        rotate_row<D, BF16, SPAN, NPK>(sbase + S::OFF_K + s * S::KV_BYTES, BN, r, sub, TPR, cv, sv);
      fence_proxy_async_smem();
      mbar_arrive(BAR_KR(s));
      if (rt == 0) DU_TRACE_EV(7, j);
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      DU_TRACE_EV(11, 0);
      mbar_expect_tx(BAR_QF, S::Q_BYTES);
#pragma unroll
      for (int blk = 0; blk < S::NBLK; ++blk)
        tma_load_3d(sbase + S::OFF_Q + blk * BM * SPAN, &tm_q, BAR_QF, blk * (SPAN / 2), q0, bh);
      int issued_k = 0, issued_v = 0;  // loads issued, for the drain below
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % NS;
        const uint32_t ph = (j / NS) & 1;
        if (j >= NS && !mbar_wait(BAR_KE(s), ph ^ 1u, failed, 30)) break;
        DU_TRACE_EV(12, j);
        mbar_expect_tx(BAR_KF(s), S::KV_BYTES);
#pragma unroll
        for (int blk = 0; blk < S::NBLK; ++blk)
          tma_load_3d(sbase + S::OFF_K + s * S::KV_BYTES + blk * BN * SPAN, &tm_k, BAR_KF(s),
                      blk * (SPAN / 2), j * BN, kv_row);
        issued_k = j + 1;
        if (j >= NS && !mbar_wait(BAR_VE(s), ph ^ 1u, failed, 31)) break;
        DU_TRACE_EV(13, j);
        mbar_expect_tx(BAR_VF(s), S::KV_BYTES);
#pragma unroll
        for (int blk = 0; blk < S::NBLK; ++blk)
          tma_load_3d(sbase + S::OFF_V + s * S::KV_BYTES + blk * BN * SPAN, &tm_v, BAR_VF(s),
                      blk * (SPAN / 2), j * BN, kv_row);
        issued_v = j + 1;
      }
      // Drain: every TMA write into this CTA's shared memory must land before the CTA exits
      // (a no-op on the normal path, where consumers already waited on each of them).
      mbar_wait_drain(BAR_QF, 0, 32);
      for (int j = (issued_k > NS ? issued_k - NS : 0); j < issued_k; ++j)
        mbar_wait_drain(BAR_KF(j % NS), (j / NS) & 1, 33);
      for (int j = (issued_v > NS ? issued_v - NS : 0); j < issued_v; ++j)
        mbar_wait_drain(BAR_VF(j % NS), (j / NS) & 1, 34);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && mbar_wait(BAR_QR, 0, failed, 40)) {
      tc_fence_after();
      for (int j = 0; j <= n_kv; ++j) {
        if (j < n_kv) {
          const int s = j % NS;
          if (!mbar_wait(BAR_KR(s), (j / NS) & 1, failed, 41)) break;
          DU_TRACE_EV(8, j);
          tc_fence_after();
          const uint32_t d_tmem = tmem + ((j & 1) ? S::TM_S1 : S::TM_S0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int blk = (kk * 32) / SPAN;
            const int inrow = (kk * 32) % SPAN;
            const uint64_t a = smem_desc(sbase + S::OFF_Q + blk * BM * SPAN + inrow, 16, 8 * SPAN, SWZ);
            const uint64_t bd =
                smem_desc(sbase + S::OFF_K + s * S::KV_BYTES + blk * BN * SPAN + inrow, 16, 8 * SPAN, SWZ);
            umma_f16_ss(d_tmem, a, bd, IDESC_QK, kk > 0 ? 1u : 0u);
          }
          umma_commit(BAR_SF(j & 1));
          umma_commit(BAR_KE(s));
        }
        if (j >= 1) {
          const int jj = j - 1;
          const int s = jj % NS;
          if (!mbar_wait(BAR_PF, jj & 1, failed, 42)) break;
          DU_TRACE_EV(9, jj);
          if (!mbar_wait(BAR_VF(s), (jj / NS) & 1, failed, 43)) break;
          DU_TRACE_EV(10, jj);
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const int blk = (kk * 32) / 128;
            const int inrow = (kk * 32) % 128;
            const uint64_t a = smem_desc(sbase + S::OFF_P + blk * BM * 128 + inrow, 16, 1024, 2);
            const uint64_t bd = smem_desc(sbase + S::OFF_V + s * S::KV_BYTES + kk * 16 * SPAN,
                                          BN * SPAN, 8 * SPAN, SWZ);
            umma_f16_ss(tmem + S::TM_O, a, bd, IDESC_PV, (jj > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(BAR_VE(s));
          umma_commit(BAR_OD);
        }
      }
    }
    if (lane == 0) {
      // Drain: all MMAs issued by this thread complete before TMEM is released.
      umma_commit(BAR_DRAIN);
      mbar_wait_drain(BAR_DRAIN, 0, 44);
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

}  // namespace du
