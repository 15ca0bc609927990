// Fused-RoPE decode for grouped-query attention on the sm_100a tensor cores: units of four or
// eight query heads sharing a KV head, head_dim 128 (the Llama-3-8B-shaped layer; group 8).
//
// Mathematics of the reference decode_kernel (dominus_ultra.py:288-413): per query head,
// softmax over the cache of (R(q_pos) q) . (R(j) k_j) * scale, then the weighted sum of v_j. The
// CUDA-core kernel (decode_sm100.cuh) spends ~70 instructions per key row on a four-head unit
// (dot products, cross-lane reductions, P.V); here both products run on tcgen05:
//   S^T = R(K) Q^T   M = 128 keys of a chunk, N = 16 (the unit's 4 or 8 heads, the rest zero), K = D.
//                    A = the K tile as TMA left it (K-major, 128-byte swizzle), rotated in place
//                    into fp16 by the CUDA cores; B = the unit's rotated fp16 query rows.
//   O  += P V        M = 128 TMEM lanes (lanes 0-3 the heads, the rest zero), N = D, K = keys;
//                    A = P in TMEM, B = the V tile (MN-major) -- the prefill kernels' P V form.
// S^T puts one key per TMEM lane, so the softmax is one thread per key. Each of the four compute
// warps keeps its own running max and sum over its 32 keys of every chunk (no cross-warp
// reduction per chunk) and writes its P rows into TMEM lanes 32w + h (its 16 packed columns of
// the chunk; the rest of those rows stay zero), so one P V product accumulates four per-warp
// partial outputs in lanes 32w + h of O. P is double-buffered. At the end of a unit's fragment
// the four (o, max, sum) partials are combined through shared memory.
//
// Warps: 0-3 softmax (warp 0 also rotates the unit's queries) and the per-fragment combine;
// 4 TMA (query header per fragment; K with the cos and sin rows of its keys per chunk); 5 TMEM
// owner and MMA issuer; 6 TMA (V per chunk); 7-10 rotate each K chunk in place as it lands, so
// that rotation and softmax run side by side (with the four softmax warps doing both, one
// warp per SM sub-partition streamed at most ~36 GB/s per SM). The work walk (whole units or flattened (unit, chunk) ranges),
// partial slots and merge are those of decode_kernel. Every mbarrier wait is bounded (du_ptx.cuh).
#pragma once

#include "decode_sm100.cuh"

namespace du {

template <int D_, int GT_ = 4>
struct DecodeTcShape {
  static constexpr int D = D_;
  static constexpr int GT = GT_;    // query heads per unit (rows of the query tile in use)
  static constexpr int NQ = 16;     // rows of the query tile (N of S^T)
  static constexpr int CK = 128;    // keys per chunk (M of S^T)
  static constexpr int SPAN = 128;  // K / V / query rows: 64-element blocks of 128 bytes
  static constexpr int NBLK = 2 * D / SPAN;
  static constexpr int TSPAN = D;   // cos / sin rows: D/2 16-bit values
  static constexpr int PAIRS = D / 16;  // 16-byte chunk pairs (i, i + D/2) per row
  static constexpr int ROWB = 2 * D;
  static constexpr int KV_BYTES = CK * ROWB;
  static constexpr int TAB_BYTES = CK * TSPAN;
  // Two rings: K with the cos / sin rows of its keys (freed once QK has read the rotated keys)
  // and V (freed after PV), refilled by their own TMA warps.
  static constexpr int OFF_K = 0;                  // within a K stage
  static constexpr int OFF_C = KV_BYTES;
  static constexpr int OFF_S = OFF_C + TAB_BYTES;
  static constexpr int KSTAGE = OFF_S + TAB_BYTES;
  static constexpr int NSTG = (D >= 128) ? 2 : 3;
  static constexpr int OFF_VR = NSTG * KSTAGE;      // V ring: NSTG x KV_BYTES
  static constexpr int OFF_Q = OFF_VR + NSTG * KV_BYTES;   // [NQ rows x D] fp16, K-major SW128
  static constexpr int Q_BYTES = NQ * ROWB;
  static constexpr int OFF_P = OFF_Q + Q_BYTES;            // P staging [4 warps][GT][32] 16-bit
  static constexpr int P_BYTES = 4 * GT * 32 * 2;
  static constexpr int NHDR = 2;
  static constexpr int HDR_Q = GT * ROWB;
  static constexpr int HDR = HDR_Q + 2 * TSPAN;           // q rows + cos row + sin row
  static constexpr int OFF_HDR = OFF_P + P_BYTES;
  static constexpr int OFF_MRG = OFF_HDR + NHDR * HDR;     // [4 warps][GT][D] o, then m, l
  static constexpr int MRG_BYTES = 4 * GT * D * 4 + 2 * 4 * GT * 4;
  static constexpr int OFF_BAR = OFF_MRG + MRG_BYTES;
  // full, empty, vfull, vempty, rk: one per stage; then sf, sc, od[2], pf[2], qr, mrg,
  // hfull[2], hempty[2], drain, fma, fmb, k0 (the CTA's first K chunk has landed; one phase)
  static constexpr int B_FULL = 0, B_EMPTY = NSTG, B_VFULL = 2 * NSTG, B_VEMPTY = 3 * NSTG,
                       B_RK = 4 * NSTG, B_SF = 5 * NSTG, B_SC = B_SF + 1, B_OD = B_SF + 2,
                       B_PF = B_SF + 4, B_QR = B_SF + 6, B_MRG = B_SF + 7, B_HFULL = B_SF + 8,
                       B_HEMPTY = B_SF + 10, B_DR = B_SF + 12, B_FMA = B_SF + 13,
                       B_FMB = B_SF + 14, B_K0 = B_SF + 15;
  static constexpr int N_BAR = B_K0 + 1;
  static constexpr int OFF_MISC = OFF_BAR + 8 * N_BAR;     // tmem address, failure flag
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int TM_S = 0;    // S^T: 16 fp32 columns
  static constexpr int TM_P = 64;   // P[2]: CK / 2 packed columns each
  static constexpr int TM_O = 256;  // O: D fp32 columns (lanes 32w + h: warp w's partial of head h)
  static constexpr int NTHREADS = 352;
  static_assert(D == 64 || D == 128, "tensor-core decode: head_dim 64 or 128");
  static_assert(GT == 4 || GT == 8, "tensor-core decode: four or eight heads per unit");
  static_assert(KSTAGE % 1024 == 0 && KV_BYTES % 1024 == 0 && OFF_Q % 1024 == 0 &&
                    Q_BYTES % 1024 == 0, "swizzled tile alignment");
  static_assert(OFF_HDR % 128 == 0 && HDR % 128 == 0 && OFF_MRG % 16 == 0, "header alignment");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(TM_P + CK <= TM_O && TM_O + D <= TMEM_COLS, "TMEM budget");
};

// v[i] for i = lane < N (a chain of selects: no indexed register array), else `other`.
template <int N>
__device__ __forceinline__ float pick(const float (&v)[N], int lane, float other) {
  float r = other;
#pragma unroll
  for (int i = 0; i < N; ++i) r = (lane == i) ? v[i] : r;
  return r;
}

template <int D, bool BF16, int GT>
__global__ void __launch_bounds__(352, 1)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_cos, const __grid_constant__ CUtensorMap tm_sin,
                     const DecodeParams p) {
  using S = DecodeTcShape<D, GT>;
  constexpr int CK = S::CK, SPAN = S::SPAN, NQ = S::NQ, PAIRS = S::PAIRS;
  constexpr uint32_t SWZ = swizzle_code(SPAN);
  constexpr uint32_t IDESC_QK = idesc_f16(128, NQ, 0, 0, 0, 0);  // fp16 R(K) x fp16 R(Q)
  constexpr uint32_t IDESC_PV = idesc_f16(128, D, BF16 ? 1 : 0, BF16 ? 1 : 0, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t sbase = (raw_u32 + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - raw_u32);
  auto bar = [&](int i) -> uint32_t { return sbase + S::OFF_BAR + 8u * static_cast<uint32_t>(i); };
  auto FULL = [&](int s) { return bar(S::B_FULL + s); };      // K + tables of a stage landed
  auto EMPTY = [&](int s) { return bar(S::B_EMPTY + s); };    // QK read it
  auto VFULL = [&](int s) { return bar(S::B_VFULL + s); };
  auto VEMPTY = [&](int s) { return bar(S::B_VEMPTY + s); };  // PV read it
  // K of a stage rotated. One barrier per stage: at a fragment boundary the MMA warp checks the
  // next fragment's first chunk only after its last PV, by which time later chunks may be
  // rotated too; rotating the stage's next chunk needs this chunk's QK, issued after the check.
  auto RK = [&](int s) { return bar(S::B_RK + s); };
  const uint32_t BAR_SF = bar(S::B_SF), BAR_SC = bar(S::B_SC);
  // P of even / odd chunks written (one barrier per P buffer: the MMA warp issues the next QK
  // before waiting for this chunk's P, so a single barrier could complete twice unseen).
  auto PF = [&](int i) { return bar(S::B_PF + i); };
  auto OD = [&](int i) { return bar(S::B_OD + i); };  // PV of even / odd chunks complete
  const uint32_t BAR_QR = bar(S::B_QR), BAR_MRG = bar(S::B_MRG);
  auto HFULL = [&](int i) { return bar(S::B_HFULL + i); };
  auto HEMPTY = [&](int i) { return bar(S::B_HEMPTY + i); };
  const uint32_t BAR_DR = bar(S::B_DR);
  // Fused merge: every consumer thread's partial is stored and fenced (FMA); the ticket's
  // verdict is in the shared word fm_word (FMB).
  const uint32_t BAR_FMA = bar(S::B_FMA), BAR_FMB = bar(S::B_FMB);
  const uint32_t BAR_K0 = bar(S::B_K0);
  volatile int* fm_word = reinterpret_cast<volatile int*>(sgen + S::OFF_MISC + 8);
  int done_t = -1;  // thread 0: this CTA's ticket on the finished-CTA counter (-1: not taken)
  const uint32_t tmem_slot = sbase + S::OFF_MISC;
  volatile int* failed = reinterpret_cast<volatile int*>(sgen + S::OFF_MISC + 4);
  float* mrg = reinterpret_cast<float*>(sgen + S::OFF_MRG);  // o [4][GT][D], m [4][GT], l [4][GT]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
#ifdef DU_TRACE
  // Debug-only timeline of the even CTAs (globaltimer ns): start, set-up done, first S ready,
  // first fragment emitted, last S ready, end.
  auto trace_ev = [&](int e) {
    if ((blockIdx.x & 1) == 0 && blockIdx.x < 148)
      g_du_trace[e * 74 + blockIdx.x / 2] = static_cast<long long>(globaltimer());
  };
  if (tid == 0) {
    trace_ev(0);
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    if ((blockIdx.x & 1) == 0 && blockIdx.x < 148) g_du_trace[6 * 74 + blockIdx.x / 2] = smid;
  }
#endif
  if (tid == 128) {
    for (int s = 0; s < S::NSTG; ++s) {
      mbar_init(FULL(s), 1);
      mbar_init(EMPTY(s), 1);
      mbar_init(VFULL(s), 1);
      mbar_init(VEMPTY(s), 1);
    }
    for (int s = 0; s < S::NSTG; ++s) mbar_init(RK(s), 128);
    mbar_init(BAR_SF, 1);
    mbar_init(BAR_SC, 128);
    mbar_init(PF(0), 128);
    mbar_init(PF(1), 128);
    mbar_init(OD(0), 1);
    mbar_init(OD(1), 1);
    mbar_init(BAR_QR, 32);
    mbar_init(BAR_MRG, 128);
    for (int i = 0; i < S::NHDR; ++i) {
      mbar_init(HFULL(i), 1);
      mbar_init(HEMPTY(i), 32);
    }
    mbar_init(BAR_DR, 1);
    mbar_init(BAR_FMA, 128);
    mbar_init(BAR_FMB, 1);
    mbar_init(BAR_K0, 1);
    *failed = 0;
    mbar_fence_init();
    fence_proxy_async_smem();
  }
  // Zero the query tile (rows GT..NQ-1 stay zero).
  if (warp < 4)
    for (int i = tid; i < S::Q_BYTES / 16; i += 128) st_shared_v4(sbase + S::OFF_Q + 16 * i, make_uint4(0, 0, 0, 0));
  __syncthreads();
  // With per-sequence lengths the launch is a programmatic dependent of the prep kernel (a
  // no-op otherwise). Everything above touches only this CTA's shared memory; once this returns
  // the prep kernel has completed and its writes (chunk offsets, appended cache rows) are
  // visible, including to the bulk copies (async proxy).
  if (p.varlen) {
    griddep_wait();
    fence_proxy_async_global();
  }
  // TMEM is taken only after the wait: a CTA that held columns while waiting could starve a
  // predecessor CTA on the same SM that has yet to allocate (tcgen05.alloc blocks).
  if (warp == 5) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sgen + S::OFF_MISC);
  // Dependents (the merge, or a caller's kernel launched as a programmatic dependent) may launch
  // once every CTA of this grid holds its columns, so none of them can take the TMEM this grid
  // still needs.
  if (tid == 0) griddep_launch_dependents();

  // Zero P in TMEM (lanes GT..127 stay zero).
  if (warp < 4) {
    const uint32_t zero[16] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
#pragma unroll
    for (int c = 0; c < CK; c += 16) tmem_st16u(tmem + lane_off + S::TM_P + c, zero);
    tmem_wait_st();
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint8_t* cosb = static_cast<const uint8_t*>(p.cos);
  const uint8_t* sinb = static_cast<const uint8_t*>(p.sin);
#ifdef DU_TRACE
  if (tid == 0) trace_ev(1);
#endif

  if (warp == 4) {
    // ------------------------------------------------------------------ TMA: headers, K + tables
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_cos);
      tma_prefetch_desc(&tm_sin);
      int g = 0, it = 0;
      bool ok = true;
      DecodeWalk walk;
      walk.init(p);
      DecodeFrag fr;
      for (; ok && walk.next(p, CK, fr); ++it) {
        const int gch = fr.unit % p.n_gchunk;
        const int bk = fr.unit / p.n_gchunk;
        const int hs = it % S::NHDR;
        if (it >= S::NHDR && !mbar_wait(HEMPTY(hs), ((it / S::NHDR) - 1) & 1, failed, 700)) break;
        const int b = bk / p.Hkv;
        const int h0 = (bk - b * p.Hkv) * p.G + gch * GT;
        const uint32_t hd = sbase + S::OFF_HDR + hs * S::HDR;
        const size_t trow = static_cast<size_t>(fr.qpos) * S::TSPAN;  // D/2 16-bit values per row
        mbar_expect_tx(HFULL(hs), static_cast<uint32_t>(S::HDR));
        bulk_load(hd, static_cast<const uint8_t*>(p.q) + (static_cast<size_t>(b) * p.Hq + h0) * S::ROWB,
                  S::HDR_Q, HFULL(hs));
        bulk_load(hd + S::HDR_Q, cosb + trow, S::TSPAN, HFULL(hs));
        bulk_load(hd + S::HDR_Q + S::TSPAN, sinb + trow, S::TSPAN, HFULL(hs));
        for (int c0 = fr.kbeg; c0 < fr.kend; c0 += CK, ++g) {
          const int s = g % S::NSTG;
          if (g >= S::NSTG && !mbar_wait(EMPTY(s), ((g / S::NSTG) - 1) & 1, failed, 701)) {
            ok = false;
            break;
          }
          const uint32_t st = sbase + s * S::KSTAGE;
          const int tpos = static_cast<int>(p.kv_pos_offset + c0);
          mbar_expect_tx(FULL(s), static_cast<uint32_t>(S::KSTAGE));
#pragma unroll
          for (int blk = 0; blk < S::NBLK; ++blk)
            tma_load_3d(st + S::OFF_K + blk * CK * SPAN, &tm_k, FULL(s), blk * (SPAN / 2), c0, bk);
          tma_load_2d(st + S::OFF_C, &tm_cos, FULL(s), 0, tpos);
          tma_load_2d(st + S::OFF_S, &tm_sin, FULL(s), 0, tpos);
        }
      }
      for (int j = (g > S::NSTG ? g - S::NSTG : 0); j < g; ++j)
        mbar_wait_drain(FULL(j % S::NSTG), (j / S::NSTG) & 1, 702);
      for (int j = (it > S::NHDR ? it - S::NHDR : 0); j < it; ++j)
        mbar_wait_drain(HFULL(j % S::NHDR), (j / S::NHDR) & 1, 703);
    }
    __syncwarp();
  } else if (warp == 6) {
    // ------------------------------------------------------------------ TMA: V
    if (lane == 0) {
      tma_prefetch_desc(&tm_v);
      int g = 0;
      bool ok = true;
      DecodeWalk walk;
      walk.init(p);
      DecodeFrag fr;
      while (ok && walk.next(p, CK, fr)) {
        const int bk = fr.unit / p.n_gchunk;
        for (int c0 = fr.kbeg; c0 < fr.kend; c0 += CK, ++g) {
          const int s = g % S::NSTG;
          if (g >= S::NSTG && !mbar_wait(VEMPTY(s), ((g / S::NSTG) - 1) & 1, failed, 704)) {
            ok = false;
            break;
          }
          // The CTA's first V waits until its first K chunk (with the tables) has landed: at the
          // start every CTA's whole ring is requested at once and the first chunk, needed first,
          // shares the bandwidth with the rest (B4 H32 Hkv8 D128 L16384 59.3 -> 58.7 us). The
          // rotation group signals that landing on a barrier with a single phase.
          if (g == 0 && !mbar_wait(BAR_K0, 0, failed, 707)) {
            ok = false;
            break;
          }
          const uint32_t st = sbase + S::OFF_VR + s * S::KV_BYTES;
          mbar_expect_tx(VFULL(s), static_cast<uint32_t>(S::KV_BYTES));
#pragma unroll
          for (int blk = 0; blk < S::NBLK; ++blk)
            tma_load_3d(st + blk * CK * SPAN, &tm_v, VFULL(s), blk * (SPAN / 2), c0, bk);
        }
      }
      for (int j = (g > S::NSTG ? g - S::NSTG : 0); j < g; ++j)
        mbar_wait_drain(VFULL(j % S::NSTG), (j / S::NSTG) & 1, 705);
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    const bool leader = elect_one();
    const uint64_t dq = smem_desc(sbase + S::OFF_Q, 16, 8 * SPAN, SWZ);
    bool ok = true;
    int g = 0, it = 0;
    DecodeWalk walk;
    walk.init(p);
    DecodeFrag fr;
    auto issue_qk = [&](int gg) {
      const uint64_t dk = smem_desc(sbase + (gg % S::NSTG) * S::KSTAGE + S::OFF_K, 16, 8 * SPAN, SWZ);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off_k = ((kk * 32) / SPAN) * CK * SPAN + (kk * 32) % SPAN;
        const uint32_t off_q = ((kk * 32) / SPAN) * NQ * SPAN + (kk * 32) % SPAN;
        umma_f16_ss(tmem + S::TM_S, dk + (off_k >> 4), dq + (off_q >> 4), IDESC_QK, kk > 0 ? 1u : 0u);
      }
      umma_commit(BAR_SF);
      umma_commit(EMPTY(gg % S::NSTG));  // the rotated keys and the tables are read
    };
    for (; ok && walk.next(p, CK, fr);) {
      const int n = (fr.kend - fr.kbeg + CK - 1) / CK;
      if (n == 0) continue;  // a sequence with no keys: nothing to multiply
      ok = __all_sync(0xffffffffu, mbar_wait(BAR_QR, it & 1, failed, 710));
      ++it;  // non-empty fragments (QR phases)
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(RK(g % S::NSTG), (g / S::NSTG) & 1, failed, 711));
      if (ok && g > 0) ok = __all_sync(0xffffffffu, mbar_wait(BAR_SC, (g - 1) & 1, failed, 712));
      if (!ok) break;
      tc_fence_after();
      if (leader) issue_qk(g);
#ifdef DU_TRACE
      if (leader && g == 0) trace_ev(9);
#endif
      __syncwarp();
      for (int j = 0; j < n; ++j) {
        const int gj = g + j;
        if (j + 1 < n) {  // QK of the next chunk, once it is rotated and S has been read
          ok = __all_sync(0xffffffffu, mbar_wait(RK((gj + 1) % S::NSTG), ((gj + 1) / S::NSTG) & 1, failed, 713));
          if (ok) ok = __all_sync(0xffffffffu, mbar_wait(BAR_SC, gj & 1, failed, 714));
          if (!ok) break;
          tc_fence_after();
          if (leader) issue_qk(gj + 1);
          __syncwarp();
        }
        ok = __all_sync(0xffffffffu, mbar_wait(PF(gj & 1), (gj >> 1) & 1, failed, 715));
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(VFULL(gj % S::NSTG), (gj / S::NSTG) & 1, failed, 717));
        if (!ok) break;
        tc_fence_after();
        if (leader) {
          const uint64_t dv = smem_desc(sbase + S::OFF_VR + (gj % S::NSTG) * S::KV_BYTES, CK * SPAN, 8 * SPAN, SWZ);
#pragma unroll
          for (int kk = 0; kk < CK / 16; ++kk)
            umma_f16_ts(tmem + S::TM_O, tmem + S::TM_P + (gj & 1) * (CK / 2) + kk * 8,
                        dv + static_cast<uint64_t>((kk * 16 * SPAN) >> 4), IDESC_PV,
                        (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(OD(gj & 1));
          umma_commit(VEMPTY(gj % S::NSTG));
        }
        __syncwarp();
      }
      g += n;
    }
    if (leader) {
      umma_commit(BAR_DR);
      mbar_wait_drain(BAR_DR, 0, 716);
    }
    __syncwarp();
  } else if (warp >= 7) {
    // ------------------------------------------------------------------ warps 7-10: K rotation
    bool ok = true;
    int g = 0;
    // Rotate the K tile of chunk gg in place (bf16/fp16 -> fp16 at the key positions): units
    // (row, chunk pair), eight per thread of warps 7-10; a quarter-warp covers one swizzled
    // 128-byte row.
    auto rotate_chunk = [&](int gg) -> bool {
      const int s = gg % S::NSTG;
      if (!__all_sync(0xffffffffu, mbar_wait(FULL(s), (gg / S::NSTG) & 1, failed, 720))) return false;
      if (gg == 0 && tid == 224) mbar_arrive(BAR_K0);
#ifdef DU_TRACE
      if (tid == 224 && gg == 0) trace_ev(7);
#endif
      const uint32_t st = sbase + s * S::KSTAGE;
#pragma unroll 2
      for (int u = tid - 224; u < CK * PAIRS; u += 128) {
        const int r = u / PAIRS, c = u % PAIRS;
        const uint32_t o1 = swz_chunk_offset<SPAN>(CK, r, c);
        const uint32_t o2 = swz_chunk_offset<SPAN>(CK, r, c + PAIRS);
        const uint32_t ot = swz_chunk_offset<S::TSPAN>(CK, r, c);
        const uint4 k1 = ld_shared_v4(st + S::OFF_K + o1);
        const uint4 k2 = ld_shared_v4(st + S::OFF_K + o2);
        const uint4 cv = ld_shared_v4(st + S::OFF_C + ot);
        const uint4 sv = ld_shared_v4(st + S::OFF_S + ot);
        const uint32_t a[4] = {k1.x, k1.y, k1.z, k1.w}, bb[4] = {k2.x, k2.y, k2.z, k2.w};
        const uint32_t ca[4] = {cv.x, cv.y, cv.z, cv.w}, sa[4] = {sv.x, sv.y, sv.z, sv.w};
        uint32_t y1[4], y2[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 x1 = unpack2<BF16>(a[e]), x2 = unpack2<BF16>(bb[e]);
          const float2 cc = unpack2<BF16>(ca[e]), ss = unpack2<BF16>(sa[e]);
          y1[e] = pack2<false>(x1.x * cc.x - x2.x * ss.x, x1.y * cc.y - x2.y * ss.y);
          y2[e] = pack2<false>(x2.x * cc.x + x1.x * ss.x, x2.y * cc.y + x1.y * ss.y);
        }
        st_shared_v4(st + S::OFF_K + o1, make_uint4(y1[0], y1[1], y1[2], y1[3]));
        st_shared_v4(st + S::OFF_K + o2, make_uint4(y2[0], y2[1], y2[2], y2[3]));
      }
      fence_proxy_async_smem();
      mbar_arrive(RK(s));
#ifdef DU_TRACE
      if (tid == 224 && gg == 0) trace_ev(8);
#endif
      return true;
    };
    DecodeWalk walk;
    walk.init(p);
    DecodeFrag fr;
    while (ok && walk.next(p, CK, fr)) {
      const int n = (fr.kend - fr.kbeg + CK - 1) / CK;
      for (int j = 0; ok && j < n; ++j) ok = rotate_chunk(g + j);
      g += n;
    }
  } else {
    // ------------------------------------------------------------------ warps 0-3
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const float sl2 = p.scale_log2;
    bool ok = true;
    int g = 0, it = 0;
    const uint32_t stage_w = sbase + S::OFF_P + warp * GT * 32 * 2;  // this warp's P staging
    uint16_t* pst = reinterpret_cast<uint16_t*>(sgen + S::OFF_P) + warp * GT * 32;
    DecodeWalk walk;
    walk.init(p);
    DecodeFrag fr;
    int qf = 0;  // non-empty fragments (QR and MRG phases)
    int fmq = 0;  // fragments through the fused-merge ticket (FMA / FMB phases)
    // The unit's output row gg, dimension d = tid, value val, natural-log lse (thread 0).
    auto emit = [&](const DecodeFrag& f, size_t orow, int gg, float val, float lse) {
      if (tid >= D) return;  // head_dim 64: threads 64..127 hold no dimension
      if (p.varlen && f.slot >= 0) {
        const size_t fs = static_cast<size_t>(f.slot) * GT + gg;  // fragment slot row
        p.o_part[fs * D + tid] = val;
        if (tid == 0) p.lse_part[fs] = lse;
      } else if (p.mode == 0 || f.slot < 0) {
        if constexpr (BF16) {
          static_cast<__nv_bfloat16*>(p.out)[orow * D + tid] = __float2bfloat16_rn(val);
        } else {
          static_cast<__half*>(p.out)[orow * D + tid] = __float2half_rn(val);
        }
      } else {
        p.o_part[(orow * p.n_split + f.slot) * D + tid] = val;
        if (tid == 0) p.lse_part[orow * p.n_split + f.slot] = lse;
        if (f.last)  // the row's unused slots weigh nothing in the merge
          for (int sl = f.slot + 1; sl < p.n_split; ++sl) {
            p.o_part[(orow * p.n_split + sl) * D + tid] = 0.f;
            if (tid == 0) p.lse_part[orow * p.n_split + sl] = -INFINITY;
          }
      }
    };
    for (; ok && walk.next(p, CK, fr); ++it) {
      const int gch = fr.unit % p.n_gchunk;
      const int bk = fr.unit / p.n_gchunk;
      const int b = bk / p.Hkv;
      const int h0 = (bk - b * p.Hkv) * p.G + gch * GT;
      const int n = (fr.kend - fr.kbeg + CK - 1) / CK;
      if (n == 0) {
        // A sequence with no keys (per-sequence lengths): release its header, zero output.
        if (warp == 0) {
          const int hs = it % S::NHDR;
          ok = __all_sync(0xffffffffu, mbar_wait(HFULL(hs), (it / S::NHDR) & 1, failed, 728));
          if (ok) mbar_arrive(HEMPTY(hs));
        }
#pragma unroll
        for (int h = 0; h < GT; ++h)
          emit(fr, static_cast<size_t>(b) * p.Hq + h0 + h, h, 0.f, -INFINITY);
        continue;
      }
      if (warp == 0) {
        // The unit's queries, rotated at the query position into the fp16 query tile.
        const int hs = it % S::NHDR;
        ok = __all_sync(0xffffffffu, mbar_wait(HFULL(hs), (it / S::NHDR) & 1, failed, 722));
        for (int u = lane; ok && u < GT * PAIRS; u += 32) {
          const uint32_t hd = sbase + S::OFF_HDR + hs * S::HDR;
          const int hh = u / PAIRS, c = u % PAIRS;
          const uint4 x1 = ld_shared_v4(hd + hh * S::ROWB + c * 16);
          const uint4 x2 = ld_shared_v4(hd + hh * S::ROWB + D + c * 16);
          const uint4 cv = ld_shared_v4(hd + S::HDR_Q + c * 16);
          const uint4 sv = ld_shared_v4(hd + S::HDR_Q + S::TSPAN + c * 16);
          const uint32_t a[4] = {x1.x, x1.y, x1.z, x1.w}, bb[4] = {x2.x, x2.y, x2.z, x2.w};
          const uint32_t ca[4] = {cv.x, cv.y, cv.z, cv.w}, sa[4] = {sv.x, sv.y, sv.z, sv.w};
          uint32_t y1[4], y2[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 u1 = unpack2<BF16>(a[e]), u2 = unpack2<BF16>(bb[e]);
            const float2 cc = unpack2<BF16>(ca[e]), ss = unpack2<BF16>(sa[e]);
            y1[e] = pack2<false>(u1.x * cc.x - u2.x * ss.x, u1.y * cc.y - u2.y * ss.y);
            y2[e] = pack2<false>(u2.x * cc.x + u1.x * ss.x, u2.y * cc.y + u1.y * ss.y);
          }
          st_shared_v4(sbase + S::OFF_Q + swz_chunk_offset<SPAN>(NQ, hh, c), make_uint4(y1[0], y1[1], y1[2], y1[3]));
          st_shared_v4(sbase + S::OFF_Q + swz_chunk_offset<SPAN>(NQ, hh, c + PAIRS), make_uint4(y2[0], y2[1], y2[2], y2[3]));
        }
        fence_proxy_async_smem();
        if (ok) {
          mbar_arrive(HEMPTY(hs));
          mbar_arrive(BAR_QR);
        }
      }
      // This warp's running max (log2 domain) and sum per head over its keys of the fragment.
      float m[GT], l[GT];
#pragma unroll
      for (int h = 0; h < GT; ++h) {
        m[h] = -1e30f;
        l[h] = 0.f;
      }
      for (int j = 0; ok && j < n; ++j) {
        const int gj = g + j;
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(BAR_SF, gj & 1, failed, 723)))) break;
#ifdef DU_TRACE
        if (tid == 0) {
          if (gj == 0) trace_ev(2);
          trace_ev(4);
        }
#endif
        tc_fence_after();
        float s16[16];
        tmem_ld16(tmem + lane_off + S::TM_S, s16);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(BAR_SC);
        const bool valid = fr.kbeg + j * CK + tid < fr.kend;
        float pe[GT], alpha[GT];
        bool moved = false;
#pragma unroll
        for (int h = 0; h < GT; ++h) {
          const float x = valid ? s16[h] * sl2 : -INFINITY;
          float mx = x;
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          const float mn = (mx > m[h] + 8.0f) ? mx : m[h];
          pe[h] = valid ? ex2(x - mn) : 0.f;
          float sum = pe[h];
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
          alpha[h] = (mn != m[h]) ? ex2(m[h] - mn) : 1.0f;
          moved |= (mn != m[h]);
          l[h] = l[h] * alpha[h] + sum;
          m[h] = mn;
          pst[h * 32 + lane] = static_cast<uint16_t>(pack2<BF16>(pe[h], 0.f) & 0xffffu);
        }
        __syncwarp();
        // P buffer gj & 1 was last read by PV(gj - 2); a moved max rescales O, which holds
        // PV(..gj - 1) of this fragment.
        if (j >= 2) ok = mbar_wait(OD(gj & 1), ((gj - 2) >> 1) & 1, failed, 724);
        if (ok && moved && j >= 1) ok = mbar_wait(OD((gj - 1) & 1), ((gj - 1) >> 1) & 1, failed, 725);
        if (!(ok = __all_sync(0xffffffffu, ok))) break;
        tc_fence_after();
        if (moved && j >= 1) {
          const float al = pick<GT>(alpha, lane, 1.0f);
#pragma unroll 1
          for (int c = 0; c < D; c += 16) {
            float o[16];
            tmem_ld16(tmem + lane_off + S::TM_O + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] *= al;
            tmem_st16(tmem + lane_off + S::TM_O + c, o);
          }
        }
        {
          // Lane h < GT: head h's 32 probabilities of this warp's keys, packed (16 columns).
          uint32_t w[16];
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 x4 = make_uint4(0, 0, 0, 0);
            if (lane < GT) x4 = ld_shared_v4(stage_w + lane * 64 + q4 * 16);
            w[4 * q4] = x4.x;
            w[4 * q4 + 1] = x4.y;
            w[4 * q4 + 2] = x4.z;
            w[4 * q4 + 3] = x4.w;
          }
          tmem_st16u(tmem + lane_off + S::TM_P + (gj & 1) * (CK / 2) + warp * 16, w);
          tmem_wait_st();
        }
        __syncwarp();
        tc_fence_before();
        mbar_arrive(PF(gj & 1));
      }
      g += n;
      if (!ok) break;
      // Combine the four warps' partials: warp w's O rows are TMEM lanes 32w + h.
      ok = __all_sync(0xffffffffu, mbar_wait(OD((g - 1) & 1), ((g - 1) >> 1) & 1, failed, 726));
      if (!ok) break;
      tc_fence_after();
      // O in batches of four 16-column loads per wait.
      constexpr int OB = (D >= 64) ? 64 : D;
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += OB) {
        float o[OB];
#pragma unroll
        for (int c = 0; c < OB; c += 16) tmem_ld16(tmem + lane_off + S::TM_O + c0 + c, o + c);
        tmem_wait_ld();
        if (lane < GT) {
          float4* dst = reinterpret_cast<float4*>(mrg + (warp * GT + lane) * D + c0);
#pragma unroll
          for (int i = 0; i < OB / 4; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        }
      }
      if (lane < GT) {
        mrg[4 * GT * D + warp * GT + lane] = pick<GT>(m, lane, 0.f);
        mrg[4 * GT * D + 4 * GT + warp * GT + lane] = pick<GT>(l, lane, 0.f);
      }
      tc_fence_before();
      mbar_arrive(BAR_MRG);
      ok = __all_sync(0xffffffffu, mbar_wait(BAR_MRG, qf & 1, failed, 727));
      ++qf;
      if (!ok) break;
      // Thread d writes dimension d of the unit's GT rows.
      const float* mw = mrg + 4 * GT * D;
      const float* lw = mw + 4 * GT;
#pragma unroll
      for (int h = 0; h < GT; ++h) {
        float M = mw[h];
#pragma unroll
        for (int w2 = 1; w2 < 4; ++w2) M = fmaxf(M, mw[w2 * GT + h]);
        float L = 0.f, A = 0.f;
#pragma unroll
        for (int w2 = 0; w2 < 4; ++w2) {
          const float wt = ex2(mw[w2 * GT + h] - M);
          L += lw[w2 * GT + h] * wt;
          A += mrg[(w2 * GT + h) * D + (tid < D ? tid : 0)] * wt;
        }
        const size_t orow = static_cast<size_t>(b) * p.Hq + h0 + h;
        emit(fr, orow, h, (L > 0.f) ? A / L : 0.f,
             (L > 0.f) ? (M + lg2(L)) * 0.69314718055994531f : -INFINITY);
      }
#ifdef DU_TRACE
      if (tid == 0 && qf == 1) trace_ev(3);
#endif
      if (p.fused_merge && !p.varlen && fr.slot >= 0) {
        // Ticket: the fragment that completes the unit merges its GT rows. The consumer threads'
        // partial stores reach thread 0 through the barrier (release / acquire in the CTA); its
        // ticket is an acquire-release add, which makes them visible device-wide before the
        // ticket and, after the last ticket, the other fragments' partials visible to this CTA.
        mbar_arrive(BAR_FMA);
        if (tid == 0) {
          int verdict = -1;
          if (mbar_wait(BAR_FMA, fmq & 1, failed, 729)) {
            const long long ub = static_cast<long long>(fr.unit) * p.cpu;
            const int nf = DecodeWalk::cta_of(p, ub + p.cpu - 1) - DecodeWalk::cta_of(p, ub) + 1;
            verdict = (atom_add_acq_rel_gpu(&p.unit_cnt[fr.unit], 1) == nf - 1) ? nf : 0;
            // After the CTA's last unit ticket, its ticket on the finished-CTA counter: the
            // counters may be zeroed once every CTA has taken its unit tickets, so this one is
            // taken now and its value read only at the end (the round trip overlaps the merge).
            DecodeWalk peek = walk;
            DecodeFrag nx;
            if (!peek.next(p, CK, nx)) done_t = atomicAdd(&p.unit_cnt[DECODE_CNT_DONE], 1);
          }
          *fm_word = verdict;
          mbar_arrive(BAR_FMB);
        }
        ok = __all_sync(0xffffffffu, mbar_wait(BAR_FMB, fmq & 1, failed, 730));
        ++fmq;
        if (!ok) break;
        const int nf = *fm_word;
        if (nf < 0) {
          ok = false;
          break;
        }
        if (nf > 0 && tid < D) {
          // Online LSE merge of the nf partials of each head, NB slots per batch of loads (all
          // of a batch's loads in flight at once: one L2 round trip per batch).
          constexpr int NB = 32 / GT;
          float M[GT], L[GT], A[GT];
#pragma unroll
          for (int h = 0; h < GT; ++h) {
            M[h] = -INFINITY;
            L[h] = 0.f;
            A[h] = 0.f;
          }
          const size_t row0 = static_cast<size_t>(b) * p.Hq + h0;
#pragma unroll 1
          for (int s0 = 0; s0 < nf; s0 += NB) {
            float lv[GT][NB], ov[GT][NB];
#pragma unroll
            for (int h = 0; h < GT; ++h)
#pragma unroll
              for (int i = 0; i < NB; ++i) {
                const bool in = s0 + i < nf;
                const size_t sr = (row0 + h) * p.n_split + s0 + i;
                lv[h][i] = in ? __ldcg(p.lse_part + sr) : -INFINITY;
                ov[h][i] = in ? __ldcg(p.o_part + sr * D + tid) : 0.f;
              }
#pragma unroll
            for (int h = 0; h < GT; ++h) {
              float mb = M[h];
#pragma unroll
              for (int i = 0; i < NB; ++i) mb = fmaxf(mb, lv[h][i]);
              if (mb == -INFINITY) continue;
              const float sc = __expf(M[h] - mb);
              L[h] *= sc;
              A[h] *= sc;
#pragma unroll
              for (int i = 0; i < NB; ++i) {
                const float w = __expf(lv[h][i] - mb);
                L[h] += w;
                A[h] = fmaf(w, ov[h][i], A[h]);
              }
              M[h] = mb;
            }
          }
#pragma unroll
          for (int h = 0; h < GT; ++h) {
            const size_t row = row0 + h;
            const float val = (L[h] > 0.f) ? A[h] / L[h] : 0.f;
            if (p.fin_kind == 2) {
              static_cast<float*>(p.fin_out)[row * D + tid] = val;
              if (tid == 0) p.fin_lse[row] = (L[h] > 0.f) ? M[h] + __logf(L[h]) : -INFINITY;
            } else if (p.fin_kind == 1) {
              static_cast<__nv_bfloat16*>(p.fin_out)[row * D + tid] = __float2bfloat16_rn(val);
            } else {
              static_cast<__half*>(p.fin_out)[row * D + tid] = __float2half_rn(val);
            }
          }
        }
      }
    }
  }

#ifdef DU_TRACE
  if (tid == 0) trace_ev(5);
#endif
  if (p.fused_merge && !p.varlen) {
    // The last CTA to take its finished-CTA ticket zeroes the counters for the next call (every
    // CTA gets here, also after a failed wait, so the counters never stay dirty). A CTA takes
    // that ticket only after all of its unit tickets, so none is taken after the zeroing.
    __syncthreads();
    if (tid == 0) {
      if (done_t < 0) done_t = atomicAdd(&p.unit_cnt[DECODE_CNT_DONE], 1);
      *fm_word = (done_t == static_cast<int>(gridDim.x) - 1) ? 1 : 0;
    }
    __syncthreads();
    if (*fm_word == 1) {
      __threadfence();
      for (int i = tid; i < p.n_units; i += S::NTHREADS) p.unit_cnt[i] = 0;
      if (tid == 0) p.unit_cnt[DECODE_CNT_DONE] = 0;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

}  // namespace du
