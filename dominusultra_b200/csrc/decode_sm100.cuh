// Fused-RoPE decode for sm_100a: persistent split-KV streaming kernel plus an LSE-weighted
// merge.
//
// One new query token per (batch, query head) attends over a KV cache, rotating the query at
// position q_pos and key j at position kv_pos_offset + j (reference: decode_kernel,
// dominus_ultra.py:288-413; query rotation :335-344, key rotation :381-395, online softmax
// :397-409). With q_pos = L and kv_pos_offset = 0 this is exactly the reference's semantics
// (the cache holds positions 0..L-1, the new token is at L and does not attend to itself).
//
// The kernel is HBM-bound, so it is laid out for streaming:
//  * a unit is one (b, kv head, group chunk) serving GT query heads of the GQA group (so each
//    KV byte is read once); a persistent grid (resident CTAs only) walks either whole units
//    round-robin or, when units are fewer than resident CTAs, equal contiguous ranges of the
//    flattened (unit, chunk) sequence (per-unit fragments with one partial slot each);
//  * a producer warp streams each item's keys in chunks of CK rows: K, V and the matching
//    cos/sin table rows are contiguous in memory, so each chunk is four cp.async.bulk copies
//    (no multicast) into a 3-stage shared-memory ring guarded by mbarriers, and it runs ahead
//    across item boundaries; the item's query rows and the cos/sin row at the query position
//    come the same way into a 2-entry header ring, so no consumer waits on a global load;
//  * four consumer warps read the ring: a few lanes share one key row and each lane takes
//    whole half-split RoPE partner chunks (elements [8c, 8c+8) and [D/2 + 8c, D/2 + 8c + 8)),
//    so the key rotation needs no shuffles; it runs two elements per instruction in the input
//    dtype (as the reference rotates in the input dtype), the rotated key and V are widened to
//    fp32 and the dot products / P V sums use packed f32x2 FMAs; scores are reduced across the
//    lanes of a row with xor-shuffles; the online softmax runs per lane group in the log2
//    domain and moves its reference max only when a score exceeds it by 2^8;
//  * at the end of an item the lane groups and warps are merged; when a unit is spread over
//    several CTAs, each fragment writes an fp32 partial (out normalised over the fragment,
//    natural-log LSE) into its slot of the row and merge_kernel combines the slots (a merge by
//    the last fragment through per-unit counters measured slower).
#pragma once

#include "du_ptx.cuh"

namespace du {

struct DecodeParams {
  const void* q;    // [B, Hq, D]
  const void* k;    // [B, Hkv, L, D]
  const void* v;    // [B, Hkv, L, D]
  const void* cos;  // [positions, D/2]
  const void* sin;  // [positions, D/2]
  void* out;        // mode 0: [B, Hq, D] in the input dtype
  float* o_part;    // mode 1: [B * Hq, n_split, D] fp32 (final when n_split == 1)
  float* lse_part;  // mode 1: [B * Hq, n_split] fp32, natural log
  int Hq;
  int Hkv;
  int L;
  int G;          // Hq / Hkv
  int n_gchunk;   // G / GT
  int n_split;    // partial slots per row (1: each unit whole in one CTA, outputs final)
  int n_units;    // B * Hkv * n_gchunk
  int cpu;        // chunks per unit = ceil(L / CK)
  long long total_chunks;  // n_units * cpu
  long long q_pos;
  long long kv_pos_offset;
  float scale_log2;
  int mode;  // 0: final output in dtype (n_split == 1); 1: fp32 partials
  // Per-sequence cache lengths (varlen != 0), prepared by decode_prep_kernel on the same stream:
  // pre[b] is the flattened chunk index where sequence b's units start (pre[B] = total), lenq[b]
  // = {keys attended, query position}. Partials go to fragment slots: fragment (unit u, CTA c)
  // writes rows (u + c) * GT + gg of o_part / lse_part (u + c grows along the flattened order,
  // so every fragment has its own slot).
  const long long* pre;
  const int2* lenq;
  const int* vl_whole;  // set by the prep kernel: whole units round-robin, final rows to out
  int B;
  int ub;  // units per sequence: Hkv * n_gchunk
  int varlen;
  // Split walk with the merge inside the split kernel (tensor-core decode, fused_merge != 0):
  // after writing a partial, a fragment takes a ticket on unit_cnt[unit]; the fragment that
  // completes the unit merges its rows into fin_out (fin_kind 0 fp16, 1 bf16, 2 fp32 with the
  // natural-log lse in fin_lse). unit_cnt[DECODE_CNT_DONE] counts finished CTAs; the last one
  // zeroes every counter, so each call leaves the counters as it found them (zero).
  int* unit_cnt;
  int fused_merge;
  void* fin_out;
  int fin_kind;
  float* fin_lse;
  // Split walk (n_split > 1, no per-sequence lengths): chunks charged to the start of every unit
  // when the CTAs' ranges are cut (0: equal ranges of the real chunks). A CTA whose range
  // reaches into a second unit finishes, combines and restarts; charging that restart as
  // frag_pen chunks gives such CTAs fewer real chunks, so they end with the others.
  int frag_pen;
};

// Workspace of the split walk: the ticket counters first (fixed size, so that calls of any
// shape find them in the same place), then the partials.
constexpr int DECODE_CNT_BYTES = 16384;
constexpr int DECODE_CNT_DONE = DECODE_CNT_BYTES / 4 - 1;  // units with a fused merge: < this

// Fewest chunks a CTA takes in the per-sequence-length walk: one-chunk fragments would cost
// more in partials than they balance.
constexpr int DECODE_VARLEN_MIN_PER = 2;

// One fragment of a CTA's work: keys [kbeg, kend) of one unit, written to partial slot `slot`,
// with the query at position qpos.
struct DecodeFrag {
  int unit, kbeg, kend, slot;
  bool last;  // the unit's last fragment
  long long qpos;
};

// The CTA's work, walked identically by its producer and consumers. With one slot per row, whole
// units are dealt round-robin. Otherwise the flattened (unit, chunk) sequence is cut into equal
// contiguous ranges, one per CTA, and each range into per-unit fragments; a unit's fragments go
// to consecutive CTAs, the first of them writing slot 0. The cut is made on a virtual sequence
// in which unit u takes positions [u (cpu + P), (u + 1)(cpu + P)), its first P = frag_pen
// positions standing for the cost of a fragment's start and the rest for its cpu chunks; with
// P = 0 per-CTA work differs by at most one chunk, whatever the unit count.
struct DecodeWalk {
  long long cur, hi;
  long long per;  // per-sequence lengths: chunks per CTA
  int b;          // per-sequence lengths: the sequence holding chunk `cur`
  bool whole;     // per-sequence lengths: whole units round-robin (no partials)
  // Chunks per CTA of the per-sequence-length walk; decode_merge_varlen_kernel uses the same.
  __device__ __forceinline__ static long long varlen_per(long long total, long long grid) {
    const long long per = (total + grid - 1) / grid;
    return per > DECODE_VARLEN_MIN_PER ? per : DECODE_VARLEN_MIN_PER;
  }
  __device__ __forceinline__ void init(const DecodeParams& p) {
    if (p.varlen) {
      whole = *p.vl_whole != 0;
      if (whole) {
        cur = blockIdx.x;
        hi = p.n_units;
        return;
      }
      // Equal ranges of the flattened chunks that are actually present (pre[B] of them).
      const long long total = p.pre[p.B];
      per = varlen_per(total, gridDim.x);
      cur = static_cast<long long>(blockIdx.x) * per;
      hi = min(total, cur + per);
      int lo = 0, up = p.B;  // pre[lo] <= cur < pre[up]
      if (cur < hi)
        while (up - lo > 1) {
          const int mid = (lo + up) >> 1;
          if (p.pre[mid] <= cur) lo = mid; else up = mid;
        }
      b = lo;
      return;
    }
    if (p.n_split == 1) {
      cur = blockIdx.x;
      hi = p.n_units;
    } else {
      const long long vt = vtotal(p);
      cur = static_cast<long long>(blockIdx.x) * vt / gridDim.x;
      hi = static_cast<long long>(blockIdx.x + 1) * vt / gridDim.x;
    }
  }
  // Length of the virtual sequence the split walk cuts.
  __device__ __forceinline__ static long long vtotal(const DecodeParams& p) {
    return static_cast<long long>(p.n_units) * (p.cpu + p.frag_pen);
  }
  // CTA whose range holds global chunk x (of the real sequence).
  __device__ __forceinline__ static int cta_of(const DecodeParams& p, long long x) {
    const long long G = gridDim.x;
    const long long vt = vtotal(p);
    const long long u = x / p.cpu;
    const long long v = u * (p.cpu + p.frag_pen) + p.frag_pen + (x - u * p.cpu);
    long long c = v * G / vt;
    if ((c + 1) * vt / G <= v) ++c;
    return static_cast<int>(c);
  }
  __device__ __forceinline__ bool next(const DecodeParams& p, int CK, DecodeFrag& f) {
    if (cur >= hi) return false;
    if (p.varlen && whole) {
      const int2 lq = p.lenq[cur / p.ub];
      f.unit = static_cast<int>(cur);
      f.kbeg = 0;
      f.kend = lq.x;
      f.slot = -1;  // final rows, written to out
      f.last = true;
      f.qpos = lq.y;
      cur += gridDim.x;
      return true;
    }
    if (p.varlen) {
      while (p.pre[b + 1] <= cur) ++b;  // every sequence has at least one chunk per unit
      const long long base = p.pre[b];
      const long long nb = (p.pre[b + 1] - base) / p.ub;  // chunks per unit of sequence b
      const long long ui = (cur - base) / nb;
      const long long ub = base + ui * nb;
      const long long e = min(hi, ub + nb);
      const int2 lq = p.lenq[b];
      f.unit = b * p.ub + static_cast<int>(ui);
      f.kbeg = static_cast<int>(cur - ub) * CK;
      f.kend = min(lq.x, static_cast<int>(e - ub) * CK);
      if (f.kend < f.kbeg) f.kend = f.kbeg;  // an empty sequence: one fragment with no keys
      f.slot = f.unit + static_cast<int>(blockIdx.x);
      f.last = (e == ub + nb);
      f.qpos = lq.y;
      cur = e;
      return true;
    }
    f.qpos = p.q_pos;
    if (p.n_split == 1) {
      f.unit = static_cast<int>(cur);
      f.kbeg = 0;
      f.kend = p.L;
      f.slot = 0;
      f.last = true;
      cur += gridDim.x;
      return true;
    }
    // Virtual positions [cur, hi): a range holding only a unit's start positions is skipped.
    const long long span = p.cpu + p.frag_pen;
    while (cur < hi) {
      const long long u = cur / span;
      const long long vb = u * span + p.frag_pen;  // the unit's first chunk
      const long long e = min(hi, (u + 1) * span);
      const long long c0 = cur > vb ? cur - vb : 0;
      const long long c1 = e > vb ? e - vb : 0;
      cur = e;
      if (c1 <= c0) continue;
      f.unit = static_cast<int>(u);
      f.kbeg = static_cast<int>(c0) * CK;
      f.kend = min(p.L, static_cast<int>(c1) * CK);
      f.slot = static_cast<int>(blockIdx.x) - cta_of(p, u * p.cpu);
      f.last = (c1 == p.cpu);
      return true;
    }
    return false;
  }
};

template <int D, int GT>
struct DecodeShape {
  // Each lane takes PPL half-split chunk pairs (2 x 8 elements each) of a key row; a single
  // head per unit leaves room in registers for two pairs, which halves the lanes per row.
  static constexpr int PPL = (GT >= 2 || D < 32) ? 1 : 2;
  static constexpr int LPR = (D / 16) / PPL;     // lanes per key row
  static constexpr int KPW = 32 / LPR;           // keys per warp step
  // Consumer warps: seven for four heads per unit (their ~220 registers allow two warps per
  // SMSP, one CTA per SM, and the producer is the eighth warp), four otherwise (two or three
  // CTAs per SM).
  static constexpr int NW = (GT >= 4) ? 7 : 4;
  // K and V stages are TMA tiles of SPAN-byte row blocks with the matching swizzle, the cos and
  // sin rows tiles of TSPAN-byte blocks; every tile starts on a 1024-byte boundary (swizzled)
  // or a 128-byte one (16-byte table rows, unswizzled).
  static constexpr int SPAN = (2 * D >= 128) ? 128 : 2 * D;
  static constexpr int NBLK = 2 * D / SPAN;
  static constexpr int TSPAN = (D >= 128) ? 128 : D;
  static constexpr int TBLK = D / TSPAN;
  static constexpr int ALIGN_ROWS_K = 1024 / SPAN;
  static constexpr int ALIGN_ROWS_T = (TSPAN >= 32) ? 1024 / TSPAN : 128 / TSPAN;
  static constexpr int ALIGN_ROWS = ALIGN_ROWS_K > ALIGN_ROWS_T ? ALIGN_ROWS_K : ALIGN_ROWS_T;
  static constexpr int CK_BASE = cx_lcm(NW * KPW, ALIGN_ROWS);
  static constexpr int CK_TARGET = 4096 / D;     // ~8 KB of K per stage
  static constexpr int CK = CK_BASE * ((CK_TARGET / CK_BASE) > 1 ? (CK_TARGET / CK_BASE) : 1);
  static constexpr int ROWB = 2 * D;        // bytes per K / V row
  static constexpr int TABB = D;            // bytes per cos / sin row (D/2 16-bit values)
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = CK * ROWB;
  static constexpr int OFF_C = 2 * CK * ROWB;
  static constexpr int OFF_S = OFF_C + CK * TABB;
  static constexpr int STAGE = ((OFF_S + CK * TABB + 1023) / 1024) * 1024;
  static constexpr int STAGE_TX = 2 * CK * ROWB + 2 * CK * TABB;  // bytes landing per stage
  static constexpr int NSTG = (3 * STAGE <= 200 * 1024) ? 3 : 2;
  static constexpr int STEPS = CK / (NW * KPW);  // steps per warp per chunk
  // Per-item header ring (2 entries): the item's GT query rows, then the cos and sin rows at
  // the query position, copied by the producer like the KV chunks.
  static constexpr int NHDR = 2;
  static constexpr int HDR_Q = GT * ROWB;
  static constexpr int HDR = ((HDR_Q + 2 * TABB + 127) / 128) * 128;
  static constexpr int OFF_HDR = NSTG * STAGE;
  static constexpr int OFF_BAR = OFF_HDR + NHDR * HDR;  // full[NSTG], empty[NSTG], merge[2],
                                                        // hfull[NHDR], hempty[NHDR], flag
  static constexpr int N_BAR = 2 * NSTG + 2 + 2 * NHDR;
  static constexpr int OFF_MERGE = OFF_BAR + 8 * N_BAR + 16;
  static constexpr int MERGE_BYTES = NW * GT * (D + 2) * 4;
  static constexpr int SMEM_BYTES = OFF_MERGE + MERGE_BYTES + 1024;  // + alignment slack
  static constexpr int NTHREADS = 32 * (NW + 1);
  static constexpr int NCONS = 32 * NW;          // consumer threads
  // Lane layout: (key slot, lane sub-index) chosen so that the 8 lanes of every quarter-warp
  // read 16-byte chunks of swizzled rows in 8 distinct bank groups. SUBMASK: lane bits that
  // differ between the lanes of one key row; KEYMASK: bits that differ between key slots.
  static constexpr int SUBMASK = (LPR <= 4) ? ((LPR - 1) << 3) : ((LPR == 8) ? 28 : 30);
  static constexpr int KEYMASK = 31 & ~SUBMASK;
  static_assert(STEPS >= 1 && CK % (NW * KPW) == 0 && CK <= 256, "chunk geometry");
  static_assert(CK % ALIGN_ROWS == 0, "tile alignment");
  static_assert((CK / NW) % (KPW < 8 ? KPW : 8) == 0, "key groups start on swizzle rows");
};

// (key slot, sub-index) of a consumer lane for LPR lanes per key row (see SUBMASK).
template <int LPR>
__device__ __forceinline__ void decode_lane_map(int lane, int& kg, int& sub) {
  if constexpr (LPR <= 4) {
    kg = (lane / (8 * LPR)) * 8 + (lane % 8);
    sub = (lane / 8) % LPR;
  } else if constexpr (LPR == 8) {
    kg = lane % 4;
    sub = (lane / 8) + 4 * ((lane / 4) % 2);
  } else {
    kg = lane % 2;
    sub = ((lane / 8) % 2) + 2 * ((lane / 2) % 4) + 8 * (lane / 16);
  }
}

template <int D, bool BF16, int GT>
// Resident CTAs per SM: three for one query head per unit (the shared-memory loads of the key
// rows are the latency to hide, so more warps per SM pay), two for two heads, one for four.
__global__ void __launch_bounds__(DecodeShape<D, GT>::NTHREADS, (GT == 1) ? 3 : ((GT == 2) ? 2 : 1))
    decode_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                  const __grid_constant__ CUtensorMap tm_cos, const __grid_constant__ CUtensorMap tm_sin,
                  const DecodeParams p) {
  static_assert(DecodeShape<D, GT>::NTHREADS <= 256 || GT < 4, "two warps per SMSP at most");
  using S = DecodeShape<D, GT>;
  constexpr int LPR = S::LPR, KPW = S::KPW, NSTG = S::NSTG, CK = S::CK, HALF = D / 2;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t sbase = (raw_u32 + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - raw_u32);
  auto FULL = [&](int s) { return sbase + S::OFF_BAR + 8u * static_cast<uint32_t>(s); };
  auto EMPTY = [&](int s) { return sbase + S::OFF_BAR + 8u * static_cast<uint32_t>(NSTG + s); };
  auto MERGE = [&](int i) { return sbase + S::OFF_BAR + 8u * static_cast<uint32_t>(2 * NSTG + i); };
  auto HFULL = [&](int i) { return sbase + S::OFF_BAR + 8u * static_cast<uint32_t>(2 * NSTG + 2 + i); };
  auto HEMPTY = [&](int i) {
    return sbase + S::OFF_BAR + 8u * static_cast<uint32_t>(2 * NSTG + 2 + S::NHDR + i);
  };
  volatile int* failed = reinterpret_cast<volatile int*>(sgen + S::OFF_BAR + 8 * S::N_BAR);
  float* sm_m = reinterpret_cast<float*>(sgen + S::OFF_MERGE);      // [NW][GT]
  float* sm_l = sm_m + S::NW * GT;                                   // [NW][GT]
  float* sm_acc = sm_l + S::NW * GT;                                 // [NW][GT][D]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
#ifdef DU_TRACE
  // Debug-only timeline of the even CTAs below 148 (globaltimer ns): start, set-up done, first
  // chunk landed (consumer warp 0), end.
  auto trace_ev = [&](int e) {
    if ((blockIdx.x & 1) == 0 && blockIdx.x < 148)
      g_du_trace[e * 74 + blockIdx.x / 2] = static_cast<long long>(globaltimer());
  };
  if (threadIdx.x == 0) trace_ev(0);
#endif
  // The merge launched after this kernel may start its launch now; it waits for our completion.
  if (threadIdx.x == 0) griddep_launch_dependents();
  const uint8_t* cosb = static_cast<const uint8_t*>(p.cos);
  const uint8_t* sinb = static_cast<const uint8_t*>(p.sin);
  // Item header: query rows of the GT heads and the cos / sin rows at the query position, into
  // header slot hs (producer thread).
  auto issue_header = [&](const DecodeFrag& f, int hs) {
    const int gch = f.unit % p.n_gchunk;
    const int bk = f.unit / p.n_gchunk;  // b * Hkv + kvh
    const int b = bk / p.Hkv;
    const int h0 = (bk - b * p.Hkv) * p.G + gch * GT;
    const uint32_t hd = sbase + S::OFF_HDR + hs * S::HDR;
    const size_t trow = static_cast<size_t>(f.qpos) * S::TABB;
    mbar_expect_tx(HFULL(hs), static_cast<uint32_t>(S::HDR_Q + 2 * S::TABB));
    bulk_load(hd, static_cast<const uint8_t*>(p.q) + (static_cast<size_t>(b) * p.Hq + h0) * S::ROWB,
              S::HDR_Q, HFULL(hs));
    bulk_load(hd + S::HDR_Q, cosb + trow, S::TABB, HFULL(hs));
    bulk_load(hd + S::HDR_Q + S::TABB, sinb + trow, S::TABB, HFULL(hs));
  };
  // Chunk c0 of unit bk into ring stage s (producer thread). Whole boxes always land (rows past
  // the cache or the tables are zero-filled and masked by the consumers), so every stage
  // completes the same byte count.
  auto issue_chunk = [&](int bk, int c0, int s) {
    const int tpos = static_cast<int>(p.kv_pos_offset + c0);
    const uint32_t st = sbase + s * S::STAGE;
    mbar_expect_tx(FULL(s), static_cast<uint32_t>(S::STAGE_TX));
#pragma unroll
    for (int blk = 0; blk < S::NBLK; ++blk) {
      tma_load_3d(st + S::OFF_K + blk * CK * S::SPAN, &tm_k, FULL(s), blk * (S::SPAN / 2), c0, bk);
      tma_load_3d(st + S::OFF_V + blk * CK * S::SPAN, &tm_v, FULL(s), blk * (S::SPAN / 2), c0, bk);
    }
#pragma unroll
    for (int tb = 0; tb < S::TBLK; ++tb) {
      tma_load_2d(st + S::OFF_C + tb * CK * S::TSPAN, &tm_cos, FULL(s), tb * (S::TSPAN / 2), tpos);
      tma_load_2d(st + S::OFF_S + tb * CK * S::TSPAN, &tm_sin, FULL(s), tb * (S::TSPAN / 2), tpos);
    }
  };
  // The producer thread initialises the barriers and, unless the lengths come from a preceding
  // kernel, issues the first item's header and first chunks before the CTA barrier, so that the
  // first loads overlap the set-up.
  int pre_g = 0;  // chunks issued before the barrier (all of the CTA's first item)
  if (warp == S::NW && lane == 0) {
    for (int s = 0; s < NSTG; ++s) {
      mbar_init(FULL(s), 1);
      mbar_init(EMPTY(s), S::NW);
    }
    mbar_init(MERGE(0), S::NCONS);  // the consumer threads, once per work item
    mbar_init(MERGE(1), S::NCONS);
    for (int i = 0; i < S::NHDR; ++i) {
      mbar_init(HFULL(i), 1);
      mbar_init(HEMPTY(i), S::NCONS);
    }
    *failed = 0;
    mbar_fence_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_cos);
    tma_prefetch_desc(&tm_sin);
    if (!p.varlen) {
      DecodeWalk w0;
      w0.init(p);
      DecodeFrag f0;
      if (w0.next(p, CK, f0)) {
        issue_header(f0, 0);
        for (int c0 = f0.kbeg; c0 < f0.kend && pre_g < NSTG; c0 += CK, ++pre_g)
          issue_chunk(f0.unit / p.n_gchunk, c0, pre_g);
      }
    }
  }
  __syncthreads();
  // Per-sequence lengths: the prep kernel (this launch's programmatic predecessor) has written
  // the chunk offsets and the appended cache rows once this returns.
  if (p.varlen) {
    griddep_wait();
    fence_proxy_async_global();  // the appended rows are read by TMA (async proxy)
  }

#ifdef DU_TRACE
  if (threadIdx.x == 0) trace_ev(1);
#endif

  if (warp == S::NW) {
    // ------------------------------------------------------------------ bulk-copy producer
    if (lane == 0) {
      int g = 0;  // chunk counter across items (ring stage / phase)
      bool ok = true;
      int it = 0;
      DecodeWalk walk;
      walk.init(p);
      DecodeFrag fr;
      for (; ok && walk.next(p, CK, fr); ++it) {
        const int bk = fr.unit / p.n_gchunk;  // b * Hkv + kvh
        const bool pre = !p.varlen && it == 0;  // header and first chunks already issued
        if (!pre) {
          const int hs = it % S::NHDR;
          if (it >= S::NHDR && !mbar_wait(HEMPTY(hs), ((it / S::NHDR) - 1) & 1, failed, 65)) {
            ok = false;
            break;
          }
          issue_header(fr, hs);
        }
        for (int c0 = fr.kbeg; c0 < fr.kend; c0 += CK, ++g) {
          if (pre && g < pre_g) continue;
          const int s = g % NSTG;
          if (g >= NSTG && !mbar_wait(EMPTY(s), ((g / NSTG) - 1) & 1, failed, 60)) {
            ok = false;
            break;
          }
          issue_chunk(bk, c0, s);
        }
      }
      // Drain: the last copies land before the CTA may exit.
      for (int j = (g > NSTG ? g - NSTG : 0); j < g; ++j) mbar_wait_drain(FULL(j % NSTG), (j / NSTG) & 1, 61);
      for (int j = (it > S::NHDR ? it - S::NHDR : 0); j < it; ++j)
        mbar_wait_drain(HFULL(j % S::NHDR), (j / S::NHDR) & 1, 66);
    }
    __syncwarp();
    return;
  }

  // -------------------------------------------------------------------- consumers (warps 0..3)
  constexpr int PPL = S::PPL;
  int kg, sub;  // key slot within a warp step; this lane's chunk pairs: sub * PPL + i, i < PPL
  decode_lane_map<LPR>(lane, kg, sub);
  int g = 0;
  bool ok = true;
  int it = 0;  // items processed by this CTA (merge-barrier phase)
  DecodeWalk walk;
  walk.init(p);
  DecodeFrag fr;
  for (; walk.next(p, CK, fr); ++it) {
    const int unit = fr.unit;
    const int split = fr.slot;
    const int gch = unit % p.n_gchunk;
    const int bk = unit / p.n_gchunk;
    const int b = bk / p.Hkv;
    const int kvh = bk - b * p.Hkv;
    const int h0 = kvh * p.G + gch * GT;
    const int kbeg = fr.kbeg;
    const int kend = fr.kend;

    // Rotated, pre-scaled query pairs (log2 domain) for this lane's chunk pairs, from the header.
    uint64_t q1[GT][PPL][4], q2[GT][PPL][4];
    {
      const int hs = it % S::NHDR;
      ok = mbar_wait(HFULL(hs), (it / S::NHDR) & 1, failed, 67);
      if (!__all_sync(0xffffffffu, ok)) break;
      const uint32_t hd = sbase + S::OFF_HDR + hs * S::HDR;
#pragma unroll
      for (int i = 0; i < PPL; ++i) {
        const int c = sub * PPL + i;
        const uint4 cv = ld_shared_v4(hd + S::HDR_Q + c * 16);
        const uint4 sv = ld_shared_v4(hd + S::HDR_Q + S::TABB + c * 16);
        const uint32_t ca[4] = {cv.x, cv.y, cv.z, cv.w};
        const uint32_t sa[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int gg = 0; gg < GT; ++gg) {
          const uint4 x1 = ld_shared_v4(hd + gg * S::ROWB + c * 16);
          const uint4 x2 = ld_shared_v4(hd + gg * S::ROWB + HALF * 2 + c * 16);
          const uint32_t xa[4] = {x1.x, x1.y, x1.z, x1.w};
          const uint32_t xb[4] = {x2.x, x2.y, x2.z, x2.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 lo = unpack2<BF16>(xa[e]);
            const float2 hi = unpack2<BF16>(xb[e]);
            const float2 cc = unpack2<BF16>(ca[e]);
            const float2 ss = unpack2<BF16>(sa[e]);
            const float sc = p.scale_log2;
            q1[gg][i][e] = f2((lo.x * cc.x - hi.x * ss.x) * sc, (lo.y * cc.y - hi.y * ss.y) * sc);
            q2[gg][i][e] = f2((hi.x * cc.x + lo.x * ss.x) * sc, (hi.y * cc.y + lo.y * ss.y) * sc);
          }
        }
      }
      mbar_arrive(HEMPTY(hs));  // header consumed: the producer may reuse the entry
    }

    float m[GT], l[GT];
    uint64_t acc[GT][PPL][8];  // f32 pairs: [0,4) first-half chunk, [4,8) second-half chunk
#pragma unroll
    for (int gg = 0; gg < GT; ++gg) {
      m[gg] = -1e30f;
      l[gg] = 0.f;
#pragma unroll
      for (int i = 0; i < PPL; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[gg][i][e] = f2(0.f, 0.f);
    }

    for (int c0 = kbeg; ok && c0 < kend; c0 += CK, ++g) {
      const int s = g % NSTG;
      ok = mbar_wait(FULL(s), (g / NSTG) & 1, failed, 62);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
#ifdef DU_TRACE
      if (threadIdx.x == 0 && g == 0) trace_ev(2);
#endif
      const int n = min(CK, kend - c0);
      const uint32_t st = sbase + s * S::STAGE;
      float sc[S::STEPS][GT];
      uint4 vx[S::STEPS][PPL][2];
#pragma unroll
      for (int u = 0; u < S::STEPS; ++u) {
        const int key = warp * (CK / S::NW) + u * KPW + kg;  // row within the chunk
        const bool valid = key < n;
        uint64_t dot[GT];
#pragma unroll
        for (int gg = 0; gg < GT; ++gg) dot[gg] = f2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < PPL; ++i) {
          const int c = sub * PPL + i;
          uint4 k1 = make_uint4(0, 0, 0, 0), k2 = k1, cv = k1, sv = k1;
          vx[u][i][0] = vx[u][i][1] = k1;
          if (valid) {
            const uint32_t o1 = swz_chunk_offset<S::SPAN>(CK, key, c);
            const uint32_t o2 = swz_chunk_offset<S::SPAN>(CK, key, c + D / 16);
            const uint32_t ot = swz_chunk_offset<S::TSPAN>(CK, key, c);
            k1 = ld_shared_v4(st + S::OFF_K + o1);
            k2 = ld_shared_v4(st + S::OFF_K + o2);
            vx[u][i][0] = ld_shared_v4(st + S::OFF_V + o1);
            vx[u][i][1] = ld_shared_v4(st + S::OFF_V + o2);
            cv = ld_shared_v4(st + S::OFF_C + ot);
            sv = ld_shared_v4(st + S::OFF_S + ot);
          }
          const uint32_t ka[4] = {k1.x, k1.y, k1.z, k1.w};
          const uint32_t kb[4] = {k2.x, k2.y, k2.z, k2.w};
          const uint32_t ca[4] = {cv.x, cv.y, cv.z, cv.w};
          const uint32_t sa[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            // Rotate two elements per instruction in the input dtype, then widen to fp32.
            uint32_t r1, r2;
            rope_rotate2<BF16>(ka[e], kb[e], ca[e], sa[e], r1, r2);
            const uint64_t k1f = widen2<BF16>(r1);
            const uint64_t k2f = widen2<BF16>(r2);
#pragma unroll
            for (int gg = 0; gg < GT; ++gg)
              dot[gg] = f2_fma(q2[gg][i][e], k2f, f2_fma(q1[gg][i][e], k1f, dot[gg]));
          }
        }
#pragma unroll
        for (int gg = 0; gg < GT; ++gg) {
          const float2 dd = f2_split(dot[gg]);
          float d = dd.x + dd.y;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1)
            if (S::SUBMASK & o) d += __shfl_xor_sync(0xffffffffu, d, o);
          sc[u][gg] = valid ? d : -INFINITY;
        }
      }
      // The stage's shared memory has been read into registers: release it to the producer.
      __syncwarp();
      if (lane == 0) mbar_arrive(EMPTY(s));
#pragma unroll
      for (int u = 0; u < S::STEPS; ++u) {
        uint64_t vf[PPL][8];
#pragma unroll
        for (int i = 0; i < PPL; ++i) {
          const uint32_t va[4] = {vx[u][i][0].x, vx[u][i][0].y, vx[u][i][0].z, vx[u][i][0].w};
          const uint32_t vb[4] = {vx[u][i][1].x, vx[u][i][1].y, vx[u][i][1].z, vx[u][i][1].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            vf[i][e] = widen2<BF16>(va[e]);
            vf[i][4 + e] = widen2<BF16>(vb[e]);
          }
        }
#pragma unroll
        for (int gg = 0; gg < GT; ++gg) {
          const float sv_ = sc[u][gg];
          // Lazy rescale: move the reference max only when the score exceeds it by 2^8.
          if (sv_ > m[gg] + 8.0f) {
            const float alpha = ex2(m[gg] - sv_);
            const uint64_t a2 = f2(alpha, alpha);
            l[gg] *= alpha;
#pragma unroll
            for (int i = 0; i < PPL; ++i)
#pragma unroll
              for (int e = 0; e < 8; ++e) acc[gg][i][e] = f2_mul(acc[gg][i][e], a2);
            m[gg] = sv_;
          }
          const float pe = ex2(sv_ - m[gg]);
          l[gg] += pe;
          const uint64_t p2 = f2(pe, pe);
#pragma unroll
          for (int i = 0; i < PPL; ++i)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[gg][i][e] = f2_fma(p2, vf[i][e], acc[gg][i][e]);
        }
      }
    }
    if (!ok) break;

    // Merge the KPW key groups of the warp (butterfly over lanes with the same chunk pairs).
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      if (!(S::KEYMASK & o)) continue;
#pragma unroll
      for (int gg = 0; gg < GT; ++gg) {
        const float mo = __shfl_xor_sync(0xffffffffu, m[gg], o);
        const float lo = __shfl_xor_sync(0xffffffffu, l[gg], o);
        const float mn = fmaxf(m[gg], mo);
        const float wa = ex2(m[gg] - mn);
        const float wb = ex2(mo - mn);
        l[gg] = l[gg] * wa + lo * wb;
        const uint64_t wa2 = f2(wa, wa), wb2 = f2(wb, wb);
#pragma unroll
        for (int i = 0; i < PPL; ++i)
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float2 a = f2_split(acc[gg][i][e]);
            const uint64_t ao = f2(__shfl_xor_sync(0xffffffffu, a.x, o), __shfl_xor_sync(0xffffffffu, a.y, o));
            acc[gg][i][e] = f2_fma(ao, wb2, f2_mul(acc[gg][i][e], wa2));
          }
        m[gg] = mn;
      }
    }
    if (kg == 0) {
#pragma unroll
      for (int gg = 0; gg < GT; ++gg) {
        if (sub == 0) {
          sm_m[warp * GT + gg] = m[gg];
          sm_l[warp * GT + gg] = l[gg];
        }
        float* a = sm_acc + (warp * GT + gg) * D;
#pragma unroll
        for (int i = 0; i < PPL; ++i) {
          const int c = sub * PPL + i;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 x1 = f2_split(acc[gg][i][e]);
            const float2 x2 = f2_split(acc[gg][i][4 + e]);
            a[8 * c + 2 * e] = x1.x;
            a[8 * c + 2 * e + 1] = x1.y;
            a[HALF + 8 * c + 2 * e] = x2.x;
            a[HALF + 8 * c + 2 * e + 1] = x2.y;
          }
        }
      }
    }
    // Bounded barrier of the consumer warps (the producer warp keeps streaming).
    mbar_arrive(MERGE(0));
    ok = mbar_wait(MERGE(0), it & 1, failed, 63);
    if (!__all_sync(0xffffffffu, ok)) break;
    for (int idx = threadIdx.x; idx < GT * D; idx += S::NCONS) {
      const int gg = idx / D;
      const int d = idx - gg * D;
      float M = sm_m[gg];
#pragma unroll
      for (int w = 1; w < S::NW; ++w) M = fmaxf(M, sm_m[w * GT + gg]);
      float Lsum = 0.f, A = 0.f;
#pragma unroll
      for (int w = 0; w < S::NW; ++w) {
        const float wt = ex2(sm_m[w * GT + gg] - M);
        Lsum += sm_l[w * GT + gg] * wt;
        A += sm_acc[(w * GT + gg) * D + d] * wt;
      }
      const size_t row = static_cast<size_t>(b) * p.Hq + h0 + gg;
      const float val = (Lsum > 0.f) ? A / Lsum : 0.f;
      if (p.varlen && split >= 0) {
        const size_t fs = static_cast<size_t>(split) * GT + gg;  // fragment slot row
        p.o_part[fs * D + d] = val;
        if (d == 0) p.lse_part[fs] = (Lsum > 0.f) ? (M + lg2(Lsum)) * 0.69314718055994531f : -INFINITY;
      } else if (p.mode == 0 || split < 0) {
        if constexpr (BF16) {
          static_cast<__nv_bfloat16*>(p.out)[row * D + d] = __float2bfloat16_rn(val);
        } else {
          static_cast<__half*>(p.out)[row * D + d] = __float2half_rn(val);
        }
      } else {
        p.o_part[(row * p.n_split + split) * D + d] = val;
        if (d == 0)
          p.lse_part[row * p.n_split + split] =
              (Lsum > 0.f) ? (M + lg2(Lsum)) * 0.69314718055994531f : -INFINITY;
        // The unit's last fragment also marks the row's unused slots empty (weight 0).
        if (fr.last)
          for (int sl = split + 1; sl < p.n_split; ++sl) {
            p.o_part[(row * p.n_split + sl) * D + d] = 0.f;
            if (d == 0) p.lse_part[row * p.n_split + sl] = -INFINITY;
          }
      }
    }
    mbar_arrive(MERGE(1));  // merge area free for the next item
    ok = mbar_wait(MERGE(1), it & 1, failed, 64);
    if (!__all_sync(0xffffffffu, ok)) break;
  }
#ifdef DU_TRACE
  if (threadIdx.x == 0) trace_ev(5);
#endif
}

constexpr int MERGE_MAX_R = 4096;

// Body of the merges: one CTA of 128 threads combines the R partials of one row, partial r at
// lse[r * l_sr] and o[r * o_sr + d]; `w` is a shared array of at least R floats.
__device__ __forceinline__ void merge_row(const float* __restrict__ o, const float* __restrict__ lse,
                                          int R, int D, long long o_sr, long long l_sr, void* out,
                                          int out_kind, float* lse_out, long long row, float* w) {
  __shared__ float red[4];
  __shared__ float s_m, s_w;
  const int tid = threadIdx.x;
  float mx = -INFINITY;
  for (int r = tid; r < R; r += 128) {
    const float v = lse[r * l_sr];
    w[r] = v;
    mx = fmaxf(mx, v);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  if (tid == 0) s_m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  const float M = s_m;
  float ws = 0.f;
  for (int r = tid; r < R; r += 128) {
    const float e = (M == -INFINITY) ? 0.f : expf(w[r] - M);
    w[r] = e;
    ws += e;
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o);
  __syncthreads();
  if ((tid & 31) == 0) red[tid >> 5] = ws;
  __syncthreads();
  if (tid == 0) s_w = red[0] + red[1] + red[2] + red[3];
  __syncthreads();
  const float W = s_w;
  const float inv = (W > 0.f) ? 1.0f / W : 0.f;
  for (int d = tid; d < D; d += 128) {
    const float* src = o + d;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    int r = 0;
    for (; r + 4 <= R; r += 4) {
      a0 = fmaf(w[r], src[r * o_sr], a0);
      a1 = fmaf(w[r + 1], src[(r + 1) * o_sr], a1);
      a2 = fmaf(w[r + 2], src[(r + 2) * o_sr], a2);
      a3 = fmaf(w[r + 3], src[(r + 3) * o_sr], a3);
    }
    for (; r < R; ++r) a0 = fmaf(w[r], src[r * o_sr], a0);
    const float A = ((a0 + a1) + (a2 + a3)) * inv;
    const long long oi = row * D + d;
    if (out_kind == 0) {
      static_cast<__half*>(out)[oi] = __float2half_rn(A);
    } else if (out_kind == 1) {
      static_cast<__nv_bfloat16*>(out)[oi] = __float2bfloat16_rn(A);
    } else {
      static_cast<float*>(out)[oi] = A;
    }
  }
  if (lse_out != nullptr && tid == 0) lse_out[row] = (W > 0.f) ? M + logf(W) : -INFINITY;
}

// LSE-weighted merge of R partials per row: lse = log(sum_r exp(lse_r)),
// out = sum_r exp(lse_r - lse) * o_r. Rows whose partials all have lse = -inf produce zeros and
// lse = -inf. out_kind: 0 fp16, 1 bf16, 2 fp32. One CTA per row: the R weights are computed in
// parallel into shared memory (R <= MERGE_MAX_R), then each thread sums its columns with
// independent loads.
__global__ void __launch_bounds__(128) merge_kernel(const float* __restrict__ o_parts,
                                                    const float* __restrict__ lse_parts, int R,
                                                    int D, long long o_sr, long long o_srow,
                                                    long long l_sr, long long l_srow, void* out,
                                                    int out_kind, float* lse_out) {
  __shared__ float w[MERGE_MAX_R];
  griddep_wait();  // the partials' producer (when launched as its dependent) has completed
  const long long row = blockIdx.x;
  merge_row(o_parts + row * o_srow, lse_parts + row * l_srow, R, D, o_sr, l_sr, out, out_kind,
            lse_out, row, w);
}

// ------------------------------------------------------------------------------------------
// Per-sequence cache lengths with the new token's K/V appended (decode over a KV cache as a
// generation loop holds it).
// ------------------------------------------------------------------------------------------
struct DecodePrepParams {
  const int* seqlens;  // [B] tokens in each sequence's cache before this step
  const void* k_new;   // [B, Hkv, D] the new token's key / value, or nullptr (no append)
  const void* v_new;
  void* k_cache;       // [B, Hkv, L, D]
  void* v_cache;
  long long* pre;      // out [B + 1]: flattened chunk offsets (DecodeParams::pre)
  int2* lenq;          // out [B]: {keys attended, query position}
  int* vl_whole;       // out: 1 = the split kernel takes whole units round-robin
  int B, Hkv, L, D, CK, ub, append;
  int whole_ok;        // the unit count allows whole units (decided on the host)
  int grid;            // CTAs of the split kernel
  long long rope_positions;
};

// A cache length s is usable when 0 <= s, the append fits (s + append <= L) and the tables hold
// the query position s. Anything else is recorded (status code 6) and the sequence is treated
// as empty: no append, no keys, zero output.
__device__ __forceinline__ bool decode_len_ok(const DecodePrepParams& p, int s) {
  return s >= 0 && s + p.append <= p.L && static_cast<long long>(s) < p.rope_positions;
}

// CTA 0 scans the per-sequence chunk counts into pre / lenq; every CTA copies its share of the
// new K / V rows (16 bytes per thread step) into row seqlens[b] of the caches.
__global__ void __launch_bounds__(256) decode_prep_kernel(const DecodePrepParams p) {
  griddep_launch_dependents();  // the split kernel may launch; it waits for this grid's writes
  __shared__ long long warp_tot[8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (blockIdx.x == 0) {
    long long carry = 0;
    for (int base = 0; base < p.B; base += 256) {
      const int b = base + tid;
      long long x = 0;
      if (b < p.B) {
        const int s = p.seqlens[b];
        const bool ok = decode_len_ok(p, s);
        if (!ok) record_error(6u, static_cast<unsigned>(b), static_cast<unsigned>(s));
        const int len = ok ? s + p.append : 0;
        p.lenq[b] = make_int2(len, ok ? s : 0);
        const int nch = (len + p.CK - 1) / p.CK;
        x = static_cast<long long>(p.ub) * (nch > 1 ? nch : 1);
      }
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const long long y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (lane == 31) warp_tot[warp] = x;
      __syncthreads();
      long long before = carry, tot = 0;
#pragma unroll
      for (int w2 = 0; w2 < 8; ++w2) {
        if (w2 < warp) before += warp_tot[w2];
        tot += warp_tot[w2];
      }
      if (b < p.B) p.pre[b + 1] = before + x;
      carry += tot;
      __syncthreads();
    }
    if (tid == 0) p.pre[0] = 0;
    // Whole units round-robin (no partials, no merge) when their load is even: the busiest CTA
    // carries at most 5/4 of the average over the CTAs that get a unit (lengths near uniform);
    // otherwise the length-balanced split walk.
    __syncthreads();
    int whole = 0;
    if (p.whole_ok) {
      const long long units = static_cast<long long>(p.B) * p.ub;
      long long mk = 0;
      for (int c = tid; c < p.grid; c += blockDim.x) {
        long long sum = 0;
        for (long long u = c; u < units; u += p.grid) {
          const int nch = (p.lenq[u / p.ub].x + p.CK - 1) / p.CK;
          sum += nch > 1 ? nch : 1;
        }
        mk = sum > mk ? sum : mk;
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        const long long y = __shfl_xor_sync(0xffffffffu, mk, o);
        mk = y > mk ? y : mk;
      }
      if (lane == 0) warp_tot[warp] = mk;
      __syncthreads();
      if (tid == 0) {
        for (int w2 = 0; w2 < 8; ++w2) mk = warp_tot[w2] > mk ? warp_tot[w2] : mk;
        const long long active = units < p.grid ? units : p.grid;
        whole = (4 * mk * active <= 5 * p.pre[p.B]) ? 1 : 0;
      }
    }
    if (tid == 0) *p.vl_whole = whole;
  }
  if (p.append) {
    const int cpr = p.D / 8;  // 16-byte pieces per row
    const long long n = static_cast<long long>(p.B) * p.Hkv * cpr;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + tid; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
      const long long r = i / cpr;  // b * Hkv + kv head
      const int c = static_cast<int>(i - r * cpr);
      const int s = p.seqlens[r / p.Hkv];
      if (!decode_len_ok(p, s)) continue;
      const long long dst = (r * p.L + s) * cpr + c;
      reinterpret_cast<uint4*>(p.k_cache)[dst] = reinterpret_cast<const uint4*>(p.k_new)[i];
      reinterpret_cast<uint4*>(p.v_cache)[dst] = reinterpret_cast<const uint4*>(p.v_new)[i];
    }
  }
}

// Merge of the fragment slots of the per-sequence-length walk: one CTA per (b, query head).
// The row's unit u spans the CTAs c0..c1 of the walk (same chunk offsets and chunks per CTA as
// DecodeWalk); fragment (u, c) wrote row (u + c) * GT + gg.
__global__ void __launch_bounds__(128) decode_merge_varlen_kernel(
    const float* __restrict__ o_parts, const float* __restrict__ lse_parts,
    const long long* __restrict__ pre, const int* __restrict__ vl_whole, int Hq, int Hkv, int GT,
    int ub, int B, int D, int split_grid, void* out, int out_kind) {
  __shared__ float w[MERGE_MAX_R];
  griddep_wait();  // the split kernel has completed
  if (*vl_whole) return;  // whole units: the split kernel wrote the final rows
  const long long row = blockIdx.x;  // b * Hq + h
  const int b = static_cast<int>(row / Hq);
  const int h = static_cast<int>(row - static_cast<long long>(b) * Hq);
  const int G = Hq / Hkv;
  const int kvh = h / G;
  const int gch = (h - kvh * G) / GT;
  const int gg = h - kvh * G - gch * GT;
  const int ui = kvh * (G / GT) + gch;  // unit within the sequence
  const long long base = pre[b];
  const long long nb = (pre[b + 1] - base) / ub;
  const long long start = base + ui * nb;
  const long long per = DecodeWalk::varlen_per(pre[B], split_grid);
  const long long c0 = start / per;
  const long long c1 = (start + nb - 1) / per;
  const long long u = static_cast<long long>(b) * ub + ui;
  const long long slot0 = (u + c0) * GT + gg;
  merge_row(o_parts + slot0 * D, lse_parts + slot0, static_cast<int>(c1 - c0 + 1), D,
            static_cast<long long>(GT) * D, GT, out, out_kind, nullptr, row, w);
}

}  // namespace du
