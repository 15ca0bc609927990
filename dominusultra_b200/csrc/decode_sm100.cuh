// Fused-RoPE decode for sm_100a: split-KV streaming kernel plus an LSE-weighted merge.
//
// One new query token per (batch, query head) attends over a KV cache, rotating the query at
// position q_pos and key j at position kv_pos_offset + j (reference: decode_kernel,
// dominus_ultra.py:288-413; query rotation :335-344, key rotation :381-395, online softmax
// :397-409). With q_pos = L and kv_pos_offset = 0 this is exactly the reference's semantics
// (the cache holds positions 0..L-1, the new token is at L and does not attend to itself).
//
// The kernel is HBM-bound, so it is laid out for streaming:
//  * a CTA owns one (b, kv head, group chunk) and one contiguous split of the cache, and
//    serves GT query heads of the GQA group at once, so each KV byte is read once per CTA;
//  * D/16 lanes share one key row; each lane streams two 16-byte chunks of K and of V
//    (elements [8c, 8c+8) and [D/2 + 8c, D/2 + 8c + 8)), which are exactly the half-split RoPE
//    partners, so the rotation needs no shuffles; loads are 128-bit and skip L1;
//  * scores are reduced across the D/16 lanes with xor-shuffles, the online softmax runs per
//    lane group in the log2 domain with one rescale per block of U keys, and the groups and
//    warps are merged at the end;
//  * with more than one split per row, each split writes an fp32 partial (out normalised over
//    the split, natural-log LSE) and merge_kernel combines them.
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
  float* o_part;    // mode 1: [B * Hq, n_split, D] fp32
  float* lse_part;  // mode 1: [B * Hq, n_split] fp32
  int Hq;
  int Hkv;
  int L;
  int G;          // Hq / Hkv
  int n_gchunk;   // G / GT
  int n_split;
  int keys_per_split;
  long long q_pos;
  long long kv_pos_offset;
  float scale_log2;
  int mode;  // 0: final output in dtype (n_split == 1); 1: fp32 partials
};

template <int D, bool BF16, int GT>
__global__ void __launch_bounds__(128) decode_split_kernel(const DecodeParams p) {
  constexpr int LPR = D / 16;      // lanes per key row
  constexpr int KPW = 32 / LPR;    // keys per warp step
  constexpr int U = (D >= 128 || GT >= 4) ? 2 : 4;  // steps per block (rows in flight)
  constexpr int NW = 4;
  constexpr int HALF = D / 2;

  __shared__ float sm_m[NW][GT];
  __shared__ float sm_l[NW][GT];
  __shared__ float sm_acc[NW][GT][D];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kg = lane / LPR;
  const int c = lane % LPR;
  const int unit = blockIdx.y;
  const int gch = unit % p.n_gchunk;
  const int bk = unit / p.n_gchunk;  // b * Hkv + kvh
  const int b = bk / p.Hkv;
  const int kvh = bk - b * p.Hkv;
  const int h0 = kvh * p.G + gch * GT;
  const int split = blockIdx.x;
  const int kbeg = split * p.keys_per_split;
  const int kend = min(p.L, kbeg + p.keys_per_split);

  const uint8_t* cosb = static_cast<const uint8_t*>(p.cos);
  const uint8_t* sinb = static_cast<const uint8_t*>(p.sin);

  // Rotated, pre-scaled query halves for this lane's 8 element pairs.
  float q1[GT][8], q2[GT][8];
  {
    const size_t trow = static_cast<size_t>(p.q_pos) * HALF * 2;
    const uint4 cv = ldg_v4(cosb + trow + c * 16);
    const uint4 sv = ldg_v4(sinb + trow + c * 16);
    const uint32_t ca[4] = {cv.x, cv.y, cv.z, cv.w};
    const uint32_t sa[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
    for (int g = 0; g < GT; ++g) {
      const uint8_t* qp =
          static_cast<const uint8_t*>(p.q) + (static_cast<size_t>(b) * p.Hq + h0 + g) * D * 2;
      const uint4 x1 = ldg_v4(qp + c * 16);
      const uint4 x2 = ldg_v4(qp + HALF * 2 + c * 16);
      const uint32_t xa[4] = {x1.x, x1.y, x1.z, x1.w};
      const uint32_t xb[4] = {x2.x, x2.y, x2.z, x2.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 lo = unpack2<BF16>(xa[i]);
        const float2 hi = unpack2<BF16>(xb[i]);
        const float2 cc = unpack2<BF16>(ca[i]);
        const float2 ss = unpack2<BF16>(sa[i]);
        q1[g][2 * i] = (lo.x * cc.x - hi.x * ss.x) * p.scale_log2;
        q1[g][2 * i + 1] = (lo.y * cc.y - hi.y * ss.y) * p.scale_log2;
        q2[g][2 * i] = (hi.x * cc.x + lo.x * ss.x) * p.scale_log2;
        q2[g][2 * i + 1] = (hi.y * cc.y + lo.y * ss.y) * p.scale_log2;
      }
    }
  }

  float m[GT], l[GT], acc[GT][16];
#pragma unroll
  for (int g = 0; g < GT; ++g) {
    m[g] = -1e30f;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[g][i] = 0.f;
  }

  const uint8_t* kb_ptr = static_cast<const uint8_t*>(p.k) + static_cast<size_t>(bk) * p.L * D * 2;
  const uint8_t* vb_ptr = static_cast<const uint8_t*>(p.v) + static_cast<size_t>(bk) * p.L * D * 2;

  for (int kb = kbeg + warp * KPW * U; kb < kend; kb += NW * KPW * U) {
    uint4 kx1[U], kx2[U], vx1[U], vx2[U], cvv[U], svv[U];
    bool valid[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int key = kb + u * KPW + kg;
      valid[u] = key < kend;
      if (valid[u]) {
        const size_t ro = static_cast<size_t>(key) * D * 2;
        kx1[u] = ldg_stream_v4(kb_ptr + ro + c * 16);
        kx2[u] = ldg_stream_v4(kb_ptr + ro + HALF * 2 + c * 16);
        vx1[u] = ldg_stream_v4(vb_ptr + ro + c * 16);
        vx2[u] = ldg_stream_v4(vb_ptr + ro + HALF * 2 + c * 16);
        const size_t trow = static_cast<size_t>(p.kv_pos_offset + key) * HALF * 2;
        cvv[u] = ldg_v4(cosb + trow + c * 16);
        svv[u] = ldg_v4(sinb + trow + c * 16);
      } else {
        kx1[u] = kx2[u] = vx1[u] = vx2[u] = cvv[u] = svv[u] = make_uint4(0, 0, 0, 0);
      }
    }
    float sc[U][GT];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t xa[4] = {kx1[u].x, kx1[u].y, kx1[u].z, kx1[u].w};
      const uint32_t xb[4] = {kx2[u].x, kx2[u].y, kx2[u].z, kx2[u].w};
      const uint32_t ca[4] = {cvv[u].x, cvv[u].y, cvv[u].z, cvv[u].w};
      const uint32_t sa[4] = {svv[u].x, svv[u].y, svv[u].z, svv[u].w};
      float k1[8], k2[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 lo = unpack2<BF16>(xa[i]);
        const float2 hi = unpack2<BF16>(xb[i]);
        const float2 cc = unpack2<BF16>(ca[i]);
        const float2 ss = unpack2<BF16>(sa[i]);
        k1[2 * i] = lo.x * cc.x - hi.x * ss.x;
        k1[2 * i + 1] = lo.y * cc.y - hi.y * ss.y;
        k2[2 * i] = hi.x * cc.x + lo.x * ss.x;
        k2[2 * i + 1] = hi.y * cc.y + lo.y * ss.y;
      }
#pragma unroll
      for (int g = 0; g < GT; ++g) {
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) d = fmaf(q1[g][i], k1[i], fmaf(q2[g][i], k2[i], d));
#pragma unroll
        for (int o = LPR / 2; o >= 1; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        sc[u][g] = valid[u] ? d : -INFINITY;
      }
    }
    float vf[U][16];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t va[4] = {vx1[u].x, vx1[u].y, vx1[u].z, vx1[u].w};
      const uint32_t vb[4] = {vx2[u].x, vx2[u].y, vx2[u].z, vx2[u].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = unpack2<BF16>(va[i]);
        const float2 bb = unpack2<BF16>(vb[i]);
        vf[u][2 * i] = a.x;
        vf[u][2 * i + 1] = a.y;
        vf[u][8 + 2 * i] = bb.x;
        vf[u][8 + 2 * i + 1] = bb.y;
      }
    }
#pragma unroll
    for (int g = 0; g < GT; ++g) {
      float mb = sc[0][g];
#pragma unroll
      for (int u = 1; u < U; ++u) mb = fmaxf(mb, sc[u][g]);
      const float mn = fmaxf(m[g], mb);
      const float alpha = ex2(m[g] - mn);
      l[g] *= alpha;
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[g][i] *= alpha;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float pe = ex2(sc[u][g] - mn);
        l[g] += pe;
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[g][i] = fmaf(pe, vf[u][i], acc[g][i]);
      }
      m[g] = mn;
    }
  }

  // Merge the KPW key groups of the warp (butterfly over lanes with the same chunk index).
#pragma unroll
  for (int o = LPR; o < 32; o <<= 1) {
#pragma unroll
    for (int g = 0; g < GT; ++g) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[g], o);
      const float lo = __shfl_xor_sync(0xffffffffu, l[g], o);
      const float mn = fmaxf(m[g], mo);
      const float wa = ex2(m[g] - mn);
      const float wb = ex2(mo - mn);
      l[g] = l[g] * wa + lo * wb;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float ao = __shfl_xor_sync(0xffffffffu, acc[g][i], o);
        acc[g][i] = acc[g][i] * wa + ao * wb;
      }
      m[g] = mn;
    }
  }
  if (kg == 0) {
#pragma unroll
    for (int g = 0; g < GT; ++g) {
      if (c == 0) {
        sm_m[warp][g] = m[g];
        sm_l[warp][g] = l[g];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        sm_acc[warp][g][8 * c + i] = acc[g][i];
        sm_acc[warp][g][HALF + 8 * c + i] = acc[g][8 + i];
      }
    }
  }
  __syncthreads();

  for (int idx = threadIdx.x; idx < GT * D; idx += blockDim.x) {
    const int g = idx / D;
    const int d = idx - g * D;
    float M = sm_m[0][g];
#pragma unroll
    for (int w = 1; w < NW; ++w) M = fmaxf(M, sm_m[w][g]);
    float Lsum = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float wt = ex2(sm_m[w][g] - M);
      Lsum += sm_l[w][g] * wt;
      A += sm_acc[w][g][d] * wt;
    }
    const size_t row = static_cast<size_t>(b) * p.Hq + h0 + g;
    const float val = (Lsum > 0.f) ? A / Lsum : 0.f;
    if (p.mode == 0) {
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
    }
  }
}

// LSE-weighted merge of R partials per row: lse = log(sum_r exp(lse_r)),
// out = sum_r exp(lse_r - lse) * o_r. Rows whose partials all have lse = -inf produce zeros and
// lse = -inf. out_kind: 0 fp16, 1 bf16, 2 fp32.
__global__ void __launch_bounds__(256) merge_kernel(const float* __restrict__ o_parts,
                                                    const float* __restrict__ lse_parts, int R,
                                                    int D, long long o_sr, long long o_srow,
                                                    long long l_sr, long long l_srow, void* out,
                                                    int out_kind, float* lse_out) {
  const long long row = blockIdx.x;
  float M = -INFINITY;
  for (int r = 0; r < R; ++r) M = fmaxf(M, lse_parts[r * l_sr + row * l_srow]);
  float W = 0.f;
  if (M != -INFINITY) {
    for (int r = 0; r < R; ++r) W += __expf(lse_parts[r * l_sr + row * l_srow] - M);
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float A = 0.f;
    if (M != -INFINITY) {
      for (int r = 0; r < R; ++r) {
        const float wt = __expf(lse_parts[r * l_sr + row * l_srow] - M);
        A = fmaf(wt, o_parts[r * o_sr + row * o_srow + d], A);
      }
      A /= W;
    }
    const long long oi = row * D + d;
    if (out_kind == 0) {
      static_cast<__half*>(out)[oi] = __float2half_rn(A);
    } else if (out_kind == 1) {
      static_cast<__nv_bfloat16*>(out)[oi] = __float2bfloat16_rn(A);
    } else {
      static_cast<float*>(out)[oi] = A;
    }
  }
  if (lse_out != nullptr && threadIdx.x == 0) lse_out[row] = (M == -INFINITY) ? M : M + logf(W);
}

}  // namespace du
