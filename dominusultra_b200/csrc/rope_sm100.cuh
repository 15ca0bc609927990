// Standalone half-split rotary embedding for sm_100a (reference rope.py:19-107, the `_rope_kernel`
// Triton program, and the rotation inside dominus_ultra.py:185-208 / :243-257).
//
//   forward  (i < D/2): y_i = x_i c_i - x_{i+D/2} s_i,   y_{i+D/2} = x_{i+D/2} c_i + x_i s_i
//   backward (the transpose): y_i = x_i c_i + x_{i+D/2} s_i, y_{i+D/2} = x_{i+D/2} c_i - x_i s_i
//
// with c_i = cos[pos, i], s_i = sin[pos, i] and, for row t of [B, H, T, D], pos = pos_offset + t
// for t < pos_split and pos_offset1 + (t - pos_split) beyond (two position segments: a rank of a
// context-parallel prefill holds two non-adjacent chunks of the sequence along T).
// The rotation runs in fp32 on 16-bit inputs and rounds once on output (the reference rounds
// the same products through its input dtype). The output is the input dtype, or fp16 for the
// attention operand path (rotated K feeding the fp16 tensor-core QK^T).
//
// Bandwidth-bound: one thread owns one 16-byte chunk of the first half and the matching chunk of
// the second half (8 + 8 elements), so a warp reads and writes whole rows with 16-byte accesses;
// the tables are small and stay in L2. Grid-stride loop over rows x D/16 chunks.
#pragma once

#include "du_ptx.cuh"

namespace du {

struct RopeParams {
  const void* x;      // [rows, D], rows = B * H * T
  const void* cos;    // [positions, D/2]
  const void* sin;    // [positions, D/2]
  void* out;          // [rows, D]
  long long rows;
  int T;
  int D;
  long long pos_offset;
  long long pos_split;    // rows t >= pos_split use the second segment (T: one segment)
  long long pos_offset1;
};

template <bool BF16, bool OUT_F16, bool BACKWARD>
__global__ void __launch_bounds__(256) rope_kernel(const RopeParams p) {
  griddep_launch_dependents();  // a prefill's attention launch may start its set-up now
  const int cpr = p.D / 16;  // chunk pairs per row
  const long long total = p.rows * cpr;
  const uint8_t* xb = static_cast<const uint8_t*>(p.x);
  const uint8_t* cb = static_cast<const uint8_t*>(p.cos);
  const uint8_t* sb = static_cast<const uint8_t*>(p.sin);
  uint8_t* ob = static_cast<uint8_t*>(p.out);
  const size_t row_bytes = static_cast<size_t>(p.D) * 2;
  const size_t tab_bytes = static_cast<size_t>(p.D);  // D/2 entries of 2 bytes
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / cpr;
    const int c = static_cast<int>(i - row * cpr);
    const long long t = row % p.T;
    const long long pos = (t < p.pos_split) ? p.pos_offset + t : p.pos_offset1 + (t - p.pos_split);
    const uint8_t* xr = xb + row * row_bytes;
    const uint4 lo = ldg_stream_v4(xr + c * 16);
    const uint4 hi = ldg_stream_v4(xr + tab_bytes + c * 16);
    const uint4 cv = ldg_v4(cb + pos * tab_bytes + c * 16);
    const uint4 sv = ldg_v4(sb + pos * tab_bytes + c * 16);
    const uint32_t la[4] = {lo.x, lo.y, lo.z, lo.w};
    const uint32_t ha[4] = {hi.x, hi.y, hi.z, hi.w};
    const uint32_t ca[4] = {cv.x, cv.y, cv.z, cv.w};
    const uint32_t sa[4] = {sv.x, sv.y, sv.z, sv.w};
    uint32_t ya[4], yb[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 l = unpack2<BF16>(la[e]);
      const float2 h = unpack2<BF16>(ha[e]);
      const float2 cc = unpack2<BF16>(ca[e]);
      const float2 ss = unpack2<BF16>(sa[e]);
      float y0, y1, z0, z1;
      if (BACKWARD) {
        y0 = l.x * cc.x + h.x * ss.x;
        y1 = l.y * cc.y + h.y * ss.y;
        z0 = h.x * cc.x - l.x * ss.x;
        z1 = h.y * cc.y - l.y * ss.y;
      } else {
        y0 = l.x * cc.x - h.x * ss.x;
        y1 = l.y * cc.y - h.y * ss.y;
        z0 = h.x * cc.x + l.x * ss.x;
        z1 = h.y * cc.y + l.y * ss.y;
      }
      if (OUT_F16) {
        ya[e] = pack2<false>(y0, y1);
        yb[e] = pack2<false>(z0, z1);
      } else {
        ya[e] = pack2<BF16>(y0, y1);
        yb[e] = pack2<BF16>(z0, z1);
      }
    }
    uint8_t* orow = ob + row * row_bytes;
    *reinterpret_cast<uint4*>(orow + c * 16) = make_uint4(ya[0], ya[1], ya[2], ya[3]);
    *reinterpret_cast<uint4*>(orow + tab_bytes + c * 16) = make_uint4(yb[0], yb[1], yb[2], yb[3]);
  }
}

}  // namespace du
