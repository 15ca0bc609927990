// Exchange of the sequence-split decode partials over NVLink peer memory, merged in the same
// kernel: the collective + merge step of the long-context decode (the KV sequence split across
// the GPUs of one node), in place of an NCCL all-gather followed by the merge launch.
//
// Every rank holds an exchange buffer (XchLayout) that the other ranks map through CUDA IPC.
// CTA c of rank r owns rows [c * rpc, (c + 1) * rpc) of the partial (D output values and the lse
// per row, fp32). It stores each value into slot r of every rank's buffer (its own included) as
// one 64-bit word: the value's bits in the low half, the call's tag (epoch + 1) in the high half.
// A 64-bit aligned store is seen whole or not at all, so a reader that finds the tag also has
// the value: no fences and no separate flags. It then merges the world's partials of its rows
// by LSE, reading each word of its own buffer until the tag matches (bounded by time), into the
// final output (and lse). The epoch lives in each rank's buffer and is advanced by the rank's
// last CTA to finish, so every call (graph replays included) finds it where the previous one
// left it; slots alternate between two parities, since a rank can run at most one call ahead of
// any other (its next merge waits for the others' words of that call). No multicast, no NVLS:
// plain loads and stores only. A CTA waits only for words that the same CTA index of the other
// ranks stores, and the grid is at most XCH_MAX_CTAS (<= the SM count), so every CTA is resident
// and the waits end unless a rank does not run the call at all (then they time out).
#pragma once

#include "du_ptx.cuh"

namespace du {

constexpr int XCH_MAX_WORLD = 8;
constexpr int XCH_MAX_CTAS = 128;

struct XchLayout {
  // [0, 256): epoch (int), finished-CTA counter (int)
  // words: uint64 [2 parities][world][rows][D + 1] (value bits | tag << 32; column D: the lse)
  static constexpr size_t DATA = 256;
  static size_t bytes(int world, int rows, int D) {
    return DATA + 2ull * world * rows * (D + 1) * 8;
  }
};

struct XchParams {
  const float* o_loc;            // [rows, D] this rank's partial
  const float* lse_loc;          // [rows]
  uint8_t* peer[XCH_MAX_WORLD];  // every rank's exchange buffer as this process maps it
  int world, rank, rows, D, rpc;
  void* out;                     // [rows, D] in out_kind (0 fp16, 1 bf16, 2 fp32)
  int out_kind;
  float* lse_out;                // [rows] natural-log lse, or nullptr
};

__device__ __forceinline__ void st_word(unsigned long long* p, unsigned long long v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// The value of word w once its tag is `tag` (false when the wait times out).
__device__ __forceinline__ bool xch_read(const unsigned long long* w, unsigned int tag, float& v,
                                         uint64_t t0, unsigned int site) {
  unsigned long long x = ld_word(w);
  uint32_t n = 0;
  while (static_cast<unsigned int>(x >> 32) != tag) {
    if ((++n & 255u) == 0u && globaltimer() - t0 > DU_WAIT_TIMEOUT_NS) {
      record_timeout(site);
      return false;
    }
    x = ld_word(w);
  }
  v = __uint_as_float(static_cast<unsigned int>(x));
  return true;
}

__global__ void __launch_bounds__(128) xch_merge_kernel(const XchParams p) {
  const int tid = threadIdx.x;
  const int c = blockIdx.x;
  uint8_t* mine = p.peer[p.rank];
  int* ctrl = reinterpret_cast<int*>(mine);
  __shared__ int s_epoch;
  if (tid == 0) s_epoch = *reinterpret_cast<volatile int*>(ctrl);
  __syncthreads();
  const int e = s_epoch;
  const int par = e & 1;
  const unsigned int tag = static_cast<unsigned int>(e + 1);
  const unsigned long long hi = static_cast<unsigned long long>(tag) << 32;
  const int r0 = c * p.rpc;
  const int r1 = min(p.rows, r0 + p.rpc);
  const int D = p.D;
  const int W = D + 1;  // words per row
  // 1) this CTA's rows of the local partial into slot `rank` of every rank's buffer
  const int n = (r1 - r0) * W;
  for (int s = 0; s < p.world; ++s) {
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(p.peer[s] + XchLayout::DATA) +
                              ((static_cast<size_t>(par) * p.world + p.rank) * p.rows + r0) * W;
    for (int i = tid; i < n; i += 128) {
      const int r = r0 + i / W, col = i % W;
      const float val = (col < D) ? p.o_loc[static_cast<size_t>(r) * D + col] : p.lse_loc[r];
      st_word(dst + i, hi | __float_as_uint(val));
    }
  }
  // 2) merge the world's partials of rows [r0, r1): thread d holds dimension d
  const unsigned long long* base = reinterpret_cast<const unsigned long long*>(mine + XchLayout::DATA) +
                                   static_cast<size_t>(par) * p.world * p.rows * W;
  const uint64_t t0 = globaltimer();
  bool ok = true;
  for (int r = r0; ok && r < r1; ++r) {
    float ls[XCH_MAX_WORLD];
    float M = -INFINITY;
    for (int s = 0; s < p.world; ++s) {
      ok = ok && xch_read(base + (static_cast<size_t>(s) * p.rows + r) * W + D, tag, ls[s], t0, 900 + s);
      M = fmaxf(M, ls[s]);
    }
    if (!ok) break;
    for (int d = tid; d < D; d += 128) {
      float L = 0.f, A = 0.f;
      for (int s = 0; s < p.world; ++s) {
        float o;
        if (!xch_read(base + (static_cast<size_t>(s) * p.rows + r) * W + d, tag, o, t0, 900 + s)) {
          ok = false;
          break;
        }
        const float w = (ls[s] == -INFINITY) ? 0.f : __expf(ls[s] - M);
        L += w;
        A = fmaf(w, o, A);
      }
      if (!ok) break;
      const float val = (L > 0.f) ? A / L : 0.f;
      const size_t idx = static_cast<size_t>(r) * D + d;
      if (p.out_kind == 2) {
        static_cast<float*>(p.out)[idx] = val;
      } else if (p.out_kind == 1) {
        static_cast<__nv_bfloat16*>(p.out)[idx] = __float2bfloat16_rn(val);
      } else {
        static_cast<__half*>(p.out)[idx] = __float2half_rn(val);
      }
      if (d == 0 && p.lse_out != nullptr) p.lse_out[r] = (L > 0.f) ? M + __logf(L) : -INFINITY;
    }
  }
  // 3) the rank's last CTA advances the epoch for the next call (every CTA has read it)
  __syncthreads();
  if (tid == 0 && atomicAdd(ctrl + 1, 1) == static_cast<int>(gridDim.x) - 1) {
    ctrl[1] = 0;
    __threadfence();
    atomicExch(ctrl, e + 1);
  }
}

}  // namespace du
