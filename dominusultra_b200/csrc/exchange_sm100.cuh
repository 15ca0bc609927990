// Exchange of the sequence-split decode partials over NVLink peer memory, merged in the same
// kernel: the collective + merge step of the long-context decode (the KV sequence split across
// the GPUs of one node), in place of an NCCL all-gather followed by the merge launch.
//
// Every rank holds an exchange buffer (XchLayout) that the other ranks map through CUDA IPC.
// CTA c of rank r owns rows [c * rpc, (c + 1) * rpc) of the partial: it stores them (o and lse,
// fp32) into slot r of every rank's buffer (its own included) with plain stores over NVLink,
// then, after a system-scope fence, raises flag [parity][r][c] on every rank to the call's
// epoch + 1. It then waits (bounded by time) until flag [parity][s][c] of its own buffer shows
// epoch + 1 for every rank s, and merges the world's partials of its rows by LSE into the final
// output (and lse). The epoch lives in each rank's buffer and is advanced by the rank's last CTA
// to finish, so every call (graph replays included) finds it where the previous one left it;
// slots and flags alternate between two parities, since a rank can run at most one call ahead
// of any other (its next merge waits for the others' flags of that call). No multicast, no
// NVLS: plain loads and stores only. Every CTA of a rank waits only for the same CTA index of
// the other ranks, and the grid is at most XCH_MAX_CTAS (<= the SM count), so all CTAs are
// resident and the waits end unless a rank does not run the call at all (then they time out).
#pragma once

#include "du_ptx.cuh"

namespace du {

constexpr int XCH_MAX_WORLD = 8;
constexpr int XCH_MAX_CTAS = 128;

struct XchLayout {
  // [0, 256): epoch (int), finished-CTA counter (int)
  // flags: int [2][XCH_MAX_WORLD][XCH_MAX_CTAS]
  // o: float [2][world][rows][D] (padded to 256 bytes); lse: float [2][world][rows]
  static constexpr size_t FLAGS = 256;
  static constexpr size_t FLAG_BYTES = 2ull * XCH_MAX_WORLD * XCH_MAX_CTAS * 4;
  static constexpr size_t DATA = FLAGS + FLAG_BYTES;
  static size_t o_bytes(int world, int rows, int D) {
    return ((2ull * world * rows * D * 4 + 255) / 256) * 256;
  }
  static size_t bytes(int world, int rows, int D) {
    return DATA + o_bytes(world, rows, D) + 2ull * world * rows * 4;
  }
};

struct XchParams {
  const float* o_loc;            // [rows, D] this rank's partial
  const float* lse_loc;          // [rows]
  uint8_t* peer[XCH_MAX_WORLD];  // every rank's exchange buffer as this process maps it
  int world, rank, rows, D, rpc;
  size_t o_bytes;                // XchLayout::o_bytes(world, rows, D)
  void* out;                     // [rows, D] in out_kind (0 fp16, 1 bf16, 2 fp32)
  int out_kind;
  float* lse_out;                // [rows] natural-log lse, or nullptr
};

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(128) xch_merge_kernel(const XchParams p) {
  const int tid = threadIdx.x;
  const int c = blockIdx.x;
  uint8_t* mine = p.peer[p.rank];
  int* ctrl = reinterpret_cast<int*>(mine);
  __shared__ int s_epoch, s_ok;
  if (tid == 0) {
    s_epoch = *reinterpret_cast<volatile int*>(ctrl);
    s_ok = 1;
  }
  __syncthreads();
  const int e = s_epoch;
  const int par = e & 1;
  const int r0 = c * p.rpc;
  const int r1 = min(p.rows, r0 + p.rpc);
  const int D = p.D;
  // 1) this CTA's rows of the local partial into slot `rank` of every rank's buffer
  for (int s = 0; s < p.world; ++s) {
    uint8_t* dst = p.peer[s];
    float* o_dst = reinterpret_cast<float*>(dst + XchLayout::DATA) +
                   (static_cast<size_t>(par) * p.world + p.rank) * p.rows * D;
    float* l_dst = reinterpret_cast<float*>(dst + XchLayout::DATA + p.o_bytes) +
                   (static_cast<size_t>(par) * p.world + p.rank) * p.rows;
    const int n4 = (r1 - r0) * D / 4;
    const float4* src4 = reinterpret_cast<const float4*>(p.o_loc + static_cast<size_t>(r0) * D);
    float4* dst4 = reinterpret_cast<float4*>(o_dst + static_cast<size_t>(r0) * D);
    for (int i = tid; i < n4; i += 128) dst4[i] = src4[i];
    for (int r = r0 + tid; r < r1; r += 128) l_dst[r] = p.lse_loc[r];
  }
  __syncthreads();
  // 2) the rows are in place on every rank: raise this CTA's flag there
  if (tid == 0) {
    __threadfence_system();
    for (int s = 0; s < p.world; ++s) {
      int* fl = reinterpret_cast<int*>(p.peer[s] + XchLayout::FLAGS) +
                (par * XCH_MAX_WORLD + p.rank) * XCH_MAX_CTAS + c;
      st_release_sys(fl, e + 1);
    }
  }
  // 3) wait for every rank's rows of this block (bounded)
  if (tid < p.world) {
    const int* fl = reinterpret_cast<const int*>(mine + XchLayout::FLAGS) +
                    (par * XCH_MAX_WORLD + tid) * XCH_MAX_CTAS + c;
    const uint64_t t0 = globaltimer();
    uint32_t n = 0;
    while (ld_acquire_sys(fl) != e + 1) {
      if ((++n & 255u) == 0u && globaltimer() - t0 > DU_WAIT_TIMEOUT_NS) {
        record_timeout(900 + tid);
        s_ok = 0;  // this block's rows are not merged; the status word records the wait
        break;
      }
    }
  }
  __syncthreads();
  if (s_ok) {
    // 4) merge the world's partials of rows [r0, r1): thread d holds dimension d
    const float* o_all = reinterpret_cast<const float*>(mine + XchLayout::DATA) +
                         static_cast<size_t>(par) * p.world * p.rows * D;
    const float* l_all = reinterpret_cast<const float*>(mine + XchLayout::DATA + p.o_bytes) +
                         static_cast<size_t>(par) * p.world * p.rows;
    for (int r = r0; r < r1; ++r) {
      float M = -INFINITY;
      for (int s = 0; s < p.world; ++s) M = fmaxf(M, __ldcg(l_all + static_cast<size_t>(s) * p.rows + r));
      for (int d = tid; d < D; d += 128) {
        float L = 0.f, A = 0.f;
        for (int s = 0; s < p.world; ++s) {
          const float ls = __ldcg(l_all + static_cast<size_t>(s) * p.rows + r);
          const float w = (ls == -INFINITY) ? 0.f : __expf(ls - M);
          L += w;
          A = fmaf(w, __ldcg(o_all + (static_cast<size_t>(s) * p.rows + r) * D + d), A);
        }
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
  }
  // 5) the rank's last CTA advances the epoch for the next call (every CTA has read it)
  __syncthreads();
  if (tid == 0 && atomicAdd(ctrl + 1, 1) == static_cast<int>(gridDim.x) - 1) {
    ctrl[1] = 0;
    __threadfence();
    atomicExch(ctrl, e + 1);
  }
}

}  // namespace du
