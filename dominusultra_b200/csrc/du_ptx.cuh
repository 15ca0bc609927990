// Thin inline-PTX wrappers for sm_100a: mbarriers with bounded waits, TMA (no multicast),
// bulk copies, tcgen05 (TMEM alloc, UMMA issue/commit, TMEM load/store) and the shared-memory
// matrix / instruction descriptors used by tcgen05.mma kind::f16.
//
// Every wait in this library is bounded: a wait that does not complete within
// DU_WAIT_TIMEOUT_NS records an error in g_du_status and returns false, so a broken pipeline
// ends the kernel instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#ifndef DU_WAIT_TIMEOUT_NS
#define DU_WAIT_TIMEOUT_NS 2000000000ull  // 2 s: far above any legitimate wait in these kernels
#endif

// Status words written by device code (the first error wins until the host resets them):
//   code 5, a bounded wait expired: [1] wait-site id, [2] blockIdx.x, [3] blockIdx.y;
//   code 6, a per-sequence cache length out of range: [1] sequence index, [2] the length.
__device__ unsigned int g_du_status[4];

#ifdef DU_TRACE
// Debug-only (DU_TRACE builds): event timestamps of the CTA at blockIdx (0, 0) [event][tile],
// and accumulators / per-CTA timelines recorded by the kernels.
__device__ long long g_du_trace[16 * 64];
#define DU_TRACE_EV(ev, j)                                                            \
  do {                                                                               \
    if (blockIdx.x == 0 && blockIdx.y == 0 && (j) < 64) g_du_trace[(ev) * 64 + (j)] = clock64(); \
  } while (0)
// Debug-only cycle accounting: slot `k` of the upper half of g_du_trace accumulates `v`.
#define DU_STAT(k, v)                                                                          \
  do {                                                                                         \
    atomicAdd(reinterpret_cast<unsigned long long*>(&g_du_trace[512 + (k)]),                  \
              static_cast<unsigned long long>(v));                                             \
  } while (0)
#else
#define DU_TRACE_EV(ev, j) \
  do {                     \
  } while (0)
#define DU_STAT(k, v) \
  do {                \
  } while (0)
#endif

namespace du {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_timeout(unsigned int site) {
  if (atomicCAS(&g_du_status[0], 0u, 5u) == 0u) {
    g_du_status[1] = site;
    g_du_status[2] = blockIdx.x;
    g_du_status[3] = blockIdx.y;
    __threadfence();
  }
}

__device__ __forceinline__ void record_error(unsigned int code, unsigned int a, unsigned int b) {
  if (atomicCAS(&g_du_status[0], 0u, code) == 0u) {
    g_du_status[1] = a;
    g_du_status[2] = b;
    g_du_status[3] = 0u;
    __threadfence();
  }
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Parity wait that lets the hardware suspend the thread for up to `hint_ns` while the phase is
// incomplete (the thread resumes when the phase completes), so waiting warps leave their issue
// slots to the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Suspend-time hint of the slow path of mbar_wait (0: plain try_wait, which the hardware may
// still suspend for a short system-defined time).
#ifndef DU_WAIT_SLEEP_NS
#define DU_WAIT_SLEEP_NS 20000u
#endif

// Bounded parity wait. `failed` is a per-CTA shared flag: once any thread of the CTA has timed
// out, every later slow wait gives up at once, so the whole CTA drains quickly.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* failed,
                                          unsigned int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  uint32_t n = 0;
  while (true) {
#if DU_WAIT_SLEEP_NS > 0
    if (mbar_try_wait_sleep(bar, parity, DU_WAIT_SLEEP_NS)) return true;
#else
    if (mbar_try_wait(bar, parity)) return true;
#endif
    if ((++n & 63u) == 0u) {
      if (*failed) return false;
      if (globaltimer() - t0 > DU_WAIT_TIMEOUT_NS) {
        record_timeout(site);
        *failed = 1;
        return false;
      }
    }
  }
}

// Non-blocking phase test: never suspends the thread.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded parity wait that polls without suspending, for single-thread MMA issuers: a
// suspended waiter can take a thousand cycles or more to resume on an SM whose other warps
// keep the issue slots busy, and every such delay lands on the tensor-core critical path.
__device__ __forceinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity, volatile int* failed,
                                               unsigned int site) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  uint32_t n = 0;
  while (true) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((++n & 255u) == 0u) {
      if (*failed) return false;
      if (globaltimer() - t0 > DU_WAIT_TIMEOUT_NS) {
        record_timeout(site);
        *failed = 1;
        return false;
      }
    }
  }
}

// Bounded wait used only while draining a CTA's own in-flight async work before exit: it
// ignores the CTA failure flag (the copies / MMAs must land before TMEM and shared memory are
// released) but still gives up after DU_WAIT_TIMEOUT_NS.
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, unsigned int site) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > DU_WAIT_TIMEOUT_NS) {
      record_timeout(site);
      return false;
    }
  }
  return true;
}

// Device-scope atomic add with acquire-release semantics: this thread's earlier writes, and those
// of threads it has synchronised with, are visible device-wide before the add; writes released
// by earlier adds on the same word are visible to this thread after it.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* addr, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}

// ---------------------------------------------------------------------------------------------
// proxy fences
// ---------------------------------------------------------------------------------------------
// Make this thread's generic-proxy shared-memory writes visible to the async proxy
// (tensor-core operand reads, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Order global-memory data seen through the generic proxy before this thread's later
// async-proxy (TMA) reads of global memory.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---------------------------------------------------------------------------------------------
// TMA (tiled, no multicast) and bulk copies
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* map, uint32_t bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* map, uint32_t bar, int c0,
                                            int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Contiguous global -> shared copy on the async proxy, completing `bytes` on `bar`
// (both addresses 16-byte aligned, size a multiple of 16). No multicast.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// ---------------------------------------------------------------------------------------------
// tcgen05: tensor memory and the 5th-generation tensor core
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Programmatic dependent launch: a kernel launched after this one with programmatic stream
// serialization may be scheduled once every CTA of this grid has executed launch_dependents;
// its griddep_wait then blocks until this grid has completed and its memory is visible (a no-op
// for a kernel launched without the attribute).
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// True in exactly one lane of the (converged) warp: the lane that issues single-thread
// tcgen05 operations while the whole warp walks the schedule.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(pred));
  return pred != 0;
}

// D[tmem] (+)= A[smem] * B[smem], kind::f16 (fp16/bf16 operands, fp32 accumulate), one CTA.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem], kind::f16: A (M x 16, 16-bit) read from tensor memory,
// two elements per 32-bit column, one row per lane.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 async operation issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns: thread i of the warp gets lane (base + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}

__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Per-warpgroup register budget change (all warps of the warpgroup execute the same one).
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------------------------------------
// UMMA descriptors
// ---------------------------------------------------------------------------------------------
// Shared-memory matrix descriptor (tcgen05 format): start address, leading/stride byte offsets
// (all >> 4), descriptor version 1 at bits [46,48), swizzle mode at bits [61,64)
// (2 = 128B, 4 = 64B, 6 = 32B).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t swizzle_mode) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(swizzle_mode & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
// fmt: 0 = fp16, 1 = bf16. major: 0 = K-major, 1 = MN-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int a_fmt, int b_fmt, int a_major,
                                                 int b_major) {
  return (1u << 4) | (static_cast<uint32_t>(a_fmt) << 7) | (static_cast<uint32_t>(b_fmt) << 10) |
         (static_cast<uint32_t>(a_major) << 15) | (static_cast<uint32_t>(b_major) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// Swizzle-mode code for a row span of `span_bytes` (128, 64 or 32).
__host__ __device__ constexpr int cx_gcd(int a, int b) { return b == 0 ? a : cx_gcd(b, a % b); }
__host__ __device__ constexpr int cx_lcm(int a, int b) { return a / cx_gcd(a, b) * b; }

__host__ __device__ constexpr uint32_t swizzle_code(int span_bytes) {
  return span_bytes == 128 ? 2u : (span_bytes == 64 ? 4u : 6u);
}

// Byte offset of 16-byte chunk `c` of row `r` inside a K-major swizzled tile of `rows` rows
// whose rows are `row_bytes` long, stored as column blocks of `span` bytes (span = min(128,
// row_bytes)); the swizzle XORs address bits [4,7) with bits [7,10) (masked to the span), the
// same pattern TMA writes for SWIZZLE_{32,64,128}B when the tile base is 1024-byte aligned.
template <int SPAN>
__device__ __forceinline__ uint32_t swz_chunk_offset(int rows, int r, int c) {
  constexpr int CPB = SPAN / 16;  // 16-byte chunks per block row
  const int blk = c / CPB;
  const uint32_t lin = static_cast<uint32_t>(r * SPAN + (c % CPB) * 16);
  const uint32_t sw = lin ^ (((lin >> 7) & static_cast<uint32_t>(CPB - 1)) << 4);
  return static_cast<uint32_t>(blk * rows * SPAN) + sw;
}

// ---------------------------------------------------------------------------------------------
// math helpers
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (Blackwell f32x2 arithmetic: one instruction for two lanes of math).
__device__ __forceinline__ uint64_t f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 f2_split(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for two values on the FMA pipe (relieves the MUFU unit, which runs 16 exponentials per
// clock per SM). x is clamped to >= -125; x = j + f with j = round(x) (added in fp32 to
// 1.5 * 2^23, which leaves j in the low mantissa bits) and f in [-1/2, 1/2]; 2^f by a cubic,
// 2^j by adding j to the exponent field. The cubic's coefficients are a minimax fit of 2^f on
// [-1/2, 1/2] (Lawson's iteratively reweighted least squares on relative error, done for this
// kernel); evaluated in fp32 its relative error is below 7.5e-5, far under the 16-bit rounding
// P receives afterwards.
__device__ __forceinline__ float2 ex2_poly2(float x0, float x1) {
  constexpr float C0 = 0x1.fff692p-1f, C1 = 0x1.62f31ap-1f, C2 = 0x1.f0de1ap-3f, C3 = 0x1.c3f76p-5f;
  const uint64_t X = f2(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t T = f2_add(X, f2(12582912.0f, 12582912.0f));
  const uint64_t J = f2_add(T, f2(-12582912.0f, -12582912.0f));
  const uint64_t F = f2_fma(J, f2(-1.0f, -1.0f), X);
  uint64_t P = f2_fma(f2(C3, C3), F, f2(C2, C2));
  P = f2_fma(P, F, f2(C1, C1));
  P = f2_fma(P, F, f2(C0, C0));
  const float2 t = f2_split(T);
  const float2 pp = f2_split(P);
  return make_float2(__uint_as_float(__float_as_uint(pp.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(pp.y) + (__float_as_uint(t.y) << 23)));
}

template <bool BF16>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if constexpr (BF16) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
  } else {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// Widen a packed pair of 16-bit values to an fp32 pair.
template <bool BF16>
__device__ __forceinline__ uint64_t widen2(uint32_t w) {
  if constexpr (BF16) {
    return f2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  } else {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
    return f2(f.x, f.y);
  }
}

// Half-split rotation of two element pairs at once in the input dtype:
// r1 = x1 * c - x2 * s, r2 = x2 * c + x1 * s (packed bf16x2 / f16x2 arithmetic).
template <bool BF16>
__device__ __forceinline__ void rope_rotate2(uint32_t x1, uint32_t x2, uint32_t c, uint32_t s,
                                             uint32_t& r1, uint32_t& r2) {
  if constexpr (BF16) {
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&x1);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&x2);
    const __nv_bfloat162 cc = *reinterpret_cast<const __nv_bfloat162*>(&c);
    const __nv_bfloat162 ss = *reinterpret_cast<const __nv_bfloat162*>(&s);
    const __nv_bfloat162 y1 = __hfma2(a, cc, __hneg2(__hmul2(b, ss)));
    const __nv_bfloat162 y2 = __hfma2(b, cc, __hmul2(a, ss));
    r1 = *reinterpret_cast<const uint32_t*>(&y1);
    r2 = *reinterpret_cast<const uint32_t*>(&y2);
  } else {
    const __half2 a = *reinterpret_cast<const __half2*>(&x1);
    const __half2 b = *reinterpret_cast<const __half2*>(&x2);
    const __half2 cc = *reinterpret_cast<const __half2*>(&c);
    const __half2 ss = *reinterpret_cast<const __half2*>(&s);
    const __half2 y1 = __hfma2(a, cc, __hneg2(__hmul2(b, ss)));
    const __half2 y2 = __hfma2(b, cc, __hmul2(a, ss));
    r1 = *reinterpret_cast<const uint32_t*>(&y1);
    r2 = *reinterpret_cast<const uint32_t*>(&y2);
  }
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// Streaming 128-bit global load that skips L1 allocation (KV cache is read once).
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ldg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

}  // namespace du
