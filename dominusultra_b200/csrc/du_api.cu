// C ABI of the B200 fused-RoPE attention library (declared in include/dominus_ultra_b200.h).
//
// This translation unit holds the host-side launchers: argument validation, TMA tensor-map
// encoding (cuTensorMapEncodeTiled reached through the runtime's driver entry point, so the
// library does not link libcuda directly), decode split planning and the kernel dispatch over
// head_dim x dtype.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <utility>
#include <string>

#include "../../include/dominus_ultra_b200.h"
#include "decode_sm100.cuh"
#include "decode_tc_sm100.cuh"
#include "exchange_sm100.cuh"
#include "prefill_fa1_sm100.cuh"
#include "prefill_fa_sm100.cuh"
#include "prefill_sm100.cuh"
#include "rope_sm100.cuh"

namespace du {

// One CTA waits on an mbarrier that nothing arrives at, bounded by timeout_ns: the timeout is
// recorded in g_du_status (site 200) and the kernel returns.
__global__ void selftest_wait_kernel(unsigned long long timeout_ns) {
  __shared__ __align__(8) unsigned long long bar;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait_sleep(b, 0, 1000u)) {
      if (globaltimer() - t0 > timeout_ns) {
        record_timeout(200);
        break;
      }
    }
  }
}

}  // namespace du

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(DU_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool valid_head_dim(int D) { return D == 16 || D == 32 || D == 64 || D == 128 || D == 256; }

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
  });
  return fn;
}

// 3-D map over a contiguous [rows_outer, T, D] 16-bit tensor: dims {D, T, rows_outer}, box
// {box_cols, box_rows, 1}, swizzle matching the box row span, zero fill out of bounds.
int encode_map(CUtensorMap* map, const void* base, int dtype, int D, int T, long long outer,
               int box_cols, int box_rows, int span_bytes) {
  auto fn = get_encode_fn();
  if (fn == nullptr) return fail(DU_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(T),
                        static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2,
                           static_cast<cuuint64_t>(T) * static_cast<cuuint64_t>(D) * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapSwizzle sw = span_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : span_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                   : CU_TENSOR_MAP_SWIZZLE_32B;
  const CUtensorMapDataType dt =
      dtype == DU_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DU_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(r));
  return DU_OK;
}

// 2-D map over a [rows, cols] 16-bit table (no swizzle): box {cols, box_rows}.
int encode_map_2d(CUtensorMap* map, const void* base, int dtype, int cols, long long rows,
                  int box_rows) {
  auto fn = get_encode_fn();
  if (fn == nullptr) return fail(DU_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      dtype == DU_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DU_ERR_CUDA, "cuTensorMapEncodeTiled (table) failed with CUresult " + std::to_string(r));
  return DU_OK;
}

// 2-D map over a [rows, cols] 16-bit table: box {box_cols, box_rows}, swizzle for a box row of
// span_bytes (16: none), zero fill out of bounds.
int encode_map_2d_sw(CUtensorMap* map, const void* base, int dtype, int cols, long long rows,
                     int box_cols, int box_rows, int span_bytes) {
  auto fn = get_encode_fn();
  if (fn == nullptr) return fail(DU_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = span_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : span_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                : span_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                   : CU_TENSOR_MAP_SWIZZLE_NONE;
  const CUtensorMapDataType dt =
      dtype == DU_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DU_ERR_CUDA, "cuTensorMapEncodeTiled (table) failed with CUresult " + std::to_string(r));
  return DU_OK;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device). The cache is
// keyed by the kernel's address: every instantiation shares one function-pointer type.
template <typename Kern>
cudaError_t ensure_smem_attr(Kern kern, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const auto key = std::make_pair(reinterpret_cast<const void*>(kern), dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key)) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.insert(key);
  return e;
}

// Launch on `st`; with `pdl` as a programmatic dependent of the stream's previous kernel (the
// kernel must call griddep_wait before touching that kernel's outputs).
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, unsigned block, size_t smem,
                          cudaStream_t st, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Launch the standalone rotary kernel over rows = B * H * T rows of D elements.
template <bool BF16, bool OUT_F16, bool BACKWARD>
int launch_rope_t(const du::RopeParams& rp, cudaStream_t st) {
  const long long total = rp.rows * (rp.D / 16);
  long long blocks = (total + 255) / 256;
  const long long cap = static_cast<long long>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  du::rope_kernel<BF16, OUT_F16, BACKWARD><<<static_cast<unsigned>(blocks), 256, 0, st>>>(rp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "rope launch");
  return DU_OK;
}

int launch_rope(const du::RopeParams& rp, bool bf16, bool out_f16, bool backward, cudaStream_t st) {
  if (bf16) {
    if (out_f16) return backward ? launch_rope_t<true, true, true>(rp, st) : launch_rope_t<true, true, false>(rp, st);
    return backward ? launch_rope_t<true, false, true>(rp, st) : launch_rope_t<true, false, false>(rp, st);
  }
  return backward ? launch_rope_t<false, false, true>(rp, st) : launch_rope_t<false, false, false>(rp, st);
}

// Registers per thread the kernel was built with, once per kernel: a setmaxnreg split that asks
// for more registers than the launch provides would never complete, so launches check it.
template <typename Kern>
int launch_registers(Kern kern) {
  static std::mutex mu;
  static std::map<const void*, int> regs;
  std::lock_guard<std::mutex> lock(mu);
  auto it = regs.find(reinterpret_cast<const void*>(kern));
  if (it != regs.end()) return it->second;
  cudaFuncAttributes attr{};
  if (cudaFuncGetAttributes(&attr, kern) != cudaSuccess) return -1;
  regs[reinterpret_cast<const void*>(kern)] = attr.numRegs;
  return attr.numRegs;
}

// Bytes of the rotated-key buffer du_prefill needs (fp16 R(K), [B, Hkv, T, D]).
size_t prefill_ws_bytes(int B, int Hkv, int T, int D) {
  if (D > 128) return 0;
  return static_cast<size_t>(B) * Hkv * T * D * 2;
}

// The two-tile attention kernel over pre-rotated fp16 keys k_rot and values v of Tkv rows per
// (b, kv head); query tiles cover rows [q_row0, q_row0 + Tq) of the T-row query tensor.
template <int D, bool BF16, bool BLOCK>
int launch_fa_t(const void* q, const void* k_rot, const void* v, du::PrefillParams prm, int B,
                int Tkv, cudaStream_t st) {
  using S = du::FaShape<D>;
  const int dtype = BF16 ? DU_DTYPE_BF16 : DU_DTYPE_F16;
  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = encode_map(&tq, q, dtype, D, prm.T, static_cast<long long>(B) * prm.Hq, S::SPAN / 2,
                       S::BM, S::SPAN)) != DU_OK)
    return rc;
  if ((rc = encode_map(&tk, k_rot, DU_DTYPE_F16, D, Tkv, static_cast<long long>(B) * prm.Hkv,
                       S::SPAN / 2, S::BN, S::SPAN)) != DU_OK)
    return rc;
  if ((rc = encode_map(&tv, v, dtype, D, Tkv, static_cast<long long>(B) * prm.Hkv, S::SPAN / 2,
                       S::BN, S::SPAN)) != DU_OK)
    return rc;
  prm.n_qtiles = (prm.Tq + 2 * S::BM - 1) / (2 * S::BM);  // query-tile pairs
  auto kern = du::prefill_fa_kernel<D, BF16, BLOCK>;
  const int regs = launch_registers(kern);
  if (regs * S::NTHREADS < 2 * 128 * S::REG_SOFTMAX + 128 * S::REG_OTHER)
    return fail(DU_ERR_CUDA, "prefill kernel built with too few registers for its split");
  cudaError_t e = ensure_smem_attr(kern, S::SMEM_BYTES);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prefill)");
  // One CTA per (query-tile pair, query head), in the kernel's group-major order.
  dim3 grid(static_cast<unsigned>(static_cast<long long>(B) * prm.Hq * prm.n_qtiles));
  // The whole-sequence path follows its key-rotation launch as a programmatic dependent: the
  // CTAs' set-up and query loads overlap the rotation; only the K producer waits for it. The
  // block form (context-parallel prefill) is launched after arbitrary work and does not.
  e = launch_kernel(kern, grid, S::NTHREADS, S::SMEM_BYTES, st, !BLOCK, tq, tk, tv, prm);
  if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
  return DU_OK;
}

template <int D, bool BF16>
int launch_prefill_t(const void* q, const void* k, const void* v, du::PrefillParams prm, int B,
                     long long rope_positions, void* ws, cudaStream_t st) {
  const int dtype = BF16 ? DU_DTYPE_BF16 : DU_DTYPE_F16;
  CUtensorMap tq, tk, tv;
  int rc;
  cudaError_t e;
  if constexpr (D <= 128) {
    // Short sequences on the one-tile kernel (at most two key tiles per CTA): the attention
    // kernel rotates its key tiles itself, so there is one launch instead of two. Every query
    // head's CTAs rotate their own copy of their KV head's tiles: per query head that is at most
    // 1.5x the rotations of a separate pass, so about 1.5 G x for a query group of G heads --
    // a few microseconds of ALU work at these lengths against a launch and its latency saved.
    using SK = du::Fa1Shape<(D <= 64) ? D : 64>;
    const bool krot = D <= 64 && prm.T <= 2 * SK::BN;
    // 1) R(K) once per (b, kv head), fp16, into the workspace.
    du::RopeParams rp{};
    rp.x = k;
    rp.cos = prm.cos;
    rp.sin = prm.sin;
    rp.out = ws;
    rp.rows = static_cast<long long>(B) * prm.Hkv * prm.T;
    rp.T = prm.T;
    rp.D = D;
    rp.pos_offset = 0;
    rp.pos_split = prm.T;
    rp.pos_offset1 = 0;
    if (!krot && (rc = launch_rope(rp, BF16, true, false, st)) != DU_OK) return rc;
    // 2) attention. Sequences up to 4096 (head_dim <= 64): one query tile per CTA, two CTAs per
    // SM, so one CTA's start-up and wind-down overlap the other's steady state (measured +3-5%
    // at S = 512-2048). Longer ones: two tiles per CTA sharing each K/V tile (+3.5% at 8192).
    constexpr bool kOneTile = D <= 64;
    if (kOneTile && prm.T <= 4096) {
      using S1 = du::Fa1Shape<kOneTile ? D : 64>;
      if ((rc = encode_map(&tq, q, dtype, D, prm.T, static_cast<long long>(B) * prm.Hq, S1::SPAN / 2,
                           S1::BM, S1::SPAN)) != DU_OK)
        return rc;
      if ((rc = encode_map(&tk, krot ? k : ws, krot ? dtype : DU_DTYPE_F16, D, prm.T,
                           static_cast<long long>(B) * prm.Hkv, S1::SPAN / 2, S1::BN, S1::SPAN)) != DU_OK)
        return rc;
      prm.krot = krot ? 1 : 0;
      if ((rc = encode_map(&tv, v, dtype, D, prm.T, static_cast<long long>(B) * prm.Hkv,
                           S1::SPAN / 2, S1::BN, S1::SPAN)) != DU_OK)
        return rc;
      prm.n_qtiles = (prm.T + S1::BM - 1) / S1::BM;
      auto kern1 = du::prefill_fa1_kernel<kOneTile ? D : 64, BF16>;
      const int regs1 = launch_registers(kern1);
      if (regs1 * S1::NTHREADS < 128 * S1::REG_SOFTMAX + 128 * S1::REG_OTHER)
        return fail(DU_ERR_CUDA, "prefill kernel built with too few registers for its split");
      e = ensure_smem_attr(kern1, S1::SMEM_BYTES);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prefill)");
      dim3 grid1(static_cast<unsigned>(B * prm.Hq), static_cast<unsigned>(prm.n_qtiles));
      // A programmatic dependent of the rotary launch (none with krot).
      e = launch_kernel(kern1, grid1, S1::NTHREADS, S1::SMEM_BYTES, st, !krot, tq, tk, tv, prm);
      if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
      e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
      return DU_OK;
    }
    return launch_fa_t<D, BF16, false>(q, ws, v, prm, B, prm.T, st);
  } else {
    (void)rope_positions;
    (void)ws;
    using S = du::PrefillShape<D>;
    if ((rc = encode_map(&tq, q, dtype, D, prm.T, static_cast<long long>(B) * prm.Hq, S::SPAN / 2,
                         S::BM, S::SPAN)) != DU_OK)
      return rc;
    if ((rc = encode_map(&tk, k, dtype, D, prm.T, static_cast<long long>(B) * prm.Hkv,
                         S::SPAN / 2, S::BN, S::SPAN)) != DU_OK)
      return rc;
    if ((rc = encode_map(&tv, v, dtype, D, prm.T, static_cast<long long>(B) * prm.Hkv,
                         S::SPAN / 2, S::BN, S::SPAN)) != DU_OK)
      return rc;
    prm.n_qtiles = (prm.T + S::BM - 1) / S::BM;
    auto kern = du::prefill_kernel<D, BF16>;
    e = ensure_smem_attr(kern, S::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prefill)");
    dim3 grid(static_cast<unsigned>(B * prm.Hq), static_cast<unsigned>(prm.n_qtiles));
    kern<<<grid, S::NTHREADS, S::SMEM_BYTES, st>>>(tq, tk, tv, prm);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
  return DU_OK;
}

struct DecodePlan {
  int GT;
  int n_gchunk;
  int n_split;   // partial slots per row; 1 = whole units round-robin, final output direct
  int n_units;
  int cpu;       // chunks per unit
  long long total_chunks;
  int grid;      // CTAs launched (the kernel's resident count per SM x SMs, or fewer)
  int frag_pen;  // chunks charged to each unit start when the split walk cuts CTA ranges
};

// Keys per ring stage of the decode kernel instantiated for (D, GT): splits are whole chunks.
template <int D>
int decode_chunk_d(int GT) {
  switch (GT) {
    case 4: return du::DecodeShape<D, 4>::CK;
    case 2: return du::DecodeShape<D, 2>::CK;
    default: return du::DecodeShape<D, 1>::CK;
  }
}

// Four- and eight-head units at head_dim 128 run on the tensor-core kernel (decode_tc_sm100.cuh), for
// du_decode, du_decode_partial and du_decode_kvcache alike.
bool decode_use_tc(int D, int GT) { return D == 128 && (GT == 4 || GT == 8); }

int decode_chunk(int D, int GT, bool tc = false) {
  if (tc && decode_use_tc(D, GT)) return du::DecodeTcShape<128>::CK;
  if (GT == 8) GT = 4;  // (eight-head units exist on the tensor-core kernel only)
  switch (D) {
    case 16: return decode_chunk_d<16>(GT);
    case 32: return decode_chunk_d<32>(GT);
    case 64: return decode_chunk_d<64>(GT);
    case 128: return decode_chunk_d<128>(GT);
    default: return decode_chunk_d<256>(GT);
  }
}

// Resident CTAs per SM the decode kernel is built for (its launch bounds): three for one query
// head per unit, two for two, one for four.
int decode_residency(int GT) { return GT == 1 ? 3 : (GT == 2 ? 2 : 1); }  // 4, 8: one

// Units are (b, kv head, group chunk of GT query heads). A persistent grid of resident CTAs
// either takes whole units round-robin (when they divide evenly over the CTAs, or are so many
// that the last round hardly matters), or cuts the flattened (unit, chunk) sequence into equal
// contiguous ranges, one per CTA; then a unit is spread over consecutive CTAs, each writing an
// fp32 partial into its own slot of the row, and merge_kernel combines the slots.
DecodePlan plan_decode(int B, int Hq, int Hkv, int L, int D) {
  DecodePlan pl{};
  const int G = Hq / Hkv;
  // Eight-head units on the tensor-core kernel read each KV byte once for groups of 8 (two
  // four-head units read it twice: B4 H64 Hkv8 L131072 D128 measured 799 us that way).
  pl.GT = (G % 8 == 0 && D == 128) ? 8 : (G % 4 == 0) ? 4 : ((G % 2 == 0) ? 2 : 1);
  pl.n_gchunk = G / pl.GT;
  const long long units = static_cast<long long>(B) * Hkv * pl.n_gchunk;
  const long long ctas = static_cast<long long>(sm_count()) * decode_residency(pl.GT);
  const int chunk = decode_chunk(D, pl.GT, true);
  pl.n_units = static_cast<int>(units);
  pl.cpu = (L + chunk - 1) / chunk;
  pl.total_chunks = units * pl.cpu;
  const long long grid = pl.total_chunks < ctas ? pl.total_chunks : ctas;
  const long long per = pl.total_chunks / grid;  // chunks per CTA, at least
  // Whole units (no partials, no merge) when they spread evenly, are plentiful, are too short to
  // be worth cutting (fragments of fewer than four chunks cost more in partials than they
  // balance), or — for the one- and two-head kernels, several CTAs per SM — when they keep at
  // least three quarters of the SMs streaming. Measured on B200, one-head units: 128 / 192 / 256
  // units 3 / 7 / 28 % faster whole than split; the four-head kernel (one CTA per SM) split is
  // faster at 128 and 320 units (3 / 21 %). Beyond the resident CTAs each CTA takes k units,
  // k = ceil(units / ctas), over ceil(units / k) CTAs (512 units: 31.2 -> 27.0 us).
  // Few, short units (fewer than four chunks per CTA over the whole grid): fragments of at
  // least four chunks on fewer CTAs, when that still spreads the work over more CTAs than whole
  // units would (B1 H32 Hkv8 L4096 D128: 8 whole units on 8 CTAs took 63.5 us).
  constexpr long long kMinPer = 4;
  const long long short_grid = pl.total_chunks / kMinPer;
  const bool short_split = per < kMinPer && short_grid >= 2 * units;
  const bool whole = !short_split &&
                     (units % ctas == 0 || units >= 8 * ctas || per < kMinPer ||
                      (pl.GT <= 2 && 4 * units >= 3LL * sm_count()));
  if (short_split) {
    pl.grid = static_cast<int>(short_grid);
    const long long sper = pl.total_chunks / short_grid;  // >= kMinPer
    long long sslots = (pl.cpu - 1 + sper - 1) / sper + 1;
    if (sslots < 2) sslots = 2;
    pl.n_split = static_cast<int>(sslots);
    return pl;
  }
  if (whole) {
    pl.n_split = 1;
    const long long k = (units + ctas - 1) / ctas;  // units per CTA
    pl.grid = static_cast<int>((units + k - 1) / k);
    return pl;
  }
  // Fewer units than CTAs: k = ctas / units CTAs per unit, so that every CTA's range lies in
  // one unit (one fragment per CTA), when that costs no more than spreading the chunks over all
  // CTAs. A CTA whose range straddles two units finishes its first fragment, combines it and
  // restarts its pipeline, about three chunks' time, and such CTAs set the kernel's end
  // (measured on the tensor-core decode, B4 H32 Hkv8 D128: one fragment per CTA on 128 CTAs
  // vs 148 CTAs, L4096 24.4 vs 29.5 us, L8192 36.8 vs 40.6, L16384 60.8 vs 61.7,
  // L32768 109.1 vs 103.5, L131072 401 vs 384).
  constexpr long long kFragPenalty = 3;
  const long long k_al = units < ctas ? ctas / units : 0;
  if (k_al >= 1 && pl.cpu >= 2 * kMinPer &&
      (pl.cpu + k_al - 1) / k_al <= (pl.total_chunks + ctas - 1) / ctas + kFragPenalty) {
    const long long k = k_al;
    pl.grid = static_cast<int>(units * k);
    pl.n_split = static_cast<int>(k);  // k == 1: whole units, final rows written directly
    return pl;
  }
  // Spread over every CTA. On the tensor-core kernel a CTA's second fragment costs a few
  // chunks' time (combine, ticket, merge, restart; a per-CTA timeline of B4 H32 Hkv8 D128
  // L16384 showed the two-fragment CTAs ending ~5 us after the others), so each unit start is
  // charged that many chunks when the ranges are cut (DecodeWalk) and such CTAs take fewer.
  // Measured (graph-timed, B200) charging 0 / 4 / 6 chunks: L16384 63.9 / 60.6 / 60.8 us,
  // eight-head units (H64) L16384 76.6 / 71.5 / 70.0, L20000 74.0 / 70.3 / 71.4, L65536
  // 196.8 / 194.2 / 193.6.
  pl.frag_pen = decode_use_tc(D, pl.GT) ? (pl.GT == 8 ? 6 : 4) : 0;
  // A CTA inside one unit holds at least vper of its chunks, so a unit spans at most this many.
  const long long vper = units * (pl.cpu + pl.frag_pen) / grid;
  long long slots = (pl.cpu - 1 + vper - 1) / vper + 1;
  if (slots < 2) slots = 2;
  pl.grid = static_cast<int>(grid);
  pl.n_split = static_cast<int>(slots);
  return pl;
}

// Split-walk workspace: ticket counters (du::DECODE_CNT_BYTES, zero between calls), then the
// partials o [B * Hq, n_split, D] and lse [B * Hq, n_split] fp32.
size_t decode_ws_bytes(const DecodePlan& pl, int B, int Hq, int D) {
  if (pl.n_split <= 1) return 0;
  const size_t rows = static_cast<size_t>(B) * Hq;
  const size_t o = rows * pl.n_split * D * sizeof(float);
  const size_t l = rows * pl.n_split * sizeof(float);
  return du::DECODE_CNT_BYTES + ((o + 255) / 256) * 256 + l;
}

template <int D, bool BF16, int GT>
int launch_decode_tc_t(const du::DecodeParams& prm, int B, long long rope_positions, int grid,
                       cudaStream_t st) {
  using S = du::DecodeTcShape<D, GT>;
  const int dtype = BF16 ? DU_DTYPE_BF16 : DU_DTYPE_F16;
  CUtensorMap tk, tv, tc, ts;
  int rc;
  const long long units = static_cast<long long>(B) * prm.Hkv;
  if ((rc = encode_map(&tk, prm.k, dtype, S::D, prm.L, units, S::SPAN / 2, S::CK, S::SPAN)) != DU_OK) return rc;
  if ((rc = encode_map(&tv, prm.v, dtype, S::D, prm.L, units, S::SPAN / 2, S::CK, S::SPAN)) != DU_OK) return rc;
  if ((rc = encode_map_2d_sw(&tc, prm.cos, dtype, S::D / 2, rope_positions, S::D / 2, S::CK, S::TSPAN)) != DU_OK)
    return rc;
  if ((rc = encode_map_2d_sw(&ts, prm.sin, dtype, S::D / 2, rope_positions, S::D / 2, S::CK, S::TSPAN)) != DU_OK)
    return rc;
  auto kern = du::decode_tc_kernel<S::D, BF16, S::GT>;
  cudaError_t e = ensure_smem_attr(kern, S::SMEM_BYTES);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode, tensor cores)");
  // With per-sequence lengths the kernel follows decode_prep_kernel as its programmatic dependent
  // (barrier set-up overlaps the prep kernel; the kernel waits before any global access and takes
  // TMEM only after the wait). Plain decode launches are ordinary: as a dependent of the previous
  // step its CTAs filled the free slots early and unbalanced the step (measured slower).
  e = launch_kernel(kern, dim3(static_cast<unsigned>(grid)), S::NTHREADS, S::SMEM_BYTES, st,
                    prm.varlen != 0, tk, tv, tc, ts, prm);
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return DU_OK;
}

template <int D, bool BF16, int GT>
int launch_decode_cuda_t(const du::DecodeParams& prm, int B, long long rope_positions, int grid,
                         cudaStream_t st) {
  using S = du::DecodeShape<D, GT>;
  const int dtype = BF16 ? DU_DTYPE_BF16 : DU_DTYPE_F16;
  CUtensorMap tk, tv, tc, ts;
  int rc;
  const long long units = static_cast<long long>(B) * prm.Hkv;
  if ((rc = encode_map(&tk, prm.k, dtype, D, prm.L, units, S::SPAN / 2, S::CK, S::SPAN)) != DU_OK) return rc;
  if ((rc = encode_map(&tv, prm.v, dtype, D, prm.L, units, S::SPAN / 2, S::CK, S::SPAN)) != DU_OK) return rc;
  if ((rc = encode_map_2d_sw(&tc, prm.cos, dtype, D / 2, rope_positions, S::TSPAN / 2, S::CK, S::TSPAN)) != DU_OK)
    return rc;
  if ((rc = encode_map_2d_sw(&ts, prm.sin, dtype, D / 2, rope_positions, S::TSPAN / 2, S::CK, S::TSPAN)) != DU_OK)
    return rc;
  auto kern = du::decode_kernel<D, BF16, GT>;
  cudaError_t e = ensure_smem_attr(kern, S::SMEM_BYTES);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode)");
  // The work walk depends on the grid size the plan chose (resident CTAs only). With per-sequence
  // lengths the kernel follows decode_prep_kernel as its programmatic dependent. Plain decode
  // launches are ordinary: as a programmatic dependent of the previous step (which triggers at
  // its start) the next step's CTAs took the free slots early and unbalanced its units
  // (B8 H32 L2048 D64: 26.5 -> 31 us).
  e = launch_kernel(kern, static_cast<unsigned>(grid), S::NTHREADS, S::SMEM_BYTES, st,
                    prm.varlen != 0, tk, tv, tc, ts, prm);
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return DU_OK;
}

// The split kernel for (D, GT): tcgen05 for four- and eight-head units at head_dim 128, the
// CUDA-core kernel otherwise.
template <int D, bool BF16, int GT>
int launch_decode_split_t(const du::DecodeParams& prm, int B, long long rope_positions, int grid,
                          cudaStream_t st) {
  if constexpr (D == 128 && (GT == 4 || GT == 8)) {
    return launch_decode_tc_t<D, BF16, GT>(prm, B, rope_positions, grid, st);
  } else if constexpr (GT == 8) {
    return fail(DU_ERR_UNSUPPORTED, "eight-head decode units need head_dim 128");
  } else {
    return launch_decode_cuda_t<D, BF16, GT>(prm, B, rope_positions, grid, st);
  }
}

template <int D, bool BF16>
int launch_decode_split_g(const du::DecodeParams& prm, int GT, int B, long long rp, int grid,
                          cudaStream_t st) {
  switch (GT) {
    case 8: return launch_decode_split_t<D, BF16, 8>(prm, B, rp, grid, st);
    case 4: return launch_decode_split_t<D, BF16, 4>(prm, B, rp, grid, st);
    case 2: return launch_decode_split_t<D, BF16, 2>(prm, B, rp, grid, st);
    default: return launch_decode_split_t<D, BF16, 1>(prm, B, rp, grid, st);
  }
}

template <bool BF16>
int launch_decode_split_d(const du::DecodeParams& prm, int GT, int D, int B, long long rp,
                          int grid, cudaStream_t st) {
  switch (D) {
    case 16: return launch_decode_split_g<16, BF16>(prm, GT, B, rp, grid, st);
    case 32: return launch_decode_split_g<32, BF16>(prm, GT, B, rp, grid, st);
    case 64: return launch_decode_split_g<64, BF16>(prm, GT, B, rp, grid, st);
    case 128: return launch_decode_split_g<128, BF16>(prm, GT, B, rp, grid, st);
    case 256: return launch_decode_split_g<256, BF16>(prm, GT, B, rp, grid, st);
    default: return fail(DU_ERR_UNSUPPORTED, "head_dim must be one of 16, 32, 64, 128, 256");
  }
}

int launch_merge(const float* o_parts, const float* lse_parts, int R, int rows, int D,
                 long long o_sr, long long o_srow, long long l_sr, long long l_srow, void* out,
                 int out_kind, float* lse_out, cudaStream_t st) {
  if (R > du::MERGE_MAX_R) return fail(DU_ERR_UNSUPPORTED, "more partials than the merge supports");
  // Launched as a programmatic dependent of the preceding kernel on the stream (the decode split
  // kernel signals at its start), so the merge's launch and set-up overlap that kernel's tail;
  // the merge waits for the producer's completion before reading the partials.
  cudaError_t e = launch_kernel(du::merge_kernel, static_cast<unsigned>(rows), 128, 0, st, true,
                                o_parts, lse_parts, R, D, o_sr, o_srow, l_sr, l_srow, out,
                                out_kind, lse_out);
  if (e != cudaSuccess) return cuda_fail(e, "merge launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "merge launch");
  return DU_OK;
}

int check_common(int B, int Hq, int Hkv, int len, int D, int dtype) {
  if (B <= 0 || Hq <= 0 || len <= 0)
    return fail(DU_ERR_INVALID, "batch, heads, and sequence length must be positive");
  if (Hkv <= 0 || Hq % Hkv != 0)
    return fail(DU_ERR_INVALID, "num_query_heads must be divisible by num_kv_heads");
  if (!valid_head_dim(D))
    return fail(DU_ERR_UNSUPPORTED, "head_dim must be a power of two between 16 and 256");
  if (dtype != DU_DTYPE_F16 && dtype != DU_DTYPE_BF16)
    return fail(DU_ERR_INVALID, "dtype must be DU_DTYPE_F16 or DU_DTYPE_BF16");
  return DU_OK;
}

// Shared body of du_decode and du_decode_partial.
int decode_impl(const void* q, const void* kc, const void* vc, const void* cos, const void* sin,
                void* out, float* out_f32, float* lse_f32, int B, int Hq, int Hkv, int L, int D,
                int dtype, float scale, long long q_pos, long long kv_off, long long rope_positions,
                void* ws, size_t ws_bytes, cudaStream_t st) {
  int rc = check_common(B, Hq, Hkv, L, D, dtype);
  if (rc != DU_OK) return rc;
  if (!q || !kc || !vc || !cos || !sin || (!out && !out_f32))
    return fail(DU_ERR_INVALID, "null pointer argument");
  if (!aligned16(q) || !aligned16(kc) || !aligned16(vc) || !aligned16(cos) || !aligned16(sin))
    return fail(DU_ERR_INVALID, "q, caches and rope tables must be 16-byte aligned");
  if (q_pos < 0 || kv_off < 0 || q_pos >= rope_positions || kv_off + L > rope_positions)
    return fail(DU_ERR_INVALID, "rope tables do not cover the query / key positions");
  if (!(scale > 0.f)) return fail(DU_ERR_INVALID, "scale must be positive");
  const DecodePlan pl = plan_decode(B, Hq, Hkv, L, D);
  du::DecodeParams prm{};
  prm.q = q;
  prm.k = kc;
  prm.v = vc;
  prm.cos = cos;
  prm.sin = sin;
  prm.Hq = Hq;
  prm.Hkv = Hkv;
  prm.L = L;
  prm.G = Hq / Hkv;
  prm.n_gchunk = pl.n_gchunk;
  prm.n_split = pl.n_split;
  prm.n_units = pl.n_units;
  prm.cpu = pl.cpu;
  prm.total_chunks = pl.total_chunks;
  prm.frag_pen = pl.frag_pen;
  prm.q_pos = q_pos;
  prm.kv_pos_offset = kv_off;
  prm.scale_log2 = scale * 1.4426950408889634f;
  const bool bf16 = dtype == DU_DTYPE_BF16;
  const long long rows = static_cast<long long>(B) * Hq;
  if (pl.n_split == 1) {
    if (out != nullptr) {
      prm.mode = 0;
      prm.out = out;
    } else {
      prm.mode = 1;
      prm.o_part = out_f32;
      prm.lse_part = lse_f32;
    }
    return bf16 ? launch_decode_split_d<true>(prm, pl.GT, D, B, rope_positions, pl.grid, st)
                : launch_decode_split_d<false>(prm, pl.GT, D, B, rope_positions, pl.grid, st);
  }
  const size_t need = decode_ws_bytes(pl, B, Hq, D);
  if (ws == nullptr || ws_bytes < need || !aligned16(ws))
    return fail(DU_ERR_WORKSPACE, "decode workspace of " + std::to_string(need) +
                                      " bytes (16-byte aligned) is required");
  uint8_t* w8 = static_cast<uint8_t*>(ws);
  float* o_part = reinterpret_cast<float*>(w8 + du::DECODE_CNT_BYTES);
  const size_t o_bytes = static_cast<size_t>(rows) * pl.n_split * D * sizeof(float);
  float* l_part = reinterpret_cast<float*>(w8 + du::DECODE_CNT_BYTES + ((o_bytes + 255) / 256) * 256);
  prm.mode = 1;
  prm.o_part = o_part;
  prm.lse_part = l_part;
  // The tensor-core decode merges in the split kernel (ticket per unit, no merge launch).
  if (decode_use_tc(D, pl.GT) && pl.n_units < du::DECODE_CNT_DONE) {
    prm.unit_cnt = reinterpret_cast<int*>(w8);
    prm.fused_merge = 1;
    if (out != nullptr) {
      prm.fin_out = out;
      prm.fin_kind = bf16 ? 1 : 0;
    } else {
      prm.fin_out = out_f32;
      prm.fin_kind = 2;
      prm.fin_lse = lse_f32;
    }
    return bf16 ? launch_decode_split_d<true>(prm, pl.GT, D, B, rope_positions, pl.grid, st)
                : launch_decode_split_d<false>(prm, pl.GT, D, B, rope_positions, pl.grid, st);
  }
  rc = bf16 ? launch_decode_split_d<true>(prm, pl.GT, D, B, rope_positions, pl.grid, st)
            : launch_decode_split_d<false>(prm, pl.GT, D, B, rope_positions, pl.grid, st);
  if (rc != DU_OK) return rc;
  if (out != nullptr)
    return launch_merge(o_part, l_part, pl.n_split, static_cast<int>(rows), D, D,
                        static_cast<long long>(pl.n_split) * D, 1, pl.n_split, out, dtype, nullptr,
                        st);
  return launch_merge(o_part, l_part, pl.n_split, static_cast<int>(rows), D, D,
                      static_cast<long long>(pl.n_split) * D, 1, pl.n_split, out_f32, DU_DTYPE_F32,
                      lse_f32, st);
}

// Rows [r0, r1) of a T-row tensor rotate at pos_offset + t below pos_split and
// pos_offset1 + (t - pos_split) from it: every position they reach must be a table row.
bool segments_covered(int T, long long split, long long off0, long long off1, long long r0,
                      long long r1, long long rope_positions) {
  (void)T;
  if (r0 >= r1) return true;
  if (r0 < split) {  // first segment: rows [r0, min(r1, split))
    const long long hi = (r1 < split ? r1 : split) - 1;
    if (off0 + r0 < 0 || off0 + hi >= rope_positions) return false;
  }
  if (r1 > split) {  // second segment: rows [max(r0, split), r1)
    const long long lo = (r0 > split ? r0 : split) - split;
    if (off1 + lo < 0 || off1 + (r1 - 1 - split) >= rope_positions) return false;
  }
  return true;
}

template <bool BF16>
int launch_fa_d(const void* q, const void* k_rot, const void* v, const du::PrefillParams& prm,
                int B, int Tkv, int D, cudaStream_t st) {
  switch (D) {
    case 16: return launch_fa_t<16, BF16, true>(q, k_rot, v, prm, B, Tkv, st);
    case 32: return launch_fa_t<32, BF16, true>(q, k_rot, v, prm, B, Tkv, st);
    case 64: return launch_fa_t<64, BF16, true>(q, k_rot, v, prm, B, Tkv, st);
    case 128: return launch_fa_t<128, BF16, true>(q, k_rot, v, prm, B, Tkv, st);
    default: return fail(DU_ERR_UNSUPPORTED, "block prefill supports head_dim 16, 32, 64, 128");
  }
}

int prefill_block_impl(const void* q, const void* k_rot, const void* v, const void* cos,
                       const void* sin, void* out, float* lse, float* acc_o, float* acc_lse,
                       int acc_mode, int B, int Hq, int Hkv, int T, int Tkv, int q_row0, int Tq,
                       int Tk, int causal, long long pos_split, long long pos_off0,
                       long long pos_off1, int D, int dtype, float scale, long long rope_positions,
                       cudaStream_t st) {
  int rc = check_common(B, Hq, Hkv, T, D, dtype);
  if (rc != DU_OK) return rc;
  if (D > 128) return fail(DU_ERR_UNSUPPORTED, "block prefill supports head_dim 16, 32, 64, 128");
  if (!q || !k_rot || !v || !cos || !sin || !out || !lse)
    return fail(DU_ERR_INVALID, "null pointer argument");
  if (!aligned16(q) || !aligned16(k_rot) || !aligned16(v) || !aligned16(cos) || !aligned16(sin) ||
      !aligned16(out))
    return fail(DU_ERR_INVALID, "q, k_rot, v, out and rope tables must be 16-byte aligned");
  if (acc_mode < 0 || acc_mode > 2) return fail(DU_ERR_INVALID, "acc_mode must be 0, 1 or 2");
  if (acc_mode != 0 && (!acc_o || !acc_lse || !aligned16(acc_o)))
    return fail(DU_ERR_INVALID, "accumulators are required (acc_o 16-byte aligned) for acc_mode 1, 2");
  if (Tkv <= 0 || Tk <= 0 || Tk > Tkv) return fail(DU_ERR_INVALID, "need 0 < Tk <= Tkv");
  if (q_row0 < 0 || Tq <= 0 || static_cast<long long>(q_row0) + Tq > T)
    return fail(DU_ERR_INVALID, "query rows [q_row0, q_row0 + Tq) must lie in [0, T)");
  if (causal && (q_row0 != 0 || Tq != T || Tk != T))
    return fail(DU_ERR_INVALID, "a causal block covers the whole query and key range (q_row0 = 0, Tq = Tk = T)");
  if (pos_split < 0) return fail(DU_ERR_INVALID, "pos_split must be non-negative");
  if (!segments_covered(T, pos_split, pos_off0, pos_off1, q_row0, static_cast<long long>(q_row0) + Tq,
                        rope_positions))
    return fail(DU_ERR_INVALID, "rope tables do not cover the query positions");
  if (!(scale > 0.f)) return fail(DU_ERR_INVALID, "scale must be positive");
  du::PrefillParams prm{};
  prm.cos = cos;
  prm.sin = sin;
  prm.out = out;
  prm.lse = lse;
  prm.Hq = Hq;
  prm.Hkv = Hkv;
  prm.T = T;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.q_row0 = q_row0;
  prm.Tq = Tq;
  prm.Tk = Tk;
  prm.causal = causal ? 1 : 0;
  prm.pos_split = pos_split;
  prm.pos_off0 = pos_off0;
  prm.pos_off1 = pos_off1;
  prm.acc_o = acc_o;
  prm.acc_lse = acc_lse;
  prm.acc_mode = acc_mode;
  return dtype == DU_DTYPE_BF16 ? launch_fa_d<true>(q, k_rot, v, prm, B, Tkv, D, st)
                                : launch_fa_d<false>(q, k_rot, v, prm, B, Tkv, D, st);
}

// Workspace of du_decode_kvcache: chunk offsets [B + 1] (int64), {len, qpos} [B] (int2), then
// the fragment-slot partials, o [(units + grid) * GT, D] and lse [(units + grid) * GT] fp32.
struct KvcacheLayout {
  size_t pre, lenq, flag, o, lse, total;
};

KvcacheLayout kvcache_layout(const DecodePlan& pl, int B, int D, int grid) {
  auto up = [](size_t x) { return ((x + 255) / 256) * 256; };
  KvcacheLayout ly{};
  const size_t slots = (static_cast<size_t>(pl.n_units) + grid) * pl.GT;
  ly.pre = 0;
  ly.lenq = up(sizeof(long long) * (static_cast<size_t>(B) + 1));
  ly.flag = ly.lenq + up(sizeof(int) * 2 * static_cast<size_t>(B));
  ly.o = ly.flag + 256;
  ly.lse = ly.o + up(slots * D * sizeof(float));
  ly.total = ly.lse + slots * sizeof(float);
  return ly;
}

int kvcache_grid(const DecodePlan& pl) { return sm_count() * decode_residency(pl.GT); }

int decode_kvcache_impl(const void* q, const void* k_new, const void* v_new, void* kc, void* vc,
                        const int* seqlens, const void* cos, const void* sin, void* out, int B,
                        int Hq, int Hkv, int L, int D, int dtype, float scale,
                        long long rope_positions, void* ws, size_t ws_bytes, cudaStream_t st) {
  int rc = check_common(B, Hq, Hkv, L, D, dtype);
  if (rc != DU_OK) return rc;
  if (!q || !kc || !vc || !seqlens || !cos || !sin || !out)
    return fail(DU_ERR_INVALID, "null pointer argument");
  if ((k_new == nullptr) != (v_new == nullptr))
    return fail(DU_ERR_INVALID, "k_new and v_new must be given together");
  const bool append = k_new != nullptr;
  if (!aligned16(q) || !aligned16(kc) || !aligned16(vc) || !aligned16(cos) || !aligned16(sin) ||
      (append && (!aligned16(k_new) || !aligned16(v_new))))
    return fail(DU_ERR_INVALID, "q, k_new, v_new, caches and rope tables must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(seqlens) & 3u) != 0)
    return fail(DU_ERR_INVALID, "cache_seqlens must be 4-byte aligned");
  if (rope_positions < 1) return fail(DU_ERR_INVALID, "rope tables must have at least one row");
  if (!(scale > 0.f)) return fail(DU_ERR_INVALID, "scale must be positive");
  const DecodePlan pl = plan_decode(B, Hq, Hkv, L, D);
  const int grid = kvcache_grid(pl);
  const KvcacheLayout ly = kvcache_layout(pl, B, D, grid);
  if (ws == nullptr || ws_bytes < ly.total || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0)
    return fail(DU_ERR_WORKSPACE, "decode_kvcache workspace of " + std::to_string(ly.total) +
                                      " bytes (256-byte aligned) is required");
  uint8_t* w8 = static_cast<uint8_t*>(ws);
  du::DecodePrepParams pp{};
  pp.seqlens = seqlens;
  pp.k_new = k_new;
  pp.v_new = v_new;
  pp.k_cache = kc;
  pp.v_cache = vc;
  pp.pre = reinterpret_cast<long long*>(w8 + ly.pre);
  pp.lenq = reinterpret_cast<int2*>(w8 + ly.lenq);
  pp.B = B;
  pp.Hkv = Hkv;
  pp.L = L;
  pp.D = D;
  pp.CK = decode_chunk(D, pl.GT, true);  // the chunk of the kernel the walk runs on
  pp.ub = Hkv * pl.n_gchunk;
  pp.append = append ? 1 : 0;
  pp.rope_positions = rope_positions;
  pp.vl_whole = reinterpret_cast<int*>(w8 + ly.flag);
  // Whole units are considered under the unit-count rule of plan_decode; the prep kernel then
  // checks that the lengths spread the load evenly.
  pp.whole_ok = (pl.GT <= 2 && 4LL * pl.n_units >= 3LL * sm_count()) ? 1 : 0;
  pp.grid = grid;
  // One CTA scans the lengths; the append spreads over enough CTAs for a 16-byte piece each.
  const long long pieces = append ? static_cast<long long>(B) * Hkv * (D / 8) : 0;
  long long pgrid = (pieces + 255) / 256;
  if (pgrid < 1) pgrid = 1;
  if (pgrid > 2LL * sm_count()) pgrid = 2LL * sm_count();
  cudaError_t e = launch_kernel(du::decode_prep_kernel, static_cast<unsigned>(pgrid), 256, 0, st,
                                false, pp);
  if (e != cudaSuccess) return cuda_fail(e, "decode prep launch");
  du::DecodeParams prm{};
  prm.q = q;
  prm.k = kc;
  prm.v = vc;
  prm.cos = cos;
  prm.sin = sin;
  prm.Hq = Hq;
  prm.Hkv = Hkv;
  prm.L = L;
  prm.G = Hq / Hkv;
  prm.n_gchunk = pl.n_gchunk;
  prm.n_split = 2;  // partials are written; slots come from the fragment walk
  prm.n_units = pl.n_units;
  prm.cpu = 0;
  prm.total_chunks = 0;
  prm.q_pos = 0;
  prm.kv_pos_offset = 0;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.mode = 1;
  prm.o_part = reinterpret_cast<float*>(w8 + ly.o);
  prm.lse_part = reinterpret_cast<float*>(w8 + ly.lse);
  prm.pre = pp.pre;
  prm.lenq = pp.lenq;
  prm.vl_whole = pp.vl_whole;
  prm.out = out;
  prm.B = B;
  prm.ub = pp.ub;
  prm.varlen = 1;
  const bool bf16 = dtype == DU_DTYPE_BF16;
  rc = bf16 ? launch_decode_split_d<true>(prm, pl.GT, D, B, rope_positions, grid, st)
            : launch_decode_split_d<false>(prm, pl.GT, D, B, rope_positions, grid, st);
  if (rc != DU_OK) return rc;
  e = launch_kernel(du::decode_merge_varlen_kernel, static_cast<unsigned>(static_cast<long long>(B) * Hq),
                    128, 0, st, true, static_cast<const float*>(prm.o_part),
                    static_cast<const float*>(prm.lse_part), static_cast<const long long*>(pp.pre),
                    static_cast<const int*>(pp.vl_whole), Hq, Hkv, pl.GT, pp.ub, B, D, grid, out,
                    dtype);
  if (e != cudaSuccess) return cuda_fail(e, "decode merge launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "decode merge launch");
  return DU_OK;
}

}  // namespace

extern "C" {

int du_version(void) { return 100; }

const char* du_last_error(void) { return g_last_error.c_str(); }

size_t du_prefill_workspace_size(int B, int Hq, int Hkv, int T, int D) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || T <= 0 || Hq % Hkv != 0 || !valid_head_dim(D)) return 0;
  return prefill_ws_bytes(B, Hkv, T, D);
}

int du_prefill(const void* q, const void* k, const void* v, const void* cos, const void* sin,
               void* out, float* lse, int B, int Hq, int Hkv, int T, int D, int dtype,
               float scale, long long rope_positions, void* workspace, size_t workspace_bytes,
               void* stream) {
  g_last_error.clear();
  int rc = check_common(B, Hq, Hkv, T, D, dtype);
  if (rc != DU_OK) return rc;
  if (!q || !k || !v || !cos || !sin || !out || !lse)
    return fail(DU_ERR_INVALID, "null pointer argument");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(cos) || !aligned16(sin) ||
      !aligned16(out) || !aligned16(lse))
    return fail(DU_ERR_INVALID, "all tensors must be 16-byte aligned");
  if (rope_positions < T) return fail(DU_ERR_INVALID, "rope tables have fewer than T positions");
  if (!(scale > 0.f)) return fail(DU_ERR_INVALID, "scale must be positive");
  if ((T + 127) / 128 > 65535) return fail(DU_ERR_UNSUPPORTED, "sequence length too large");
  const size_t need = prefill_ws_bytes(B, Hkv, T, D);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)))
    return fail(DU_ERR_WORKSPACE, "prefill workspace of " + std::to_string(need) +
                                      " bytes (16-byte aligned) is required");
  du::PrefillParams prm{};
  prm.cos = cos;
  prm.sin = sin;
  prm.out = out;
  prm.lse = lse;
  prm.Hq = Hq;
  prm.Hkv = Hkv;
  prm.T = T;
  prm.n_qtiles = (T + 127) / 128;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.q_row0 = 0;
  prm.Tq = T;
  prm.Tk = T;
  prm.causal = 1;
  prm.pos_split = T;
  prm.pos_off0 = 0;
  prm.pos_off1 = 0;
  prm.acc_mode = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = dtype == DU_DTYPE_BF16;
  void* ws = workspace;
  switch (D) {
    case 16: return bf16 ? launch_prefill_t<16, true>(q, k, v, prm, B, rope_positions, ws, st)
                         : launch_prefill_t<16, false>(q, k, v, prm, B, rope_positions, ws, st);
    case 32: return bf16 ? launch_prefill_t<32, true>(q, k, v, prm, B, rope_positions, ws, st)
                         : launch_prefill_t<32, false>(q, k, v, prm, B, rope_positions, ws, st);
    case 64: return bf16 ? launch_prefill_t<64, true>(q, k, v, prm, B, rope_positions, ws, st)
                         : launch_prefill_t<64, false>(q, k, v, prm, B, rope_positions, ws, st);
    case 128: return bf16 ? launch_prefill_t<128, true>(q, k, v, prm, B, rope_positions, ws, st)
                          : launch_prefill_t<128, false>(q, k, v, prm, B, rope_positions, ws, st);
    case 256: return bf16 ? launch_prefill_t<256, true>(q, k, v, prm, B, rope_positions, ws, st)
                          : launch_prefill_t<256, false>(q, k, v, prm, B, rope_positions, ws, st);
    default: return fail(DU_ERR_UNSUPPORTED, "head_dim must be one of 16, 32, 64, 128, 256");
  }
}

int du_rope(const void* x, const void* cos, const void* sin, void* out, int B, int H, int T, int D,
            int dtype, int out_dtype, long long pos_offset, long long rope_positions, int backward,
            void* stream) {
  return du_rope_segments(x, cos, sin, out, B, H, T, D, dtype, out_dtype, T, pos_offset, 0,
                          rope_positions, backward, stream);
}

int du_rope_segments(const void* x, const void* cos, const void* sin, void* out, int B, int H,
                     int T, int D, int dtype, int out_dtype, long long pos_split,
                     long long pos_offset, long long pos_offset1, long long rope_positions,
                     int backward, void* stream) {
  g_last_error.clear();
  if (B <= 0 || H <= 0 || T <= 0) return fail(DU_ERR_INVALID, "batch, heads, and sequence length must be positive");
  if (!valid_head_dim(D))
    return fail(DU_ERR_UNSUPPORTED, "head_dim must be a power of two between 16 and 256");
  if (dtype != DU_DTYPE_F16 && dtype != DU_DTYPE_BF16)
    return fail(DU_ERR_INVALID, "dtype must be DU_DTYPE_F16 or DU_DTYPE_BF16");
  if (out_dtype != dtype && out_dtype != DU_DTYPE_F16)
    return fail(DU_ERR_INVALID, "out_dtype must be the input dtype or DU_DTYPE_F16");
  if (!x || !cos || !sin || !out) return fail(DU_ERR_INVALID, "null pointer argument");
  if (!aligned16(x) || !aligned16(cos) || !aligned16(sin) || !aligned16(out))
    return fail(DU_ERR_INVALID, "all tensors must be 16-byte aligned");
  if (pos_split < 0 || pos_split > T) return fail(DU_ERR_INVALID, "pos_split must be in [0, T]");
  if (!segments_covered(T, pos_split, pos_offset, pos_offset1, 0, T, rope_positions))
    return fail(DU_ERR_INVALID, "rope tables do not cover the positions");
  du::RopeParams rp{};
  rp.x = x;
  rp.cos = cos;
  rp.sin = sin;
  rp.out = out;
  rp.rows = static_cast<long long>(B) * H * T;
  rp.T = T;
  rp.D = D;
  rp.pos_offset = pos_offset;
  rp.pos_split = pos_split;
  rp.pos_offset1 = pos_offset1;
  return launch_rope(rp, dtype == DU_DTYPE_BF16, out_dtype == DU_DTYPE_F16 && dtype != DU_DTYPE_F16,
                     backward != 0, static_cast<cudaStream_t>(stream));
}

size_t du_decode_workspace_size(int B, int Hq, int Hkv, int L, int D) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || L <= 0 || Hq % Hkv != 0 || !valid_head_dim(D)) return 0;
  return decode_ws_bytes(plan_decode(B, Hq, Hkv, L, D), B, Hq, D);
}

int du_decode(const void* q, const void* k_cache, const void* v_cache, const void* cos,
              const void* sin, void* out, int B, int Hq, int Hkv, int L, int D, int dtype,
              float scale, long long rope_positions, void* workspace, size_t workspace_bytes,
              void* stream) {
  g_last_error.clear();
  if (out == nullptr) return fail(DU_ERR_INVALID, "null pointer argument");
  return decode_impl(q, k_cache, v_cache, cos, sin, out, nullptr, nullptr, B, Hq, Hkv, L, D,
                     dtype, scale, L, 0, rope_positions, workspace, workspace_bytes,
                     static_cast<cudaStream_t>(stream));
}

int du_prefill_block(const void* q, const void* k_rot, const void* v, const void* cos,
                     const void* sin, void* out, float* lse, float* acc_o, float* acc_lse,
                     int acc_mode, int B, int Hq, int Hkv, int T, int Tkv, int q_row0, int Tq,
                     int Tk, int causal, long long pos_split, long long pos_off0,
                     long long pos_off1, int D, int dtype, float scale, long long rope_positions,
                     void* stream) {
  g_last_error.clear();
  return prefill_block_impl(q, k_rot, v, cos, sin, out, lse, acc_o, acc_lse, acc_mode, B, Hq, Hkv,
                            T, Tkv, q_row0, Tq, Tk, causal, pos_split, pos_off0, pos_off1, D,
                            dtype, scale, rope_positions, static_cast<cudaStream_t>(stream));
}

size_t du_decode_kvcache_workspace_size(int B, int Hq, int Hkv, int L, int D) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || L <= 0 || Hq % Hkv != 0 || !valid_head_dim(D)) return 0;
  const DecodePlan pl = plan_decode(B, Hq, Hkv, L, D);
  return kvcache_layout(pl, B, D, kvcache_grid(pl)).total;
}

int du_decode_kvcache(const void* q, const void* k_new, const void* v_new, void* k_cache,
                      void* v_cache, const int* cache_seqlens, const void* cos, const void* sin,
                      void* out, int B, int Hq, int Hkv, int L, int D, int dtype, float scale,
                      long long rope_positions, void* workspace, size_t workspace_bytes,
                      void* stream) {
  g_last_error.clear();
  return decode_kvcache_impl(q, k_new, v_new, k_cache, v_cache, cache_seqlens, cos, sin, out, B,
                             Hq, Hkv, L, D, dtype, scale, rope_positions, workspace,
                             workspace_bytes, static_cast<cudaStream_t>(stream));
}

int du_decode_partial(const void* q, const void* k_shard, const void* v_shard, const void* cos,
                      const void* sin, float* out_f32, float* lse_f32, int B, int Hq, int Hkv,
                      int L_shard, int D, int dtype, float scale, long long q_pos,
                      long long kv_pos_offset, long long rope_positions, void* workspace,
                      size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (out_f32 == nullptr || lse_f32 == nullptr)
    return fail(DU_ERR_INVALID, "null pointer argument");
  return decode_impl(q, k_shard, v_shard, cos, sin, nullptr, out_f32, lse_f32, B, Hq, Hkv,
                     L_shard, D, dtype, scale, q_pos, kv_pos_offset, rope_positions, workspace,
                     workspace_bytes, static_cast<cudaStream_t>(stream));
}

int du_merge_partials(const float* o_parts, const float* lse_parts, int R, int rows, int D,
                      long long o_stride_r, long long o_stride_row, long long lse_stride_r,
                      long long lse_stride_row, void* out, int out_dtype, float* lse_out,
                      void* stream) {
  g_last_error.clear();
  if (R <= 0 || rows <= 0 || D <= 0) return fail(DU_ERR_INVALID, "R, rows and D must be positive");
  if (!o_parts || !lse_parts || !out) return fail(DU_ERR_INVALID, "null pointer argument");
  if (out_dtype != DU_DTYPE_F16 && out_dtype != DU_DTYPE_BF16 && out_dtype != DU_DTYPE_F32)
    return fail(DU_ERR_INVALID, "out_dtype must be DU_DTYPE_F16, BF16 or F32");
  return launch_merge(o_parts, lse_parts, R, rows, D, o_stride_r, o_stride_row, lse_stride_r,
                      lse_stride_row, out, out_dtype, lse_out, static_cast<cudaStream_t>(stream));
}


// --------------------------------------------------------------------------------------------
// Peer-memory exchange of sequence-split decode partials (exchange_sm100.cuh)
// --------------------------------------------------------------------------------------------
size_t du_exchange_buffer_bytes(int world, int rows, int D) {
  if (world < 1 || world > du::XCH_MAX_WORLD || rows <= 0 || D <= 0 || D % 4 != 0) return 0;
  return du::XchLayout::bytes(world, rows, D);
}

int du_exchange_buffer_alloc(size_t bytes, void** ptr) {
  g_last_error.clear();
  if (ptr == nullptr || bytes == 0) return fail(DU_ERR_INVALID, "null pointer or zero size");
  *ptr = nullptr;
  // Its own allocation, so that a CUDA IPC handle covers exactly this buffer.
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(exchange buffer)");
  e = cudaMemset(*ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return cuda_fail(e, "cudaMemset(exchange buffer)");
  }
  return DU_OK;
}

int du_exchange_buffer_free(void* ptr) {
  g_last_error.clear();
  if (ptr == nullptr) return DU_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? DU_OK : cuda_fail(e, "cudaFree(exchange buffer)");
}

int du_ipc_get_handle(const void* ptr, void* handle64) {
  g_last_error.clear();
  if (ptr == nullptr || handle64 == nullptr) return fail(DU_ERR_INVALID, "null pointer argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle64, &h, sizeof(h));
  return DU_OK;
}

int du_ipc_open_handle(const void* handle64, void** ptr) {
  g_last_error.clear();
  if (ptr == nullptr || handle64 == nullptr) return fail(DU_ERR_INVALID, "null pointer argument");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? DU_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int du_ipc_close_handle(void* ptr) {
  g_last_error.clear();
  if (ptr == nullptr) return DU_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? DU_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int du_exchange_merge(const float* o_local, const float* lse_local, void* const* buffers, int world,
                      int rank, int rows, int D, void* out, int out_dtype, float* lse_out,
                      void* stream) {
  g_last_error.clear();
  if (world < 1 || world > du::XCH_MAX_WORLD)
    return fail(DU_ERR_UNSUPPORTED, "world must be between 1 and " + std::to_string(du::XCH_MAX_WORLD));
  if (rank < 0 || rank >= world) return fail(DU_ERR_INVALID, "rank must be in [0, world)");
  if (rows <= 0 || D <= 0 || D % 4 != 0) return fail(DU_ERR_INVALID, "rows must be positive and D a multiple of 4");
  if (!o_local || !lse_local || !buffers || !out) return fail(DU_ERR_INVALID, "null pointer argument");
  if (!aligned16(o_local)) return fail(DU_ERR_INVALID, "o_local must be 16-byte aligned");
  if (out_dtype != DU_DTYPE_F16 && out_dtype != DU_DTYPE_BF16 && out_dtype != DU_DTYPE_F32)
    return fail(DU_ERR_INVALID, "out_dtype must be DU_DTYPE_F16, BF16 or F32");
  du::XchParams p{};
  for (int r = 0; r < world; ++r) {
    if (buffers[r] == nullptr || reinterpret_cast<uintptr_t>(buffers[r]) % 256 != 0)
      return fail(DU_ERR_INVALID, "every exchange buffer must be non-null and 256-byte aligned");
    p.peer[r] = static_cast<uint8_t*>(buffers[r]);
  }
  p.o_loc = o_local;
  p.lse_loc = lse_local;
  p.world = world;
  p.rank = rank;
  p.rows = rows;
  p.D = D;
  const int grid0 = rows < du::XCH_MAX_CTAS ? rows : du::XCH_MAX_CTAS;
  p.rpc = (rows + grid0 - 1) / grid0;
  const int grid = (rows + p.rpc - 1) / p.rpc;
  p.out = out;
  p.out_kind = out_dtype == DU_DTYPE_F32 ? 2 : (out_dtype == DU_DTYPE_BF16 ? 1 : 0);
  p.lse_out = lse_out;
  du::xch_merge_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? DU_OK : cuda_fail(e, "exchange merge launch");
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Decode without device allocation (du_decode_noalloc)
// ---------------------------------------------------------------------------------------------
// For callers that cannot allocate device memory (a foreign runtime binding this C ABI with no
// CUDA allocator, or a serving loop that must not call cudaMalloc once running), the split-KV
// partials live in this fixed array instead of a caller-provided workspace. It is part of the
// library's device image, so every GPU that loads the library holds these 4 MiB until exit.
// In host code `g_du_noalloc_scratch` is only a host-side stand-in for the symbol; the device
// address comes from cudaGetSymbolAddress below, once per device.
static __device__ __align__(256) unsigned char g_du_noalloc_scratch[DU_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
// Per device: the array's address and the id of the context it was looked up in. A device's
// primary context can be destroyed and created again (cudaDeviceReset), which loads this
// library's device image afresh, possibly at another address: the id tells the two apart.
struct NoallocSlot {
  unsigned long long ctx_id;
  void* ptr;
};
NoallocSlot g_noalloc_slot[kNoallocMaxDevices] = {};

// Unique id of the calling thread's current context (false if none is current or the driver
// entry points are unavailable).
bool current_context_id(unsigned long long* id) {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  if (get_current == nullptr || get_id == nullptr) return false;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
  return get_id(ctx, id) == CUDA_SUCCESS;
}

// Device address of the scratch array on the current device. It is looked up with
// cudaGetSymbolAddress (the return code checked) on the first call in each context of the
// device, with that device current, and reused while the same context stays current; the
// first call on a device must therefore not happen inside a stream capture.
int noalloc_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kNoallocMaxDevices)
    return fail(DU_ERR_UNSUPPORTED, "device index beyond the no-allocation scratch table");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  unsigned long long id = 0;
  NoallocSlot& slot = g_noalloc_slot[dev];
  if (slot.ptr != nullptr && current_context_id(&id) && id == slot.ctx_id) {
    *out = slot.ptr;
    return DU_OK;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_du_noalloc_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-allocation scratch)");
  // The lookup made the device's context current; without an id the address is not cached.
  if (current_context_id(&id)) {
    slot.ctx_id = id;
    slot.ptr = p;
  } else {
    slot.ptr = nullptr;
  }
  *out = p;
  return DU_OK;
}

}  // namespace

extern "C" {

int du_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const void* cos,
                      const void* sin, void* out, int B, int Hq, int Hkv, int L, int D,
                      int dtype, float scale, long long rope_positions, void* stream) {
  g_last_error.clear();
  if (out == nullptr) return fail(DU_ERR_INVALID, "null pointer argument");
  int rc = check_common(B, Hq, Hkv, L, D, dtype);
  if (rc != DU_OK) return rc;
  const size_t need = decode_ws_bytes(plan_decode(B, Hq, Hkv, L, D), B, Hq, D);
  if (need > DU_NOALLOC_SCRATCH_BYTES)
    return fail(DU_ERR_WORKSPACE, "this decode needs " + std::to_string(need) +
                                      " bytes of split scratch; du_decode_noalloc holds at most " +
                                      std::to_string(DU_NOALLOC_SCRATCH_BYTES) +
                                      " bytes (use du_decode with a workspace)");
  void* scratch = nullptr;
  if (need > 0) {
    rc = noalloc_scratch_address(&scratch);
    if (rc != DU_OK) return rc;
  }
  // Nothing is cleared here: the split kernel writes every partial before it is read, and the
  // ticket counters at the start of the array are zero at load and left zero by every call.
  // Calls sharing the array must not overlap on the GPU.
  return decode_impl(q, k_cache, v_cache, cos, sin, out, nullptr, nullptr, B, Hq, Hkv, L, D,
                     dtype, scale, L, 0, rope_positions, scratch, need,
                     static_cast<cudaStream_t>(stream));
}

#ifdef DU_TRACE
// Debug builds only: copy the prefill event trace (16 x 64 timestamps) to the host.
int du_trace_read(long long* out) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_du_trace, sizeof(long long) * 16 * 64);
  return e == cudaSuccess ? DU_OK : DU_ERR_CUDA;
}
int du_trace_reset(void) {
  static long long zeros[16 * 64] = {};
  cudaError_t e = cudaMemcpyToSymbol(g_du_trace, zeros, sizeof(zeros));
  return e == cudaSuccess ? DU_OK : DU_ERR_CUDA;
}
#endif

int du_selftest_wait_timeout(int timeout_us, void* stream) {
  g_last_error.clear();
  if (timeout_us < 1 || timeout_us > 1000000)
    return fail(DU_ERR_INVALID, "timeout_us must be in [1, 1000000]");
  du::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned long long>(timeout_us) * 1000ull);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "selftest launch");
  return DU_OK;
}

int du_read_status(unsigned int* words4, int reset) {
  g_last_error.clear();
  unsigned int h[4] = {0, 0, 0, 0};
  cudaError_t e = cudaMemcpyFromSymbol(h, g_du_status, sizeof(h));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(status)");
  if (words4 != nullptr) std::memcpy(words4, h, sizeof(h));
  if (reset) {
    const unsigned int z[4] = {0, 0, 0, 0};
    e = cudaMemcpyToSymbol(g_du_status, z, sizeof(z));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(status)");
  }
  return DU_OK;
}

}  // extern "C"
