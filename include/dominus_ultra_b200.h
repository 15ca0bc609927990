/*
 * dominus_ultra_b200.h -- C ABI of the B200 (sm_100a) fused-RoPE causal attention library.
 *
 * Plain pointers, sizes and a CUDA stream handle; no framework types. All entry points are
 * asynchronous on `stream` (a cudaStream_t passed as void*), never synchronise, and return
 * DU_OK (0) or a DU_ERR_* code; du_last_error() then describes the failure. Arguments are
 * validated before any launch.
 *
 * Layouts (row-major, contiguous, 16-byte aligned base pointers):
 *   q        [B, Hq, T, D]         k, v      [B, Hkv, T, D]
 *   cos, sin [positions, D/2]      (half-split RoPE tables, same dtype as q)
 *   out      [B, Hq, T, D]         lse       [B, Hq, T] fp32, natural log
 * Query head h reads KV head h / (Hq / Hkv). D is one of 16, 32, 64, 128, 256.
 * dtype: DU_DTYPE_F16 or DU_DTYPE_BF16 for q/k/v/cos/sin/out.
 */
#ifndef DOMINUS_ULTRA_B200_H
#define DOMINUS_ULTRA_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DU_OK 0
#define DU_ERR_INVALID 1     /* bad argument (shape, alignment, dtype, null pointer) */
#define DU_ERR_UNSUPPORTED 2 /* valid but not built (e.g. head_dim outside 16..256) */
#define DU_ERR_CUDA 3        /* a CUDA runtime / driver call failed */
#define DU_ERR_WORKSPACE 4   /* workspace missing or too small */
#define DU_ERR_TIMEOUT 5     /* a bounded device-side wait expired (see du_read_status) */
#define DU_STATUS_BAD_SEQLEN 6 /* device status only: a per-sequence cache length out of range */

#define DU_DTYPE_F16 0
#define DU_DTYPE_BF16 1
#define DU_DTYPE_F32 2

/* Library version, major * 10000 + minor * 100 + patch. */
int du_version(void);

/* Description of the last error on the calling host thread ("" if none). */
const char* du_last_error(void);

/*
 * Workspace bytes du_prefill needs for these sizes: the rotated keys R(K) as fp16
 * [B, Hkv, T, D] for head_dim <= 128, 0 for head_dim 256.
 */
size_t du_prefill_workspace_size(int B, int Hq, int Hkv, int T, int D);

/*
 * Causal fused-RoPE prefill. Replaces the launch of `prefill_kernel` in
 * `dominus_ultra_prefill` (reference dominus_ultra.py:416-501, kernel :119-285).
 * Rows use positions 0..T-1 of the tables; `rope_positions` is the table length (>= T).
 * `scale` is the softmax scale (the reference uses 1/sqrt(D), dominus_ultra.py:475).
 * For head_dim <= 128 the keys are rotated once per (b, kv head) into `workspace` (see
 * du_prefill_workspace_size; DU_ERR_WORKSPACE when missing or too small), then the attention
 * kernel reads them; queries are rotated inside the attention kernel.
 */
int du_prefill(const void* q, const void* k, const void* v, const void* cos, const void* sin,
               void* out, float* lse, int B, int Hq, int Hkv, int T, int D, int dtype,
               float scale, long long rope_positions, void* workspace, size_t workspace_bytes,
               void* stream);

/*
 * Standalone half-split RoPE over x [B, H, T, D] (contiguous): row t rotates at position
 * pos_offset + t of the tables (pos_offset + T <= rope_positions). backward != 0 applies the
 * transpose rotation (the gradient of the forward one). Replaces the launch of `_rope_kernel`
 * in the reference rope.py:19-107 (`apply_rope` / `apply_rope_backward`, :179-220), one tensor
 * per call. out_dtype is dtype, or DU_DTYPE_F16 for a bf16 input (rotated operands for an
 * fp16 tensor-core product). out may alias x.
 */
int du_rope(const void* x, const void* cos, const void* sin, void* out, int B, int H, int T, int D,
            int dtype, int out_dtype, long long pos_offset, long long rope_positions, int backward,
            void* stream);

/*
 * du_rope with two position segments: row t of [B, H, T, D] rotates at pos_offset + t for
 * t < pos_split and at pos_offset1 + (t - pos_split) from pos_split on (0 <= pos_split <= T).
 * A rank of a context-parallel prefill holds two non-adjacent chunks of the sequence along T
 * (zigzag sharding) and rotates its keys once with this. du_rope(..., pos_offset, ...) equals
 * du_rope_segments(..., pos_split = T, pos_offset, 0, ...).
 */
int du_rope_segments(const void* x, const void* cos, const void* sin, void* out, int B, int H,
                     int T, int D, int dtype, int out_dtype, long long pos_split,
                     long long pos_offset, long long pos_offset1, long long rope_positions,
                     int backward, void* stream);

/*
 * One block of a context-parallel (ring) prefill (no counterpart in the reference, which is
 * single-GPU; it generalises prefill_kernel, dominus_ultra.py:119-285, to a query range against
 * a key range). head_dim 16..128.
 *   q [B, Hq, T, D] (input dtype, rotated here), k_rot [B, Hkv, Tkv, D] fp16 keys already
 *   rotated at their absolute positions (du_rope_segments, out_dtype DU_DTYPE_F16),
 *   v [B, Hkv, Tkv, D] (input dtype).
 *   Query rows [q_row0, q_row0 + Tq) attend to keys [0, Tk). causal != 0: key t is visible to
 *   query row t' iff t <= t' (then q_row0 = 0 and Tq = Tk = T); causal == 0: every key is
 *   visible. Query row t rotates at pos_off0 + t (t < pos_split) or pos_off1 + (t - pos_split).
 *   out [B, Hq, T, D] and lse [B, Hq, T] (natural log) are written for the block's rows only.
 *   acc_mode 0: out / lse are this block's attention. acc_mode 1: they also overwrite the fp32
 *   accumulators acc_o [B, Hq, T, D] / acc_lse [B, Hq, T]. acc_mode 2: the block is LSE-merged
 *   into the accumulators (a row with acc_lse = -inf takes the block alone) and out / lse
 *   receive the merged result, so after a row's last block out / lse are final.
 */
int du_prefill_block(const void* q, const void* k_rot, const void* v, const void* cos,
                     const void* sin, void* out, float* lse, float* acc_o, float* acc_lse,
                     int acc_mode, int B, int Hq, int Hkv, int T, int Tkv, int q_row0, int Tq,
                     int Tk, int causal, long long pos_split, long long pos_off0,
                     long long pos_off1, int D, int dtype, float scale, long long rope_positions,
                     void* stream);

/*
 * Workspace bytes du_decode / du_decode_partial need for these sizes on the current device
 * (0 when every row's cache is handled by one CTA). The workspace must be zero-filled before
 * its first use (e.g. cudaMemsetAsync once after allocating it): its first 16 KB hold the
 * counters with which the CTAs of a split decode find the last fragment of each unit, and
 * every call leaves them zero again, so one buffer serves any number of calls of any shape.
 */
size_t du_decode_workspace_size(int B, int Hq, int Hkv, int L, int D);

/*
 * Decode: one new query token per (batch, head) against a KV cache of length L.
 * Replaces the launch of `decode_kernel` in `dominus_ultra_decode` (reference
 * dominus_ultra.py:504-583, kernel :288-413): the query rotates at position L, cached key j at
 * position j, no mask. q [B, Hq, D] (the reference's [B, Hq, 1, D]), caches [B, Hkv, L, D],
 * out [B, Hq, D]. `rope_positions` must be >= L + 1.
 */
int du_decode(const void* q, const void* k_cache, const void* v_cache, const void* cos,
              const void* sin, void* out, int B, int Hq, int Hkv, int L, int D, int dtype,
              float scale, long long rope_positions, void* workspace, size_t workspace_bytes,
              void* stream);

/*
 * Workspace bytes du_decode_kvcache needs for these sizes on the current device (never 0).
 */
size_t du_decode_kvcache_workspace_size(int B, int Hq, int Hkv, int L, int D);

/*
 * Decode step of a generation loop over a KV cache of capacity L with per-sequence lengths,
 * optionally appending the new token's key and value first (no counterpart in the reference:
 * its decode_kernel, dominus_ultra.py:288-413, takes one length for every sequence, the whole
 * cache, and excludes the current token, :350). cache_seqlens [B] int32 on the device holds the
 * tokens already cached per sequence, s_b; it is read on the device, so the call never
 * synchronises and a captured CUDA graph stays valid as the lengths grow.
 *   - k_new, v_new [B, Hkv, D] (or both NULL): when given, written to row s_b of k_cache /
 *     v_cache, and the query attends to keys 0..s_b; otherwise to keys 0..s_b-1.
 *   - The query rotates at position s_b, cached key j at position j (as du_decode with L = s_b).
 *   - q [B, Hq, D], caches [B, Hkv, L, D] (written only at row s_b), out [B, Hq, D].
 *   - A sequence needs 0 <= s_b, s_b + (k_new != NULL) <= L and s_b < rope_positions. A
 *     length outside that is not an argument error (the host never sees it): the sequence is
 *     treated as empty (zero output, nothing appended) and du_read_status reports code 6 with
 *     the sequence index and the length. An empty sequence without an append gives zeros.
 * workspace: du_decode_kvcache_workspace_size bytes, 256-byte aligned.
 */
int du_decode_kvcache(const void* q, const void* k_new, const void* v_new, void* k_cache,
                      void* v_cache, const int* cache_seqlens, const void* cos, const void* sin,
                      void* out, int B, int Hq, int Hkv, int L, int D, int dtype, float scale,
                      long long rope_positions, void* workspace, size_t workspace_bytes,
                      void* stream);

/*
 * Decode over one shard of a KV sequence (no counterpart in the reference, which has no
 * multi-GPU path; it generalises decode_kernel, dominus_ultra.py:288-413, by position
 * offsets). Key j of the shard rotates at kv_pos_offset + j, the query at q_pos. Writes fp32
 * out_f32 [B, Hq, D] normalised over the shard and lse_f32 [B, Hq] (natural log) for a later
 * du_merge_partials. Requires q_pos and kv_pos_offset + L_shard - 1 < rope_positions.
 */
int du_decode_partial(const void* q, const void* k_shard, const void* v_shard, const void* cos,
                      const void* sin, float* out_f32, float* lse_f32, int B, int Hq, int Hkv,
                      int L_shard, int D, int dtype, float scale, long long q_pos,
                      long long kv_pos_offset, long long rope_positions, void* workspace,
                      size_t workspace_bytes, void* stream);

/*
 * LSE-weighted merge of R partial results per row (no counterpart in the reference):
 * lse = log(sum_r exp(lse_r)), out = sum_r exp(lse_r - lse) * o_r.
 * Partial r of row i lives at o_parts[r * o_stride_r + i * o_stride_row + d] and
 * lse_parts[r * lse_stride_r + i * lse_stride_row] (strides in elements).
 * out [rows, D] in out_dtype (DU_DTYPE_F16 / BF16 / F32); lse_out [rows] may be NULL.
 */
int du_merge_partials(const float* o_parts, const float* lse_parts, int R, int rows, int D,
                      long long o_stride_r, long long o_stride_row, long long lse_stride_r,
                      long long lse_stride_row, void* out, int out_dtype, float* lse_out,
                      void* stream);

/*
 * Collective + merge step of the sequence-split decode over NVLink peer memory (no counterpart
 * in the reference, which runs on one GPU; it replaces the NCCL all-gather of the packed
 * partials followed by du_merge_partials). Every rank of one node owns an exchange buffer of
 * du_exchange_buffer_bytes(world, rows, D) bytes from du_exchange_buffer_alloc (zero-filled, its
 * own cudaMalloc allocation so that a CUDA IPC handle covers it), publishes its handle
 * (du_ipc_get_handle, 64 bytes) and opens the others' (du_ipc_open_handle). du_exchange_merge
 * then takes this rank's fp32 partial (o_local [rows, D], lse_local [rows], e.g. from
 * du_decode_partial), stores it into slot `rank` of every rank's buffer, waits (bounded) for the
 * other ranks' slots, and writes the LSE merge of all `world` partials into out [rows, D]
 * (out_dtype) and, when non-NULL, lse_out [rows] (natural log). buffers[r] is rank r's buffer as
 * this process maps it (its own allocation for r == rank). Every rank must make the same calls,
 * in the same order, with the same world, rows and D; a rank may run at most one call ahead of
 * another. A wait that expires is reported by du_read_status (code 5, sites 900 + rank) and
 * leaves that block's rows unwritten. world <= 8, D a multiple of 4.
 */
size_t du_exchange_buffer_bytes(int world, int rows, int D);
int du_exchange_buffer_alloc(size_t bytes, void** ptr);
int du_exchange_buffer_free(void* ptr);
int du_ipc_get_handle(const void* ptr, void* handle64);
int du_ipc_open_handle(const void* handle64, void** ptr);
int du_ipc_close_handle(void* ptr);
int du_exchange_merge(const float* o_local, const float* lse_local, void* const* buffers, int world,
                      int rank, int rows, int D, void* out, int out_dtype, float* lse_out,
                      void* stream);

/*
 * Decode that allocates nothing. No counterpart in the reference: it exists for callers that
 * cannot allocate device memory themselves -- hosts that bind this C ABI from another runtime
 * without a CUDA allocator, and serving loops that must not call cudaMalloc once they are
 * running (it can block on the device and fail under memory pressure).
 *
 * Same arguments, semantics and output as du_decode, minus the workspace: the split-KV
 * partials go to a fixed scratch array of DU_NOALLOC_SCRATCH_BYTES (4 MiB) compiled into this
 * library, which every GPU that loads the library holds until the process exits. Sizes whose
 * partials need more than that (du_decode_workspace_size above DU_NOALLOC_SCRATCH_BYTES) are
 * rejected with DU_ERR_WORKSPACE before anything is launched. On a 148-SM B200 every shape
 * with head_dim <= 128, B <= 16 and Hq <= 128 fits; large batches of many heads do not
 * (e.g. B 64, Hq 32, Hkv 8, L 8192 at head_dim 256, or B 64, Hq 128 at head_dim 128).
 * The first call on a device, and the first after its context is re-created (for instance by
 * cudaDeviceReset), looks up that device's address of the array (cudaGetSymbolAddress, with
 * the device current); make that first call before any stream capture. All calls on a device
 * share the one array, which keeps what the last call left: the partials are always written
 * before they are read, and the ticket counters at its start (with which the tensor-core
 * decode merges a unit's partials) are zero when the library loads and are returned to zero
 * by every call, so no call clears anything. Calls that may overlap on the GPU -- on
 * different streams, or from different host threads -- race on the array; serialise them.
 * Calls issued one after the other on one stream do not overlap.
 */
#define DU_NOALLOC_SCRATCH_BYTES (4u << 20)
int du_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const void* cos,
                      const void* sin, void* out, int B, int Hq, int Hkv, int L, int D,
                      int dtype, float scale, long long rope_positions, void* stream);

/*
 * Failure-detection self-test (no counterpart in the reference): launches one CTA whose
 * bounded wait can never complete -- an mbarrier nothing arrives at -- with a limit of
 * timeout_us microseconds (1..1000000). The kernel records DU_ERR_TIMEOUT in the status words
 * (wait site 200) and returns; nothing faults or hangs, and the context stays usable.
 */
int du_selftest_wait_timeout(int timeout_us, void* stream);

/*
 * Read the device status words (the first device-side error since the last reset):
 *   words[0] = 0 ok;
 *   DU_ERR_TIMEOUT: a bounded wait expired, [1] wait site, [2..3] block index;
 *   DU_STATUS_BAD_SEQLEN: du_decode_kvcache met a cache length out of range, [1] sequence
 *   index, [2] the length (as unsigned).
 * Synchronises the current device. reset != 0 clears them. Returns DU_OK or DU_ERR_CUDA.
 */
int du_read_status(unsigned int* words4, int reset);

#ifdef __cplusplus
}
#endif

#endif /* DOMINUS_ULTRA_B200_H */
