/*
 * iris_b200.h -- C ABI of the B200-native (sm_100a) INT4 paged KV-cache kernels.
 *
 * Drop-in replacement for the two device hot paths of Hunter2030ZeRo/Iris-Kernel:
 *
 *   write: src/iris_kernel/fused_kv.py:419-597 (_rope_int4_paged_append kernel,
 *          launched by fused_rope_int4_paged_append, fused_kv.py:600-780)
 *   read:  src/iris_kernel/fused_attention.py:11-220 (_int4_paged_decode_attention
 *          kernel, launched by fused_int4_paged_decode_attention, :437-525)
 *
 * All pointers are device pointers unless stated otherwise; tensors are
 * dense row-major (C-contiguous).  `stream` is a cudaStream_t (NULL = legacy
 * default stream).  Every call is asynchronous on `stream`; the return value
 * reports host-side argument/launch problems only (IRIS_OK == 0).  Problems
 * that need the data to detect (bad slots, bad page ids, ...) are OR-ed into
 * the caller's device `error_word` (int32, IRIS_ERR_* bits) by the kernels,
 * which never read or write out of bounds: offending tokens / pages are
 * skipped (write path) or replaced by page 0 (read path).
 *
 * Cache layout (identical to the reference, README.md:76-84):
 *   k_data, v_data   [num_pages, page_size, Hkv, D/2]   uint8, low nibble first,
 *                                                      signed INT4 in [-7, 7]
 *   k_scale, v_scale [num_pages, page_size, Hkv, D/32]  fp16, one per 32 values
 */
#ifndef IRIS_B200_H_
#define IRIS_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define IRIS_API __attribute__((visibility("default")))
#else
#define IRIS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes returned by the entry points ------------------------- */
#define IRIS_OK 0
#define IRIS_EINVAL 1          /* bad argument (shape / null pointer)            */
#define IRIS_EUNSUPPORTED 2    /* shape outside the kernel's supported set        */
#define IRIS_EALIGN 3          /* a pointer is not aligned as required            */
#define IRIS_ECUDA 4           /* a CUDA runtime / driver call failed             */
#define IRIS_EWORKSPACE 5      /* workspace too small                             */

/* ---- bits OR-ed into the device error word ------------------------------ */
#define IRIS_ERR_SLOT_RANGE 0x1        /* slot >= num_pages*page_size        (IndexError) */
#define IRIS_ERR_POS_NEGATIVE 0x2      /* position < 0                       (IndexError) */
#define IRIS_ERR_POS_RANGE 0x4         /* position >= max_position           (IndexError) */
#define IRIS_ERR_DUP_SLOT 0x8          /* two tokens target one slot         (ValueError) */
#define IRIS_ERR_SEQ_LEN 0x10          /* seq_len <= 0                       (ValueError) */
#define IRIS_ERR_BLOCK_TABLE 0x20      /* block_table row shorter than needed (ValueError) */
#define IRIS_ERR_PAGE_ID 0x40          /* page id outside [0, num_pages)     (IndexError) */
#define IRIS_ERR_PIPELINE_TIMEOUT 0x80 /* a bounded wait gave up             (RuntimeError) */

/* Library version (major*10000 + minor*100 + patch). */
IRIS_API int iris_b200_version(void);

/*
 * Self-test of the kernels' failure path: one thread waits, with the decode
 * pipeline's bounded wait, on a barrier phase that nothing completes, gives
 * up after limit_ns (0 < limit_ns <= 2e9) and ORs IRIS_ERR_PIPELINE_TIMEOUT
 * into *error_word.  No fault, no hang; the context stays usable.
 */
IRIS_API int iris_b200_selftest_bounded_wait(int32_t* error_word, int64_t limit_ns, void* stream);

/*
 * Self-test of the write path's division-free quantiser over its whole finite
 * domain.  For every group absmax with non-negative finite fp16 bit pattern
 * in [amax_lo, amax_hi) (0 <= amax_lo < amax_hi <= 0x7C00) and every fp16 x
 * with |x| <= amax, the append's quantiser (scale = fp16(max(amax/7, 2^-14))
 * from a Markstein-corrected reciprocal, q from a corrected reciprocal and a
 * round-half-even magic add) is compared with the reference's arithmetic in
 * IEEE operations (torch_eager_kv.py:77-86: amax / 7.0, x / scale, round,
 * clamp).  Adds to counts[0] the 8-value packed words that differ, to
 * counts[1] the amax values whose fp16 scale differs and to counts[2] the
 * words compared (device pointer to three uint64, zeroed by the caller).
 * No counterpart in the reference.
 */
IRIS_API int iris_b200_selftest_quantizer_sweep(int32_t amax_lo, int32_t amax_hi, unsigned long long* counts,
                                                void* stream);

/* Human-readable text for a status code. */
IRIS_API const char* iris_b200_status_string(int status);

/* Name and text of the last CUDA error an entry point of this library hit on
 * the calling thread ("" if none); explains an IRIS_ECUDA status. */
IRIS_API const char* iris_b200_last_cuda_error(void);

/* ======================================================================
 * WRITE PATH
 * ====================================================================== */

/* Bytes of device workspace iris_b200_append_check needs (slot bitmap). */
IRIS_API size_t iris_b200_append_check_workspace_bytes(int64_t num_pages, int32_t page_size);

/*
 * Range / duplicate validation of an append batch, on the device.  Replaces
 * the host-synchronising checks of fused_kv.py:741-759 (torch.unique +
 * three any() calls).  For every token with slot >= 0 it checks
 * slot < num_pages*page_size, 0 <= position < max_position, and that no two
 * tokens share a slot, OR-ing IRIS_ERR_* bits into *error_word.  `workspace`
 * (>= iris_b200_append_check_workspace_bytes) is cleared by this call.
 */
IRIS_API int iris_b200_append_check(const int32_t* positions, const int32_t* slot_mapping, int64_t num_tokens,
                           int64_t max_position, int64_t num_pages, int32_t page_size, void* workspace,
                           size_t workspace_bytes, int32_t* error_word, void* stream);

/*
 * Fused RoPE(K) + group-32 symmetric INT4 quantisation of K and V + low-
 * nibble-first packing + paged append.  Replaces the _rope_int4_paged_append
 * launch of fused_kv.py:766-780; bit-exact with torch_eager_append
 * (torch_eager_kv.py:110-337): identical packed bytes and fp16 scales.
 *
 *   key, value  [num_tokens, num_kv_heads, head_dim] fp16
 *   positions, slot_mapping [num_tokens] int32 (slot < 0: token skipped)
 *   cos_cache, sin_cache [max_position, head_dim/2] fp16 (rotary_dim == head_dim)
 *   head_dim % 64 == 0, group size 32.
 * Slots / positions out of range are skipped and reported in *error_word
 * (may be NULL).  Batches of more than IRIS_APPEND_INLINE_CHECK_TOKENS tokens
 * are not checked for duplicate slots here (use iris_b200_append_check first,
 * on the same stream and error word): when *error_word already holds a slot,
 * position or duplicate bit as the kernel starts, the call writes nothing, so
 * a batch the check rejected leaves the cache untouched without a host round
 * trip in between.  Batches of at most IRIS_APPEND_INLINE_CHECK_TOKENS tokens
 * get the whole iris_b200_append_check validation inside this call (one
 * launch; a batch it rejects is not written and its bits are recorded), so
 * the separate check may be skipped for them.
 */
#define IRIS_APPEND_INLINE_CHECK_TOKENS 128
IRIS_API int iris_b200_rope_int4_paged_append(const void* key, const void* value, const int32_t* positions,
                                     const int32_t* slot_mapping, const void* cos_cache, const void* sin_cache,
                                     void* k_data, void* v_data, void* k_scale, void* v_scale, int64_t num_tokens,
                                     int32_t num_kv_heads, int32_t head_dim, int64_t max_position,
                                     int64_t num_pages, int32_t page_size, int32_t* error_word, void* stream);

/*
 * Group-32 symmetric INT4 quantisation + low-nibble-first packing of a
 * contiguous fp16 tensor, without RoPE or paging.  Replaces the
 * _quantize_pack_int4_g32 launch of fused_quantize_pack_int4
 * (fused_kv.py:300-416); bit-exact with quantize_int4_groupwise + pack_int4
 * (torch_eager_kv.py:52-107).
 *
 *   x      [rows, head_dim] fp16 (rows = T * H), 16-byte aligned
 *   packed [rows, head_dim/2] uint8, 16-byte aligned
 *   scales [rows, head_dim/32] fp16
 *   head_dim a multiple of 32 (the Python wrapper keeps the reference's
 *   multiple-of-64 rule).
 */
IRIS_API int iris_b200_int4_quantize_pack(const void* x, void* packed, void* scales, int64_t rows, int32_t head_dim,
                                          void* stream);

/*
 * FP16 paged append (the unquantised baseline write path): RoPE over the
 * first rotary_dim dims of K (fp16 rounding after every operation, the rest
 * of K passed through) and V copied, into k_cache / v_cache
 * [num_pages, page_size, num_kv_heads, head_dim] fp16.  Replaces the
 * _rope_fp16_paged_append launch of fused_rope_fp16_append
 * (fused_kv.py:153-297); bit-exact with the reference test's eager
 * expectation (apply_rope, torch_eager_kv.py:6-49, then a scatter).
 * rotary_dim even and <= head_dim; slot < 0 skips the token.  Run
 * iris_b200_append_check first on the same stream and error word: a batch it
 * rejects is not written (as for the INT4 append).  As for the INT4 append,
 * batches of at most IRIS_APPEND_INLINE_CHECK_TOKENS tokens are validated
 * inside this call, and the separate check may be skipped for them.
 */
IRIS_API int iris_b200_rope_fp16_paged_append(const void* key, const void* value, const int32_t* positions,
                                              const int32_t* slot_mapping, const void* cos_cache,
                                              const void* sin_cache, void* k_cache, void* v_cache, int64_t num_tokens,
                                              int32_t num_kv_heads, int32_t head_dim, int32_t rotary_dim,
                                              int64_t max_position, int64_t num_pages, int32_t page_size,
                                              int32_t* error_word, void* stream);

/* ======================================================================
 * READ PATH
 * ====================================================================== */

/* Output forms of the decode. */
#define IRIS_DECODE_OUT_FP16 0 /* output [B, Hq, D] fp16 = softmax(QK^T) V (reference form) */
#define IRIS_DECODE_OUT_LSE 1  /* out_o [B, Hq, D] fp32 normalised + out_lse [B, Hq] fp32,
                                  log2-sum-exp2 of the scaled logits (for split-context merge) */

/* Bytes of device workspace iris_b200_int4_paged_decode needs. */
IRIS_API size_t iris_b200_decode_workspace_bytes(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                        int32_t device);

/*
 * INT4 paged decode attention (one query token per sequence, GQA/MQA/MHA).
 * Replaces the _int4_paged_decode_attention launch of
 * fused_attention.py:508-524 with the semantics of
 * torch_eager_int4_paged_decode_attention (torch_eager_attention.py:154-239):
 * page lookup, nibble unpack, group dequantisation, QK, softmax and PV with
 * FP32 accumulation.  Work is split over the GPU's SMs in page units
 * (split-KV); partial (m, l, O) records live in `workspace` and are merged by
 * a combine kernel in the same call.
 *
 *   query        [B, Hq, D] fp16                 D in {64, 128}
 *   block_table  int32, row b at block_table + b*block_table_stride,
 *                max_pages_per_seq valid columns
 *   seq_lens     [B] int32 (> 0)
 *   page_size 16, group 32, Hq % Hkv == 0, Hq/Hkv <= 16
 *   softmax_scale > 0 (the reference's default is D^-0.5)
 *   out_mode IRIS_DECODE_OUT_FP16: `output` [B, Hq, D] fp16, out_lse unused
 *   out_mode IRIS_DECODE_OUT_LSE : `output` [B, Hq, D] fp32, out_lse [B, Hq] fp32
 * k_data / v_data / k_scale / v_scale must be 16-byte aligned.
 */
IRIS_API int iris_b200_int4_paged_decode(const void* query, const void* k_data, const void* v_data, const void* k_scale,
                                const void* v_scale, const int32_t* block_table, int64_t block_table_stride,
                                const int32_t* seq_lens, void* output, float* out_lse, int32_t out_mode,
                                int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                int64_t num_pages, int32_t page_size, int32_t max_pages_per_seq,
                                float softmax_scale, void* workspace, size_t workspace_bytes, int32_t* error_word,
                                void* stream);

/* Bytes of device workspace iris_b200_fp16_paged_decode needs. */
IRIS_API size_t iris_b200_fp16_decode_workspace_bytes(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                                      int32_t head_dim, int32_t device);

/*
 * Matched FP16 paged decode attention (the INT4 decode's baseline).
 * Replaces the _fp16_paged_decode_attention launch of
 * fused_attention.py:528-582 with the semantics of
 * torch_eager_fp16_paged_decode_attention (torch_eager_attention.py:243-294):
 * softmax(scale * q.k) v over the sequence's fp16 K/V, FP32 accumulation.
 * Same schedule, workspace rules, outputs and error word as
 * iris_b200_int4_paged_decode, with
 *   k_cache, v_cache [num_pages, 16, Hkv, D] fp16, 16-byte aligned.
 */
IRIS_API int iris_b200_fp16_paged_decode(const void* query, const void* k_cache, const void* v_cache,
                                         const int32_t* block_table, int64_t block_table_stride,
                                         const int32_t* seq_lens, void* output, float* out_lse, int32_t out_mode,
                                         int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                         int64_t num_pages, int32_t page_size, int32_t max_pages_per_seq,
                                         float softmax_scale, void* workspace, size_t workspace_bytes,
                                         int32_t* error_word, void* stream);

/* Size of the scratch array iris_b200_int4_paged_decode_noalloc uses (32 MiB). */
#define IRIS_DECODE_NOALLOC_SCRATCH_BYTES (32u << 20)

/*
 * iris_b200_int4_paged_decode for callers that cannot allocate device memory.
 * No counterpart in the reference (its decode allocates nothing but its
 * output; this library's split-KV decode needs a workspace).
 *
 * Same arguments and results as iris_b200_int4_paged_decode, without the
 * workspace: the scratch (page prefix sums, split-KV partial records) is a
 * static __device__ array of IRIS_DECODE_NOALLOC_SCRATCH_BYTES inside the
 * library, held by every GPU that loads the library until the process exits.
 * For callers that are handed their tensors and may not call cudaMalloc or an
 * allocating library routine themselves (plugins in frameworks that own all
 * device memory, code running in allocator or stream callbacks, serving loops
 * that forbid allocation after start-up).
 *   - Nothing is allocated; returns IRIS_EWORKSPACE, before touching the
 *     array, when the problem needs more scratch than the array holds.  The
 *     need is sized by the problem's pages P = batch * max_pages_per_seq: at
 *     most max(min(P, 48), ceil(min(P, 128) / 2), ceil(P / 4)) split-KV
 *     ranges (and never more than the GPU-wide maximum that
 *     iris_b200_decode_workspace_bytes assumes), each holding two records of
 *     num_q_heads * (head_dim + 1) floats.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.  The address (like the library's cached
 *     launch shapes and tensor maps) is kept for the life of the process and
 *     does not survive cudaDeviceReset or a re-created primary context.
 *   - All calls share the one array: calls whose work overlaps on the GPU
 *     (other streams, other host threads) race.  Each call rewrites the
 *     parts it reads, so no state carries over between calls.
 */
IRIS_API int iris_b200_int4_paged_decode_noalloc(const void* query, const void* k_data, const void* v_data,
                                                 const void* k_scale, const void* v_scale,
                                                 const int32_t* block_table, int64_t block_table_stride,
                                                 const int32_t* seq_lens, void* output, float* out_lse,
                                                 int32_t out_mode, int32_t batch, int32_t num_q_heads,
                                                 int32_t num_kv_heads, int32_t head_dim, int64_t num_pages,
                                                 int32_t page_size, int32_t max_pages_per_seq, float softmax_scale,
                                                 int32_t* error_word, void* stream);

/*
 * Merge `num_parts` log-sum-exp-form partial results (as produced with
 * IRIS_DECODE_OUT_LSE) into the final fp16 output:
 *   parts_o [num_parts, rows, D] fp32, parts_lse [num_parts, rows] fp32,
 *   output [rows, D] fp16, rows = B*Hq.
 * A part with lse = -inf for a row contributes nothing to that row.
 * Used after an all-gather of per-GPU partials in split-context decode.  No
 * counterpart in the reference (split-KV is out of its scope, README.md:425).
 */
IRIS_API int iris_b200_merge_lse_partials(const float* parts_o, const float* parts_lse, int32_t num_parts, int64_t rows,
                                 int32_t head_dim, void* output, void* stream);

/*
 * Same merge over one packed buffer, the layout a single all-gather of the
 * per-GPU partials produces: part k occupies rows*(D+1) floats starting at
 * parts + k*rows*(D+1), O [rows, D] first and lse [rows] after it.  A part
 * whose lse is -inf for a row (a GPU that held none of that sequence's
 * tokens) is skipped for that row; its O need not be written.  No counterpart
 * in the reference.
 */
IRIS_API int iris_b200_merge_lse_packed(const float* parts, int32_t num_parts, int64_t rows, int32_t head_dim,
                                        void* output, void* stream);

/* ======================================================================
 * SPLIT-CONTEXT MERGE OVER NVLINK PEER MEMORY
 * ====================================================================== */

/*
 * No counterpart in the reference (single GPU). In split-context decode each
 * GPU computes, for the whole batch, a log-sum-exp partial (IRIS_DECODE_OUT_LSE:
 * O [rows, D] fp32, lse [rows] fp32, rows = B*Hq) over its own context splits;
 * every GPU needs their merge. These calls replace an all-gather + merge: one
 * kernel per GPU and step publishes this GPU's partial in its exchange buffer,
 * which the other GPUs have mapped (CUDA IPC), and merges every GPU's partial
 * read straight from its memory over NVLink.
 *
 * Per step every GPU calls iris_b200_xchg_merge once, after the kernel that
 * wrote its partial, on the same stream; all GPUs run the same steps in the
 * same order. The buffer holds two slots used on alternate steps, so a step
 * never waits for the others to finish reading. Waits are bounded: a GPU that
 * does not arrive within limit_ns sets IRIS_ERR_PIPELINE_TIMEOUT, after which
 * the exchange must be rebuilt.
 */
#define IRIS_IPC_HANDLE_BYTES 64
#define IRIS_XCHG_HEADER_BYTES 256

/* Bytes of one GPU's exchange buffer (header + two slots); 0 for a bad shape. */
IRIS_API size_t iris_b200_xchg_buffer_bytes(int64_t rows, int32_t head_dim);

/* Allocate (cudaMalloc, so that its IPC handle covers exactly it) and zero an
 * exchange buffer on the current device; free it. */
IRIS_API int iris_b200_xchg_alloc(size_t bytes, void** buf);
IRIS_API int iris_b200_xchg_free(void* buf);

/* CUDA IPC: write buf's handle (IRIS_IPC_HANDLE_BYTES, host memory); map a
 * peer's buffer from its handle (returns the device address here); unmap. */
IRIS_API int iris_b200_ipc_export(const void* buf, void* handle);
IRIS_API int iris_b200_ipc_open(const void* handle, void** peer_buf);
IRIS_API int iris_b200_ipc_close(void* peer_buf);

/* One step's merge on GPU my_rank: publish this GPU's partial (local_o [rows,
 * head_dim] fp32, 16-byte aligned; local_lse [rows] fp32), wait (bounded by
 * limit_ns) for every GPU's, and merge all num_ranks partials into output
 * [rows, head_dim] fp16. bufs: host array of num_ranks (<= 8) device
 * addresses, this GPU's buffer at my_rank and the mapped peer buffers
 * elsewhere. A part whose lse is -inf for a row (no tokens of that sequence)
 * is skipped. A cooperative launch of at most one CTA per SM. */
IRIS_API int iris_b200_xchg_merge(void* const* bufs, int32_t num_ranks, int32_t my_rank, int64_t rows,
                                  int32_t head_dim, const float* local_o, const float* local_lse, void* output,
                                  int32_t* error_word, int64_t limit_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* IRIS_B200_H_ */
