/*
 * pkv_b200.h -- C ABI of libpagedkv_b200.so, the B200 (sm_100a) device data
 * path of a paged KV cache.
 *
 * This is the drop-in seam for the `KvBackend` trait of paged-kv-core
 * (crates/paged-kv-core/src/backend.rs:23-124): a host-language backend
 * implements the trait by calling these functions, beside the unchanged
 * `CpuBackend`, `BlockAllocator`, `BlockTable` and `Scheduler`. Plain
 * pointers, sizes and status codes only; no C++ exceptions cross it.
 *
 * Pool layout (identical to CpuBackend, crates/paged-kv-core/src/cpu.rs:13-21):
 * two planes, K and V, each [num_layers][num_blocks][block_size][entry] in
 * the pool dtype, entry = num_kv_heads*head_dim (or, for shard r of G, the
 * contiguous slice [r*E/G, (r+1)*E/G) of it).
 *
 * Error model: every function returns a pkv_status. The variant's two fields
 * (e.g. InvalidLayer{layer, num_layers}) and a readable message are kept per
 * thread; fetch them with pkv_last_error_fields() / pkv_last_error().
 * Host-buffer entry points validate in the same order as CpuBackend and the
 * trait's default batch methods, and, like them, leave the effects of the
 * items before a failing item in place.
 *
 * Threading: one backend handle is used by one host thread at a time (the
 * trait's mutating methods take &mut self). Host-buffer methods issue their
 * work on the handle's own blocking CUDA stream, which is ordered with the
 * legacy default stream; device entry points use the stream they are given.
 * Per-handle device state is shared by the calls that use it: the device
 * error word (all entry points), the split workspace of the attention entry
 * points and the sequence order of pkv_paged_attention_plan_dev. Calls on
 * one handle that run concurrently on different streams share them too, so
 * give one handle's device calls one stream (or order the streams) when the
 * error word or attention's partial results must stay apart, and do not
 * remake a plan while attention calls that read it run on another stream
 * (they could read a mix of the two orders and skip a sequence).
 */
#ifndef PKV_B200_H
#define PKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* One status per CacheError variant (crates/paged-kv-core/src/error.rs:12-46). */
typedef enum pkv_status {
    PKV_OK = 0,
    PKV_ERR_OUT_OF_BLOCKS = 1,       /* OutOfBlocks{requested, available}  error.rs:14 */
    PKV_ERR_INVALID_BLOCK = 2,       /* InvalidBlock{id, num_blocks}       error.rs:17 */
    PKV_ERR_BLOCK_NOT_ALLOCATED = 3, /* BlockNotAllocated{id}              error.rs:20 */
    PKV_ERR_REFCOUNT_OVERFLOW = 4,   /* RefCountOverflow{id, max}          error.rs:24 */
    PKV_ERR_SLOT_OUT_OF_RANGE = 5,   /* SlotOutOfRange{slot, block_size}   error.rs:27 */
    PKV_ERR_SHAPE_MISMATCH = 6,      /* ShapeMismatch{expected, actual}    error.rs:31 */
    PKV_ERR_INVALID_LAYER = 7,       /* InvalidLayer{layer, num_layers}    error.rs:34 */
    PKV_ERR_UNKNOWN_SEQUENCE = 8,    /* UnknownSequence{id}                error.rs:38 */
    PKV_ERR_DEVICE = 9               /* Device(String)                     error.rs:45 */
} pkv_status;

/* Element types of the pool and of caller buffers. CacheConfig only carries
 * dtype_bytes (config.rs:19-20); the type tag tells bf16 from f16.
 * PKV_FP8_E4M3 (dtype_bytes 1) has no counterpart in the reference, whose
 * CpuBackend is f32 only (cpu.rs:22-25): an fp8 pool stores OCP E4M3 codes,
 * E4M3(x * (1/scale)) per (layer, kv head) -- see pkv_set_kv_scales. f32,
 * bf16 and f16 rows are quantised on the way in and dequantised on the way
 * out; E4M3 rows (raw codes) move unchanged and only to or from fp8 pools. */
typedef enum pkv_dtype { PKV_F32 = 0, PKV_BF16 = 1, PKV_F16 = 2, PKV_FP8_E4M3 = 3 } pkv_dtype;

/* CacheConfig (crates/paged-kv-core/src/config.rs:8-21), field for field. */
typedef struct pkv_config {
    uint64_t num_blocks;
    uint64_t block_size;
    uint64_t num_kv_heads;
    uint64_t head_dim;
    uint64_t num_layers;
    uint64_t dtype_bytes;
} pkv_config;

/* PhysicalSlot (crates/paged-kv-core/src/types.rs:40-43); BlockId widened to 64 bits. */
typedef struct pkv_slot {
    uint64_t block;
    uint64_t slot;
} pkv_slot;

typedef struct pkv_backend pkv_backend;

/* ---- errors ------------------------------------------------------------ */

/* Message of the last failing call on this thread ("" after success). */
const char *pkv_last_error(void);
/* Status of the last call on this thread; writes the variant's two fields
 * (0 where the variant has fewer). */
int pkv_last_error_fields(int64_t *field0, int64_t *field1);

/* ---- lifecycle (CudaBackend::new, crates/paged-kv-cuda/src/backend.rs:63-92) ---- */

/* Allocate a zero-filled pool on `device`. dtype must agree with
 * cfg->dtype_bytes. num_shards = 1 gives the whole pool; otherwise this
 * backend holds shard `shard_rank` (contiguous entry slice) and every
 * host/device K/V buffer passed to it holds that slice only. */
int pkv_create(const pkv_config *cfg, int dtype, int device, int shard_rank, int num_shards,
               pkv_backend **out);
int pkv_destroy(pkv_backend *b);

/* ---- metadata ------------------------------------------------------------ */

/* KvBackend::config (backend.rs:25): the full, unsharded geometry. */
int pkv_get_config(const pkv_backend *b, pkv_config *out);
/* KvBackend::allocated_bytes (backend.rs:118-120): this backend's pool bytes. */
uint64_t pkv_allocated_bytes(const pkv_backend *b);
/* KvBackend::device_name (backend.rs:123); starts with "cuda:". */
int pkv_device_name(const pkv_backend *b, char *buf, uint64_t buf_len);
/* Shard geometry: elements per entry held here and their offset in the full entry. */
int pkv_shard_info(const pkv_backend *b, int *shard_rank, int *num_shards, uint64_t *elem_offset,
                   uint64_t *shard_entry_elems);
/* Device addresses of the K and V planes (for attention kernels and checks). */
int pkv_device_planes(const pkv_backend *b, void **k_plane, void **v_plane);

/* ---- KvBackend methods over host buffers ----------------------------------
 * Lengths are element counts of the caller's buffers; host_dtype is their
 * element type. Data converted to a narrower pool type is rounded to nearest
 * even; widening is exact. The call returns once the host buffers have been
 * consumed; device work may still be running on the backend's stream. */

/* KvBackend::write_kv (backend.rs:34-40; CpuBackend cpu.rs:95-111). */
int pkv_write_kv(pkv_backend *b, uint64_t layer, pkv_slot dst, const void *k, uint64_t k_len,
                 const void *v, uint64_t v_len, int host_dtype);
/* KvBackend::write_kv_batch (backend.rs:55-74) -> one reshape_and_cache launch
 * (replaces CudaBackend::write_kv_batch, crates/paged-kv-cuda/src/backend.rs:147-209). */
int pkv_write_kv_batch(pkv_backend *b, uint64_t layer, const pkv_slot *dsts, uint64_t count,
                       const void *k, uint64_t k_len, const void *v, uint64_t v_len,
                       int host_dtype);
/* KvBackend::read_kv (backend.rs:82-88; cpu.rs:113-129). Synchronous; copies
 * only the requested entry (the reference copies the whole plane,
 * crates/paged-kv-cuda/src/backend.rs:211-242). */
int pkv_read_kv(pkv_backend *b, uint64_t layer, pkv_slot src, void *k_out, uint64_t k_len,
                void *v_out, uint64_t v_len, int host_dtype);
/* KvBackend::copy_block (backend.rs:97; cpu.rs:131-149). */
int pkv_copy_block(pkv_backend *b, uint64_t src, uint64_t dst);
/* KvBackend::copy_blocks (backend.rs:104-109) -> batched copy_blocks kernel
 * (replaces crates/paged-kv-cuda/src/backend.rs:251-293). pairs = [count][2]
 * (src, dst). Same result as applying the pairs one after another, chains
 * included. */
int pkv_copy_blocks(pkv_backend *b, const uint64_t *pairs, uint64_t count);
/* KvBackend::zero_block (backend.rs:115; cpu.rs:151-160;
 * crates/paged-kv-cuda/src/backend.rs:295-320). */
int pkv_zero_block(pkv_backend *b, uint64_t block);
/* Batched zero_block: one launch for many blocks (the reference launches once per block). */
int pkv_zero_blocks(pkv_backend *b, const uint64_t *blocks, uint64_t count);

/* ---- device entry points (inputs already in device memory) ----------------
 * stream: a cudaStream_t; NULL is the legacy default stream, as everywhere in
 * CUDA. These do not synchronise. Bad indices found on the device are skipped
 * and recorded in the backend's device error word (pkv_device_error). */

/* reshape_and_cache (crates/paged-kv-cuda/kernels/kernels.cu:31-60).
 * layer >= 0: k, v are [num_tokens][entry] rows (row pitch src_token_stride
 * elements) written into that layer. layer == -1: k, v are
 * [num_layers][num_tokens][entry] (layer pitch src_layer_stride elements) and
 * every layer is written in one launch. slot_mapping[t] = block*block_size +
 * slot; a negative slot skips the token (padding). src_dtype may differ from
 * the pool dtype (rounded to nearest even when narrowing; quantised with the
 * pool's scales into an fp8 pool). */
int pkv_reshape_and_cache_dev(pkv_backend *b, int64_t layer, const void *k, const void *v,
                              int64_t src_token_stride, int64_t src_layer_stride,
                              const int64_t *slot_mapping, int64_t num_tokens, int src_dtype,
                              void *stream);
/* copy_blocks (kernels.cu:62-92). pairs = [count][2] int64 (src, dst) in
 * device memory. The pairs must not chain (no dst is another pair's src or
 * dst), which copy-on-write pairs never do; src == dst is a no-op. */
int pkv_copy_blocks_dev(pkv_backend *b, const int64_t *pairs, int64_t count, void *stream);
/* Scales of an fp8 (E4M3) pool; no counterpart in the reference. k_scales
 * and v_scales are [num_layers][num_kv_heads] (count = num_layers *
 * num_kv_heads, full heads even for a shard). Element x of layer l, kv head
 * h is stored as E4M3(x * inv) with inv = 1.0f / scale[l][h] (f32 division),
 * the product an f32 multiply, and the conversion rounding to nearest even
 * and saturating at +-448; reads return code * scale. Every scale starts at
 * 1.0. Each scale must be finite and positive with a finite reciprocal
 * (else PKV_ERR_DEVICE); a wrong count is ShapeMismatch{expected, count};
 * pools of other types reject the call. Applies to writes issued after it
 * returns (it synchronises the backend's stream). */
int pkv_set_kv_scales(pkv_backend *b, const float *k_scales, const float *v_scales,
                      uint64_t count);
/* Engines that copy_blocks can run on (no counterpart in the reference, whose
 * copy_blocks_kernel, kernels.cu:62-92, has one scalar form). Both give the
 * same pool bytes.
 *   PKV_COPY_VECTOR: every thread moves 16-byte vectors through registers.
 *   PKV_COPY_BULK:   one thread per CTA drives the SM's bulk-copy (TMA)
 *                    engine, global -> shared -> global, in runs of up to
 *                    32 KiB; needs a block plane (block_size * entry bytes)
 *                    that splits into 16-byte multiples of at most 32 KiB.
 *   PKV_COPY_AUTO:   the engine that measured faster on B200 for the pool's
 *                    geometry (the default). */
typedef enum pkv_copy_engine {
    PKV_COPY_AUTO = 0,
    PKV_COPY_VECTOR = 1,
    PKV_COPY_BULK = 2
} pkv_copy_engine;
/* Selects the engine of every later copy_blocks and zero_blocks call on this
 * backend (host and device entry points). Under PKV_COPY_BULK, zero_blocks
 * issues bulk stores of a zeroed shared-memory run; the geometry rule is the
 * same. Unknown engines, and PKV_COPY_BULK for a geometry it cannot take, are
 * rejected with PKV_ERR_DEVICE and leave the engine as it was. */
int pkv_set_copy_engine(pkv_backend *b, int engine);
/* zero_block (kernels.cu:94-110), batched: blocks = [count] int64 in device memory. */
int pkv_zero_blocks_dev(pkv_backend *b, const int64_t *blocks, int64_t count, void *stream);
/* One scheduler step's copy_blocks and zero_blocks in one launch (the
 * reference issues copy_blocks then zero_block per block,
 * crates/paged-kv-cuda/src/backend.rs:251-320). All arrays are int64 in
 * device memory. The pairs are given grouped by source: source i
 * (srcs[i]) is copied to dsts[dst_offsets[i] .. dst_offsets[i + 1]) and,
 * if zero_src[i] is nonzero, zeroed after its copies; zero_ids are further
 * blocks to zero. Equivalent to copy_blocks of every (srcs[i], dst) pair
 * followed by zero_blocks of the zeroed sources and zero_ids, provided that
 * no destination is a source, a zeroed block or repeated (the step driver
 * checks this and otherwise issues the two calls). Bad ids are recorded in
 * the device error word (index: the pair's position in dsts, or
 * dst_offsets[num_srcs] + the position in zero_ids) and skipped. */
int pkv_copy_zero_blocks_dev(pkv_backend *b, const int64_t *srcs, const int64_t *dst_offsets,
                             const int64_t *dsts, const int64_t *zero_src, int64_t num_srcs,
                             const int64_t *zero_ids, int64_t num_zero, void *stream);
/* Slot resolution (no device counterpart in the reference; host rule
 * BlockTable::slot_for_position, block_table.rs:97-101, flattened as
 * crates/paged-kv-cuda/src/backend.rs:172-175). Sequence q has ctx_lens[q]
 * cached tokens and new_lens[q] new ones; block_tables is [num_seqs][table_stride]
 * int32. Writes cu_seqlens[0..num_seqs] (exclusive prefix of new_lens, int32)
 * and slot_mapping[0..num_tokens). num_tokens must equal sum(new_lens).
 * Tokens whose logical block lies past table_stride or whose table entry is
 * outside the pool get slot -1 and are recorded in the device error word. */
int pkv_resolve_slots_dev(pkv_backend *b, const int32_t *block_tables, int64_t table_stride,
                          const int32_t *ctx_lens, const int32_t *new_lens, int64_t num_seqs,
                          int64_t num_tokens, int32_t *cu_seqlens, int64_t *slot_mapping,
                          void *stream);
/* Slot resolution fused with reshape_and_cache: one launch per step, the
 * slots computed inline (no slot_mapping round trip through memory). Same
 * arguments and results as pkv_resolve_slots_dev followed by
 * pkv_reshape_and_cache_dev(layer, k, v, ...); slot_mapping is an optional
 * output (NULL: not written) for kernels that read the cache afterwards.
 * src_dtype must equal the pool dtype, except that an fp8 pool also takes
 * f32/bf16/f16 rows and quantises them in the same launch. */
int pkv_resolve_and_cache_dev(pkv_backend *b, const int32_t *block_tables, int64_t table_stride,
                              const int32_t *ctx_lens, const int32_t *new_lens, int64_t num_seqs,
                              int64_t num_tokens, int32_t *cu_seqlens, int64_t *slot_mapping,
                              int64_t layer, const void *k, const void *v,
                              int64_t src_token_stride, int64_t src_layer_stride, int src_dtype,
                              void *stream);
/* One scheduler step's whole cache write in one launch (no counterpart in
 * the reference; its StepOutcome carries both kinds of token,
 * crates/paged-kv-core/src/scheduler.rs:57-86): the num_tokens tokens of the
 * sequences given by block tables (admitted prompts), resolved as
 * pkv_resolve_and_cache_dev does, then num_direct tokens whose slots the
 * host already has (decoded tokens: direct_slots, int64, device memory;
 * negative skipped, past the pool recorded as InvalidBlock at the token's
 * index). k and v hold num_tokens + num_direct rows, the resolved tokens'
 * first. Equivalent to pkv_resolve_and_cache_dev followed by
 * pkv_reshape_and_cache_dev of the direct tokens; pools of the source's
 * type only (an fp8 pool is refused). slot_mapping, if given, receives the
 * resolved tokens' slots. */
int pkv_resolve_and_cache_mixed_dev(pkv_backend *b, const int32_t *block_tables,
                                    int64_t table_stride, const int32_t *ctx_lens,
                                    const int32_t *new_lens, int64_t num_seqs, int64_t num_tokens,
                                    int32_t *cu_seqlens, int64_t *slot_mapping,
                                    const int64_t *direct_slots, int64_t num_direct, int64_t layer,
                                    const void *k, const void *v, int64_t src_token_stride,
                                    int64_t src_layer_stride, int src_dtype, void *stream);
/* Decode attention over layer `layer` of the pool: one query token per
 * sequence. No counterpart in the reference, which leaves paged_attention
 * off its trait until its signature is settled
 * (crates/paged-kv-core/src/backend.rs:18-22); this one fixes the open
 * choices as: scores and softmax in f32, output in the pool dtype, and an
 * optional log-sum-exp per (sequence, head) as the partial softmax state that
 * chunked prefill merges.
 *
 * q and out are [num_seqs][num_q_heads][head_dim] in the pool dtype (bf16 or
 * f16 pools), q with row pitch q_seq_stride elements (<= 0: dense), out
 * dense; num_q_heads counts the query heads of the kv heads held by this
 * backend (a shard must hold whole kv heads) and is a multiple of them: query
 * head qh reads kv head qh / (num_q_heads / kv_heads), at most 16 per kv
 * head. Sequence s attends to its context_lens[s] cached tokens, token t in
 * block block_tables[s][t / 16] slot t % 16 (block_size must be 16; head_dim
 * 64, 128 or 256). max_context_len bounds every context_lens[s] (a longer one
 * is recorded as ShapeMismatch in the device error word and yields zeros) and
 * must fit the tables (<= table_stride * 16). lse (optional, f32
 * [num_seqs][num_q_heads]) receives log(sum exp(scale * q.k)); an empty
 * context gives a zero output and lse = -inf. Block ids outside the pool are
 * recorded (InvalidBlock) and their tokens skipped. softmax_scale must be
 * finite and positive.
 *
 * Long contexts are split over several CTAs whose partial results live in a
 * per-handle device workspace. A call that needs more workspace than every
 * earlier call on the handle synchronises the device and allocates it
 * (cudaMalloc), which a stream capture does not allow: run the largest shape
 * once before capturing attention calls into a CUDA graph. The other
 * device-pointer entry points allocate nothing per call. */
int pkv_paged_attention_dev(pkv_backend *b, int64_t layer, const void *q, int64_t q_seq_stride,
                            int64_t num_seqs, int64_t num_q_heads, const int32_t *block_tables,
                            int64_t table_stride, const int32_t *context_lens,
                            int64_t max_context_len, float softmax_scale, void *out, float *lse,
                            void *stream);
/* pkv_paged_attention_dev with the type of q and out given (a pkv_dtype):
 * over a bf16 or f16 pool it must be the pool dtype; over an fp8 (E4M3) pool
 * it is PKV_BF16 or PKV_F16, and attention reads the dequantised cache,
 * code * scale with the per-(layer, kv head) scales of pkv_set_kv_scales.
 * The codes enter the tensor cores as f16 (exact for every E4M3 value), and
 * so do the queries, scaled by a power of two into f16 range; the scores,
 * softmax and output accumulate in f32. Otherwise as pkv_paged_attention_dev.
 * No counterpart in the reference (no attention, no fp8 format). */
int pkv_paged_attention_typed_dev(pkv_backend *b, int64_t layer, const void *q, int query_dtype,
                                  int64_t q_seq_stride, int64_t num_seqs, int64_t num_q_heads,
                                  const int32_t *block_tables, int64_t table_stride,
                                  const int32_t *context_lens, int64_t max_context_len,
                                  float softmax_scale, void *out, float *lse, void *stream);
/* pkv_paged_attention_typed_dev with q_len query tokens per sequence (the
 * verification step of speculative decoding, or a short chunk of prefill):
 * query token i of sequence s sits at position context_lens[s] - q_len + i
 * (its own K/V already in the cache) and attends keys 0 .. that position.
 * q and out are [num_seqs * q_len][num_q_heads][head_dim], token i of
 * sequence s at row s * q_len + i; q_token_stride is q's row pitch in
 * elements (<= 0: dense); lse is [num_seqs * q_len][num_q_heads]. Needs
 * 1 <= q_len and q_len * (num_q_heads / kv_heads) <= 16. A context shorter
 * than q_len is recorded as ShapeMismatch and yields zeros. q_len 1 is
 * pkv_paged_attention_typed_dev. No counterpart in the reference. */
int pkv_paged_attention_multi_dev(pkv_backend *b, int64_t layer, const void *q, int query_dtype,
                                  int64_t q_len, int64_t q_token_stride, int64_t num_seqs,
                                  int64_t num_q_heads, const int32_t *block_tables,
                                  int64_t table_stride, const int32_t *context_lens,
                                  int64_t max_context_len, float softmax_scale, void *out,
                                  float *lse, void *stream);

/* Schedule for the paged attention calls that follow (a decode step's
 * layers): reads context_lens on the device and orders the sequences by
 * descending length, so that each layer's grid starts with its long
 * sequences and ends with its short ones instead of waiting on a long one
 * that happened to come last. Later pkv_paged_attention_dev / _typed_dev /
 * _multi_dev calls on this handle with the same context_lens pointer,
 * num_seqs and max_context_len use it; other calls run in launch order. The
 * plan only schedules: the results are the same bit for bit, also when
 * context_lens has changed since, so plan once per step after the lengths
 * are written. The first plan on a handle allocates 256 KiB of device
 * memory. No counterpart in the reference. */
int pkv_paged_attention_plan_dev(pkv_backend *b, const int32_t *context_lens, int64_t num_seqs,
                                 int64_t max_context_len, void *stream);

/* Order-independent 64-bit digests of this backend's K and V planes (the
 * element's global index in the full plane and its f32-widened bits, summed;
 * zeros contribute nothing). Digests of the shards of one pool add up
 * (mod 2^64) to the digest of the whole pool. Synchronous. */
int pkv_digest(pkv_backend *b, uint64_t *k_digest, uint64_t *v_digest, void *stream);

/* Digests (as pkv_digest) that this backend's planes would have if the given
 * rows (arguments as pkv_reshape_and_cache_dev; negative slots skipped) had
 * been written into an all-zero pool. With distinct slots, comparing this to
 * pkv_digest after the write verifies the pool without reading it back.
 * Synchronous. */
int pkv_digest_rows_dev(pkv_backend *b, int64_t layer, const void *k, const void *v,
                        int64_t src_token_stride, int64_t src_layer_stride,
                        const int64_t *slot_mapping, int64_t num_tokens, int src_dtype,
                        uint64_t *k_digest, uint64_t *v_digest, void *stream);

/* Slot resolution + reshape_and_cache that allocates nothing. No counterpart
 * in the reference.
 *
 * For callers that cannot call cudaMalloc: for example a plugin running
 * inside an inference engine that has already reserved (nearly) all HBM for
 * its own memory pool and hands out only the buffers it owns. The caller
 * passes every input and output, including the pool planes (laid out as a
 * backend created with the same config, dtype and shard would lay them out)
 * and cu_seqlens[num_seqs + 1]; the intermediate slot mapping and the device
 * error word live in a fixed static device array of
 * PKV_NOALLOC_SCRATCH_BYTES, which every GPU that loads the library holds
 * until the process exits. Results are those of pkv_resolve_slots_dev
 * followed by pkv_reshape_and_cache_dev.
 *
 * - num_tokens above PKV_NOALLOC_MAX_TOKENS is rejected (ShapeMismatch{max,
 *   num_tokens}) before any device work; more than 57,344 sequences is
 *   rejected as by pkv_resolve_slots_dev (PKV_ERR_DEVICE).
 * - Pools and sources of f32, bf16 and f16 only: an fp8 (E4M3) pool or
 *   source is rejected with PKV_ERR_DEVICE, because quantising needs the
 *   per-(layer, kv head) scales that only a backend holds
 *   (pkv_resolve_and_cache_dev writes fp8 pools).
 * - Strides are checked as by pkv_reshape_and_cache_dev: a token stride
 *   shorter than the entry, or (layer = -1) a layer stride shorter than
 *   num_tokens x token stride, is ShapeMismatch.
 * - Runs on the current device; the first call on a device looks up the
 *   scratch array's device address, so make that first call before any
 *   stream capture. The address is kept for the life of the process: calls
 *   after cudaDeviceReset on that device are not supported.
 * - All calls on a device share the scratch array: calls whose work overlaps
 *   on the GPU race. Each call clears what it needs before use.
 * - device_status (optional, device memory, 2 x int64) receives {status,
 *   index} of the first bad index met on the device (0 = none). */
#define PKV_NOALLOC_MAX_TOKENS 131072
#define PKV_NOALLOC_SCRATCH_BYTES (256 + 8 * PKV_NOALLOC_MAX_TOKENS)
int pkv_resolve_and_cache_noalloc(const pkv_config *cfg, int pool_dtype, int shard_rank,
                                  int num_shards, void *k_plane, void *v_plane,
                                  const int32_t *block_tables, int64_t table_stride,
                                  const int32_t *ctx_lens, const int32_t *new_lens,
                                  int64_t num_seqs, int64_t num_tokens, int32_t *cu_seqlens,
                                  int64_t layer, const void *k, const void *v,
                                  int64_t src_token_stride, int64_t src_layer_stride,
                                  int src_dtype, int64_t *device_status, void *stream);

/* Worker threads of the backend's host stager. Large host-buffer writes
 * (pkv_write_kv_batch / pkv_write_kv of at least 1 MiB of rows) use it when
 * the rows are in pageable memory, or are f32 rows for a bf16 pool: the
 * workers copy (or narrow to bf16) the caller's rows into a 32 MiB ring of
 * pinned chunks while earlier chunks cross the host link, and the call
 * returns once every row has been read. Environment, read by pkv_create:
 * PKV_HOST_THREADS=n sets the count (default: one per host core, at most
 * 16, and at most half the ring's chunks); PKV_HOST_STAGING=off copies from
 * the caller's buffer instead; PKV_STAGE_CHUNK_KIB and PKV_STAGE_SLOTS size
 * the ring (default 1,024 KiB x 32, at most 64 chunks). No
 * counterpart in the reference (its CudaBackend copies each slice with a
 * fresh device allocation, crates/paged-kv-cuda/src/backend.rs:177-180). */
int pkv_host_threads(const pkv_backend *b, int *threads);

/* f32 -> bf16 on the host, round to nearest even (NaN as CUDA's
 * __float2bfloat16_rn gives it): the narrowing the host stager applies to
 * f32 rows bound for a bf16 pool before they cross the host link, with the
 * same results as the device conversion. dst receives bf16 bit patterns.
 * No counterpart in the reference (its pool is f32). */
int pkv_f32_to_bf16(const float *src, uint16_t *dst, uint64_t n);

/* Wait for all work issued on the backend's stream. */
int pkv_sync(pkv_backend *b);
/* Synchronise, then read and clear the device error word. Returns PKV_OK if no
 * device entry point met a bad index since the last call; otherwise the
 * status of the first one met and, in *index, the token/pair/block index it
 * was met at. */
int pkv_device_error(pkv_backend *b, int64_t *index);

#ifdef __cplusplus
}
#endif

#endif /* PKV_B200_H */
