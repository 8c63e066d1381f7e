// pkv_internal.hpp -- launch descriptors shared by the backend and the kernels.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace pkv {

// Element type tags; values match pkv_dtype in include/pkv_b200.h.
enum class DType : int { F32 = 0, BF16 = 1, F16 = 2, FP8_E4M3 = 3 };

inline int dtype_size(DType t) {
    switch (t) {
        case DType::F32: return 4;
        case DType::FP8_E4M3: return 1;
        default: return 2;
    }
}

// Quantisation of an fp8 (E4M3) pool: element e of an entry held by this
// backend belongs to kv head (elem_offset + e) / head_dim, and layer l of
// head h stores E4M3(x * inv[l * heads + h]). Unused for other pool types.
struct Fp8Scales {
    const float *k_inv = nullptr;  // [num_layers][heads], device memory
    const float *v_inv = nullptr;
    long long heads = 0;
    long long head_dim = 0;
    long long elem_offset = 0;
};

// Largest sequence count slot resolution takes in one call: the prefix of
// new_lens is built in one CTA's shared memory.
constexpr long long kMaxResolveSeqs = 56 * 1024;

// First bad index met by a device entry point. `code` is a pkv_status;
// `index` is the token / pair / block index it was met at.
struct DevError {
    int code;
    int pad;
    long long index;
};

// One reshape_and_cache launch: rows of `entry_elems` elements, read from
// k/v (src_dtype) and scattered to the pool planes (pool_dtype) at
// slot_mapping. Strides are in elements of the source type.
struct ReshapeLaunch {
    const void *k;
    const void *v;
    long long src_token_stride;
    long long src_layer_stride;  // used when num_layers > 1
    void *k_pool;                // plane base
    void *v_pool;
    long long first_layer;       // layer written by layer 0 of the source
    long long num_layers;        // layers written by this launch
    long long slots_per_layer;   // num_blocks * block_size
    long long entry_elems;       // elements per entry held by this backend
    const long long *slots;
    long long num_tokens;
    DType src_dtype;
    DType pool_dtype;
    DevError *err;
    Fp8Scales fp8;  // pool_dtype == FP8_E4M3 with another src_dtype
};

// Batched block copy over every layer and both planes; pairs is [num_pairs][2].
struct CopyLaunch {
    void *k_pool;
    void *v_pool;
    long long num_layers;
    long long num_blocks;
    long long block_bytes;  // block_size * entry_elems * elem size, one plane, one layer
    const long long *pairs;
    long long num_pairs;
    DevError *err;
};

struct ZeroLaunch {
    void *k_pool;
    void *v_pool;
    long long num_layers;
    long long num_blocks;
    long long block_bytes;
    const long long *blocks;
    long long num_ids;
    DevError *err;
};

// A step's copy-on-write pairs and freed blocks in one launch. The pairs
// are grouped by source: source i is read once and written to
// dsts[dst_off[i] .. dst_off[i + 1]), then zeroed when zero_src[i] is set
// (the step frees it); zero_ids are the step's other freed blocks.
struct CopyZeroLaunch {
    void *k_pool;
    void *v_pool;
    long long num_layers;
    long long num_blocks;
    long long block_bytes;
    const long long *srcs;      // [num_srcs]
    const long long *dst_off;   // [num_srcs + 1]
    const long long *dsts;      // [dst_off[num_srcs]]
    const long long *zero_src;  // [num_srcs]: nonzero to zero the source after its copies
    long long num_srcs;
    const long long *zero_ids;  // [num_zero]
    long long num_zero;
    DevError *err;
};

struct ResolveLaunch {
    const int *tables;
    long long table_stride;
    const int *ctx_lens;
    const int *new_lens;
    long long num_seqs;
    long long num_tokens;
    long long block_size;
    long long num_blocks;
    int *cu_seqlens;
    long long *slots;
    DevError *err;
};

struct DigestLaunch {
    const void *k_pool;
    const void *v_pool;
    long long rows;            // num_layers * num_blocks * block_size
    long long entry_elems;     // per shard
    long long full_entry;      // unsharded entry
    long long elem_offset;     // this shard's offset in the full entry
    DType pool_dtype;
    unsigned long long *out;   // [2]: K digest, V digest (accumulated)
};

// Slot resolution fused with reshape_and_cache (same element type in and out).
struct ResolveCacheLaunch {
    const int *tables;
    long long table_stride;
    const int *ctx_lens;
    const int *new_lens;
    long long num_seqs;
    long long num_tokens;
    long long block_size;
    long long num_blocks;
    int *cu_seqlens;             // [num_seqs + 1], written
    long long *slots_out;        // [num_tokens] or null
    const void *k;
    const void *v;
    long long src_token_stride_bytes;
    long long src_layer_stride_bytes;
    void *k_pool;
    void *v_pool;
    long long first_layer;
    long long num_layers;
    long long slots_per_layer;
    long long entry_bytes;  // pool bytes per entry
    DevError *err;
    // Quantising form (fp8 pool, wider source): element types and scales.
    DType src_dtype = DType::F32;
    DType pool_dtype = DType::F32;
    long long entry_elems = 0;
    Fp8Scales fp8;
    // Tokens whose slots the host already knows (a step's decoded tokens),
    // after the resolved ones: token num_tokens + j reads source row
    // num_tokens + j and goes to direct_slots[j] (negative: skipped).
    const long long *direct_slots = nullptr;
    long long num_direct = 0;
};

// Digest of rows as a scatter into an empty pool would store them.
struct DigestRowsLaunch {
    const void *k;
    const void *v;
    long long src_token_stride;  // elements
    long long src_layer_stride;  // elements
    const long long *slots;
    long long num_tokens;
    long long num_layers;
    long long first_layer;
    long long slots_per_layer;
    long long entry_elems;
    long long full_entry;
    long long elem_offset;
    DType src_dtype;
    DType pool_dtype;
    unsigned long long *out;  // [2], accumulated
    Fp8Scales fp8;
};

// Decode attention over one layer of the pool (pkv_attention.cu): one query
// token per sequence, GQA groups of `group` query heads per kv head.
struct AttnLaunch {
    const void *q;             // [num_seqs * q_len][num_q_heads][head_dim], row pitch q_seq_stride
    long long q_seq_stride;    // elements between consecutive query tokens
    void *out;                 // [num_seqs * q_len][num_q_heads][head_dim], contiguous
    float *lse;                // [num_seqs * q_len][num_q_heads] natural-log sum of exp, or null
    const int *tables;         // [num_seqs][table_stride]
    long long table_stride;
    const int *ctx;            // [num_seqs] tokens in the cache per sequence
    int num_seqs;
    int kv_heads;              // kv heads held by this backend
    int group;                 // query heads per kv head
    // Query tokens per sequence (q_len * group <= 16): token i of sequence s
    // sits at position ctx[s] - q_len + i and attends keys 0 .. that position.
    int q_len = 1;
    int num_q_heads;           // kv_heads * group
    int layer_row0;            // layer * num_blocks * block_size: first pool row of the layer
    int num_blocks;
    int max_ctx;
    int blocks_per_split;
    int num_splits;
    float scale_log2;          // softmax scale * log2(e)
    float *part_o;             // [num_seqs * q_len][num_q_heads][num_splits][head_dim] when num_splits > 1
    float *part_lse;           // [num_seqs * q_len][num_q_heads][num_splits], base-2
    // fp8 pools: dequantisation scales [num_layers][num_kv_heads] (device
    // memory) and the index of this layer's first kv head held here.
    const float *k_scale = nullptr;
    const float *v_scale = nullptr;
    long long scale_row = 0;
    // Optional order of the sequences (pkv_paged_attention_plan_dev): grid
    // slot z runs sequence order[z]. Any permutation gives the same results.
    const unsigned *order = nullptr;
    DevError *err;
};

int num_sms(int device);

cudaError_t launch_reshape(const ReshapeLaunch &a, int sms, cudaStream_t s);
cudaError_t launch_copy_blocks(const CopyLaunch &a, cudaStream_t s);
// copy_blocks through the SM's bulk-copy engine (pkv_bulk_copy.cu); supported
// when a block's plane splits into 16-byte-aligned runs of at most 32 KiB.
bool bulk_copy_supported(const CopyLaunch &a);
cudaError_t launch_copy_blocks_bulk(const CopyLaunch &a, int sms, cudaStream_t s);
cudaError_t launch_zero_blocks(const ZeroLaunch &a, cudaStream_t s);
cudaError_t launch_copy_zero(const CopyZeroLaunch &a, cudaStream_t s);
// zero_blocks through the bulk-copy engine (pkv_bulk_copy.cu).
bool bulk_zero_supported(const ZeroLaunch &a);
cudaError_t launch_zero_blocks_bulk(const ZeroLaunch &a, int sms, cudaStream_t s);
cudaError_t launch_resolve_slots(const ResolveLaunch &a, int sms, cudaStream_t s);
cudaError_t launch_resolve_cache(const ResolveCacheLaunch &a, int sms, cudaStream_t s);
cudaError_t launch_digest(const DigestLaunch &a, int sms, cudaStream_t s);
cudaError_t launch_digest_rows(const DigestRowsLaunch &a, int sms, cudaStream_t s);

// Paged decode attention (pkv_attention.cu). `tmaps` points at two
// CUtensorMap objects (K plane, V plane) built by make_attention_tmaps.
cudaError_t make_attention_tmaps(void *k_plane, void *v_plane, DType dtype, long long entry_elems,
                                 long long rows, int head_dim,
                                 void *tmaps_out /* 2 x 128 bytes, 64-aligned */);
int attention_splits(long long num_pairs, int max_ctx, int sms, int *blocks_per_split, bool fp8);
// The sequences ordered by descending block count (ctx entries outside
// [0, max_ctx] count as empty, as the attention kernel treats them):
// order[num_seqs].
cudaError_t launch_attention_plan(const int *ctx, int num_seqs, int max_ctx, unsigned *order,
                                  cudaStream_t s);
// pool: the pool dtype; query: the type of q and out (the pool dtype for
// bf16/f16 pools; bf16 or f16 over an fp8 pool).
cudaError_t launch_paged_attention(const AttnLaunch &a, const void *tmaps, DType pool, DType query,
                                   int head_dim, cudaStream_t s);

// fp8 (E4M3) pools (pkv_fp8.cu): quantising scatter, fused slot resolution +
// quantising scatter, and the digests of E4M3 planes and rows.
cudaError_t launch_reshape_fp8(const ReshapeLaunch &a, int sms, cudaStream_t s);
cudaError_t launch_resolve_cache_fp8(const ResolveCacheLaunch &a, int sms, cudaStream_t s);
cudaError_t launch_digest_fp8(const DigestLaunch &a, int sms, cudaStream_t s);
cudaError_t launch_digest_rows_fp8(const DigestRowsLaunch &a, int sms, cudaStream_t s);

}  // namespace pkv
