// pkv_capi.cpp -- the extern "C" surface declared in include/pkv_b200.h.
// Each entry point records its status (code, the CacheError variant's fields
// and a message) in thread-local storage and returns the code; no exception
// crosses the boundary. Each call that reaches the backend is an NVTX range
// named after the entry point (visible to Nsight Systems; free without a
// tool attached).

#include <cstring>

#include "pkv_b200.h"
#include "pkv_backend.hpp"

struct pkv_backend {
    std::unique_ptr<pkv::B200Backend> impl;
};

namespace {
thread_local pkv::Status g_last;
}  // namespace

// Records the status of the C-ABI call that is returning on this thread.
int pkv::finish(pkv::Status s) {
    g_last = std::move(s);
    return g_last.code;
}

using pkv::finish;
using pkv::guarded;

namespace {

int null_handle() { return finish(pkv::error(PKV_ERR_DEVICE, 0, 0, "null backend handle")); }

bool valid_dtype(int t) { return t >= PKV_F32 && t <= PKV_FP8_E4M3; }

int bad_dtype() { return finish(pkv::error(PKV_ERR_DEVICE, 0, 0, "unknown dtype tag")); }

cudaStream_t as_stream(void *s) { return static_cast<cudaStream_t>(s); }

}  // namespace

extern "C" {

const char *pkv_last_error(void) { return g_last.msg.c_str(); }

int pkv_last_error_fields(int64_t *field0, int64_t *field1) {
    if (field0) *field0 = g_last.a;
    if (field1) *field1 = g_last.b;
    return g_last.code;
}

int pkv_create(const pkv_config *cfg, int dtype, int device, int shard_rank, int num_shards,
               pkv_backend **out) {
    if (!cfg || !out) return finish(pkv::error(PKV_ERR_DEVICE, 0, 0, "null argument"));
    *out = nullptr;
    if (!valid_dtype(dtype)) return bad_dtype();
    return guarded("pkv_create", [&] {
        std::unique_ptr<pkv::B200Backend> impl;
        pkv::Status s = pkv::B200Backend::create(*cfg, static_cast<pkv::DType>(dtype), device,
                                                 shard_rank, num_shards, &impl);
        if (s.ok()) *out = new pkv_backend{std::move(impl)};
        return s;
    });
}

int pkv_destroy(pkv_backend *b) {
    delete b;
    return finish(pkv::Status::Ok());
}

int pkv_get_config(const pkv_backend *b, pkv_config *out) {
    if (!b || !out) return null_handle();
    *out = b->impl->config();
    return finish(pkv::Status::Ok());
}

uint64_t pkv_allocated_bytes(const pkv_backend *b) { return b ? b->impl->allocated_bytes() : 0; }

int pkv_device_name(const pkv_backend *b, char *buf, uint64_t buf_len) {
    if (!b || !buf || buf_len == 0) return null_handle();
    const std::string n = b->impl->device_name();
    const size_t m = std::min<size_t>(n.size(), buf_len - 1);
    std::memcpy(buf, n.data(), m);
    buf[m] = '\0';
    return finish(pkv::Status::Ok());
}

int pkv_shard_info(const pkv_backend *b, int *rank, int *num_shards, uint64_t *elem_offset,
                   uint64_t *shard_entry_elems) {
    if (!b) return null_handle();
    if (rank) *rank = b->impl->shard_rank();
    if (num_shards) *num_shards = b->impl->num_shards();
    if (elem_offset) *elem_offset = b->impl->elem_offset();
    if (shard_entry_elems) *shard_entry_elems = b->impl->entry_elems();
    return finish(pkv::Status::Ok());
}

int pkv_device_planes(const pkv_backend *b, void **k_plane, void **v_plane) {
    if (!b) return null_handle();
    if (k_plane) *k_plane = b->impl->k_plane();
    if (v_plane) *v_plane = b->impl->v_plane();
    return finish(pkv::Status::Ok());
}

int pkv_write_kv(pkv_backend *b, uint64_t layer, pkv_slot dst, const void *k, uint64_t k_len,
                 const void *v, uint64_t v_len, int host_dtype) {
    if (!b) return null_handle();
    if (!valid_dtype(host_dtype)) return bad_dtype();
    return guarded("pkv_write_kv", [&] {
        return b->impl->write_kv(layer, dst, k, k_len, v, v_len, static_cast<pkv::DType>(host_dtype));
    });
}

int pkv_write_kv_batch(pkv_backend *b, uint64_t layer, const pkv_slot *dsts, uint64_t count,
                       const void *k, uint64_t k_len, const void *v, uint64_t v_len,
                       int host_dtype) {
    if (!b) return null_handle();
    if (!valid_dtype(host_dtype)) return bad_dtype();
    return guarded("pkv_write_kv_batch", [&] {
        return b->impl->write_kv_batch(layer, dsts, count, k, k_len, v, v_len,
                                       static_cast<pkv::DType>(host_dtype));
    });
}

int pkv_read_kv(pkv_backend *b, uint64_t layer, pkv_slot src, void *k_out, uint64_t k_len,
                void *v_out, uint64_t v_len, int host_dtype) {
    if (!b) return null_handle();
    if (!valid_dtype(host_dtype)) return bad_dtype();
    return guarded("pkv_read_kv", [&] {
        return b->impl->read_kv(layer, src, k_out, k_len, v_out, v_len,
                                static_cast<pkv::DType>(host_dtype));
    });
}

int pkv_copy_block(pkv_backend *b, uint64_t src, uint64_t dst) {
    if (!b) return null_handle();
    return guarded("pkv_copy_block", [&] { return b->impl->copy_block(src, dst); });
}

int pkv_copy_blocks(pkv_backend *b, const uint64_t *pairs, uint64_t count) {
    if (!b) return null_handle();
    return guarded("pkv_copy_blocks", [&] { return b->impl->copy_blocks(pairs, count); });
}

int pkv_zero_block(pkv_backend *b, uint64_t block) {
    if (!b) return null_handle();
    return guarded("pkv_zero_block", [&] { return b->impl->zero_block(block); });
}

int pkv_zero_blocks(pkv_backend *b, const uint64_t *blocks, uint64_t count) {
    if (!b) return null_handle();
    return guarded("pkv_zero_blocks", [&] { return b->impl->zero_blocks(blocks, count); });
}

int pkv_reshape_and_cache_dev(pkv_backend *b, int64_t layer, const void *k, const void *v,
                              int64_t src_token_stride, int64_t src_layer_stride,
                              const int64_t *slot_mapping, int64_t num_tokens, int src_dtype,
                              void *stream) {
    if (!b) return null_handle();
    if (!valid_dtype(src_dtype)) return bad_dtype();
    return guarded("pkv_reshape_and_cache_dev", [&] {
        return b->impl->reshape_and_cache_dev(layer, k, v, src_token_stride, src_layer_stride,
                                              slot_mapping, num_tokens,
                                              static_cast<pkv::DType>(src_dtype), as_stream(stream));
    });
}

int pkv_copy_blocks_dev(pkv_backend *b, const int64_t *pairs, int64_t count, void *stream) {
    if (!b) return null_handle();
    return guarded("pkv_copy_blocks_dev", [&] { return b->impl->copy_blocks_dev(pairs, count, as_stream(stream)); });
}

int pkv_set_kv_scales(pkv_backend *b, const float *k_scales, const float *v_scales,
                      uint64_t count) {
    if (!b) return null_handle();
    return guarded("pkv_set_kv_scales", [&] { return b->impl->set_kv_scales(k_scales, v_scales, count); });
}

int pkv_paged_attention_dev(pkv_backend *b, int64_t layer, const void *q, int64_t q_seq_stride,
                            int64_t num_seqs, int64_t num_q_heads, const int32_t *block_tables,
                            int64_t table_stride, const int32_t *context_lens,
                            int64_t max_context_len, float softmax_scale, void *out, float *lse,
                            void *stream) {
    if (!b) return null_handle();
    return guarded("pkv_paged_attention_dev", [&] {
        return b->impl->paged_attention_dev(layer, q, b->impl->dtype(), q_seq_stride, num_seqs,
                                            num_q_heads, block_tables, table_stride, context_lens,
                                            max_context_len, softmax_scale, out, lse,
                                            as_stream(stream));
    });
}

int pkv_paged_attention_typed_dev(pkv_backend *b, int64_t layer, const void *q, int query_dtype,
                                  int64_t q_seq_stride, int64_t num_seqs, int64_t num_q_heads,
                                  const int32_t *block_tables, int64_t table_stride,
                                  const int32_t *context_lens, int64_t max_context_len,
                                  float softmax_scale, void *out, float *lse, void *stream) {
    if (!b) return null_handle();
    if (!valid_dtype(query_dtype)) return bad_dtype();
    return guarded("pkv_paged_attention_typed_dev", [&] {
        return b->impl->paged_attention_dev(layer, q, static_cast<pkv::DType>(query_dtype),
                                            q_seq_stride, num_seqs, num_q_heads, block_tables,
                                            table_stride, context_lens, max_context_len,
                                            softmax_scale, out, lse, as_stream(stream));
    });
}

int pkv_paged_attention_multi_dev(pkv_backend *b, int64_t layer, const void *q, int query_dtype,
                                  int64_t q_len, int64_t q_token_stride, int64_t num_seqs,
                                  int64_t num_q_heads, const int32_t *block_tables,
                                  int64_t table_stride, const int32_t *context_lens,
                                  int64_t max_context_len, float softmax_scale, void *out,
                                  float *lse, void *stream) {
    if (!b) return null_handle();
    if (!valid_dtype(query_dtype)) return bad_dtype();
    return guarded("pkv_paged_attention_multi_dev", [&] {
        return b->impl->paged_attention_dev(layer, q, static_cast<pkv::DType>(query_dtype),
                                            q_token_stride, num_seqs, num_q_heads, block_tables,
                                            table_stride, context_lens, max_context_len,
                                            softmax_scale, out, lse, as_stream(stream), q_len);
    });
}

int pkv_paged_attention_plan_dev(pkv_backend *b, const int32_t *context_lens, int64_t num_seqs,
                                 int64_t max_context_len, void *stream) {
    if (!b) return null_handle();
    return guarded("pkv_paged_attention_plan_dev", [&] {
        return b->impl->paged_attention_plan_dev(context_lens, num_seqs, max_context_len,
                                                 as_stream(stream));
    });
}

int pkv_set_copy_engine(pkv_backend *b, int engine) {
    if (!b) return null_handle();
    return guarded("pkv_set_copy_engine", [&] { return b->impl->set_copy_engine(engine); });
}

int pkv_zero_blocks_dev(pkv_backend *b, const int64_t *blocks, int64_t count, void *stream) {
    if (!b) return null_handle();
    return guarded("pkv_zero_blocks_dev", [&] { return b->impl->zero_blocks_dev(blocks, count, as_stream(stream)); });
}

int pkv_resolve_and_cache_mixed_dev(pkv_backend *b, const int32_t *block_tables,
                                    int64_t table_stride, const int32_t *ctx_lens,
                                    const int32_t *new_lens, int64_t num_seqs, int64_t num_tokens,
                                    int32_t *cu_seqlens, int64_t *slot_mapping,
                                    const int64_t *direct_slots, int64_t num_direct, int64_t layer,
                                    const void *k, const void *v, int64_t src_token_stride,
                                    int64_t src_layer_stride, int src_dtype, void *stream) {
    if (!b) return null_handle();
    if (!valid_dtype(src_dtype)) return bad_dtype();
    return guarded("pkv_resolve_and_cache_mixed_dev", [&] {
        return b->impl->resolve_and_cache_dev(block_tables, table_stride, ctx_lens, new_lens,
                                              num_seqs, num_tokens, cu_seqlens, slot_mapping,
                                              layer, k, v, src_token_stride, src_layer_stride,
                                              static_cast<pkv::DType>(src_dtype),
                                              as_stream(stream), direct_slots, num_direct);
    });
}

int pkv_copy_zero_blocks_dev(pkv_backend *b, const int64_t *srcs, const int64_t *dst_offsets,
                             const int64_t *dsts, const int64_t *zero_src, int64_t num_srcs,
                             const int64_t *zero_ids, int64_t num_zero, void *stream) {
    if (!b) return null_handle();
    return guarded("pkv_copy_zero_blocks_dev", [&] {
        return b->impl->copy_zero_dev(srcs, dst_offsets, dsts, zero_src, num_srcs, zero_ids,
                                      num_zero, as_stream(stream));
    });
}

int pkv_resolve_slots_dev(pkv_backend *b, const int32_t *block_tables, int64_t table_stride,
                          const int32_t *ctx_lens, const int32_t *new_lens, int64_t num_seqs,
                          int64_t num_tokens, int32_t *cu_seqlens, int64_t *slot_mapping,
                          void *stream) {
    if (!b) return null_handle();
    return guarded("pkv_resolve_slots_dev", [&] {
        return b->impl->resolve_slots_dev(block_tables, table_stride, ctx_lens, new_lens, num_seqs,
                                          num_tokens, cu_seqlens, slot_mapping, as_stream(stream));
    });
}

int pkv_resolve_and_cache_dev(pkv_backend *b, const int32_t *block_tables, int64_t table_stride,
                              const int32_t *ctx_lens, const int32_t *new_lens, int64_t num_seqs,
                              int64_t num_tokens, int32_t *cu_seqlens, int64_t *slot_mapping,
                              int64_t layer, const void *k, const void *v,
                              int64_t src_token_stride, int64_t src_layer_stride, int src_dtype,
                              void *stream) {
    if (!b) return null_handle();
    if (!valid_dtype(src_dtype)) return bad_dtype();
    return guarded("pkv_resolve_and_cache_dev", [&] {
        return b->impl->resolve_and_cache_dev(block_tables, table_stride, ctx_lens, new_lens,
                                              num_seqs, num_tokens, cu_seqlens, slot_mapping,
                                              layer, k, v, src_token_stride, src_layer_stride,
                                              static_cast<pkv::DType>(src_dtype),
                                              as_stream(stream));
    });
}

int pkv_digest(pkv_backend *b, uint64_t *k_digest, uint64_t *v_digest, void *stream) {
    if (!b || !k_digest || !v_digest) return null_handle();
    return guarded("pkv_digest", [&] { return b->impl->digest(k_digest, v_digest, as_stream(stream)); });
}

int pkv_digest_rows_dev(pkv_backend *b, int64_t layer, const void *k, const void *v,
                        int64_t src_token_stride, int64_t src_layer_stride,
                        const int64_t *slot_mapping, int64_t num_tokens, int src_dtype,
                        uint64_t *k_digest, uint64_t *v_digest, void *stream) {
    if (!b || !k_digest || !v_digest) return null_handle();
    if (!valid_dtype(src_dtype)) return bad_dtype();
    return guarded("pkv_digest_rows_dev", [&] {
        return b->impl->digest_rows(layer, k, v, src_token_stride, src_layer_stride, slot_mapping,
                                    num_tokens, static_cast<pkv::DType>(src_dtype), k_digest,
                                    v_digest, as_stream(stream));
    });
}

int pkv_host_threads(const pkv_backend *b, int *threads) {
    if (!b || !threads) return null_handle();
    *threads = b->impl->host_threads();
    return finish(pkv::Status::Ok());
}

int pkv_f32_to_bf16(const float *src, uint16_t *dst, uint64_t n) {
    if (n > 0 && (!src || !dst)) return finish(pkv::error(PKV_ERR_DEVICE, 0, 0, "null argument"));
    return guarded("pkv_f32_to_bf16", [&] {
        pkv::narrow_f32_to_bf16(dst, src, n);
        return pkv::Status::Ok();
    });
}

int pkv_sync(pkv_backend *b) {
    if (!b) return null_handle();
    return guarded("pkv_sync", [&] { return b->impl->sync(); });
}

int pkv_device_error(pkv_backend *b, int64_t *index) {
    if (!b) return null_handle();
    return guarded("pkv_device_error", [&] { return b->impl->take_device_error(index); });
}

}  // extern "C"
