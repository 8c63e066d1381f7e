// pkv_backend.hpp -- B200Backend: the KvBackend trait of paged-kv-core
// (crates/paged-kv-core/src/backend.rs:23-124) implemented over the sm_100a
// kernels, with CpuBackend's validation order and error variants
// (crates/paged-kv-core/src/cpu.rs:55-87) so that callers cannot tell the two
// apart except by speed.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <exception>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "pkv_b200.h"
#include "pkv_internal.hpp"
#include "pkv_stage.hpp"

namespace pkv {

// Result of one backend call: a pkv_status plus the CacheError variant's fields.
struct Status {
    int code = PKV_OK;
    int64_t a = 0;
    int64_t b = 0;
    std::string msg;
    bool ok() const { return code == PKV_OK; }
    static Status Ok() { return {}; }
};

Status error(int code, int64_t a, int64_t b, std::string msg);
Status device_error(const std::string &what, cudaError_t e);
// Stores `s` as this thread's last status (pkv_last_error*) and returns its code.
int finish(Status s);

// One NVTX range per C-ABI call, named after the entry point.
struct NvtxRange {
    explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
};

// Runs the body of a C-ABI entry point inside its NVTX range and records its
// status; no exception crosses the boundary (host allocation failures become
// PKV_ERR_DEVICE).
template <typename F>
int guarded(const char *name, F &&f) {
    NvtxRange range(name);
    try {
        return finish(f());
    } catch (const std::bad_alloc &) {
        return finish(error(PKV_ERR_DEVICE, 0, 0, "host out of memory"));
    } catch (const std::exception &e) {
        return finish(error(PKV_ERR_DEVICE, 0, 0, e.what()));
    }
}

class B200Backend {
   public:
    static Status create(const pkv_config &cfg, DType dtype, int device, int shard_rank,
                         int num_shards, std::unique_ptr<B200Backend> *out);
    ~B200Backend();
    B200Backend(const B200Backend &) = delete;
    B200Backend &operator=(const B200Backend &) = delete;

    // ---- KvBackend ----
    const pkv_config &config() const { return cfg_; }
    Status write_kv(uint64_t layer, pkv_slot dst, const void *k, uint64_t k_len, const void *v,
                    uint64_t v_len, DType host);
    Status write_kv_batch(uint64_t layer, const pkv_slot *dsts, uint64_t count, const void *k,
                          uint64_t k_len, const void *v, uint64_t v_len, DType host);
    Status read_kv(uint64_t layer, pkv_slot src, void *k_out, uint64_t k_len, void *v_out,
                   uint64_t v_len, DType host);
    Status copy_block(uint64_t src, uint64_t dst);
    Status copy_blocks(const uint64_t *pairs, uint64_t count);
    Status zero_block(uint64_t block);
    Status zero_blocks(const uint64_t *blocks, uint64_t count);
    uint64_t allocated_bytes() const;
    std::string device_name() const;

    // ---- device entry points ----
    Status reshape_and_cache_dev(int64_t layer, const void *k, const void *v, int64_t tok_stride,
                                 int64_t layer_stride, const int64_t *slots, int64_t num_tokens,
                                 DType src, cudaStream_t s);
    Status copy_blocks_dev(const int64_t *pairs, int64_t count, cudaStream_t s);
    Status zero_blocks_dev(const int64_t *blocks, int64_t count, cudaStream_t s);
    Status copy_zero_dev(const int64_t *srcs, const int64_t *dst_off, const int64_t *dsts,
                         const int64_t *zero_src, int64_t num_srcs, const int64_t *zero_ids,
                         int64_t num_zero, cudaStream_t s);
    Status set_copy_engine(int engine);
    Status set_kv_scales(const float *k_scales, const float *v_scales, uint64_t count);
    // query: the type of q and out; the pool dtype for bf16/f16 pools, bf16
    // or f16 over an fp8 pool. q_len: query tokens per sequence (the last
    // q_len positions of its context, causal among themselves).
    Status paged_attention_dev(int64_t layer, const void *q, DType query, int64_t q_seq_stride,
                               int64_t num_seqs, int64_t num_q_heads, const int32_t *tables,
                               int64_t table_stride, const int32_t *ctx, int64_t max_ctx,
                               float softmax_scale, void *out, float *lse, cudaStream_t s,
                               int64_t q_len = 1);
    // Longest-first order of the sequences for the attention calls that
    // follow with the same ctx buffer, num_seqs and max_ctx (scheduling only).
    Status paged_attention_plan_dev(const int32_t *ctx, int64_t num_seqs, int64_t max_ctx, cudaStream_t s);
    Status resolve_slots_dev(const int32_t *tables, int64_t table_stride, const int32_t *ctx,
                             const int32_t *new_lens, int64_t num_seqs, int64_t num_tokens,
                             int32_t *cu, int64_t *slots, cudaStream_t s);
    Status resolve_and_cache_dev(const int32_t *tables, int64_t table_stride, const int32_t *ctx,
                                 const int32_t *new_lens, int64_t num_seqs, int64_t num_tokens,
                                 int32_t *cu, int64_t *slots_out, int64_t layer, const void *k,
                                 const void *v, int64_t tok_stride, int64_t layer_stride,
                                 DType src, cudaStream_t s, const int64_t *direct_slots = nullptr,
                                 int64_t num_direct = 0);
    Status digest(uint64_t *k, uint64_t *v, cudaStream_t s);
    Status digest_rows(int64_t layer, const void *k, const void *v, int64_t tok_stride,
                       int64_t layer_stride, const int64_t *slots, int64_t num_tokens, DType src,
                       uint64_t *kd, uint64_t *vd, cudaStream_t s);
    Status sync();
    Status take_device_error(int64_t *index);

    // ---- geometry ----
    uint64_t entry_elems() const { return shard_entry_; }
    uint64_t full_entry_elems() const { return cfg_.num_kv_heads * cfg_.head_dim; }
    uint64_t elem_offset() const { return shard_rank_ * shard_entry_; }
    int shard_rank() const { return shard_rank_; }
    // Workers the stager runs with (it caps them at half its ring's slots).
    int host_threads() const {
        return std::max(1, std::min(host_threads_, std::min(stage_slots_, HostStager::kMaxSlots) / 2));
    }
    int num_shards() const { return num_shards_; }
    void *k_plane() const { return k_plane_; }
    void *v_plane() const { return v_plane_; }
    DType dtype() const { return dtype_; }
    cudaStream_t stream() const { return stream_; }

   private:
    B200Backend() = default;

    uint64_t slots_per_layer() const { return cfg_.num_blocks * cfg_.block_size; }
    uint64_t entry_bytes() const { return shard_entry_ * dtype_size(dtype_); }
    uint64_t block_bytes() const { return cfg_.block_size * entry_bytes(); }
    Status validate_block(uint64_t block) const;
    Status validate(uint64_t layer, pkv_slot at) const;
    Status ensure_device_stage(size_t bytes);
    Status ensure_scatter_stage(int buf, size_t bytes);
    Status ensure_host_stage(size_t bytes);
    Status launch_scatter(uint64_t layer, const pkv_slot *dsts, uint64_t count, const void *k,
                          const void *v, DType host);
    bool host_pinned(const void *p) const;
    Status stager(HostStager **out);
    Status launch_copy_pairs(const uint64_t *pairs, uint64_t count);
    Status launch_zero_ids(const uint64_t *blocks, uint64_t count);
    cudaError_t launch_copy(const CopyLaunch &a, cudaStream_t st) const;
    cudaError_t launch_zero(const ZeroLaunch &a, cudaStream_t st) const;
    Fp8Scales fp8_scales() const;
    Status fp8_source_error() const;
    Status upload_inv_scales();
    Status check(const char *what, cudaError_t e) const;

    pkv_config cfg_{};
    DType dtype_ = DType::F32;
    int device_ = 0;
    int sms_ = 148;
    int shard_rank_ = 0;
    int copy_engine_ = PKV_COPY_AUTO;
    int num_shards_ = 1;
    uint64_t shard_entry_ = 0;
    void *k_plane_ = nullptr;
    void *v_plane_ = nullptr;
    cudaStream_t stream_ = nullptr;
    DevError *d_err_ = nullptr;
    unsigned long long *d_digest_ = nullptr;
    // Reused staging (the reference allocates fresh device buffers per call).
    void *d_stage_ = nullptr;
    size_t d_stage_bytes_ = 0;
    void *h_stage_ = nullptr;  // pinned
    size_t h_stage_bytes_ = 0;
    cudaEvent_t h_stage_free_ = nullptr;  // last H2D out of h_stage_ has finished
    cudaEvent_t inputs_consumed_ = nullptr;
    // Host-path K/V uploads run on their own stream into two alternating
    // staging buffers, so that a call's upload overlaps the scatter of the
    // call before it; scatter_free_[i] marks the end of the last scatter
    // that read buffer i.
    cudaStream_t copy_stream_ = nullptr;
    void *d_scatter_[2] = {nullptr, nullptr};
    size_t d_scatter_bytes_[2] = {0, 0};
    cudaEvent_t scatter_free_[2] = {nullptr, nullptr};
    int scatter_turn_ = 0;
    std::vector<uint64_t> seen_;  // one bit per slot of a layer: duplicate detection
    // Host stager for large host-buffer writes (made on first use).
    static constexpr uint64_t kStageMinBytes = 1u << 20;
    std::unique_ptr<HostStager> stager_;
    bool host_staging_ = true;
    int host_threads_ = 16;
    size_t stage_chunk_bytes_ = 1u << 20;
    int stage_slots_ = 32;
    // fp8 pools: [num_layers][num_kv_heads] scales on the host, and their f32
    // reciprocals on the device (K's, then V's).
    std::vector<float> k_scale_, v_scale_;
    float *d_inv_ = nullptr;
    // Paged attention: TMA descriptors of the K and V planes (built on first
    // use) and the split workspace (grown on demand).
    alignas(64) unsigned char tmaps_[256] = {};
    bool tmaps_ready_ = false;
    float *d_attn_ws_ = nullptr;
    size_t d_attn_ws_bytes_ = 0;
    // The attention plan (sequence order, 65,535 entries) and the call shape
    // it was made for.
    unsigned *d_plan_ = nullptr;
    const int32_t *plan_ctx_ = nullptr;
    int64_t plan_seqs_ = -1, plan_max_ctx_ = -1;
    std::string gpu_name_;
};

}  // namespace pkv
