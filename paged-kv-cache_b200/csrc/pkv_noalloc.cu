// pkv_noalloc.cu -- pkv_resolve_and_cache_noalloc: slot resolution followed
// by reshape_and_cache for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc at all: a plugin that runs inside an
// inference engine which has already reserved (almost) all HBM for its own
// pool, or code that only receives buffers from such a manager. The regular
// path needs scratch that the library allocates (the backend's slot_mapping
// buffer and device error word). This entry point keeps that scratch in a
// fixed file-scope __device__ array instead, so it allocates nothing; the
// caller passes every input and output, including the pool planes.
//
// The scratch array is PKV_NOALLOC_SCRATCH_BYTES per GPU that loads the
// library and stays allocated until the process exits. All calls on a device
// share it: two calls whose work overlaps on the GPU (different streams, no
// ordering between them) race on it and may corrupt each other's slots.

#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "pkv_b200.h"
#include "pkv_backend.hpp"
#include "pkv_internal.hpp"

namespace {

constexpr size_t kErrBytes = 256;  // DevError, padded to keep the slots 256-byte aligned
constexpr size_t kScratchBytes = kErrBytes + sizeof(long long) * PKV_NOALLOC_MAX_TOKENS;
static_assert(kScratchBytes == PKV_NOALLOC_SCRATCH_BYTES, "header and scratch size disagree");
constexpr int kMaxDevices = 64;

// The scratch itself: [DevError | pad][slot_mapping of up to PKV_NOALLOC_MAX_TOKENS tokens].
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

// Device address of g_scratch on each device, looked up on the first call
// made with that device current (host code cannot use the symbol itself: on
// the host it names a stand-in, not device memory). A failed lookup is not
// remembered, so a later call tries again. The address belongs to the
// device's current context: calls after cudaDeviceReset are not supported.
std::mutex g_mu;
void *g_addr[kMaxDevices];

cudaError_t scratch_for(int device, void **out) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[device]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess) return e;
        g_addr[device] = p;
    }
    *out = g_addr[device];
    return cudaSuccess;
}

using pkv::error;
using pkv::Status;

Status resolve_and_cache_noalloc(const pkv_config *cfg, int pool_dtype, int shard_rank,
                                 int num_shards, void *k_plane, void *v_plane,
                                 const int32_t *block_tables, int64_t table_stride,
                                 const int32_t *ctx_lens, const int32_t *new_lens,
                                 int64_t num_seqs, int64_t num_tokens, int32_t *cu_seqlens,
                                 int64_t layer, const void *k, const void *v,
                                 int64_t src_token_stride, int64_t src_layer_stride,
                                 int src_dtype, int64_t *device_status, cudaStream_t s) {
    if (!cfg) return error(PKV_ERR_DEVICE, 0, 0, "null config");
    if (pool_dtype == PKV_FP8_E4M3 || src_dtype == PKV_FP8_E4M3)
        return error(PKV_ERR_DEVICE, 0, 0,
                     "pkv_resolve_and_cache_noalloc writes f32, bf16 and f16 pools only: an fp8 "
                     "(E4M3) pool needs the per-(layer, kv head) scales that a backend holds "
                     "(use pkv_resolve_and_cache_dev)");
    if (pool_dtype < PKV_F32 || pool_dtype > PKV_F16 || src_dtype < PKV_F32 || src_dtype > PKV_F16)
        return error(PKV_ERR_DEVICE, 0, 0, "unknown dtype tag");
    const auto pdt = static_cast<pkv::DType>(pool_dtype);
    if (cfg->dtype_bytes != (uint64_t)pkv::dtype_size(pdt))
        return error(PKV_ERR_DEVICE, 0, 0, "dtype_bytes does not match the pool dtype");
    const uint64_t full = cfg->num_kv_heads * cfg->head_dim;
    if (num_shards < 1 || shard_rank < 0 || shard_rank >= num_shards || full % num_shards != 0 ||
        cfg->block_size == 0)
        return error(PKV_ERR_DEVICE, 0, 0, "invalid geometry or shard");
    if (layer < -1 || (layer >= 0 && (uint64_t)layer >= cfg->num_layers))
        return error(PKV_ERR_INVALID_LAYER, layer, (int64_t)cfg->num_layers, "invalid layer");
    if (num_tokens < 0 || num_seqs < 0 || table_stride < 0)
        return error(PKV_ERR_SHAPE_MISMATCH, 0, -1, "negative size");
    if (num_tokens > PKV_NOALLOC_MAX_TOKENS)
        return error(PKV_ERR_SHAPE_MISMATCH, PKV_NOALLOC_MAX_TOKENS, num_tokens,
                     "pkv_resolve_and_cache_noalloc takes at most " +
                         std::to_string(PKV_NOALLOC_MAX_TOKENS) + " tokens per call, got " +
                         std::to_string(num_tokens));
    // Same limit, code and words as pkv_resolve_slots_dev / pkv_resolve_and_cache_dev.
    if (num_seqs > pkv::kMaxResolveSeqs)
        return error(PKV_ERR_DEVICE, 0, 0,
                     "slot resolution handles at most " + std::to_string(pkv::kMaxResolveSeqs) +
                         " sequences per call");
    const uint64_t entry = full / num_shards;
    if (src_token_stride <= 0) src_token_stride = (int64_t)entry;
    if ((uint64_t)src_token_stride < entry)
        return error(PKV_ERR_SHAPE_MISMATCH, (int64_t)entry, src_token_stride,
                     "token stride shorter than an entry");
    if (layer == -1 && src_layer_stride <= 0) src_layer_stride = src_token_stride * num_tokens;
    // As pkv_reshape_and_cache_dev: a layer's rows must not overlap the next layer's.
    if (layer == -1 && src_layer_stride < src_token_stride * num_tokens)
        return error(PKV_ERR_SHAPE_MISMATCH, src_token_stride * num_tokens, src_layer_stride,
                     "layer stride shorter than a layer's rows");
    if (!cu_seqlens || (num_seqs > 0 && (!ctx_lens || !new_lens)) ||
        (num_tokens > 0 && (!block_tables || !k || !v || !k_plane || !v_plane)))
        return error(PKV_ERR_DEVICE, 0, 0, "null device pointer");

    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return pkv::device_error("cudaGetDevice", e);
    if (device < 0 || device >= kMaxDevices) return error(PKV_ERR_DEVICE, 0, 0, "device index too large");
    void *scratch = nullptr;
    if ((e = scratch_for(device, &scratch)) != cudaSuccess)
        return pkv::device_error("cudaGetSymbolAddress", e);
    auto *err = static_cast<pkv::DevError *>(scratch);
    auto *slots = reinterpret_cast<long long *>(static_cast<unsigned char *>(scratch) + kErrBytes);
    const int sms = pkv::num_sms(device);

    // The scratch keeps the previous call's contents: clear the error word,
    // and set every slot to -1 (skip) so that tokens the resolution rejects
    // are never written with a stale slot.
    if ((e = cudaMemsetAsync(err, 0, sizeof(pkv::DevError), s)) != cudaSuccess ||
        (num_tokens > 0 && (e = cudaMemsetAsync(slots, 0xFF, num_tokens * sizeof(long long), s)) != cudaSuccess))
        return pkv::device_error("clearing scratch", e);

    pkv::ResolveLaunch r{};
    r.tables = block_tables;
    r.table_stride = table_stride;
    r.ctx_lens = ctx_lens;
    r.new_lens = new_lens;
    r.num_seqs = num_seqs;
    r.num_tokens = num_tokens;
    r.block_size = (long long)cfg->block_size;
    r.num_blocks = (long long)cfg->num_blocks;
    r.cu_seqlens = cu_seqlens;
    r.slots = slots;
    r.err = err;
    if ((e = pkv::launch_resolve_slots(r, sms, s)) != cudaSuccess)
        return pkv::device_error("resolve_slots", e);

    if (num_tokens > 0) {
        pkv::ReshapeLaunch a{};
        a.k = k;
        a.v = v;
        a.src_token_stride = src_token_stride;
        a.src_layer_stride = layer == -1 ? src_layer_stride : 0;
        a.k_pool = k_plane;
        a.v_pool = v_plane;
        a.first_layer = layer == -1 ? 0 : layer;
        a.num_layers = layer == -1 ? (long long)cfg->num_layers : 1;
        a.slots_per_layer = (long long)(cfg->num_blocks * cfg->block_size);
        a.entry_elems = (long long)entry;
        a.slots = slots;
        a.num_tokens = num_tokens;
        a.src_dtype = static_cast<pkv::DType>(src_dtype);
        a.pool_dtype = pdt;
        a.err = err;
        if ((e = pkv::launch_reshape(a, sms, s)) != cudaSuccess)
            return pkv::device_error("reshape_and_cache", e);
    }
    // {status, index} of the first bad index met, for callers that want it.
    if (device_status &&
        (e = cudaMemcpyAsync(device_status, err, sizeof(pkv::DevError), cudaMemcpyDeviceToDevice, s)) != cudaSuccess)
        return pkv::device_error("copying the device status", e);
    return Status::Ok();
}

}  // namespace

extern "C" int pkv_resolve_and_cache_noalloc(
    const pkv_config *cfg, int pool_dtype, int shard_rank, int num_shards, void *k_plane,
    void *v_plane, const int32_t *block_tables, int64_t table_stride, const int32_t *ctx_lens,
    const int32_t *new_lens, int64_t num_seqs, int64_t num_tokens, int32_t *cu_seqlens,
    int64_t layer, const void *k, const void *v, int64_t src_token_stride,
    int64_t src_layer_stride, int src_dtype, int64_t *device_status, void *stream) {
    return pkv::guarded("pkv_resolve_and_cache_noalloc", [&] {
        return resolve_and_cache_noalloc(cfg, pool_dtype, shard_rank, num_shards, k_plane, v_plane,
                                         block_tables, table_stride, ctx_lens, new_lens, num_seqs,
                                         num_tokens, cu_seqlens, layer, k, v, src_token_stride,
                                         src_layer_stride, src_dtype, device_status,
                                         static_cast<cudaStream_t>(stream));
    });
}
