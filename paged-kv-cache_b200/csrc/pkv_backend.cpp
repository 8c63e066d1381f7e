// pkv_backend.cpp -- host side of the B200 KvBackend: validation in the
// reference's order, staging, copy-pair scheduling and kernel launches.

#include "pkv_backend.hpp"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <unordered_map>

namespace pkv {

Status error(int code, int64_t a, int64_t b, std::string msg) {
    Status s;
    s.code = code;
    s.a = a;
    s.b = b;
    s.msg = std::move(msg);
    return s;
}

Status device_error(const std::string &what, cudaError_t e) {
    // Reset the runtime's last-error state, so that a recoverable failure
    // (an allocation that did not fit) is not reported again by the next
    // launch's cudaGetLastError.
    cudaGetLastError();
    return error(PKV_ERR_DEVICE, 0, 0, what + ": " + cudaGetErrorString(e));
}

namespace {

struct DeviceGuard {
    int prev = -1;
    int want;
    explicit DeviceGuard(int d) : want(d) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != want) cudaSetDevice(want);
    }
    ~DeviceGuard() {
        if (prev >= 0 && prev != want) cudaSetDevice(prev);
    }
};

constexpr size_t kAlign = 256;
size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Messages worded as the reference's CacheError Display impl (error.rs:42-76).
std::string msg_invalid_block(uint64_t id, uint64_t n) {
    return "invalid block #" + std::to_string(id) + ": pool holds " + std::to_string(n) + " blocks";
}
std::string msg_slot(uint64_t slot, uint64_t bs) {
    return "slot " + std::to_string(slot) + " out of range for block size " + std::to_string(bs);
}
std::string msg_shape(uint64_t e, uint64_t a) {
    return "shape mismatch: expected " + std::to_string(e) + " elements, got " + std::to_string(a);
}
std::string msg_layer(uint64_t l, uint64_t n) {
    return "invalid layer " + std::to_string(l) + ": model has " + std::to_string(n) + " layers";
}

// Exact f32 value of an E4M3 code (OCP OFP8 E4M3: bias 7, 3 mantissa bits,
// exponent 0 holds m * 2^-9, S.1111.111 is NaN).
float e4m3_to_f32(uint8_t q) {
    const uint32_t sign = uint32_t(q & 0x80) << 24, e = (q >> 3) & 0xfu, m = q & 7u;
    uint32_t bits;
    if (e == 15 && m == 7) {
        bits = sign | 0x7fc00000u;
    } else if (e == 0) {
        const float v = float(m) * (1.0f / 512.0f);
        std::memcpy(&bits, &v, 4);
        bits |= sign;
    } else {
        bits = sign | ((e + 120u) << 23) | (m << 20);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

float host_to_f32(const void *p, uint64_t i, DType t) {
    switch (t) {
        case DType::FP8_E4M3: return e4m3_to_f32(static_cast<const uint8_t *>(p)[i]);
        case DType::F32: return static_cast<const float *>(p)[i];
        case DType::BF16: {
            uint32_t bits = uint32_t(static_cast<const uint16_t *>(p)[i]) << 16;
            float f;
            std::memcpy(&f, &bits, 4);
            return f;
        }
        case DType::F16: return __half2float(static_cast<const __half *>(p)[i]);
    }
    return 0.f;
}

void host_from_f32(void *p, uint64_t i, DType t, float f) {
    switch (t) {
        case DType::F32: static_cast<float *>(p)[i] = f; break;
        case DType::BF16: static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(f); break;
        case DType::F16: static_cast<__half *>(p)[i] = __float2half_rn(f); break;
        case DType::FP8_E4M3: break;  // never a conversion target on the host
    }
}

// Convert `n` elements between host types (exact when widening, round to
// nearest even when narrowing); same type is a plain copy.
void host_convert(void *dst, DType dt, const void *src, DType st, uint64_t n) {
    if (dt == st) {
        std::memcpy(dst, src, n * dtype_size(st));
        return;
    }
    for (uint64_t i = 0; i < n; ++i) host_from_f32(dst, i, dt, host_to_f32(src, i, st));
}

}  // namespace

// ---------------------------------------------------------------------------
// construction: CudaBackend::new (crates/paged-kv-cuda/src/backend.rs:63-92)

Status B200Backend::create(const pkv_config &cfg, DType dtype, int device, int shard_rank,
                           int num_shards, std::unique_ptr<B200Backend> *out) {
    if (static_cast<int>(dtype) < 0 || static_cast<int>(dtype) > 3)
        return error(PKV_ERR_DEVICE, 0, 0, "invalid config: unknown dtype tag");
    if (cfg.dtype_bytes != static_cast<uint64_t>(dtype_size(dtype)))
        return error(PKV_ERR_DEVICE, 0, 0,
                     "invalid config: dtype_bytes " + std::to_string(cfg.dtype_bytes) +
                         " does not match the pool dtype (" + std::to_string(dtype_size(dtype)) +
                         " bytes)");
    if (num_shards < 1 || shard_rank < 0 || shard_rank >= num_shards)
        return error(PKV_ERR_DEVICE, 0, 0, "invalid shard: rank " + std::to_string(shard_rank) +
                                               " of " + std::to_string(num_shards));
    const uint64_t full_entry = cfg.num_kv_heads * cfg.head_dim;
    if (full_entry % static_cast<uint64_t>(num_shards) != 0)
        return error(PKV_ERR_DEVICE, 0, 0,
                     "invalid shard: entry of " + std::to_string(full_entry) +
                         " elements does not split into " + std::to_string(num_shards) + " shards");
    if (cfg.block_size == 0)
        return error(PKV_ERR_DEVICE, 0, 0, "invalid config: block_size must be positive");
    // Plane size must fit comfortably in signed 64-bit byte offsets.
    const long double plane_bytes = (long double)cfg.num_layers * cfg.num_blocks * cfg.block_size *
                                    (full_entry / num_shards) * dtype_size(dtype);
    if (plane_bytes > (long double)(1ull << 60))
        return error(PKV_ERR_DEVICE, 0, 0, "invalid config: pool too large");

    std::unique_ptr<B200Backend> b(new B200Backend());
    b->cfg_ = cfg;
    b->dtype_ = dtype;
    b->device_ = device;
    b->shard_rank_ = shard_rank;
    b->num_shards_ = num_shards;
    b->shard_entry_ = full_entry / num_shards;

    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess) return device_error("no CUDA device", e);
    if (device < 0 || device >= ndev)
        return error(PKV_ERR_DEVICE, 0, 0, "device " + std::to_string(device) + " not present");
    DeviceGuard g(device);
    cudaDeviceProp prop{};
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess)
        return device_error("cudaGetDeviceProperties", e);
    b->gpu_name_ = prop.name;
    b->sms_ = num_sms(device);
    // Host staging of large host-buffer writes: PKV_HOST_STAGING=off copies
    // straight from the caller's buffer instead (as the reference does);
    // PKV_HOST_THREADS sets the stager's worker count (default: one per
    // host core, up to 16).
    if (const char *m = std::getenv("PKV_HOST_STAGING")) b->host_staging_ = std::strcmp(m, "off") != 0;
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    b->host_threads_ = (int)std::min(16u, hw);
    if (const char *t = std::getenv("PKV_HOST_THREADS")) {
        const int n = std::atoi(t);
        if (n > 0) b->host_threads_ = std::min(n, HostStager::kMaxSlots / 2);
    }
    // Ring geometry (tuning): PKV_STAGE_CHUNK_KIB per chunk, PKV_STAGE_SLOTS chunks.
    if (const char *c = std::getenv("PKV_STAGE_CHUNK_KIB")) {
        const long n = std::atol(c);
        if (n > 0) b->stage_chunk_bytes_ = size_t(n) << 10;
    }
    if (const char *c = std::getenv("PKV_STAGE_SLOTS")) {
        const int n = std::atoi(c);
        if (n > 0) b->stage_slots_ = n;
    }
    // A blocking stream: host-buffer calls stay ordered with work that callers
    // issue on the legacy default stream.
    if ((e = cudaStreamCreateWithFlags(&b->stream_, cudaStreamDefault)) != cudaSuccess)
        return device_error("cudaStreamCreate", e);
    // Uploads of the caller's host rows into private staging need no order
    // with other streams' work: a non-blocking stream.
    if ((e = cudaStreamCreateWithFlags(&b->copy_stream_, cudaStreamNonBlocking)) != cudaSuccess)
        return device_error("cudaStreamCreate", e);
    if ((e = cudaEventCreateWithFlags(&b->h_stage_free_, cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&b->inputs_consumed_, cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&b->scatter_free_[0], cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&b->scatter_free_[1], cudaEventDisableTiming)) != cudaSuccess)
        return device_error("cudaEventCreate", e);

    const size_t plane = static_cast<size_t>(plane_bytes);
    if (plane > 0) {
        if ((e = cudaMalloc(&b->k_plane_, plane)) != cudaSuccess ||
            (e = cudaMalloc(&b->v_plane_, plane)) != cudaSuccess)
            return device_error("allocating a pool of 2 x " + std::to_string(plane) + " bytes", e);
        // alloc_zeros (crates/paged-kv-cuda/src/backend.rs:84-85).
        if ((e = cudaMemsetAsync(b->k_plane_, 0, plane, b->stream_)) != cudaSuccess ||
            (e = cudaMemsetAsync(b->v_plane_, 0, plane, b->stream_)) != cudaSuccess)
            return device_error("zeroing the pool", e);
    }
    if ((e = cudaMalloc(&b->d_err_, sizeof(DevError) + 2 * sizeof(unsigned long long))) !=
        cudaSuccess)
        return device_error("cudaMalloc", e);
    b->d_digest_ = reinterpret_cast<unsigned long long *>(b->d_err_ + 1);
    if ((e = cudaMemsetAsync(b->d_err_, 0, sizeof(DevError), b->stream_)) != cudaSuccess)
        return device_error("cudaMemset", e);
    if (dtype == DType::FP8_E4M3) {
        // Per (layer, kv head) scales of K and V, 1.0 until pkv_set_kv_scales.
        const size_t n = cfg.num_layers * cfg.num_kv_heads;
        b->k_scale_.assign(n, 1.0f);
        b->v_scale_.assign(n, 1.0f);
        // [k_inv][v_inv][k_scale][v_scale]: inverses for the quantising
        // writes, scales for attention's dequantisation.
        if ((e = cudaMalloc(&b->d_inv_, 4 * std::max<size_t>(n, 1) * sizeof(float))) != cudaSuccess)
            return device_error("allocating fp8 scales", e);
        Status st = b->upload_inv_scales();
        if (!st.ok()) return st;
    }
    if ((e = cudaStreamSynchronize(b->stream_)) != cudaSuccess) return device_error("init", e);
    *out = std::move(b);
    return Status::Ok();
}

B200Backend::~B200Backend() {
    DeviceGuard g(device_);
    stager_.reset();  // joins its workers; their copies are on copy_stream_
    if (stream_) cudaStreamSynchronize(stream_);
    if (copy_stream_) cudaStreamSynchronize(copy_stream_);
    if (k_plane_) cudaFree(k_plane_);
    if (v_plane_) cudaFree(v_plane_);
    if (d_err_) cudaFree(d_err_);
    if (d_inv_) cudaFree(d_inv_);
    if (d_attn_ws_) cudaFree(d_attn_ws_);
    if (d_plan_) cudaFree(d_plan_);
    if (d_stage_) cudaFree(d_stage_);
    if (h_stage_) cudaFreeHost(h_stage_);
    if (h_stage_free_) cudaEventDestroy(h_stage_free_);
    if (inputs_consumed_) cudaEventDestroy(inputs_consumed_);
    for (int i = 0; i < 2; ++i) {
        if (d_scatter_[i]) cudaFree(d_scatter_[i]);
        if (scatter_free_[i]) cudaEventDestroy(scatter_free_[i]);
    }
    if (copy_stream_) cudaStreamDestroy(copy_stream_);
    if (stream_) cudaStreamDestroy(stream_);
}

Status B200Backend::check(const char *what, cudaError_t e) const {
    if (e == cudaSuccess) return Status::Ok();
    return ::pkv::device_error(what, e);
}

uint64_t B200Backend::allocated_bytes() const {
    // CacheConfig::total_bytes (config.rs:74-76) for this backend's share of the entry.
    return 2 * cfg_.num_layers * cfg_.num_blocks * cfg_.block_size * shard_entry_ * cfg_.dtype_bytes;
}

std::string B200Backend::device_name() const {
    static const char *names[] = {"f32", "bf16", "f16", "fp8_e4m3"};
    std::string s = "cuda:" + std::to_string(device_) + " (" + gpu_name_ + ", " +
                    names[static_cast<int>(dtype_)];
    if (num_shards_ > 1)
        s += ", shard " + std::to_string(shard_rank_) + "/" + std::to_string(num_shards_);
    s += ", " + std::to_string(allocated_bytes() / (1024 * 1024)) + " MiB pool)";
    return s;
}

// validate_block (cpu.rs:72-80) and validate (cpu.rs:55-70).
Status B200Backend::validate_block(uint64_t block) const {
    if (block >= cfg_.num_blocks)
        return error(PKV_ERR_INVALID_BLOCK, (int64_t)block, (int64_t)cfg_.num_blocks,
                     msg_invalid_block(block, cfg_.num_blocks));
    return Status::Ok();
}

Status B200Backend::validate(uint64_t layer, pkv_slot at) const {
    if (layer >= cfg_.num_layers)
        return error(PKV_ERR_INVALID_LAYER, (int64_t)layer, (int64_t)cfg_.num_layers,
                     msg_layer(layer, cfg_.num_layers));
    Status s = validate_block(at.block);
    if (!s.ok()) return s;
    if (at.slot >= cfg_.block_size)
        return error(PKV_ERR_SLOT_OUT_OF_RANGE, (int64_t)at.slot, (int64_t)cfg_.block_size,
                     msg_slot(at.slot, cfg_.block_size));
    return Status::Ok();
}

Status B200Backend::ensure_device_stage(size_t bytes) {
    if (bytes <= d_stage_bytes_) return Status::Ok();
    cudaError_t e = cudaStreamSynchronize(stream_);  // old buffer may still be read
    if (e != cudaSuccess) return device_error("cudaStreamSynchronize", e);
    const size_t want = std::max(bytes, d_stage_bytes_ + d_stage_bytes_ / 2);
    if (d_stage_) cudaFree(d_stage_);
    d_stage_ = nullptr;
    d_stage_bytes_ = 0;
    if ((e = cudaMalloc(&d_stage_, want)) != cudaSuccess)
        return device_error("allocating " + std::to_string(want) + " bytes of staging", e);
    d_stage_bytes_ = want;
    return Status::Ok();
}

Status B200Backend::ensure_scatter_stage(int buf, size_t bytes) {
    if (bytes <= d_scatter_bytes_[buf]) return Status::Ok();
    // The old buffer may still be written by an upload or read by a scatter.
    cudaError_t e;
    if ((e = cudaStreamSynchronize(copy_stream_)) != cudaSuccess ||
        (e = cudaStreamSynchronize(stream_)) != cudaSuccess)
        return device_error("cudaStreamSynchronize", e);
    const size_t want = std::max(bytes, d_scatter_bytes_[buf] + d_scatter_bytes_[buf] / 2);
    if (d_scatter_[buf]) cudaFree(d_scatter_[buf]);
    d_scatter_[buf] = nullptr;
    d_scatter_bytes_[buf] = 0;
    if ((e = cudaMalloc(&d_scatter_[buf], want)) != cudaSuccess)
        return device_error("allocating " + std::to_string(want) + " bytes of staging", e);
    d_scatter_bytes_[buf] = want;
    return Status::Ok();
}

Status B200Backend::ensure_host_stage(size_t bytes) {
    cudaError_t e = cudaEventSynchronize(h_stage_free_);
    if (e != cudaSuccess) return device_error("cudaEventSynchronize", e);
    if (bytes <= h_stage_bytes_) return Status::Ok();
    if (h_stage_) cudaFreeHost(h_stage_);
    h_stage_ = nullptr;
    h_stage_bytes_ = 0;
    const size_t want = std::max<size_t>(bytes, 64 * 1024);
    if ((e = cudaMallocHost(&h_stage_, want)) != cudaSuccess)
        return device_error("allocating pinned staging", e);
    h_stage_bytes_ = want;
    return Status::Ok();
}

bool B200Backend::host_pinned(const void *p) const {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();  // not a CUDA-known pointer: pageable
        return false;
    }
    return at.type == cudaMemoryTypeHost;
}

Status B200Backend::stager(HostStager **out) {
    if (!stager_)
        stager_.reset(new HostStager(device_, copy_stream_, host_threads_, stage_chunk_bytes_,
                                     stage_slots_));
    *out = stager_.get();
    return Status::Ok();
}

// ---------------------------------------------------------------------------
// reshape_and_cache over host buffers

Status B200Backend::launch_scatter(uint64_t layer, const pkv_slot *dsts, uint64_t count,
                                   const void *k, const void *v, DType host) {
    if (count == 0) return Status::Ok();
    DeviceGuard g(device_);
    // Large batches from pageable memory, and f32 rows for a bf16 pool, go
    // through the host stager: worker threads copy (or narrow to bf16, which
    // halves the link bytes) into pinned chunks while earlier chunks upload.
    // Pinned rows of the pool's own type are copied straight from the caller.
    const bool narrow = host == DType::F32 && dtype_ == DType::BF16;
    bool staged = false;
    if (host_staging_ && count * shard_entry_ * dtype_size(host) >= kStageMinBytes)
        staged = narrow || !host_pinned(k) || !host_pinned(v);
    const DType sd = staged && narrow ? DType::BF16 : host;  // type of the rows on the device
    const size_t row_bytes = shard_entry_ * dtype_size(sd);
    const size_t slot_bytes = round_up(count * sizeof(int64_t), kAlign);
    const size_t kv_bytes = round_up(count * row_bytes, kAlign);
    const int buf = scatter_turn_;
    Status s = ensure_scatter_stage(buf, slot_bytes + 2 * kv_bytes);
    if (s.ok()) s = ensure_host_stage(count * sizeof(int64_t));
    if (!s.ok()) {
        // A batch whose first destination is invalid writes nothing and needs
        // no staging: report the validation error, as CpuBackend would.
        Status first = validate(layer, dsts[0]);
        return first.ok() ? s : first;
    }
    scatter_turn_ ^= 1;
    char *d = static_cast<char *>(d_scatter_[buf]);
    int64_t *d_slots = reinterpret_cast<int64_t *>(d);
    char *d_k = d + slot_bytes;
    char *d_v = d_k + kv_bytes;

    // The K/V rows go to the device first, on the upload stream, so that the
    // copy engine moves them while the host validates the destinations and
    // builds the slot list, and while the previous call's scatter (which read
    // the other staging buffer) still runs. Rows past a failing destination
    // are copied too but never scattered.
    cudaError_t e;
    if (staged) {
        HostStager *hs = nullptr;
        Status st = stager(&hs);
        if (!st.ok()) return st;
        const uint64_t n = count * shard_entry_;
        if ((e = cudaStreamWaitEvent(copy_stream_, scatter_free_[buf], 0)) ||
            (e = hs->begin(k, host, d_k, sd, n)) || (e = hs->begin(v, host, d_v, sd, n))) {
            hs->wait();  // never return while a worker may still read the caller's rows
            return device_error("staging K/V", e);
        }
    } else if ((e = cudaStreamWaitEvent(copy_stream_, scatter_free_[buf], 0)) ||
               (e = cudaMemcpyAsync(d_k, k, count * row_bytes, cudaMemcpyHostToDevice, copy_stream_)) ||
               (e = cudaMemcpyAsync(d_v, v, count * row_bytes, cudaMemcpyHostToDevice, copy_stream_)) ||
               (e = cudaEventRecord(inputs_consumed_, copy_stream_))) {
        cudaStreamSynchronize(copy_stream_);  // never return while a copy may still read the caller's rows
        return device_error("staging K/V", e);
    }
    // The caller's slices are borrowed: return only once they have been read
    // (by the copy engine, or by the stager's workers, whose pinned chunks
    // may still be uploading when this call returns).
    auto finish_with = [&](Status st) {
        const cudaError_t w = staged ? stager_->wait() : cudaEventSynchronize(inputs_consumed_);
        if (st.ok() && w != cudaSuccess) return device_error("staging K/V", w);
        return st;
    };

    // Validation in CpuBackend's order (cpu.rs:55-70); the items before the
    // first bad one are applied, as by the trait's default loop (backend.rs:70-72).
    uint64_t valid = 0;
    Status bad;
    for (; valid < count; ++valid) {
        bad = validate(layer, dsts[valid]);
        if (!bad.ok()) break;
    }
    if (valid == 0) return finish_with(bad);

    // Combined slot index block*block_size + slot (crates/paged-kv-cuda/src/backend.rs:172-175).
    // Within one batch the last write to a slot wins, as in the sequential
    // default write_kv_batch; earlier duplicates become padding (-1).
    int64_t *hs = static_cast<int64_t *>(h_stage_);
    for (uint64_t i = 0; i < valid; ++i) hs[i] = (int64_t)(dsts[i].block * cfg_.block_size + dsts[i].slot);
    if (valid > 1) {
        if (seen_.size() * 64 < slots_per_layer()) seen_.assign((slots_per_layer() + 63) / 64, 0);
        for (uint64_t i = valid; i-- > 0;) {
            const uint64_t x = (uint64_t)hs[i];
            uint64_t &w = seen_[x >> 6];
            const uint64_t bit = 1ull << (x & 63);
            if (w & bit) hs[i] = -1;
            else w |= bit;
        }
        for (uint64_t i = 0; i < valid; ++i)
            if (hs[i] >= 0) seen_[(uint64_t)hs[i] >> 6] = 0;
    }
    if (staged) {
        // Every chunk's copy is issued once wait() returns.
        if ((e = stager_->wait()) || (e = cudaEventRecord(inputs_consumed_, copy_stream_)))
            return finish_with(device_error("staging K/V", e));
    }
    if ((e = cudaMemcpyAsync(d_slots, hs, valid * sizeof(int64_t), cudaMemcpyHostToDevice, stream_)) ||
        (e = cudaEventRecord(h_stage_free_, stream_)) ||
        (e = cudaStreamWaitEvent(stream_, inputs_consumed_, 0)))
        return finish_with(device_error("staging slots", e));

    ReshapeLaunch a{};
    a.k = d_k;
    a.v = d_v;
    a.src_token_stride = (long long)shard_entry_;
    a.src_layer_stride = 0;
    a.k_pool = k_plane_;
    a.v_pool = v_plane_;
    a.first_layer = (long long)layer;
    a.num_layers = 1;
    a.slots_per_layer = (long long)slots_per_layer();
    a.entry_elems = (long long)shard_entry_;
    a.slots = reinterpret_cast<const long long *>(d_slots);
    a.num_tokens = (long long)valid;
    a.src_dtype = sd;
    a.pool_dtype = dtype_;
    a.err = d_err_;
    a.fp8 = fp8_scales();
    if ((e = launch_reshape(a, sms_, stream_)) != cudaSuccess ||
        (e = cudaEventRecord(scatter_free_[buf], stream_)) != cudaSuccess)
        return finish_with(device_error("reshape_and_cache", e));
    return finish_with(bad);
}

// write_kv (cpu.rs:95-111): validate, then K length, then V length.
Status B200Backend::write_kv(uint64_t layer, pkv_slot dst, const void *k, uint64_t k_len,
                             const void *v, uint64_t v_len, DType host) {
    if (host == DType::FP8_E4M3 && dtype_ != DType::FP8_E4M3) return fp8_source_error();
    Status s = validate(layer, dst);
    if (!s.ok()) return s;
    if (k_len != shard_entry_)
        return error(PKV_ERR_SHAPE_MISMATCH, (int64_t)shard_entry_, (int64_t)k_len, msg_shape(shard_entry_, k_len));
    if (v_len != shard_entry_)
        return error(PKV_ERR_SHAPE_MISMATCH, (int64_t)shard_entry_, (int64_t)v_len, msg_shape(shard_entry_, v_len));
    return launch_scatter(layer, &dst, 1, k, v, host);
}

// write_kv_batch (backend.rs:55-74): K shape, V shape, then per-token
// validation in order; tokens before the first invalid one are written.
Status B200Backend::write_kv_batch(uint64_t layer, const pkv_slot *dsts, uint64_t count,
                                   const void *k, uint64_t k_len, const void *v, uint64_t v_len,
                                   DType host) {
    if (host == DType::FP8_E4M3 && dtype_ != DType::FP8_E4M3) return fp8_source_error();
    const uint64_t expected = count * shard_entry_;
    if (k_len != expected)
        return error(PKV_ERR_SHAPE_MISMATCH, (int64_t)expected, (int64_t)k_len, msg_shape(expected, k_len));
    if (v_len != expected)
        return error(PKV_ERR_SHAPE_MISMATCH, (int64_t)expected, (int64_t)v_len, msg_shape(expected, v_len));
    return launch_scatter(layer, dsts, count, k, v, host);
}

// read_kv (cpu.rs:113-129): only the requested entry crosses PCIe.
Status B200Backend::read_kv(uint64_t layer, pkv_slot src, void *k_out, uint64_t k_len, void *v_out,
                            uint64_t v_len, DType host) {
    if (host == DType::FP8_E4M3 && dtype_ != DType::FP8_E4M3) return fp8_source_error();
    Status s = validate(layer, src);
    if (!s.ok()) return s;
    if (k_len != shard_entry_)
        return error(PKV_ERR_SHAPE_MISMATCH, (int64_t)shard_entry_, (int64_t)k_len, msg_shape(shard_entry_, k_len));
    if (v_len != shard_entry_)
        return error(PKV_ERR_SHAPE_MISMATCH, (int64_t)shard_entry_, (int64_t)v_len, msg_shape(shard_entry_, v_len));
    DeviceGuard g(device_);
    const size_t eb = entry_bytes();
    if (!(s = ensure_host_stage(2 * eb)).ok()) return s;
    const size_t off = ((layer * cfg_.num_blocks + src.block) * cfg_.block_size + src.slot) * eb;
    char *h = static_cast<char *>(h_stage_);
    cudaError_t e;
    if ((e = cudaMemcpyAsync(h, static_cast<char *>(k_plane_) + off, eb, cudaMemcpyDeviceToHost, stream_)) ||
        (e = cudaMemcpyAsync(h + eb, static_cast<char *>(v_plane_) + off, eb, cudaMemcpyDeviceToHost, stream_)) ||
        (e = cudaEventRecord(h_stage_free_, stream_)) || (e = cudaStreamSynchronize(stream_)))
        return device_error("read_kv", e);
    if (dtype_ == DType::FP8_E4M3 && host != DType::FP8_E4M3) {
        // Dequantise: the widened code times its (layer, kv head) scale.
        const uint64_t hd = cfg_.head_dim, base = layer * cfg_.num_kv_heads, off0 = elem_offset();
        for (uint64_t i = 0; i < shard_entry_; ++i) {
            const uint64_t sc = base + (off0 + i) / hd;
            host_from_f32(k_out, i, host, e4m3_to_f32(static_cast<uint8_t>(h[i])) * k_scale_[sc]);
            host_from_f32(v_out, i, host, e4m3_to_f32(static_cast<uint8_t>(h[eb + i])) * v_scale_[sc]);
        }
        return Status::Ok();
    }
    host_convert(k_out, host, h, dtype_, shard_entry_);
    host_convert(v_out, host, h + eb, dtype_, shard_entry_);
    return Status::Ok();
}

Fp8Scales B200Backend::fp8_scales() const {
    Fp8Scales f;
    if (dtype_ != DType::FP8_E4M3) return f;
    const long long n = (long long)(cfg_.num_layers * cfg_.num_kv_heads);
    f.k_inv = d_inv_;
    f.v_inv = d_inv_ + std::max<long long>(n, 1);
    f.heads = (long long)cfg_.num_kv_heads;
    f.head_dim = (long long)cfg_.head_dim;
    f.elem_offset = (long long)elem_offset();
    return f;
}

Status B200Backend::fp8_source_error() const {
    return error(PKV_ERR_DEVICE, 0, 0, "E4M3 rows can only be written to (or read from) an fp8 pool");
}

Status B200Backend::upload_inv_scales() {
    const size_t n = k_scale_.size(), stride = std::max<size_t>(n, 1);
    std::vector<float> inv(4 * stride, 1.0f);
    for (size_t i = 0; i < n; ++i) {
        inv[i] = 1.0f / k_scale_[i];  // IEEE f32 division, rounded to nearest even
        inv[stride + i] = 1.0f / v_scale_[i];
        inv[2 * stride + i] = k_scale_[i];
        inv[3 * stride + i] = v_scale_[i];
    }
    DeviceGuard g(device_);
    cudaError_t e;
    if ((e = cudaMemcpyAsync(d_inv_, inv.data(), inv.size() * sizeof(float), cudaMemcpyHostToDevice,
                             stream_)) != cudaSuccess ||
        (e = cudaStreamSynchronize(stream_)) != cudaSuccess)
        return device_error("uploading fp8 scales", e);
    return Status::Ok();
}

Status B200Backend::set_kv_scales(const float *k_scales, const float *v_scales, uint64_t count) {
    if (dtype_ != DType::FP8_E4M3)
        return error(PKV_ERR_DEVICE, 0, 0, "kv scales apply to fp8 (E4M3) pools only");
    const uint64_t n = cfg_.num_layers * cfg_.num_kv_heads;
    if (count != n) return error(PKV_ERR_SHAPE_MISMATCH, (int64_t)n, (int64_t)count, msg_shape(n, count));
    if (n > 0 && (!k_scales || !v_scales)) return error(PKV_ERR_DEVICE, 0, 0, "null scale array");
    for (uint64_t i = 0; i < n; ++i)
        for (float x : {k_scales[i], v_scales[i]})
            if (!(x > 0.0f) || !std::isfinite(x) || !std::isfinite(1.0f / x))
                return error(PKV_ERR_DEVICE, (int64_t)i, 0,
                             "kv scale " + std::to_string(i) + " must be finite and positive, with a finite reciprocal");
    k_scale_.assign(k_scales, k_scales + n);
    v_scale_.assign(v_scales, v_scales + n);
    return upload_inv_scales();
}

// ---------------------------------------------------------------------------
// copy_blocks

// Launch pairs (all valid) so that the result equals applying them one after
// another (backend.rs:104-109). Self-copies are dropped (cpu.rs:134-136).
// Pairs go into waves: a pair waits for every earlier pair that writes its
// source, reads its destination or writes its destination. Copy-on-write
// pairs always have fresh destinations, so they form a single wave.
Status B200Backend::launch_copy_pairs(const uint64_t *pairs, uint64_t count) {
    std::vector<int64_t> flat;
    std::vector<int> wave;
    flat.reserve(2 * count);
    wave.reserve(count);
    std::unordered_map<uint64_t, int> last_write, last_read;
    int max_wave = 0;
    for (uint64_t i = 0; i < count; ++i) {
        const uint64_t src = pairs[2 * i], dst = pairs[2 * i + 1];
        if (src == dst) continue;
        int w = 0;
        auto it = last_write.find(src);
        if (it != last_write.end()) w = std::max(w, it->second + 1);
        it = last_read.find(dst);
        if (it != last_read.end()) w = std::max(w, it->second + 1);
        it = last_write.find(dst);
        if (it != last_write.end()) w = std::max(w, it->second + 1);
        last_write[dst] = w;
        auto r = last_read.find(src);
        if (r == last_read.end()) last_read[src] = w;
        else r->second = std::max(r->second, w);
        flat.push_back((int64_t)src);
        flat.push_back((int64_t)dst);
        wave.push_back(w);
        max_wave = std::max(max_wave, w);
    }
    const uint64_t n = wave.size();
    if (n == 0) return Status::Ok();
    DeviceGuard g(device_);
    Status s = ensure_device_stage(round_up(n * 16, kAlign));
    if (!s.ok()) return s;
    if (!(s = ensure_host_stage(n * 16)).ok()) return s;
    int64_t *h = static_cast<int64_t *>(h_stage_);
    std::vector<std::pair<uint64_t, uint64_t>> ranges;  // [begin, end) per wave
    uint64_t pos = 0;
    for (int w = 0; w <= max_wave; ++w) {
        const uint64_t begin = pos;
        for (uint64_t i = 0; i < n; ++i)
            if (wave[i] == w) {
                h[2 * pos] = flat[2 * i];
                h[2 * pos + 1] = flat[2 * i + 1];
                ++pos;
            }
        if (pos > begin) ranges.emplace_back(begin, pos);
    }
    cudaError_t e;
    if ((e = cudaMemcpyAsync(d_stage_, h, n * 16, cudaMemcpyHostToDevice, stream_)) ||
        (e = cudaEventRecord(h_stage_free_, stream_)))
        return device_error("staging copy pairs", e);
    for (auto &r : ranges) {
        CopyLaunch a{};
        a.k_pool = k_plane_;
        a.v_pool = v_plane_;
        a.num_layers = (long long)cfg_.num_layers;
        a.num_blocks = (long long)cfg_.num_blocks;
        a.block_bytes = (long long)block_bytes();
        a.pairs = static_cast<const long long *>(d_stage_) + 2 * r.first;
        a.num_pairs = (long long)(r.second - r.first);
        a.err = d_err_;
        if ((e = launch_copy(a, stream_)) != cudaSuccess) return device_error("copy_blocks", e);
    }
    return Status::Ok();
}

// copy_block (cpu.rs:131-149).
Status B200Backend::copy_block(uint64_t src, uint64_t dst) {
    Status s = validate_block(src);
    if (!s.ok()) return s;
    if (!(s = validate_block(dst)).ok()) return s;
    if (src == dst) return Status::Ok();
    const uint64_t pair[2] = {src, dst};
    return launch_copy_pairs(pair, 1);
}

// copy_blocks (backend.rs:104-109): pairs before the first invalid one apply.
Status B200Backend::copy_blocks(const uint64_t *pairs, uint64_t count) {
    uint64_t valid = 0;
    Status bad;
    for (; valid < count; ++valid) {
        bad = validate_block(pairs[2 * valid]);
        if (!bad.ok()) break;
        bad = validate_block(pairs[2 * valid + 1]);
        if (!bad.ok()) break;
    }
    Status s = launch_copy_pairs(pairs, valid);
    if (!s.ok()) return s;
    return bad;
}

// ---------------------------------------------------------------------------
// zero_block

Status B200Backend::launch_zero_ids(const uint64_t *blocks, uint64_t count) {
    if (count == 0) return Status::Ok();
    DeviceGuard g(device_);
    Status s = ensure_device_stage(round_up(count * 8, kAlign));
    if (!s.ok()) return s;
    if (!(s = ensure_host_stage(count * 8)).ok()) return s;
    std::memcpy(h_stage_, blocks, count * 8);
    cudaError_t e;
    if ((e = cudaMemcpyAsync(d_stage_, h_stage_, count * 8, cudaMemcpyHostToDevice, stream_)) ||
        (e = cudaEventRecord(h_stage_free_, stream_)))
        return device_error("staging block ids", e);
    ZeroLaunch a{};
    a.k_pool = k_plane_;
    a.v_pool = v_plane_;
    a.num_layers = (long long)cfg_.num_layers;
    a.num_blocks = (long long)cfg_.num_blocks;
    a.block_bytes = (long long)block_bytes();
    a.blocks = static_cast<const long long *>(d_stage_);
    a.num_ids = (long long)count;
    a.err = d_err_;
    if ((e = launch_zero(a, stream_)) != cudaSuccess) return device_error("zero_blocks", e);
    return Status::Ok();
}

// zero_block (cpu.rs:151-160).
Status B200Backend::zero_block(uint64_t block) {
    Status s = validate_block(block);
    if (!s.ok()) return s;
    return launch_zero_ids(&block, 1);
}

Status B200Backend::zero_blocks(const uint64_t *blocks, uint64_t count) {
    uint64_t valid = 0;
    Status bad;
    for (; valid < count; ++valid) {
        bad = validate_block(blocks[valid]);
        if (!bad.ok()) break;
    }
    Status s = launch_zero_ids(blocks, valid);
    if (!s.ok()) return s;
    return bad;
}

// ---------------------------------------------------------------------------
// device entry points

Status B200Backend::reshape_and_cache_dev(int64_t layer, const void *k, const void *v,
                                          int64_t tok_stride, int64_t layer_stride,
                                          const int64_t *slots, int64_t num_tokens, DType src,
                                          cudaStream_t st) {
    if (layer < -1 || (layer >= 0 && (uint64_t)layer >= cfg_.num_layers))
        return error(PKV_ERR_INVALID_LAYER, layer, (int64_t)cfg_.num_layers,
                     msg_layer((uint64_t)layer, cfg_.num_layers));
    if (num_tokens < 0)
        return error(PKV_ERR_SHAPE_MISMATCH, 0, num_tokens, "negative token count");
    if (num_tokens == 0) return Status::Ok();
    if (!k || !v || !slots) return error(PKV_ERR_DEVICE, 0, 0, "null device pointer");
    if (static_cast<int>(src) < 0 || static_cast<int>(src) > 3)
        return error(PKV_ERR_DEVICE, 0, 0, "unknown source dtype tag");
    if (src == DType::FP8_E4M3 && dtype_ != DType::FP8_E4M3) return fp8_source_error();
    if (tok_stride <= 0) tok_stride = (int64_t)shard_entry_;
    if ((uint64_t)tok_stride < shard_entry_)
        return error(PKV_ERR_SHAPE_MISMATCH, (int64_t)shard_entry_, tok_stride,
                     "token stride shorter than an entry");
    const bool all = layer == -1;
    if (all && layer_stride <= 0) layer_stride = tok_stride * num_tokens;
    if (all && layer_stride < tok_stride * num_tokens)
        return error(PKV_ERR_SHAPE_MISMATCH, tok_stride * num_tokens, layer_stride,
                     "layer stride shorter than a layer's rows");
    DeviceGuard g(device_);
    ReshapeLaunch a{};
    a.k = k;
    a.v = v;
    a.src_token_stride = tok_stride;
    a.src_layer_stride = all ? layer_stride : 0;
    a.k_pool = k_plane_;
    a.v_pool = v_plane_;
    a.first_layer = all ? 0 : layer;
    a.num_layers = all ? (long long)cfg_.num_layers : 1;
    a.slots_per_layer = (long long)slots_per_layer();
    a.entry_elems = (long long)shard_entry_;
    a.slots = reinterpret_cast<const long long *>(slots);
    a.num_tokens = num_tokens;
    a.src_dtype = src;
    a.pool_dtype = dtype_;
    a.err = d_err_;
    a.fp8 = fp8_scales();
    return check("reshape_and_cache", launch_reshape(a, sms_, st));
}

Status B200Backend::copy_blocks_dev(const int64_t *pairs, int64_t count, cudaStream_t st) {
    if (count < 0) return error(PKV_ERR_SHAPE_MISMATCH, 0, count, "negative pair count");
    if (count == 0) return Status::Ok();
    if (!pairs) return error(PKV_ERR_DEVICE, 0, 0, "null device pointer");
    DeviceGuard g(device_);
    CopyLaunch a{};
    a.k_pool = k_plane_;
    a.v_pool = v_plane_;
    a.num_layers = (long long)cfg_.num_layers;
    a.num_blocks = (long long)cfg_.num_blocks;
    a.block_bytes = (long long)block_bytes();
    a.pairs = reinterpret_cast<const long long *>(pairs);
    a.num_pairs = count;
    a.err = d_err_;
    return check("copy_blocks", launch_copy(a, st));
}

cudaError_t B200Backend::launch_copy(const CopyLaunch &a, cudaStream_t st) const {
    // AUTO takes the register path: on B200 both engines reach the copy peak
    // for 16 KiB plane-blocks, and the vector kernel needs no shared memory.
    if (copy_engine_ == PKV_COPY_BULK) return launch_copy_blocks_bulk(a, sms_, st);
    return launch_copy_blocks(a, st);
}

cudaError_t B200Backend::launch_zero(const ZeroLaunch &a, cudaStream_t st) const {
    if (copy_engine_ == PKV_COPY_BULK) return launch_zero_blocks_bulk(a, sms_, st);
    return launch_zero_blocks(a, st);
}

Status B200Backend::set_copy_engine(int engine) {
    if (engine != PKV_COPY_AUTO && engine != PKV_COPY_VECTOR && engine != PKV_COPY_BULK)
        return error(PKV_ERR_DEVICE, 0, 0, "unknown copy engine " + std::to_string(engine));
    if (engine == PKV_COPY_BULK) {
        CopyLaunch a{};
        a.k_pool = k_plane_;
        a.v_pool = v_plane_;
        a.block_bytes = (long long)block_bytes();
        if (!bulk_copy_supported(a))
            return error(PKV_ERR_DEVICE, 0, 0,
                         "bulk copy engine needs block planes that split into 16-byte runs of "
                         "at most 32 KiB; this pool has " +
                             std::to_string(block_bytes()) + "-byte block planes");
    }
    copy_engine_ = engine;
    return Status::Ok();
}

Status B200Backend::zero_blocks_dev(const int64_t *blocks, int64_t count, cudaStream_t st) {
    if (count < 0) return error(PKV_ERR_SHAPE_MISMATCH, 0, count, "negative block count");
    if (count == 0) return Status::Ok();
    if (!blocks) return error(PKV_ERR_DEVICE, 0, 0, "null device pointer");
    DeviceGuard g(device_);
    ZeroLaunch a{};
    a.k_pool = k_plane_;
    a.v_pool = v_plane_;
    a.num_layers = (long long)cfg_.num_layers;
    a.num_blocks = (long long)cfg_.num_blocks;
    a.block_bytes = (long long)block_bytes();
    a.blocks = reinterpret_cast<const long long *>(blocks);
    a.num_ids = count;
    a.err = d_err_;
    return check("zero_blocks", launch_zero(a, st));
}

Status B200Backend::copy_zero_dev(const int64_t *srcs, const int64_t *dst_off, const int64_t *dsts,
                                  const int64_t *zero_src, int64_t num_srcs,
                                  const int64_t *zero_ids, int64_t num_zero, cudaStream_t st) {
    if (num_srcs < 0 || num_zero < 0)
        return error(PKV_ERR_SHAPE_MISMATCH, 0, std::min(num_srcs, num_zero), "negative count");
    if (num_srcs == 0 && num_zero == 0) return Status::Ok();
    if ((num_srcs > 0 && (!srcs || !dst_off || !dsts || !zero_src)) || (num_zero > 0 && !zero_ids))
        return error(PKV_ERR_DEVICE, 0, 0, "null device pointer");
    DeviceGuard g(device_);
    CopyZeroLaunch a{};
    a.k_pool = k_plane_;
    a.v_pool = v_plane_;
    a.num_layers = (long long)cfg_.num_layers;
    a.num_blocks = (long long)cfg_.num_blocks;
    a.block_bytes = (long long)block_bytes();
    a.srcs = reinterpret_cast<const long long *>(srcs);
    a.dst_off = reinterpret_cast<const long long *>(dst_off);
    a.dsts = reinterpret_cast<const long long *>(dsts);
    a.zero_src = reinterpret_cast<const long long *>(zero_src);
    a.num_srcs = num_srcs;
    a.zero_ids = reinterpret_cast<const long long *>(zero_ids);
    a.num_zero = num_zero;
    a.err = d_err_;
    return check("copy_zero_blocks", launch_copy_zero(a, st));
}

Status B200Backend::resolve_slots_dev(const int32_t *tables, int64_t table_stride,
                                      const int32_t *ctx, const int32_t *new_lens,
                                      int64_t num_seqs, int64_t num_tokens, int32_t *cu,
                                      int64_t *slots, cudaStream_t st) {
    if (num_seqs < 0 || num_tokens < 0 || table_stride < 0)
        return error(PKV_ERR_SHAPE_MISMATCH, 0, std::min({num_seqs, num_tokens, table_stride}),
                     "negative size");
    if (num_seqs > kMaxResolveSeqs)
        return error(PKV_ERR_DEVICE, 0, 0,
                     "slot resolution handles at most " + std::to_string(kMaxResolveSeqs) +
                         " sequences per call");
    if (num_tokens > std::numeric_limits<int32_t>::max())
        return error(PKV_ERR_SHAPE_MISMATCH, std::numeric_limits<int32_t>::max(), num_tokens,
                     "too many tokens for int32 cu_seqlens");
    if (!cu || (num_seqs > 0 && (!ctx || !new_lens)) || (num_tokens > 0 && (!tables || !slots)))
        return error(PKV_ERR_DEVICE, 0, 0, "null device pointer");
    DeviceGuard g(device_);
    ResolveLaunch a{};
    a.tables = tables;
    a.table_stride = table_stride;
    a.ctx_lens = ctx;
    a.new_lens = new_lens;
    a.num_seqs = num_seqs;
    a.num_tokens = num_tokens;
    a.block_size = (long long)cfg_.block_size;
    a.num_blocks = (long long)cfg_.num_blocks;
    a.cu_seqlens = cu;
    a.slots = reinterpret_cast<long long *>(slots);
    a.err = d_err_;
    return check("resolve_slots", launch_resolve_slots(a, sms_, st));
}

Status B200Backend::resolve_and_cache_dev(const int32_t *tables, int64_t table_stride,
                                          const int32_t *ctx, const int32_t *new_lens,
                                          int64_t num_seqs, int64_t num_tokens, int32_t *cu,
                                          int64_t *slots_out, int64_t layer, const void *k,
                                          const void *v, int64_t tok_stride,
                                          int64_t layer_stride, DType src, cudaStream_t st,
                                          const int64_t *direct_slots, int64_t num_direct) {
    if (layer < -1 || (layer >= 0 && (uint64_t)layer >= cfg_.num_layers))
        return error(PKV_ERR_INVALID_LAYER, layer, (int64_t)cfg_.num_layers,
                     msg_layer((uint64_t)layer, cfg_.num_layers));
    if (num_seqs < 0 || num_tokens < 0 || table_stride < 0)
        return error(PKV_ERR_SHAPE_MISMATCH, 0, std::min({num_seqs, num_tokens, table_stride}),
                     "negative size");
    if (num_seqs > kMaxResolveSeqs)
        return error(PKV_ERR_DEVICE, 0, 0,
                     "slot resolution handles at most " + std::to_string(kMaxResolveSeqs) +
                         " sequences per call");
    if (num_tokens > std::numeric_limits<int32_t>::max())
        return error(PKV_ERR_SHAPE_MISMATCH, std::numeric_limits<int32_t>::max(), num_tokens,
                     "too many tokens for int32 cu_seqlens");
    const bool quantise = dtype_ == DType::FP8_E4M3 && src != DType::FP8_E4M3;
    if (static_cast<int>(src) < 0 || static_cast<int>(src) > 3)
        return error(PKV_ERR_DEVICE, 0, 0, "unknown source dtype tag");
    if (src != dtype_ && !quantise)
        return error(PKV_ERR_DEVICE, 0, 0,
                     "the fused path moves bytes, or quantises into an fp8 pool: source dtype "
                     "must equal the pool dtype (use pkv_resolve_slots_dev + "
                     "pkv_reshape_and_cache_dev to convert)");
    if (num_direct < 0)
        return error(PKV_ERR_SHAPE_MISMATCH, 0, num_direct, "negative direct token count");
    if (num_direct > 0 && quantise)
        return error(PKV_ERR_DEVICE, 0, 0,
                     "host-slot tokens in the fused step are for pools of the source's type; "
                     "an fp8 pool takes them through pkv_reshape_and_cache_dev");
    if (num_tokens + num_direct > std::numeric_limits<int32_t>::max())
        return error(PKV_ERR_SHAPE_MISMATCH, std::numeric_limits<int32_t>::max(),
                     num_tokens + num_direct, "too many tokens for one step");
    if (!cu || (num_seqs > 0 && (!ctx || !new_lens)) ||
        (num_tokens > 0 && (!tables || !k || !v)) ||
        (num_direct > 0 && (!direct_slots || !k || !v)))
        return error(PKV_ERR_DEVICE, 0, 0, "null device pointer");
    const int64_t rows = num_tokens + num_direct;  // source rows the launch reads
    if (tok_stride <= 0) tok_stride = (int64_t)shard_entry_;
    if ((uint64_t)tok_stride < shard_entry_)
        return error(PKV_ERR_SHAPE_MISMATCH, (int64_t)shard_entry_, tok_stride,
                     "token stride shorter than an entry");
    const bool all = layer == -1;
    if (all && layer_stride <= 0) layer_stride = tok_stride * rows;
    if (all && layer_stride < tok_stride * rows)
        return error(PKV_ERR_SHAPE_MISMATCH, tok_stride * rows, layer_stride,
                     "layer stride shorter than a layer's rows");
    DeviceGuard g(device_);
    const int es = dtype_size(src);
    ResolveCacheLaunch a{};
    a.tables = tables;
    a.table_stride = table_stride;
    a.ctx_lens = ctx;
    a.new_lens = new_lens;
    a.num_seqs = num_seqs;
    a.num_tokens = num_tokens;
    a.block_size = (long long)cfg_.block_size;
    a.num_blocks = (long long)cfg_.num_blocks;
    a.cu_seqlens = cu;
    a.slots_out = reinterpret_cast<long long *>(slots_out);
    a.k = k;
    a.v = v;
    a.src_token_stride_bytes = tok_stride * es;
    a.src_layer_stride_bytes = all ? layer_stride * es : 0;
    a.k_pool = k_plane_;
    a.v_pool = v_plane_;
    a.first_layer = all ? 0 : layer;
    a.num_layers = all ? (long long)cfg_.num_layers : 1;
    a.slots_per_layer = (long long)slots_per_layer();
    a.entry_bytes = (long long)entry_bytes();
    a.err = d_err_;
    a.direct_slots = reinterpret_cast<const long long *>(direct_slots);
    a.num_direct = num_direct;
    if (quantise) {
        a.src_dtype = src;
        a.pool_dtype = dtype_;
        a.entry_elems = (long long)shard_entry_;
        a.fp8 = fp8_scales();
        return check("resolve_and_cache", launch_resolve_cache_fp8(a, sms_, st));
    }
    return check("resolve_and_cache", launch_resolve_cache(a, sms_, st));
}

// Decode attention over one layer (no counterpart in the reference: the
// trait leaves paged_attention for later, crates/paged-kv-core/src/backend.rs:18-22).
Status B200Backend::paged_attention_dev(int64_t layer, const void *q, DType query, int64_t q_seq_stride,
                                        int64_t num_seqs, int64_t num_q_heads,
                                        const int32_t *tables, int64_t table_stride,
                                        const int32_t *ctx, int64_t max_ctx, float softmax_scale,
                                        void *out, float *lse, cudaStream_t st, int64_t q_len) {
    if (layer < 0 || (uint64_t)layer >= cfg_.num_layers)
        return error(PKV_ERR_INVALID_LAYER, layer, (int64_t)cfg_.num_layers,
                     msg_layer((uint64_t)layer, cfg_.num_layers));
    if (dtype_ == DType::FP8_E4M3) {
        if (query != DType::BF16 && query != DType::F16)
            return error(PKV_ERR_DEVICE, 0, 0, "attention over an fp8 pool takes bf16 or f16 queries");
    } else if (dtype_ != DType::BF16 && dtype_ != DType::F16) {
        return error(PKV_ERR_DEVICE, 0, 0, "paged attention reads bf16, f16 or fp8 (E4M3) pools");
    } else if (query != dtype_) {
        return error(PKV_ERR_DEVICE, 0, 0, "queries must have the pool dtype (bf16 or f16)");
    }
    if (cfg_.block_size != 16)
        return error(PKV_ERR_DEVICE, 0, 0, "paged attention needs block_size 16");
    const uint64_t hd = cfg_.head_dim;
    if (hd != 64 && hd != 128 && hd != 256)
        return error(PKV_ERR_DEVICE, 0, 0, "paged attention supports head_dim 64, 128 or 256");
    if (elem_offset() % hd != 0 || shard_entry_ % hd != 0)
        return error(PKV_ERR_DEVICE, 0, 0, "paged attention needs whole kv heads in this shard");
    const int64_t kv = (int64_t)(shard_entry_ / hd);
    if (num_seqs < 0 || num_q_heads <= 0 || num_q_heads % kv != 0)
        return error(PKV_ERR_SHAPE_MISMATCH, kv, num_q_heads,
                     "query heads must be a positive multiple of the kv heads held here");
    const int64_t group = num_q_heads / kv;
    if (group > 16)
        return error(PKV_ERR_DEVICE, 0, 0, "paged attention supports at most 16 query heads per kv head");
    if (q_len < 1 || q_len * group > 16)
        return error(PKV_ERR_DEVICE, 0, 0,
                     "paged attention takes 1 <= q_len and q_len * (query heads per kv head) <= 16");
    if (num_seqs == 0) return Status::Ok();
    if (num_seqs > 65535) return error(PKV_ERR_DEVICE, 0, 0, "at most 65535 sequences per call");
    if (max_ctx < 0 || table_stride < 0 || max_ctx > table_stride * (int64_t)cfg_.block_size ||
        max_ctx > std::numeric_limits<int32_t>::max() - 16)
        return error(PKV_ERR_SHAPE_MISMATCH, table_stride * (int64_t)cfg_.block_size, max_ctx,
                     "max_context_len exceeds the block tables");
    if (q_seq_stride <= 0) q_seq_stride = num_q_heads * (int64_t)hd;
    if (q_seq_stride < num_q_heads * (int64_t)hd || q_seq_stride % 8 != 0)
        return error(PKV_ERR_SHAPE_MISMATCH, num_q_heads * (int64_t)hd, q_seq_stride,
                     "query row pitch must cover the heads and be a multiple of 8 elements");
    if (!q || !out || !tables || !ctx) return error(PKV_ERR_DEVICE, 0, 0, "null device pointer");
    if (reinterpret_cast<uintptr_t>(q) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
        return error(PKV_ERR_DEVICE, 0, 0, "query and output must be 16-byte aligned");
    if (!std::isfinite(softmax_scale) || !(softmax_scale > 0.0f))
        return error(PKV_ERR_DEVICE, 0, 0, "softmax scale must be finite and positive");
    const long long rows = (long long)(cfg_.num_layers * cfg_.num_blocks * cfg_.block_size);
    if (rows >= (1ll << 31)) return error(PKV_ERR_DEVICE, 0, 0, "pool too tall for paged attention");
    DeviceGuard g(device_);
    cudaError_t e;
    if (!tmaps_ready_) {
        if ((e = make_attention_tmaps(k_plane_, v_plane_, dtype_, (long long)shard_entry_, rows,
                                      (int)hd, tmaps_)) != cudaSuccess)
            return device_error("building the attention tensor maps", e);
        tmaps_ready_ = true;
    }
    AttnLaunch a{};
    a.q = q;
    a.q_seq_stride = q_seq_stride;
    a.out = out;
    a.lse = lse;
    a.tables = tables;
    a.table_stride = table_stride;
    a.ctx = ctx;
    a.num_seqs = (int)num_seqs;
    a.kv_heads = (int)kv;
    a.group = (int)group;
    a.q_len = (int)q_len;
    a.num_q_heads = (int)num_q_heads;
    a.layer_row0 = (int)(layer * (int64_t)(cfg_.num_blocks * cfg_.block_size));
    a.num_blocks = (int)cfg_.num_blocks;
    a.max_ctx = (int)max_ctx;
    a.num_splits = attention_splits((long long)num_seqs * kv, (int)max_ctx, sms_, &a.blocks_per_split,
                                    dtype_ == DType::FP8_E4M3);
    a.scale_log2 = softmax_scale * 1.4426950408889634f;
    if (dtype_ == DType::FP8_E4M3) {
        const long long stride = std::max<long long>((long long)(cfg_.num_layers * cfg_.num_kv_heads), 1);
        a.k_scale = d_inv_ + 2 * stride;
        a.v_scale = d_inv_ + 3 * stride;
        a.scale_row = layer * (long long)cfg_.num_kv_heads + (long long)(elem_offset() / hd);
    }
    a.err = d_err_;
    if (d_plan_ && plan_ctx_ == ctx && plan_seqs_ == num_seqs && plan_max_ctx_ == max_ctx) a.order = d_plan_;
    if (a.num_splits > 1) {
        const size_t parts = (size_t)num_seqs * q_len * num_q_heads * a.num_splits;
        const size_t need = parts * (hd + 1) * sizeof(float);
        if (need > d_attn_ws_bytes_) {
            // The old workspace may still be read by attention work in flight.
            if ((e = cudaDeviceSynchronize()) != cudaSuccess) return device_error("cudaDeviceSynchronize", e);
            const size_t want = std::max(need, d_attn_ws_bytes_ + d_attn_ws_bytes_ / 2);
            if (d_attn_ws_) cudaFree(d_attn_ws_);
            d_attn_ws_ = nullptr;
            d_attn_ws_bytes_ = 0;
            if ((e = cudaMalloc(&d_attn_ws_, want)) != cudaSuccess)
                return device_error("allocating the attention workspace", e);
            d_attn_ws_bytes_ = want;
        }
        a.part_o = d_attn_ws_;
        a.part_lse = d_attn_ws_ + parts * hd;
    }
    return check("paged_attention", launch_paged_attention(a, tmaps_, dtype_, query, (int)hd, st));
}

Status B200Backend::paged_attention_plan_dev(const int32_t *ctx, int64_t num_seqs, int64_t max_ctx,
                                             cudaStream_t st) {
    plan_ctx_ = nullptr;  // no plan unless this one is made
    if (num_seqs < 0 || num_seqs > 65535)
        return error(PKV_ERR_DEVICE, 0, 0, "at most 65535 sequences per call");
    if (max_ctx < 0 || max_ctx > std::numeric_limits<int32_t>::max() - 16)
        return error(PKV_ERR_SHAPE_MISMATCH, 0, max_ctx, "max_context_len out of range");
    if (num_seqs == 0) return Status::Ok();
    if (!ctx) return error(PKV_ERR_DEVICE, 0, 0, "null device pointer");
    DeviceGuard g(device_);
    cudaError_t e;
    if (!d_plan_ && (e = cudaMalloc(&d_plan_, 65536 * sizeof(unsigned))) != cudaSuccess) {
        d_plan_ = nullptr;
        return device_error("allocating the attention plan", e);
    }
    if ((e = launch_attention_plan(ctx, (int)num_seqs, (int)max_ctx, d_plan_, st)) != cudaSuccess)
        return check("paged_attention_plan", e);
    plan_ctx_ = ctx;
    plan_seqs_ = num_seqs;
    plan_max_ctx_ = max_ctx;
    return Status::Ok();
}

Status B200Backend::digest(uint64_t *k, uint64_t *v, cudaStream_t st) {
    DeviceGuard g(device_);
    cudaStream_t s = st;
    unsigned long long host[2] = {0, 0};
    cudaError_t e;
    if ((e = cudaMemsetAsync(d_digest_, 0, 2 * sizeof(unsigned long long), s)) != cudaSuccess)
        return device_error("digest", e);
    DigestLaunch a{};
    a.k_pool = k_plane_;
    a.v_pool = v_plane_;
    a.rows = (long long)(cfg_.num_layers * slots_per_layer());
    a.entry_elems = (long long)shard_entry_;
    a.full_entry = (long long)full_entry_elems();
    a.elem_offset = (long long)elem_offset();
    a.pool_dtype = dtype_;
    a.out = d_digest_;
    if ((e = launch_digest(a, sms_, s)) != cudaSuccess) return device_error("digest", e);
    if ((e = cudaMemcpyAsync(host, d_digest_, sizeof(host), cudaMemcpyDeviceToHost, s)) ||
        (e = cudaStreamSynchronize(s)))
        return device_error("digest", e);
    *k = host[0];
    *v = host[1];
    return Status::Ok();
}

Status B200Backend::digest_rows(int64_t layer, const void *k, const void *v, int64_t tok_stride,
                                int64_t layer_stride, const int64_t *slots, int64_t num_tokens,
                                DType src, uint64_t *kd, uint64_t *vd, cudaStream_t st) {
    if (layer < -1 || (layer >= 0 && (uint64_t)layer >= cfg_.num_layers))
        return error(PKV_ERR_INVALID_LAYER, layer, (int64_t)cfg_.num_layers,
                     msg_layer((uint64_t)layer, cfg_.num_layers));
    if (num_tokens < 0) return error(PKV_ERR_SHAPE_MISMATCH, 0, num_tokens, "negative token count");
    if (num_tokens > 0 && (!k || !v || !slots)) return error(PKV_ERR_DEVICE, 0, 0, "null device pointer");
    if (tok_stride <= 0) tok_stride = (int64_t)shard_entry_;
    const bool all = layer == -1;
    if (all && layer_stride <= 0) layer_stride = tok_stride * num_tokens;
    DeviceGuard g(device_);
    unsigned long long host[2] = {0, 0};
    cudaError_t e;
    if ((e = cudaMemsetAsync(d_digest_, 0, sizeof(host), st)) != cudaSuccess)
        return device_error("digest_rows", e);
    DigestRowsLaunch a{};
    a.k = k;
    a.v = v;
    a.src_token_stride = tok_stride;
    a.src_layer_stride = all ? layer_stride : 0;
    a.slots = reinterpret_cast<const long long *>(slots);
    a.num_tokens = num_tokens;
    a.num_layers = all ? (long long)cfg_.num_layers : 1;
    a.first_layer = all ? 0 : layer;
    a.slots_per_layer = (long long)slots_per_layer();
    a.entry_elems = (long long)shard_entry_;
    a.full_entry = (long long)full_entry_elems();
    a.elem_offset = (long long)elem_offset();
    a.src_dtype = src;
    a.pool_dtype = dtype_;
    a.out = d_digest_;
    a.fp8 = fp8_scales();
    if ((e = launch_digest_rows(a, sms_, st)) != cudaSuccess) return device_error("digest_rows", e);
    if ((e = cudaMemcpyAsync(host, d_digest_, sizeof(host), cudaMemcpyDeviceToHost, st)) ||
        (e = cudaStreamSynchronize(st)))
        return device_error("digest_rows", e);
    *kd = host[0];
    *vd = host[1];
    return Status::Ok();
}

Status B200Backend::sync() {
    DeviceGuard g(device_);
    return check("cudaStreamSynchronize", cudaStreamSynchronize(stream_));
}

Status B200Backend::take_device_error(int64_t *index) {
    DeviceGuard g(device_);
    DevError h{};
    cudaError_t e;
    if ((e = cudaDeviceSynchronize()) || (e = cudaMemcpy(&h, d_err_, sizeof(h), cudaMemcpyDeviceToHost)) ||
        (e = cudaMemset(d_err_, 0, sizeof(DevError))))
        return ::pkv::device_error("reading the device error word", e);
    if (index) *index = h.index;
    if (h.code == PKV_OK) return Status::Ok();
    return error(h.code, h.index, 0,
                 "device entry point met a bad index at " + std::to_string(h.index));
}

}  // namespace pkv
