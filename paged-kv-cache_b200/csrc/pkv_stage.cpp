// pkv_stage.cpp -- HostStager (see pkv_stage.hpp).

#include "pkv_stage.hpp"

#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstring>

namespace pkv {

namespace {

// Round to nearest even on the bit pattern: adding 0x7fff plus the lowest
// kept bit carries into the kept half exactly when the dropped half is above
// one half ulp, or equal to it with an odd kept half. Finite values past the
// largest bf16 round to infinity, infinities stay, subnormals round like any
// other value (bf16 and f32 share the exponent range). Returns whether any
// element was a NaN, whose bits this does not give.
__attribute__((target_clones("avx512f", "avx2", "default")))
bool narrow_rne(uint16_t *__restrict dst, const float *__restrict src, uint64_t n) {
    uint32_t nan_seen = 0;
    for (uint64_t i = 0; i < n; ++i) {
        uint32_t u;
        std::memcpy(&u, src + i, 4);
        nan_seen |= (u & 0x7fffffffu) > 0x7f800000u;
        dst[i] = static_cast<uint16_t>((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
    }
    return nan_seen != 0;
}

}  // namespace

void narrow_f32_to_bf16(uint16_t *dst, const float *src, uint64_t n) {
    if (!narrow_rne(dst, src, n)) return;
    for (uint64_t i = 0; i < n; ++i)
        if (std::isnan(src[i])) {
            const __nv_bfloat16 b = __float2bfloat16_rn(src[i]);
            std::memcpy(dst + i, &b, 2);
        }
}

HostStager::HostStager(int device, cudaStream_t upload_stream, int threads, size_t chunk_bytes,
                       int slots)
    : device_(device),
      stream_(upload_stream),
      chunk_bytes_(std::max<size_t>(4096, chunk_bytes / 4096 * 4096)),
      slots_(std::max(2, std::min(slots, kMaxSlots))) {
    for (int s = 0; s < kMaxSlots; ++s) issued_[s] = -1;
    // Each worker holds at most one slot, and a slot waits only on the chunk
    // taken slots_ chunks before it: up to slots_ / 2 workers stream.
    threads = std::max(1, std::min(threads, slots_ / 2));
    for (int i = 0; i < threads; ++i) workers_.emplace_back([this] { run(); });
}

HostStager::~HostStager() {
    {
        std::lock_guard<std::mutex> lk(mu_);
        stop_ = true;
    }
    cv_jobs_.notify_all();
    cv_done_.notify_all();
    for (auto &t : workers_) t.join();
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device_);
    for (auto &e : slot_free_)
        if (e) {
            cudaEventSynchronize(e);
            cudaEventDestroy(e);
        }
    if (ring_) cudaFreeHost(ring_);
    cudaSetDevice(prev);
}

cudaError_t HostStager::ensure_ring() {
    if (ring_) return cudaSuccess;
    cudaError_t e;
    for (auto &ev : slot_free_)
        if (!ev && (e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming)) != cudaSuccess) return e;
    void *p = nullptr;
    if ((e = cudaMallocHost(&p, size_t(slots_) * chunk_bytes_)) != cudaSuccess) return e;
    ring_ = static_cast<char *>(p);
    return cudaSuccess;
}

cudaError_t HostStager::begin(const void *src, DType in, void *dst, DType out, uint64_t elems) {
    if (elems == 0) return cudaSuccess;
    if (!(in == out || (in == DType::F32 && out == DType::BF16))) return cudaErrorInvalidValue;
    const cudaError_t e = ensure_ring();
    if (e != cudaSuccess) return e;
    const uint64_t in_size = dtype_size(in), out_size = dtype_size(out);
    const uint64_t per = chunk_bytes_ / out_size;
    {
        std::lock_guard<std::mutex> lk(mu_);
        for (uint64_t off = 0; off < elems; off += per) {
            jobs_.push_back(Job{static_cast<const char *>(src) + off * in_size,
                                static_cast<char *>(dst) + off * out_size,
                                std::min(per, elems - off), in, out, next_seq_++});
            ++queued_;
        }
    }
    cv_jobs_.notify_all();
    return cudaSuccess;
}

cudaError_t HostStager::wait() {
    std::unique_lock<std::mutex> lk(mu_);
    cv_done_.wait(lk, [&] { return done_ == queued_; });
    const cudaError_t e = err_;
    err_ = cudaSuccess;
    return e;
}

void HostStager::run() {
    cudaSetDevice(device_);
    for (;;) {
        Job j;
        int s;
        {
            std::unique_lock<std::mutex> lk(mu_);
            cv_jobs_.wait(lk, [&] { return stop_ || !jobs_.empty(); });
            if (jobs_.empty()) return;  // stopping
            j = jobs_.front();
            jobs_.pop_front();
            s = int(j.seq % slots_);
            // The slot's previous chunk was taken before this one; wait until
            // its copy has been issued, so that the slot's event covers it.
            cv_done_.wait(lk, [&] { return issued_[s] >= j.seq - slots_; });
        }
        char *buf = ring_ + size_t(s) * chunk_bytes_;
        cudaError_t e = cudaEventSynchronize(slot_free_[s]);  // its copy has left the slot
        if (e == cudaSuccess) {
            if (j.in == j.out)
                std::memcpy(buf, j.src, j.elems * dtype_size(j.in));
            else
                narrow_f32_to_bf16(reinterpret_cast<uint16_t *>(buf),
                                   reinterpret_cast<const float *>(j.src), j.elems);
            e = cudaMemcpyAsync(j.dst, buf, j.elems * dtype_size(j.out), cudaMemcpyHostToDevice,
                                stream_);
        }
        if (e == cudaSuccess) e = cudaEventRecord(slot_free_[s], stream_);
        {
            std::lock_guard<std::mutex> lk(mu_);
            issued_[s] = j.seq;
            ++done_;
            if (e != cudaSuccess && err_ == cudaSuccess) err_ = e;
        }
        cv_done_.notify_all();
    }
}

}  // namespace pkv
