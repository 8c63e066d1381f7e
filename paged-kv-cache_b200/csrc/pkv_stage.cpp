// pkv_stage.cpp -- HostStager (see pkv_stage.hpp).

#include "pkv_stage.hpp"

#include <cuda_bf16.h>
#include <immintrin.h>

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

// The same rounding, 16 elements per step with AVX2, written to the pinned
// ring with streaming (non-temporal) stores: the ring is read next by the
// copy engine, not by this core, so its lines need not be fetched into the
// cache first. Fences before returning, so the copy that follows sees them.
__attribute__((target("avx2")))
bool narrow_rne_stream(uint16_t *dst, const float *src, uint64_t n) {
    uint64_t i = 0;
    uint32_t nan_seen = 0;
    auto one_elem = [&](uint64_t j) {
        uint32_t u;
        std::memcpy(&u, src + j, 4);
        nan_seen |= (u & 0x7fffffffu) > 0x7f800000u;
        dst[j] = static_cast<uint16_t>((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
    };
    while (i < n && (reinterpret_cast<uintptr_t>(dst + i) & 31)) one_elem(i++);
    const __m256i bias = _mm256_set1_epi32(0x7fff), one = _mm256_set1_epi32(1),
                  magnitude = _mm256_set1_epi32(0x7fffffff), inf = _mm256_set1_epi32(0x7f800000);
    __m256i nan_acc = _mm256_setzero_si256();
    for (; i + 16 <= n; i += 16) {
        __m256i a = _mm256_loadu_si256(reinterpret_cast<const __m256i *>(src + i));
        __m256i b = _mm256_loadu_si256(reinterpret_cast<const __m256i *>(src + i + 8));
        nan_acc = _mm256_or_si256(nan_acc, _mm256_cmpgt_epi32(_mm256_and_si256(a, magnitude), inf));
        nan_acc = _mm256_or_si256(nan_acc, _mm256_cmpgt_epi32(_mm256_and_si256(b, magnitude), inf));
        a = _mm256_srli_epi32(
            _mm256_add_epi32(_mm256_add_epi32(a, bias), _mm256_and_si256(_mm256_srli_epi32(a, 16), one)), 16);
        b = _mm256_srli_epi32(
            _mm256_add_epi32(_mm256_add_epi32(b, bias), _mm256_and_si256(_mm256_srli_epi32(b, 16), one)), 16);
        // packus interleaves the 128-bit halves: a0-3 b0-3 | a4-7 b4-7.
        const __m256i packed = _mm256_permute4x64_epi64(_mm256_packus_epi32(a, b), 0xD8);
        _mm256_stream_si256(reinterpret_cast<__m256i *>(dst + i), packed);
    }
    while (i < n) one_elem(i++);
    _mm_sfence();
    return nan_seen != 0 || !_mm256_testz_si256(nan_acc, nan_acc);
}

// memcpy with streaming stores (32-byte aligned destination runs).
__attribute__((target("avx2")))
void copy_stream(char *dst, const char *src, uint64_t bytes) {
    uint64_t i = 0;
    const uint64_t head = std::min<uint64_t>(bytes, (32 - (reinterpret_cast<uintptr_t>(dst) & 31)) & 31);
    std::memcpy(dst, src, head);
    i = head;
    for (; i + 64 <= bytes; i += 64) {
        const __m256i a = _mm256_loadu_si256(reinterpret_cast<const __m256i *>(src + i));
        const __m256i b = _mm256_loadu_si256(reinterpret_cast<const __m256i *>(src + i + 32));
        _mm256_stream_si256(reinterpret_cast<__m256i *>(dst + i), a);
        _mm256_stream_si256(reinterpret_cast<__m256i *>(dst + i + 32), b);
    }
    std::memcpy(dst + i, src + i, bytes - i);
    _mm_sfence();
}

const bool g_avx2 = __builtin_cpu_supports("avx2");

void fix_nans(uint16_t *dst, const float *src, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i)
        if (std::isnan(src[i])) {
            const __nv_bfloat16 b = __float2bfloat16_rn(src[i]);
            std::memcpy(dst + i, &b, 2);
        }
}

// Fill of one ring chunk: narrowing or a plain copy.
void fill_chunk(char *buf, const char *src, uint64_t elems, DType in, DType out) {
    if (in == out) {
        if (g_avx2) copy_stream(buf, src, elems * dtype_size(in));
        else std::memcpy(buf, src, elems * dtype_size(in));
        return;
    }
    auto *d = reinterpret_cast<uint16_t *>(buf);
    const auto *f = reinterpret_cast<const float *>(src);
    if (g_avx2 ? narrow_rne_stream(d, f, elems) : narrow_rne(d, f, elems)) fix_nans(d, f, elems);
}

}  // namespace

void narrow_f32_to_bf16(uint16_t *dst, const float *src, uint64_t n) {
    if (narrow_rne(dst, src, n)) fix_nans(dst, src, n);
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
            fill_chunk(buf, j.src, j.elems, j.in, j.out);
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
