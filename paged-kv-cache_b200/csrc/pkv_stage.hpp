// pkv_stage.hpp -- HostStager: uploads K/V rows from caller-owned host memory
// (pageable or pinned) through a ring of pinned chunks that host worker
// threads fill, so that the trait's host-buffer entry points
// (write_kv_batch with &[f32] slices, crates/paged-kv-core/src/backend.rs:55-74)
// keep the host link busy without the caller pinning anything.
//
// A chunk is filled by one worker (a copy, or f32 -> bf16 narrowing with
// round to nearest even, which halves the bytes that cross the link), then
// sent by cudaMemcpyAsync on the upload stream; the slot's event marks the
// end of that copy before the slot is filled again. Chunks are taken in
// order, so a worker waiting for its slot waits only on earlier chunks.
#pragma once

#include <cuda_runtime.h>

#include <condition_variable>
#include <cstdint>
#include <deque>
#include <mutex>
#include <thread>
#include <vector>

#include "pkv_internal.hpp"

namespace pkv {

// f32 -> bf16 bits, round to nearest even; NaN as the CUDA host conversion
// gives it (__float2bfloat16_rn).
void narrow_f32_to_bf16(uint16_t *dst, const float *src, uint64_t n);

class HostStager {
   public:
    // `chunk_bytes` (a multiple of 4 KiB) and `slots` size the pinned ring.
    HostStager(int device, cudaStream_t upload_stream, int threads, size_t chunk_bytes,
               int slots);
    ~HostStager();
    HostStager(const HostStager &) = delete;
    HostStager &operator=(const HostStager &) = delete;

    // Queues the upload of `elems` elements from host `src` (type `in`) to
    // device `dst` (type `out`: `in`, or BF16 when `in` is F32). Returns
    // once the chunks are queued; wait() returns once every queued chunk has
    // been read from `src` and its copy issued on the upload stream.
    cudaError_t begin(const void *src, DType in, void *dst, DType out, uint64_t elems);
    cudaError_t wait();

    int threads() const { return (int)workers_.size(); }

    static constexpr int kMaxSlots = 64;

   private:
    struct Job {
        const char *src;
        char *dst;
        uint64_t elems;
        DType in, out;
        int64_t seq;  // global chunk number; slot = seq % slots_
    };
    void run();
    cudaError_t ensure_ring();

    int device_;
    cudaStream_t stream_;
    size_t chunk_bytes_;    // staged bytes per chunk
    int slots_;
    char *ring_ = nullptr;  // slots_ x chunk_bytes_, pinned
    cudaEvent_t slot_free_[kMaxSlots] = {};
    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable cv_jobs_, cv_done_;
    std::deque<Job> jobs_;
    int64_t issued_[kMaxSlots];  // last chunk whose copy left slot i (issued)
    int64_t next_seq_ = 0;
    int64_t queued_ = 0, done_ = 0;
    cudaError_t err_ = cudaSuccess;
    bool stop_ = false;
};

}  // namespace pkv
