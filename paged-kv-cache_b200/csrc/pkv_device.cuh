// pkv_device.cuh -- device helpers shared by the kernel files: error
// recording, the block-wide scan of per-sequence lengths, the slot rule, and
// the launch-shape helpers of the scatter kernels.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <initializer_list>

#include "pkv_internal.hpp"

namespace pkv {

constexpr int kThreads = 256;

// pkv_status values recorded on the device.
constexpr int kInvalidBlock = 2;
constexpr int kSlotOutOfRange = 5;
constexpr int kShapeMismatch = 6;

__device__ __forceinline__ void record_error(DevError *e, int code, long long index) {
    if (atomicCAS(&e->code, 0, code) == 0) e->index = index;
}

// splitmix64 finaliser (Steele, Lea & Flood, 2014): the per-element hash of
// the plane digests, mix64(((index * 2 + plane) * golden) + f32 bits).
__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ unsigned long long elem_hash(long long gidx, int plane, unsigned bits) {
    return mix64(((unsigned long long)gidx * 2 + plane) * 0x9E3779B97F4A7C15ull + bits);
}

__device__ __forceinline__ int warp_inclusive_scan(int x) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    return x;
}

// Exclusive prefix of new_lens into s_cu[0..num_seqs] (one contiguous
// segment per thread, then warp shuffles); sets *s_bad when a length or a
// context is negative. Every thread of the CTA must call it.
__device__ __forceinline__ void scan_lengths(const int *__restrict__ ctx,
                                             const int *__restrict__ nnew, int num_seqs,
                                             int *s_cu, int *s_warp, int *s_bad) {
    const int tid = threadIdx.x;
    if (tid == 0) *s_bad = 0;
    __syncthreads();
    const int seg = (num_seqs + kThreads - 1) / kThreads;
    const int b0 = min(num_seqs, tid * seg);
    const int b1 = min(num_seqs, b0 + seg);
    int local = 0;
    for (int q = b0; q < b1; ++q) {
        const int n = __ldg(nnew + q);
        if (n < 0 || __ldg(ctx + q) < 0) *s_bad = 1;
        local += max(n, 0);
    }
    const int incl = warp_inclusive_scan(local);
    if ((tid & 31) == 31) s_warp[tid >> 5] = incl;
    __syncthreads();
    if (tid < 32) {
        const int w = tid < kThreads / 32 ? s_warp[tid] : 0;
        const int wi = warp_inclusive_scan(w);
        if (tid < kThreads / 32) s_warp[tid] = wi - w;
    }
    __syncthreads();
    int run = s_warp[tid >> 5] + incl - local;
    for (int q = b0; q < b1; ++q) {
        s_cu[q] = run;
        run += max(__ldg(nnew + q), 0);
    }
    if (b1 == num_seqs && b0 < b1) s_cu[num_seqs] = run;
    if (num_seqs == 0 && tid == 0) s_cu[0] = 0;
    __syncthreads();
}

// Programmatic dependent launch. A grid launched with programmatic stream
// serialization may be set up while the previous grid in its stream still
// runs; griddepcontrol.wait then holds it until that grid has completed and
// its writes are visible (a no-op for a grid launched the ordinary way), so
// stream order is kept and only the launch and set-up overlap. Called first,
// by every thread, before any global memory access. The kernels that use it
// release their dependents only by exiting: a release at entry let the next
// step's CTAs take SM slots while this step's still streamed, and the decode
// step got slower (bf16: 5.91 -> 5.98 us, against 5.64 us with the release at
// exit).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launches kern<<<grid, block, smem, st>>>(args...) with programmatic stream
// serialization (the kernel starts with pdl_enter()).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Combined slot of packed token t: its sequence by binary search over the
// prefix, then BlockTable::slot_for_position. -1 (and an error record when
// `report`) for a logical block past the table or a table entry outside the pool.
__device__ __forceinline__ long long slot_of_token(long long t, const int *s_cu, int num_seqs,
                                                   const int *__restrict__ ctx,
                                                   const int *__restrict__ tables,
                                                   long long table_stride, long long block_size,
                                                   long long num_blocks, DevError *err, bool report) {
    int lo = 0, hi = num_seqs - 1;
    while (lo < hi) {  // last q with s_cu[q] <= t; that sequence has new_lens > 0
        const int mid = (lo + hi + 1) >> 1;
        if (s_cu[mid] <= t) lo = mid;
        else hi = mid - 1;
    }
    const long long pos = (long long)__ldg(ctx + lo) + (t - s_cu[lo]);
    const long long lb = pos / block_size;
    const long long off = pos - lb * block_size;
    if (lb >= table_stride) {
        if (report) record_error(err, kSlotOutOfRange, t);
        return -1;
    }
    const long long blk = __ldg(tables + (long long)lo * table_stride + lb);
    if (blk < 0 || blk >= num_blocks) {
        if (report) record_error(err, kInvalidBlock, t);
        return -1;
    }
    return blk * block_size + off;
}

inline bool aligned(const void *p, long long a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Layers per grid.y chunk of a scatter launch. Layers are split only when
// the (token, vector) items alone cannot fill one wave of resident CTAs, and
// never below 4 layers per chunk, so every thread keeps 4 layers' K and V
// loads in flight and the per-CTA set-up is paid for over several layers.
inline int layers_per_chunk(long long items, long long num_layers, int sms, long long *chunks) {
    const long long wave = (long long)sms * 4 * kThreads;
    const long long needed = (wave + std::max<long long>(items, 1) - 1) / std::max<long long>(items, 1);
    const long long cap = std::max<long long>(1, (num_layers + 3) / 4);
    const long long c = std::min<long long>(std::max<long long>(needed, 1), cap);
    const int lpc = (int)((num_layers + c - 1) / c);
    *chunks = (num_layers + lpc - 1) / lpc;
    return lpc;
}

// Largest power-of-two vector width (<= 16 bytes) dividing every byte offset.
inline int pick_vector_bytes(long long elem_bytes, std::initializer_list<long long> byte_quantities,
                      std::initializer_list<const void *> ptrs) {
    int vb = 16;
    while (vb > elem_bytes) {
        bool ok = true;
        for (long long q : byte_quantities) ok = ok && (q % vb == 0);
        for (const void *p : ptrs) ok = ok && aligned(p, vb);
        if (ok) break;
        vb /= 2;
    }
    return vb;
}

}  // namespace pkv
