// pkv_bulk_copy.cu -- copy_blocks through the bulk-copy (TMA) engine.
//
// A block's plane for one layer is block_size*entry contiguous bytes (16 KiB
// at Qwen2-7B geometry), so a copy-on-write copy is a handful of large
// contiguous moves. Here one thread per CTA hands them to the SM's bulk-copy
// engine: cp.async.bulk global -> shared (completing on an mbarrier), then
// cp.async.bulk shared -> global, through a ring of kStages shared-memory
// buffers so that loads of later chunks overlap stores of earlier ones. Each
// CTA reads only for itself, with no tensor map: plain 1-D bulk copies of
// 16-byte-aligned runs.
//
// Same work and results as copy_blocks_kernel (pkv_kernels.cu); pairs with an
// id outside the pool are skipped and recorded, self-copies are skipped. Every
// wait on an mbarrier is bounded: past the budget the kernel records an error,
// drains its own stores and returns.

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "pkv_internal.hpp"

namespace pkv {
namespace {

#ifndef PKV_BULK_STAGES
#define PKV_BULK_STAGES 4
#endif
#ifndef PKV_BULK_CHUNK_MAX
#define PKV_BULK_CHUNK_MAX (32 * 1024)
#endif
#ifndef PKV_BULK_CTAS_PER_SM
#define PKV_BULK_CTAS_PER_SM 4
#endif
constexpr int kStages = PKV_BULK_STAGES;           // shared-memory buffers per CTA
constexpr long long kChunkMax = PKV_BULK_CHUNK_MAX;  // bytes per bulk copy, at most
constexpr int kCtasPerSm = PKV_BULK_CTAS_PER_SM;
constexpr int kInvalidBlock = 2;
constexpr int kDevice = 9;
constexpr long long kWaitBudgetCycles = 4000000000ll;  // about 2 s at 2 GHz

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record(DevError *e, int code, long long index) {
    if (atomicCAS(&e->code, 0, code) == 0) e->index = index;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the barrier's phase to complete, for at most kWaitBudgetCycles.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kWaitBudgetCycles) return false;
    return true;
}

__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gmem_src, uint32_t bytes,
                                          uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void bulk_store(void *gmem_dst, const void *smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
                 "r"(smem_u32(smem_src)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// All but the newest committed store group have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all_but_one() {
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

struct Item {
    const char *src;
    char *dst;
    bool live;
};

__global__ void __launch_bounds__(32)
copy_blocks_bulk_kernel(char *__restrict__ kp, char *__restrict__ vp, long long pool_layer,
                        long long block_bytes, int subs, int chunk_bytes,
                        const long long *__restrict__ pairs, long long num_pairs,
                        long long num_blocks, int num_layers, DevError *err) {
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ __align__(8) uint64_t bars[kStages];
    if (threadIdx.x != 0) return;  // one thread drives the copy engine

    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

    const long long items = num_pairs * num_layers * 2 * subs;
    const long long first = blockIdx.x, stride = gridDim.x;
    const long long mine = items > first ? (items - first + stride - 1) / stride : 0;

    // Item i of this CTA -> (pair, layer, plane, sub-chunk): source and destination.
    auto decode = [&](long long i) -> Item {
        long long x = first + i * stride;
        const int sub = (int)(x % subs);
        x /= subs;
        const int plane = (int)(x & 1);
        x >>= 1;
        const int layer = (int)(x % num_layers);
        const long long pair = x / num_layers;
        const long long s = __ldg(pairs + 2 * pair), d = __ldg(pairs + 2 * pair + 1);
        if (s < 0 || s >= num_blocks || d < 0 || d >= num_blocks) {
            if (sub == 0 && plane == 0 && layer == 0) record(err, kInvalidBlock, pair);
            return {nullptr, nullptr, false};
        }
        if (s == d) return {nullptr, nullptr, false};
        char *base = (plane ? vp : kp) + layer * pool_layer + (long long)sub * chunk_bytes;
        return {base + s * block_bytes, base + d * block_bytes, true};
    };

    Item stage[kStages];
    uint32_t phase[kStages];
    for (int s = 0; s < kStages; ++s) phase[s] = 0;
    auto issue = [&](long long i) {
        const int s = (int)(i % kStages);
        stage[s] = decode(i);
        if (stage[s].live) {
            mbar_expect_tx(&bars[s], (uint32_t)chunk_bytes);
            bulk_load(ring + (size_t)s * chunk_bytes, stage[s].src, (uint32_t)chunk_bytes, &bars[s]);
        }
    };

    for (long long i = 0; i < (mine < kStages ? mine : kStages); ++i) issue(i);
    for (long long n = 0; n < mine; ++n) {
        const int s = (int)(n % kStages);
        if (stage[s].live) {
            if (!mbar_wait_bounded(&bars[s], phase[s] & 1)) {
                // A load did not land within the budget: record it, give the
                // other loads still in flight the same bounded wait, let this
                // CTA's stores drain, and leave.
                record(err, kDevice, first + n * stride);
                const long long issued = n == 0 ? kStages : n - 1 + kStages;  // items < issued
                for (long long m = n + 1; m < issued && m < mine; ++m) {
                    const int t = (int)(m % kStages);
                    if (stage[t].live) mbar_wait_bounded(&bars[t], phase[t] & 1);
                }
                bulk_wait_all();
                return;
            }
            phase[s] ^= 1;
            // The load wrote this buffer through the async proxy; order that
            // before the store reads it.
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            bulk_store(stage[s].dst, ring + (size_t)s * chunk_bytes, (uint32_t)chunk_bytes);
        }
        bulk_commit();
        bulk_wait_read_all_but_one();  // the previous item's buffer is free again
        if (n >= 1 && n - 1 + kStages < mine) issue(n - 1 + kStages);
    }
    bulk_wait_all();
}

// zero_blocks on the same engine. Every CTA fills one chunk of shared
// memory with zeros, and lane 0 of each warp hands the engine bulk stores of
// that chunk over its share of the (block, layer, plane, sub-chunk) items:
// one instruction per up to 32 KiB, with no register data and no loads, so a
// few hundred issuing lanes keep the write path busy. Ids outside the pool
// are skipped and recorded. Only the stores' reads of the shared chunk are
// waited for (the hardware wait on this thread's bulk groups), so the CTA
// can exit; the writes themselves complete in stream order.
constexpr int kZeroWarps = 4;
constexpr int kZeroGroupsInFlight = 8;

__global__ void __launch_bounds__(kZeroWarps * 32)
zero_blocks_bulk_kernel(char *__restrict__ kp, char *__restrict__ vp, long long pool_layer,
                        long long block_bytes, int subs, int chunk_bytes,
                        const long long *__restrict__ ids, long long num_ids, long long num_blocks,
                        int num_layers, DevError *err) {
    extern __shared__ __align__(128) unsigned char zeros[];
    for (int i = threadIdx.x * 16; i < chunk_bytes; i += blockDim.x * 16)
        *reinterpret_cast<uint4 *>(zeros + i) = make_uint4(0, 0, 0, 0);
    // The zeros were written through the generic proxy; the bulk stores read
    // them through the async proxy.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if ((threadIdx.x & 31) != 0) return;

    const long long items = num_ids * num_layers * 2 * subs;
    const long long stride = (long long)gridDim.x * kZeroWarps;
    for (long long x0 = (long long)blockIdx.x * kZeroWarps + (threadIdx.x >> 5); x0 < items;
         x0 += stride) {
        long long x = x0;
        const int sub = (int)(x % subs);
        x /= subs;
        const int plane = (int)(x & 1);
        x >>= 1;
        const int layer = (int)(x % num_layers);
        const long long idx = x / num_layers;
        const long long blk = __ldg(ids + idx);
        if (blk < 0 || blk >= num_blocks) {
            if (sub == 0 && plane == 0 && layer == 0) record(err, kInvalidBlock, idx);
            continue;
        }
        bulk_store((plane ? vp : kp) + layer * pool_layer + blk * block_bytes +
                       (long long)sub * chunk_bytes,
                   zeros, (uint32_t)chunk_bytes);
        bulk_commit();
        asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kZeroGroupsInFlight) : "memory");
    }
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

}  // namespace

// Bytes moved per bulk copy: the block's plane, or the largest equal part of
// it up to 32 KiB that is a multiple of 16 bytes; 0 if there is none.
static long long bulk_chunk_bytes(long long block_bytes) {
    for (long long parts = 1; parts <= block_bytes / 16; ++parts) {
        if (block_bytes % parts) continue;
        const long long c = block_bytes / parts;
        if (c <= kChunkMax && c % 16 == 0) return c;
    }
    return 0;
}

bool bulk_copy_supported(const CopyLaunch &a) {
    return bulk_chunk_bytes(a.block_bytes) > 0 &&
           reinterpret_cast<uintptr_t>(a.k_pool) % 16 == 0 &&
           reinterpret_cast<uintptr_t>(a.v_pool) % 16 == 0;
}

cudaError_t launch_copy_blocks_bulk(const CopyLaunch &a, int sms, cudaStream_t st) {
    if (a.num_pairs <= 0 || a.num_layers <= 0 || a.block_bytes <= 0) return cudaSuccess;
    const long long chunk = bulk_chunk_bytes(a.block_bytes);
    if (chunk == 0) return cudaErrorInvalidValue;
    const int subs = (int)(a.block_bytes / chunk);
    const size_t smem = (size_t)kStages * (size_t)chunk;
    cudaError_t e = cudaFuncSetAttribute(copy_blocks_bulk_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const long long items = a.num_pairs * a.num_layers * 2 * subs;
    // As many CTAs as fit on the GPU at once (each holds kStages chunks of shared memory).
    const long long per_sm = std::max<long long>(
        1, std::min<long long>(kCtasPerSm, (227 * 1024) / (long long)(smem + 1024)));
    const long long grid = std::min<long long>(items, (long long)sms * per_sm);
    copy_blocks_bulk_kernel<<<(unsigned)grid, 32, smem, st>>>(
        static_cast<char *>(a.k_pool), static_cast<char *>(a.v_pool), a.num_blocks * a.block_bytes,
        a.block_bytes, subs, (int)chunk, a.pairs, a.num_pairs, a.num_blocks, (int)a.num_layers,
        a.err);
    return cudaGetLastError();
}

}  // namespace pkv

namespace pkv {

bool bulk_zero_supported(const ZeroLaunch &a) {
    return bulk_chunk_bytes(a.block_bytes) > 0 &&
           reinterpret_cast<uintptr_t>(a.k_pool) % 16 == 0 &&
           reinterpret_cast<uintptr_t>(a.v_pool) % 16 == 0;
}

cudaError_t launch_zero_blocks_bulk(const ZeroLaunch &a, int sms, cudaStream_t st) {
    if (a.num_ids <= 0 || a.num_layers <= 0 || a.block_bytes <= 0) return cudaSuccess;
    const long long chunk = bulk_chunk_bytes(a.block_bytes);
    if (chunk == 0) return cudaErrorInvalidValue;
    const int subs = (int)(a.block_bytes / chunk);
    if (chunk > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(zero_blocks_bulk_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)chunk);
        if (e != cudaSuccess) return e;
    }
    const long long items = a.num_ids * a.num_layers * 2 * subs;
    const long long warps = (long long)sms * 2 * kZeroWarps;  // two CTAs per SM
    const long long grid = std::max<long long>(1, (std::min(items, warps) + kZeroWarps - 1) / kZeroWarps);
    zero_blocks_bulk_kernel<<<(unsigned)grid, kZeroWarps * 32, (size_t)chunk, st>>>(
        static_cast<char *>(a.k_pool), static_cast<char *>(a.v_pool), a.num_blocks * a.block_bytes,
        a.block_bytes, subs, (int)chunk, a.blocks, a.num_ids, a.num_blocks, (int)a.num_layers, a.err);
    return cudaGetLastError();
}

}  // namespace pkv
