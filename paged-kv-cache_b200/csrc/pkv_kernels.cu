// pkv_kernels.cu -- sm_100a kernels of the paged KV cache data path.
//
// All four operations are pure data movement bounded by HBM bandwidth, so
// the kernels are built around wide (16-byte) coalesced loads and stores,
// several independent loads in flight per thread, streaming cache hints on
// data that is touched once, and 64-bit address arithmetic throughout (a
// 150 GB pool holds more than 2^31 elements per plane).
//
// Pool addressing is the reference's (crates/paged-kv-cuda/kernels/kernels.cu:11-14,
// crates/paged-kv-core/src/cpu.rs:45-53):
//   element (layer, block, slot, i) of a plane sits at
//   ((layer*num_blocks + block)*block_size + slot)*entry + i
// and, since block*block_size + slot is exactly the combined slot index s of
// slot_mapping, at (layer*slots_per_layer + s)*entry + i.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "pkv_device.cuh"
#include "pkv_internal.hpp"

namespace pkv {
namespace {

// ---- element conversion ---------------------------------------------------

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }

template <typename D>
__device__ __forceinline__ D from_f32(float f);
template <>
__device__ __forceinline__ float from_f32<float>(float f) { return f; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float f) { return __float2bfloat16_rn(f); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float f) { return __float2half_rn(f); }

// ---- reshape_and_cache: same element type, byte copy ------------------------
//
// Work item = (token, vector of V within the entry). A thread resolves its
// token's slot once and then moves its vector for every layer of its layer
// chunk (blockIdx.y), UNROLL layers' K and V loads in flight at a time.
// Consecutive threads cover consecutive vectors of one entry, so every warp
// reads and writes whole contiguous runs.

template <typename V, int UNROLL, int MIN_CTAS>
__global__ void __launch_bounds__(kThreads, MIN_CTAS)
reshape_copy_kernel(const char *__restrict__ k, const char *__restrict__ v, long long src_tok,
                    long long src_layer, char *__restrict__ kp, char *__restrict__ vp,
                    long long pool_layer, const long long *__restrict__ slots, long long num_tokens,
                    long long num_slots, int nvec, long long entry_bytes, int num_layers,
                    int layers_per_chunk, DevError *err) {
    const long long total = num_tokens * nvec;
    const int l0 = blockIdx.y * layers_per_chunk;
    const int l1 = min(num_layers, l0 + layers_per_chunk);
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long it = (long long)blockIdx.x * blockDim.x + threadIdx.x; it < total; it += stride) {
        const long long t = it / nvec;
        const int vec = (int)(it - t * nvec);
        const long long s = __ldg(slots + t);
        if (s < 0) continue;  // padding token
        if (s >= num_slots) {
            if (vec == 0 && blockIdx.y == 0) record_error(err, kInvalidBlock, t);
            continue;
        }
        const long long col = (long long)vec * sizeof(V);
        const char *ks = k + t * src_tok + l0 * src_layer + col;
        const char *vs = v + t * src_tok + l0 * src_layer + col;
        char *kd = kp + l0 * pool_layer + s * entry_bytes + col;
        char *vd = vp + l0 * pool_layer + s * entry_bytes + col;
        int l = l0;
        for (; l + UNROLL <= l1; l += UNROLL) {
            V kr[UNROLL], vr[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                kr[u] = __ldcs(reinterpret_cast<const V *>(ks + u * src_layer));
                vr[u] = __ldcs(reinterpret_cast<const V *>(vs + u * src_layer));
            }
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                __stcs(reinterpret_cast<V *>(kd + u * pool_layer), kr[u]);
                __stcs(reinterpret_cast<V *>(vd + u * pool_layer), vr[u]);
            }
            ks += UNROLL * src_layer;
            vs += UNROLL * src_layer;
            kd += UNROLL * pool_layer;
            vd += UNROLL * pool_layer;
        }
        for (; l < l1; ++l) {
            const V kr = __ldcs(reinterpret_cast<const V *>(ks));
            const V vr = __ldcs(reinterpret_cast<const V *>(vs));
            __stcs(reinterpret_cast<V *>(kd), kr);
            __stcs(reinterpret_cast<V *>(vd), vr);
            ks += src_layer;
            vs += src_layer;
            kd += pool_layer;
            vd += pool_layer;
        }
    }
}

// ---- reshape_and_cache with element conversion ------------------------------
//
// Work item = (token, group of PER elements). PER = 8 moves 16-byte vectors
// of 16-bit types (and pairs of them for f32); PER = 1 is the fallback for
// entries that are not a multiple of 8 elements or are misaligned.

template <int BYTES>
struct Raw {
    uint4 q[BYTES / 16];
};

template <typename S, typename D, int PER>
__global__ void __launch_bounds__(kThreads)
reshape_convert_kernel(const S *__restrict__ k, const S *__restrict__ v, long long src_tok,
                       long long src_layer, D *__restrict__ kp, D *__restrict__ vp,
                       long long pool_layer, const long long *__restrict__ slots,
                       long long num_tokens, long long num_slots, long long entry, int num_layers,
                       int layers_per_chunk, DevError *err) {
    const long long groups = entry / PER;
    const long long total = num_tokens * groups;
    const int l0 = blockIdx.y * layers_per_chunk;
    const int l1 = min(num_layers, l0 + layers_per_chunk);
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long it = (long long)blockIdx.x * blockDim.x + threadIdx.x; it < total; it += stride) {
        const long long t = it / groups;
        const long long g = it - t * groups;
        const long long s = __ldg(slots + t);
        if (s < 0) continue;
        if (s >= num_slots) {
            if (g == 0 && blockIdx.y == 0) record_error(err, kInvalidBlock, t);
            continue;
        }
        for (int l = l0; l < l1; ++l) {
            const long long so = t * src_tok + l * src_layer + g * PER;
            const long long dof = l * pool_layer + s * entry + g * PER;
            if constexpr (PER == 8) {
                Raw<8 * sizeof(S)> rk, rv;
#pragma unroll
                for (int q = 0; q < (int)(8 * sizeof(S) / 16); ++q) {
                    rk.q[q] = __ldcs(reinterpret_cast<const uint4 *>(k + so) + q);
                    rv.q[q] = __ldcs(reinterpret_cast<const uint4 *>(v + so) + q);
                }
                const S *ek = reinterpret_cast<const S *>(&rk);
                const S *ev = reinterpret_cast<const S *>(&rv);
                Raw<8 * sizeof(D)> wk, wv;
                D *ok = reinterpret_cast<D *>(&wk);
                D *ov = reinterpret_cast<D *>(&wv);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    ok[e] = from_f32<D>(to_f32(ek[e]));
                    ov[e] = from_f32<D>(to_f32(ev[e]));
                }
#pragma unroll
                for (int q = 0; q < (int)(8 * sizeof(D) / 16); ++q) {
                    __stcs(reinterpret_cast<uint4 *>(kp + dof) + q, wk.q[q]);
                    __stcs(reinterpret_cast<uint4 *>(vp + dof) + q, wv.q[q]);
                }
            } else {
                kp[dof] = from_f32<D>(to_f32(k[so]));
                vp[dof] = from_f32<D>(to_f32(v[so]));
            }
        }
    }
}

// ---- copy_blocks -------------------------------------------------------------
//
// One CTA per (pair, layer, plane, chunk of kThreads*UNROLL vectors); a
// block's plane for one layer is block_size*entry contiguous elements, so
// each CTA streams one contiguous run from src to dst.

template <typename V, int UNROLL>
__global__ void __launch_bounds__(kThreads)
copy_blocks_kernel(char *__restrict__ kp, char *__restrict__ vp, long long pool_layer,
                   long long block_bytes, const long long *__restrict__ pairs, long long num_blocks,
                   int num_layers, int chunks, DevError *err) {
    long long x = blockIdx.x;
    const int chunk = (int)(x % chunks);
    x /= chunks;
    const int plane = (int)(x & 1);
    x >>= 1;
    const int layer = (int)(x % num_layers);
    const long long pair = x / num_layers;
    const long long src = __ldg(pairs + 2 * pair);
    const long long dst = __ldg(pairs + 2 * pair + 1);
    if (src < 0 || src >= num_blocks || dst < 0 || dst >= num_blocks) {
        if (threadIdx.x == 0 && chunk == 0 && plane == 0 && layer == 0)
            record_error(err, kInvalidBlock, pair);
        return;
    }
    if (src == dst) return;
    char *base = (plane ? vp : kp) + layer * pool_layer;
    const V *s = reinterpret_cast<const V *>(base + src * block_bytes);
    V *d = reinterpret_cast<V *>(base + dst * block_bytes);
    const long long nvec = block_bytes / (long long)sizeof(V);
    const long long v0 = (long long)chunk * kThreads * UNROLL + threadIdx.x;
    V r[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
        const long long i = v0 + (long long)u * kThreads;
        if (i < nvec) r[u] = __ldcs(s + i);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
        const long long i = v0 + (long long)u * kThreads;
        if (i < nvec) __stcs(d + i, r[u]);
    }
}

// ---- zero_blocks -------------------------------------------------------------

template <typename V, int UNROLL>
__global__ void __launch_bounds__(kThreads)
zero_blocks_kernel(char *__restrict__ kp, char *__restrict__ vp, long long pool_layer,
                   long long block_bytes, const long long *__restrict__ ids, long long num_blocks,
                   int num_layers, int chunks, DevError *err) {
    long long x = blockIdx.x;
    const int chunk = (int)(x % chunks);
    x /= chunks;
    const int plane = (int)(x & 1);
    x >>= 1;
    const int layer = (int)(x % num_layers);
    const long long idx = x / num_layers;
    const long long blk = __ldg(ids + idx);
    if (blk < 0 || blk >= num_blocks) {
        if (threadIdx.x == 0 && chunk == 0 && plane == 0 && layer == 0)
            record_error(err, kInvalidBlock, idx);
        return;
    }
    V *d = reinterpret_cast<V *>((plane ? vp : kp) + layer * pool_layer + blk * block_bytes);
    const long long nvec = block_bytes / (long long)sizeof(V);
    const long long v0 = (long long)chunk * kThreads * UNROLL + threadIdx.x;
    V z;
    memset(&z, 0, sizeof(V));
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
        const long long i = v0 + (long long)u * kThreads;
        if (i < nvec) __stcs(d + i, z);
    }
}

// ---- copy_blocks + zero_blocks of one step, one launch ----------------------
//
// One CTA per (entry, layer, plane, chunk of kThreads * UNROLL vectors), as
// copy_blocks_kernel. Entries [0, num_srcs) are sources: the CTA loads its
// chunk of the source plane once, stores it to each of the source's
// destinations and then, if the step frees the source, stores zeros over it
// (the same thread loaded those addresses first, so the copy reads the old
// contents). Entries past num_srcs zero one freed block each. Bad ids are
// recorded (index: the position in dsts of the pair, or dst_off[num_srcs] +
// the position in zero_ids) and skipped.

template <typename V, int UNROLL>
__global__ void __launch_bounds__(kThreads)
copy_zero_kernel(char *__restrict__ kp, char *__restrict__ vp, long long pool_layer,
                 long long block_bytes, const CopyZeroLaunch a, int num_layers, int chunks) {
    long long x = blockIdx.x;
    const int chunk = (int)(x % chunks);
    x /= chunks;
    const int plane = (int)(x & 1);
    x >>= 1;
    const int layer = (int)(x % num_layers);
    const long long entry = x / num_layers;
    const bool report = threadIdx.x == 0 && chunk == 0 && plane == 0 && layer == 0;
    char *base = (plane ? vp : kp) + layer * pool_layer;
    const long long nvec = block_bytes / (long long)sizeof(V);
    const long long v0 = (long long)chunk * kThreads * UNROLL + threadIdx.x;
    V z;
    memset(&z, 0, sizeof(V));
    if (entry >= a.num_srcs) {
        const long long zi = entry - a.num_srcs;
        const long long blk = __ldg(a.zero_ids + zi);
        if (blk < 0 || blk >= a.num_blocks) {
            if (report) record_error(a.err, kInvalidBlock, __ldg(a.dst_off + a.num_srcs) + zi);
            return;
        }
        V *d = reinterpret_cast<V *>(base + blk * block_bytes);
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const long long i = v0 + (long long)u * kThreads;
            if (i < nvec) __stcs(d + i, z);
        }
        return;
    }
    const long long src = __ldg(a.srcs + entry);
    const long long d0 = __ldg(a.dst_off + entry), d1 = __ldg(a.dst_off + entry + 1);
    if (src < 0 || src >= a.num_blocks) {
        if (report) record_error(a.err, kInvalidBlock, d0);
        return;
    }
    V *s = reinterpret_cast<V *>(base + src * block_bytes);
    V r[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
        const long long i = v0 + (long long)u * kThreads;
        if (i < nvec) r[u] = __ldcs(s + i);
    }
    for (long long d = d0; d < d1; ++d) {
        const long long dst = __ldg(a.dsts + d);
        if (dst < 0 || dst >= a.num_blocks) {
            if (report) record_error(a.err, kInvalidBlock, d);
            continue;
        }
        if (dst == src) continue;
        V *o = reinterpret_cast<V *>(base + dst * block_bytes);
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const long long i = v0 + (long long)u * kThreads;
            if (i < nvec) __stcs(o + i, r[u]);
        }
    }
    if (__ldg(a.zero_src + entry)) {
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const long long i = v0 + (long long)u * kThreads;
            if (i < nvec) __stcs(s + i, z);
        }
    }
}

// ---- copy_blocks / zero_blocks over small block planes ---------------------
//
// A head-sharded pool has small block planes (2 KiB per plane and layer at
// 8 shards of Qwen2-7B's 512-element entry). One CTA per plane would move a
// few hundred bytes; instead `group` consecutive units (unit u = (pair or
// block index, layer, plane), u = (index * L + layer) * 2 + plane) share a
// CTA of kThreads * UNROLL vectors, consecutive threads on consecutive
// vectors of a unit. `shift` is log2(nvec) when nvec is a power of two.

struct UnitGroups {
    int nvec;   // vectors per unit (a block plane)
    int group;  // units per CTA
    int shift;  // log2(nvec) or -1
    int num_layers;
    unsigned num_units;  // < 2^31 (checked by the launcher)
};

// Unit, vector, index (pair or block id slot), layer and plane of this
// thread's u-th vector; false past the group or the last unit.
__device__ __forceinline__ bool group_unit(const UnitGroups &m, int u, int &vec, unsigned &idx,
                                           int &layer, int &plane) {
    const int local = u * kThreads + (int)threadIdx.x;
    const int du = m.shift >= 0 ? local >> m.shift : local / m.nvec;
    if (du >= m.group) return false;
    vec = local - du * m.nvec;
    const unsigned unit = blockIdx.x * (unsigned)m.group + (unsigned)du;
    if (unit >= m.num_units) return false;
    plane = (int)(unit & 1u);
    const unsigned lp = unit >> 1;
    idx = lp / (unsigned)m.num_layers;
    layer = (int)(lp - idx * (unsigned)m.num_layers);
    return true;
}

template <typename V, int UNROLL>
__global__ void __launch_bounds__(kThreads)
copy_blocks_grouped_kernel(char *__restrict__ kp, char *__restrict__ vp, long long pool_layer,
                           long long block_bytes, const long long *__restrict__ pairs,
                           long long num_blocks, UnitGroups m, DevError *err) {
    V r[UNROLL];
    V *dst_at[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
        dst_at[u] = nullptr;
        int vec, layer, plane;
        unsigned pair;
        if (!group_unit(m, u, vec, pair, layer, plane)) continue;
        const long long src = __ldg(pairs + 2 * (long long)pair);
        const long long dst = __ldg(pairs + 2 * (long long)pair + 1);
        if (src < 0 || src >= num_blocks || dst < 0 || dst >= num_blocks) {
            if (vec == 0 && plane == 0 && layer == 0) record_error(err, kInvalidBlock, pair);
            continue;
        }
        if (src == dst) continue;
        char *base = (plane ? vp : kp) + layer * pool_layer;
        r[u] = __ldcs(reinterpret_cast<const V *>(base + src * block_bytes) + vec);
        dst_at[u] = reinterpret_cast<V *>(base + dst * block_bytes) + vec;
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
        if (dst_at[u]) __stcs(dst_at[u], r[u]);
}

template <typename V, int UNROLL>
__global__ void __launch_bounds__(kThreads)
zero_blocks_grouped_kernel(char *__restrict__ kp, char *__restrict__ vp, long long pool_layer,
                           long long block_bytes, const long long *__restrict__ ids,
                           long long num_blocks, UnitGroups m, DevError *err) {
    V z;
    memset(&z, 0, sizeof(V));
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
        int vec, layer, plane;
        unsigned idx;
        if (!group_unit(m, u, vec, idx, layer, plane)) continue;
        const long long blk = __ldg(ids + idx);
        if (blk < 0 || blk >= num_blocks) {
            if (vec == 0 && plane == 0 && layer == 0) record_error(err, kInvalidBlock, idx);
            continue;
        }
        __stcs(reinterpret_cast<V *>((plane ? vp : kp) + layer * pool_layer + blk * block_bytes) + vec, z);
    }
}

// ---- slot resolution -----------------------------------------------------------
//
// Every CTA scans new_lens into shared memory (exclusive prefix, one
// contiguous segment per thread, then warp shuffles), so no CTA waits for
// another; CTA 0 also publishes cu_seqlens. Each token then finds its
// sequence by binary search over the prefix and applies
// BlockTable::slot_for_position (block_table.rs:97-101); the scan and the
// slot rule live in pkv_device.cuh.

__global__ void __launch_bounds__(kThreads)
resolve_slots_kernel(const int *__restrict__ tables, long long table_stride,
                     const int *__restrict__ ctx, const int *__restrict__ nnew, int num_seqs,
                     long long num_tokens, long long block_size, long long num_blocks,
                     int *__restrict__ cu_out, long long *__restrict__ slots, DevError *err) {
    extern __shared__ int s_cu[];  // num_seqs + 1
    __shared__ int s_warp[kThreads / 32];
    __shared__ int s_bad;
    const int tid = threadIdx.x;
    scan_lengths(ctx, nnew, num_seqs, s_cu, s_warp, &s_bad);

    const long long total = s_cu[num_seqs];
    if (blockIdx.x == 0) {
        for (int q = tid; q <= num_seqs; q += kThreads) cu_out[q] = s_cu[q];
        if (tid == 0) {
            if (s_bad) record_error(err, kShapeMismatch, -1);
            else if (total != num_tokens) record_error(err, kShapeMismatch, total);
        }
    }
    if (s_bad || total != num_tokens) return;

    const long long stride = (long long)gridDim.x * kThreads;
    for (long long t = (long long)blockIdx.x * kThreads + tid; t < num_tokens; t += stride)
        slots[t] = slot_of_token(t, s_cu, num_seqs, ctx, tables, table_stride, block_size,
                                 num_blocks, err, true);
}

// ---- slot resolution fused with reshape_and_cache ------------------------------
//
// One launch per step: every CTA scans new_lens, and each (token, vector)
// work item resolves its token's slot inline (no slot_mapping round trip
// through HBM) before moving its vector for every layer of its chunk, as
// reshape_copy_kernel does. The vector-0 threads of layer chunk 0 also
// publish the slot (when asked) so attention can use it.

// Moves item (t, vec)'s vector for layers [l0, l1) to slot s, UNROLL
// layers' K and V loads in flight at a time; the first `have` layers' rows
// are already in kr/vr.
template <typename V, int UNROLL>
__device__ __forceinline__ void move_item(const ResolveCacheLaunch &a, int nvec, int l0, int l1,
                                          long long t, int vec, long long s, V (&kr)[UNROLL],
                                          V (&vr)[UNROLL], int have) {
    const long long entry_bytes = (long long)nvec * sizeof(V);
    const long long pool_layer = a.slots_per_layer * entry_bytes;
    const long long src_tok = a.src_token_stride_bytes, src_layer = a.src_layer_stride_bytes;
    const long long col = (long long)vec * sizeof(V);
    const char *ks = static_cast<const char *>(a.k) + t * src_tok + l0 * src_layer + col;
    const char *vs = static_cast<const char *>(a.v) + t * src_tok + l0 * src_layer + col;
    char *kd = static_cast<char *>(a.k_pool) + (a.first_layer + l0) * pool_layer + s * entry_bytes + col;
    char *vd = static_cast<char *>(a.v_pool) + (a.first_layer + l0) * pool_layer + s * entry_bytes + col;
    int l = l0;
    if (have > 0) {
#pragma unroll
        for (int u = 0; u < UNROLL; ++u)
            if (u < have) {
                __stcs(reinterpret_cast<V *>(kd + u * pool_layer), kr[u]);
                __stcs(reinterpret_cast<V *>(vd + u * pool_layer), vr[u]);
            }
        ks += have * src_layer;
        vs += have * src_layer;
        kd += have * pool_layer;
        vd += have * pool_layer;
        l += have;
    }
    for (; l + UNROLL <= l1; l += UNROLL) {
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            kr[u] = __ldcs(reinterpret_cast<const V *>(ks + u * src_layer));
            vr[u] = __ldcs(reinterpret_cast<const V *>(vs + u * src_layer));
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            __stcs(reinterpret_cast<V *>(kd + u * pool_layer), kr[u]);
            __stcs(reinterpret_cast<V *>(vd + u * pool_layer), vr[u]);
        }
        ks += UNROLL * src_layer;
        vs += UNROLL * src_layer;
        kd += UNROLL * pool_layer;
        vd += UNROLL * pool_layer;
    }
    for (; l < l1; ++l) {
        const V k1 = __ldcs(reinterpret_cast<const V *>(ks));
        const V v1 = __ldcs(reinterpret_cast<const V *>(vs));
        __stcs(reinterpret_cast<V *>(kd), k1);
        __stcs(reinterpret_cast<V *>(vd), v1);
        ks += src_layer;
        vs += src_layer;
        kd += pool_layer;
        vd += pool_layer;
    }
}

// The general step: scan new_lens, then resolve and move every item of the
// grid-stride loop. Every thread of the CTA must call it.
template <typename V, int UNROLL>
__device__ __forceinline__ void resolve_cache_general(const ResolveCacheLaunch &a, int nvec,
                                                      int layers_per_chunk) {
    extern __shared__ int s_cu[];
    __shared__ int s_warp[kThreads / 32];
    __shared__ int s_bad;
    scan_lengths(a.ctx_lens, a.new_lens, (int)a.num_seqs, s_cu, s_warp, &s_bad);
    const long long total_tokens = s_cu[a.num_seqs];
    if (blockIdx.x == 0 && blockIdx.y == 0) {
        for (int q = threadIdx.x; q <= a.num_seqs; q += kThreads) a.cu_seqlens[q] = s_cu[q];
        if (threadIdx.x == 0) {
            if (s_bad) record_error(a.err, kShapeMismatch, -1);
            else if (total_tokens != a.num_tokens) record_error(a.err, kShapeMismatch, total_tokens);
        }
    }
    if (s_bad || total_tokens != a.num_tokens) return;

    const long long entry_bytes = (long long)nvec * sizeof(V);
    const long long pool_layer = a.slots_per_layer * entry_bytes;
    const int l0 = blockIdx.y * layers_per_chunk;
    const int l1 = min((int)a.num_layers, l0 + layers_per_chunk);
    const long long src_tok = a.src_token_stride_bytes, src_layer = a.src_layer_stride_bytes;
    const char *kbase = static_cast<const char *>(a.k);
    const char *vbase = static_cast<const char *>(a.v);
    char *kp = static_cast<char *>(a.k_pool) + a.first_layer * pool_layer;
    char *vp = static_cast<char *>(a.v_pool) + a.first_layer * pool_layer;
    const long long total = (a.num_tokens + a.num_direct) * nvec;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long it = (long long)blockIdx.x * blockDim.x + threadIdx.x; it < total; it += stride) {
        const long long t = it / nvec;
        const int vec = (int)(it - t * nvec);
        const bool lead = vec == 0 && blockIdx.y == 0;
        long long s;
        if (t < a.num_tokens) {
            s = slot_of_token(t, s_cu, (int)a.num_seqs, a.ctx_lens, a.tables, a.table_stride,
                              a.block_size, a.num_blocks, a.err, lead);
            if (lead && a.slots_out) a.slots_out[t] = s;
        } else {  // a host-known slot, as reshape_copy_kernel takes it
            s = __ldg(a.direct_slots + (t - a.num_tokens));
            if (s >= a.slots_per_layer) {
                if (lead) record_error(a.err, kInvalidBlock, t);
                continue;
            }
        }
        if (s < 0) continue;
        const long long col = (long long)vec * sizeof(V);
        const char *ks = kbase + t * src_tok + l0 * src_layer + col;
        const char *vs = vbase + t * src_tok + l0 * src_layer + col;
        char *kd = kp + l0 * pool_layer + s * entry_bytes + col;
        char *vd = vp + l0 * pool_layer + s * entry_bytes + col;
        int l = l0;
        for (; l + UNROLL <= l1; l += UNROLL) {
            V kr[UNROLL], vr[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                kr[u] = __ldcs(reinterpret_cast<const V *>(ks + u * src_layer));
                vr[u] = __ldcs(reinterpret_cast<const V *>(vs + u * src_layer));
            }
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                __stcs(reinterpret_cast<V *>(kd + u * pool_layer), kr[u]);
                __stcs(reinterpret_cast<V *>(vd + u * pool_layer), vr[u]);
            }
            ks += UNROLL * src_layer;
            vs += UNROLL * src_layer;
            kd += UNROLL * pool_layer;
            vd += UNROLL * pool_layer;
        }
        for (; l < l1; ++l) {
            const V kr = __ldcs(reinterpret_cast<const V *>(ks));
            const V vr = __ldcs(reinterpret_cast<const V *>(vs));
            __stcs(reinterpret_cast<V *>(kd), kr);
            __stcs(reinterpret_cast<V *>(vd), vr);
            ks += src_layer;
            vs += src_layer;
            kd += pool_layer;
            vd += pool_layer;
        }
    }
}

// The same, compiled on its own: the decode kernel's rarely taken fallback,
// so that its registers do not weigh on the decode path.
template <typename V, int UNROLL>
__device__ __noinline__ void resolve_cache_general_call(ResolveCacheLaunch a, int nvec,
                                                        int layers_per_chunk) {
    resolve_cache_general<V, UNROLL>(a, nvec, layers_per_chunk);
}

template <typename V, int UNROLL, int MIN_CTAS>
__global__ void __launch_bounds__(kThreads, MIN_CTAS)
resolve_cache_kernel(ResolveCacheLaunch a, int nvec, int layers_per_chunk) {
    pdl_wait();
    resolve_cache_general<V, UNROLL>(a, nvec, layers_per_chunk);
}

// A decode step (one new token per sequence, num_tokens == num_seqs, one
// work item per thread): token t is sequence t's token, at position
// ctx_lens[t], so no scan is needed. Each thread issues its context length
// and its rows' loads first, then the CTA checks with one barrier that every
// new_lens is 1 (and every context non-negative); only the block-table load
// and the stores remain after it. If the check fails, every CTA (they all
// read the same lengths) takes the general path instead.
template <typename V, int UNROLL>
__global__ void __launch_bounds__(kThreads, 4)
resolve_cache_decode_kernel(ResolveCacheLaunch a, int nvec, int layers_per_chunk) {
    pdl_wait();
    const long long it = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const bool active = it < a.num_tokens * nvec;
    const int l0 = blockIdx.y * layers_per_chunk;
    const int l1 = min((int)a.num_layers, l0 + layers_per_chunk);
    const int have = min(UNROLL, l1 - l0);
    long long t = 0;
    int vec = 0, pos = 0;
    V kr[UNROLL], vr[UNROLL];
    if (active) {
        t = it / nvec;
        vec = (int)(it - t * nvec);
        pos = __ldg(a.ctx_lens + t);
        const long long off = t * a.src_token_stride_bytes + l0 * a.src_layer_stride_bytes +
                              (long long)vec * sizeof(V);
#pragma unroll
        for (int u = 0; u < UNROLL; ++u)
            if (u < have) {
                kr[u] = __ldcs(reinterpret_cast<const V *>(static_cast<const char *>(a.k) + off +
                                                           u * a.src_layer_stride_bytes));
                vr[u] = __ldcs(reinterpret_cast<const V *>(static_cast<const char *>(a.v) + off +
                                                           u * a.src_layer_stride_bytes));
            }
    }
    int ok = 1;
    for (int q = threadIdx.x; q < a.num_seqs; q += kThreads)
        ok &= (__ldg(a.new_lens + q) == 1) & (__ldg(a.ctx_lens + q) >= 0);
    if (!__syncthreads_and(ok)) {
        resolve_cache_general_call<V, UNROLL>(a, nvec, layers_per_chunk);
        return;
    }
    if (blockIdx.x == 0 && blockIdx.y == 0)
        for (int q = threadIdx.x; q <= a.num_seqs; q += kThreads) a.cu_seqlens[q] = q;
    if (!active) return;
    // BlockTable::slot_for_position (block_table.rs:97-101) of position pos.
    const bool lead = vec == 0 && blockIdx.y == 0;
    const long long lb = pos / a.block_size;
    long long s = -1;
    if (lb >= a.table_stride) {
        if (lead) record_error(a.err, kSlotOutOfRange, t);
    } else {
        const long long blk = __ldg(a.tables + t * a.table_stride + lb);
        if (blk < 0 || blk >= a.num_blocks) {
            if (lead) record_error(a.err, kInvalidBlock, t);
        } else {
            s = blk * a.block_size + (pos - lb * a.block_size);
        }
    }
    if (lead && a.slots_out) a.slots_out[t] = s;
    if (s < 0) return;
    move_item<V, UNROLL>(a, nvec, l0, l1, t, vec, s, kr, vr, have);
}

// ---- digest --------------------------------------------------------------------
// splitmix64 finaliser over (global index, bits): mix64 in pkv_device.cuh.

__device__ __forceinline__ unsigned widen_bits(const float *p, long long i) { return __float_as_uint(p[i]); }
__device__ __forceinline__ unsigned widen_bits(const __nv_bfloat16 *p, long long i) {
    return (unsigned)(*reinterpret_cast<const unsigned short *>(p + i)) << 16;
}
__device__ __forceinline__ unsigned widen_bits(const __half *p, long long i) {
    return __float_as_uint(__half2float(p[i]));
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
digest_kernel(const T *__restrict__ kp, const T *__restrict__ vp, long long rows, long long entry,
              long long full_entry, long long elem_offset, unsigned long long *out) {
    const int plane = blockIdx.y;
    const T *p = plane ? vp : kp;
    const long long total = rows * entry;
    unsigned long long acc = 0;
    const long long stride = (long long)gridDim.x * kThreads;
    for (long long i = (long long)blockIdx.x * kThreads + threadIdx.x; i < total; i += stride) {
        const unsigned bits = widen_bits(p, i);
        if (bits == 0) continue;
        const long long r = i / entry;
        const long long gidx = r * full_entry + elem_offset + (i - r * entry);
        acc += mix64(((unsigned long long)gidx * 2 + plane) * 0x9E3779B97F4A7C15ull + bits);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0 && acc) atomicAdd(out + plane, acc);
}

// Digest that a pool would have after `num_layers` layers of rows were
// scattered through `slots` into it while it was empty: the same per-element
// hash, over the value as the pool would store it.
__device__ __forceinline__ unsigned widen_value(float x) { return __float_as_uint(x); }
__device__ __forceinline__ unsigned widen_value(__nv_bfloat16 x) {
    return (unsigned)(*reinterpret_cast<const unsigned short *>(&x)) << 16;
}
__device__ __forceinline__ unsigned widen_value(__half x) { return __float_as_uint(__half2float(x)); }

template <typename S, typename D>
__global__ void __launch_bounds__(kThreads)
digest_rows_kernel(const S *__restrict__ k, const S *__restrict__ v, long long tok_stride,
                   long long layer_stride, const long long *__restrict__ slots, long long num_tokens,
                   long long entry, long long num_layers, long long first_layer,
                   long long slots_per_layer, long long full_entry, long long elem_offset,
                   unsigned long long *out) {
    const int plane = blockIdx.y;
    const S *src = plane ? v : k;
    const long long total = num_layers * num_tokens * entry;
    unsigned long long acc = 0;
    const long long stride = (long long)gridDim.x * kThreads;
    for (long long i = (long long)blockIdx.x * kThreads + threadIdx.x; i < total; i += stride) {
        const long long r = i / entry;
        const long long e = i - r * entry;
        const long long l = r / num_tokens;
        const long long t = r - l * num_tokens;
        const long long s = __ldg(slots + t);
        if (s < 0 || s >= slots_per_layer) continue;
        const D d = from_f32<D>(to_f32(src[l * layer_stride + t * tok_stride + e]));
        const unsigned bits = widen_value(d);
        if (bits == 0) continue;
        const long long gidx = ((first_layer + l) * slots_per_layer + s) * full_entry + elem_offset + e;
        acc += mix64(((unsigned long long)gidx * 2 + plane) * 0x9E3779B97F4A7C15ull + bits);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0 && acc) atomicAdd(out + plane, acc);
}

// ---- helpers ---------------------------------------------------------------------


template <typename S, typename D>
cudaError_t launch_convert(const ReshapeLaunch &a, dim3 grid_chunks, int layers_per_chunk,
                           bool per8, int sms, cudaStream_t st) {
    const long long per = per8 ? 8 : 1;
    const long long total = a.num_tokens * (a.entry_elems / per);
    long long bx = std::min<long long>((total + kThreads - 1) / kThreads, (long long)sms * 64);
    dim3 grid((unsigned)std::max<long long>(bx, 1), grid_chunks.y);
    const long long pool_layer = a.slots_per_layer * a.entry_elems;
    D *kp = static_cast<D *>(a.k_pool) + a.first_layer * pool_layer;
    D *vp = static_cast<D *>(a.v_pool) + a.first_layer * pool_layer;
    if (per8)
        reshape_convert_kernel<S, D, 8><<<grid, kThreads, 0, st>>>(
            static_cast<const S *>(a.k), static_cast<const S *>(a.v), a.src_token_stride,
            a.src_layer_stride, kp, vp, pool_layer, a.slots, a.num_tokens, a.slots_per_layer,
            a.entry_elems, (int)a.num_layers, layers_per_chunk, a.err);
    else
        reshape_convert_kernel<S, D, 1><<<grid, kThreads, 0, st>>>(
            static_cast<const S *>(a.k), static_cast<const S *>(a.v), a.src_token_stride,
            a.src_layer_stride, kp, vp, pool_layer, a.slots, a.num_tokens, a.slots_per_layer,
            a.entry_elems, (int)a.num_layers, layers_per_chunk, a.err);
    return cudaGetLastError();
}

template <typename S>
cudaError_t launch_convert_from(const ReshapeLaunch &a, dim3 g, int lpc, bool per8, int sms,
                                cudaStream_t st) {
    switch (a.pool_dtype) {
        case DType::F32: return launch_convert<S, float>(a, g, lpc, per8, sms, st);
        case DType::BF16: return launch_convert<S, __nv_bfloat16>(a, g, lpc, per8, sms, st);
        case DType::F16: return launch_convert<S, __half>(a, g, lpc, per8, sms, st);
        default: return cudaErrorInvalidValue;
    }
}

template <typename V>
cudaError_t launch_copy_v(const ReshapeLaunch &a, long long entry_bytes, int layers_per_chunk,
                          int chunks_y, int sms, cudaStream_t st) {
    const int es = dtype_size(a.pool_dtype);
    const int nvec = (int)(entry_bytes / (long long)sizeof(V));
    const long long total = a.num_tokens * nvec;
    // Enough CTAs to cover every item once, up to a cap past which threads loop.
    long long bx = std::min<long long>((total + kThreads - 1) / kThreads, (long long)sms * 256);
    dim3 grid((unsigned)std::max<long long>(bx, 1), (unsigned)chunks_y);
    const long long pool_layer = a.slots_per_layer * entry_bytes;
    char *kp = static_cast<char *>(a.k_pool) + a.first_layer * pool_layer;
    char *vp = static_cast<char *>(a.v_pool) + a.first_layer * pool_layer;
    // Launches that move several layers per item and span more than one
    // wave run at 2 CTAs per SM with up to 128 registers a thread (100 used):
    // the all-layer scatter of a 65,536-token chunk reaches 1.007 of the copy
    // peak against 0.973 at 4 CTAs per SM. A per-layer call (the trait's
    // write_kv_batch) has one layer per item and keeps 4: measured end to end
    // from pinned host rows, where each layer's scatter overlaps the next
    // layer's upload, the 2-CTA form lost 1.3 % of the host link.
    const bool wide = (long long)grid.x * grid.y > (long long)sms * 4 && layers_per_chunk >= 4;
    auto kern = wide ? reshape_copy_kernel<V, 4, 2> : reshape_copy_kernel<V, 4, 4>;
    kern<<<grid, kThreads, 0, st>>>(
        static_cast<const char *>(a.k), static_cast<const char *>(a.v), a.src_token_stride * es,
        a.src_layer_stride * es, kp, vp, pool_layer, a.slots, a.num_tokens, a.slots_per_layer,
        nvec, entry_bytes, (int)a.num_layers, layers_per_chunk, a.err);
    return cudaGetLastError();
}


}  // namespace

int num_sms(int device) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
        n = 148;
    return n;
}

cudaError_t launch_reshape(const ReshapeLaunch &a, int sms, cudaStream_t st) {
    if (a.num_tokens <= 0 || a.num_layers <= 0 || a.entry_elems <= 0) return cudaSuccess;
    if (a.pool_dtype == DType::FP8_E4M3 && a.src_dtype != DType::FP8_E4M3)
        return launch_reshape_fp8(a, sms, st);  // quantising scatter (pkv_fp8.cu)
    if (a.src_dtype == DType::FP8_E4M3 && a.pool_dtype != DType::FP8_E4M3)
        return cudaErrorInvalidValue;  // E4M3 rows go only into E4M3 pools
    const int es = dtype_size(a.pool_dtype);
    const long long entry_bytes = a.entry_elems * es;
    const long long items = a.num_tokens * std::max<long long>(1, entry_bytes / 16);
    long long chunks;
    const int lpc = layers_per_chunk(items, a.num_layers, sms, &chunks);

    if (a.src_dtype == a.pool_dtype) {
        const int vb = pick_vector_bytes(
            es, {entry_bytes, a.src_token_stride * es, a.num_layers > 1 ? a.src_layer_stride * es : 0},
            {a.k, a.v});
        switch (vb) {
            case 16: return launch_copy_v<uint4>(a, entry_bytes, lpc, (int)chunks, sms, st);
            case 8: return launch_copy_v<uint2>(a, entry_bytes, lpc, (int)chunks, sms, st);
            case 4: return launch_copy_v<unsigned int>(a, entry_bytes, lpc, (int)chunks, sms, st);
            default: return launch_copy_v<unsigned short>(a, entry_bytes, lpc, (int)chunks, sms, st);
        }
    }
    const int ss = dtype_size(a.src_dtype);
    const bool per8 = a.entry_elems % 8 == 0 && a.src_token_stride % 8 == 0 &&
                      (a.num_layers == 1 || a.src_layer_stride % 8 == 0) && aligned(a.k, 16) &&
                      aligned(a.v, 16) && ss * 8 % 16 == 0;
    dim3 g(1, (unsigned)chunks);
    switch (a.src_dtype) {
        case DType::F32: return launch_convert_from<float>(a, g, lpc, per8, sms, st);
        case DType::BF16: return launch_convert_from<__nv_bfloat16>(a, g, lpc, per8, sms, st);
        case DType::F16: return launch_convert_from<__half>(a, g, lpc, per8, sms, st);
        default: return cudaErrorInvalidValue;
    }
}

namespace {
// Small block planes (at most half of a CTA's kThreads * U vectors) go to
// the grouped kernels; larger ones take one CTA per (unit, chunk).
template <typename V, int U>
bool small_planes(long long block_bytes, long long num_layers, long long units, UnitGroups &m,
                  long long &grid) {
    const long long nvec = block_bytes / (long long)sizeof(V);
    if (nvec * 2 > kThreads * U || units >= (1ll << 31)) return false;
    m.nvec = (int)nvec;
    m.group = (int)(kThreads * U / nvec);
    m.shift = (nvec & (nvec - 1)) == 0 ? __builtin_ctzll((unsigned long long)nvec) : -1;
    m.num_layers = (int)num_layers;
    m.num_units = (unsigned)units;
    grid = (units + m.group - 1) / m.group;
    return true;
}

template <typename V>
cudaError_t copy_v(const CopyLaunch &a, cudaStream_t st) {
    constexpr int U = 4;
    UnitGroups m;
    long long grid;
    if (small_planes<V, U>(a.block_bytes, a.num_layers, a.num_pairs * a.num_layers * 2, m, grid)) {
        copy_blocks_grouped_kernel<V, U><<<(unsigned)grid, kThreads, 0, st>>>(
            static_cast<char *>(a.k_pool), static_cast<char *>(a.v_pool),
            a.num_blocks * a.block_bytes, a.block_bytes, a.pairs, a.num_blocks, m, a.err);
        return cudaGetLastError();
    }
    const long long nvec = a.block_bytes / (long long)sizeof(V);
    const int chunks = (int)((nvec + kThreads * U - 1) / (kThreads * U));
    grid = a.num_pairs * a.num_layers * 2 * chunks;
    copy_blocks_kernel<V, U><<<(unsigned)grid, kThreads, 0, st>>>(
        static_cast<char *>(a.k_pool), static_cast<char *>(a.v_pool),
        a.num_blocks * a.block_bytes, a.block_bytes, a.pairs, a.num_blocks, (int)a.num_layers,
        chunks, a.err);
    return cudaGetLastError();
}
template <typename V>
cudaError_t zero_v(const ZeroLaunch &a, cudaStream_t st) {
    constexpr int U = 4;
    UnitGroups m;
    long long grid;
    if (small_planes<V, U>(a.block_bytes, a.num_layers, a.num_ids * a.num_layers * 2, m, grid)) {
        zero_blocks_grouped_kernel<V, U><<<(unsigned)grid, kThreads, 0, st>>>(
            static_cast<char *>(a.k_pool), static_cast<char *>(a.v_pool),
            a.num_blocks * a.block_bytes, a.block_bytes, a.blocks, a.num_blocks, m, a.err);
        return cudaGetLastError();
    }
    const long long nvec = a.block_bytes / (long long)sizeof(V);
    const int chunks = (int)((nvec + kThreads * U - 1) / (kThreads * U));
    grid = a.num_ids * a.num_layers * 2 * chunks;
    zero_blocks_kernel<V, U><<<(unsigned)grid, kThreads, 0, st>>>(
        static_cast<char *>(a.k_pool), static_cast<char *>(a.v_pool),
        a.num_blocks * a.block_bytes, a.block_bytes, a.blocks, a.num_blocks, (int)a.num_layers,
        chunks, a.err);
    return cudaGetLastError();
}
}  // namespace

cudaError_t launch_copy_zero(const CopyZeroLaunch &a, cudaStream_t st) {
    const long long entries = a.num_srcs + a.num_zero;
    if (entries <= 0 || a.num_layers <= 0 || a.block_bytes <= 0) return cudaSuccess;
    const int vb = pick_vector_bytes(2, {a.block_bytes}, {a.k_pool, a.v_pool});
    auto go = [&](auto vec) {
        using V = decltype(vec);
        constexpr int U = 4;
        const long long nvec = a.block_bytes / (long long)sizeof(V);
        const int chunks = (int)((nvec + kThreads * U - 1) / (kThreads * U));
        const long long grid = entries * a.num_layers * 2 * chunks;
        if (grid >= (1ll << 31)) return cudaErrorInvalidValue;
        copy_zero_kernel<V, U><<<(unsigned)grid, kThreads, 0, st>>>(
            static_cast<char *>(a.k_pool), static_cast<char *>(a.v_pool),
            a.num_blocks * a.block_bytes, a.block_bytes, a, (int)a.num_layers, chunks);
        return cudaGetLastError();
    };
    switch (vb) {
        case 16: return go(uint4{});
        case 8: return go(uint2{});
        case 4: return go(0u);
        default: return go((unsigned short)0);
    }
}

cudaError_t launch_copy_blocks(const CopyLaunch &a, cudaStream_t st) {
    if (a.num_pairs <= 0 || a.num_layers <= 0 || a.block_bytes <= 0) return cudaSuccess;
    const int vb = pick_vector_bytes(2, {a.block_bytes}, {a.k_pool, a.v_pool});
    switch (vb) {
        case 16: return copy_v<uint4>(a, st);
        case 8: return copy_v<uint2>(a, st);
        case 4: return copy_v<unsigned int>(a, st);
        default: return copy_v<unsigned short>(a, st);
    }
}

cudaError_t launch_zero_blocks(const ZeroLaunch &a, cudaStream_t st) {
    if (a.num_ids <= 0 || a.num_layers <= 0 || a.block_bytes <= 0) return cudaSuccess;
    const int vb = pick_vector_bytes(2, {a.block_bytes}, {a.k_pool, a.v_pool});
    switch (vb) {
        case 16: return zero_v<uint4>(a, st);
        case 8: return zero_v<uint2>(a, st);
        case 4: return zero_v<unsigned int>(a, st);
        default: return zero_v<unsigned short>(a, st);
    }
}

cudaError_t launch_resolve_slots(const ResolveLaunch &a, int sms, cudaStream_t st) {
    const size_t smem = (size_t)(a.num_seqs + 1) * sizeof(int);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(resolve_slots_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    long long bx = std::min<long long>((a.num_tokens + kThreads - 1) / kThreads, (long long)sms * 4);
    bx = std::max<long long>(bx, 1);
    resolve_slots_kernel<<<(unsigned)bx, kThreads, smem, st>>>(
        a.tables, a.table_stride, a.ctx_lens, a.new_lens, (int)a.num_seqs, a.num_tokens,
        a.block_size, a.num_blocks, a.cu_seqlens, a.slots, a.err);
    return cudaGetLastError();
}

cudaError_t launch_digest(const DigestLaunch &a, int sms, cudaStream_t st) {
    const long long total = a.rows * a.entry_elems;
    if (total <= 0) return cudaSuccess;
    if (a.pool_dtype == DType::FP8_E4M3) return launch_digest_fp8(a, sms, st);
    long long bx = std::min<long long>((total + kThreads - 1) / kThreads, (long long)sms * 16);
    dim3 grid((unsigned)std::max<long long>(bx, 1), 2);
    switch (a.pool_dtype) {
        case DType::F32:
            digest_kernel<float><<<grid, kThreads, 0, st>>>(
                static_cast<const float *>(a.k_pool), static_cast<const float *>(a.v_pool), a.rows,
                a.entry_elems, a.full_entry, a.elem_offset, a.out);
            break;
        case DType::BF16:
            digest_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(
                static_cast<const __nv_bfloat16 *>(a.k_pool),
                static_cast<const __nv_bfloat16 *>(a.v_pool), a.rows, a.entry_elems, a.full_entry,
                a.elem_offset, a.out);
            break;
        case DType::F16:
            digest_kernel<__half><<<grid, kThreads, 0, st>>>(
                static_cast<const __half *>(a.k_pool), static_cast<const __half *>(a.v_pool),
                a.rows, a.entry_elems, a.full_entry, a.elem_offset, a.out);
            break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

namespace {
template <typename S, typename D>
cudaError_t digest_rows_sd(const DigestRowsLaunch &a, int sms, cudaStream_t st) {
    const long long total = a.num_layers * a.num_tokens * a.entry_elems;
    long long bx = std::min<long long>((total + kThreads - 1) / kThreads, (long long)sms * 16);
    dim3 grid((unsigned)std::max<long long>(bx, 1), 2);
    digest_rows_kernel<S, D><<<grid, kThreads, 0, st>>>(
        static_cast<const S *>(a.k), static_cast<const S *>(a.v), a.src_token_stride,
        a.src_layer_stride, a.slots, a.num_tokens, a.entry_elems, a.num_layers, a.first_layer,
        a.slots_per_layer, a.full_entry, a.elem_offset, a.out);
    return cudaGetLastError();
}
template <typename S>
cudaError_t digest_rows_s(const DigestRowsLaunch &a, int sms, cudaStream_t st) {
    switch (a.pool_dtype) {
        case DType::F32: return digest_rows_sd<S, float>(a, sms, st);
        case DType::BF16: return digest_rows_sd<S, __nv_bfloat16>(a, sms, st);
        case DType::F16: return digest_rows_sd<S, __half>(a, sms, st);
        default: return cudaErrorInvalidValue;
    }
}
}  // namespace

cudaError_t launch_digest_rows(const DigestRowsLaunch &a, int sms, cudaStream_t st) {
    if (a.num_layers * a.num_tokens * a.entry_elems <= 0) return cudaSuccess;
    if (a.pool_dtype == DType::FP8_E4M3) return launch_digest_rows_fp8(a, sms, st);
    switch (a.src_dtype) {
        case DType::F32: return digest_rows_s<float>(a, sms, st);
        case DType::BF16: return digest_rows_s<__nv_bfloat16>(a, sms, st);
        case DType::F16: return digest_rows_s<__half>(a, sms, st);
        default: return cudaErrorInvalidValue;
    }
}

namespace {
template <typename V>
cudaError_t resolve_cache_v(const ResolveCacheLaunch &a, long long entry_bytes, int sms,
                            cudaStream_t st) {
    const int nvec = (int)(entry_bytes / (long long)sizeof(V));
    const long long items = (a.num_tokens + a.num_direct) * nvec;
    long long chunks;
    const int lpc = layers_per_chunk(items, a.num_layers, sms, &chunks);
    long long bx = std::min<long long>((items + kThreads - 1) / kThreads, (long long)sms * 256);
    dim3 grid((unsigned)std::max<long long>(bx, 1), (unsigned)chunks);
    // A launch that fits one wave at 4 CTAs per SM (a decode step) keeps
    // that residency. Larger ones (a prefill chunk) run at 2 CTAs per SM with
    // up to 128 registers a thread: fewer write streams in flight per SM.
    // Measured on B200 (65,536-token chunk, alternating builds): 1.004 of the
    // copy peak, against 0.989 at 3 CTAs per SM (80 registers) and 0.974 at 4
    // (64 registers); 2 layers in flight instead of 4 at 2 CTAs per SM: 0.927.
    const bool one_wave = (long long)grid.x * grid.y <= (long long)sms * 4;
    // One new token per sequence with every item in the first pass of the
    // grid: the decode form, which skips the scan when the lengths allow.
    const bool decode = a.num_tokens == a.num_seqs && a.num_direct == 0 &&
                        (long long)bx * kThreads >= items;
    auto kern = decode ? resolve_cache_decode_kernel<V, 4>
                : one_wave ? resolve_cache_kernel<V, 4, 4> : resolve_cache_kernel<V, 4, 2>;
    const size_t smem = (size_t)(a.num_seqs + 1) * sizeof(int);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(kern, grid, dim3(kThreads), smem, st, a, nvec, lpc);
}
}  // namespace

cudaError_t launch_resolve_cache(const ResolveCacheLaunch &a, int sms, cudaStream_t st) {
    const long long entry_bytes = a.entry_bytes;
    if (a.num_layers <= 0 || entry_bytes <= 0) return cudaSuccess;
    const int vb = pick_vector_bytes(2, {entry_bytes, a.src_token_stride_bytes,
                                         a.num_layers > 1 ? a.src_layer_stride_bytes : 0},
                                     {a.k, a.v});
    switch (vb) {
        case 16: return resolve_cache_v<uint4>(a, entry_bytes, sms, st);
        case 8: return resolve_cache_v<uint2>(a, entry_bytes, sms, st);
        case 4: return resolve_cache_v<unsigned int>(a, entry_bytes, sms, st);
        default: return resolve_cache_v<unsigned short>(a, entry_bytes, sms, st);
    }
}

}  // namespace pkv
