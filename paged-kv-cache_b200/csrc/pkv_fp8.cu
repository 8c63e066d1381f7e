// pkv_fp8.cu -- fp8 (E4M3) pools: quantising reshape_and_cache, the fused
// slot resolution + quantising scatter, and digests of E4M3 planes.
//
// The reference stores f32 only (crates/paged-kv-core/src/cpu.rs:22-25);
// crates/paged-kv-core/src/config.rs:19 leaves room for 1-byte elements.
// Here an fp8 pool keeps the reference's layout and addressing with 1-byte
// E4M3 elements. Element x of layer l, kv head h is stored as
//   E4M3(x * inv[l][h]),  inv = 1 / scale, the f32 reciprocal computed on the host,
// with the f32 product rounded to nearest even and the E4M3 conversion
// rounding to nearest even and saturating at +-448 (PTX cvt .satfinite).
// Reads multiply the widened code by the scale.
//
// Bytes per token-layer: 2 planes x entry x (source bytes + 1), e.g. 6 B per
// element pair for a bf16 source instead of 8 B for a bf16 pool: the same
// HBM-bound kernels move a third more tokens per second.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "pkv_device.cuh"
#include "pkv_internal.hpp"

namespace pkv {
namespace {

// E4M3 codes of two f32 values, `lo` in the low byte. The PTX conversion
// writes its first source operand to the upper byte.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
    unsigned short r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ uint32_t e4m3(float x) { return e4m3x2(x, 0.0f) & 0xffu; }

// f32 bits of an E4M3 code (exact): sign, exponent bias 7 -> 127, 3 mantissa
// bits; exponent 0 holds m * 2^-9; S.1111.111 is NaN.
__device__ __forceinline__ unsigned e4m3_f32_bits(unsigned q) {
    const unsigned sign = (q & 0x80u) << 24, e = (q >> 3) & 0xfu, m = q & 7u;
    if (e == 15 && m == 7) return sign | 0x7fc00000u;
    if (e == 0) return sign | __float_as_uint((float)m * (1.0f / 512.0f));
    return sign | ((e + 120u) << 23) | (m << 20);
}

__device__ __forceinline__ float src_f32(float x) { return x; }
__device__ __forceinline__ float src_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float src_f32(__half x) { return __half2float(x); }

__device__ __forceinline__ uint32_t word(const uint4 &v, int j) {
    return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

// The two 16-bit elements of a 32-bit word as f32 (exact widening).
__device__ __forceinline__ float lo_f32(uint32_t w, __nv_bfloat16 *) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f32(uint32_t w, __nv_bfloat16 *) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float lo_f32(uint32_t w, __half *) {
    return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
}
__device__ __forceinline__ float hi_f32(uint32_t w, __half *) {
    return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

// 16 source elements (16 * sizeof(S) bytes, 16-byte aligned) as raw words.
template <typename S>
struct Group16 {
    static constexpr int kWords = (int)(16 * sizeof(S) / 16);
    uint4 w[kWords];
    __device__ __forceinline__ void load(const char *p) {
#pragma unroll
        for (int q = 0; q < kWords; ++q) w[q] = __ldcs(reinterpret_cast<const uint4 *>(p) + q);
    }
    // E4M3 codes of the 16 elements times `inv`, in element order.
    __device__ __forceinline__ uint4 quantise(float inv) const {
        float f[16];
#pragma unroll
        for (int q = 0; q < kWords; ++q)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t x = word(w[q], j);
                if constexpr (sizeof(S) == 4) {
                    f[q * 4 + j] = __uint_as_float(x);
                } else {
                    f[q * 8 + 2 * j] = lo_f32(x, (S *)nullptr);
                    f[q * 8 + 2 * j + 1] = hi_f32(x, (S *)nullptr);
                }
            }
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            o[j] = e4m3x2(__fmul_rn(f[4 * j], inv), __fmul_rn(f[4 * j + 1], inv)) |
                   (e4m3x2(__fmul_rn(f[4 * j + 2], inv), __fmul_rn(f[4 * j + 3], inv)) << 16);
        return make_uint4(o[0], o[1], o[2], o[3]);
    }
};

// Moves one work item -- PER elements of one token's entry, starting at
// element `e0` -- for layers [l0, l1): loads UNROLL layers' K and V before
// storing them. Source pointers are byte addresses of layer l0's elements;
// pool pointers of layer l0's codes. `layer_base` is the absolute layer of
// l0 for the scale lookup.
template <typename S, int PER, int UNROLL>
__device__ __forceinline__ void quantise_layers(const char *ks, const char *vs, long long src_layer,
                                                uint8_t *kd, uint8_t *vd, long long pool_layer,
                                                int l0, int l1, long long layer_base, long long e0,
                                                const Fp8Scales &sc) {
    const long long head = (sc.elem_offset + e0) / sc.head_dim;
    const float *ki = sc.k_inv + (layer_base + l0) * sc.heads + head;
    const float *vi = sc.v_inv + (layer_base + l0) * sc.heads + head;
    int l = l0;
    if constexpr (PER == 16) {
        for (; l + UNROLL <= l1; l += UNROLL) {
            Group16<S> kg[UNROLL], vg[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                kg[u].load(ks + u * src_layer);
                vg[u].load(vs + u * src_layer);
            }
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                __stcs(reinterpret_cast<uint4 *>(kd + u * pool_layer), kg[u].quantise(__ldg(ki + u * sc.heads)));
                __stcs(reinterpret_cast<uint4 *>(vd + u * pool_layer), vg[u].quantise(__ldg(vi + u * sc.heads)));
            }
            ks += UNROLL * src_layer;
            vs += UNROLL * src_layer;
            kd += UNROLL * pool_layer;
            vd += UNROLL * pool_layer;
            ki += UNROLL * sc.heads;
            vi += UNROLL * sc.heads;
        }
        for (; l < l1; ++l) {
            Group16<S> kg, vg;
            kg.load(ks);
            vg.load(vs);
            __stcs(reinterpret_cast<uint4 *>(kd), kg.quantise(__ldg(ki)));
            __stcs(reinterpret_cast<uint4 *>(vd), vg.quantise(__ldg(vi)));
            ks += src_layer;
            vs += src_layer;
            kd += pool_layer;
            vd += pool_layer;
            ki += sc.heads;
            vi += sc.heads;
        }
    } else {
        for (; l < l1; ++l) {
            const float k = src_f32(*reinterpret_cast<const S *>(ks));
            const float v = src_f32(*reinterpret_cast<const S *>(vs));
            *kd = (uint8_t)e4m3(__fmul_rn(k, __ldg(ki)));
            *vd = (uint8_t)e4m3(__fmul_rn(v, __ldg(vi)));
            ks += src_layer;
            vs += src_layer;
            kd += pool_layer;
            vd += pool_layer;
            ki += sc.heads;
            vi += sc.heads;
        }
    }
}

// ---- reshape_and_cache into an fp8 pool ------------------------------------
//
// Work item = (token, group of PER elements): the token's slot is read once,
// then the group is quantised and stored for every layer of the chunk
// (blockIdx.y). Consecutive threads take consecutive groups of one entry.

template <typename S, int PER, int UNROLL>
__global__ void __launch_bounds__(kThreads)
reshape_fp8_kernel(const char *__restrict__ k, const char *__restrict__ v, long long src_tok,
                   long long src_layer, uint8_t *__restrict__ kp, uint8_t *__restrict__ vp,
                   long long pool_layer, const long long *__restrict__ slots, long long num_tokens,
                   long long num_slots, long long groups, long long entry, int num_layers,
                   int layers_per_chunk, long long first_layer, Fp8Scales sc, DevError *err) {
    const long long total = num_tokens * groups;
    const int l0 = blockIdx.y * layers_per_chunk;
    const int l1 = min(num_layers, l0 + layers_per_chunk);
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long it = (long long)blockIdx.x * blockDim.x + threadIdx.x; it < total; it += stride) {
        const long long t = it / groups;
        const long long g = it - t * groups;
        const long long s = __ldg(slots + t);
        if (s < 0) continue;  // padding token
        if (s >= num_slots) {
            if (g == 0 && blockIdx.y == 0) record_error(err, kInvalidBlock, t);
            continue;
        }
        const long long e0 = g * PER;
        quantise_layers<S, PER, UNROLL>(k + t * src_tok + l0 * src_layer + e0 * (long long)sizeof(S),
                                        v + t * src_tok + l0 * src_layer + e0 * (long long)sizeof(S),
                                        src_layer, kp + l0 * pool_layer + s * entry + e0,
                                        vp + l0 * pool_layer + s * entry + e0, pool_layer, l0, l1,
                                        first_layer, e0, sc);
    }
}

// ---- slot resolution fused with the quantising scatter ------------------------
//
// resolve_cache_kernel (pkv_kernels.cu) with E4M3 stores: every CTA scans
// new_lens, each (token, group) item resolves its slot on chip and quantises
// its group for every layer of its chunk.

template <typename S, int PER, int UNROLL>
__device__ __forceinline__ void resolve_cache_fp8_general(const ResolveCacheLaunch &a,
                                                          long long groups, int layers_per_chunk) {
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

    const long long entry = a.entry_elems;  // one byte per element
    const long long pool_layer = a.slots_per_layer * entry;
    const int l0 = blockIdx.y * layers_per_chunk;
    const int l1 = min((int)a.num_layers, l0 + layers_per_chunk);
    const long long src_tok = a.src_token_stride_bytes, src_layer = a.src_layer_stride_bytes;
    const char *kbase = static_cast<const char *>(a.k);
    const char *vbase = static_cast<const char *>(a.v);
    uint8_t *kp = static_cast<uint8_t *>(a.k_pool) + a.first_layer * pool_layer;
    uint8_t *vp = static_cast<uint8_t *>(a.v_pool) + a.first_layer * pool_layer;
    const long long total = a.num_tokens * groups;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long it = (long long)blockIdx.x * blockDim.x + threadIdx.x; it < total; it += stride) {
        const long long t = it / groups;
        const long long g = it - t * groups;
        const bool lead = g == 0 && blockIdx.y == 0;
        const long long s = slot_of_token(t, s_cu, (int)a.num_seqs, a.ctx_lens, a.tables,
                                          a.table_stride, a.block_size, a.num_blocks, a.err, lead);
        if (lead && a.slots_out) a.slots_out[t] = s;
        if (s < 0) continue;
        const long long e0 = g * PER;
        quantise_layers<S, PER, UNROLL>(
            kbase + t * src_tok + l0 * src_layer + e0 * (long long)sizeof(S),
            vbase + t * src_tok + l0 * src_layer + e0 * (long long)sizeof(S), src_layer,
            kp + l0 * pool_layer + s * entry + e0, vp + l0 * pool_layer + s * entry + e0, pool_layer,
            l0, l1, a.first_layer, e0, a.fp8);
    }
}

template <typename S, int PER, int UNROLL, int MIN_CTAS>
__global__ void __launch_bounds__(kThreads, MIN_CTAS)
resolve_cache_fp8_kernel(ResolveCacheLaunch a, long long groups, int layers_per_chunk) {
    pdl_wait();
    resolve_cache_fp8_general<S, PER, UNROLL>(a, groups, layers_per_chunk);
}

// The general form compiled on its own: the decode kernel's rarely taken
// fallback, so that its registers do not weigh on the decode path.
template <typename S, int UNROLL>
__device__ __noinline__ void resolve_cache_fp8_general_call(ResolveCacheLaunch a, long long groups,
                                                            int layers_per_chunk) {
    resolve_cache_fp8_general<S, 16, UNROLL>(a, groups, layers_per_chunk);
}

// Decode form (num_tokens == num_seqs, one 16-element group per thread), as
// resolve_cache_decode_kernel (pkv_kernels.cu): the context length and the
// first UNROLL layers' source groups are loaded before one barrier vote
// checks that every new_lens is 1 and every context non-negative; the
// general form runs otherwise.
template <typename S, int UNROLL>
__global__ void __launch_bounds__(kThreads, 4)
resolve_cache_fp8_decode_kernel(ResolveCacheLaunch a, long long groups, int layers_per_chunk) {
    pdl_wait();
    const long long it = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const bool active = it < a.num_tokens * groups;
    const int l0 = blockIdx.y * layers_per_chunk;
    const int l1 = min((int)a.num_layers, l0 + layers_per_chunk);
    const int have = min(UNROLL, l1 - l0);
    const long long src_tok = a.src_token_stride_bytes, src_layer = a.src_layer_stride_bytes;
    long long t = 0, e0 = 0;
    int pos = 0;
    Group16<S> kg[UNROLL], vg[UNROLL];
    if (active) {
        t = it / groups;
        e0 = (it - t * groups) * 16;
        pos = __ldg(a.ctx_lens + t);
        const long long off = t * src_tok + l0 * src_layer + e0 * (long long)sizeof(S);
#pragma unroll
        for (int u = 0; u < UNROLL; ++u)
            if (u < have) {
                kg[u].load(static_cast<const char *>(a.k) + off + u * src_layer);
                vg[u].load(static_cast<const char *>(a.v) + off + u * src_layer);
            }
    }
    int ok = 1;
    for (int q = threadIdx.x; q < a.num_seqs; q += kThreads)
        ok &= (__ldg(a.new_lens + q) == 1) & (__ldg(a.ctx_lens + q) >= 0);
    if (!__syncthreads_and(ok)) {
        resolve_cache_fp8_general_call<S, UNROLL>(a, groups, layers_per_chunk);
        return;
    }
    if (blockIdx.x == 0 && blockIdx.y == 0)
        for (int q = threadIdx.x; q <= a.num_seqs; q += kThreads) a.cu_seqlens[q] = q;
    if (!active) return;
    // BlockTable::slot_for_position (block_table.rs:97-101) of position pos.
    const bool lead = e0 == 0 && blockIdx.y == 0;
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
    const long long entry = a.entry_elems;  // one byte per element
    const long long pool_layer = a.slots_per_layer * entry;
    const Fp8Scales &sc = a.fp8;
    const long long head = (sc.elem_offset + e0) / sc.head_dim;
    const float *ki = sc.k_inv + (a.first_layer + l0) * sc.heads + head;
    const float *vi = sc.v_inv + (a.first_layer + l0) * sc.heads + head;
    uint8_t *kd = static_cast<uint8_t *>(a.k_pool) + (a.first_layer + l0) * pool_layer + s * entry + e0;
    uint8_t *vd = static_cast<uint8_t *>(a.v_pool) + (a.first_layer + l0) * pool_layer + s * entry + e0;
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
        if (u < have) {
            __stcs(reinterpret_cast<uint4 *>(kd + u * pool_layer), kg[u].quantise(__ldg(ki + u * sc.heads)));
            __stcs(reinterpret_cast<uint4 *>(vd + u * pool_layer), vg[u].quantise(__ldg(vi + u * sc.heads)));
        }
    if (l0 + have < l1) {
        const long long off = t * src_tok + (l0 + have) * src_layer + e0 * (long long)sizeof(S);
        quantise_layers<S, 16, UNROLL>(static_cast<const char *>(a.k) + off,
                                       static_cast<const char *>(a.v) + off, src_layer,
                                       kd + have * pool_layer, vd + have * pool_layer, pool_layer,
                                       l0 + have, l1, a.first_layer, e0, sc);
    }
}

// ---- digests -------------------------------------------------------------------
// The plane digest of pkv_kernels.cu over widened E4M3 codes (unscaled), and
// the digest of rows as the quantising scatter would store them.

__global__ void __launch_bounds__(kThreads)
digest_fp8_kernel(const uint8_t *__restrict__ kp, const uint8_t *__restrict__ vp, long long rows,
                  long long entry, long long full_entry, long long elem_offset,
                  unsigned long long *out) {
    const int plane = blockIdx.y;
    const uint8_t *p = plane ? vp : kp;
    const long long total = rows * entry;
    unsigned long long acc = 0;
    const long long stride = (long long)gridDim.x * kThreads;
    for (long long i = (long long)blockIdx.x * kThreads + threadIdx.x; i < total; i += stride) {
        const unsigned bits = e4m3_f32_bits(p[i]);
        if (bits == 0) continue;
        const long long r = i / entry;
        acc += elem_hash(r * full_entry + elem_offset + (i - r * entry), plane, bits);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0 && acc) atomicAdd(out + plane, acc);
}

template <typename S>
__global__ void __launch_bounds__(kThreads)
digest_rows_fp8_kernel(const S *__restrict__ k, const S *__restrict__ v, long long tok_stride,
                       long long layer_stride, const long long *__restrict__ slots,
                       long long num_tokens, long long entry, long long num_layers,
                       long long first_layer, long long slots_per_layer, long long full_entry,
                       Fp8Scales sc, unsigned long long *out) {
    const int plane = blockIdx.y;
    const S *src = plane ? v : k;
    const float *inv = plane ? sc.v_inv : sc.k_inv;
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
        unsigned bits;
        if constexpr (sizeof(S) == 1) {  // rows that already hold E4M3 codes
            bits = e4m3_f32_bits(src[l * layer_stride + t * tok_stride + e]);
        } else {
            const long long head = (sc.elem_offset + e) / sc.head_dim;
            const float x = src_f32(src[l * layer_stride + t * tok_stride + e]);
            bits = e4m3_f32_bits(e4m3(__fmul_rn(x, __ldg(inv + (first_layer + l) * sc.heads + head))));
        }
        if (bits == 0) continue;
        const long long gidx = ((first_layer + l) * slots_per_layer + s) * full_entry + sc.elem_offset + e;
        acc += elem_hash(gidx, plane, bits);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0 && acc) atomicAdd(out + plane, acc);
}

// ---- launchers -------------------------------------------------------------------

// Whether 16-element groups apply: whole groups per entry and per head, and
// 16-byte aligned source rows.
bool groups_of_16(long long entry, const Fp8Scales &sc, long long src_elem_bytes,
                  std::initializer_list<long long> src_byte_strides,
                  std::initializer_list<const void *> ptrs) {
    if (entry % 16 || sc.head_dim % 16 || sc.elem_offset % 16) return false;
    for (long long q : src_byte_strides)
        if (q % 16) return false;
    for (const void *p : ptrs)
        if (!aligned(p, 16)) return false;
    return src_elem_bytes * 16 % 16 == 0;
}

// Layers per thread kept in flight: about 128 bytes of K and V loads.
template <typename S>
constexpr int unroll_for() { return sizeof(S) == 4 ? 1 : 2; }

template <typename S>
cudaError_t reshape_fp8_s(const ReshapeLaunch &a, int sms, cudaStream_t st) {
    const long long ss = (long long)sizeof(S);
    const long long entry = a.entry_elems;
    const bool g16 = groups_of_16(entry, a.fp8, ss,
                                  {a.src_token_stride * ss, a.num_layers > 1 ? a.src_layer_stride * ss : 0},
                                  {a.k, a.v, a.k_pool, a.v_pool});
    const long long per = g16 ? 16 : 1;
    const long long groups = entry / per;
    const long long items = a.num_tokens * groups;
    long long chunks;
    const int lpc = layers_per_chunk(items, a.num_layers, sms, &chunks);
    const long long bx = std::min<long long>((items + kThreads - 1) / kThreads, (long long)sms * 256);
    dim3 grid((unsigned)std::max<long long>(bx, 1), (unsigned)chunks);
    const long long pool_layer = a.slots_per_layer * entry;
    uint8_t *kp = static_cast<uint8_t *>(a.k_pool) + a.first_layer * pool_layer;
    uint8_t *vp = static_cast<uint8_t *>(a.v_pool) + a.first_layer * pool_layer;
    const char *k = static_cast<const char *>(a.k), *v = static_cast<const char *>(a.v);
    if (g16)
        reshape_fp8_kernel<S, 16, unroll_for<S>()><<<grid, kThreads, 0, st>>>(
            k, v, a.src_token_stride * ss, a.src_layer_stride * ss, kp, vp, pool_layer, a.slots,
            a.num_tokens, a.slots_per_layer, groups, entry, (int)a.num_layers, lpc, a.first_layer,
            a.fp8, a.err);
    else
        reshape_fp8_kernel<S, 1, 1><<<grid, kThreads, 0, st>>>(
            k, v, a.src_token_stride * ss, a.src_layer_stride * ss, kp, vp, pool_layer, a.slots,
            a.num_tokens, a.slots_per_layer, groups, entry, (int)a.num_layers, lpc, a.first_layer,
            a.fp8, a.err);
    return cudaGetLastError();
}

template <typename S>
cudaError_t resolve_cache_fp8_s(const ResolveCacheLaunch &a, int sms, cudaStream_t st) {
    const long long entry = a.entry_elems;
    const bool g16 = groups_of_16(entry, a.fp8, (long long)sizeof(S),
                                  {a.src_token_stride_bytes, a.num_layers > 1 ? a.src_layer_stride_bytes : 0},
                                  {a.k, a.v, a.k_pool, a.v_pool});
    const long long groups = entry / (g16 ? 16 : 1);
    const long long items = a.num_tokens * groups;
    long long chunks;
    const int lpc = layers_per_chunk(items, a.num_layers, sms, &chunks);
    const long long bx = std::min<long long>((items + kThreads - 1) / kThreads, (long long)sms * 256);
    dim3 grid((unsigned)std::max<long long>(bx, 1), (unsigned)chunks);
    const size_t smem = (size_t)(a.num_seqs + 1) * sizeof(int);
    // As resolve_cache_kernel: one wave keeps 4 CTAs per SM, larger launches
    // run at 3 with more registers a thread.
    const bool one_wave = (long long)grid.x * grid.y <= (long long)sms * 4;
    // One new token per sequence, every item in the first pass: the decode form.
    const bool decode = g16 && a.num_tokens == a.num_seqs && (long long)bx * kThreads >= items;
    auto kern = decode ? resolve_cache_fp8_decode_kernel<S, unroll_for<S>()>
                : g16 ? (one_wave ? resolve_cache_fp8_kernel<S, 16, unroll_for<S>(), 4>
                                  : resolve_cache_fp8_kernel<S, 16, unroll_for<S>(), 3>)
                      : resolve_cache_fp8_kernel<S, 1, 1, 4>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(kern, grid, dim3(kThreads), smem, st, a, groups, lpc);
}

template <typename S>
cudaError_t digest_rows_fp8_s(const DigestRowsLaunch &a, int sms, cudaStream_t st) {
    const long long total = a.num_layers * a.num_tokens * a.entry_elems;
    long long bx = std::min<long long>((total + kThreads - 1) / kThreads, (long long)sms * 16);
    dim3 grid((unsigned)std::max<long long>(bx, 1), 2);
    digest_rows_fp8_kernel<S><<<grid, kThreads, 0, st>>>(
        static_cast<const S *>(a.k), static_cast<const S *>(a.v), a.src_token_stride,
        a.src_layer_stride, a.slots, a.num_tokens, a.entry_elems, a.num_layers, a.first_layer,
        a.slots_per_layer, a.full_entry, a.fp8, a.out);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_reshape_fp8(const ReshapeLaunch &a, int sms, cudaStream_t st) {
    if (a.num_tokens <= 0 || a.num_layers <= 0 || a.entry_elems <= 0) return cudaSuccess;
    if (a.pool_dtype != DType::FP8_E4M3 || a.fp8.head_dim <= 0) return cudaErrorInvalidValue;
    switch (a.src_dtype) {
        case DType::F32: return reshape_fp8_s<float>(a, sms, st);
        case DType::BF16: return reshape_fp8_s<__nv_bfloat16>(a, sms, st);
        case DType::F16: return reshape_fp8_s<__half>(a, sms, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_resolve_cache_fp8(const ResolveCacheLaunch &a, int sms, cudaStream_t st) {
    if (a.num_layers <= 0 || a.entry_elems <= 0) return cudaSuccess;
    if (a.pool_dtype != DType::FP8_E4M3 || a.fp8.head_dim <= 0) return cudaErrorInvalidValue;
    switch (a.src_dtype) {
        case DType::F32: return resolve_cache_fp8_s<float>(a, sms, st);
        case DType::BF16: return resolve_cache_fp8_s<__nv_bfloat16>(a, sms, st);
        case DType::F16: return resolve_cache_fp8_s<__half>(a, sms, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_digest_fp8(const DigestLaunch &a, int sms, cudaStream_t st) {
    const long long total = a.rows * a.entry_elems;
    if (total <= 0) return cudaSuccess;
    long long bx = std::min<long long>((total + kThreads - 1) / kThreads, (long long)sms * 16);
    dim3 grid((unsigned)std::max<long long>(bx, 1), 2);
    digest_fp8_kernel<<<grid, kThreads, 0, st>>>(
        static_cast<const uint8_t *>(a.k_pool), static_cast<const uint8_t *>(a.v_pool), a.rows,
        a.entry_elems, a.full_entry, a.elem_offset, a.out);
    return cudaGetLastError();
}

cudaError_t launch_digest_rows_fp8(const DigestRowsLaunch &a, int sms, cudaStream_t st) {
    if (a.num_layers * a.num_tokens * a.entry_elems <= 0) return cudaSuccess;
    switch (a.src_dtype) {
        case DType::F32: return digest_rows_fp8_s<float>(a, sms, st);
        case DType::BF16: return digest_rows_fp8_s<__nv_bfloat16>(a, sms, st);
        case DType::F16: return digest_rows_fp8_s<__half>(a, sms, st);
        case DType::FP8_E4M3: return digest_rows_fp8_s<uint8_t>(a, sms, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace pkv
