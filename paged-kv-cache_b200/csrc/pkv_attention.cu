// pkv_attention.cu -- decode attention over the paged pool: the cache's
// consumer (the reference leaves `paged_attention` off its trait and lists it
// as the next kernel: crates/paged-kv-core/src/backend.rs:18-22, README.md
// roadmap).
//
// One new query token per sequence. For sequence s with ctx[s] cached tokens
// (the new token's K/V already written by reshape_and_cache) and query head
// qh of kv head h = qh / group:
//   out[s][qh] = softmax(scale * q[s][qh] . K[s][0..ctx)) . V[s][0..ctx)
// where token t of the sequence sits in pool block table[s][t / 16], slot
// t % 16, of layer `layer`.
//
// B200 mapping. The work is bounded by HBM (every cached K/V byte of the
// layer is read once); per token and kv head it is 2 x group x head_dim
// multiply-adds for QK and again for PV.
// - Grid (split, kv head, sequence). A split is up to `blocks_per_split`
//   pool blocks; a short sequence uses fewer splits. Each of the 4 warps of a
//   CTA takes every 4th block of the split.
// - Loads: each warp runs its own ring of 3 stages. A stage is one pool
//   block of one kv head, K then V (16 rows x head_dim), brought from the
//   pool by TMA tile copies (cp.async.bulk.tensor.2d) straight from the
//   block table's block id, 128-byte swizzled, completing on an mbarrier.
//   Waits are bounded.
// - Math: mma.sync m16n8k16 (bf16 or f16 in, f32 accumulate). The M rows
//   are the group's query heads (padded to 16), so one K/V tile serves the
//   whole group. Scores stay in registers; the online softmax rescales the
//   f32 output accumulators only when a row maximum rises; P is rounded to
//   the input type for the PV product (as flash attention does).
// - Warps are merged through shared memory; splits through a small
//   workspace and a combine kernel (skipped when one split suffices).

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <type_traits>

#include "pkv_device.cuh"
#include "pkv_internal.hpp"

namespace pkv {
namespace {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kMaxStages = 6;
// Pool blocks per split, at most: a CTA has a fixed cost (queries, barrier
// set-up, the first copies' round trip, the warp merge), so long splits pay
// best. Measured on the config-2 batch (bf16, one launch per layer, early
// form): 16 / 32 / 64 / 128 blocks gave 0.65 / 0.82 / 0.89 / 0.90 of peak;
// later, with the plan and 28 layers per step, 256 against 128 blocks gave
// 1.052 against 0.994 (bf16) and 0.962 against 0.811 (fp8, whose blocks are
// half the bytes); 512 for fp8 gave 0.949.
#ifndef PKV_ATTN_SPLIT_BLOCKS
#define PKV_ATTN_SPLIT_BLOCKS 256
#endif
#ifndef PKV_ATTN_SPLIT_BLOCKS_FP8
#define PKV_ATTN_SPLIT_BLOCKS_FP8 256
#endif
// Block ids a lane prefetches: splits of up to 128 * kIdsPerLane blocks.
constexpr int kIdsPerLane =
    ((PKV_ATTN_SPLIT_BLOCKS > PKV_ATTN_SPLIT_BLOCKS_FP8 ? PKV_ATTN_SPLIT_BLOCKS
                                                        : PKV_ATTN_SPLIT_BLOCKS_FP8) + 127) / 128;
constexpr int kTok = 16;                 // tokens per pool block
constexpr int kDeviceCode = 9;           // PKV_ERR_DEVICE
constexpr long long kAttnWaitCycles = 4000000000ll;  // about 2 s at 2 GHz

// Tile geometry. A tile is one pool block of one kv head: 16 rows of D
// elements, brought in as boxes of 16 rows x up to 128 bytes, swizzled in
// 16-byte chunks (128-byte rows: chunk c of row r at c ^ (r % 8); the 64-byte
// rows of a 64-dim fp8 head: c ^ ((r / 2) % 4)). fp8 tiles are half as big,
// so three stages a warp leave room for four CTAs per SM: the same bytes in
// flight as two CTAs of bf16 tiles, and 16 warps to hide the conversions.
template <int D, bool FP8, int STAGES>
struct AttnGeom {
    static constexpr int kElemBytes = FP8 ? 1 : 2;
    static constexpr int kRowBytes = D * kElemBytes;                       // one head's row
    static constexpr int kBoxRow = kRowBytes < 128 ? kRowBytes : 128;      // bytes per box row
    static constexpr int kBoxElems = kBoxRow / kElemBytes;
    static constexpr int kBoxes = kRowBytes / kBoxRow;                     // boxes per tile
    static constexpr int kBoxBytes = kTok * kBoxRow;
    static constexpr int kTileBytes = kBoxes * kBoxBytes;                  // 16 tokens x D elements
    static constexpr int kStages = STAGES;
    static constexpr int kStageBytes = 2 * kTileBytes;                     // K tile, then V tile
    static constexpr int kRingBytes = kStages * kStageBytes;
    static constexpr int kQPitch = (D + 8) * 2;               // padded: conflict-free ldmatrix
    static constexpr int kQBytes = 16 * kQPitch;
    static constexpr int kOBytes = kAttnWarps * 16 * D * 4;   // per-warp partial outputs
    static constexpr int kStatBytes = 2 * kAttnWarps * 16 * 4;
    static constexpr int kSmem = 1024 + kAttnWarps * kRingBytes + kQBytes;
    static_assert(kStages <= kMaxStages, "stage masks");
    static_assert(kOBytes + kStatBytes <= kAttnWarps * kRingBytes, "combine must fit the rings");

    // Byte offset of 16-byte chunk c of row r within a box.
    __device__ static constexpr int chunk_at(int r, int c) {
        return kBoxRow == 128 ? r * 128 + ((c ^ (r & 7)) << 4) : r * kBoxRow + ((c ^ ((r >> 1) & 3)) << 4);
    }
};

// Stages per warp and CTAs per SM of each form: the bytes in flight per SM
// stay 4 warps x 3 stages x 2 CTAs of bf16/f16 tiles, spread over as many
// CTAs as registers allow, so that one CTA's set-up and merge overlap the
// others' streaming.
template <int D, bool FP8>
__host__ __device__ constexpr int attn_stages(int nt) {
    return (D <= 128 && !FP8) ? 2 : 3;
}
template <int D, bool FP8>
__host__ __device__ constexpr int attn_min_ctas(int nt) {
    return D > 128 ? 2 : FP8 ? (nt == 1 ? 4 : 3) : 3;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
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

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kAttnWaitCycles) return false;
    return true;
}

// One box of a 2-D tensor map (x = element column, y = row) into shared memory.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// ldmatrix of four 8x8 b16 matrices from a shared-memory address.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// Transpose of an 8x8 b16 matrix held one row pair per lane (lane t: row
// t / 4, elements 2(t % 4), +1) into the same layout.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

// 2^x by the SFU (PTX ex2.approx.ftz; 2^-inf = +0). The weights it feeds
// are rounded to bf16/f16 before P.V, far coarser than its error.
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Four E4M3 codes (byte 0 first) as two f16 pairs: bytes 0, 1 -> lo (byte 0
// in the low half), bytes 2, 3 -> hi. Exact: every E4M3 value is an f16 value.
__device__ __forceinline__ uint32_t e4m3x2_lo_to_f16x2(uint32_t codes) {
    uint32_t y;
    asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, a;\n\t}"
        : "=r"(y) : "r"(codes));
    return y;
}
__device__ __forceinline__ uint32_t e4m3x2_hi_to_f16x2(uint32_t codes) {
    uint32_t y;
    asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, b;\n\t}"
        : "=r"(y) : "r"(codes));
    return y;
}
__device__ __forceinline__ void e4m3x4_to_f16x2x2(uint32_t codes, uint32_t &lo, uint32_t &hi) {
    lo = e4m3x2_lo_to_f16x2(codes);
    hi = e4m3x2_hi_to_f16x2(codes);
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);

template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&c)[4], const uint32_t (&a)[4],
                                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <>
__device__ __forceinline__ void mma16816<__half>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                                 uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two f32 values as a packed pair of T, `lo` in the low half.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_float(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_float<__half>(float x) { return __float2half_rn(x); }

// Sequence length as the kernels use it: out-of-range lengths (and, with
// several query tokens per sequence, a context shorter than the query
// tokens) are recorded once and treated as empty.
__device__ __forceinline__ int checked_ctx(const AttnLaunch &a, int seq, bool report) {
    const int ctx = __ldg(a.ctx + seq);
    if (ctx < 0 || ctx > a.max_ctx || (a.q_len > 1 && ctx < a.q_len)) {
        if (report) record_error(a.err, kShapeMismatch, seq);
        return 0;
    }
    return ctx;
}

// T: query and output type. FP8: the pool holds E4M3 codes with per-(layer,
// kv head) scales; the tiles are converted to f16 in registers and the math
// runs in f16 (queries too, scaled by a power of two into f16 range), with
// the K scale folded into the softmax scale and the V scale into the output.
// MQ: several query tokens per sequence (a.q_len > 1), causal among
// themselves; without it the kernel is the one-token decode form.
template <typename T, int D, int NT, bool FP8, bool MQ>
__global__ void __launch_bounds__(kAttnThreads, attn_min_ctas<D, FP8>(NT))
paged_attention_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                       const AttnLaunch a) {
    using G = AttnGeom<D, FP8, attn_stages<D, FP8>(NT)>;
    using C = std::conditional_t<FP8, __half, T>;  // tensor-core operand type
    constexpr int kStages = G::kStages;
    extern __shared__ unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bars[kAttnWarps][kStages];
    __shared__ int s_failed;
    __shared__ int s_qmax;  // fp8: max |q| of the group, as f32 bits
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char *qs = smem + kAttnWarps * G::kRingBytes;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, kvh = blockIdx.y;
    pdl_wait();  // launched as a programmatic dependent of the previous grid (a layer's combine)
    // With a plan, grid slot z (dispatched in z order) takes the sequence
    // the plan put there, the longest first.
    int seq = blockIdx.z;
    if (a.order) {
        seq = (int)__ldg(a.order + blockIdx.z);
        if (seq >= a.num_seqs) return;  // not a sequence (a plan made while the lengths changed)
    }
    const int ctx = checked_ctx(a, seq, threadIdx.x == 0 && split == 0 && kvh == 0);
    const int nblk = (ctx + kTok - 1) / kTok;
    const int b0 = split * a.blocks_per_split;
    const int b1 = min(nblk, b0 + a.blocks_per_split);
    // The combine kernel (launched as a programmatic dependent of this grid)
    // may be scheduled from here on; it waits for this grid's completion.
    // Without splits the next grid is another layer's attention, released
    // only as this grid's CTAs exit.
    if (a.num_splits > 1) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (split > 0 && b0 >= b1) return;  // beyond this sequence's splits: the combine skips it

    // Query tile: row r < cols is query token r / group (of the sequence's
    // q_len) and head kvh * group + r % group; other rows zero.
    const int cols = MQ ? a.q_len * a.group : a.group;
    const T *q = static_cast<const T *>(a.q) + (long long)seq * (MQ ? a.q_len : 1) * a.q_seq_stride +
                 (long long)kvh * a.group * D;
    auto q_row = [&](int r) {
        if constexpr (MQ) {
            const int i = r / a.group;
            return q + (long long)i * a.q_seq_stride + (long long)(r - i * a.group) * D;
        } else {
            return q + (long long)r * D;
        }
    };
    float c = a.scale_log2;
    float v_scale = 1.f;
    if constexpr (FP8) {
        // f16 holds every E4M3 code exactly; the queries are brought into
        // its range by 2^-e (e > 0 only when some |q| >= 2^14), and 2^e
        // joins the K scale in the softmax scale.
        if (threadIdx.x == 0) s_qmax = 0;
        __syncthreads();
        float mx = 0.f;
        for (int i = threadIdx.x; i < cols * (D / 8); i += kAttnThreads) {
            const int r = i / (D / 8), cc = i - r * (D / 8);
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(q_row(r)) + cc);
            const T *e = reinterpret_cast<const T *>(&v);
#pragma unroll
            for (int k = 0; k < 8; ++k) mx = fmaxf(mx, fabsf(to_float(e[k])));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) atomicMax(&s_qmax, __float_as_int(mx));  // non-negative: int order
        __syncthreads();
        const float qmax = __int_as_float(s_qmax);
        int ex = 0;
        if (qmax < INFINITY) frexpf(qmax, &ex);
        const int e = max(0, ex - 14);
        const float down = ldexpf(1.f, -e);
        c *= __ldg(a.k_scale + a.scale_row + kvh) * ldexpf(1.f, e);
        v_scale = __ldg(a.v_scale + a.scale_row + kvh);
        for (int i = threadIdx.x; i < 16 * (D / 8); i += kAttnThreads) {
            const int r = i / (D / 8), cc = i - r * (D / 8);
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r < cols) {
                const uint4 x = __ldg(reinterpret_cast<const uint4 *>(q_row(r)) + cc);
                const T *xe = reinterpret_cast<const T *>(&x);
                uint32_t *w = reinterpret_cast<uint32_t *>(&v);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    w[k] = pack2<__half>(to_float(xe[2 * k]) * down, to_float(xe[2 * k + 1]) * down);
            }
            *reinterpret_cast<uint4 *>(qs + r * G::kQPitch + cc * 16) = v;
        }
    } else {
        for (int i = threadIdx.x; i < 16 * (D / 8); i += kAttnThreads) {
            const int r = i / (D / 8), cc = i - r * (D / 8);
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r < cols) v = __ldg(reinterpret_cast<const uint4 *>(q_row(r)) + cc);
            *reinterpret_cast<uint4 *>(qs + r * G::kQPitch + cc * 16) = v;
        }
    }
    if (lane == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&bars[warp][s]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x == 0) s_failed = 0;
    __syncthreads();

    // Queries as the B operand of S^T = K . Q^T: for n-tile nt (query heads
    // 8nt..8nt+7) and k-step ks, qb = {Q[h][16ks + 2j..], Q[h][16ks + 8 + 2j..]}.
    // fp8 tiles order each k-step's 16 dims as the K fragments arrive
    // (below): logical k 2j, 2j+1 are dims 4j, 4j+1 and logical k 2j+8, 2j+9
    // are dims 4j+2, 4j+3, so qb = Q[h][16ks + 4j .. 16ks + 4j + 3].
    uint32_t qb[NT][D / 16][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        if constexpr (FP8) {
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
                const uint2 w = *reinterpret_cast<const uint2 *>(
                    qs + (nt * 8 + (lane >> 2)) * G::kQPitch + (ks * 16 + (lane & 3) * 4) * 2);
                qb[nt][ks][0] = w.x;
                qb[nt][ks][1] = w.y;
            }
        } else {
#pragma unroll
            for (int kp = 0; kp < D / 32; ++kp) {  // two k-steps per ldmatrix.x4
                uint32_t r[4];
                const int row = nt * 8 + (lane & 7);
                ldsm_x4(r, smem_u32(qs + row * G::kQPitch + (kp * 4 + (lane >> 3)) * 16));
                qb[nt][2 * kp][0] = r[0];
                qb[nt][2 * kp][1] = r[1];
                qb[nt][2 * kp + 1][0] = r[2];
                qb[nt][2 * kp + 1][1] = r[3];
            }
        }
    }

    unsigned char *ring = smem + warp * G::kRingBytes;
    const uint32_t ring_u32 = smem_u32(ring);
    const int first = b0 + warp;
    const int count = first < b1 ? (b1 - first + kAttnWarps - 1) / kAttnWarps : 0;
    const int *table = a.tables + (long long)seq * a.table_stride;

    // ldmatrix row addresses within a tile; the box is an immediate added
    // per step.
    //  bf16/f16: chunk 2*ks + c of row `tok` sits at box ks / 4, chunk
    //  ((2*ks) mod 8) ^ (c ^ (tok mod 8)), so four offsets per lane cover
    //  every k-step. K is the A operand of S^T (rows = tokens, k = dims):
    //  matrix m of an x4 load is (tokens 8(m&1).., dims of chunk 2ks + (m>>1)).
    //  V^T is the A operand of O^T (rows = dims, k = tokens), loaded
    //  transposed: matrix m is (tokens 8(m>>1).., dims of chunk 2mt + (m&1)).
    //  fp8: a 16-byte chunk is 16 dims of a token; one x4 load (as b16 pairs)
    //  covers chunks 2p, 2p+1: matrix m is (tokens 8(m&1).., chunk 2p + (m>>1)),
    //  the same addresses for K and (transposed) for V.
    constexpr int kOffs = FP8 ? (G::kBoxRow / 32 < 1 ? 1 : G::kBoxRow / 32) : 4;
    uint32_t koff[kOffs], voff[kOffs];
    if constexpr (FP8) {
        const int tok = (lane & 7) + (((lane >> 3) & 1) << 3), half = lane >> 4;
#pragma unroll
        for (int pp = 0; pp < kOffs; ++pp) {
            koff[pp] = G::chunk_at(tok, 2 * pp + half);
            voff[pp] = G::kTileBytes + koff[pp];
        }
    } else {
        const int kt = (((lane >> 3) & 1) << 3) + (lane & 7), kx = (lane >> 4) ^ (kt & 7);
        const int vt = ((lane >> 4) << 3) + (lane & 7), vx = ((lane >> 3) & 1) ^ (vt & 7);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            koff[kk] = kt * 128 + (((2 * kk) ^ kx) << 4);
            voff[kk] = G::kTileBytes + vt * 128 + (((2 * kk) ^ vx) << 4);
        }
    }

    // This warp's block ids, up to kIdsPerLane per lane (count <= 32 x
    // kIdsPerLane), read once so that no table load sits in the block loop.
    int my_blk[kIdsPerLane];
#pragma unroll
    for (int r = 0; r < kIdsPerLane; ++r)
        my_blk[r] = lane + 32 * r < count ? __ldg(table + first + kAttnWarps * (lane + 32 * r)) : -1;
    uint32_t live = 0;   // bit s: stage s holds a block in flight (block id inside the pool)
    uint32_t dirty = 0;  // bit s: stage s's V rows were zeroed by generic stores
    auto issue = [&](int i, int st) {  // st == i % kStages
        int mine = my_blk[0];
#pragma unroll
        for (int r = 1; r < kIdsPerLane; ++r)
            if ((i >> 5) == r) mine = my_blk[r];
        const int blk = __shfl_sync(0xffffffffu, mine, i & 31);
        if (blk < 0 || blk >= a.num_blocks) {
            if (lane == 0) record_error(a.err, kInvalidBlock, seq);
            live &= ~(1u << st);
            return;
        }
        live |= 1u << st;
        const bool fence = (dirty >> st) & 1u;
        dirty &= ~(1u << st);
        if (lane == 0) {
            unsigned char *buf = ring + st * G::kStageBytes;
            uint64_t *bar = &bars[warp][st];
            // The tail of a sequence zeroes V rows with generic stores; those
            // come before the async-proxy writes of the next copy into the
            // buffer. (Its ldmatrix reads have completed: their values fed
            // the mma that issued before this, and the warp synchronised.)
            if (fence) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_expect_tx(bar, (uint32_t)G::kStageBytes);
            const int y = a.layer_row0 + blk * kTok;
#pragma unroll
            for (int hf = 0; hf < G::kBoxes; ++hf) {
                tma_load_2d(buf + hf * G::kBoxBytes, &tk, kvh * D + hf * G::kBoxElems, y, bar);
                tma_load_2d(buf + G::kTileBytes + hf * G::kBoxBytes, &tv, kvh * D + hf * G::kBoxElems, y, bar);
            }
        }
    };

    // O^T accumulators: o[nt][mt] is the m16n8 tile (dims 16mt.., query heads
    // 8nt..); this lane holds dims 16mt + g (+8) of heads 8nt + 2j (+1), with
    // g = lane / 4, j = lane % 4 (fp8: dims 16mt + 2g (+1), the order the V
    // fragments arrive in). Reference points (base-2 units: a raw score
    // times c) and sums per query head: [nt][hc] is head 8nt + 2j + hc.
    float o[NT][D / 16][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.f;
    // With several query tokens the reference points start at -FLT_MAX
    // rather than -inf, so that a head whose scores are all masked in a block
    // (a query token before the block's first key) keeps finite arithmetic:
    // its weights are 2^-inf = 0. With one token every block holds a key of
    // every head.
    float mc[NT][2], l_run[NT][2];
    constexpr float kM0 = MQ ? -FLT_MAX : -INFINITY;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) mc[nt][0] = mc[nt][1] = kM0, l_run[nt][0] = l_run[nt][1] = 0.f;
    // Query token index of this lane's two columns per n-tile, 4 bits each
    // (q_len * group <= 16); padding columns take the last token's limit.
    uint32_t qcols = 0;
    if constexpr (MQ) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
                const int col = nt * 8 + (lane & 3) * 2 + hc;
                qcols |= (uint32_t)(col < cols ? col / a.group : a.q_len - 1) << (4 * (2 * nt + hc));
            }
    }
    uint32_t phase = 0;  // bit s: parity of stage s's next completion
    bool failed = false;

    int issued = 0;
#pragma unroll
    for (int i = 0; i < kStages; ++i)
        if (i < count) issue(issued++, i);

    // Block n of this warp sits in stage n % kStages; the loop is unrolled
    // by the stage count so that each stage's index, barrier, buffer and
    // phase bit are constants. Block n + kStages, issued after block n is
    // consumed, reuses block n's stage.
    auto consume = [&](const int n, const int st) {
        bool ready = false;
        if ((live >> st) & 1u) {
            uint64_t *bar = &bars[warp][st];
            const uint32_t par = (phase >> st) & 1u;
            ready = mbar_try_wait(bar, par) || mbar_wait_bounded(bar, par);
            phase ^= 1u << st;
            if (!ready && !failed) {
                failed = true;  // stop issuing; the loop still waits out the loads in flight
                if (lane == 0) {
                    record_error(a.err, kDeviceCode, seq);
                    s_failed = 1;
                }
            }
        }
        if (ready && !failed) {
            const uint32_t kb = ring_u32 + st * G::kStageBytes;
            const int kb0 = (first + kAttnWarps * n) * kTok;  // the block's first key
            const int valid = min(kTok, ctx - kb0);

            // S^T[token][head] for the block's 16 tokens, even and odd
            // k-steps in separate accumulators (shorter mma chains).
            float sc[NT][4], s2[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = s2[nt][0] = s2[nt][1] = s2[nt][2] = s2[nt][3] = 0.f;
            if constexpr (FP8) {
#pragma unroll
                for (int pp = 0; pp < D / 32; ++pp) {
                    // r0/r1: tokens g, g+8, dims 32pp + 4j..+3; r2/r3: the
                    // next 16 dims. Low code pair -> k 2j, 2j+1; high -> 2j+8, 2j+9.
                    uint32_t r[4];
                    ldsm_x4(r, kb + koff[pp % kOffs] + (pp / kOffs) * G::kBoxBytes);
                    uint32_t ae[4], ao[4];
                    e4m3x4_to_f16x2x2(r[0], ae[0], ae[2]);
                    e4m3x4_to_f16x2x2(r[1], ae[1], ae[3]);
                    e4m3x4_to_f16x2x2(r[2], ao[0], ao[2]);
                    e4m3x4_to_f16x2x2(r[3], ao[1], ao[3]);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        mma16816<C>(sc[nt], ae, qb[nt][2 * pp][0], qb[nt][2 * pp][1]);
                        mma16816<C>(s2[nt], ao, qb[nt][2 * pp + 1][0], qb[nt][2 * pp + 1][1]);
                    }
                }
            } else {
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    uint32_t r[4];
                    ldsm_x4(r, kb + koff[ks & 3] + (ks >> 2) * G::kBoxBytes);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
                        mma16816<C>((ks & 1) ? s2[nt] : sc[nt], r, qb[nt][ks][0], qb[nt][ks][1]);
                }
            }
            const int g = lane >> 2;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) sc[nt][e] += s2[nt][e];
            // Zeroes the V rows past the sequence's end (they may hold
            // anything, NaN included) so that their zero weights contribute
            // exactly 0.
            auto zero_tail = [&]() {
                unsigned char *vb = ring + st * G::kStageBytes + G::kTileBytes;
                constexpr int kChunks = G::kBoxRow / 16;  // per row and box
                for (int i = lane; i < (kTok - valid) * G::kBoxes * kChunks; i += 32) {
                    const int r = valid + i / (G::kBoxes * kChunks), cc = i % (G::kBoxes * kChunks);
                    *reinterpret_cast<uint4 *>(vb + (cc / kChunks) * G::kBoxBytes + r * G::kBoxRow +
                                               (cc % kChunks) * 16) = make_uint4(0, 0, 0, 0);
                }
                dirty |= 1u << st;
                __syncwarp();
            };
            if constexpr (MQ) {
                // Token i attends keys up to ctx - q_len + i; last0 is token
                // 0's limit relative to the block. Where some token's limit
                // falls inside the block, mask each column past its own.
                const int last0 = ctx - a.q_len - kb0;
                if (last0 < kTok - 1) {
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int hc = 0; hc < 2; ++hc) {
                            const int lim = last0 + (int)((qcols >> (4 * (2 * nt + hc))) & 15u);
                            if (g > lim) sc[nt][hc] = -INFINITY;
                            if (g + 8 > lim) sc[nt][2 + hc] = -INFINITY;
                        }
                    if (valid < kTok) zero_tail();
                }
            } else if (valid < kTok) {
                // The sequence ends inside this block: mask the tokens past
                // its end.
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    if (g >= valid) sc[nt][0] = sc[nt][1] = -INFINITY;
                    if (g + 8 >= valid) sc[nt][2] = sc[nt][3] = -INFINITY;
                }
                zero_tail();
            }
            // Online softmax per query head (a column of S^T, spread over the
            // 8 lanes with the same j) in base 2: p = 2^(s * c - m). The
            // reference point m moves only when some score of the head
            // exceeds it by more than 8 (2^8 in weight), so most blocks skip
            // the rescale, and each lane tests only its own scores: the
            // head's exact maximum (3 shuffles) is taken on the rare path
            // alone. Weights stay below 2^8, which f32 sums and bf16/f16
            // weights hold with the same relative precision as weights below 1.
            bool grew = false;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int hc = 0; hc < 2; ++hc)  // always on the first block (m = -inf)
                    grew |= fmaf(fmaxf(sc[nt][hc], sc[nt][2 + hc]), c, -mc[nt][hc]) > 8.0f;
            if (__any_sync(0xffffffffu, grew)) {
                // Move every head's reference point to its maximum: rescale
                // its sum and output by 2^(m_old - m_new).
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int hc = 0; hc < 2; ++hc) {
                        float mx = fmaxf(sc[nt][hc], sc[nt][2 + hc]);
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                        // Finite: one token's blocks all hold a key of the
                        // head; several tokens' mc starts at -FLT_MAX.
                        const float m_new = fmaxf(mc[nt][hc], mx * c);
                        const float corr = ex2(mc[nt][hc] - m_new);
                        l_run[nt][hc] *= corr;
#pragma unroll
                        for (int mt = 0; mt < D / 16; ++mt) {
                            o[nt][mt][hc] *= corr;
                            o[nt][mt][2 + hc] *= corr;
                        }
                        mc[nt][hc] = m_new;
                    }
            }
            // P^T as the B operand of O^T = V^T . P^T: pack this lane's
            // weights (tokens g, g+8 of heads 2j, 2j+1) and transpose each
            // 8x8 half in registers to (tokens 2j.., head g).
            uint32_t pb[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    sc[nt][e] = ex2(fmaf(sc[nt][e], c, -mc[nt][e & 1]));
                    l_run[nt][e & 1] += sc[nt][e];
                }
                pb[nt][0] = movmatrix_trans(pack2<C>(sc[nt][0], sc[nt][1]));
                pb[nt][1] = movmatrix_trans(pack2<C>(sc[nt][2], sc[nt][3]));
            }
            if constexpr (FP8) {
#pragma unroll
                for (int qq = 0; qq < D / 32; ++qq) {
                    // Transposed b16 pairs: lane (g, j) holds tokens 2j, 2j+1
                    // (+8 in r1/r3) at dims 2g, 2g+1 of chunk 2qq (r0/r1) and
                    // 2qq+1 (r2/r3). Regrouped by dim, each pair of tokens is
                    // one f16x2: row g of the m-tile is dim 2g, row g+8 is 2g+1.
                    uint32_t r[4];
                    ldsm_x4_trans(r, kb + voff[qq % kOffs] + (qq / kOffs) * G::kBoxBytes);
                    uint32_t va[4], vb2[4];
                    e4m3x4_to_f16x2x2(__byte_perm(r[0], 0, 0x3120), va[0], va[1]);
                    e4m3x4_to_f16x2x2(__byte_perm(r[1], 0, 0x3120), va[2], va[3]);
                    e4m3x4_to_f16x2x2(__byte_perm(r[2], 0, 0x3120), vb2[0], vb2[1]);
                    e4m3x4_to_f16x2x2(__byte_perm(r[3], 0, 0x3120), vb2[2], vb2[3]);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        mma16816<C>(o[nt][2 * qq], va, pb[nt][0], pb[nt][1]);
                        mma16816<C>(o[nt][2 * qq + 1], vb2, pb[nt][0], pb[nt][1]);
                    }
                }
            } else {
#pragma unroll
                for (int mt = 0; mt < D / 16; ++mt) {
                    uint32_t r[4];
                    ldsm_x4_trans(r, kb + voff[mt & 3] + (mt >> 2) * G::kBoxBytes);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) mma16816<C>(o[nt][mt], r, pb[nt][0], pb[nt][1]);
                }
            }
        }
        __syncwarp();
        if (!failed && issued < count) issue(issued++, st);
    };
    for (int n0 = 0; n0 < issued; n0 += kStages) {
#pragma unroll
        for (int st = 0; st < kStages; ++st)
            if (n0 + st < issued) consume(n0 + st, st);
    }

    // Per-head sums over the 8 lanes (g = 0..7) that share a head.
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
            l_run[nt][hc] += __shfl_xor_sync(0xffffffffu, l_run[nt][hc], 4);
            l_run[nt][hc] += __shfl_xor_sync(0xffffffffu, l_run[nt][hc], 8);
            l_run[nt][hc] += __shfl_xor_sync(0xffffffffu, l_run[nt][hc], 16);
        }

    // Merge the four warps through shared memory (the rings are free now).
    __syncthreads();
    float *om = reinterpret_cast<float *>(smem);             // [warp][16][D]
    float *mm = om + kAttnWarps * 16 * D;                     // [warp][16]
    float *ll = mm + kAttnWarps * 16;                         // [warp][16]
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = nt * 8 + (lane & 3) * 2 + (e & 1);
                const int d = FP8 ? mt * 16 + (lane >> 2) * 2 + (e >> 1) : mt * 16 + (lane >> 2) + (e >> 1) * 8;
                om[(warp * 16 + row) * D + d] = o[nt][mt][e];
            }
    if (lane < 4) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
                const int row = nt * 8 + lane * 2 + hc;
                mm[warp * 16 + row] = mc[nt][hc];  // base-2 units, as the merge expects
                ll[warp * 16 + row] = l_run[nt][hc];
            }
    }
    __syncthreads();
    failed = s_failed != 0;  // a timed-out wait in any warp voids the CTA's result
    for (int idx = threadIdx.x; idx < cols * D; idx += kAttnThreads) {
        const int row = idx / D, d = idx - row * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, mm[w * 16 + row]);
        float L = 0.f, acc = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kAttnWarps; ++w) {
                const float f = exp2f(mm[w * 16 + row] - M);
                L += ll[w * 16 + row] * f;
                acc += om[(w * 16 + row) * D + d] * f;
            }
        }
        const float val = (L > 0.f && !failed) ? acc / L * v_scale : 0.f;
        const float lse2 = (L > 0.f && !failed) ? M + log2f(L) : -INFINITY;
        const int qi = MQ ? row / a.group : 0;  // query token of the row
        const long long qh = (long long)kvh * a.group + (row - qi * a.group);
        const long long sq = ((long long)seq * (MQ ? a.q_len : 1) + qi) * a.num_q_heads + qh;
        if (a.num_splits == 1) {
            static_cast<T *>(a.out)[sq * D + d] = from_float<T>(val);
            if (d == 0 && a.lse) a.lse[sq] = lse2 * 0.69314718055994531f;
        } else {
            a.part_o[(sq * a.num_splits + split) * D + d] = val;
            if (d == 0) a.part_lse[sq * a.num_splits + split] = lse2;
        }
    }
}

// Merges the splits of one sequence, all its query tokens and heads: per
// (token, head) row the weights 2^(lse_i - max) / sum go to shared memory,
// then every thread combines float4 runs of the partial outputs.
template <typename T, int D>
__global__ void __launch_bounds__(256)
paged_attention_combine_kernel(const AttnLaunch a) {
    extern __shared__ float s_w[];  // [q_len * num_q_heads][num_splits]
    // Launched as a programmatic dependent of the attention grid: its CTAs
    // can take SM slots while the attention's last CTAs run, and wait here
    // until that grid has completed and its partials are visible.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int seq = blockIdx.x;
    const int ctx = checked_ctx(a, seq, false);
    const int nblk = (ctx + kTok - 1) / kTok;
    const int used = max(1, (nblk + a.blocks_per_split - 1) / a.blocks_per_split);
    const int rows = a.q_len * a.num_q_heads;  // the sequence's output rows, contiguous
    for (int h = threadIdx.x; h < rows; h += blockDim.x) {
        const long long sq = (long long)seq * rows + h;
        const float *lse = a.part_lse + sq * a.num_splits;
        float M = -INFINITY;
        for (int i = 0; i < used; ++i) M = fmaxf(M, lse[i]);
        float den = 0.f;
        if (M != -INFINITY)
            for (int i = 0; i < used; ++i) den += exp2f(lse[i] - M);
        for (int i = 0; i < used; ++i)
            s_w[h * a.num_splits + i] = den > 0.f ? exp2f(lse[i] - M) / den : 0.f;
        if (a.lse) a.lse[sq] = den > 0.f ? (M + log2f(den)) * 0.69314718055994531f : -INFINITY;
    }
    __syncthreads();
    for (int it = threadIdx.x; it < rows * (D / 4); it += blockDim.x) {
        const int h = it / (D / 4), d4 = it - h * (D / 4);
        const long long sq = (long long)seq * rows + h;
        const float4 *po = reinterpret_cast<const float4 *>(a.part_o + sq * a.num_splits * D) + d4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int i = 0; i < used; ++i) {
            const float w = s_w[h * a.num_splits + i];
            const float4 v = __ldcs(po + i * (D / 4));
            acc.x += v.x * w;
            acc.y += v.y * w;
            acc.z += v.z * w;
            acc.w += v.w * w;
        }
        uint2 packed;
        packed.x = pack2<T>(acc.x, acc.y);
        packed.y = pack2<T>(acc.z, acc.w);
        *reinterpret_cast<uint2 *>(static_cast<T *>(a.out) + sq * D + d4 * 4) = packed;
    }
}

template <typename T, int D, int NT, bool FP8, bool MQ>
cudaError_t launch_main(const AttnLaunch &a, const CUtensorMap *maps, cudaStream_t st) {
    using G = AttnGeom<D, FP8, attn_stages<D, FP8>(NT)>;
    auto kern = paged_attention_kernel<T, D, NT, FP8, MQ>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)a.num_splits, (unsigned)a.kv_heads, (unsigned)a.num_seqs);
    return launch_pdl(kern, grid, dim3(kAttnThreads), G::kSmem, st, maps[0], maps[1], a);
}

template <typename T, int D, bool FP8>
cudaError_t launch_td(const AttnLaunch &a, const CUtensorMap *maps, cudaStream_t st) {
    if (a.q_len < 1 || a.q_len * a.group > 16) return cudaErrorInvalidValue;
    const bool nt1 = a.q_len * a.group <= 8;
    cudaError_t e = a.q_len == 1 ? (nt1 ? launch_main<T, D, 1, FP8, false>(a, maps, st)
                                        : launch_main<T, D, 2, FP8, false>(a, maps, st))
                                 : (nt1 ? launch_main<T, D, 1, FP8, true>(a, maps, st)
                                        : launch_main<T, D, 2, FP8, true>(a, maps, st));
    if (e != cudaSuccess) return e;
    if (a.num_splits > 1) {
        const size_t smem = (size_t)a.q_len * a.num_q_heads * a.num_splits * sizeof(float);
        if (smem > 227 * 1024) return cudaErrorInvalidValue;
        if (smem > 48 * 1024 &&
            (e = cudaFuncSetAttribute(paged_attention_combine_kernel<T, D>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
            return e;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)a.num_seqs);
        cfg.blockDim = dim3(256);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, paged_attention_combine_kernel<T, D>, a);
    }
    return e;
}

template <typename T, bool FP8>
cudaError_t launch_t(const AttnLaunch &a, const CUtensorMap *maps, int head_dim, cudaStream_t st) {
    switch (head_dim) {
        case 64: return launch_td<T, 64, FP8>(a, maps, st);
        case 128: return launch_td<T, 128, FP8>(a, maps, st);
        case 256: return launch_td<T, 256, FP8>(a, maps, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t make_attention_tmaps(void *k_plane, void *v_plane, DType dtype, long long entry_elems,
                                 long long rows, int head_dim, void *tmaps_out) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess) return e;
    if (!fn || q != cudaDriverEntryPointSuccess) return cudaErrorNotSupported;
    auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    const bool fp8 = dtype == DType::FP8_E4M3;
    const CUtensorMapDataType t = fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                  : dtype == DType::BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int eb = fp8 ? 1 : 2;
    // The plane as [rows][entry] elements; a box is 16 rows x 128 bytes
    // (64 bf16/f16 or 128 E4M3 elements), or the 64 bytes of a 64-dim fp8
    // head with the 64-byte swizzle (AttnGeom::chunk_at).
    const int box_bytes = std::min(head_dim * eb, 128);
    const cuuint64_t dims[2] = {(cuuint64_t)entry_elems, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)entry_elems * eb};
    const cuuint32_t box[2] = {(cuuint32_t)(box_bytes / eb), (cuuint32_t)kTok};
    const cuuint32_t elem_strides[2] = {1, 1};
    const CUtensorMapSwizzle swz = box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    CUtensorMap *maps = static_cast<CUtensorMap *>(tmaps_out);
    void *planes[2] = {k_plane, v_plane};
    for (int i = 0; i < 2; ++i) {
        const CUresult r = encode(&maps[i], t, 2, planes[i], dims, strides, box, elem_strides,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    }
    return cudaSuccess;
}

namespace {
// One CTA: counting sort of the sequences by block count, largest first
// (counts above kPlanKeys - 1 share a bucket after a right shift). Each
// thread owns kPlanKeys / kPlanThreads consecutive buckets of the descending
// key order, so the bucket starts are one block-wide exclusive scan.
constexpr int kPlanThreads = 1024;
constexpr int kPlanKeys = 4096;
constexpr int kPlanPer = kPlanKeys / kPlanThreads;
__global__ void __launch_bounds__(kPlanThreads)
attention_plan_kernel(const int *__restrict__ ctx, int num_seqs, int max_ctx, int shift,
                      unsigned *__restrict__ order) {
    __shared__ unsigned s_count[kPlanKeys];  // indexed by descending key: kPlanKeys - 1 - key
    __shared__ unsigned s_warp[kPlanThreads / 32];
    pdl_wait();
    for (int k = threadIdx.x; k < kPlanKeys; k += kPlanThreads) s_count[k] = 0;
    __syncthreads();
    auto slot = [&](int s) {
        const int c = __ldg(ctx + s);
        const int nblk = (c < 0 || c > max_ctx) ? 0 : (c + kTok - 1) / kTok;
        return kPlanKeys - 1 - min(kPlanKeys - 1, nblk >> shift);
    };
    for (int s = threadIdx.x; s < num_seqs; s += kPlanThreads) atomicAdd(&s_count[slot(s)], 1u);
    __syncthreads();
    // Exclusive scan of the counts in slot order (descending keys).
    unsigned c[kPlanPer], sum = 0;
#pragma unroll
    for (int i = 0; i < kPlanPer; ++i) sum += (c[i] = s_count[threadIdx.x * kPlanPer + i]);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned x = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        unsigned w = s_warp[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        s_warp[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    unsigned at = x - sum + (warp > 0 ? s_warp[warp - 1] : 0u);
#pragma unroll
    for (int i = 0; i < kPlanPer; ++i) {
        s_count[threadIdx.x * kPlanPer + i] = at;
        at += c[i];
    }
    __syncthreads();
    // The lengths are read again here; should a caller rewrite them while
    // this runs, positions past the end are dropped rather than written.
    for (int s = threadIdx.x; s < num_seqs; s += kPlanThreads) {
        const unsigned pos = atomicAdd(&s_count[slot(s)], 1u);
        if (pos < (unsigned)num_seqs) order[pos] = (unsigned)s;
    }
}
}  // namespace

cudaError_t launch_attention_plan(const int *ctx, int num_seqs, int max_ctx, unsigned *order,
                                  cudaStream_t st) {
    if (num_seqs <= 0) return cudaSuccess;
    const int max_blocks = (max_ctx + kTok - 1) / kTok;
    int shift = 0;
    while ((max_blocks >> shift) >= kPlanKeys) ++shift;
    return launch_pdl(attention_plan_kernel, dim3(1), dim3(kPlanThreads), 0, st, ctx, num_seqs, max_ctx,
                      shift, order);
}

int attention_splits(long long num_pairs, int max_ctx, int sms, int *blocks_per_split, bool fp8) {
    const int max_blocks = (max_ctx + kTok - 1) / kTok;
    // At least one block per warp per split, at most PKV_ATTN_SPLIT_BLOCKS
    // (PKV_ATTN_SPLIT_BLOCKS_FP8 for fp8 tiles); fewer blocks per split while
    // the (sequence, kv head) pairs alone cannot fill two CTAs per SM.
    int p = fp8 ? PKV_ATTN_SPLIT_BLOCKS_FP8 : PKV_ATTN_SPLIT_BLOCKS;
    while (p > kAttnWarps && num_pairs * ((max_blocks + p - 1) / p) < 2LL * sms) p /= 2;
    *blocks_per_split = p;
    return std::max(1, (max_blocks + p - 1) / p);
}

cudaError_t launch_paged_attention(const AttnLaunch &a, const void *tmaps, DType pool, DType query,
                                   int head_dim, cudaStream_t st) {
    if (a.num_seqs <= 0 || a.kv_heads <= 0) return cudaSuccess;
    const CUtensorMap *maps = static_cast<const CUtensorMap *>(tmaps);
    if (pool == DType::FP8_E4M3) {
        if (query == DType::BF16) return launch_t<__nv_bfloat16, true>(a, maps, head_dim, st);
        if (query == DType::F16) return launch_t<__half, true>(a, maps, head_dim, st);
        return cudaErrorInvalidValue;
    }
    if (query != pool) return cudaErrorInvalidValue;
    switch (pool) {
        case DType::BF16: return launch_t<__nv_bfloat16, false>(a, maps, head_dim, st);
        case DType::F16: return launch_t<__half, false>(a, maps, head_dim, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace pkv
