/*
 * pkv_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, single-threaded restatement of the reference's host-memory
 * backend (`CpuBackend`, crates/paged-kv-core/src/cpu.rs) together with the
 * default batch methods of the `KvBackend` trait
 * (crates/paged-kv-core/src/backend.rs) and the logical->physical slot rule of
 * `BlockTable` (crates/paged-kv-core/src/block_table.rs).
 *
 * It is the checker that the CUDA data path is compared against, bit for bit.
 * Only the tests, the smoke check and the CPU-baseline leg of the benchmark
 * load it; the product library never links it and has no CPU fallback.
 *
 * Parity pinning: every known-answer test that cpu.rs, block_table.rs and the
 * never-run CUDA oracle tests (crates/paged-kv-cuda/src/backend.rs:345-416)
 * hold is replayed against this file by tests/test_oracle_pins.py.
 *
 * Storage is f32 whatever dtype_bytes says, exactly like CpuBackend
 * (cpu.rs:22-25); an fp8 pool (orc_set_fp8, no counterpart in the reference)
 * stores the widened E4M3 codes in the same f32 planes. Element index:
 *   ((((layer*num_blocks + block)*block_size + slot)*num_kv_heads + head)*head_dim) + d
 * (cpu.rs:13-21, cpu.rs:45-53).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Status codes: one per CacheError variant (crates/paged-kv-core/src/error.rs:12-46).
 * Numbering matches include/pkv_b200.h. */
enum {
    ORC_OK = 0,
    ORC_OUT_OF_BLOCKS = 1,
    ORC_INVALID_BLOCK = 2,
    ORC_BLOCK_NOT_ALLOCATED = 3,
    ORC_REFCOUNT_OVERFLOW = 4,
    ORC_SLOT_OUT_OF_RANGE = 5,
    ORC_SHAPE_MISMATCH = 6,
    ORC_INVALID_LAYER = 7,
    ORC_UNKNOWN_SEQUENCE = 8,
    ORC_DEVICE = 9,
};

/* CacheConfig (crates/paged-kv-core/src/config.rs:8-21). */
typedef struct orc_config {
    uint64_t num_blocks, block_size, num_kv_heads, head_dim, num_layers, dtype_bytes;
} orc_config;

/* PhysicalSlot (crates/paged-kv-core/src/types.rs:40-43). */
typedef struct orc_slot {
    uint64_t block, slot;
} orc_slot;

typedef struct orc_backend {
    orc_config cfg;
    float *k, *v;     /* cpu.rs:27-31 */
    int64_t err_a, err_b; /* the failing variant's two fields */
    /* fp8 (E4M3) pools only: per (layer, kv head) scales and their f32
     * reciprocals; NULL for the f32/bf16/f16 pools of the reference. */
    float *k_scale, *v_scale, *k_inv, *v_inv;
} orc_backend;

static uint64_t entry_elems(const orc_config *c) { return c->num_kv_heads * c->head_dim; } /* config.rs:50-52 */
static uint64_t block_elems(const orc_config *c) { return c->block_size * entry_elems(c); } /* config.rs:56-58 */
static uint64_t layer_elems(const orc_config *c) { return c->num_blocks * block_elems(c); } /* config.rs:62-64 */

static int fail(orc_backend *b, int code, int64_t a, int64_t bb) {
    b->err_a = a;
    b->err_b = bb;
    return code;
}

/* CpuBackend::new (cpu.rs:34-41): both planes zero-filled. */
orc_backend *orc_new(const orc_config *cfg) {
    orc_backend *b = (orc_backend *)calloc(1, sizeof(orc_backend));
    if (!b) return NULL;
    b->cfg = *cfg;
    uint64_t plane = cfg->num_layers * layer_elems(cfg);
    b->k = (float *)calloc(plane ? plane : 1, sizeof(float));
    b->v = (float *)calloc(plane ? plane : 1, sizeof(float));
    if (!b->k || !b->v) {
        free(b->k);
        free(b->v);
        free(b);
        return NULL;
    }
    return b;
}

void orc_free(orc_backend *b) {
    if (!b) return;
    free(b->k);
    free(b->v);
    free(b->k_scale);
    free(b->v_scale);
    free(b->k_inv);
    free(b->v_inv);
    free(b);
}

/*
 * fp8 (E4M3) pools. The reference has none: CpuBackend stores f32 whatever
 * dtype_bytes says (cpu.rs:22-25), and config.rs:19 only leaves room for
 * 1-byte elements. This is the oracle of the device's quantising writes.
 *
 * Format: E4M3 of the OCP 8-bit floating point specification (OFP8, 2023):
 * 1 sign bit, 4 exponent bits with bias 7, 3 mantissa bits; exponent 0 holds
 * the subnormals m * 2^-9; S.1111.111 is NaN; there are no infinities and the
 * largest finite magnitude is 448 (S.1111.110).
 *
 * Encoding of an f32 value: round to nearest, ties to even; magnitudes that
 * would round past 448, and infinities, saturate to +-448 ("satfinite"); NaN
 * encodes as S.1111.111 with the input's sign; -0.0 encodes as 0x80.
 */
uint8_t orc_e4m3_from_f32(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    const uint8_t sign = (uint8_t)((u >> 24) & 0x80);
    const uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return sign | 0x7f;          /* NaN */
    if (a >= 0x43e00000u) return sign | 0x7e;         /* |x| >= 448: saturate */
    const int e = (int)(a >> 23) - 127;               /* unbiased exponent */
    if (e < -6) {
        /* Below the smallest normal 2^-6: m * 2^-9, m = round(|x| * 512). The
         * scaling by 512 is exact and y < 8, so y - floor(y) is exact too. */
        float ax;
        memcpy(&ax, &a, 4);
        const float y = ax * 512.0f;
        uint32_t m = (uint32_t)y;
        const float frac = y - (float)m;
        if (frac > 0.5f || (frac == 0.5f && (m & 1u))) ++m;
        return sign | (uint8_t)m; /* m == 8 is 2^-6, the smallest normal: still right */
    }
    /* Normal: keep 3 of the 23 mantissa bits, round on the other 20. A carry
     * out of the mantissa moves into the exponent field, which is again the
     * correctly rounded value; below 448 it never reaches S.1111.111. */
    const uint32_t mant = a & 0x7fffffu;
    const uint32_t keep = mant >> 20, rest = mant & 0xfffffu, half = 0x80000u;
    uint32_t q = ((uint32_t)(e + 7) << 3) | keep;
    if (rest > half || (rest == half && (keep & 1u))) ++q;
    return sign | (uint8_t)q;
}

/* Exact value of an E4M3 code as f32. */
float orc_e4m3_to_f32(uint8_t q) {
    const uint32_t sign = (uint32_t)(q & 0x80) << 24;
    const uint32_t e = (q >> 3) & 0xfu, m = q & 7u;
    uint32_t bits;
    if (e == 15 && m == 7) {
        bits = sign | 0x7fc00000u;
    } else if (e == 0) {
        float v = (float)m * (1.0f / 512.0f); /* exact */
        memcpy(&bits, &v, 4);
        bits |= sign;
    } else {
        bits = sign | ((e - 7 + 127) << 23) | (m << 20);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

void orc_e4m3_from_f32_array(const float *x, uint64_t n, uint8_t *out) {
    for (uint64_t i = 0; i < n; ++i) out[i] = orc_e4m3_from_f32(x[i]);
}

/* Makes this an fp8 pool: later writes store widen(E4M3(x * inv)) with
 * inv = 1.0f / scale of the element's (layer, kv head), an f32 division and
 * an f32 multiply, each rounded to nearest even; reads return the stored
 * value times the scale. The planes hold the widened E4M3 values, so copies,
 * zeroing and digests are unchanged. scales are [num_layers][num_kv_heads]. */
int orc_set_fp8(orc_backend *b, const float *k_scales, const float *v_scales) {
    const uint64_t n = b->cfg.num_layers * b->cfg.num_kv_heads;
    float **dst[4] = {&b->k_scale, &b->v_scale, &b->k_inv, &b->v_inv};
    for (int i = 0; i < 4; ++i) {
        free(*dst[i]);
        *dst[i] = (float *)malloc((n ? n : 1) * sizeof(float));
        if (!*dst[i]) return fail(b, ORC_DEVICE, 0, 0);
    }
    for (uint64_t i = 0; i < n; ++i) {
        b->k_scale[i] = k_scales[i];
        b->v_scale[i] = v_scales[i];
        b->k_inv[i] = 1.0f / k_scales[i];
        b->v_inv[i] = 1.0f / v_scales[i];
    }
    return ORC_OK;
}

/* Stores one entry of `layer` at plane offset `off`, quantised when fp8. */
static void store_entry(orc_backend *b, float *plane, const float *inv, uint64_t layer,
                        uint64_t off, const float *src) {
    const uint64_t n = b->cfg.num_kv_heads * b->cfg.head_dim;
    if (!inv) {
        memcpy(plane + off, src, n * sizeof(float));
        return;
    }
    for (uint64_t i = 0; i < n; ++i) {
        const float r = inv[layer * b->cfg.num_kv_heads + i / b->cfg.head_dim];
        plane[off + i] = orc_e4m3_to_f32(orc_e4m3_from_f32(src[i] * r));
    }
}

static void load_entry(orc_backend *b, const float *plane, const float *scale, uint64_t layer,
                       uint64_t off, float *out) {
    const uint64_t n = b->cfg.num_kv_heads * b->cfg.head_dim;
    if (!scale) {
        memcpy(out, plane + off, n * sizeof(float));
        return;
    }
    for (uint64_t i = 0; i < n; ++i)
        out[i] = plane[off + i] * scale[layer * b->cfg.num_kv_heads + i / b->cfg.head_dim];
}

float *orc_k_plane(orc_backend *b) { return b->k; }
float *orc_v_plane(orc_backend *b) { return b->v; }
uint64_t orc_plane_elems(const orc_backend *b) { return b->cfg.num_layers * layer_elems(&b->cfg); }
void orc_last_fields(const orc_backend *b, int64_t *a, int64_t *bb) {
    *a = b->err_a;
    *bb = b->err_b;
}

/* block_offset (cpu.rs:45-48) and slot_offset (cpu.rs:51-53). */
static uint64_t block_offset(const orc_backend *b, uint64_t layer, uint64_t block) {
    return (layer * b->cfg.num_blocks + block) * block_elems(&b->cfg);
}
static uint64_t slot_offset(const orc_backend *b, uint64_t layer, orc_slot at) {
    return block_offset(b, layer, at.block) + at.slot * entry_elems(&b->cfg);
}

/* validate_block (cpu.rs:72-80). */
static int validate_block(orc_backend *b, uint64_t block) {
    if (block >= b->cfg.num_blocks)
        return fail(b, ORC_INVALID_BLOCK, (int64_t)block, (int64_t)b->cfg.num_blocks);
    return ORC_OK;
}

/* validate (cpu.rs:55-70): layer, then block, then slot. */
static int validate(orc_backend *b, uint64_t layer, orc_slot at) {
    if (layer >= b->cfg.num_layers)
        return fail(b, ORC_INVALID_LAYER, (int64_t)layer, (int64_t)b->cfg.num_layers);
    int rc = validate_block(b, at.block);
    if (rc) return rc;
    if (at.slot >= b->cfg.block_size)
        return fail(b, ORC_SLOT_OUT_OF_RANGE, (int64_t)at.slot, (int64_t)b->cfg.block_size);
    return ORC_OK;
}

/* check_len (cpu.rs:82-87). */
static int check_len(orc_backend *b, uint64_t expected, uint64_t actual) {
    if (expected != actual) return fail(b, ORC_SHAPE_MISMATCH, (int64_t)expected, (int64_t)actual);
    return ORC_OK;
}

/* write_kv (cpu.rs:95-111): validate, K length, V length, then copy. */
int orc_write_kv(orc_backend *b, uint64_t layer, orc_slot dst, const float *k, uint64_t k_len,
                 const float *v, uint64_t v_len) {
    int rc = validate(b, layer, dst);
    if (rc) return rc;
    uint64_t n = entry_elems(&b->cfg);
    if ((rc = check_len(b, n, k_len))) return rc;
    if ((rc = check_len(b, n, v_len))) return rc;
    uint64_t off = slot_offset(b, layer, dst);
    store_entry(b, b->k, b->k_inv, layer, off, k);
    store_entry(b, b->v, b->v_inv, layer, off, v);
    return ORC_OK;
}

/* Default KvBackend::write_kv_batch (backend.rs:55-74): K shape, V shape,
 * then write_kv per token in order, stopping at the first error (tokens
 * before it stay written). */
int orc_write_kv_batch(orc_backend *b, uint64_t layer, const orc_slot *dsts, uint64_t count,
                       const float *k, uint64_t k_len, const float *v, uint64_t v_len) {
    uint64_t n = entry_elems(&b->cfg);
    uint64_t expected = count * n;
    if (k_len != expected) return fail(b, ORC_SHAPE_MISMATCH, (int64_t)expected, (int64_t)k_len);
    if (v_len != expected) return fail(b, ORC_SHAPE_MISMATCH, (int64_t)expected, (int64_t)v_len);
    for (uint64_t i = 0; i < count; ++i) {
        int rc = orc_write_kv(b, layer, dsts[i], k + i * n, n, v + i * n, n);
        if (rc) return rc;
    }
    return ORC_OK;
}

/* read_kv (cpu.rs:113-129). */
int orc_read_kv(orc_backend *b, uint64_t layer, orc_slot src, float *k_out, uint64_t k_len,
                float *v_out, uint64_t v_len) {
    int rc = validate(b, layer, src);
    if (rc) return rc;
    uint64_t n = entry_elems(&b->cfg);
    if ((rc = check_len(b, n, k_len))) return rc;
    if ((rc = check_len(b, n, v_len))) return rc;
    uint64_t off = slot_offset(b, layer, src);
    load_entry(b, b->k, b->k_scale, layer, off, k_out);
    load_entry(b, b->v, b->v_scale, layer, off, v_out);
    return ORC_OK;
}

/* copy_block (cpu.rs:131-149): validate src, validate dst, self-copy is a
 * no-op, else copy every layer's K and V block (copy_within; src != dst so
 * the ranges never overlap). */
int orc_copy_block(orc_backend *b, uint64_t src, uint64_t dst) {
    int rc;
    if ((rc = validate_block(b, src))) return rc;
    if ((rc = validate_block(b, dst))) return rc;
    if (src == dst) return ORC_OK;
    uint64_t n = block_elems(&b->cfg);
    for (uint64_t layer = 0; layer < b->cfg.num_layers; ++layer) {
        uint64_t s = block_offset(b, layer, src), d = block_offset(b, layer, dst);
        memmove(b->k + d, b->k + s, n * sizeof(float));
        memmove(b->v + d, b->v + s, n * sizeof(float));
    }
    return ORC_OK;
}

/* Default KvBackend::copy_blocks (backend.rs:104-109): sequential, stop at
 * the first error. pairs is [count][2] = (src, dst). */
int orc_copy_blocks(orc_backend *b, const uint64_t *pairs, uint64_t count) {
    for (uint64_t i = 0; i < count; ++i) {
        int rc = orc_copy_block(b, pairs[2 * i], pairs[2 * i + 1]);
        if (rc) return rc;
    }
    return ORC_OK;
}

/* zero_block (cpu.rs:151-160). */
int orc_zero_block(orc_backend *b, uint64_t block) {
    int rc = validate_block(b, block);
    if (rc) return rc;
    uint64_t n = block_elems(&b->cfg);
    for (uint64_t layer = 0; layer < b->cfg.num_layers; ++layer) {
        uint64_t off = block_offset(b, layer, block);
        memset(b->k + off, 0, n * sizeof(float)); /* fill(0.0): +0.0 is all-zero bits */
        memset(b->v + off, 0, n * sizeof(float));
    }
    return ORC_OK;
}

/* A loop of zero_block, stopping at the first error. */
int orc_zero_blocks(orc_backend *b, const uint64_t *blocks, uint64_t count) {
    for (uint64_t i = 0; i < count; ++i) {
        int rc = orc_zero_block(b, blocks[i]);
        if (rc) return rc;
    }
    return ORC_OK;
}

/* allocated_bytes = CacheConfig::total_bytes (backend.rs:118-120, config.rs:68-76). */
uint64_t orc_allocated_bytes(const orc_backend *b) {
    return 2 * b->cfg.num_layers * layer_elems(&b->cfg) * b->cfg.dtype_bytes;
}

/*
 * Slot resolution, the oracle of the device kernel that builds slot_mapping
 * from block tables.
 *
 * For sequence q, with ctx[q] tokens already cached and n_new[q] new tokens,
 * token j (0 <= j < n_new[q]) sits at logical position pos = ctx[q] + j. Its
 * physical address is BlockTable::slot_for_position (block_table.rs:97-101):
 *   block = table[q][pos / block_size], slot = pos % block_size,
 * flattened into vLLM's combined index block*block_size + slot exactly as the
 * reference CUDA backend builds slot_mapping (cuda/src/backend.rs:172-175).
 * cu[q] = sum_{r<q} n_new[r] (the packed offset of sequence q), cu[S] = T.
 *
 * Inputs that the reference would panic on (a logical block past the table's
 * end, a table entry outside the pool) resolve to -1 and count as errors;
 * the return value is the number of such tokens, or -1 if some n_new < 0 or
 * ctx < 0, or -2 if the total differs from num_tokens.
 */
int64_t orc_resolve_slots(const int32_t *tables, int64_t table_stride, const int32_t *ctx,
                          const int32_t *n_new, int64_t num_seqs, int64_t num_tokens,
                          int64_t block_size, int64_t num_blocks, int32_t *cu, int64_t *slots) {
    int64_t total = 0;
    for (int64_t q = 0; q < num_seqs; ++q) {
        if (n_new[q] < 0 || ctx[q] < 0) return -1;
        cu[q] = (int32_t)total;
        total += n_new[q];
    }
    cu[num_seqs] = (int32_t)total;
    if (total != num_tokens) return -2;
    int64_t bad = 0;
    for (int64_t q = 0; q < num_seqs; ++q) {
        for (int64_t j = 0; j < n_new[q]; ++j) {
            int64_t pos = (int64_t)ctx[q] + j;
            int64_t lb = pos / block_size, off = pos % block_size;
            int64_t out = -1;
            if (lb < table_stride) {
                int64_t blk = tables[q * table_stride + lb];
                if (blk >= 0 && blk < num_blocks) out = blk * block_size + off;
            }
            if (out < 0) ++bad;
            slots[cu[q] + j] = out;
        }
    }
    return bad;
}

/*
 * Order-independent plane digest, used to verify pools (and shards of pools)
 * without moving them. Each element contributes mix(p, x) where p is the
 * element's flat index in the FULL (unsharded) plane, doubled plus the plane
 * id (K = 0, V = 1), and x is the element's value widened to f32 bits; +0.0
 * contributes nothing, so an all-zero pool digests to 0 and a pool's digest
 * is the wrapping sum of its shards' digests.
 * The mixer is the splitmix64 finaliser (Steele, Lea & Flood, 2014).
 */
static uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint64_t elem_hash(uint64_t p, uint32_t plane, uint32_t bits) {
    if (bits == 0) return 0;
    uint64_t key = (p * 2 + plane) * 0x9E3779B97F4A7C15ull + bits;
    return mix64(key);
}

/* Digest of a full f32 plane of `elems` elements. */
uint64_t orc_digest_plane(const float *plane, uint64_t elems, uint32_t plane_id) {
    uint64_t acc = 0;
    for (uint64_t i = 0; i < elems; ++i) {
        uint32_t bits;
        memcpy(&bits, plane + i, 4);
        acc += elem_hash(i, plane_id, bits);
    }
    return acc;
}

/* Digest that a plane would have after scattering rows `src` ([count][E] f32)
 * of one layer to distinct combined slots, into an otherwise-zero plane.
 * Used to check full-size runs whose pools do not fit on the host. */
uint64_t orc_digest_rows(const float *src, uint64_t count, uint64_t entry, const int64_t *slots,
                         uint64_t layer, uint64_t slots_per_layer, uint32_t plane_id) {
    uint64_t acc = 0;
    for (uint64_t t = 0; t < count; ++t) {
        if (slots[t] < 0) continue;
        uint64_t base = (layer * slots_per_layer + (uint64_t)slots[t]) * entry;
        for (uint64_t e = 0; e < entry; ++e) {
            uint32_t bits;
            memcpy(&bits, src + t * entry + e, 4);
            acc += elem_hash(base + e, plane_id, bits);
        }
    }
    return acc;
}
