/*
 * pkv_host.h -- C ABI of the native host bookkeeping that feeds the device
 * data path: BlockAllocator, BlockTable and Scheduler of paged-kv-core,
 * restated in C++ inside libpagedkv_b200.so.
 *
 * A Rust caller keeps the reference's own crate for these; they exist here
 * so that the data path can be driven by real allocator/scheduler traces
 * (copy-on-write beams, continuous-batching churn) from C or Python. Status
 * codes and per-thread error fields are those of pkv_b200.h. No GPU is used.
 */
#ifndef PKV_HOST_H
#define PKV_HOST_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct pkv_allocator pkv_allocator;
typedef struct pkv_table pkv_table;
typedef struct pkv_scheduler pkv_scheduler;

/* ---- BlockAllocator (crates/paged-kv-core/src/allocator.rs:24-241) ---- */
pkv_allocator *pkv_allocator_new(uint64_t num_blocks);                      /* :40-55 */
void pkv_allocator_free(pkv_allocator *a);
int pkv_allocator_allocate(pkv_allocator *a, uint32_t *out);                /* :90-105 */
int pkv_allocator_allocate_many(pkv_allocator *a, uint64_t n, uint32_t *out); /* :113-126 */
int pkv_allocator_incref(pkv_allocator *a, uint32_t id, uint32_t *new_count); /* :132-148 */
int pkv_allocator_decref(pkv_allocator *a, uint32_t id, uint32_t *new_count); /* :152-170 */
int pkv_allocator_ref_count(const pkv_allocator *a, uint32_t id, uint32_t *count); /* :181-184 */
uint64_t pkv_allocator_num_free(const pkv_allocator *a);                    /* :63-65 */
uint64_t pkv_allocator_total_allocated(const pkv_allocator *a);             /* :85-87 */
/* check_invariants (:213-240): PKV_OK, or PKV_ERR_DEVICE with the reason in pkv_last_error(). */
int pkv_allocator_check_invariants(const pkv_allocator *a);
/* Reference counts of n blocks at once (0 for free blocks); InvalidBlock on an id out of range. */
int pkv_allocator_ref_counts(const pkv_allocator *a, const uint32_t *ids, uint64_t n, uint32_t *out);

/* ---- BlockTable (crates/paged-kv-core/src/block_table.rs:20-240) ---- */
pkv_table *pkv_table_new(uint64_t block_size);                              /* :46-52 */
void pkv_table_free_handle(pkv_table *t);
uint64_t pkv_table_num_tokens(const pkv_table *t);
uint64_t pkv_table_num_blocks(const pkv_table *t);
/* Copies up to cap block ids; returns the table's block count. */
uint64_t pkv_table_blocks(const pkv_table *t, uint32_t *out, uint64_t cap);
/* append (:135-160): the slot goes to *block and *slot; *cow = 1 with *cow_src,
 * *cow_dst when the shared tail was made private. */
int pkv_table_append(pkv_table *t, pkv_allocator *a, uint32_t *block, uint64_t *slot, int *cow,
                     uint32_t *cow_src, uint32_t *cow_dst);
/* append_many (:169-209): all-or-nothing; slots ([n] blocks and offsets) and
 * copies ([*num_copies][2]) are optional outputs (may be NULL). */
int pkv_table_append_many(pkv_table *t, pkv_allocator *a, uint64_t n, uint32_t *blocks,
                          uint64_t *slots, uint32_t *copies, uint64_t *num_copies);
int pkv_table_resolve(const pkv_table *t, uint64_t position, uint32_t *block, uint64_t *slot); /* :107-115 */
int pkv_table_fork(const pkv_table *t, pkv_allocator *a, pkv_table **child);              /* :218-227 */
int pkv_table_release(pkv_table *t, pkv_allocator *a);                                    /* free, :233-239 */

/* ---- Scheduler (crates/paged-kv-core/src/scheduler.rs:117-358) ---- */

/* StepOutcome (scheduler.rs:72-86). Arrays are owned by the scheduler and
 * stay valid until its next step or destruction. decoded_* are parallel
 * arrays; decoded_cow[i] = 1 when decoded_cow_src/dst[i] hold a copy. */
typedef struct pkv_step_outcome {
    const uint64_t *admitted;
    uint64_t num_admitted;
    const uint64_t *decoded_id;
    const uint32_t *decoded_block;
    const uint64_t *decoded_slot;
    const int32_t *decoded_cow;
    const uint32_t *decoded_cow_src;
    const uint32_t *decoded_cow_dst;
    uint64_t num_decoded;
    const uint64_t *preempted;
    uint64_t num_preempted;
    const uint64_t *finished;
    uint64_t num_finished;
    const uint32_t *freed_blocks; /* blocks whose refcount reached 0 this step (not in the reference's outcome) */
    uint64_t num_freed;
    /* Per admitted sequence (in admitted order): the context length it was
     * admitted with and its block table right after admission, as
     * admitted_blocks[admitted_table_offsets[i] .. admitted_table_offsets[i+1]).
     * The reference's admit discards append_many's slots (scheduler.rs:235-236);
     * these tables are what device slot resolution rebuilds them from. */
    const uint64_t *admitted_ctx;
    const uint64_t *admitted_table_offsets; /* num_admitted + 1 entries */
    const uint32_t *admitted_blocks;
} pkv_step_outcome;

pkv_scheduler *pkv_scheduler_new(uint64_t num_blocks, uint64_t block_size, uint64_t max_batch_size); /* :128-136 */
void pkv_scheduler_free(pkv_scheduler *s);
int pkv_scheduler_add_request(pkv_scheduler *s, uint64_t id, uint64_t prompt_len, uint64_t max_new_tokens); /* :196-213 */
int pkv_scheduler_step(pkv_scheduler *s, pkv_step_outcome *out);                                        /* :218-226 */
int pkv_scheduler_fork_sequence(pkv_scheduler *s, uint64_t parent, uint64_t child, uint64_t max_new_tokens); /* :342-357 */
uint64_t pkv_scheduler_num_running(const pkv_scheduler *s);
uint64_t pkv_scheduler_num_waiting(const pkv_scheduler *s);
double pkv_scheduler_pool_utilization(const pkv_scheduler *s);
/* running_snapshot (:178-189), flattened for the device: per running
 * sequence its id, token count and generated count (arrays of
 * pkv_scheduler_num_running entries) and its block table, row-major into
 * tables[num_running][table_stride] padded with -1. Fails with
 * ShapeMismatch{needed stride, table_stride} if a table is longer. */
int pkv_scheduler_running(const pkv_scheduler *s, uint64_t *ids, uint64_t *tokens,
                          uint64_t *generated, int32_t *tables, uint64_t table_stride);

#ifdef __cplusplus
}
#endif

#endif /* PKV_HOST_H */
