// pkv_host.cpp -- native host bookkeeping that produces the inputs of the
// device data path: BlockAllocator (crates/paged-kv-core/src/allocator.rs),
// BlockTable (block_table.rs) and Scheduler (scheduler.rs), with the same
// policies, orderings and error variants, behind include/pkv_host.h.

#include <cstdint>
#include <deque>
#include <string>
#include <vector>

#include "pkv_backend.hpp"
#include "pkv_host.h"

namespace pkv {
namespace host {
namespace {

constexpr uint32_t kMaxRef = 0xFFFF;  // u16 counter, allocator.rs:6-7

Status out_of_blocks(uint64_t requested, uint64_t available) {
    return error(PKV_ERR_OUT_OF_BLOCKS, (int64_t)requested, (int64_t)available,
                 "out of KV blocks: requested " + std::to_string(requested) + ", only " +
                     std::to_string(available) + " free");
}
Status invalid_block(uint64_t id, uint64_t n) {
    return error(PKV_ERR_INVALID_BLOCK, (int64_t)id, (int64_t)n,
                 "invalid block #" + std::to_string(id) + ": pool holds " + std::to_string(n) + " blocks");
}
Status not_allocated(uint64_t id) {
    return error(PKV_ERR_BLOCK_NOT_ALLOCATED, (int64_t)id, 0,
                 "block #" + std::to_string(id) + " is not allocated (refcount 0)");
}

}  // namespace

struct Allocator {
    uint64_t num_blocks;
    std::vector<uint32_t> free_list;  // LIFO stack, top at the back
    std::vector<uint16_t> rc;
    uint64_t total_allocated = 0;
    std::vector<uint32_t> *freed_log = nullptr;

    explicit Allocator(uint64_t n) : num_blocks(n), rc(n, 0) {
        free_list.reserve(n);
        for (uint64_t i = n; i-- > 0;) free_list.push_back((uint32_t)i);  // block 0 on top
    }
    Status validate(uint64_t id) const {
        return id >= num_blocks ? invalid_block(id, num_blocks) : Status::Ok();
    }
    Status allocate(uint32_t *out) {
        if (free_list.empty()) return out_of_blocks(1, 0);
        const uint32_t id = free_list.back();
        free_list.pop_back();
        rc[id] = 1;
        ++total_allocated;
        *out = id;
        return Status::Ok();
    }
    Status allocate_many(uint64_t n, uint32_t *out) {
        if (free_list.size() < n) return out_of_blocks(n, free_list.size());
        for (uint64_t i = 0; i < n; ++i) allocate(out + i);
        return Status::Ok();
    }
    Status incref(uint64_t id, uint32_t *nc) {
        Status s = validate(id);
        if (!s.ok()) return s;
        if (rc[id] == 0) return not_allocated(id);
        if (rc[id] == kMaxRef)
            return error(PKV_ERR_REFCOUNT_OVERFLOW, (int64_t)id, kMaxRef,
                         "refcount overflow on block #" + std::to_string(id) + " (max 65535)");
        if (nc) *nc = ++rc[id];
        else ++rc[id];
        return Status::Ok();
    }
    Status decref(uint64_t id, uint32_t *nc) {
        Status s = validate(id);
        if (!s.ok()) return s;
        if (rc[id] == 0) return not_allocated(id);
        const uint16_t n = --rc[id];
        if (n == 0) {
            free_list.push_back((uint32_t)id);
            if (freed_log) freed_log->push_back((uint32_t)id);
        }
        if (nc) *nc = n;
        return Status::Ok();
    }
    Status is_shared(uint64_t id, bool *shared) const {
        Status s = validate(id);
        if (!s.ok()) return s;
        *shared = rc[id] > 1;
        return Status::Ok();
    }
    Status check_invariants() const {
        std::vector<char> seen(num_blocks, 0);
        for (uint32_t id : free_list) {
            if (id >= num_blocks)
                return error(PKV_ERR_DEVICE, 0, 0, "free list holds out-of-range block #" + std::to_string(id));
            if (seen[id])
                return error(PKV_ERR_DEVICE, 0, 0, "block #" + std::to_string(id) + " appears twice on the free list");
            if (rc[id] != 0)
                return error(PKV_ERR_DEVICE, 0, 0, "block #" + std::to_string(id) +
                                                       " is on the free list but has refcount " +
                                                       std::to_string(rc[id]));
            seen[id] = 1;
        }
        for (uint64_t i = 0; i < num_blocks; ++i)
            if (rc[i] == 0 && !seen[i])
                return error(PKV_ERR_DEVICE, 0, 0, "block #" + std::to_string(i) + " has refcount 0 but is not free");
        return Status::Ok();
    }
};

struct Table {
    std::vector<uint32_t> blocks;
    uint64_t num_tokens = 0;
    uint64_t block_size;

    explicit Table(uint64_t bs) : block_size(bs) {}

    bool last_block_has_room() const {  // block_table.rs:90-92
        return !blocks.empty() && num_tokens % block_size != 0;
    }

    // append (block_table.rs:135-160).
    Status append(Allocator &a, uint32_t *blk, uint64_t *slot, bool *cow, uint32_t *src, uint32_t *dst) {
        *cow = false;
        if (last_block_has_room()) {
            const uint32_t tail = blocks.back();
            bool shared = false;
            Status s = a.is_shared(tail, &shared);
            if (!s.ok()) return s;
            if (shared) {
                uint32_t fresh = 0;
                if (!(s = a.allocate(&fresh)).ok()) return s;
                if (!(s = a.decref(tail, nullptr)).ok()) return s;
                blocks.back() = fresh;
                *cow = true;
                *src = tail;
                *dst = fresh;
            }
        } else {
            uint32_t fresh = 0;
            Status s = a.allocate(&fresh);
            if (!s.ok()) return s;
            blocks.push_back(fresh);
        }
        *blk = blocks[num_tokens / block_size];
        *slot = num_tokens % block_size;
        ++num_tokens;
        return Status::Ok();
    }

    // append_many (block_table.rs:169-209): all-or-nothing. Tokens that land
    // in a tail this call has already made private need no allocator call,
    // so they advance in runs.
    Status append_many(Allocator &a, uint64_t n, uint32_t *out_blk, uint64_t *out_slot,
                       std::vector<uint32_t> *copies) {
        const std::vector<uint32_t> saved = blocks;
        const uint64_t saved_tokens = num_tokens;
        uint64_t done = 0;
        while (done < n) {
            uint32_t b, s, d;
            uint64_t o;
            bool cow;
            Status st = append(a, &b, &o, &cow, &s, &d);
            if (!st.ok()) {
                for (size_t i = std::min(blocks.size(), saved.size()); i < blocks.size(); ++i)
                    a.decref(blocks[i], nullptr);  // errors ignored, as the reference does
                blocks = saved;
                num_tokens = saved_tokens;
                return st;
            }
            if (out_blk) out_blk[done] = b;
            if (out_slot) out_slot[done] = o;
            if (cow && copies) {
                copies->push_back(s);
                copies->push_back(d);
            }
            ++done;
            // The tail is now private: fill the rest of it without the allocator.
            const uint64_t room = (block_size - num_tokens % block_size) % block_size;
            const uint64_t run = std::min(room, n - done);
            for (uint64_t i = 0; i < run; ++i) {
                if (out_blk) out_blk[done + i] = blocks.back();
                if (out_slot) out_slot[done + i] = (num_tokens + i) % block_size;
            }
            num_tokens += run;
            done += run;
        }
        return Status::Ok();
    }

    Status fork(Allocator &a, Table *child) const {  // block_table.rs:218-227
        for (uint32_t b : blocks) {
            Status s = a.incref(b, nullptr);
            if (!s.ok()) return s;
        }
        child->blocks = blocks;
        child->num_tokens = num_tokens;
        child->block_size = block_size;
        return Status::Ok();
    }

    Status release(Allocator &a) {  // block_table.rs:233-239
        for (uint32_t b : blocks) {
            Status s = a.decref(b, nullptr);
            if (!s.ok()) return s;
        }
        blocks.clear();
        num_tokens = 0;
        return Status::Ok();
    }
};

struct Pending {
    uint64_t id, context_len, max_new_tokens;
};

struct Running {
    uint64_t id;
    Table table;
    uint64_t max_new_tokens;
    uint64_t generated;
};

struct Scheduler {
    Allocator alloc;
    uint64_t block_size, max_batch;
    std::deque<Pending> waiting;
    std::vector<Running> running;
    // Last outcome.
    std::vector<uint64_t> admitted, preempted, finished, dec_id, dec_slot;
    std::vector<uint32_t> dec_block, dec_src, dec_dst, freed_raw, freed, adm_blocks;
    std::vector<uint64_t> adm_ctx, adm_off;
    std::vector<int32_t> dec_cow;

    Scheduler(uint64_t nb, uint64_t bs, uint64_t mb) : alloc(nb), block_size(bs), max_batch(mb) {}

    Status add_request(uint64_t id, uint64_t prompt, uint64_t max_new) {  // scheduler.rs:196-213
        const uint64_t cap = alloc.num_blocks * block_size;
        const uint64_t fin = prompt + max_new;
        if (fin > cap) return out_of_blocks((fin + block_size - 1) / block_size, alloc.num_blocks);
        waiting.push_back({id, prompt, max_new});
        return Status::Ok();
    }

    Status admit() {  // scheduler.rs:228-253
        while (running.size() < max_batch && !waiting.empty()) {
            const Pending p = waiting.front();
            Table t(block_size);
            Status s = t.append_many(alloc, p.context_len, nullptr, nullptr, nullptr);
            if (s.code == PKV_ERR_OUT_OF_BLOCKS) break;
            if (!s.ok()) return s;
            waiting.pop_front();
            admitted.push_back(p.id);
            adm_ctx.push_back(p.context_len);
            adm_blocks.insert(adm_blocks.end(), t.blocks.begin(), t.blocks.end());
            adm_off.push_back(adm_blocks.size());
            running.push_back({p.id, std::move(t), p.max_new_tokens, 0});
        }
        return Status::Ok();
    }

    void drop_decoded(uint64_t id) {
        size_t w = 0;
        for (size_t r = 0; r < dec_id.size(); ++r) {
            if (dec_id[r] == id) continue;
            dec_id[w] = dec_id[r];
            dec_block[w] = dec_block[r];
            dec_slot[w] = dec_slot[r];
            dec_cow[w] = dec_cow[r];
            dec_src[w] = dec_src[r];
            dec_dst[w] = dec_dst[r];
            ++w;
        }
        dec_id.resize(w);
        dec_block.resize(w);
        dec_slot.resize(w);
        dec_cow.resize(w);
        dec_src.resize(w);
        dec_dst.resize(w);
    }

    Status preempt_last() {  // scheduler.rs:299-317, victim = newest = last
        Running seq = std::move(running.back());
        running.pop_back();
        drop_decoded(seq.id);
        preempted.push_back(seq.id);
        const uint64_t ctx = seq.table.num_tokens;
        const uint64_t rem = seq.max_new_tokens - seq.generated;
        Status s = seq.table.release(alloc);
        if (!s.ok()) return s;
        waiting.push_front({seq.id, ctx, rem});
        return Status::Ok();
    }

    // decode (scheduler.rs:255-297). Preemption only ever removes the last
    // running sequence, so position i keeps naming the snapshot's i-th
    // sequence for as long as i < running.size().
    Status decode() {
        const size_t n = running.size();
        for (size_t i = 0; i < n; ++i) {
            if (i >= running.size()) break;
            for (;;) {
                uint32_t b, src = 0, dst = 0;
                uint64_t o;
                bool cow;
                Status s = running[i].table.append(alloc, &b, &o, &cow, &src, &dst);
                if (s.ok()) {
                    dec_id.push_back(running[i].id);
                    dec_block.push_back(b);
                    dec_slot.push_back(o);
                    dec_cow.push_back(cow ? 1 : 0);
                    dec_src.push_back(src);
                    dec_dst.push_back(dst);
                    ++running[i].generated;
                    break;
                }
                if (s.code != PKV_ERR_OUT_OF_BLOCKS) return s;
                const bool self = running.size() - 1 == i;
                if (!(s = preempt_last()).ok()) return s;
                if (self) break;  // the sequence being advanced was the victim
            }
        }
        return Status::Ok();
    }

    Status retire() {  // scheduler.rs:319-331, order-preserving compaction
        size_t w = 0;
        for (size_t r = 0; r < running.size(); ++r) {
            if (running[r].generated >= running[r].max_new_tokens) {
                finished.push_back(running[r].id);
                Status s = running[r].table.release(alloc);
                if (!s.ok()) return s;
            } else {
                if (w != r) running[w] = std::move(running[r]);
                ++w;
            }
        }
        running.resize(w, Running{0, Table(block_size), 0, 0});
        return Status::Ok();
    }

    Status step(pkv_step_outcome *out) {  // scheduler.rs:218-226
        admitted.clear();
        preempted.clear();
        finished.clear();
        dec_id.clear();
        dec_block.clear();
        dec_slot.clear();
        dec_cow.clear();
        dec_src.clear();
        dec_dst.clear();
        freed_raw.clear();
        freed.clear();
        adm_ctx.clear();
        adm_blocks.clear();
        adm_off.assign(1, 0);
        alloc.freed_log = &freed_raw;
        Status s = admit();
        if (s.ok()) s = decode();
        if (s.ok()) s = retire();
        alloc.freed_log = nullptr;
        // Blocks released this step and still free at its end.
        for (uint32_t b : freed_raw)
            if (alloc.rc[b] == 0) {
                alloc.rc[b] = kMaxRef;  // mark to dedupe
                freed.push_back(b);
            }
        for (uint32_t b : freed) alloc.rc[b] = 0;
        if (out) {
            out->admitted = admitted.data();
            out->num_admitted = admitted.size();
            out->decoded_id = dec_id.data();
            out->decoded_block = dec_block.data();
            out->decoded_slot = dec_slot.data();
            out->decoded_cow = dec_cow.data();
            out->decoded_cow_src = dec_src.data();
            out->decoded_cow_dst = dec_dst.data();
            out->num_decoded = dec_id.size();
            out->preempted = preempted.data();
            out->num_preempted = preempted.size();
            out->finished = finished.data();
            out->num_finished = finished.size();
            out->freed_blocks = freed.data();
            out->num_freed = freed.size();
            out->admitted_ctx = adm_ctx.data();
            out->admitted_table_offsets = adm_off.data();
            out->admitted_blocks = adm_blocks.data();
        }
        return s;
    }

    Status fork_sequence(uint64_t parent, uint64_t child, uint64_t max_new) {  // :342-357
        for (auto &r : running)
            if (r.id == parent) {
                Table t(block_size);
                Status s = r.table.fork(alloc, &t);
                if (!s.ok()) return s;
                running.push_back({child, std::move(t), max_new, 0});
                return Status::Ok();
            }
        return error(PKV_ERR_UNKNOWN_SEQUENCE, (int64_t)parent, 0,
                     "no sequence with id seq" + std::to_string(parent) + " is running or waiting");
    }
};

}  // namespace host
}  // namespace pkv

struct pkv_allocator {
    pkv::host::Allocator a;
};
struct pkv_table {
    pkv::host::Table t;
};
struct pkv_scheduler {
    pkv::host::Scheduler s;
};

using pkv::finish;

extern "C" {

pkv_allocator *pkv_allocator_new(uint64_t num_blocks) {
    if (num_blocks > 0xFFFFFFFFull) return nullptr;
    return new pkv_allocator{pkv::host::Allocator(num_blocks)};
}
void pkv_allocator_free(pkv_allocator *a) { delete a; }
int pkv_allocator_allocate(pkv_allocator *a, uint32_t *out) { return finish(a->a.allocate(out)); }
int pkv_allocator_allocate_many(pkv_allocator *a, uint64_t n, uint32_t *out) {
    return finish(a->a.allocate_many(n, out));
}
int pkv_allocator_incref(pkv_allocator *a, uint32_t id, uint32_t *nc) { return finish(a->a.incref(id, nc)); }
int pkv_allocator_decref(pkv_allocator *a, uint32_t id, uint32_t *nc) { return finish(a->a.decref(id, nc)); }
int pkv_allocator_ref_count(const pkv_allocator *a, uint32_t id, uint32_t *count) {
    pkv::Status s = a->a.validate(id);
    if (s.ok() && count) *count = a->a.rc[id];
    return finish(s);
}
uint64_t pkv_allocator_num_free(const pkv_allocator *a) { return a->a.free_list.size(); }
uint64_t pkv_allocator_total_allocated(const pkv_allocator *a) { return a->a.total_allocated; }
int pkv_allocator_check_invariants(const pkv_allocator *a) { return finish(a->a.check_invariants()); }
int pkv_allocator_ref_counts(const pkv_allocator *a, const uint32_t *ids, uint64_t n, uint32_t *out) {
    for (uint64_t i = 0; i < n; ++i) {
        pkv::Status s = a->a.validate(ids[i]);
        if (!s.ok()) return finish(s);
        out[i] = a->a.rc[ids[i]];
    }
    return finish(pkv::Status::Ok());
}

pkv_table *pkv_table_new(uint64_t block_size) {
    if (block_size == 0) return nullptr;
    return new pkv_table{pkv::host::Table(block_size)};
}
void pkv_table_free_handle(pkv_table *t) { delete t; }
uint64_t pkv_table_num_tokens(const pkv_table *t) { return t->t.num_tokens; }
uint64_t pkv_table_num_blocks(const pkv_table *t) { return t->t.blocks.size(); }
uint64_t pkv_table_blocks(const pkv_table *t, uint32_t *out, uint64_t cap) {
    const uint64_t n = t->t.blocks.size();
    for (uint64_t i = 0; i < n && i < cap; ++i) out[i] = t->t.blocks[i];
    return n;
}
int pkv_table_append(pkv_table *t, pkv_allocator *a, uint32_t *block, uint64_t *slot, int *cow,
                     uint32_t *cow_src, uint32_t *cow_dst) {
    bool c = false;
    uint32_t s = 0, d = 0;
    const int rc = finish(t->t.append(a->a, block, slot, &c, &s, &d));
    if (cow) *cow = c ? 1 : 0;
    if (cow_src) *cow_src = s;
    if (cow_dst) *cow_dst = d;
    return rc;
}
int pkv_table_append_many(pkv_table *t, pkv_allocator *a, uint64_t n, uint32_t *blocks,
                          uint64_t *slots, uint32_t *copies, uint64_t *num_copies) {
    std::vector<uint32_t> cp;
    const int rc = finish(t->t.append_many(a->a, n, blocks, slots, &cp));
    if (rc == PKV_OK) {
        if (copies)
            for (size_t i = 0; i < cp.size(); ++i) copies[i] = cp[i];
        if (num_copies) *num_copies = cp.size() / 2;
    }
    return rc;
}
int pkv_table_resolve(const pkv_table *t, uint64_t position, uint32_t *block, uint64_t *slot) {
    if (position >= t->t.num_tokens)
        return finish(pkv::error(PKV_ERR_SLOT_OUT_OF_RANGE, (int64_t)position, (int64_t)t->t.num_tokens,
                                 "slot " + std::to_string(position) + " out of range for block size " +
                                     std::to_string(t->t.num_tokens)));
    *block = t->t.blocks[position / t->t.block_size];
    *slot = position % t->t.block_size;
    return finish(pkv::Status::Ok());
}
int pkv_table_fork(const pkv_table *t, pkv_allocator *a, pkv_table **child) {
    auto *c = new pkv_table{pkv::host::Table(t->t.block_size)};
    const int rc = finish(t->t.fork(a->a, &c->t));
    if (rc != PKV_OK) {
        delete c;
        c = nullptr;
    }
    *child = c;
    return rc;
}
int pkv_table_release(pkv_table *t, pkv_allocator *a) { return finish(t->t.release(a->a)); }

pkv_scheduler *pkv_scheduler_new(uint64_t num_blocks, uint64_t block_size, uint64_t max_batch_size) {
    if (block_size == 0 || num_blocks > 0xFFFFFFFFull) return nullptr;
    return new pkv_scheduler{pkv::host::Scheduler(num_blocks, block_size, max_batch_size)};
}
void pkv_scheduler_free(pkv_scheduler *s) { delete s; }
int pkv_scheduler_add_request(pkv_scheduler *s, uint64_t id, uint64_t prompt_len, uint64_t max_new) {
    return finish(s->s.add_request(id, prompt_len, max_new));
}
int pkv_scheduler_step(pkv_scheduler *s, pkv_step_outcome *out) { return finish(s->s.step(out)); }
int pkv_scheduler_fork_sequence(pkv_scheduler *s, uint64_t parent, uint64_t child, uint64_t max_new) {
    return finish(s->s.fork_sequence(parent, child, max_new));
}
uint64_t pkv_scheduler_num_running(const pkv_scheduler *s) { return s->s.running.size(); }
uint64_t pkv_scheduler_num_waiting(const pkv_scheduler *s) { return s->s.waiting.size(); }
double pkv_scheduler_pool_utilization(const pkv_scheduler *s) {
    const auto &a = s->s.alloc;
    return a.num_blocks ? double(a.num_blocks - a.free_list.size()) / double(a.num_blocks) : 0.0;
}
int pkv_scheduler_running(const pkv_scheduler *s, uint64_t *ids, uint64_t *tokens,
                          uint64_t *generated, int32_t *tables, uint64_t stride) {
    const auto &run = s->s.running;
    uint64_t need = 0;
    for (const auto &r : run) need = std::max<uint64_t>(need, r.table.blocks.size());
    if (tables && need > stride)
        return finish(pkv::error(PKV_ERR_SHAPE_MISMATCH, (int64_t)need, (int64_t)stride,
                                 "block tables need a stride of " + std::to_string(need)));
    for (size_t i = 0; i < run.size(); ++i) {
        if (ids) ids[i] = run[i].id;
        if (tokens) tokens[i] = run[i].table.num_tokens;
        if (generated) generated[i] = run[i].generated;
        if (tables) {
            int32_t *row = tables + i * stride;
            const auto &b = run[i].table.blocks;
            for (uint64_t j = 0; j < stride; ++j) row[j] = j < b.size() ? (int32_t)b[j] : -1;
        }
    }
    return finish(pkv::Status::Ok());
}

}  // extern "C"
