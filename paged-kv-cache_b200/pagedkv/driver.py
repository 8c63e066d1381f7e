"""The StepOutcome driver: applies StepPlans (pagedkv.traces) to a B200Backend.

One step issues, on one CUDA stream and in the order the scheduler's
contract requires (crates/paged-kv-core/src/scheduler.rs:57-63):

1. copy_blocks of the step's copy-on-write pairs (in dependency waves, so
   pairs that chain within the step keep their sequential meaning),
2.+3. slot resolution for the sequences given as block tables fused with
   their all-layer reshape_and_cache (one launch), then one all-layer
   reshape_and_cache for the tokens whose slots the host supplied,
4. zero_blocks of the blocks freed this step.

Step metadata travels host -> device through reused pinned buffers; nothing
is allocated per step once the buffers have grown to the largest step.
"""

from __future__ import annotations

import numpy as np

from .backend import B200Backend
from .traces import StepPlan


class _Staging:
    """A ring of pinned host buffers and one device buffer of int64 words,
    grown on demand. The host reuses a pinned buffer only once the copy out of
    it has finished, `ring` steps later, so it can stage a step while the GPU
    is still busy with the previous ones. The device buffer is rewritten in
    stream order, after the kernels of earlier steps have read it."""

    def __init__(self, dev, ring: int = 4):
        import torch

        self.torch = torch
        self.dev = dev
        self.host = [torch.empty(0, dtype=torch.int64).pin_memory() for _ in range(ring)]
        self.events = [None] * ring
        self.turn = 0
        self.device = torch.empty(0, dtype=torch.int64, device=dev)

    def upload_packed(self, packed: np.ndarray, stream):
        """Copy one int64 buffer to the device on `stream`; returns its device view."""
        torch = self.torch
        total = packed.size
        i = self.turn % len(self.host)
        self.turn += 1
        if self.events[i] is not None:
            self.events[i].synchronize()  # the copy out of this pinned buffer is done
        if self.host[i].numel() < total:
            self.host[i] = torch.empty(2 * total, dtype=torch.int64).pin_memory()
        if self.device.numel() < total:
            self.device = torch.empty(2 * total, dtype=torch.int64, device=self.dev)
        self.host[i].numpy()[:total] = packed
        with torch.cuda.stream(stream):
            self.device[:total].copy_(self.host[i][:total], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
            self.events[i] = ev
        return self.device[:total]

    def upload(self, arrays: list[np.ndarray], stream):
        """Copy the int arrays (as int64 words, each 8-byte aligned) to the device
        on `stream`; returns a device int64 view per array."""
        torch = self.torch
        words = [(a.nbytes + 7) // 8 for a in arrays]
        total = max(sum(words), 1)
        i = self.turn % len(self.host)
        self.turn += 1
        if self.events[i] is not None:
            self.events[i].synchronize()  # the copy out of this pinned buffer is done
        if self.host[i].numel() < total:
            self.host[i] = torch.empty(2 * total, dtype=torch.int64).pin_memory()
        if self.device.numel() < total:
            self.device = torch.empty(2 * total, dtype=torch.int64, device=self.dev)
        hb = self.host[i].numpy().view(np.uint8)
        off = 0
        for a, w in zip(arrays, words):
            hb[off * 8: off * 8 + a.nbytes] = np.ascontiguousarray(a).view(np.uint8).ravel()
            off += w
        with torch.cuda.stream(stream):
            self.device[:total].copy_(self.host[i][:total], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
            self.events[i] = ev
        out, off = [], 0
        for w in words:
            out.append(self.device[off: off + w])
            off += w
        return out


def _pool_dtype_matches(backend: B200Backend, t) -> bool:
    import torch

    return {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}.get(t.dtype) == backend.dtype_tag


def copy_waves(copies: np.ndarray):
    """Orders a step's copy pairs into waves that may each run fully in
    parallel and, applied one after another, give the result of applying
    the pairs sequentially (the trait's default copy_blocks loop,
    crates/paged-kv-core/src/backend.rs:104-109).

    Copy-on-write pairs within one scheduler step can chain: a block freed
    earlier in the step (an old beam, a preempted sequence) can come back
    off the free list as a later pair's destination while an earlier pair
    still reads it as its source. A pair goes one wave after every earlier
    pair that writes its source, reads its destination or writes its
    destination. Self-copies are dropped. Returns (ordered pairs [P'][2],
    [(start, count)] per wave)."""
    copies = np.asarray(copies, np.int64).reshape(-1, 2)
    if len(copies) == 0:
        return np.zeros((0, 2), np.int64), []
    src, dst = copies[:, 0], copies[:, 1]
    if (src != dst).all() and np.unique(dst).size == len(dst) and \
            np.intersect1d(src, dst, assume_unique=False).size == 0:
        # No pair writes a block another pair reads or writes: one wave.
        return np.ascontiguousarray(copies), [(0, len(copies))]
    last_write: dict[int, int] = {}
    last_read: dict[int, int] = {}
    keep, wave = [], []
    for i, (src, dst) in enumerate(copies.tolist()):
        if src == dst:
            continue
        w = max(last_write.get(src, -1), last_read.get(dst, -1), last_write.get(dst, -1)) + 1
        last_write[dst] = w
        last_read[src] = max(last_read.get(src, -1), w)
        keep.append(i)
        wave.append(w)
    if not keep:
        return np.zeros((0, 2), np.int64), []
    wave = np.asarray(wave)
    order = np.argsort(wave, kind="stable")
    ordered = np.ascontiguousarray(copies[np.asarray(keep)[order]], dtype=np.int64)
    counts = np.bincount(wave)
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
    return ordered, [(int(a), int(c)) for a, c in zip(starts, counts) if c]


def group_copy_zero(copies: np.ndarray, zero: np.ndarray, token_blocks: np.ndarray):
    """The arrays of one fused copy + zero launch (pkv_copy_zero_blocks_dev)
    for a step whose copies form one wave, or None when the step needs the
    two separate launches: a destination that is zeroed, or a zeroed block
    that receives one of the step's tokens (zeroing runs before the token
    writes in the fused form, after them in the separate one).

    Returns (srcs, dst_offsets, dsts, zero_src, zero_only): the distinct
    sources in order of first use, each one's destinations in pair order, a
    flag for the sources the step frees, and the other freed blocks."""
    copies = np.asarray(copies, np.int64).reshape(-1, 2)
    zero = np.asarray(zero, np.int64)
    if len(copies) == 0 or len(zero) == 0:
        return None
    if np.isin(copies[:, 1], zero).any() or np.isin(zero, token_blocks).any():
        return None
    srcs, first, inv = np.unique(copies[:, 0], return_index=True, return_inverse=True)
    by_first = np.argsort(first, kind="stable")  # sources in order of first use
    rank = np.empty_like(by_first)
    rank[by_first] = np.arange(len(by_first))
    group = rank[inv]
    order = np.argsort(group, kind="stable")
    dsts = np.ascontiguousarray(copies[order, 1])
    offs = np.concatenate([[0], np.cumsum(np.bincount(group, minlength=len(srcs)))]).astype(np.int64)
    srcs = np.ascontiguousarray(srcs[by_first])
    zero_src = np.isin(srcs, zero).astype(np.int64)
    zero_only = np.ascontiguousarray(zero[~np.isin(zero, srcs)])
    return srcs, offs, dsts, zero_src, zero_only


class DeviceStepper:
    """Runs StepPlans on `backend`. With timing=True each step also records
    CUDA events around its four phases; ``phase_ms()`` sums them."""

    PHASES = ("copy_blocks", "resolve_and_cache", "reshape_and_cache", "zero_blocks")

    def __init__(self, backend: B200Backend, stream=None, timing: bool = False,
                 fuse_copy_zero: bool = True, fuse_mixed: bool = True):
        import torch

        self.torch = torch
        self.b = backend
        self.dev = torch.device("cuda", backend.device)
        self.stream = stream or torch.cuda.current_stream(self.dev)
        self.stage = _Staging(self.dev)
        self.slots = torch.empty(0, dtype=torch.int64, device=self.dev)
        self.cu = torch.empty(0, dtype=torch.int32, device=self.dev)
        self.launches = 0
        self.timing = timing
        self.events: list[list] = []
        # Steps whose copies form one wave and whose zeroes touch neither a
        # destination nor a written block run copies and zeroes as one launch.
        self.fuse_copy_zero = fuse_copy_zero
        self.fused_steps = 0
        # Steps with both resolved and host-slot tokens write them in one
        # launch when the rows do not wrap.
        self.fuse_mixed = fuse_mixed
        self.mixed_steps = 0

    def _mark(self, marks: list) -> None:
        if self.timing:
            e = self.torch.cuda.Event(enable_timing=True)
            e.record(self.stream)
            marks.append(e)

    def phase_ms(self) -> dict:
        """Summed milliseconds per phase and in total over the recorded steps."""
        self.stream.synchronize()
        out = {p: 0.0 for p in self.PHASES}
        for m in self.events:
            for i, p in enumerate(self.PHASES):
                out[p] += m[i].elapsed_time(m[i + 1])
        if self.events:
            out["total"] = self.events[0][0].elapsed_time(self.events[-1][-1])
        return out

    def step_ms(self) -> list[float]:
        """Device milliseconds of each recorded step (first to last phase mark)."""
        self.stream.synchronize()
        return [m[0].elapsed_time(m[-1]) for m in self.events]

    def reset_timing(self) -> None:
        self.events = []

    def _ensure(self, t: int, s: int):
        torch = self.torch
        if self.slots.numel() < t:
            self.slots = torch.empty(max(2 * t, 1024), dtype=torch.int64, device=self.dev)
        if self.cu.numel() < s + 1:
            self.cu = torch.empty(max(2 * (s + 1), 1024), dtype=torch.int32, device=self.dev)

    def prepare(self, plan: StepPlan) -> "Prepared":
        """Host-side work of a step done ahead of time: copy waves and one
        packed buffer of every array the device needs."""
        return Prepared(plan, self.b.config().block_size, self.fuse_copy_zero)

    def make_resident(self, prepared: list["Prepared"]):
        """Uploads the metadata of every prepared step into one device buffer
        (for replaying a trace whose inputs are already in HBM); returns the
        buffer, which must outlive the steps' apply()."""
        torch = self.torch
        total = sum(p.packed.size for p in prepared)
        buf = torch.empty(max(total, 1), dtype=torch.int64, device=self.dev)
        host = torch.from_numpy(np.concatenate([p.packed for p in prepared]) if prepared else
                                np.zeros(1, np.int64))
        buf[:host.numel()].copy_(host)
        off = 0
        for p in prepared:
            p.resident = buf[off:off + p.packed.size]
            off += p.packed.size
        return buf

    def apply(self, plan, k, v) -> int:
        """Runs one step (a StepPlan, or one made ready by prepare()). k, v:
        device [L][R][entry] rows; token i of the step reads row i % R
        (R >= the step's token count keeps every row distinct)."""
        torch = self.torch
        p = plan if isinstance(plan, Prepared) else self.prepare(plan)
        b, st = self.b, self.stream
        tr, d, t, s = p.tr, p.d, p.t, p.s
        self._ensure(t, s)
        # A step made resident (make_resident) reads its metadata where it
        # already lies on the device; otherwise it is uploaded now.
        dev = p.resident if p.resident is not None else self.stage.upload_packed(p.packed, st)
        d_copies, d_tables, d_ctx, d_new, d_direct, d_zero = (dev[a:c] for a, c in p.spans[:6])
        n = 0
        marks: list = []
        self._mark(marks)
        if p.fused is not None:  # copies and zeroes in one launch
            d_srcs, d_off, d_dsts, d_zsrc, d_zonly = (dev[a:c] for a, c in p.spans[6:])
            ns, nz = p.fused
            b.copy_zero_blocks_dev(d_srcs, d_off, d_dsts, d_zsrc, d_zonly, num_srcs=ns,
                                   num_zero=nz, stream=st)
            n += 1
            self.fused_steps += 1
        else:
            for start, count in p.waves:
                b.copy_blocks_dev(d_copies[2 * start:], count=count, stream=st)
                n += 1
        self._mark(marks)
        rows = k.shape[1]
        fused = s and tr <= rows and k.dtype == v.dtype and _pool_dtype_matches(b, k)
        mixed = fused and d and t <= rows and self.fuse_mixed
        if mixed:
            # Resolved and host-slot tokens in one launch: token i reads row i.
            b.resolve_and_cache_mixed(d_tables.view(torch.int32)[: p.table_elems].view(p.table_shape),
                                      d_ctx.view(torch.int32)[:s], d_new.view(torch.int32)[:s], tr,
                                      self.cu, d_direct, d, k[:, :t], v[:, :t],
                                      slots_out=self.slots[:tr], stream=st)
            n += 1
            self.mixed_steps += 1
        elif fused:
            # Slots resolved inline by the scatter itself; they are also
            # published into self.slots for later readers of the cache.
            b.resolve_and_cache(d_tables.view(torch.int32)[: p.table_elems].view(p.table_shape),
                                d_ctx.view(torch.int32)[:s], d_new.view(torch.int32)[:s], tr,
                                self.cu, k[:, :tr], v[:, :tr], slots_out=self.slots[:tr],
                                stream=st)
            n += 1
        elif s:
            b.resolve_slots(d_tables.view(torch.int32)[: p.table_elems].view(p.table_shape),
                            d_ctx.view(torch.int32)[:s], d_new.view(torch.int32)[:s], tr,
                            self.cu, self.slots[:max(tr, 1)], stream=st)
            n += 1
        self._mark(marks)
        # Token i reads row i % rows: scatter in runs that do not wrap. Tokens
        # past the resolved ones take their slots straight from the uploaded
        # list; after a separate resolution every slot is in self.slots.
        start = t if mixed else (tr if fused or not s else 0)
        if not fused and s and d:
            with torch.cuda.stream(st):
                self.slots[tr:t].copy_(d_direct[:d], non_blocking=True)
        while start < t:
            r0 = start % rows
            c = min(rows - r0, t - start)
            slots = self.slots[start:start + c] if start < tr or (s and not fused) else \
                d_direct[start - tr:start - tr + c]
            b.reshape_and_cache(k[:, r0:r0 + c], v[:, r0:r0 + c], slots, stream=st)
            n += 1
            start += c
        self._mark(marks)
        if p.nzero and p.fused is None:
            b.zero_blocks_dev(d_zero, count=p.nzero, stream=st)
            n += 1
        self._mark(marks)
        if self.timing:
            self.events.append(marks)
        self.launches += n
        return n


class Prepared:
    """A StepPlan with its host-side work done: copy waves computed (or the
    copies grouped by source for one fused copy + zero launch) and every
    array packed, as 8-byte-aligned int64 words, into one buffer."""

    def __init__(self, plan: StepPlan, block_size: int = 16, fuse_copy_zero: bool = True):
        tables = np.ascontiguousarray(plan.tables, np.int32)
        copies, self.waves = copy_waves(plan.copies)
        self.fused = None
        extra = []
        if fuse_copy_zero and len(self.waves) == 1 and len(plan.zero):
            written = np.concatenate([np.unique(tables[tables >= 0]).astype(np.int64),
                                      np.asarray(plan.direct_slots, np.int64) // block_size])
            g = group_copy_zero(copies, plan.zero, written)
            if g is not None:
                extra = list(g)
                self.fused = (len(g[0]), len(g[4]))
        parts = [copies, tables, np.ascontiguousarray(plan.ctx, np.int32),
                 np.ascontiguousarray(plan.new, np.int32),
                 np.ascontiguousarray(plan.direct_slots, np.int64),
                 np.ascontiguousarray(plan.zero, np.int64), *extra]
        words = [(a.nbytes + 7) // 8 for a in parts]
        self.packed = np.zeros(max(sum(words), 1), np.int64)
        raw = self.packed.view(np.uint8)
        self.spans, off = [], 0
        for a, w in zip(parts, words):
            raw[off * 8: off * 8 + a.nbytes] = a.view(np.uint8).ravel()
            self.spans.append((off, off + w))
            off += w
        self.tr, self.d = plan.resolved_tokens, len(plan.direct_slots)
        self.t, self.s = self.tr + self.d, len(plan.new)
        self.table_shape, self.table_elems = tables.shape, tables.size
        self.nzero = len(plan.zero)
        self.resident = None  # device view of `packed`, once made resident
