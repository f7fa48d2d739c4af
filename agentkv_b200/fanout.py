"""FanoutGraph — a Tree-of-Thought fan-out replayed as one CUDA graph.

Agent frameworks fork the same shape of tree over and over (a root forked K
ways for a few levels, every child copy-on-writing the block it will extend
and appending a few blocks).  FanoutGraph records that step once — the host
-> device copy of the root block tables, SlabAllocator.fanout_tree (one
alloc batch, the plan — one launch for all levels when children append
blocks — one inc_ref and one dec_ref batch), the block copies and, optionally,
the frees of every child — and each run() replays it: the caller's host root
tables go in, every child's block table and the status word come back to
host memory, one synchronisation per call.  With appended blocks the levels'
copy-on-write pairs are independent and are copied in one launch after the
last level's plan (merge=True); otherwise each level's copy follows its
plan.

Capturing executes nothing, so the allocator sees exactly the operations of
the runs, in order: ids, refcounts and the free list stay those of the
reference's per-child calls.  run_many() pipelines a sequence of runs over
two recorded instances, hiding the host's read-back and relaunch behind the
other instance's replay; with per_replay=k it replays instances that hold k
consecutive fan-outs each, so that each fan-out's planning (on the
allocator's side stream) overlaps the previous fan-out's copy, which a
replay boundary would otherwise hold back.  Requirements: the roots' table
lengths are fixed at construction, and nothing else uses the allocator
between runs on another stream.

With a `copier` (sharded.ShardedCopier) the fan-out takes part in
partitioned planning: the allocator covers this rank's range of block ids
(starting at `id_base`), the recorded step all-gathers every rank's pair
list after its plan and copies all of them on `pool`, this rank's head slice
of every rank's blocks.  Every rank replays its graph the same number of
times, in the same order.
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import _native as N
from . import kernels as K
from .allocator import SlabAllocator


class FanoutGraph:
    def __init__(self, alloc: SlabAllocator, root_lens, levels: int, fanout: int, append: int, *,
                 pool: Optional[torch.Tensor] = None, free_children: bool = False, variant: int = 0,
                 merge: bool = True, copier=None, id_base: int = 0, per_replay: int = 1) -> None:
        self.alloc = alloc
        self.per_replay = int(per_replay)
        if self.per_replay < 1:
            raise ValueError(f"FanoutGraph: per_replay={per_replay} < 1")
        self.copier, self.id_base = copier, int(id_base)
        if copier is not None and not (merge and int(append) >= 1):
            raise ValueError("FanoutGraph: partitioned planning copies every level in one launch "
                             "(merge=True, append >= 1)")
        self.dev = alloc.device
        self.levels, self.fanout, self.append = int(levels), int(fanout), int(append)
        self.root_lens = np.asarray(root_lens, np.int64)
        if (self.root_lens < 1).any():
            raise ValueError("FanoutGraph: every root needs at least one block")
        self.pool = pool if pool is not None else alloc._kv_data
        self.free_children = free_children
        self.variant = variant
        self.merge = merge
        # fixed shapes of every level
        lens = self.root_lens
        self.level_off = []
        n_child_entries = 0
        for _ in range(self.levels):
            off = np.zeros(len(lens) + 1, np.int64)
            np.cumsum(lens, out=off[1:])
            self.level_off.append(torch.from_numpy(off).to(self.dev))
            lens = np.repeat(lens + self.append, self.fanout)
            n_child_entries += int(lens.sum())
        self.child_lens = lens
        self.n_child_entries = n_child_entries
        self.n_root_entries = int(self.root_lens.sum())
        # per_replay fan-outs' roots / tables back to back
        k = self.per_replay
        self.h_roots = torch.empty(k * self.n_root_entries, dtype=torch.int32, pin_memory=True)
        self.h_tables = torch.empty(k * n_child_entries, dtype=torch.int32, pin_memory=True)
        self.h_status = torch.empty(N.STATUS_BYTES // 4, dtype=torch.int32, pin_memory=True)
        self._h_status_np = self.h_status.numpy()  # read after each replay without a tensor op
        self._h_roots_np = self.h_roots.numpy()
        self.d_roots = torch.empty(k * self.n_root_entries, dtype=torch.int32, device=self.dev)
        # copy errors land in the allocator's status word when both share a device;
        # the copies are then the only launches that use its work counter, so
        # the automatic choice takes the claimed variant
        self._copy_status = alloc._status if self.pool.device == alloc.device else None
        if self.variant == N.VARIANT_AUTO and self._copy_status is not None and self.pool.device.type == "cuda":
            self.variant = K.claimed_variant(self.pool)
        self.copies_per_run = int(sum(len(self.root_lens) * self.fanout ** (lv + 1) for lv in range(self.levels)))
        self.launches_per_run = 0
        self._twin: Optional["FanoutGraph"] = None  # run_many's second instance
        self._grouped: dict = {}  # run_many(per_replay=k): instances of k fan-outs each
        with torch.cuda.device(self.dev):  # kernels prepared and graph recorded on the allocator's GPU
            N.check(N.lib.akv_prepare())
            self._note_replay()  # nothing of the allocator's own log may land in the recording
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
                self._record()

    def _record(self) -> None:
        # Allocator kernels on a side stream; each level's copy on the
        # capture stream waits only for that level's plan.  Allocator kernels
        # never touch pool bytes, so they overlap the copies — the next
        # fan-out's planning included, when a replay holds several.
        cs = torch.cuda.current_stream(self.dev)
        meta = self._meta = torch.cuda.Stream(self.dev)
        meta.wait_stream(cs)
        keep, launches = [], 0
        for r in range(self.per_replay):
            kept, n = self._record_one(cs, meta, r)
            keep.append(kept)
            launches += n
        cs.wait_stream(meta)
        self.h_status.copy_(self.alloc._status, non_blocking=True)
        self._keep = keep  # every fan-out's device buffers live as long as the graph
        self.launches_per_run = launches

    def _record_one(self, cs, meta, r: int):
        """Records fan-out r of a replay: its roots in, its plan and refcount
        batches on `meta`, its copy on `cs`, its tables out."""
        R, T = self.n_root_entries, self.n_child_entries
        d_roots = self.d_roots[r * R:(r + 1) * R]
        events = []
        local = gathered = None
        if self.copier is not None:
            # the gather starts as soon as the last level is planned, before the
            # refcount batches, so the copy waits for the plan and the gather only
            local = torch.empty((self.copies_per_run, 2), dtype=torch.int32, device=self.dev)
            gathered = torch.empty((self.copier.world * self.copies_per_run, 2), dtype=torch.int32, device=self.dev)
        with torch.cuda.stream(meta):
            d_roots.copy_(self.h_roots[r * R:(r + 1) * R], non_blocking=True)

            def on_level(lvl):
                if gathered is not None and lvl == self.levels - 1:
                    self.copier.gather_pairs(local, self.id_base, gathered)  # every rank's pairs, global ids
                ev = torch.cuda.Event()
                ev.record(meta)
                events.append(ev)

            res = self.alloc.fanout_tree(d_roots, self.root_lens, self.levels, self.fanout, self.append,
                                         level_offsets=self.level_off, on_level=on_level, pairs_out=local)
            launches = res["launches"]
            tables = res.get("all_tables")
            if tables is None:
                tables = torch.cat(res["child_tables"])
            if self.free_children:
                self.alloc.dec_ref_batch(tables)
                launches += 4
            self.h_tables[r * T:(r + 1) * T].copy_(tables, non_blocking=True)
        if self.pool.device.type != "meta" and events:
            if self.merge and res["independent"]:
                # every level's pairs in one launch once the last level is planned
                # (and, with a copier, once every rank's pairs are here)
                cs.wait_event(events[-1])
                K.copy_blocks(self.pool, res["all_pairs"] if gathered is None else gathered, variant=self.variant,
                              status=self._copy_status)
                launches += 1
            else:
                for lvl, pairs in enumerate(res["pairs"]):
                    cs.wait_event(events[lvl])
                    K.copy_blocks(self.pool, pairs, variant=self.variant, status=self._copy_status)
                    launches += 1
        return (res, tables, events, local, gathered), launches

    @property
    def h2d_bytes(self) -> int:
        return self.h_roots.numel() * 4

    @property
    def d2h_bytes(self) -> int:
        return (self.h_tables.numel() + self.h_status.numel()) * 4

    def run(self, root_tables, copy: bool = True) -> np.ndarray:
        """Fan out from `root_tables` (host ints, the roots' tables
        concatenated); returns every child's block table concatenated, level
        by level, children in (parent, child) order.  An instance recorded
        with per_replay=k takes k fan-outs' roots back to back and returns
        their tables back to back.  With copy=False the result is a view of
        the pinned read-back buffer, valid until the next run()."""
        roots = np.asarray(root_tables, np.int32).reshape(-1)
        if roots.size != self.h_roots.numel():
            raise ValueError(f"FanoutGraph.run: expected {self.h_roots.numel()} root ids, got {roots.size}")
        self._h_roots_np[:] = roots
        with torch.cuda.device(self.dev):
            self._note_replay()
            self.graph.replay()
            torch.cuda.current_stream(self.dev).synchronize()
        if self._h_status_np[0]:
            self.alloc.check()
        out = self.h_tables.numpy()
        return out.copy() if copy else out

    def _note_replay(self) -> None:
        """A replay runs allocator batches on the device: the allocator's
        per-call log goes first, and its host mirror is reloaded when next
        needed."""
        if self.alloc is not None:
            with self.alloc._lock:
                self.alloc._device_op()

    def _instance(self, per_replay: int) -> "FanoutGraph":
        return FanoutGraph(self.alloc, self.root_lens, self.levels, self.fanout, self.append,
                           pool=self.pool, free_children=self.free_children, variant=self.variant,
                           merge=self.merge, copier=self.copier, id_base=self.id_base, per_replay=per_replay)

    def _twin_graph(self) -> "FanoutGraph":
        if self._twin is None:
            self._twin = self._instance(getattr(self, "per_replay", 1))
        return self._twin

    def run_many(self, roots_list, on_result=None, per_replay: int = 1) -> list:
        """run() on each entry of `roots_list` (one fan-out's roots each) in
        turn, with the same results (each child table array, in order),
        keeping the GPU busy: two recorded instances alternate, so that while
        one replays, the host reads the other's child tables and writes its
        next roots.  With per_replay=k the instances hold k fan-outs each
        (recorded once per k and kept), so a fan-out's planning overlaps the
        copy of the one before it inside a replay; a final len % k runs go
        through one-fan-out instances.  The replays are ordered on one
        stream, so the allocator sees the runs one after another exactly as
        with run().  With `on_result` each run's tables go to
        on_result(i, tables) instead — a view of the pinned read-back buffer,
        valid during the call — and nothing is kept (long sequences of runs
        without a copy of every table)."""
        k = int(per_replay)
        if k < 1:
            raise ValueError(f"FanoutGraph.run_many: per_replay={per_replay} < 1")
        own_k = getattr(self, "per_replay", 1)
        n_roots = self.h_roots.numel() // own_k
        arrays = []
        for roots in roots_list:
            r = np.asarray(roots, np.int32).reshape(-1)
            if r.size != n_roots:
                raise ValueError(f"FanoutGraph.run_many: expected {n_roots} root ids, got {r.size}")
            arrays.append(r)
        outs: list = []
        n_grouped = (len(arrays) // k) * k if k > 1 else 0
        if n_grouped:
            pair = self._grouped.get(k)
            if pair is None:
                pair = self._grouped[k] = (self._instance(k), self._instance(k))
            self._pipelined(pair, arrays[:n_grouped], k, on_result, outs, 0)
        if n_grouped < len(arrays):
            if own_k == 1:
                pair = (self, self._twin_graph())
            else:
                pair = self._grouped.get(1)
                if pair is None:
                    pair = self._grouped[1] = (self._instance(1), self._instance(1))
            self._pipelined(pair, arrays[n_grouped:], 1, on_result, outs, n_grouped)
        return outs

    def _pipelined(self, graphs, arrays, k: int, on_result, outs: list, first: int) -> None:
        """Replays `graphs` (two instances of k fan-outs each) alternately
        over `arrays` (a multiple of k fan-outs' roots), reading each
        instance's tables back before it is replayed again."""
        n_roots = arrays[0].size
        with torch.cuda.device(self.dev):
            stream = torch.cuda.current_stream(self.dev)
            done = (torch.cuda.Event(), torch.cuda.Event())
            held = [False, False]
            runs_done = [first]

            def collect(j: int) -> None:
                done[j].synchronize()
                g = graphs[j]
                if g._h_status_np[0]:
                    self.alloc.check()
                tabs = g.h_tables.numpy()
                per = tabs.size // k
                for r in range(k):
                    t = tabs[r * per:(r + 1) * per]
                    if on_result is None:
                        outs.append(t.copy())
                    else:
                        on_result(runs_done[0], t)
                    runs_done[0] += 1
                held[j] = False

            n_rep = len(arrays) // k
            for b in range(n_rep):
                j = b % 2
                if held[j]:
                    collect(j)  # replay b - 2, before this instance is reused
                g = graphs[j]
                for r in range(k):
                    g._h_roots_np[r * n_roots:(r + 1) * n_roots] = arrays[b * k + r]
                self._note_replay()
                g.graph.replay()
                done[j].record(stream)
                held[j] = True
            for b in (n_rep - 2, n_rep - 1):
                if b >= 0 and held[b % 2]:
                    collect(b % 2)
