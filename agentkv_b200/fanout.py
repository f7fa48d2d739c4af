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
other instance's replay.  Requirements: the roots' table lengths are
fixed at construction, and nothing else uses the allocator between runs on
another stream.

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
                 merge: bool = True, copier=None, id_base: int = 0) -> None:
        self.alloc = alloc
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
        self.h_roots = torch.empty(int(self.root_lens.sum()), dtype=torch.int32, pin_memory=True)
        self.h_tables = torch.empty(n_child_entries, dtype=torch.int32, pin_memory=True)
        self.h_status = torch.empty(N.STATUS_BYTES // 4, dtype=torch.int32, pin_memory=True)
        self._h_status_np = self.h_status.numpy()  # read after each replay without a tensor op
        self._h_roots_np = self.h_roots.numpy()
        self.d_roots = torch.empty(int(self.root_lens.sum()), dtype=torch.int32, device=self.dev)
        # copy errors land in the allocator's status word when both share a device
        self._copy_status = alloc._status if self.pool.device == alloc.device else None
        self.copies_per_run = int(sum(len(self.root_lens) * self.fanout ** (lv + 1) for lv in range(self.levels)))
        self.launches_per_run = 0
        self._twin: Optional["FanoutGraph"] = None  # run_many's second instance
        with torch.cuda.device(self.dev):  # kernels prepared and graph recorded on the allocator's GPU
            N.check(N.lib.akv_prepare())
            self._note_replay()  # nothing of the allocator's own log may land in the recording
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
                self._record()

    def _record(self) -> None:
        # Allocator kernels on a side stream; each level's copy on the
        # capture stream waits only for that level's plan.  Allocator kernels
        # never touch pool bytes, so they overlap the copies.
        cs = torch.cuda.current_stream(self.dev)
        meta = self._meta = torch.cuda.Stream(self.dev)
        meta.wait_stream(cs)
        events = []
        local = gathered = None
        if self.copier is not None:
            # the gather starts as soon as the last level is planned, before the
            # refcount batches, so the copy waits for the plan and the gather only
            local = torch.empty((self.copies_per_run, 2), dtype=torch.int32, device=self.dev)
            gathered = torch.empty((self.copier.world * self.copies_per_run, 2), dtype=torch.int32, device=self.dev)
        with torch.cuda.stream(meta):
            self.d_roots.copy_(self.h_roots, non_blocking=True)

            def on_level(lvl):
                if gathered is not None and lvl == self.levels - 1:
                    self.copier.gather_pairs(local, self.id_base, gathered)  # every rank's pairs, global ids
                ev = torch.cuda.Event()
                ev.record(meta)
                events.append(ev)

            res = self.alloc.fanout_tree(self.d_roots, self.root_lens, self.levels, self.fanout, self.append,
                                         level_offsets=self.level_off, on_level=on_level, pairs_out=local)
            launches = res["launches"]
            tables = res.get("all_tables")
            if tables is None:
                tables = torch.cat(res["child_tables"])
            if self.free_children:
                self.alloc.dec_ref_batch(tables)
                launches += 4
            self.h_tables.copy_(tables, non_blocking=True)
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
        cs.wait_stream(meta)
        self.h_status.copy_(self.alloc._status, non_blocking=True)
        self._keep = (res, tables, events, gathered)
        self.launches_per_run = launches

    @property
    def h2d_bytes(self) -> int:
        return self.h_roots.numel() * 4

    @property
    def d2h_bytes(self) -> int:
        return (self.h_tables.numel() + self.h_status.numel()) * 4

    def run(self, root_tables, copy: bool = True) -> np.ndarray:
        """Fan out from `root_tables` (host ints, the roots' tables
        concatenated); returns every child's block table concatenated, level
        by level, children in (parent, child) order.  With copy=False the
        result is a view of the pinned read-back buffer, valid until the next
        run()."""
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

    def _twin_graph(self) -> "FanoutGraph":
        if self._twin is None:
            self._twin = FanoutGraph(self.alloc, self.root_lens, self.levels, self.fanout, self.append,
                                     pool=self.pool, free_children=self.free_children, variant=self.variant,
                                     merge=self.merge, copier=self.copier, id_base=self.id_base)
        return self._twin

    def run_many(self, roots_list, on_result=None) -> list:
        """run() on each entry of `roots_list` in turn, with the same results
        (each child table array, in order), keeping the GPU busy: two
        recorded instances of the fan-out alternate, so that while one
        replays, the host reads the other's child tables and writes its next
        roots.  The replays are ordered on one stream, so the allocator sees
        the runs one after another exactly as with run().  With `on_result`
        each run's tables go to on_result(i, tables) instead — a view of the
        pinned read-back buffer, valid during the call — and nothing is kept
        (long sequences of runs without a copy of every table)."""
        graphs = (self, self._twin_graph())
        n_roots = self.h_roots.numel()
        outs = []
        with torch.cuda.device(self.dev):
            stream = torch.cuda.current_stream(self.dev)
            done = (torch.cuda.Event(), torch.cuda.Event())
            held = [False, False]
            runs_done = [0]

            def collect(j: int) -> None:
                done[j].synchronize()
                g = graphs[j]
                if g._h_status_np[0]:
                    self.alloc.check()
                if on_result is None:
                    outs.append(g.h_tables.numpy().copy())
                else:
                    on_result(runs_done[0], g.h_tables.numpy())
                runs_done[0] += 1
                held[j] = False

            for i, roots in enumerate(roots_list):
                j = i % 2
                r = np.asarray(roots, np.int32).reshape(-1)
                if r.size != n_roots:
                    raise ValueError(f"FanoutGraph.run_many: expected {n_roots} root ids, got {r.size}")
                if held[j]:
                    collect(j)  # run i - 2, before this instance is reused
                graphs[j]._h_roots_np[:] = r
                self._note_replay()
                graphs[j].graph.replay()
                done[j].record(stream)
                held[j] = True
            n = len(roots_list)
            for i in (n - 2, n - 1):
                if i >= 0 and held[i % 2]:
                    collect(i % 2)
        return outs
