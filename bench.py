"""Benchmark of the B200 block-movement path on the Tree-of-Thought workload.

Workload (one "step"): a Llama-3-8B-shaped KV pool (32 layers, 8 KV heads,
head_dim 128, block 16, bf16: 2 MiB per block, 60,000 blocks, seeded N(0,1)
contents, 117 GiB).  A root holding a 4096-token prefix (256 blocks) is forked
8 ways for 3 levels; every child copy-on-writes the last block it inherited
and appends 64 tokens (4 blocks) — 8 + 64 + 512 = 584 CoW copies of 2 MiB —
then all 584 children are freed, returning the pool to its starting shape.
On device: one akv_alloc_batch for every level's ids, one
akv_fanout_tree_plan for all three levels (child tables, the forks' inc_ref
list, CoW pairs, CoW dec_ref list), one akv_incref_batch, one
akv_decref_batch, one akv_copy_blocks of all 584 pairs, and one
akv_decref_batch for the frees; two consecutive steps are recorded as one
CUDA graph (the second step's planning overlaps the first step's copy).
Block ids, refcounts and the free list end exactly as after the reference's
per-child calls (checked by the tests).

Metric: CoW block-copy GB/s = 2 x bytes_per_block x copies / step time
(read + write), whole step timed (metadata kernels included), inputs resident
in HBM; each step touches ~2.4 GB, above the 126 MB L2.

With N GPUs (torchrun, one process per GPU) the pool is sharded by KV head:
each rank holds an 8/N-head slice of every block, and the step runs N trees
(60,000 x N blocks), so the bytes each GPU moves per step stay constant
(weak scaling).  Every rank runs the same deterministic allocator kernels on
its own copy of the block metadata, so all ranks derive identical (src, dst)
pair lists with no collective in the step, and each copies its own slice
(--plan bcast-level / bcast-once instead let rank 0 plan and broadcast the
pair lists over NCCL).

Also reported: `e2e` (the same step through the public FanoutGraph API: the
root tables copied in from pinned host memory, every child's block table and
the status word copied back, one CUDA graph replay and one synchronisation
per step; eager host-driven calls under --no-graph or a broadcast plan), the
copy kernel's roofline, the CPU baseline (the oracle's C
restatement of the reference path on the host cores), clocks sampled during
the timed region, and optionally (--match) the match_prefix stress figure.

`--impl reference` times the reference algorithm's CPU path (the oracle port
with multi-threaded block copies) on the same workload and prints the same
JSON line with "impl": "reference".
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

from agentkv_b200 import workloads as W  # noqa: E402

METRIC = ("CoW block-copy GB/s (% HBM peak) at Llama-3-8B KV shape, Tree-of-Thought fan-out 8x3; "
          "match_prefix queries/s under match_prefix")

try:  # event records inside CUDA graphs (timing the copy launches of the timed replays)
    from cuda.bindings import runtime as _RT
except Exception:  # noqa: BLE001 - without it the copy launch is timed outside the graph
    _RT = None


def _record_in_graph(event, stream) -> None:
    """Record `event` on `stream` so that, during a capture, the graph gets an
    event-record node (a timing point read after each replay)."""
    err = _RT.cudaEventRecordWithFlags(event.cuda_event, stream.cuda_stream, _RT.cudaEventRecordExternal)
    code = err[0] if isinstance(err, tuple) else err
    if int(code) != 0:
        raise RuntimeError(f"cudaEventRecordWithFlags: {code}")
UNIT = "GB/s"
MATCH_DEFAULT_CHUNKS = 8
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--variant", type=int, default=0, help="copy kernel: 0 auto, 1 vec, 2 bulk")
    ap.add_argument("--blocks", type=int, default=W.LLAMA3_8B_GEOMETRY[0], help="blocks per tree/GPU")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-pipeline", action="store_true",
                    help="e2e: time FanoutGraph.run per step only (no run_many)")
    ap.add_argument("--no-graph", action="store_true", help="launch every kernel from Python each step")
    ap.add_argument("--trees", type=int, default=0, help="fan-outs per step (default: one per GPU)")
    ap.add_argument("--heads-per-rank", type=int, default=0, help="KV heads per rank (default: 8 / GPUs)")
    ap.add_argument("--plan", default=None, choices=["bcast-level", "bcast-once", "replicated", "sharded"],
                    help="N > 1: each rank plans its own trees in its own range of block ids and the ranks "
                         "all-gather the pair lists (sharded, the default); every rank runs the same "
                         "deterministic allocator for every tree (replicated, no collective in the step); or "
                         "rank 0 plans and broadcasts each level's pairs / all pairs once")
    ap.add_argument("--graph-nccl", type=int, default=1,
                    help="N > 1: capture the step, NCCL pair broadcast included, as a CUDA graph")
    ap.add_argument("--graph-steps", type=int, default=8,
                    help="consecutive fan-outs recorded in one CUDA graph (the next fan-out's planning overlaps "
                         "the current copy)")
    ap.add_argument("--copy-levels", default="merged", choices=["merged", "per-level"],
                    help="copy every level's CoW pairs in one launch after the last plan, or one launch per "
                         "level as soon as its plan is ready")
    ap.add_argument("--fanouts-per-step", type=int, default=256,
                    help="Tree-of-Thought fan-outs per bench step (a step is a batch of consecutive fan-outs, "
                         "so that the timed region lasts about a second)")
    ap.add_argument("--no-sweep", action="store_true", help="leave out the disjoint-pair copy/zero sweep")
    ap.add_argument("--no-match", action="store_true", help="leave out the match_prefix figure")
    ap.add_argument("--match", action="store_true", help="(kept for old command lines: the figure is on by default)")
    ap.add_argument("--match-seconds", type=float, default=1.0,
                    help="match_prefix: time batches for at least this long")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--match-seqs", type=int, default=W.MatchSpec.n_sequences)
    ap.add_argument("--match-runs", type=int, default=1,
                    help="match_prefix follows unary chains a run at a time (0: one hash probe per hop)")
    ap.add_argument("--match-queries", type=int, default=W.MatchSpec.n_queries)
    ap.add_argument("--match-chunks", type=int, default=0, choices=[0, 1, 2, 4, 8, 16],
                    help="match_prefix verify width: 32-token compares per lane per step (0: the default)")
    ap.add_argument("--match-pipelined", type=int, default=-1,
                    help="match_prefix verify rounds two in flight (1) or one (0); -1: the default")
    ap.add_argument("--match-split", type=int, default=0,
                    help="match_prefix splits queries into token ranges, one warp each (default 0: one warp per "
                         "query, measured faster on this workload)")
    ap.add_argument("--match-staged", type=int, default=0,
                    help="match_prefix as the two-launch staged lookup (chase, then windows over the grid)")
    ap.add_argument("--match-window-tokens", type=int, default=0,
                    help="staged lookup window in tokens: 256, 512 or 1024 (0: the library's default)")
    ap.add_argument("--match-tokens-per-range", type=int, default=0,
                    help="match_prefix split range in tokens, a multiple of 32 (0: the library's default)")
    ap.add_argument("--case", default="tot", choices=["tot", "sweep", "match", "layers", "hf", "react", "percall"],
                    help="tot: the headline step; sweep: batched copy/zero sweep; match: match_prefix on the "
                         "stress tree; layers: copies on vLLM's per-layer cache layout; hf: the HF cache's "
                         "per-layer K/V gather; react: the ReAct multi-agent trace at the Llama-3-70B shape, "
                         "head-sharded under torchrun; percall: per-call latency of the reference-facing API "
                         "(each prints its own line)")
    ap.add_argument("--batches", default="1,8,64,512,4096", help="sweep batch sizes")
    ap.add_argument("--react-steps-per-launch", type=int, default=10,
                    help="react: trace steps applied per akv_agent_steps launch")
    ap.add_argument("--rotations", type=int, default=8, help="sweep: distinct pair sets cycled")
    return ap.parse_args()


def match_chunks_arg(args) -> int:
    """--match-chunks with --match-pipelined folded in (the C ABI's chunks
    argument: the width, OR-ed with AKV_MATCH_PIPELINED)."""
    c = args.match_chunks
    if args.match_pipelined == 1:
        c = (c or MATCH_DEFAULT_CHUNKS) | 0x100
    return c


def measured_peak():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


# ── clocks ───────────────────────────────────────────────────────────────────
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except FileNotFoundError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.rows = [r.split(", ") for r in out.strip().splitlines() if r.strip()]
        else:
            self.rows = []

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for name, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ── the device step ──────────────────────────────────────────────────────────
class ToTBench:
    """One ToT fan-out + free per step on device-resident block tables.

    Rank 0 runs the allocator kernels (alloc, fan-out plan, inc_ref, dec_ref)
    on a side stream; the copies run on the current stream, each level's copy
    waiting only for that level's plan.  Allocator kernels never read or write
    pool bytes, so they overlap the copies; every copy is ordered after the
    previous ones on its stream, which keeps a block that is freed and handed
    out again from being overwritten before an older copy has read it."""

    def __init__(self, rank: int, world: int, blocks_per_tree: int, variant: int, trees: int = 0,
                 heads_per_rank: int = 0, plan: str = "bcast-once", merge: bool = True):
        import torch

        from agentkv_b200.allocator import SlabAllocator
        from agentkv_b200.config import PoolConfig

        self.torch = torch
        self.rank, self.world = rank, world
        self.dev = torch.device("cuda", torch.cuda.current_device())
        n, bs, L, H, D, dt = W.LLAMA3_8B_GEOMETRY
        if H % world:
            raise SystemExit(f"--gpus {world} must divide the {H} KV heads")
        self.spec = W.ToTSpec()
        self.trees = trees or world
        self.n_blocks = blocks_per_tree * self.trees
        self.slice_heads = heads_per_rank or H // world
        self.plan = plan if world > 1 or plan == "sharded" else "replicated"
        # all levels' pairs in one copy launch once the last level is planned
        # (valid because appended blocks make the levels' pairs independent)
        self.merge = merge and self.spec.appended_blocks >= 1 and self.plan != "bcast-level"
        self.planner = rank == 0 or self.plan in ("replicated", "sharded")
        if self.plan == "sharded" and (self.trees % world or not self.merge):
            raise SystemExit(f"--plan sharded: {self.trees} trees must split evenly over {world} ranks "
                             "(and the levels' pairs go in one launch)")
        # the trees this rank plans: all of them, or its own under --plan sharded
        self.plan_trees = self.trees // world if self.plan == "sharded" else self.trees
        # this rank's head slice of every block: [N, L, 2, H/world, bs, D]
        self.pool = torch.empty((self.n_blocks, L, 2, self.slice_heads, bs, D), dtype=torch.bfloat16,
                                device=self.dev)
        g = torch.Generator(device=self.dev)
        g.manual_seed(1234 + rank)
        self.pool.normal_(generator=g)
        self.slice_bytes = L * 2 * self.slice_heads * bs * D * 2
        self.variant = variant
        self.alloc = None
        self.pairs_per_level = [self.trees * c for c in self.spec.children_per_level()]
        root_len = self.spec.root_tokens // bs
        # parent table lengths per level are fixed by the workload
        self.level_lens = []
        lens = np.full(self.plan_trees, root_len, np.int64)
        for _ in range(self.spec.levels):
            self.level_lens.append(lens)
            lens = np.repeat(lens + self.spec.appended_blocks, self.spec.fanout)
        self.level_off = []
        for lens in self.level_lens:
            off = np.zeros(len(lens) + 1, np.int64)
            np.cumsum(lens, out=off[1:])
            self.level_off.append(torch.from_numpy(off).to(self.dev))
        self.pairs_bufs = [torch.empty((n, 2), dtype=torch.int32, device=self.dev) for n in self.pairs_per_level]
        self.all_pairs_buf = torch.empty((sum(self.pairs_per_level), 2), dtype=torch.int32, device=self.dev)
        from agentkv_b200.sharded import ShardedCopier, partition

        self.copier = ShardedCopier(self.pool)
        # --plan sharded: this rank's allocator covers its own range of the ids
        self.id_base, plan_blocks = (partition(self.n_blocks, rank, world) if self.plan == "sharded"
                                     else (0, self.n_blocks))
        self.send_buf = torch.empty((sum(self.pairs_per_level) // world, 2), dtype=torch.int32, device=self.dev)
        if self.planner:
            cfg = PoolConfig(total_blocks=plan_blocks, block_size=bs, num_layers=L, num_kv_heads=H,
                             head_dim=D, dtype=dt, device="meta")
            self.alloc = SlabAllocator(cfg)
            self.root_tables = self.alloc.alloc_batch(root_len * self.plan_trees)
            self.alloc.check()
            self.root_host = self.root_tables.cpu().pin_memory()
            self.meta = torch.cuda.Stream(self.dev)
            n_child_entries = sum(int(x.sum()) * self.spec.fanout + len(x) * self.spec.fanout *
                                  self.spec.appended_blocks for x in self.level_lens)
            self.host_tables = torch.empty(n_child_entries, dtype=torch.int32, pin_memory=True)
            self.host_status = torch.empty(8, dtype=torch.int32, pin_memory=True)
        self.launches_per_step = 0
        self.copy_events = []
        self.last_pairs = None
        # (start, end) event pairs recorded inside captured graphs around each
        # step's copy launch; after a replay they hold that replay's times
        self.graph_marks = []
        self._mark_pool = []
        self.mark_graphs = _RT is not None

    def join(self):
        """Make the current stream wait for the allocator stream."""
        if self.planner:
            self.torch.cuda.current_stream(self.dev).wait_stream(self.meta)

    def step(self, e2e=False, time_copies=False, capture=False, chain=False):
        """Returns (h2d_bytes, d2h_bytes) of the host-driven variant.  With
        chain=True (the second step of a captured pair) the allocator stream
        continues from the previous step's allocator work without waiting for
        its copy: the next fan-out's planning touches only block metadata, so
        it overlaps the previous copy; copies stay ordered on one stream."""
        torch = self.torch
        from agentkv_b200 import kernels as K

        cs = torch.cuda.current_stream(self.dev)
        h2d = d2h = 0
        launches = 0
        events = []
        if self.planner:
            if capture and not chain:
                self.meta.wait_stream(cs)  # fork the allocator stream into the capture
            with torch.cuda.stream(self.meta):
                if e2e:
                    roots = self.root_host.to(self.dev, non_blocking=True)
                    h2d += self.root_host.numel() * 4
                else:
                    roots = self.root_tables

                local = gathered = None
                if self.plan == "sharded":
                    # every rank's pairs in global ids, gathered as soon as the last
                    # level is planned; new buffers per fan-out (the copy stream may
                    # still read the last ones)
                    local = torch.empty_like(self.send_buf)
                    gathered = torch.empty_like(self.all_pairs_buf)
                    gathered.record_stream(cs)

                def on_level(lvl):
                    if gathered is not None and lvl == self.spec.levels - 1:
                        self.copier.gather_pairs(local, self.id_base, gathered, send=self.send_buf)
                    ev = torch.cuda.Event()
                    ev.record(self.meta)
                    events.append(ev)

                res = self.alloc.fanout_tree(roots, self.level_lens[0], self.spec.levels, self.spec.fanout,
                                             self.spec.appended_blocks, level_offsets=self.level_off,
                                             on_level=on_level, pairs_out=local)
                launches += res["launches"]
                frees = res.get("all_tables")
                if frees is None:
                    frees = torch.cat(res["child_tables"])
                self.alloc.dec_ref_batch(frees)  # every child freed, in creation order
                launches += 4
                if e2e:
                    self.host_tables.copy_(frees, non_blocking=True)
                    self.host_status.copy_(self.alloc._status, non_blocking=True)
                    d2h += self.host_tables.numel() * 4 + self.host_status.numel() * 4
        level_pairs = []
        if self.merge:
            if self.plan == "bcast-once":
                if self.rank == 0:
                    res["all_pairs"].record_stream(cs)
                    cs.wait_event(events[-1])
                    allp = res["all_pairs"]
                else:
                    allp = None
                allp = self.copier.share_pairs(allp, sum(self.pairs_per_level), out=self.all_pairs_buf)
            elif self.plan == "sharded":
                allp = gathered
                cs.wait_event(events[-1])  # recorded after the gather was issued
            else:
                allp = res["all_pairs"]
                allp.record_stream(cs)
                cs.wait_event(events[-1])
            if time_copies:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(cs)
            marks = self._graph_marks() if capture else None
            if marks is not None:
                _record_in_graph(marks[0], cs)
            self.copier.copy(allp, variant=self.variant)
            if marks is not None:
                _record_in_graph(marks[1], cs)
                self.graph_marks.append(marks)
            self.last_pairs = allp
            launches += 1
            if time_copies:
                e1.record(cs)
                self.copy_events.append((e0, e1, allp.shape[0]))
            if capture:
                self.join()
            if e2e and self.planner:
                self.join()
                torch.cuda.synchronize(self.dev)
                if int(self.host_status[0]):
                    self.alloc.check()
            self.launches_per_step = launches
            return h2d, d2h
        if self.plan == "bcast-once":
            # one broadcast of every level's pairs once the last level is planned
            if self.rank == 0:
                for p_ in res["pairs"]:
                    p_.record_stream(cs)
                cs.wait_event(events[-1])
                allp = torch.cat(res["pairs"])
            else:
                allp = None
            allp = self.copier.share_pairs(allp, sum(self.pairs_per_level), out=self.all_pairs_buf)
            level_pairs = list(torch.split(allp, self.pairs_per_level))
        for lvl, n_pairs in enumerate(self.pairs_per_level):
            if self.plan == "bcast-once":
                pairs = level_pairs[lvl]
            elif self.planner:
                pairs = res["pairs"][lvl]
                pairs.record_stream(cs)
                cs.wait_event(events[lvl])
                if self.plan == "bcast-level":
                    pairs = self.copier.share_pairs(pairs, n_pairs, out=self.pairs_bufs[lvl])
            else:  # bcast-level, receiving rank
                pairs = self.copier.share_pairs(None, n_pairs, out=self.pairs_bufs[lvl])
            if time_copies:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(cs)
            self.copier.copy(pairs, variant=self.variant)
            launches += 1
            if time_copies:
                e1.record(cs)
                self.copy_events.append((e0, e1, n_pairs))
        if capture:
            self.join()
        if e2e and self.planner:
            self.join()
            torch.cuda.synchronize(self.dev)  # the host reads its tables and the status
            if int(self.host_status[0]):
                self.alloc.check()
        self.launches_per_step = launches
        return h2d, d2h

    def _graph_marks(self):
        """The next pre-created pair of timing events for a copy launch
        recorded into a graph (None when graph marks are off)."""
        return self._mark_pool.pop(0) if self._mark_pool else None

    def _make_marks(self, n: int) -> None:
        """Create and record n event pairs outside any capture (timing events
        must exist before a capture records them)."""
        torch = self.torch
        self._mark_pool = []
        if not self.mark_graphs:
            return
        for _ in range(n):
            pair = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for e in pair:
                e.record()
            self._mark_pool.append(pair)
        torch.cuda.synchronize(self.dev)

    def capture(self, steps: int = 1):
        """Record `steps` consecutive steps as one CUDA graph; returns the
        graph.  With N ranks every rank captures its own steps (the pair
        broadcast included) and the ranks replay in lockstep."""
        torch = self.torch
        g = torch.cuda.CUDAGraph()
        self._make_marks(steps)
        self.graph_marks = []
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            for i in range(steps):
                self.step(capture=True, chain=i > 0)
        self._mark_pool = []
        return g

    def copy_bytes_per_step_global(self):
        """Algorithmic bytes of all copies of one step, all ranks together."""
        return sum(self.pairs_per_level) * 2 * self.slice_bytes * self.world


def timed_steps(run_steps, steps, warmup, world, join=None):
    """timed() for a runner that takes a step count (graphs holding several
    steps): the same barriers, events and max over ranks, EXACTLY `steps`
    steps in the timed region."""
    import torch

    run_steps(warmup)
    if join is not None:
        join()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    run_steps(steps)
    if join is not None:
        join()
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    return ms, wall


def timed(fn, steps, warmup, world, join=None):
    import torch

    for _ in range(warmup):
        fn()
    if join is not None:
        join()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(steps):
        fn()
    if join is not None:
        join()
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    return ms, wall


# ── CPU path (oracle port of the reference algorithm) ────────────────────────
def cpu_tot_run(trees: int, steps: int, warmup: int, threads: int, max_seconds: float | None = None):
    """The reference's per-child sequence on the host: fork inc_refs, CoW
    (alloc, copy 2 MiB, dec_ref), 4 allocs; then every child freed.  Uses the
    oracle's C restatement of the allocator and multi-threaded block copies
    on a host pool of 4096 blocks (enough for the 3,176 blocks one fan-out
    touches); `trees` fan-outs run back to back per step.  Returns GB/s on
    the compulsory bytes (each distinct source read once, each destination
    written once: the GPU figure's count), steps, seconds, bytes per block,
    threads and GB/s on the algorithmic 2 x bytes per pair."""
    from oracle import oracle as O

    n, bs, L, H, D, _ = W.LLAMA3_8B_GEOMETRY
    bpb = L * 2 * H * bs * D * 2
    spec = W.ToTSpec()
    host_blocks = 4096
    pool = np.empty((host_blocks, bpb), np.uint8)
    for i in range(0, host_blocks, 512):  # touch every page
        pool[i : i + 512] = (i // 512) & 0xFF
    a = O.OracleAllocator(host_blocks)
    root = a.alloc_seq(spec.root_tokens // bs)

    def one_tree():
        level = [root]
        kids = []
        for _ in range(spec.levels):
            nxt = []
            for parent in level:
                for _ in range(spec.fanout):
                    a.inc_ref_seq(parent)  # fork
                    new = a.alloc_seq(1)  # ensure_mutable_block: alloc ...
                    O.copy_blocks(pool, bpb, np.array([[parent[-1], new[0]]], np.int32), threads)
                    a.dec_ref_seq(parent[-1:])  # ... copy, dec_ref
                    app = a.alloc_seq(spec.appended_blocks)
                    nxt.append(np.concatenate([parent[:-1], new, app]).astype(np.int32))
            kids.extend(nxt)
            level = nxt
        for c in kids:
            a.dec_ref_seq(c)

    def one_step():
        for _ in range(trees):
            one_tree()

    if threads <= 0:
        # use the thread count that copies fastest on this host (one step each)
        best = None
        for t in cpu_thread_candidates():
            threads = t
            t0 = time.perf_counter()
            one_step()
            dt = time.perf_counter() - t0
            if best is None or dt < best[0]:
                best = (dt, t)
        threads = best[1]
    for _ in range(warmup):
        one_step()
    times = []
    t_start = time.perf_counter()
    for i in range(steps):
        t0 = time.perf_counter()
        one_step()
        times.append(time.perf_counter() - t0)
        if max_seconds is not None and time.perf_counter() - t_start > max_seconds and i + 1 >= 2:
            break
    copies = trees * sum(spec.children_per_level())
    sources = trees * sum(spec.fanout ** lvl for lvl in range(spec.levels))
    gbs = bpb * (sources + copies) * len(times) / sum(times) / 1e9
    gbs_alg = 2 * bpb * copies * len(times) / sum(times) / 1e9
    return gbs, len(times), sum(times), bpb, threads, gbs_alg


def host_cpu() -> dict:
    """The host's CPU model string and logical CPU count, reported beside
    every CPU baseline."""
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    if not model:
        import platform

        model = platform.processor() or platform.machine()
    return {"cpu_model": model, "logical_cpus": os.cpu_count()}


def cpu_thread_candidates():
    n = os.cpu_count() or 1
    return sorted({t for t in (1, 4, 8, 16, 32, 64, n) if t <= n})


def reference_arm(args, rank, world):
    """The reference algorithm's CPU path (the oracle's C restatement, block
    copies over the host's threads) on the Tree-of-Thought workload; rank 0
    alone.  A bench step of the GPU arm is --fanouts-per-step fan-outs; here
    each step is a bounded sample of `world` fan-outs (the GPU arm's per-rank
    work), timed on the same compulsory bytes."""
    if rank != 0:
        return
    gbs, steps, secs, bpb, threads, gbs_alg = cpu_tot_run(world, args.steps, args.warmup, 0)
    sample = (f"{world} Tree-of-Thought fan-out(s) per step ({world * 584} CoW copies of {bpb} B), "
              f"host pool of 4096 blocks, {steps} steps in {secs:.1f} s")
    n_, bs, L, H, D, _ = W.LLAMA3_8B_GEOMETRY
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(1e3 * secs / steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded token ids and pool bytes)",
        "config": {"workload": "tot_8b_fanout", "pool_blocks": n_ * world, "fanouts_per_step": world,
                   "trees_per_fanout": world, "bytes_per_block": bpb, "cow_copies_per_fanout": 584 * world,
                   "bytes_counted": "compulsory: each distinct source block read once + each destination "
                                    "written once",
                   "parallelism": "host threads", "heads_per_rank": H},
        "algorithmic_gbs": round(gbs_alg, 3),
        "cpu_baseline": {"value": round(gbs, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample, "host": host_cpu()},
        "e2e": {"value": round(gbs, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ── match_prefix figure ──────────────────────────────────────────────────────
MATCH_NODE_BYTES = 32  # per visited node: its child slot (16 B) + edge offset and length, rounded up


def match_compulsory_bytes(parent, edge_len, children, queries, out_node, out_cmp) -> dict:
    """Compulsory DRAM bytes of one match_prefix batch: 4 B per query token
    compared (the reference loop's comparison count), 4 B per distinct edge
    token the batch touches (every edge on a matched path in full, the
    partially compared child of each path end as far as it was compared) and
    MATCH_NODE_BYTES per distinct visited node.  `parent`, `edge_len` and
    `children` map node ids of the host tree; `out_node` / `out_cmp` are the
    batch's results.  A query with no credited match (node -1) is counted
    from the root."""
    depth = {0: 0}
    full = {0}
    partial: dict = {}
    q_bytes = 0

    def depth_of(u: int) -> int:
        stack = []
        v = u
        while v not in depth:
            stack.append(v)
            v = parent[v]
        d = depth[v]
        for w in reversed(stack):
            d += int(edge_len[w])
            depth[w] = d
        return d

    for q, u, c in zip(queries, out_node, out_cmp):
        c = int(c)
        q_bytes += 4 * c
        u = int(u) if int(u) >= 0 else 0
        v = u
        while v not in full:  # once a node is in, so are its ancestors
            full.add(v)
            v = parent[v]
        d = depth_of(u)
        rest = c - d
        if rest > 0 and d < len(q):
            ch = children[u].get(int(q[d]))
            if ch is not None:
                partial[ch] = max(partial.get(ch, 0), min(rest, int(edge_len[ch])))
    edge_tokens = sum(int(edge_len[v]) for v in full) + sum(n for v, n in partial.items() if v not in full)
    nodes = len(full | set(partial))
    return {"query_bytes": q_bytes, "edge_bytes": 4 * edge_tokens, "node_bytes": MATCH_NODE_BYTES * nodes,
            "total": q_bytes + 4 * edge_tokens + MATCH_NODE_BYTES * nodes, "nodes": nodes}


def match_cpu_baseline(pool, batches, gpu_results, max_seconds: float) -> dict:
    """The oracle's C restatement of _match_prefix_locked, one host thread,
    over the same tree and batches (repeated until max_seconds); also checks
    its answers against the GPU's."""
    from oracle import oracle as O

    nodes = pool._tree._shared_nodes
    n = max(nodes) + 1
    child_ptr = np.zeros(n + 1, np.int64)
    keys, ids, toks = [], [], []
    edge_off = np.zeros(n, np.int64)
    edge_len = np.zeros(n, np.int32)
    pos = 0
    for nid in range(n):
        nd = nodes.get(nid)
        if nd is not None:
            for k in sorted(nd.children):
                keys.append(k)
                ids.append(nd.children[k])
            e = np.asarray(nd.edge, np.int32)
            edge_off[nid], edge_len[nid] = pos, len(e)
            toks.append(e)
            pos += len(e)
        child_ptr[nid + 1] = len(keys)
    csr = {"child_ptr": child_ptr, "child_key": np.asarray(keys or [0], np.int32),
           "child_id": np.asarray(ids or [0], np.int32), "edge_off": edge_off, "edge_len": edge_len,
           "edge_tokens": np.concatenate(toks) if pos else np.zeros(1, np.int32)}
    packed = [O.pack_queries(b) for b in batches]
    same = True
    for (flat, off), (g_node, g_len) in zip(packed, gpu_results):
        o_node, o_len, _ = O.match_prefix_csr(csr, flat, off, 16)
        same &= bool(np.array_equal(o_len, g_len) and np.array_equal(np.where(o_len > 0, o_node, -1),
                                                                      np.where(g_len > 0, g_node, -1)))
    done = 0
    t0 = time.perf_counter()
    while True:
        flat, off = packed[done % len(packed)]
        O.match_prefix_csr(csr, flat, off, 16)
        done += 1
        secs = time.perf_counter() - t0
        if secs >= max_seconds:
            break
    nq = len(batches[0])
    # the reference's own loop, in Python, on the first queries of batch 0
    py_tree = O.csr_children(csr)
    py_done, py_secs = 0, 0.0
    while py_done < len(batches[0]) and py_secs < max_seconds / 2:
        chunk = [q.tolist() for q in batches[0][py_done:py_done + 16]]  # the reference's token lists
        t1 = time.perf_counter()
        O.match_prefix_py(py_tree, chunk, 16)
        py_secs += time.perf_counter() - t1
        py_done += len(chunk)
    return {"value": round(done * nq / secs, 1), "unit": "queries/s", "cores": 1, "kind": "port",
            "sample": f"{done} batches of {nq} queries on the same tree, {secs:.1f} s, one host thread "
                      f"(the oracle's C restatement)",
            "same_answers_as_gpu": same, "host": host_cpu(),
            "python_loop": {"value": round(py_done / py_secs, 1), "unit": "queries/s",
                            "sample": f"{py_done} queries of batch 0, {py_secs:.1f} s: the reference's loop "
                                      f"in pure Python, one thread"}}


def match_figure(steps: int, warmup: int, n_seqs: int = W.MatchSpec.n_sequences,
                 n_queries: int = W.MatchSpec.n_queries, rank: int = 0, world: int = 1,
                 use_runs: bool = True, cpu_seconds: float = 0.0, chunks: int = 0, split: bool = False,
                 tokens_per_item: int = 0, min_seconds: float = 0.0, staged: bool = False,
                 window_tokens: int = 0) -> dict:
    """match_prefix on the stress tree (the one-warp walk; with staged=True
    the two-launch lookup, akv_match_prefix_staged).  With N ranks, rank 0 builds the tree
    through the pool API and broadcasts it (TreeReplicaSync) to every rank's
    replica; each rank then matches its own 4096-query batches (weak
    scaling), timed as the max over ranks.  Rank 0 adds the kernel's
    roofline (compulsory bytes of its batches, match_compulsory_bytes) and,
    at one rank with cpu_seconds > 0, the CPU baseline."""
    import torch

    from agentkv_b200 import AgentKVPool, PoolConfig
    from agentkv_b200.device_tree import DeviceTree, longest_first, pack_queries
    from agentkv_b200.sharded_tree import TreeReplicaSync

    spec = W.MatchSpec(n_sequences=n_seqs, n_queries=n_queries)
    prefixes = W.match_prefixes(spec)
    corpus = W.match_sequences(spec, prefixes)
    dev = torch.device("cuda", torch.cuda.current_device())
    build_s = 0.0
    n_nodes = None
    if rank == 0:
        total_blocks = sum(-(-len(s) // 16) for s in corpus) + 16
        cfg = PoolConfig(total_blocks=total_blocks, block_size=16, num_layers=1, num_kv_heads=1, head_dim=1,
                         dtype="float16", device="meta")
        pool = AgentKVPool(config=cfg)
        t0 = time.perf_counter()
        for seq in corpus:
            h = pool.create_root(seq)
            pool.allocate_blocks(h, -(-len(seq) // 16) - len(pool.get_block_ids(h)))
            share = (len(seq) // 16) * 16 - h.shared_match_len
            if share > 0:
                pool.commit_prefix(h, share)
        build_s = time.perf_counter() - t0
        tree = pool._tree._dev_tree
        n_nodes = len(pool._tree._shared_nodes)
    else:
        tree = DeviceTree(dev)
    t0 = time.perf_counter()
    if world > 1:
        TreeReplicaSync(tree).sync()
    else:
        tree.flush()
    torch.cuda.synchronize()
    sync_s = time.perf_counter() - t0
    batches = [W.match_queries(spec, corpus, prefixes, batch=rank * 4 + b) for b in range(4)]
    packed = [pack_queries(q, dev) for q in batches]
    orders = [longest_first(off, dev) for _, off in packed]
    nq = spec.n_queries
    # the split lookups' range plans (host: the lengths in launch order)
    from agentkv_b200.device_tree import split_plan

    plans = [split_plan(np.sort(np.asarray([len(q) for q in b_], np.int64))[::-1], tokens_per_item)
             if split else None for b_ in batches]
    node = torch.empty(nq, dtype=torch.int32, device=dev)
    mlen = torch.empty(nq, dtype=torch.int32, device=dev)
    cmp_ = torch.empty(nq, dtype=torch.int64, device=dev)
    totals = [int(off[-1].item()) for _, off in packed]
    lookup = {"staged": staged, "window_tokens": window_tokens}
    compared = []
    qtokens = []
    results = []
    for (tok, off), order, plan, nt in zip(packed, orders, plans, totals):
        tree.match(tok, off, nq, 16, node, mlen, cmp_, order=order, runs=use_runs, chunks=chunks, plan=plan,
                   n_tokens=nt, **lookup)
        compared.append(int(cmp_.sum()))
        qtokens.append(int(off[-1]))
        results.append((node.cpu().numpy(), mlen.cpu().numpy(), cmp_.cpu().numpy()))
    tree.check()
    alg = None
    if rank == 0:
        shared = pool._tree._shared_nodes
        parent = {k: v.parent_id for k, v in shared.items()}
        elen = {k: v.edge_len for k, v in shared.items()}
        kids = {k: v.children for k, v in shared.items()}
        per = [match_compulsory_bytes(parent, elen, kids, q, r[0], r[2]) for q, r in zip(batches, results)]
        alg = {k: int(statistics.mean(p[k] for p in per)) for k in per[0]}

    def run():
        for (tok, off), order, plan, nt in zip(packed, orders, plans, totals):
            tree.match(tok, off, nq, 16, node, mlen, cmp_, order=order, runs=use_runs, chunks=chunks, plan=plan,
                       n_tokens=nt, **lookup)

    # enough repetitions of the rotation for min_seconds (the same count on every rank)
    ms_probe, _ = timed(run, 3, warmup, 1)
    steps = max(steps, int(np.ceil(min_seconds / max(ms_probe / 3e3, 1e-6))))
    if world > 1:
        t = torch.tensor([steps], dtype=torch.int64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        steps = int(t.item())
    sampler = ClockSampler(torch.cuda.current_device())
    with sampler:
        ms, wall = timed(run, steps, warmup, world)
    clocks = sampler.summary()
    per_batch_ms = ms / (steps * len(packed))
    (tok0, off0), order0, plan0 = packed[0], orders[0], plans[0]

    def run_warm():  # one batch again and again: its query tokens stay in L2
        for _ in range(len(packed)):
            tree.match(tok0, off0, nq, 16, node, mlen, cmp_, order=order0, runs=use_runs, chunks=chunks,
                       plan=plan0, n_tokens=totals[0], **lookup)

    ms_w, _ = timed(run_warm, steps, warmup, world)
    warm_ms = ms_w / (steps * len(packed))
    tok_cmp = statistics.mean(compared)
    if world > 1:
        t = torch.tensor([tok_cmp], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t)
        tok_cmp = float(t) / world
    roofline = cpu = e2e = None
    if rank == 0 and world == 1:
        # through the public call with host queries: pack into the pinned
        # stage, upload, look up, read the answers back (one batch per call)
        for b in range(len(batches)):  # every batch of the rotation once: the stage has grown to the largest
            pool.match_prefix_batch(batches[b])
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        reps = 2 * len(batches)
        for i in range(reps):
            pool.match_prefix_batch(batches[i % len(batches)])
        e2e_s = (time.perf_counter() - t0) / reps
        # where the time goes: the host packing (and its sliced upload) alone
        stage = pool._tree._dev_tree._stage
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        stage.pack(batches[0])
        pack_ms = (time.perf_counter() - t0) * 1e3
        torch.cuda.synchronize()
        upload_ms = (time.perf_counter() - t0) * 1e3
        h2d = int(statistics.mean(qtokens)) * 4 + (nq + 1) * 8 + nq * 4
        e2e = {"value": round(nq / e2e_s, 1), "unit": "queries/s", "ms_per_batch": round(e2e_s * 1e3, 3),
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": nq * 8,
               "host_pack_ms": round(pack_ms, 3), "pack_and_upload_ms": round(upload_ms, 3),
               "api": "AgentKVPool.match_prefix_batch (host token lists in, numpy answers out)"}
    if rank == 0:
        peak, peak_kind = measured_peak()
        achieved = alg["total"] / (per_batch_ms / 1e3) / 1e9
        roofline = {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "traffic": MATCH_TRAFFIC_NCU[n_seqs][0] if (use_runs and not split and n_seqs in MATCH_TRAFFIC_NCU)
            else None,
            "peak_source": peak_kind,
            "kernel": (f"akv match_prefix_split (k_match_split), one {nq}-query batch" if split
                       else f"akv match_prefix_staged (k_match_chase + k_match_verify), one {nq}-query batch"
                       if staged else f"akv match_prefix (k_match), one {nq}-query batch"),
            "algorithmic_bytes_per_launch": alg,
            "note": "compulsory bytes: 4 B per query token compared, 4 B per distinct edge token touched, "
                    f"{MATCH_NODE_BYTES} B per distinct visited node (rank 0's batches); the kernel is "
                    "bound by dependent-load latency and issue, not by DRAM bandwidth",
        }
        if world == 1 and cpu_seconds > 0:
            cpu = match_cpu_baseline(pool, batches, [(r[0], r[1]) for r in results], cpu_seconds)
    return {
        "metric": "match_prefix queries/s (stress tree)",
        "value": round(world * nq / (per_batch_ms / 1e3), 1),
        "unit": "queries/s",
        "n_gpus": world,
        "scaling": "weak",
        "tokens_compared_per_ms": round(world * tok_cmp / per_batch_ms, 1),
        "tokens_compared_per_ms_per_gpu": round(tok_cmp / per_batch_ms, 1),
        "ms_per_batch": round(per_batch_ms, 4),
        "l2": f"{len(packed)} batches in rotation ({len(packed)} x {int(statistics.mean(qtokens)) * 4 / 1e6:.0f} MB "
              f"of query tokens, above the 126 MB L2); warm: batch 0 repeated",
        "batches_timed": steps * len(packed),
        "wall_s_timed": round(wall, 3),
        "clocks": clocks,
        "warm_ms_per_batch": round(warm_ms, 4),
        "warm_queries_per_s": round(world * nq / (warm_ms / 1e3), 1),
        "warm_tokens_compared_per_ms_per_gpu": round(compared[0] / warm_ms, 1),
        "batch_per_gpu": nq,
        "tree_nodes": n_nodes,
        "tree_build_s": round(build_s, 1),
        "replica_sync_s": round(sync_s, 2),
        "query_tokens_per_batch": int(statistics.mean(qtokens)),
        "unary_runs": bool(use_runs),
        "verify_chunks": (chunks & 0xFF) or (4 if split else 8),
        "verify_flags": {"pipelined": bool(chunks & 0x100), "prefetch": bool(chunks & 0x200)},
        "staged": {"window_tokens": window_tokens or 512} if staged else None,
        "split": ({"tokens_per_range": plans[0].tokens_per_range, "ranges_per_batch": plans[0].n_items}
                  if split else None),
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
    }


# ── copy / zero sweep ────────────────────────────────────────────────────────
def sweep_case(args) -> None:
    """Batched copy and zero over disjoint random pairs of a Llama-3-8B-shaped
    pool of --blocks blocks (sweep_figure), beside the reference's GPU path
    without Triton (one dst.copy_(src) per pair)."""
    import torch

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    n_blocks, bs, L, H, D, _ = W.LLAMA3_8B_GEOMETRY
    n_blocks = args.blocks
    pool = torch.empty((n_blocks, L, 2, H, bs, D), dtype=torch.bfloat16, device=dev)
    pool.normal_(generator=torch.Generator(device=dev).manual_seed(3))
    bpb = L * 2 * H * bs * D * 2
    out = {"case": "copy_zero_sweep", "variant": args.variant}
    out.update(sweep_figure(pool, bpb, [int(x) for x in args.batches.split(",")], args.rotations, args.steps,
                            args.warmup, variant=args.variant, torch_path=True))
    print(json.dumps(out), flush=True)


def layers_case(args) -> None:
    """Batched block copies on vLLM's per-layer cache layout at the
    Llama-3-8B shape: 32 layers, each one [2, N, 16, 8, 128] bf16 tensor
    (K and V), so a 2 MiB block is 64 spans of 32 KiB in 64 tensors; the
    blocks_to_copy pairs go to kernels.copy_blocks_vllm (one launch)."""
    import torch

    from agentkv_b200 import kernels as K

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _, bs, L, H, D, _ = W.LLAMA3_8B_GEOMETRY
    n_blocks = min(args.blocks, 30_000)
    gen = torch.Generator(device=dev).manual_seed(5)
    kv = []
    for _ in range(L):
        t = torch.empty((2, n_blocks, bs, H, D), dtype=torch.bfloat16, device=dev)
        t.normal_(generator=gen)
        kv.append(t)
    keys, values = [t[0] for t in kv], [t[1] for t in kv]
    bpb = L * 2 * bs * H * D * 2
    peak, peak_kind = measured_peak()
    out = {"case": "vllm_layer_caches", "variant": args.variant, "layers": L, "cache_blocks": n_blocks, "bytes_per_block": bpb,
           "span_bytes": bpb // (2 * L), "peak_gbs": peak, "peak_source": peak_kind, "batches": {}}
    for n in [int(x) for x in args.batches.split(",")]:
        if 2 * n > n_blocks:
            continue
        sets = [torch.from_numpy(W.copy_sweep_pairs(n, n_blocks, rotation=r)).to(dev)
                for r in range(args.rotations)]
        for i in range(args.warmup):
            K.copy_blocks_vllm(keys, values, sets[i % len(sets)], variant=args.variant)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            K.copy_blocks_vllm(keys, values, sets[i % len(sets)], variant=args.variant)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        K.raise_for_status(K._status_buffer(dev))
        gbs = 2 * bpb * n / (ms / 1e3) / 1e9
        out["batches"][str(n)] = {"copy_ms": round(ms, 5), "copy_gbs": round(gbs, 1),
                                  "copy_frac": round(gbs / peak, 4)}
    print(json.dumps(out), flush=True)


def hf_case(args) -> None:
    """The HF cache's per-layer K/V assembly at the Llama-3-8B shape: a
    4096-token sequence in 256 blocks scattered over a pool of up to 4096
    (--blocks), all 32 layers (one decode
    step's gathers), kernels.kv_gather against the reference's GPU path for
    the same result (indexing gather, permute, reshape, truncation)."""
    import torch

    from agentkv_b200 import kernels as K

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _, bs, L, H, D, _ = W.LLAMA3_8B_GEOMETRY
    n_blocks, n_tok = max(320, min(args.blocks, 4096)), 4096  # room for the decode steps' new blocks
    pool = torch.empty((n_blocks, L, 2, H, bs, D), dtype=torch.bfloat16, device=dev)
    pool.normal_(generator=torch.Generator(device=dev).manual_seed(7))
    rng = np.random.default_rng(7)
    tables = [torch.from_numpy(rng.permutation(n_blocks)[: n_tok // bs].astype(np.int32)).to(dev)
              for _ in range(4)]
    tables_l = [t.long() for t in tables]

    def ours(i):
        for layer in range(L):
            K.kv_gather(pool, tables[i % 4], layer, n_tok)

    def torch_path(i):
        for layer in range(L):
            data = pool[tables_l[i % 4], layer]
            k = data[:, 0].permute(1, 0, 2, 3).reshape(1, H, -1, D)[:, :, :n_tok]
            v = data[:, 1].permute(1, 0, 2, 3).reshape(1, H, -1, D)[:, :, :n_tok]
            del k, v

    k0, v0 = K.kv_gather(pool, tables[0], 5, n_tok)
    data = pool[tables_l[0], 5]
    assert torch.equal(k0, data[:, 0].permute(1, 0, 2, 3).reshape(1, H, -1, D))
    assert torch.equal(v0, data[:, 1].permute(1, 0, 2, 3).reshape(1, H, -1, D))
    res = {}
    for name, fn in (("kv_gather", ours), ("torch_index_permute", torch_path)):
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        alg = 2 * 2 * H * n_tok * D * 2 * L  # read + write of K and V, all layers
        res[name] = {"ms_per_decode_step": round(ms, 4), "us_per_layer": round(ms * 1e3 / L, 2),
                     "gbs_algorithmic": round(alg / (ms / 1e3) / 1e9, 1)}
    peak, peak_kind = measured_peak()
    res["kv_gather"]["frac"] = round(res["kv_gather"]["gbs_algorithmic"] / peak, 4)
    res["kv_gather"]["timing"] = "events around the host loop of 32 calls (launch-bound)"
    # the kernels alone: the 32 layers' gathers of each table recorded as a
    # CUDA graph, the 4 graphs (tables) replayed in turn
    graphs = []
    for i in range(4):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            ours(i)
        graphs.append(g)
    for g in graphs:
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(args.steps, 20)
    e0.record()
    for i in range(reps):
        graphs[i % 4].replay()
    e1.record()
    torch.cuda.synchronize()
    ms_g = e0.elapsed_time(e1) / reps
    alg = 2 * 2 * H * n_tok * D * 2 * L
    res["kv_gather_kernels"] = {"ms_per_decode_step": round(ms_g, 4), "us_per_layer": round(ms_g * 1e3 / L, 2),
                                "gbs_algorithmic": round(alg / (ms_g / 1e3) / 1e9, 1),
                                "frac": round(alg / (ms_g / 1e3) / 1e9 / peak, 4),
                                "timing": "32 launches per CUDA graph replay, 4 tables in turn (device time)"}
    del graphs
    del pool
    res["update_e2e"] = hf_update_figure(n_blocks, n_tok, args.steps, args.warmup)
    res["update_e2e_append_only"] = hf_update_figure(n_blocks, n_tok, args.steps, args.warmup, append_only=True)
    res["update_reference_torch_path"] = hf_reference_update_figure(n_blocks, n_tok, args.steps, args.warmup)
    res["update_speedup_vs_reference_torch_path"] = round(
        res["update_reference_torch_path"]["ms_per_decode_step"] / res["update_e2e"]["ms_per_decode_step"], 2)
    res["update_speedup_note"] = ("the torch arm times the reference's row writes and indexed gather only; "
                                  "update_e2e also includes the pool calls (block allocation, the "
                                  "copy-on-write check, the block tables), so the ratio understates ours")
    print(json.dumps({"case": "hf_cache_gather", "tokens": n_tok, "layers": L, "heads": H, "head_dim": D,
                      "peak_gbs": peak, "peak_source": peak_kind, **res,
                      "speedup": round(res["torch_index_permute"]["ms_per_decode_step"] /
                                       res["kv_gather"]["ms_per_decode_step"], 2)}), flush=True)


def hf_update_figure(n_blocks: int, n_tok: int, steps: int, warmup: int, append_only: bool = False) -> dict:
    """Decode steps through the public call, AgentKVCache.update on every
    layer (block allocation and copy-on-write checks on layer 0, the new
    token's rows written, the layer's K/V assembled): an agent forked from a
    committed n_tok-token prompt held as a 16-node shared chain, one new
    token per step, host logic included."""
    import torch

    from agentkv_b200 import AgentKVPool, PoolConfig
    from agentkv_b200.hf_cache import AgentKVCache

    dev = torch.device("cuda", torch.cuda.current_device())
    _, bs, L, H, D, _ = W.LLAMA3_8B_GEOMETRY
    pool = AgentKVPool(config=PoolConfig(total_blocks=n_blocks, block_size=bs, num_layers=L, num_kv_heads=H,
                                         head_dim=D, dtype="bfloat16", device="cuda"))
    root = pool.create_root(list(range(n_tok)))
    pool.allocate_blocks(root, n_tok // bs)
    for _ in range(16):
        pool.commit_prefix(root, n_tok // 16)
    cache = AgentKVCache(pool, pool.fork(root), append_only=append_only)
    k = torch.randn((1, H, 1, D), generator=torch.Generator(device=dev).manual_seed(8), device=dev,
                    dtype=torch.float32).to(torch.bfloat16)

    def step():
        for layer in range(L):
            cache.update(k, k, layer)

    for _ in range(max(3, warmup)):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) / steps
    ms = e0.elapsed_time(e1) / steps
    return {"ms_per_decode_step": round(ms, 4), "us_per_layer": round(ms * 1e3 / L, 2),
            "host_wall_ms_per_step": round(wall * 1e3, 4), "tokens_at_start": n_tok,
            "api": f"AgentKVCache.update(append_only={append_only}), every layer, one new token per step"}


def hf_reference_update_figure(n_blocks: int, n_tok: int, steps: int, warmup: int) -> dict:
    """The data movement of the reference's AgentKVCache.update on the GPU,
    restated in torch (agentkv/hf_cache.py:100-153): per layer, the new
    token's K and V rows written by indexed assignment, then the layer's
    blocks gathered by advanced indexing, permuted, reshaped and cut to the
    sequence length — one new token per step on an n_tok-token agent, the
    same pool and table shape as hf_update_figure (its pool calls excluded)."""
    import torch

    dev = torch.device("cuda", torch.cuda.current_device())
    _, bs, L, H, D, _ = W.LLAMA3_8B_GEOMETRY
    pool = torch.zeros((n_blocks, L, 2, H, bs, D), dtype=torch.bfloat16, device=dev)
    rng = np.random.default_rng(9)
    ids = rng.permutation(n_blocks)[: n_tok // bs + 8].tolist()
    k = torch.randn((1, H, 1, D), generator=torch.Generator(device=dev).manual_seed(9), device=dev,
                    dtype=torch.float32).to(torch.bfloat16)
    state = {"seen": n_tok}

    def step():
        seen = state["seen"]
        nxt = seen + 1
        table = torch.tensor(ids[: -(-nxt // bs)], dtype=torch.long, device=dev)
        b, pos = ids[seen // bs], seen % bs
        for layer in range(L):
            pool[b, layer, 0, :, pos, :] = k[0, :, 0, :]
            pool[b, layer, 1, :, pos, :] = k[0, :, 0, :]
            data = pool[table, layer]
            out_k = data[:, 0].permute(1, 0, 2, 3).reshape(1, H, -1, D)[:, :, :nxt]
            out_v = data[:, 1].permute(1, 0, 2, 3).reshape(1, H, -1, D)[:, :, :nxt]
            del out_k, out_v
        state["seen"] = nxt if nxt < n_tok + 100 else n_tok

    for _ in range(max(3, warmup)):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return {"ms_per_decode_step": round(ms, 4), "us_per_layer": round(ms * 1e3 / L, 2),
            "api": "torch restatement of the reference's per-layer row writes + indexed gather"}


def copy_kernel_name(pool, variant: int) -> str:
    """What the copy launches of the step run, for the config record."""
    from agentkv_b200 import _native as N
    from agentkv_b200 import kernels as K

    v = K.claimed_variant(pool) if variant == N.VARIANT_AUTO else variant
    bpb = pool[0].numel() * pool.element_size()
    if v == N.VARIANT_CLAIMED_32K:
        return "k_copy_bulk 32 KiB x 6 per SM, items claimed 128 KiB at a time"
    if v == N.VARIANT_CLAIMED_16K:
        return "k_copy_bulk 16 KiB x 12 per SM, items claimed 128 KiB at a time"
    if v in (N.VARIANT_AUTO, N.VARIANT_BULK):
        return ("k_copy_bulk 16 KiB x 12 per SM, items dealt round robin" if bpb >= (2 << 20)
                else "k_copy_bulk 32 KiB x 6 per SM, items dealt round robin")
    return f"copy variant {v}"


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch,
# from ncu captures of the same launch (constants: they describe the kernel
# as captured, not the run that prints them).
COPY_TRAFFIC_NCU = {
    584: (1319668736, "ncu: the 584-pair Tree-of-Thought copy launch (k_copy_bulk<32768,6,OnePool,0,4>, items "
                      "claimed), 3,200-block pool"),
}
MATCH_TRAFFIC_NCU = {
    2000: (52336896, "ncu: one 4,096-query k_match batch (16-byte verify rounds, one query per CTA) on the "
                     "2,000-sequence stress tree"),
}


# ── ReAct multi-agent trace ──────────────────────────────────────────────────
class _ReActPool:
    """The call set workloads.react_setup / react_step drive: the pool's own
    calls plus residual_len(handle)."""

    def __init__(self, pool) -> None:
        self.pool = pool

    def __getattr__(self, name):
        return getattr(self.pool, name)

    @staticmethod
    def residual_len(h) -> int:
        return len(h.residual_blocks)


class _ReActOracle:
    """The same call set on the oracle (OracleTree over OracleAllocator)."""

    def __init__(self, n_blocks: int, block_size: int, copy_cb) -> None:
        from oracle import oracle as O

        self.alloc = O.OracleAllocator(n_blocks)
        self.tree = O.OracleTree(self.alloc, block_size, copy_cb=copy_cb)

    def __getattr__(self, name):
        return getattr(self.tree, name)

    def allocate_blocks(self, h, n) -> None:
        for _ in range(n):
            self.tree.allocate_block(h)

    def maybe_advance_epoch(self) -> None:
        self.alloc.maybe_advance_epoch()

    @staticmethod
    def residual_len(h) -> int:
        return len(h.residual)


def react_cpu_baseline(spec, heads: int, max_seconds: float) -> dict:
    """The oracle playing the same trace on the host (one thread), each CoW
    copy moving one head slice's bytes between blocks of a 64-block host
    pool (ids taken modulo 64): steps per second over a bounded sample."""
    from oracle import oracle as O

    n_, bs, L, _, D, _ = W.LLAMA3_70B_GEOMETRY
    bpb = L * 2 * heads * bs * D * 2
    host = np.zeros((64, bpb), np.uint8)
    host[:] = np.arange(64, dtype=np.uint8)[:, None]
    copied = [0]

    def copy_cb(src, dst):
        a, b = src % 64, dst % 64
        if a != b:
            O.copy_blocks(host, bpb, np.array([[a, b]], np.int32))
        copied[0] += 1

    api = _ReActOracle(n_, bs, copy_cb)
    root, agents = W.react_setup(api, spec)
    done = 0
    t0 = time.perf_counter()
    for actions in W.react_trace(spec):
        W.react_step(api, root, agents, actions)
        done += 1
        if time.perf_counter() - t0 >= max_seconds:
            break
    secs = time.perf_counter() - t0
    return {"value": round(done / secs, 2), "unit": "steps/s", "cores": 1, "kind": "port",
            "sample": f"{done} of {spec.steps} trace steps ({copied[0]} CoW copies of {bpb} B), {secs:.1f} s",
            "host": host_cpu()}


def percall_timings(api, prompt, query, copy_hook: bool, reps: int, match_fn, free_match=None) -> dict:
    """Median microseconds per call of the reference-facing per-call API on
    `api` (AgentKVPool, or the oracle's tree with the same call set): the
    vLLM adapter's calls (fork, allocate_block, ensure_mutable_block on a
    shared last block, free) and the SGLang adapter's match_prefix.  One
    round: fork the root, allocate a block, copy-on-write the last
    inherited block, look the query up, free the child (and the match's
    handle).  The root keeps 128 residual blocks, so a fork increments 128
    refcounts and the copy-on-write copies a 2 MiB block."""
    times = {k: [] for k in ("fork", "allocate_block", "ensure_mutable_block", "match_prefix", "free")}
    root = api.create_root(prompt)
    need = -(-len(prompt) // 16)
    for _ in range(need):
        api.allocate_block(root)
    api.commit_prefix(root, len(prompt) // 2)  # half the prompt shared, half the root's own blocks
    pc = time.perf_counter
    for i in range(reps + 3):
        t0 = pc()
        child = api.fork(root)
        t1 = pc()
        api.allocate_block(child)
        t2 = pc()
        api.ensure_mutable_block(child, -2)
        t3 = pc()
        h, _ = match_fn(query)
        t4 = pc()
        api.free(child)
        t5 = pc()
        if h is not None and free_match is not None:
            free_match(h)
        if i >= 3:
            for k, (a, b) in zip(times, ((t0, t1), (t1, t2), (t2, t3), (t3, t4), (t4, t5))):
                times[k].append((b - a) * 1e6)
    return {k: round(statistics.median(v), 2) for k, v in times.items()}


def percall_case(args) -> None:
    """Per-call latency of the reference-facing API (the calls the reference's
    vLLM and SGLang adapters make one at a time: fork, allocate_block,
    ensure_mutable_block, match_prefix, free) on a metadata-only pool and on
    a CUDA pool at the Llama-3-8B shape, with and without the copy_block hook
    the vLLM adapter installs, beside the oracle's restatement of the
    reference's per-call path on the host (kind "port": its allocator is the
    C restatement, its tree Python, as the reference's is)."""
    import torch

    from agentkv_b200 import AgentKVPool, PoolConfig
    from oracle import oracle as O

    torch.cuda.set_device(0)
    n_, bs, L, H, D, dt = W.LLAMA3_8B_GEOMETRY
    rng = np.random.default_rng(7)
    prompt = rng.integers(0, 128256, size=4096).tolist()
    query = prompt[:3000] + rng.integers(0, 128256, size=500).tolist()
    reps = max(50, args.steps * 10)
    out = {"case": "percall", "unit": "us per call (median)", "reps": reps,
           "workload": "4096-token root (256 blocks), its first 2048 tokens committed to the tree; per round: "
                       "fork it, allocate a block, copy-on-write the child's last inherited block, match_prefix "
                       "a 3500-token query sharing 3000 tokens with the root, free the child", "pools": {}}
    for name, device, blocks in (("meta", "meta", 60000), ("cuda", "cuda", 1024)):
        for hook in (False, True):
            pool = AgentKVPool(config=PoolConfig(total_blocks=blocks, block_size=bs, num_layers=L, num_kv_heads=H,
                                                 head_dim=D, dtype=dt, device=device))
            pairs = []
            if hook:
                orig = pool._allocator.copy_block

                def record(src, dst, orig=orig):
                    pairs.append((src.block_id, dst.block_id))
                    orig(src, dst)

                pool._allocator.copy_block = record
            tree = pool._tree
            res = percall_timings(pool, prompt, query, hook, reps, tree.match_prefix, free_match=pool.free)
            torch.cuda.synchronize()
            out["pools"][f"{name}{' + copy_block hook' if hook else ''}"] = res
            del pool
    # the reference's per-call path restated on the host: Python tree, C allocator
    oa = O.OracleAllocator(60000)
    ot = O.OracleTree(oa, bs)

    def ofree(h):
        ot.free(h)

    res = percall_timings(ot, prompt, query, False, reps, ot.match_prefix, free_match=ofree)
    # and with the 2 MiB block copies on a host pool, as a device="cpu" pool does them
    bpb = L * 2 * H * bs * D * 2
    host_pool = np.zeros((1024, bpb), np.uint8)
    oa2 = O.OracleAllocator(1024)
    ot2 = O.OracleTree(oa2, bs, copy_cb=lambda s_, d_: np.copyto(host_pool[d_], host_pool[s_]))
    res2 = percall_timings(ot2, prompt, query, False, reps, ot2.match_prefix, free_match=ot2.free)
    out["cpu_baseline"] = {"kind": "port", "cores": 1, "value": res,
                           "sample": f"{reps} rounds on a 60,000-block metadata pool, one host thread",
                           "with_copies": res2, "host": host_cpu()}
    print(json.dumps(out), flush=True)


def react_case(args) -> None:
    """The ReAct multi-agent trace (a 16,384-token shared prefix, 32 agents,
    1,000 steps of forks, CoW tail copies, frees, appends and epoch advances)
    at the Llama-3-70B KV shape (40,000 blocks).  Rank 0 holds the agents'
    block tables on the device (DeviceAgents) and applies
    --react-steps-per-launch trace steps per akv_agent_steps launch; each
    step's copy-on-write pairs (a count + pairs buffer written by that
    launch) are broadcast to every rank, which copies its KV-head slice of
    those blocks (akv_copy_blocks_counted reads the count on the device).  One
    bench step = one trace step; warm-up and timed steps are consecutive
    steps of the trace.  Beside it, `percall`: the same steps through the
    pool's per-call API on a metadata-only pool with the vLLM adapter's
    copy_block hook recording the pairs (rank 0, one GPU)."""
    import torch

    from agentkv_b200 import AgentKVPool, PoolConfig
    from agentkv_b200.agents import DeviceAgents
    from agentkv_b200.sharded import ShardedCopier

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    spec = W.ReActSpec()
    n_, bs, L, H, D, dt = W.LLAMA3_70B_GEOMETRY
    # 8 heads do not fit one GPU (200 GB): one GPU holds the 4-head slice of a 2-GPU run
    heads = H // max(world, 2)
    slice_bytes = L * 2 * heads * bs * D * 2
    pool_slice = torch.empty((n_, L, 2, heads, bs, D), dtype=torch.bfloat16, device=dev)
    copier = ShardedCopier(pool_slice)
    buf = copier.batch_buffer(spec.agents)  # at most one CoW per agent per step
    trace = W.react_trace(spec)
    warmup = max(3, args.warmup)
    steps = max(1, min(args.steps, spec.steps - warmup))
    per_launch = max(1, args.react_steps_per_launch)
    pairs_done = [0]
    state = {"next": 0, "rows": None, "row": 0}

    def meta_pool():
        return AgentKVPool(config=PoolConfig(total_blocks=n_, block_size=bs, num_layers=L, num_kv_heads=H,
                                             head_dim=D, dtype=dt, device="meta"))

    if rank == 0:
        meta = meta_pool()
        root, agents = W.react_setup(_ReActPool(meta), spec)
        dev_agents = DeviceAgents(meta, root, agents)

    def one_step():
        if rank == 0:
            rows = state["rows"]
            if rows is None or state["row"] >= rows.shape[0]:
                i = state["next"]
                state["rows"] = rows = dev_agents.steps(trace[i:i + per_launch], pairs_cap=spec.agents)
                state["next"] = i + rows.shape[0]
                state["row"] = 0
            b = rows[state["row"]]  # this step's count + pairs, written by the launch
            state["row"] += 1
        else:
            b = buf
        copier.share_batch(b)
        copier.copy_batch(b)

    sampler = ClockSampler(local)
    with sampler:
        for _ in range(warmup):
            one_step()
        ms, wall = timed(one_step, steps, 0, world)
    clocks = sampler.summary()
    n_pairs_timed = None
    if rank == 0:
        dev_agents.check()
    cpu = percall = None
    if rank == 0 and world == 1:
        # the per-call pattern on the same trace steps (timed alone, no copies)
        meta2 = meta_pool()
        step_pairs = []
        orig = meta2._allocator.copy_block

        def record(src, dst):
            step_pairs.append((src.block_id, dst.block_id))
            orig(src, dst)

        meta2._allocator.copy_block = record
        api = _ReActPool(meta2)
        root2, agents2 = W.react_setup(api, spec)
        for i in range(warmup):
            W.react_step(api, root2, agents2, trace[i])
        step_pairs.clear()
        t0 = time.perf_counter()
        for i in range(warmup, warmup + steps):
            W.react_step(api, root2, agents2, trace[i])
        pc_s = time.perf_counter() - t0
        n_pairs_timed = len(step_pairs)
        percall = {"value": round(steps / pc_s, 2), "unit": "steps/s", "ms_per_step": round(1e3 * pc_s / steps, 4),
                   "api": "AgentKVPool per-call API (free / fork / ensure_mutable_block / allocate_block / "
                          "maybe_advance_epoch) on a metadata pool, copy_block hook recording the pairs; host "
                          "wall time, no copies"}
        if not args.no_cpu_baseline:
            cpu = react_cpu_baseline(spec, heads, args.cpu_seconds)
    if rank == 0:
        step_ms = ms / steps
        line = {
            "case": "react_70b",
            "metric": "ReAct trace steps/s (32 agents, Llama-3-70B KV)",
            "value": round(steps / (ms / 1e3), 2),
            "unit": "steps/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": warmup,
            "ms_per_step": round(step_ms, 4),
            "higher_is_better": True,
            "scaling": "strong" if world > 1 else None,
            "dtype": "bf16",
            "data": "synthetic (seeded trace; pool contents uninitialised: the copies move bytes, nothing reads "
                    "them)",
            "config": {"workload": "react_70b", "pool_blocks": n_, "heads_per_rank": heads,
                       "bytes_per_block_per_rank": slice_bytes,
                       "parallelism": f"kv-head shard x{world}" if world > 1 else
                                      "single GPU, 4 of 8 KV heads (the full pool is 200 GB)",
                       "trace_steps": f"{warmup}..{warmup + steps - 1} of {spec.steps}",
                       "api": f"DeviceAgents: {per_launch} trace steps per akv_agent_steps launch, each step's "
                              f"pairs broadcast and copied (akv_copy_blocks_counted)"},
            "percall": percall,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "wall_s_timed": round(wall, 3),
        }
        if n_pairs_timed is not None:
            line["cow_pairs_per_step"] = round(n_pairs_timed / steps, 2)
            line["copy_gbs_per_rank"] = round(n_pairs_timed * 2 * slice_bytes / (ms / 1e3) / 1e9, 1)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


# ── main arm ─────────────────────────────────────────────────────────────────
def tot_compulsory_bytes(bench) -> tuple:
    """(compulsory, algorithmic) bytes of one step's copies on this rank:
    compulsory = every distinct source block read once + every destination
    written once (the bytes HBM must move however the copies are scheduled;
    the 8 children of a parent copy the same source), algorithmic = 2 x
    bytes per pair.  Counted from the step's own pair list when the copy is
    one launch, else from the workload's shape."""
    per_tree_pairs = sum(bench.spec.children_per_level())
    if bench.merge and bench.last_pairs is not None:
        p = bench.last_pairs.cpu().numpy()
        n_src = len(np.unique(p[:, 0]))
        n_dst = len(np.unique(p[:, 1]))
        assert n_dst == len(p), "a destination repeats within a step"
    else:
        # every parent of every level is one source: 1 + 8 + 64 per tree
        n_src = bench.trees * sum(bench.spec.fanout ** lvl for lvl in range(bench.spec.levels))
        n_dst = bench.trees * per_tree_pairs
    comp = (n_src + n_dst) * bench.slice_bytes
    alg = 2 * bench.trees * per_tree_pairs * bench.slice_bytes
    return comp, alg, n_src, n_dst


def sweep_figure(pool, bpb: int, batches, rotations: int, steps: int, warmup: int, variant: int = 0,
                 torch_path: bool = False) -> dict:
    """Batched copy and zero over seeded disjoint random (src, dst) pairs of
    `pool` (config 3's pair sets): per batch size, `rotations` distinct pair
    sets cycled so small batches do not stay in L2; CUDA events over `steps`
    launches after `warmup`.  GB/s = (read + write) bytes / time for the copy
    (every pair's blocks are distinct, so these are also its compulsory
    bytes), write bytes / time for the zero.  After timing, the last set's
    destinations are checked equal to their sources (copy) and all zero bits
    (zero)."""
    import torch

    from agentkv_b200 import kernels as K

    dev = pool.device
    n_blocks = pool.shape[0]
    peak, peak_kind = measured_peak()
    out = {"pool_blocks": n_blocks, "bytes_per_block": bpb, "peak_gbs": peak, "peak_source": peak_kind,
           "rotations": rotations, "launches_timed": steps, "batches": {}}
    for n in batches:
        if 2 * n > n_blocks:
            continue
        sets = [torch.from_numpy(W.copy_sweep_pairs(n, n_blocks, rotation=r)).to(dev) for r in range(rotations)]
        dsts = [p_[:, 1].contiguous() for p_ in sets]
        zv = variant if variant <= 2 else 0  # zero has no tuning shapes
        for i in range(warmup):
            K.copy_blocks(pool, sets[i % len(sets)], variant=variant)
            K.zero_blocks(pool, dsts[i % len(dsts)], variant=zv)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            K.copy_blocks(pool, sets[i % len(sets)], variant=variant)
        e1.record()
        torch.cuda.synchronize()
        c_ms = e0.elapsed_time(e1) / steps
        last = sets[(steps - 1) % len(sets)]
        flat = pool.view(n_blocks, -1)
        probe = last[:: max(1, n // 16)].long()
        copied_ok = bool(torch.equal(flat[probe[:, 1]], flat[probe[:, 0]]))
        e0.record()
        for i in range(steps):
            K.zero_blocks(pool, dsts[i % len(dsts)], variant=zv)
        e1.record()
        torch.cuda.synchronize()
        z_ms = e0.elapsed_time(e1) / steps
        zlast = dsts[(steps - 1) % len(dsts)][:: max(1, n // 16)].long()
        zero_ok = bool((flat[zlast].view(torch.int16) == 0).all())
        K.raise_for_status(K._status_buffer(dev))
        c_gbs = 2 * bpb * n / (c_ms / 1e3) / 1e9
        z_gbs = bpb * n / (z_ms / 1e3) / 1e9
        row = {"copy_ms": round(c_ms, 5), "copy_gbs": round(c_gbs, 1), "copy_frac": round(c_gbs / peak, 4),
               "zero_ms": round(z_ms, 5), "zero_gbs": round(z_gbs, 1), "zero_frac": round(z_gbs / peak, 4),
               "copied_equal": copied_ok, "zeroed_all_bits": zero_ok}
        if torch_path:
            # the reference's GPU path without Triton: one dst.copy_(src) per pair
            # (agentkv/core/triton_kernels.py:194-196 via SlabAllocator.copy_block)
            host_sets = [p_.cpu().tolist() for p_ in sets]
            reps = max(1, min(steps, 4096 // n))
            for s_, d_ in host_sets[0]:
                pool[d_].copy_(pool[s_])
            torch.cuda.synchronize()
            e0.record()
            for i in range(reps):
                for s_, d_ in host_sets[i % len(host_sets)]:
                    pool[d_].copy_(pool[s_])
            e1.record()
            torch.cuda.synchronize()
            t_ms = e0.elapsed_time(e1) / reps
            row.update({"torch_per_pair_ms": round(t_ms, 5),
                        "torch_per_pair_gbs": round(2 * bpb * n / (t_ms / 1e3) / 1e9, 1)})
        out["batches"][str(n)] = row
    return out


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return
    if args.case == "sweep":
        sweep_case(args)
        return
    if args.case == "layers":
        layers_case(args)
        return
    if args.case == "hf":
        hf_case(args)
        return
    if args.case == "react":
        react_case(args)
        return
    if args.case == "percall":
        percall_case(args)
        return
    if args.case == "match":
        import torch

        torch.cuda.set_device(local)
        if world > 1:
            import datetime

            torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                                 device_id=torch.device("cuda", local))
        fig = match_figure(args.steps, args.warmup, args.match_seqs, args.match_queries, rank, world,
                           use_runs=bool(args.match_runs),
                           cpu_seconds=0.0 if args.no_cpu_baseline else args.cpu_seconds,
                           chunks=match_chunks_arg(args), split=bool(args.match_split),
                           tokens_per_item=args.match_tokens_per_range, min_seconds=args.match_seconds,
                           staged=bool(args.match_staged), window_tokens=args.match_window_tokens)
        if rank == 0:
            print(json.dumps(fig), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    import torch

    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    plan = args.plan or ("sharded" if world > 1 else "replicated")
    bench = ToTBench(rank, world, args.blocks, args.variant, args.trees, args.heads_per_rank, plan,
                     merge=args.copy_levels == "merged")
    F = max(1, args.fanouts_per_step)
    graph = None
    if not args.no_graph and (world == 1 or args.graph_nccl):
        for _ in range(2):  # load every kernel and settle the allocator pools before capture
            bench.step()
        bench.join()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        # --graph-steps consecutive fan-outs per graph (each fan-out's
        # planning overlaps the previous one's copy) and a one-fan-out graph
        # for the remainder
        gs = max(1, args.graph_steps)
        graph2 = bench.capture(gs) if gs > 1 else None
        marks2 = list(bench.graph_marks)
        graph = bench.capture(1)
        marks1 = list(bench.graph_marks)

        def run_fanouts(n):
            if graph2 is not None:
                for _ in range(n // gs):
                    graph2.replay()
                n %= gs
            for _ in range(n):
                graph.replay()
    else:
        def run_fanouts(n):
            for _ in range(n):
                bench.step()
        graph2 = None
        marks1 = marks2 = []

    def run_steps(n):  # one bench step = F consecutive fan-outs
        run_fanouts(n * F)

    use_graph = graph is not None
    sampler = ClockSampler(local)
    with sampler:
        ms, wall = timed_steps(run_steps, args.steps, args.warmup, world, join=bench.join)
    if bench.alloc is not None:
        # every fan-out frees what it allocated: only the roots remain allocated
        bench.alloc.check()
        st = bench.alloc.stats()
        assert st["allocated_blocks"] == len(bench.root_host), st
        assert st["pending_reclamation"] == 0, st
    clocks = sampler.summary()
    step_ms = ms / args.steps
    fanout_ms = step_ms / F
    # the copy launches of the last timed replay, timed inside the graph
    live_marks = []
    if use_graph:
        gs = max(1, args.graph_steps)
        live_marks = marks2 if (graph2 is not None and (args.steps * F) % gs == 0) else marks1
    live_copy_ms = [a.elapsed_time(b) for a, b in live_marks]

    # copy-kernel roofline: per-launch durations with events on this stream
    bench.copy_events = []
    for _ in range(3):
        bench.step(time_copies=True)
    bench.join()
    torch.cuda.synchronize()
    comp_rank, alg_rank, n_src, n_dst = tot_compulsory_bytes(bench)
    comp_step = comp_rank * world * F  # all ranks, one bench step
    alg_step = alg_rank * world * F
    value_gbs = comp_step / (step_ms / 1e3) / 1e9
    per_level = {}
    for (e0, e1, n) in bench.copy_events:
        per_level.setdefault(n, []).append(e0.elapsed_time(e1))
    peak, peak_kind = measured_peak()
    big = max(per_level)
    big_ms = statistics.mean(per_level[big])
    copy_timing = "events around eager launches"
    alone_ms = None
    if bench.merge and bench.last_pairs is not None:
        # The eager launches above can wait on the host between their start
        # event and the kernel; replaying a graph of the same copy launch back
        # to back keeps the stream busy, so the events bracket device time.
        gc = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gc, capture_error_mode="thread_local"):
            bench.copier.copy(bench.last_pairs, variant=args.variant)
        for _ in range(3):
            gc.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            gc.replay()
        e1.record()
        torch.cuda.synchronize()
        alone_ms = e0.elapsed_time(e1) / 10
        del gc
        if live_copy_ms:
            big_ms = statistics.mean(live_copy_ms)
            copy_timing = (f"events recorded inside the timed CUDA graph around the copy launches of the last "
                           f"timed replay ({len(live_copy_ms)} launches)")
        else:
            big_ms = alone_ms
            copy_timing = "events around 10 back-to-back graph replays of the step's copy launch"
        per_level[big] = [big_ms]
    one_launch = bench.merge and bench.last_pairs is not None
    launch_comp = comp_rank if one_launch else None
    achieved = (launch_comp if one_launch else 2 * bench.slice_bytes * big) / (big_ms / 1e3) / 1e9
    # the constant describes the claimed copy the automatic choice launches
    traffic = (COPY_TRAFFIC_NCU.get(big) if (bench.slice_heads == 8 and bench.trees == 1 and one_launch
                                             and args.variant == 0) else None)

    # per-rank breakdown (every rank takes part in the gather)
    per_rank = None
    if world > 1:
        mine = torch.tensor([step_ms, big_ms, alone_ms or 0.0], dtype=torch.float64, device="cuda")
        allr = [torch.zeros_like(mine) for _ in range(world)]
        torch.distributed.all_gather(allr, mine)
        per_rank = {"fanout_ms": [round(float(t[0]) / F, 4) for t in allr],
                    "copy_launch_ms_in_step": [round(float(t[1]), 4) for t in allr],
                    "copy_launch_ms_alone": [round(float(t[2]), 4) for t in allr]}

    e2e = None
    if not args.no_e2e:
        res = {}
        graph_e2e = bench.plan in ("replicated", "sharded") and use_graph
        if graph_e2e:
            # the public FanoutGraph API: host root tables in, every child's
            # table and the status word back to host memory, one graph replay
            # (under --plan sharded the graph also all-gathers the pair lists)
            from agentkv_b200.fanout import FanoutGraph

            fg = FanoutGraph(bench.alloc, bench.level_lens[0], bench.spec.levels, bench.spec.fanout,
                             bench.spec.appended_blocks, pool=bench.pool, free_children=True,
                             variant=args.variant,
                             copier=bench.copier if bench.plan == "sharded" else None, id_base=bench.id_base)
            roots_np = bench.root_host.numpy()
            res["io"] = (fg.h2d_bytes, fg.d2h_bytes)
            e2e_api = "FanoutGraph.run (one CUDA graph replay and one wait per fan-out)"

            def e2e_fanout():
                fg.run(roots_np, copy=False)
        else:
            e2e_api = "SlabAllocator.fanout_tree + copy_blocks from host tables (eager)"

            def e2e_fanout():
                res["io"] = bench.step(e2e=True)

        pc_fanouts = max(3, min(F * args.steps // 2, 400))
        e_ms, _ = timed(e2e_fanout, pc_fanouts, max(3, args.warmup), world, join=bench.join)
        e_fanout = e_ms / pc_fanouts
        h2d, d2h = res["io"]
        e2e = {"value": round(comp_rank * world / (e_fanout / 1e3) / 1e9, 2), "unit": UNIT,
               "h2d_bytes_per_step": int(h2d) * F, "d2h_bytes_per_step": int(d2h) * F,
               "ms_per_step": round(e_fanout * F, 4), "api": e2e_api,
               "fanouts_timed": pc_fanouts}
        if graph_e2e and not args.no_pipeline:
            # the same fan-outs through FanoutGraph.run_many: two recorded
            # instances of --graph-steps fan-outs each alternate, so the host's
            # read-back of one replay and its relaunch hide behind the other's
            # replay, and inside a replay each fan-out's planning overlaps the
            # previous copy (each fan-out still copies its roots in from pinned
            # memory and its tables back to the host, where the host reads them)
            seen = [0]
            k_rep = max(1, args.graph_steps)

            def on_result(i, tables):
                seen[0] += int(tables[-1] >= 0)

            try:
                fg.run_many([roots_np] * (2 * k_rep + 1), per_replay=k_rep)  # records the instances, warms up
                n_many = args.steps * F
                p_ms, _ = timed(lambda: fg.run_many([roots_np] * n_many, on_result=on_result, per_replay=k_rep),
                                1, 0, world, join=bench.join)
                p_fanout = p_ms / n_many
                assert seen[0] == n_many, seen
                e2e["per_call"] = {k: e2e[k] for k in ("value", "ms_per_step", "api", "fanouts_timed")}
                e2e.update({"value": round(comp_rank * world / (p_fanout / 1e3) / 1e9, 2),
                            "ms_per_step": round(p_fanout * F, 4), "fanouts_timed": n_many,
                            "api": f"FanoutGraph.run_many ({n_many} fan-outs in one call, two graph "
                                   f"instances of {k_rep} fan-outs alternating)"})
            except Exception as exc:  # noqa: BLE001 - the per-call figure stands; say why
                e2e["pipelined_error"] = repr(exc)[:200]
        if graph_e2e:
            torch.cuda.synchronize()
            fg = None  # its graphs (with NCCL calls under --plan sharded) go before the process group

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, n_fan, secs, bpb, threads, gbs_alg = cpu_tot_run(1, 1000, 1, 0, max_seconds=args.cpu_seconds)
        cpu = {"value": round(gbs, 3), "unit": UNIT, "cores": threads, "kind": "port",
               "algorithmic_gbs": round(gbs_alg, 3),
               "sample": f"{n_fan} Tree-of-Thought fan-outs ({n_fan * 584} CoW copies of {bpb} B) on a "
                         f"4096-block host pool, {secs:.1f} s; GB/s on the same compulsory bytes as the "
                         f"GPU figure", "host": host_cpu()}

    sweep = None
    if world == 1 and not args.no_sweep:
        n_, bs, L, H, D, _ = W.LLAMA3_8B_GEOMETRY
        sweep = sweep_figure(bench.pool, bench.slice_bytes, [512, 4096], args.rotations, 20, 3,
                             variant=args.variant)
        sweep["workload"] = "copy_zero_sweep_8b (seeded disjoint pairs on the same 60,000-block pool)"

    match = None
    if rank == 0 and world == 1 and not args.no_match:
        del graph, graph2
        graph = graph2 = None
        torch.cuda.synchronize()
        match = match_figure(args.warmup, args.warmup, args.match_seqs, args.match_queries,
                             cpu_seconds=0.0 if args.no_cpu_baseline else args.cpu_seconds,
                             chunks=match_chunks_arg(args), split=bool(args.match_split),
                             tokens_per_item=args.match_tokens_per_range, min_seconds=args.match_seconds,
                           staged=bool(args.match_staged), window_tokens=args.match_window_tokens)

    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    del graph, graph2, run_steps, run_fanouts  # a graph holding NCCL calls must go before the process group
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value_gbs, 2),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(step_ms, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded token ids, seeded N(0,1) pool contents)",
            "config": {
                "workload": "tot_8b_fanout",
                "pool_blocks": bench.n_blocks,
                "fanouts_per_step": F,
                "trees_per_fanout": bench.trees,
                "bytes_per_block": bench.slice_bytes * world,
                "cow_copies_per_fanout": sum(bench.pairs_per_level),
                "bytes_counted": (f"compulsory: {n_src} distinct source blocks read once + {n_dst} destination "
                                  f"blocks written per fan-out and rank ({comp_rank} B); the per-pair figure "
                                  f"(2 x bytes_per_block per pair, {alg_rank} B) is algorithmic_gbs"),
                "parallelism": f"kv-head shard x{world}" if world > 1 else "single GPU",
                "pair_lists": bench.plan if world > 1 else "local",
                "heads_per_rank": bench.slice_heads,
                "l2": "inputs larger than L2 (each fan-out touches ~1.4 GB per GPU)",
                "copy_variant": args.variant,
                "copy_kernel": copy_kernel_name(bench.pool, args.variant),
                "copy_levels": "merged" if bench.merge else "per-level",
                "cuda_graph": use_graph,
                "fanouts_per_graph": max(1, args.graph_steps) if use_graph else None,
            },
            "algorithmic_gbs": round(alg_step / (step_ms / 1e3) / 1e9, 2),
            "fanout_ms": round(fanout_ms, 5),
            "roofline": {
                "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic[0] if traffic else None,
                "traffic_source": traffic[1] if traffic else None,
                "kernel": f"akv copy_blocks (k_copy_bulk), {big}-pair launch", "peak_source": peak_kind,
                "launch_timing": copy_timing,
                "launch_ms": round(big_ms, 4),
                "launch_ms_alone": round(alone_ms, 4) if alone_ms else None,
                "compulsory_bytes_per_launch": launch_comp,
                "algorithmic_bytes_per_launch": 2 * bench.slice_bytes * big,
                "algorithmic_gbs": round(2 * bench.slice_bytes * big / (big_ms / 1e3) / 1e9, 1),
                "dram_gbs": round(traffic[0] / (big_ms / 1e3) / 1e9, 1) if traffic else None,
                "per_level_ms": {str(k): round(statistics.mean(v), 4) for k, v in sorted(per_level.items())},
                "note": "achieved = compulsory bytes (distinct sources + destinations) / launch time; the 8 "
                        "children of a parent copy one source, so L2 serves 7 of 8 source reads and the "
                        "algorithmic per-pair figure exceeds the HBM peak",
            },
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": bench.launches_per_step * F * args.steps,
            "clocks": clocks,
            "wall_s_timed": round(wall, 3),
        }
        if per_rank is not None:
            line["per_rank"] = per_rank
        if sweep is not None:
            line["sweep"] = sweep
        if match is not None:
            line["match_prefix"] = match
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
