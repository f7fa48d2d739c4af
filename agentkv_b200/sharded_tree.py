"""Replicas of the shared radix tree on every GPU of a node, so that
match_prefix queries spread over the ranks.

Rank `src` owns the tree (the DualRadixTree of its pool).  Its device replica
records every change as a delta (DeviceTree.take_delta); `TreeReplicaSync`
broadcasts each delta over the process group — NCCL over NVLink on GPUs —
and every rank applies it to its own DeviceTree with akv_tree_apply, so all
replicas hold identical arrays and each rank answers its queries locally
(akv_match_prefix), with no exchange per query.

Wire format of one delta: an int64 header
    [kind, n_tokens, tok_lo, token_cap, node_cap, slot_cap, n_slot_rows, n_node_rows,
     run_nodes, n_runs]
(kind -1 = nothing changed, 0 = incremental, 1 = full, 2 = commands), then,
skipping empty arrays, for a full delta tokens[n_tokens] i32,
edge_off[node_cap] i64, edge_len[node_cap] i32, slots[slot_cap x 4] i32; for
an incremental one the appended tokens[n_tokens - tok_lo] i32, slot rows
[n x 5] i32 and node rows [n x 3] i64; for commands (every change since the
last share was one of the host tree's inserts or prunes, and nothing was
resized) the command records [n x 8] i64 and their tokens i32 (the
n_slot_rows / n_node_rows fields carry their counts), which every replica
applies itself with akv_tree_commands — a commit then travels as its tokens
and a few ids instead of the rows it changed.  When the owner's unary-chain runs were rebuilt since the last
share (run_nodes >= 0), run_head[run_nodes] i32 and run entries
[n_runs x 4] i32 follow, sent straight from the owner's device arrays; a
replica whose tree changed without new runs drops its runs and matches with
the hash table alone.
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from .device_tree import DeviceTree

KIND_NONE, KIND_INCREMENTAL, KIND_FULL, KIND_COMMANDS = -1, 0, 1, 2


class TreeReplicaSync:
    def __init__(self, tree: DeviceTree, group=None, src: int = 0) -> None:
        """`tree`: the owner's DeviceTree on rank src, an empty DeviceTree (the
        replica) on every other rank."""
        import torch.distributed as dist

        self.tree = tree
        self.device = tree.device
        self.group = group
        self.src = src
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self._sent_runs = 0  # the owner's runs_version last sent
        if self.rank == src:
            tree.track_peers()
        else:
            tree.as_replica()

    def _bcast(self, t: torch.Tensor) -> None:
        import torch.distributed as dist

        if self.world > 1 and t.numel():
            dist.broadcast(t, src=self.src, group=self.group)

    def share(self, runs: bool = True) -> Optional[dict]:
        """Collective: rank src takes its pending delta and sends it; every
        rank returns the delta with its arrays as tensors on its device (None
        when nothing changed).  With runs=True the owner rebuilds its stale
        unary-chain runs when DeviceTree.want_runs says a rebuild pays (or
        the caller built them) and sends them when they changed since the
        last share (keys "run_head" / "runs" of the result)."""
        dev = self.device
        send_runs = None
        if self.rank == self.src:
            d = self.tree.take_commands(peers=True) if self.tree.device_commands else None
            if d is None:
                self.tree._peers.drop_commands()
                d = self.tree.take_delta(peers=True)
            if d is None:
                head = [KIND_NONE, self.tree.n_tokens, self.tree.n_tokens, 0, 0, 0, 0, 0]
            elif "commands" in d:
                head = [KIND_COMMANDS, d["n_tokens"], d["tok_lo"], 0, 0, 0, len(d["commands"]), len(d["payload"])]
            elif d["full"]:
                head = [KIND_FULL, d["n_tokens"], 0, d["token_cap"], len(d["off"]), len(d["slots"]), 0, 0]
            else:
                head = [KIND_INCREMENTAL, d["n_tokens"], d["tok_lo"], 0, 0, 0, len(d["su"]), len(d["nu"])]
            if runs and self.tree.want_runs():
                self.tree.build_runs()
            if runs and self.tree.d_run_head is not None and self.tree.runs_version != self._sent_runs:
                send_runs = (self.tree.d_run_head, self.tree.d_runs)
                head += [send_runs[0].numel(), send_runs[1].shape[0]]
                self._sent_runs = self.tree.runs_version
            else:
                head += [-1, 0]
            hdr = torch.tensor(head, dtype=torch.int64, device=dev)
        else:
            d = None
            hdr = torch.empty(10, dtype=torch.int64, device=dev)
        self._bcast(hdr)
        kind, n_tok, tok_lo, tok_cap, node_cap, slot_cap, n_su, n_nu, run_nodes, n_runs = \
            (int(x) for x in hdr.cpu())
        run_arrays = {}
        if run_nodes >= 0:
            rh, re_ = send_runs if send_runs is not None else (
                torch.empty(run_nodes, dtype=torch.int32, device=dev),
                torch.empty((n_runs, 4), dtype=torch.int32, device=dev))
            self._bcast(rh)
            self._bcast(re_)
            run_arrays = {"run_head": rh, "runs": re_}
        if kind == KIND_NONE:
            if not run_arrays:
                return None
            # new runs of an unchanged tree: an empty incremental delta carries them
            empty = torch.empty(0, dtype=torch.int32, device=dev)
            return {"full": False, "n_tokens": n_tok, "tok_lo": tok_lo, "tokens": empty,
                    "su": empty.view(0, 5), "nu": empty.to(torch.int64).view(0, 3), **run_arrays}
        if kind == KIND_COMMANDS:
            out = {"n_tokens": n_tok, "tok_lo": tok_lo}
            for name, n, dtype in (("commands", n_su * 8, torch.int64), ("payload", n_nu, torch.int32)):
                if d is not None:
                    t = torch.from_numpy(np.ascontiguousarray(d[name]).reshape(-1)).to(dev, dtype=dtype)
                else:
                    t = torch.empty(n, dtype=dtype, device=dev)
                self._bcast(t)
                out[name] = t
            out["commands"] = out["commands"].view(-1, 8)
            out.update(run_arrays)
            return out
        if kind == KIND_FULL:
            spec = [("tokens", n_tok, torch.int32), ("off", node_cap, torch.int64),
                    ("len", node_cap, torch.int32), ("slots", slot_cap * 4, torch.int32)]
        else:
            spec = [("tokens", n_tok - tok_lo, torch.int32), ("su", n_su * 5, torch.int32),
                    ("nu", n_nu * 3, torch.int64)]
        out = {"full": kind == KIND_FULL, "n_tokens": n_tok, "tok_lo": tok_lo, "token_cap": tok_cap}
        for name, n, dtype in spec:
            if d is not None:
                t = torch.from_numpy(np.ascontiguousarray(d[name]).reshape(-1)).to(dev, dtype=dtype)
            else:
                t = torch.empty(n, dtype=dtype, device=dev)
            self._bcast(t)
            out[name] = t
        if kind == KIND_INCREMENTAL:
            out["su"] = out["su"].view(-1, 5)
            out["nu"] = out["nu"].view(-1, 3)
        out.update(run_arrays)
        return out

    def sync(self, runs: bool = True) -> None:
        """Collective: bring every rank's device replica (and, with runs=True,
        its unary-chain runs) up to date with the owner's tree."""
        d = self.share(runs)
        if d is None:
            return
        if "commands" in d:
            if self.rank == self.src:
                self.tree.flush()  # the owner's own arrays: its local commands (never applied twice)
            else:
                self.tree.apply_commands(d)
        else:
            self.tree.apply_delta(d)  # rows are idempotent: the owner may apply them again
        if self.rank != self.src and "run_head" in d:
            self.tree.set_runs(d["run_head"], d["runs"])


def query_range(n_queries: int, rank: int, world: int) -> tuple:
    """Rank `rank`'s contiguous share [lo, hi) of a batch of n_queries."""
    base, extra = divmod(n_queries, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def match_split(sync: TreeReplicaSync, queries, block_size: int, *, gather: bool = True):
    """One batch spread over the ranks: each rank matches its contiguous range
    on its own replica; with gather=True (a collective) every rank returns
    the whole batch's (node ids, match lengths), else its own range's.  On
    the owner's rank the lookup runs on the owner's DeviceTree directly:
    call it where the pool's tree is not being changed by another thread
    (between commits, as after sync())."""
    import torch.distributed as dist

    from .device_tree import match_batch

    lo, hi = query_range(len(queries), sync.rank, sync.world)
    node, mlen = match_batch(sync.tree, queries[lo:hi], block_size)
    if not gather or sync.world == 1:
        return node, mlen
    dev = sync.device
    width = query_range(len(queries), 0, sync.world)[1]  # the largest share
    mine = torch.full((2, width), -1, dtype=torch.int32, device=dev)
    mine[0, : hi - lo] = torch.from_numpy(node).to(dev)
    mine[1, : hi - lo] = torch.from_numpy(mlen).to(dev)
    parts = [torch.empty_like(mine) for _ in range(sync.world)]
    dist.all_gather(parts, mine, group=sync.group)
    out_n, out_l = [], []
    for r, p in enumerate(parts):
        a, b = query_range(len(queries), r, sync.world)
        p = p.cpu().numpy()
        out_n.append(p[0, : b - a])
        out_l.append(p[1, : b - a])
    return np.concatenate(out_n), np.concatenate(out_l)
