"""Host-side logic of the KV-head sharded pool with 2 CPU ranks (gloo).

Rank 0 plans a batch of copy-on-write pairs (with the oracle's allocator as
the planner stand-in on CPU), shares it through ShardedCopier.share_pairs,
and each rank applies the pairs to its own head slice (with the oracle's
copy, since the product copy kernel needs a GPU).  Reassembled, the slices
must equal the full pool after the same copies: sharding by head loses
nothing and the broadcast delivers rank 0's exact list.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from agentkv_b200 import sharded as S

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O

        n, L, H, bs, D = 24, 2, 4, 4, 8
        g = torch.Generator().manual_seed(5)
        full = torch.randint(-(2**30), 2**30, (n, L, 2, H, bs, D), dtype=torch.int32, generator=g)
        mine = S.head_slice(full, rank, world).contiguous()
        copier = S.ShardedCopier(mine)
        if rank == 0:
            a = O.OracleAllocator(n)
            a.alloc_batch(8)
            src = np.arange(n - 8, n, dtype=np.int32)
            dst = a.alloc_batch(8)
            pairs = torch.from_numpy(np.stack([src, dst], 1).astype(np.int32))
        else:
            pairs = None
        got = copier.share_pairs(pairs, 8)
        host = mine.numpy().view(np.uint8).reshape(n, -1).copy()
        O.copy_blocks(host, host.shape[1], got.numpy())
        mine_after = torch.from_numpy(host.view(np.int32).reshape(mine.shape))
        parts = [torch.empty_like(mine_after) for _ in range(world)]
        dist.all_gather(parts, mine_after)
        all_pairs = [torch.empty_like(got) for _ in range(world)]
        dist.all_gather(all_pairs, got)
        if rank == 0:
            fhost = full.numpy().view(np.uint8).reshape(n, -1).copy()
            O.copy_blocks(fhost, fhost.shape[1], got.numpy())
            want = torch.from_numpy(fhost.view(np.int32).reshape(full.shape))
            re = torch.cat(parts, dim=3)
            q.put((bool(torch.equal(re, want)), bool(torch.equal(all_pairs[0], all_pairs[1]))))
    finally:
        dist.destroy_process_group()


def _partition_worker(rank, world, port, q):
    """Partitioned planning: each rank plans its own range of block ids with
    an allocator over that range alone; the gathered pairs, in global ids,
    are every rank's pairs in rank order, and every slice takes all of them."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O

        n, L, H, bs, D = 32, 2, 4, 4, 8
        g = torch.Generator().manual_seed(9)
        full = torch.randint(-(2**30), 2**30, (n, L, 2, H, bs, D), dtype=torch.int32, generator=g)
        mine = S.head_slice(full, rank, world).contiguous()
        copier = S.ShardedCopier(mine)
        base, count = S.partition(n, rank, world)
        a = O.OracleAllocator(count)
        roots = a.alloc_batch(3 + rank)  # the ranks' plans differ
        kids = a.alloc_batch(5)
        local = np.stack([np.resize(roots, 5), kids], 1).astype(np.int32)
        out = torch.empty((world * 5, 2), dtype=torch.int32)
        got = copier.gather_pairs(torch.from_numpy(local), base, out)
        everyone = [torch.empty((5, 2), dtype=torch.int32) for _ in range(world)]
        dist.all_gather(everyone, torch.from_numpy(local + base))
        host = mine.numpy().view(np.uint8).reshape(n, -1).copy()
        O.copy_blocks(host, host.shape[1], got.numpy())
        mine_after = torch.from_numpy(host.view(np.int32).reshape(mine.shape))
        parts = [torch.empty_like(mine_after) for _ in range(world)]
        dist.all_gather(parts, mine_after)
        if rank == 0:
            fhost = full.numpy().view(np.uint8).reshape(n, -1).copy()
            O.copy_blocks(fhost, fhost.shape[1], got.numpy())
            want = torch.from_numpy(fhost.view(np.int32).reshape(full.shape))
            in_range = all(((p_ >= r * count) & (p_ < (r + 1) * count)).all() for r, p_ in enumerate(everyone))
            q.put((bool(torch.equal(got, torch.cat(everyone))) and bool(in_range),
                   bool(torch.equal(torch.cat(parts, dim=3), want))))
    finally:
        dist.destroy_process_group()


def _batch_worker(rank, world, port, q, golden):
    """Variable-size batches (count + pairs in one buffer) of the ReAct
    trace's recorded pairs, one broadcast per step."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O

        g = np.load(golden)
        so = g["step_off"][:151]
        n = int(g["pairs"][: so[-1]].max()) + 1
        gen = torch.Generator().manual_seed(6)
        full = torch.randint(-(2**30), 2**30, (n, 1, 2, 4, 2, 4), dtype=torch.int32, generator=gen)
        mine = S.head_slice(full, rank, world).contiguous()
        copier = S.ShardedCopier(mine)
        buf = copier.batch_buffer(32)
        host = mine.numpy().view(np.uint8).reshape(n, -1).copy()
        counts = []
        for i in range(len(so) - 1):
            if rank == 0:
                copier.pack_batch(g["pairs"][so[i]:so[i + 1]], buf)
            copier.share_batch(buf)
            k = int(copier.batch_count(buf)[0])
            counts.append(k)
            O.copy_blocks(host, host.shape[1], copier.batch_pairs(buf)[:k].numpy())
        mine_after = torch.from_numpy(host.view(np.int32).reshape(mine.shape))
        parts = [torch.empty_like(mine_after) for _ in range(world)]
        dist.all_gather(parts, mine_after)
        if rank == 0:
            fhost = full.numpy().view(np.uint8).reshape(n, -1).copy()
            O.copy_blocks(fhost, fhost.shape[1], g["pairs"][: so[-1]])
            want = torch.from_numpy(fhost.view(np.int32).reshape(full.shape))
            q.put((bool(torch.equal(torch.cat(parts, dim=3), want)), counts == np.diff(so).tolist()))
    finally:
        dist.destroy_process_group()


class _HostReplica:
    """What akv_tree_apply does to a replica's arrays, on the host."""

    def __init__(self):
        self.tokens = self.off = self.len = self.slots = None
        self.runs = ()
        self.n = 0

    def apply(self, d):
        if d["full"]:
            self.tokens = np.zeros(int(d["token_cap"]), np.int32)
            self.n = int(d["n_tokens"])
            self.tokens[: self.n] = d["tokens"].numpy()
            self.off = d["off"].numpy().copy()
            self.len = d["len"].numpy().copy()
            self.slots = d["slots"].numpy().reshape(-1, 4).copy()
            return
        lo, hi = int(d["tok_lo"]), int(d["n_tokens"])
        self.tokens[lo:hi] = d["tokens"].numpy()
        self.n = hi
        for r in d["su"].numpy():
            self.slots[r[0]] = r[1:]
        for r in d["nu"].numpy():
            self.off[r[0]] = r[1]
            self.len[r[0]] = r[2]

    def digest(self):
        import hashlib

        h = hashlib.sha256()
        for a in (self.tokens[: self.n], self.off, self.len, self.slots, *self.runs):
            h.update(np.ascontiguousarray(a).tobytes())
        return int.from_bytes(h.digest()[:7], "little")


def _tree_worker(rank, world, port, q):
    """Rank 0 mutates a tree (nodes, edges, child slots, splits, deletions,
    growth and rehash); after every round the deltas reach rank 1, whose
    replica (unary-chain runs included) must equal rank 0's arrays."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from agentkv_b200.device_tree import DeviceTree
        from agentkv_b200.sharded_tree import TreeReplicaSync

        tree = DeviceTree(torch.device("cpu"), node_cap=8, slot_cap=16, token_cap=32)
        sync = TreeReplicaSync(tree)
        rep = _HostReplica()
        rng = np.random.default_rng(9)
        nodes = {0: None}  # node id -> (parent, first token)
        next_id = 1
        ok = True
        for rnd in range(40):
            if rank == 0:
                for _ in range(int(rng.integers(0, 12))):
                    op = rng.integers(0, 10)
                    if op < 6 or len(nodes) < 3:
                        parent = int(rng.choice(list(nodes)))
                        toks = rng.integers(0, 1000, size=int(rng.integers(1, 40)), dtype=np.int32)
                        off = tree.append_tokens(toks)
                        tree.set_node(next_id, off, len(toks))
                        tree.set_child(parent, int(toks[0]), next_id, len(toks))
                        nodes[next_id] = (parent, int(toks[0]))
                        next_id += 1
                    elif op < 8:
                        nid = int(rng.choice([k for k in nodes if k]))
                        o, ln = int(tree.h_off[nid]), int(tree.h_len[nid])
                        if ln > 1:
                            tree.set_node(nid, o + 1, ln - 1)
                    else:
                        nid = int(rng.choice([k for k in nodes if k]))
                        parent, tok = nodes.pop(nid)
                        tree.del_child(parent, tok)
                        tree.clear_node(nid)
            if rank == 0:
                tree.build_runs()  # current runs on every share, so each one travels
            d = sync.share()
            if rank == 0:
                rep.tokens, rep.n = tree.h_tokens, tree.n_tokens
                rep.off, rep.len, rep.slots = tree.h_off, tree.h_len, tree.h_slots
                rep.runs = (tree.d_run_head.numpy(), tree.d_runs.numpy())
            elif d is not None:
                rep.apply(d)
                if "run_head" in d:  # the owner's unary-chain runs, rebuilt after its changes
                    rep.runs = (d["run_head"].numpy().copy(), d["runs"].numpy().copy())
            dig = torch.tensor([rep.digest()], dtype=torch.int64)
            both = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
            dist.all_gather(both, dig)
            ok &= bool(both[0] == both[1])
        if rank == 0:
            q.put((ok, next_id))
    finally:
        dist.destroy_process_group()


def test_tree_replica_deltas_gloo():
    ok, n_nodes = _run(_tree_worker)
    assert n_nodes > 100
    assert ok, "a replica built from the broadcast deltas differs from the owner's arrays"


def _run(target, extra=()):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, WORLD, port, q, *extra)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return q.get(timeout=5)


def test_variable_batches_gloo(golden_dir):
    same_pool, counts_ok = _run(_batch_worker, (str(golden_dir / "react_70b.npz"),))
    assert counts_ok, "receivers decoded other pair counts"
    assert same_pool, "reassembled head slices differ from the unsharded copies"


def test_sharded_pairs_and_slices_gloo():
    same_pool, same_pairs = _run(_worker)
    assert same_pairs, "ranks saw different pair lists"
    assert same_pool, "reassembled head slices differ from the unsharded copy"


def test_partitioned_planning_gloo():
    same_pairs, same_pool = _run(_partition_worker)
    assert same_pairs, "the gathered pairs are not every rank's pairs in rank order, in global ids"
    assert same_pool, "reassembled head slices differ from the unsharded copy of every rank's pairs"


def test_partition_math():
    assert S.partition(120, 0, 2) == (0, 60) and S.partition(120, 1, 2) == (60, 60)
    assert S.partition(480000, 7, 8) == (420000, 60000)
    for bad in ((10, 0, 3), (8, 2, 2), (8, -1, 2)):
        with pytest.raises(ValueError):
            S.partition(*bad)
    copier = S.ShardedCopier(torch.zeros(4, 1, 2, 1, 1, 1))
    with pytest.raises(ValueError):  # out must hold world x n pairs
        copier.gather_pairs(torch.zeros((3, 2), dtype=torch.int32), 0, torch.empty((4, 2), dtype=torch.int32))
    got = copier.gather_pairs(torch.tensor([[1, 2]], dtype=torch.int32), 5, torch.empty((1, 2), dtype=torch.int32))
    assert got.tolist() == [[6, 7]]


def test_head_slicing_math():
    assert S.heads_per_rank(8, 8) == 1 and S.heads_per_rank(8, 2) == 4
    with pytest.raises(ValueError):
        S.heads_per_rank(8, 3)
    assert S.slice_shape(100, 32, 8, 16, 128, 4) == (100, 32, 2, 2, 16, 128)
    full = torch.arange(2 * 1 * 2 * 8 * 1 * 1).reshape(2, 1, 2, 8, 1, 1)
    parts = [S.head_slice(full, r, 4) for r in range(4)]
    assert torch.equal(torch.cat(parts, dim=3), full)


def _match_split_worker(rank, world, port, q):
    """Rank 0 owns a tree built by DualRadixTree's inserts; TreeReplicaSync
    brings rank 1's replica (and the owner's unary-chain runs) up to date
    between insert rounds; match_split spreads a query batch over the ranks
    and all-gathers the answers.  The tree kernels run as their CPU model."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        sys.path.insert(0, os.path.dirname(__file__))
        from agentkv_b200 import _native as N
        from agentkv_b200 import device_tree as DT
        from agentkv_b200 import workloads as W
        from agentkv_b200.allocator import BlockHandle
        from agentkv_b200.config import PoolConfig
        from agentkv_b200.radix_tree import ROOT_NODE_ID, DualRadixTree, SharedNode
        from agentkv_b200.sharded_tree import TreeReplicaSync, match_split
        from oracle import oracle as O
        from test_host_runs import _csr_of
        from tree_kernel_model import TreeKernelModel

        model = TreeKernelModel(N.lib)
        N.lib = model
        DT.stream_handle = lambda dev: 0
        cpu = torch.device("cpu")
        spec = W.MatchSpec(n_prefixes=8, prefix_min=64, prefix_max=192, n_sequences=160, total_min=32,
                           total_max=400, n_queries=75)
        prefixes = W.match_prefixes(spec)
        corpus = W.match_sequences(spec, prefixes)
        queries = W.match_queries(spec, corpus, prefixes, batch=0, n=spec.n_queries)
        if rank == 0:
            tree = object.__new__(DualRadixTree)
            tree._cfg = PoolConfig(total_blocks=64, block_size=16, num_layers=1, num_kv_heads=1, head_dim=1,
                                   dtype="float16", device="meta")
            tree._dev_tree = dt = DT.DeviceTree(cpu, node_cap=8, slot_cap=16, token_cap=64)
            tree._shared_nodes = {ROOT_NODE_ID: SharedNode(ROOT_NODE_ID, -1, dt)}
            dt.set_node(ROOT_NODE_ID, 0, 0)
            tree._next_node_id = 1
        else:
            dt = DT.DeviceTree(cpu)
        sync = TreeReplicaSync(dt)
        ok = True
        for lo in range(0, len(corpus), 40):
            if rank == 0:
                for seq in corpus[lo:lo + 40]:
                    n = (len(seq) // 16) * 16
                    tree._insert_shared_locked(ROOT_NODE_ID, np.asarray(seq[:n], np.int32),
                                               [BlockHandle(b) for b in range(n // 16)])
                dt.build_runs()
            sync.sync()
            node, mlen = match_split(sync, queries, 16)
            if rank == 0:
                flat, q_off = O.pack_queries([x.tolist() for x in queries])
                want = O.match_prefix_csr(_csr_of(tree._shared_nodes), flat, q_off, 16)
                ok &= bool(np.array_equal(mlen, want[1]) and
                           np.array_equal(np.where(mlen > 0, node, -1), np.where(want[1] > 0, want[0], -1)))
        hops = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(hops, torch.tensor([model.run_hops], dtype=torch.int64))
        if rank == 0:
            q.put((ok, [int(h) for h in hops]))
    finally:
        dist.destroy_process_group()


def test_match_split_over_replicas_gloo():
    ok, hops = _run(_match_split_worker)
    assert ok, "match_split over two replicas differs from the oracle's match on the owner's tree"
    assert min(hops) > 100, hops  # both ranks' lookups followed unary-chain runs
