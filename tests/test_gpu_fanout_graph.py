"""FanoutGraph (a Tree-of-Thought fan-out replayed as one CUDA graph) against
the oracle's per-child sequence.

The oracle runs the reference's calls child by child — fork, then
ensure_mutable_block(child, -1) copying the shared block, then `append`
allocate_block calls, level after level — and frees every child in creation
order.  After every replay the returned child tables, the refcounts, the
free list, the reclaimer queues and counters, and the pool bytes must equal
the oracle's.  The Llama-3-8B Tree-of-Thought case is also checked against
the reference's own recorded fan-out.
"""

import json

import numpy as np
import pytest
import torch

from agentkv_b200 import AgentKVPool, PoolConfig
from agentkv_b200 import workloads as W
from agentkv_b200.fanout import FanoutGraph
from oracle import oracle as O

from test_gpu_alloc import assert_same_as_oracle

pytestmark = pytest.mark.gpu


def _oracle_fanout(tree, roots, levels, fanout, append, free):
    parents, made = roots, []
    for _ in range(levels):
        kids = []
        for p in parents:
            for _ in range(fanout):
                c = tree.fork(p)
                tree.ensure_mutable_block(c, -1)
                for _ in range(append):
                    tree.allocate_block(c)
                kids.append(c)
        made += kids
        parents = kids
    tables = np.concatenate([np.asarray(c.residual, np.int32) for c in made])
    if free:
        for c in made:
            tree.free(c)
    return tables


@pytest.mark.parametrize("merge", [True, False])
@pytest.mark.parametrize("free", [True, False])
@pytest.mark.parametrize("root_lens,levels,fanout,append", [
    ([3, 5], 2, 3, 2),
    ([1], 3, 4, 0),
    ([2, 1, 4], 1, 5, 1),
])
def test_fanout_graph_matches_oracle(root_lens, levels, fanout, append, free, merge):
    n_blocks = 1024
    cfg = PoolConfig(total_blocks=n_blocks, block_size=16, num_layers=2, num_kv_heads=2, head_dim=64,
                     dtype="bfloat16", device="cuda")
    pool = AgentKVPool(config=cfg)
    a = pool._allocator
    a._kv_data.view(torch.int16).random_(-30000, 30000)
    host = a._kv_data.view(torch.uint8).reshape(n_blocks, -1).cpu().numpy().copy()
    bpb = host.shape[1]

    o = O.OracleAllocator(n_blocks, cfg.epoch_interval)
    tree = O.OracleTree(o, 16, copy_cb=lambda s, d: O.copy_blocks(host, bpb, np.array([[s, d]], np.int32)))
    roots = []
    for ln in root_lens:
        h = tree.create_root([])
        for _ in range(ln):
            tree.allocate_block(h)
        roots.append(h)
    d_roots = a.alloc_batch(sum(root_lens)).cpu().numpy()
    want_roots = np.concatenate([np.asarray(h.residual, np.int32) for h in roots])
    np.testing.assert_array_equal(d_roots, want_roots)

    fg = FanoutGraph(a, root_lens, levels, fanout, append, free_children=free, merge=merge)
    assert fg.copies_per_run == len(root_lens) * sum(fanout ** (lv + 1) for lv in range(levels))
    for run in range(3):
        got = fg.run(d_roots)
        want = _oracle_fanout(tree, roots, levels, fanout, append, free)
        np.testing.assert_array_equal(got, want, err_msg=f"tables, run {run}")
        assert_same_as_oracle(a, o, f"run {run}")
        dev = a._kv_data.view(torch.uint8).reshape(n_blocks, -1).cpu().numpy()
        assert np.array_equal(dev, host), f"pool bytes, run {run}"


def test_fanout_graph_tot_8b_reference_fixture(golden_dir):
    """The Llama-3-8B Tree-of-Thought fan-out (a 256-block root forked 8 ways
    for 3 levels, 4 blocks appended per child) equals the reference's
    recorded tables, refcounts and free list; with the frees in the graph,
    every replay returns the refcounts to the reference's freed state and
    follows the oracle's per-child sequence."""
    g = np.load(golden_dir / "tot_8b.npz")
    spec = W.ToTSpec()
    N_, bs, L, H, D, dt = W.LLAMA3_8B_GEOMETRY
    cfg = PoolConfig(total_blocks=N_, block_size=bs, num_layers=L, num_kv_heads=H, head_dim=D, dtype=dt,
                     device="meta")
    a = AgentKVPool(config=cfg)._allocator
    root_len = spec.root_tokens // bs
    roots = a.alloc_batch(root_len).cpu().numpy()
    fg = FanoutGraph(a, [root_len], spec.levels, spec.fanout, spec.appended_blocks)
    np.testing.assert_array_equal(fg.run(roots), g["tables"])
    np.testing.assert_array_equal(a.ref_counts(), g["ref_fanout"])
    np.testing.assert_array_equal(a.free_list(), g["free_fanout"])
    st = json.loads(str(g["stats_fanout"]))
    for k in ("free_blocks", "allocated_blocks", "peak_allocated", "total_allocs", "epoch"):
        assert a.stats()[k] == st[k], k
    a.dec_ref_batch(torch.from_numpy(g["tables"]).to(a.device))
    a.check()
    np.testing.assert_array_equal(a.free_list(), g["free_freed"])

    # with the frees in the graph: the first replay ends in the reference's
    # freed state; later replays (the freed ids now sit at the other end of
    # the free list) follow the oracle's per-child sequence
    a2 = AgentKVPool(config=cfg)._allocator
    roots2 = a2.alloc_batch(root_len).cpu().numpy()
    fg2 = FanoutGraph(a2, [root_len], spec.levels, spec.fanout, spec.appended_blocks, free_children=True)
    o = O.OracleAllocator(N_, cfg.epoch_interval)
    tree = O.OracleTree(o, bs)
    root = tree.create_root([])
    for _ in range(root_len):
        tree.allocate_block(root)
    for run in range(3):
        got = fg2.run(roots2)
        if run == 0:
            np.testing.assert_array_equal(got, g["tables"])
            np.testing.assert_array_equal(a2.free_list(), g["free_freed"])
        want = _oracle_fanout(tree, [root], spec.levels, spec.fanout, spec.appended_blocks, True)
        np.testing.assert_array_equal(got, want, err_msg=f"run {run}")
        np.testing.assert_array_equal(a2.ref_counts(), g["ref_freed"])
        assert_same_as_oracle(a2, o, f"run {run}")


def test_fanout_graph_exhaustion_raises():
    cfg = PoolConfig(total_blocks=40, block_size=4, num_layers=1, num_kv_heads=1, head_dim=4,
                     dtype="float16", device="cuda")
    a = AgentKVPool(config=cfg)._allocator
    roots = a.alloc_batch(2).cpu().numpy()
    fg = FanoutGraph(a, [2], 2, 3, 1)  # 24 blocks per replay, children kept
    fg.run(roots)
    with pytest.raises(MemoryError):
        fg.run(roots)
    with pytest.raises(ValueError):
        fg.run(roots[:1])


@pytest.mark.parametrize("root_lens,levels,fanout,append", [
    ([3, 1, 5, 2], 3, 3, 2), ([1], 4, 2, 1), ([7], 1, 6, 3), ([2, 2], 2, 1, 1),
])
def test_fused_tree_plan_equals_level_plans(root_lens, levels, fanout, append):
    """fanout_tree's one-launch plan (append >= 1) against fanout_level run
    level by level: identical child tables, pairs, refcounts, free lists."""
    def run(per_level):
        cfg = PoolConfig(total_blocks=4096, block_size=16, num_layers=1, num_kv_heads=1, head_dim=8,
                         dtype="float16", device="meta")
        a = AgentKVPool(config=cfg)._allocator
        roots = a.alloc_batch(sum(root_lens))
        if per_level:
            tables, pairs = [], []
            t, lens = roots, np.asarray(root_lens)
            for _ in range(levels):
                off = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)])).to(a.device)
                r = a.fanout_level(t, off, lens, fanout, append)
                tables.append(r["child_tables"])
                pairs.append(r["pairs"])
                t, lens = r["child_tables"], r["child_lens"]
        else:
            r = a.fanout_tree(roots, root_lens, levels, fanout, append)
            tables, pairs = r["child_tables"], r["pairs"]
        a.check()
        return ([t.cpu().numpy() for t in tables], [p.cpu().numpy() for p in pairs],
                a.ref_counts(), a.free_list(), a.stats())

    t1, p1, r1, f1, s1 = run(False)
    t2, p2, r2, f2, s2 = run(True)
    for x, y in zip(t1, t2):
        np.testing.assert_array_equal(x, y)
    for x, y in zip(p1, p2):
        np.testing.assert_array_equal(x.reshape(-1, 2), y.reshape(-1, 2))
    np.testing.assert_array_equal(r1, r2)
    np.testing.assert_array_equal(f1, f2)
    for k in ("free_blocks", "allocated_blocks", "peak_allocated", "total_allocs", "epoch"):
        assert s1[k] == s2[k], k


def test_fanout_edge_cases():
    """No levels, no children, a single level of one child: the graph and
    the allocator behave like the reference's (empty) call sequences."""
    cfg = PoolConfig(total_blocks=64, block_size=4, num_layers=1, num_kv_heads=1, head_dim=4, dtype="float16",
                     device="cuda")
    a = AgentKVPool(config=cfg)._allocator
    roots = a.alloc_batch(2).cpu().numpy()
    before = (a.ref_counts().copy(), a.free_list().copy())
    for levels, fanout in ((0, 3), (2, 0)):
        fg = FanoutGraph(a, [2], levels, fanout, 1, free_children=True)
        assert fg.run(roots).size == 0
        np.testing.assert_array_equal(a.ref_counts(), before[0])
        np.testing.assert_array_equal(a.free_list(), before[1])
    o = O.OracleAllocator(64)
    tree = O.OracleTree(o, 4)
    r = tree.create_root([])
    tree.allocate_block(r)
    tree.allocate_block(r)
    fg = FanoutGraph(a, [2], 1, 1, 1, free_children=False)
    got = fg.run(roots)
    want = _oracle_fanout(tree, [r], 1, 1, 1, False)
    np.testing.assert_array_equal(got, want)
    assert_same_as_oracle(a, o, "one child")
    with pytest.raises(ValueError):
        FanoutGraph(a, [0], 1, 2, 1)


@pytest.mark.parametrize("merge,per_replay", [(True, 1), (False, 1), (True, 3), (False, 2)])
def test_run_many_matches_oracle(merge, per_replay):
    """FanoutGraph.run_many (two recorded instances alternating, each holding
    per_replay fan-outs, the runs left over through one-fan-out instances)
    returns, for each of its runs in order, what the oracle's per-child
    sequence gives, and leaves the allocator, the reclaimer and the pool
    bytes as the oracle leaves them; runs mixed with run() stay in
    sequence."""
    n_blocks, root_lens, levels, fanout, append = 1024, [3, 2], 2, 3, 1
    cfg = PoolConfig(total_blocks=n_blocks, block_size=16, num_layers=2, num_kv_heads=2, head_dim=64,
                     dtype="bfloat16", device="cuda")
    a = AgentKVPool(config=cfg)._allocator
    a._kv_data.view(torch.int16).random_(-30000, 30000)
    host = a._kv_data.view(torch.uint8).reshape(n_blocks, -1).cpu().numpy().copy()
    bpb = host.shape[1]
    o = O.OracleAllocator(n_blocks, cfg.epoch_interval)
    tree = O.OracleTree(o, 16, copy_cb=lambda s, d: O.copy_blocks(host, bpb, np.array([[s, d]], np.int32)))
    roots = []
    for ln in root_lens:
        h = tree.create_root([])
        for _ in range(ln):
            tree.allocate_block(h)
        roots.append(h)
    d_roots = a.alloc_batch(sum(root_lens)).cpu().numpy()
    fg = FanoutGraph(a, root_lens, levels, fanout, append, free_children=True, merge=merge)
    for n_runs in (1, 5, 2, 7):
        got = fg.run_many([d_roots] * n_runs, per_replay=per_replay)
        assert len(got) == n_runs
        for r in range(n_runs):
            want = _oracle_fanout(tree, roots, levels, fanout, append, True)
            np.testing.assert_array_equal(got[r], want, err_msg=f"{n_runs} runs, run {r}")
        got1 = fg.run(d_roots)
        np.testing.assert_array_equal(got1, _oracle_fanout(tree, roots, levels, fanout, append, True))
        assert_same_as_oracle(a, o, f"after {n_runs} runs")
        dev = a._kv_data.view(torch.uint8).reshape(n_blocks, -1).cpu().numpy()
        assert np.array_equal(dev, host)
    with pytest.raises(ValueError, match="root ids"):
        fg.run_many([d_roots[:-1]])
