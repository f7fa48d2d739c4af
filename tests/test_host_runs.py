"""The device tree's unary-chain runs and the match path's host side on
CPU: the runs' invariants after random changes and under DualRadixTree's
own inserts (first build in full, then incremental), the rebuild policy,
and — with the tree kernels replaced by their CPU model
(tree_kernel_model.py) — the whole host orchestration of a lookup
(deltas, replica sync, runs) against the oracle's C match."""

import numpy as np
import pytest

from agentkv_b200 import workloads as W
from agentkv_b200.config import PoolConfig


def _check_runs(tree, tag):
    """Every node with exactly one child points at entries that walk its
    unary chain through the first node without exactly one child (each
    entry {child, first token, child's edge length, entries left}); every
    other node points nowhere."""
    head = tree.d_run_head.numpy()
    runs = tree.d_runs.numpy()
    kids = {}
    for (p, t), s in tree._slot_of.items():
        kids.setdefault(p, []).append((int(tree.h_slots[s, 2]), t, int(tree.h_slots[s, 3])))
    assert sum(len(c) == 1 for c in kids.values()) == tree._n_unary, tag
    for u in range(len(head)):
        ch = kids.get(u, [])
        if len(ch) != 1:
            assert head[u] == -1, (tag, u)
            continue
        i, node = int(head[u]), u
        rem = int(runs[i, 3])
        assert rem >= 1 and i + rem <= len(runs), (tag, u)
        for j in range(rem):
            c, t, ln, r = (int(x) for x in runs[i + j])
            assert r == rem - j, (tag, u, j)
            assert kids[node] == [(c, t, ln)], (tag, u, j)
            node = c
        assert len(kids.get(node, [])) != 1, (tag, u)  # the chain ends at a non-unary node
    assert all(u < len(head) for u, c in kids.items() if len(c) == 1), tag


def test_unary_runs_follow_the_chains():
    """DeviceTree.build_runs, first in full and then by rewriting only the
    chains through changed nodes: after every few random changes (new
    children, edge splits that put a node between a parent and its child,
    removed leaves), every node with exactly one child walks its chain and
    no other node has a run; larger change batches take the full build."""
    import torch

    from agentkv_b200.device_tree import DeviceTree

    rng = np.random.default_rng(11)
    for trial in range(6):
        tree = DeviceTree(torch.device("cpu"), node_cap=8, slot_cap=16, token_cap=32)
        nodes = {0: None}  # node -> (parent, first token)
        nxt = 1
        builds = 0
        full = []
        full_runs = tree._full_runs
        tree._full_runs = lambda n: (full.append(n), full_runs(n))
        for step in range(400):
            op = rng.integers(0, 10)
            if op < 5 or len(nodes) < 3:
                parent = int(rng.choice(list(nodes)))
                toks = rng.integers(0, 30, size=int(rng.integers(1, 6)), dtype=np.int32)
                if (parent, int(toks[0])) in tree._slot_of:
                    continue
                tree.set_node(nxt, tree.append_tokens(toks), len(toks))
                tree.set_child(parent, int(toks[0]), nxt, len(toks))
                nodes[nxt] = (parent, int(toks[0]))
                nxt += 1
            elif op < 8:
                # split the edge into child c: parent -> mid -> c
                c = int(rng.choice([k for k in nodes if k]))
                parent, tok = nodes[c]
                ln = int(tree.h_len[c])
                if ln < 2:
                    continue
                k = int(rng.integers(1, ln))
                off = int(tree.h_off[c])
                t2 = int(tree.h_tokens[off + k])
                tree.set_node(nxt, off, k)
                tree.set_node(c, off + k, ln - k)
                tree.set_child(parent, tok, nxt, k)
                tree.set_child(nxt, t2, c, ln - k)
                nodes[nxt] = (parent, tok)
                nodes[c] = (nxt, t2)
                nxt += 1
            else:
                nid = int(rng.choice([k for k in nodes if k]))
                if nid in tree._kids:
                    continue  # only leaves are removed
                parent, tok = nodes.pop(nid)
                tree.del_child(parent, tok)
                tree.clear_node(nid)
            every = 150 if trial == 5 else int(rng.integers(1, 6))  # the last trial: > 64 changes per build
            if step % every == 0:
                tree.build_runs()
                builds += 1
                _check_runs(tree, (trial, step))
        tree.build_runs()
        _check_runs(tree, (trial, "end"))
        assert tree._n_entries >= tree._n_unary
        if trial < 5:
            assert builds > 20 and len(full) == 1  # the first build in full, every later one incremental
        else:
            assert len(full) >= 2  # a batch of more than 64 changed nodes took a full build
        assert not tree._runs_dirty
        tree.set_child(0, 12345, 1, 1)
        assert tree._runs_dirty
    # an empty tree has no runs; child links that loop are refused
    empty = DeviceTree(torch.device("cpu"), node_cap=8, slot_cap=16, token_cap=32)
    empty.build_runs()
    assert (empty.d_run_head.numpy() == -1).all()
    loop = DeviceTree(torch.device("cpu"), node_cap=8, slot_cap=16, token_cap=32)
    for nid in (1, 2):
        loop.set_node(nid, loop.append_tokens(np.array([nid], np.int32)), 1)
    loop.set_child(0, 1, 1, 1)
    loop.set_child(1, 2, 2, 1)
    loop.set_child(2, 1, 1, 1)
    with pytest.raises(RuntimeError, match="cycle"):
        loop.build_runs()
    # a loop made after the first build is refused by the incremental update too
    loop2 = DeviceTree(torch.device("cpu"), node_cap=8, slot_cap=16, token_cap=32)
    for nid in (1, 2):
        loop2.set_node(nid, loop2.append_tokens(np.array([nid], np.int32)), 1)
    loop2.set_child(0, 1, 1, 1)
    loop2.set_child(1, 2, 2, 1)
    loop2.build_runs()
    loop2.set_child(2, 1, 1, 1)
    with pytest.raises(RuntimeError, match="cycle"):
        loop2.build_runs()


def test_run_rebuild_policy():
    """DeviceTree.want_runs: a never-built tree builds; current runs are used;
    after a change the one-probe-per-hop lookups pay rent, the coming one
    counted at the last batch's time, until it reaches the cost of the
    rebuild due (the last incremental one, or the last full one when more
    than 64 nodes changed); every change restarts the count; a replica uses
    runs only while it holds the owner's."""
    import torch

    from agentkv_b200.device_tree import DeviceTree

    t = DeviceTree(torch.device("cpu"), node_cap=8, slot_cap=16, token_cap=32)
    t.set_node(1, t.append_tokens(np.array([5, 6], np.int32)), 2)
    t.set_child(0, 5, 1, 2)
    assert t.want_runs()  # never built
    t.build_runs()
    assert t.want_runs() and t._full_ms is not None
    t._patch_ms = 2.0  # an incremental rebuild costs 2 ms
    t.note_lookup(0.5, True)
    t.set_node(2, t.append_tokens(np.array([7], np.int32)), 1)
    t.set_child(1, 7, 2, 1)
    assert not t.want_runs()  # 0 + 0.5 < 2
    t.note_lookup(0.7, False)
    assert not t.want_runs()  # 0.7 + 0.7 < 2
    t.set_child(1, 8, 2, 1)  # a change: the rent starts over
    t.note_lookup(0.7, False)
    assert not t.want_runs()
    t.note_lookup(0.7, False)
    assert t.want_runs()  # 1.4 + 0.7 >= 2
    t.build_runs()
    assert t.want_runs() and not t._runs_dirty
    t._patch_ms = 0.05  # a cheap incremental rebuild: the next change rebuilds at once
    t.set_child(2, 9, 1, 1)
    assert t.want_runs()
    # a change touching more than 64 nodes needs a full build: priced at the full build's time
    t._full_ms = 50.0
    for p in range(3, 80):
        t.set_child(p, 5, p + 1, 1)
    t.note_lookup(1.0, False)
    assert not t.want_runs()

    r = DeviceTree(torch.device("cpu"), node_cap=8, slot_cap=16, token_cap=32)
    r.as_replica()
    assert not r.want_runs()
    r.set_runs(t.d_run_head, t.d_runs)
    assert r.want_runs()


def test_unary_runs_under_the_tree_insert_logic():
    """The incremental run updates follow DualRadixTree's own inserts —
    children added, edges split on block boundaries with the split node put
    between parent and child, the split==0 overwrite that orphans a subtree,
    exact re-commits — on a CPU device tree: after every few inserts of the
    stress workload's sequences (prefix sharing, block-floored lengths) the
    runs walk every unary chain."""
    import torch

    from agentkv_b200.allocator import BlockHandle
    from agentkv_b200.device_tree import DeviceTree
    from agentkv_b200.radix_tree import ROOT_NODE_ID, DualRadixTree, SharedNode

    spec = W.MatchSpec(n_prefixes=12, prefix_min=32, prefix_max=160, n_sequences=300, total_min=16,
                       total_max=320, n_queries=1)
    prefixes = W.match_prefixes(spec)
    corpus = W.match_sequences(spec, prefixes)
    tree = object.__new__(DualRadixTree)
    tree._cfg = PoolConfig(total_blocks=64, block_size=16, num_layers=1, num_kv_heads=1, head_dim=1,
                           dtype="float16", device="meta")
    tree._dev_tree = dt = DeviceTree(torch.device("cpu"), node_cap=8, slot_cap=16, token_cap=64)
    tree._shared_nodes = {ROOT_NODE_ID: SharedNode(ROOT_NODE_ID, -1, dt)}
    dt.set_node(ROOT_NODE_ID, 0, 0)
    tree._next_node_id = 1
    rng = np.random.default_rng(4)
    full = []
    full_runs = dt._full_runs
    dt._full_runs = lambda n: (full.append(n), full_runs(n))
    for i, seq in enumerate(corpus):
        n = (len(seq) // 16) * 16
        if rng.random() < 0.2:  # a commit cut inside the shared prefix (split == 0 cases included)
            n = int(rng.integers(0, n // 16 + 1)) * 16
        if n:
            tree._insert_shared_locked(ROOT_NODE_ID, np.asarray(seq[:n], np.int32),
                                       [BlockHandle(b) for b in range(n // 16)])
        if i % 3 == 0:
            dt.build_runs()
            _check_runs(dt, i)
    dt.build_runs()
    _check_runs(dt, "end")
    assert dt._n_unary > 20 and len(full) == 1
    # and a from-scratch build gives the same chains
    fresh_head = dt.d_run_head.numpy().copy()
    fresh_runs = dt.d_runs.numpy().copy()
    dt._runs_dirty = True
    dt._full_runs(len(fresh_head))
    for u in np.flatnonzero(fresh_head >= 0):
        a, b = int(fresh_head[u]), int(dt._h_run_head[u])
        r = int(fresh_runs[a, 3])
        assert r == int(dt._h_runs[b, 3])
        np.testing.assert_array_equal(fresh_runs[a:a + r], dt._h_runs[b:b + r])


def _csr_of(shared_nodes) -> dict:
    """The oracle's CSR arrays of a host tree's nodes (children, edges)."""
    n = max(shared_nodes) + 1
    child_ptr = np.zeros(n + 1, np.int64)
    keys, ids, toks = [], [], []
    edge_off = np.zeros(n, np.int64)
    edge_len = np.zeros(n, np.int32)
    pos = 0
    for nid in range(n):
        nd = shared_nodes.get(nid)
        if nd is not None:
            for k in sorted(nd.children):
                keys.append(k)
                ids.append(nd.children[k])
            e = np.asarray(nd.edge, np.int32)
            edge_off[nid], edge_len[nid] = pos, len(e)
            toks.append(e)
            pos += len(e)
        child_ptr[nid + 1] = len(keys)
    return {"child_ptr": child_ptr, "child_key": np.asarray(keys or [0], np.int32),
            "child_id": np.asarray(ids or [0], np.int32), "edge_off": edge_off, "edge_len": edge_len,
            "edge_tokens": np.concatenate(toks) if pos else np.zeros(1, np.int32)}


def test_tree_orchestration_with_kernel_model(monkeypatch):
    """The host side of match_prefix end to end on CPU, the two tree kernels
    replaced by their CPU model (tests/tree_kernel_model.py): DualRadixTree
    inserts mirrored into an owner DeviceTree (full and incremental deltas),
    a replica fed by TreeReplicaSync deltas with the owner's unary-chain runs,
    and batched lookups under the rebuild policy, with runs and without, whole
    and split into ranges of 32 to 96 tokens — all equal to the oracle's C
    match over the same host tree, comparison counts included."""
    import torch

    from agentkv_b200 import _native as N
    from agentkv_b200 import device_tree as DT
    from agentkv_b200.allocator import BlockHandle
    from agentkv_b200.radix_tree import ROOT_NODE_ID, DualRadixTree, SharedNode
    from agentkv_b200.sharded_tree import TreeReplicaSync
    from oracle import oracle as O
    from tree_kernel_model import TreeKernelModel

    model = TreeKernelModel(N.lib)
    monkeypatch.setattr(N, "lib", model)
    monkeypatch.setattr(DT, "stream_handle", lambda dev: 0)
    cpu = torch.device("cpu")
    spec = W.MatchSpec(n_prefixes=10, prefix_min=64, prefix_max=256, n_sequences=240, total_min=32,
                       total_max=480, n_queries=96)
    prefixes = W.match_prefixes(spec)
    corpus = W.match_sequences(spec, prefixes)
    tree = object.__new__(DualRadixTree)
    tree._cfg = PoolConfig(total_blocks=64, block_size=16, num_layers=1, num_kv_heads=1, head_dim=1,
                           dtype="float16", device="meta")
    tree._dev_tree = owner = DT.DeviceTree(cpu, node_cap=8, slot_cap=16, token_cap=64)
    tree._shared_nodes = {ROOT_NODE_ID: SharedNode(ROOT_NODE_ID, -1, owner)}
    owner.set_node(ROOT_NODE_ID, 0, 0)
    tree._next_node_id = 1
    sync = TreeReplicaSync(owner)
    replica = DT.DeviceTree(cpu)
    replica.as_replica()
    queries = W.match_queries(spec, corpus, prefixes, batch=0, n=spec.n_queries)
    flat, q_off = O.pack_queries([q.tolist() for q in queries])
    rng = np.random.default_rng(8)
    checks = 0
    for i, seq in enumerate(corpus):
        n = (len(seq) // 16) * 16
        if rng.random() < 0.2:
            n = int(rng.integers(0, n // 16 + 1)) * 16
        if n:
            tree._insert_shared_locked(ROOT_NODE_ID, np.asarray(seq[:n], np.int32),
                                       [BlockHandle(b) for b in range(n // 16)])
        if i % 7 == 6:
            if i % 2:
                owner.build_runs()  # else the policy decides whether new runs travel
            d = sync.share()
            if d is not None:
                replica.apply_shared(d)
                if "run_head" in d:
                    replica.set_runs(d["run_head"], d["runs"])
        if i % 21 == 20:
            want = O.match_prefix_csr(_csr_of(tree._shared_nodes), flat, q_off, 16)
            want_node = np.where(want[1] > 0, want[0], -1)
            # the split lookup at the default range and at ranges far shorter
            # than the queries (many ranges per query, stops in any of them);
            # the staged lookup at every window size
            for t, runs, tpi in ((owner, None, -1), (owner, False, -1), (replica, None, -1), (owner, None, 0),
                                 (owner, True, 32), (replica, False, 64), (owner, None, 96),
                                 (owner, None, "s0"), (replica, True, "s256"), (owner, False, "s1024")):
                staged = isinstance(tpi, str)
                node, mlen, cmp_ = DT.match_batch(
                    t, queries, 16, with_compared=True, runs=runs, split=not staged and tpi >= 0,
                    tokens_per_range=0 if staged else max(tpi, 0), staged=staged,
                    window_tokens=int(tpi[1:]) if staged else 0)
                np.testing.assert_array_equal(mlen, want[1], err_msg=f"{i} {runs} {tpi}")
                np.testing.assert_array_equal(np.where(mlen > 0, node, -1), want_node)
                np.testing.assert_array_equal(cmp_, want[2])
            checks += 1
    assert checks >= 10 and model.run_hops > 1000, (checks, model.run_hops)
    assert model.split_ranges > 20 * checks * len(queries), model.split_ranges
    assert model.staged_windows > 3 * checks * len(queries), model.staged_windows
    # the replica's arrays equal the owner's after a final sync
    owner.build_runs()
    d = sync.share()
    if d is not None:
        replica.apply_shared(d)
        if "run_head" in d:
            replica.set_runs(d["run_head"], d["runs"])
    owner.flush()
    n = owner.n_tokens
    assert torch.equal(replica.d_tokens[:n], owner.d_tokens[:n])
    assert torch.equal(replica.d_slots, owner.d_slots)
    assert torch.equal(replica.d_off, owner.d_off) and torch.equal(replica.d_len, owner.d_len)
    assert torch.equal(replica.d_run_head, owner.d_run_head) and torch.equal(replica.d_runs, owner.d_runs)
