"""Host-side logic that needs no GPU: config validation (same rules and
messages as the reference), the device-tree mirror's hash table and
unary-chain runs, pair validation, the seeded workload generators, the
bench's byte counts and CPU baselines, and — with the tree kernels replaced
by their CPU model (tree_kernel_model.py) and the allocator answered by the
oracle (oracle_slab.py) — the package's tree logic replaying the
reference's recorded traces and the match path's host orchestration."""

import json

import numpy as np
import pytest

from agentkv_b200 import workloads as W
from agentkv_b200.config import PoolConfig
from agentkv_b200.device_tree import DELETED, EMPTY, tree_hash


class TestPoolConfig:
    def test_bytes_per_block(self):
        c = PoolConfig(total_blocks=10, block_size=16, num_layers=32, num_kv_heads=8, head_dim=128,
                       dtype="bfloat16", device="cuda")
        assert c.bytes_per_block == 2 * 1024 * 1024
        assert c.total_bytes == 10 * c.bytes_per_block

    @pytest.mark.parametrize("kw,msg", [
        ({"dtype": "int8"}, "dtype must be one of"),
        ({"block_size": 12}, "power of 2"),
        ({"block_size": 0}, "power of 2"),
        ({"total_blocks": 0}, "total_blocks must be > 0"),
        ({"max_agents": 0}, "max_agents must be > 0"),
    ])
    def test_validation(self, kw, msg):
        with pytest.raises(ValueError, match=msg):
            PoolConfig(**kw)

    def test_from_capacity_rounds_down_to_power_of_two(self):
        c = PoolConfig.from_capacity_gb(1.0, num_layers=32, num_kv_heads=8, head_dim=128, dtype="float16")
        assert c.total_blocks == 512  # 1 GiB / 2 MiB
        c = PoolConfig.from_capacity_gb(0.9, num_layers=32, num_kv_heads=8, head_dim=128)
        assert c.total_blocks == 256
        with pytest.raises(ValueError, match="too small"):
            PoolConfig.from_capacity_gb(1e-9)

    def test_repr(self):
        assert "GiB" in repr(PoolConfig(total_blocks=4, device="cpu"))


def _kernel_style_lookup(slots, parent, token):
    """The device lookup rule: 32-slot windows from the hash; first hit wins,
    an empty slot before any hit ends the probe."""
    mask = len(slots) - 1
    h = tree_hash(parent, token)
    for w in range(len(slots) // 32 + 1):
        win = [(h + w * 32 + lane) & mask for lane in range(32)]
        hits = [i for i, s in enumerate(win) if slots[s, 0] == parent and slots[s, 1] == token]
        empties = [i for i, s in enumerate(win) if slots[s, 0] == EMPTY]
        if hits:
            return int(slots[win[hits[0]], 2]) if not empties or hits[0] < empties[0] else -1
        if empties:
            return -1
    return -1


def test_device_tree_hash_table_mirror():
    from agentkv_b200.device_tree import DeviceTree
    import torch

    t = DeviceTree(torch.device("cpu"), slot_cap=64)
    ref = {}
    rng = np.random.default_rng(5)
    for step in range(3000):
        p, k = int(rng.integers(0, 40)), int(rng.integers(0, 12))
        if rng.random() < 0.65:
            c = int(rng.integers(1, 10_000))
            t.set_child(p, k, c, 3)
            ref[(p, k)] = c
        else:
            t.del_child(p, k)
            ref.pop((p, k), None)
        if step % 97 == 0:
            for pp in range(40):
                for kk in range(12):
                    assert _kernel_style_lookup(t.h_slots, pp, kk) == ref.get((pp, kk), -1)
    assert t.live == len(ref)
    assert 2 * (t.live + t.dead) <= len(t.h_slots)
    assert (t.h_slots[:, 0] >= DELETED).all()


def test_device_tree_arena_and_nodes():
    from agentkv_b200.device_tree import DeviceTree
    import torch

    t = DeviceTree(torch.device("cpu"), node_cap=2, token_cap=4)
    o1 = t.append_tokens(np.arange(5))
    o2 = t.append_tokens(np.arange(100, 103))
    assert (o1, o2) == (0, 5)
    t.set_node(7, o2, 3)
    assert t.edge(o2, 3).tolist() == [100, 101, 102]
    assert len(t.h_off) >= 8 and t.h_len[7] == 3


def test_validate_pairs():
    from agentkv_b200.kernels import validate_pairs

    validate_pairs([[0, 1], [2, 3], [4, 4]], 5)
    with pytest.raises(ValueError, match="out of range"):
        validate_pairs([[0, 5]], 5)
    with pytest.raises(ValueError, match="appears twice"):
        validate_pairs([[0, 1], [2, 1]], 5)
    with pytest.raises(ValueError, match="read as another"):
        validate_pairs([[0, 1], [1, 2]], 5)


def test_workloads_are_deterministic():
    a = W.copy_sweep_pairs(512)
    b = W.copy_sweep_pairs(512)
    np.testing.assert_array_equal(a, b)
    assert len(np.unique(a)) == 1024 and a.max() < 60_000
    assert not np.array_equal(a, W.copy_sweep_pairs(512, rotation=1))
    spec = W.MatchSpec(n_sequences=50, n_queries=16)
    s1, s2 = W.match_sequences(spec), W.match_sequences(spec)
    assert all(np.array_equal(x, y) for x, y in zip(s1, s2))
    assert all(512 <= len(x) <= 8192 for x in s1)
    assert W.quickstart_queries() == W.quickstart_queries()
    assert len(W.tot_root_tokens()) == 4096


def test_query_ranges_cover_the_batch():
    from agentkv_b200.sharded_tree import query_range

    for n in (0, 1, 7, 256, 4096, 4097):
        for w in (1, 2, 3, 8):
            r = [query_range(n, i, w) for i in range(w)]
            assert r[0][0] == 0 and r[-1][1] == n
            assert all(r[i][1] == r[i + 1][0] for i in range(w - 1))
            sizes = [b - a for a, b in r]
            assert max(sizes) - min(sizes) <= 1


def test_layer_cache_table_validation():
    """The host checks behind copy_blocks_layers (CPU tensors stand in for
    device caches: only shapes, strides and addresses are looked at)."""
    import torch

    from agentkv_b200 import kernels as K

    K._CACHE_TABLES.clear()
    kv = [torch.zeros(2, 10, 4, 2, 8, dtype=torch.float16) for _ in range(3)]
    caches = [t[0] for t in kv] + [t[1] for t in kv]
    table, n, block_bytes, stride = K._cache_table(caches)
    assert (n, block_bytes, stride) == (10, 4 * 2 * 8 * 2, 4 * 2 * 8 * 2)
    assert table.tolist() == [c.data_ptr() for c in caches]
    assert K._cache_table(caches)[0] is table  # same tensors: cached
    assert K._cache_table([t[0] for t in kv] + [t[1] for t in kv])[0] is table  # new views, same memory
    with pytest.raises(ValueError):
        K._cache_table(caches + [torch.zeros(9, 4, 2, 8, dtype=torch.float16)])  # block count differs
    with pytest.raises(ValueError):
        K._cache_table([torch.zeros(10, 3, 2, dtype=torch.float16)])  # 12-byte blocks
    with pytest.raises(ValueError):
        K._cache_table([torch.zeros(10, 8, dtype=torch.float16)[:, :4]])  # 8-byte blocks 16 bytes apart
    with pytest.raises(ValueError):
        K._cache_table([])


def test_hf_script_and_states_are_deterministic():
    from agentkv_b200 import workloads as W

    spec = W.HFSpec()
    ev = W.hf_script(spec)
    assert ev[:2] == [("prefill", 0, 10), ("commit", 0, 8)]
    assert sum(1 for e in ev if e[0] == "fork") == spec.forks
    k1, v1 = W.hf_states(spec, 7, 1, 3)
    k2, v2 = W.hf_states(spec, 7, 1, 3)
    assert k1.shape == (1, spec.num_kv_heads, 3, spec.head_dim) and (k1 == k2).all() and (v1 == v2).all()
    tr = W.react_trace(W.ReActSpec(steps=5))
    assert len(tr) == 5 and all(len(st) == 32 for st in tr)
    assert all(t != s for st in tr for _, s, t in st)


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


def test_match_compulsory_bytes():
    """The match roofline's byte count on a hand-built tree: root -> 1
    (8-token edge) -> {2, 3} (4-token edges).  A: both edges of 0-1-2
    compared in full; B: edge 1 in full, 2 tokens of edge 3; C: a mismatch
    after 3 tokens of edge 1 (no credited match)."""
    import bench

    parent = {0: -1, 1: 0, 2: 1, 3: 1}
    edge_len = {0: 0, 1: 8, 2: 4, 3: 4}
    children = {0: {10: 1}, 1: {20: 2, 30: 3}, 2: {}, 3: {}}
    qa = np.array([10] + [1] * 7 + [20, 2, 2, 2, 5, 5])
    qb = np.array([10] + [1] * 7 + [30, 7, 7])
    qc = np.array([10, 1, 1, 9])
    got = bench.match_compulsory_bytes(parent, edge_len, children, [qa, qb, qc],
                                       np.array([2, 1, -1]), np.array([12, 10, 3]))
    assert got["query_bytes"] == 4 * (12 + 10 + 3)
    assert got["edge_bytes"] == 4 * (8 + 4 + 2)  # edge 1 once, edge 2 in full, 2 tokens of edge 3
    assert got["nodes"] == 4
    assert got["total"] == 100 + 56 + 4 * bench.MATCH_NODE_BYTES


def test_match_cpu_baseline_on_a_host_tree():
    """bench.match_cpu_baseline flattens a host tree (nodes with .children and
    .edge) for the oracle's C match and reports queries/s; answers equal to
    the given ones are flagged as such, a planted difference is not."""
    from types import SimpleNamespace

    import bench
    from oracle import oracle as O

    ot = O.OracleTree(O.OracleAllocator(256), 16)
    rng = np.random.default_rng(3)
    seqs = [rng.integers(0, 40, size=int(rng.integers(16, 80))).tolist() for _ in range(30)]
    for s in seqs:
        h = ot.create_root(s)
        while len(ot.get_block_ids(h)) < -(-len(s) // 16):
            ot.allocate_block(h)
        share = (len(s) // 16) * 16 - h.shared_match_len
        if share > 0:
            ot.commit_prefix(h, share)
    batch = [np.asarray(s[: int(rng.integers(1, len(s) + 1))] + [99], np.int32) for s in seqs]
    want = [ot.match(q.tolist()) for q in batch]
    node = np.array([w[0] for w in want], np.int32)
    mlen = np.array([w[1] for w in want], np.int32)
    pool = SimpleNamespace(_tree=SimpleNamespace(_shared_nodes=ot.nodes))
    res = bench.match_cpu_baseline(pool, [batch], [(node, mlen)], 0.05)
    assert res["same_answers_as_gpu"] and res["value"] > 0 and res["cores"] == 1
    assert mlen.max() > 0
    planted = mlen.copy()
    planted[int(np.argmax(mlen))] = 0
    assert not bench.match_cpu_baseline(pool, [batch], [(node, planted)], 0.01)["same_answers_as_gpu"]


def test_run_rebuild_policy():
    """DeviceTree.want_runs: a never-built tree builds; current runs are used;
    after a change the one-probe-per-hop lookups pay rent, the coming one
    counted at the last batch's time, until it reaches the last rebuild's
    cost; every change restarts the count; a replica uses runs only while it
    holds the owner's."""
    import torch

    from agentkv_b200.device_tree import DeviceTree

    t = DeviceTree(torch.device("cpu"), node_cap=8, slot_cap=16, token_cap=32)
    t.set_node(1, t.append_tokens(np.array([5, 6], np.int32)), 2)
    t.set_child(0, 5, 1, 2)
    assert t.want_runs()  # never built
    t.build_runs()
    assert t.want_runs() and t._build_ms is not None
    t._build_ms = 2.0  # a rebuild costs 2 ms
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
    t._build_ms = 0.05  # a cheap incremental rebuild: the next change rebuilds at once
    t.set_child(2, 9, 1, 1)
    assert t.want_runs()

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


def test_react_cpu_baseline_plays_the_trace():
    """bench.react_cpu_baseline drives the oracle through the ReAct trace with
    the same call set the parity tests use, and reports steps/s over a
    bounded sample."""
    import bench

    spec = W.ReActSpec(steps=30)
    res = bench.react_cpu_baseline(spec, 1, 60.0)
    assert res["unit"] == "steps/s" and res["value"] > 0 and res["kind"] == "port"
    assert res["sample"].startswith("30 of 30 trace steps")


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
    and batched lookups under the rebuild policy, with runs and without —
    all equal to the oracle's C match over the same host tree, comparison
    counts included."""
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
                replica.apply_delta(d)
                if "run_head" in d:
                    replica.set_runs(d["run_head"], d["runs"])
        if i % 21 == 20:
            want = O.match_prefix_csr(_csr_of(tree._shared_nodes), flat, q_off, 16)
            want_node = np.where(want[1] > 0, want[0], -1)
            for t, runs in ((owner, None), (owner, False), (replica, None)):
                node, mlen, cmp_ = DT.match_batch(t, queries, 16, with_compared=True, runs=runs)
                np.testing.assert_array_equal(mlen, want[1], err_msg=f"{i} {runs}")
                np.testing.assert_array_equal(np.where(mlen > 0, node, -1), want_node)
                np.testing.assert_array_equal(cmp_, want[2])
            checks += 1
    assert checks >= 10 and model.run_hops > 1000, (checks, model.run_hops)
    # the replica's arrays equal the owner's after a final sync
    owner.build_runs()
    d = sync.share()
    if d is not None:
        replica.apply_delta(d)
        if "run_head" in d:
            replica.set_runs(d["run_head"], d["runs"])
    owner.flush()
    n = owner.n_tokens
    assert torch.equal(replica.d_tokens[:n], owner.d_tokens[:n])
    assert torch.equal(replica.d_slots, owner.d_slots)
    assert torch.equal(replica.d_off, owner.d_off) and torch.equal(replica.d_len, owner.d_len)
    assert torch.equal(replica.d_run_head, owner.d_run_head) and torch.equal(replica.d_runs, owner.d_runs)


def test_serving_lifecycle_on_the_oracle():
    """The serving-lifecycle schedule (tests/serving_pattern.py) on the
    oracle: deterministic, with page hits that return the committed blocks,
    misses, aborts, finishes and evictions; the allocated count it reads
    agrees with the oracle's own counter."""
    from serving_pattern import OracleServeAPI, serve

    a = serve(OracleServeAPI(512, 16))
    assert a == serve(OracleServeAPI(512, 16))
    kinds = {o[0] for o in a}
    assert {"hit", "miss", "abort", "finish", "evict"} <= kinds, kinds
    assert sum(1 for o in a if o[0] == "hit") >= 10
    assert all(o[1] >= 0 for o in a if o[0] == "evict")
    # hits hand back the committed prefix's blocks, one id per whole page
    assert all(len(o[3]) == o[2] // 16 and o[2] > 0 for o in a if o[0] == "hit")
    api = OracleServeAPI(512, 16)
    serve(api)
    assert api.allocated_blocks == api.alloc.state()["allocated_blocks"]
    assert a[-1] == ("end", api.free_blocks, api.allocated_blocks)


def test_package_exports_the_reference_names():
    """The names the reference package exports at its top level
    (agentkv/__init__.py) and the triton_kernels helpers resolve here."""
    import agentkv_b200
    from agentkv_b200 import kernels as K

    for name in ("AgentKVPool", "CoWRadixTree", "DualRadixTree", "SlabAllocator", "PoolConfig",
                 "AgentKVCache", "__version__"):
        assert getattr(agentkv_b200, name) is not None, name
    assert agentkv_b200.CoWRadixTree is agentkv_b200.DualRadixTree
    assert K.is_triton_available() is False
    assert callable(K.copy_block) and callable(K.zero_block) and callable(K.kernel_info)


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_tree_host_logic_replays_reference_traces(golden_dir, seed, monkeypatch):
    """The package's host-side tree logic (agentkv_b200/radix_tree.py:
    handles, shared nodes, inserts with their split / overwrite quirks,
    prunes, CoW dispatch, error checks) replays the reference's recorded
    tree traces on CPU — the allocator answered by the oracle
    (tests/oracle_slab.py), the tree kernels by their CPU model — with every
    result, error, block table, tree node, refcount, free-list entry and
    block digest as recorded."""
    import hashlib

    import torch

    from agentkv_b200 import _native as N
    from agentkv_b200 import device_tree as DT
    from agentkv_b200.allocator import BlockHandle
    from agentkv_b200.radix_tree import DualRadixTree
    from oracle_slab import OracleSlab
    from tree_kernel_model import TreeKernelModel

    monkeypatch.setattr(N, "lib", TreeKernelModel(N.lib))
    monkeypatch.setattr(DT, "stream_handle", lambda dev: 0)
    g = json.loads((golden_dir / f"tree_trace_{seed}.json").read_text())
    n, bs = g["n_blocks"], g["block_size"]
    cfg = PoolConfig(total_blocks=n, block_size=bs, num_layers=1, num_kv_heads=2, head_dim=4,
                     dtype="float16", device="meta", epoch_interval=7)
    torch.manual_seed(seed)
    kv = torch.randn((n, 1, 2, 2, bs, 4), dtype=torch.float32).half()
    slab = OracleSlab(kv, 7)
    tree = DualRadixTree(slab, cfg)
    T_CREATE, T_FORK, T_ALLOC, T_COW, T_APPEND, T_COMMIT, T_FREE, T_MATCH, T_ADVANCE, T_ZERO = range(10)
    live = {}
    states = {step: st for step, st in g["states"]}
    for step, rec in enumerate(g["ops"]):
        op = rec["op"]
        err = None
        try:
            if op == T_CREATE:
                h = tree.create_root(rec["tokens"])
                live[h.handle_id] = h
                assert [h.handle_id, h.shared_node_id, h.shared_match_len] == rec["out"]
            elif op == T_FORK:
                c = tree.fork(live[rec["h"]])
                live[c.handle_id] = c
                assert c.handle_id == rec["out"]
            elif op == T_ALLOC:
                h = live[rec["h"]]
                tree.allocate_block(h)
                assert h.residual_blocks[-1].block_id == rec["out"]
            elif op == T_COW:
                h = live[rec["h"]]
                tree.ensure_mutable_block(h, rec["idx"])
                assert h.residual_blocks[rec["idx"]].block_id == rec["out"]
            elif op == T_APPEND:
                tree.append_tokens(live[rec["h"]], rec["tokens"])
            elif op == T_COMMIT:
                h = live[rec["h"]]
                tree.commit_prefix(h, rec["length"])
                assert [h.shared_node_id, h.shared_match_len] == rec["out"]
            elif op == T_FREE:
                tree.free(live.pop(rec["h"]))
            elif op == T_MATCH:
                mh, mlen = tree.match_prefix(rec["tokens"])
                got = [-1 if mh is None else mh.handle_id, mlen, -1 if mh is None else mh.shared_node_id]
                assert got == rec["out"]
                if mh is not None:
                    live[mh.handle_id] = mh
            elif op == T_ADVANCE:
                slab.maybe_advance_epoch()
            elif op == T_ZERO:
                slab.zero_block(BlockHandle(rec["block"]))
        except (ValueError, MemoryError) as e:
            err = e
        assert (err is not None) == ("error" in rec), f"step {step}: {rec} -> {err!r}"
        if step in states:
            st = states[step]
            assert {str(k): tree.get_block_ids(h) for k, h in sorted(live.items())} == st["tables"]
            assert {str(k): [h.shared_node_id, h.shared_match_len] for k, h in sorted(live.items())} == st["shared"]
            nodes = {str(nid): {"parent": nd.parent_id, "edge": nd.edge_tokens,
                                "blocks": [b.block_id for b in nd.blocks],
                                "children": sorted([int(k), int(v)] for k, v in nd.children.items()),
                                "ref": nd.ref_count}
                     for nid, nd in sorted(tree._shared_nodes.items())}
            assert nodes == st["nodes"]
            ost = slab.o.state()
            assert ost["ref_counts"].tolist() == st["ref"]
            assert ost["free_list"].tolist() == st["free"]
            for k in ("active_handles", "shared_nodes", "shared_blocks"):
                if k in st["stats"]:
                    assert tree.stats()[k] == st["stats"][k], k
    digests = [hashlib.sha256(kv[i].numpy().tobytes()).hexdigest() for i in range(n)]
    assert digests == g["block_sha256"]


@pytest.mark.parametrize("seed", [1, 2, 7, 13, 17, 42, 137, 999])
def test_tree_host_logic_replays_reference_stress_runner(golden_dir, seed, monkeypatch):
    """The reference stress runner's recorded calls (tests/stress_replay.py)
    through the package's tree logic on CPU, the allocator answered by the
    oracle and the tree kernels by their CPU model: every handle id, block
    id and exhaustion as recorded, and the recorded end state."""
    import torch

    from agentkv_b200 import _native as N
    from agentkv_b200 import device_tree as DT
    from agentkv_b200.radix_tree import DualRadixTree
    from oracle_slab import OracleSlab
    from stress_replay import replay
    from tree_kernel_model import TreeKernelModel

    monkeypatch.setattr(N, "lib", TreeKernelModel(N.lib))
    monkeypatch.setattr(DT, "stream_handle", lambda dev: 0)
    g = np.load(golden_dir / f"stress_{seed}.npz")
    cfg = PoolConfig(total_blocks=512, block_size=4, num_layers=2, num_kv_heads=2, head_dim=8, dtype="float16",
                     device="meta")
    slab = OracleSlab(torch.zeros((512, 2, 2, 2, 4, 8), dtype=torch.float16), cfg.epoch_interval)
    tree = DualRadixTree(slab, cfg)
    replay(g, tree, slab.maybe_advance_epoch, lambda e: isinstance(e, MemoryError) and "exhausted" in str(e))
    st = slab.o.state()
    np.testing.assert_array_equal(st["ref_counts"], g["ref"])
    np.testing.assert_array_equal(st["free_list"], g["free"])


def test_hf_cache_host_logic_replays_reference_session(golden_dir, monkeypatch):
    """The package's HuggingFace cache logic (agentkv_b200/hf_cache.py: block
    allocation on layer 0, copy-on-write checks in the reference's order,
    slot arithmetic, truncation) replays the reference's recorded session on
    CPU — the pool's allocator answered by the oracle, the tree kernels by
    their CPU model, and the KV scatter / gather by their contract in torch
    indexing — with every K/V output, block table, sequence length and pool
    byte as recorded."""
    import torch

    from agentkv_b200 import _native as N
    from agentkv_b200 import device_tree as DT
    from agentkv_b200 import kernels as K
    from agentkv_b200.hf_cache import AgentKVCache
    from agentkv_b200.pool import AgentKVPool
    from agentkv_b200.radix_tree import DualRadixTree
    from oracle_slab import OracleSlab
    from tree_kernel_model import TreeKernelModel

    def kv_scatter(kv, slots, layer, k, v, status=None):
        bs = kv.shape[4]
        for i, slot in enumerate(slots.tolist()):
            kv[slot // bs, layer, 0, :, slot % bs] = k[0, :, i].to(kv.dtype)
            kv[slot // bs, layer, 1, :, slot % bs] = v[0, :, i].to(kv.dtype)

    def kv_gather(kv, table, layer, n_tokens, status=None):
        x = kv[table.long(), layer]  # [blocks, 2, H, bs, D]
        nb, _, h, bs, d = x.shape
        k = x[:, 0].permute(1, 0, 2, 3).reshape(1, h, nb * bs, d)[:, :, :n_tokens]
        v = x[:, 1].permute(1, 0, 2, 3).reshape(1, h, nb * bs, d)[:, :, :n_tokens]
        return k.contiguous(), v.contiguous()

    monkeypatch.setattr(N, "lib", TreeKernelModel(N.lib))
    monkeypatch.setattr(DT, "stream_handle", lambda dev: 0)
    monkeypatch.setattr(K, "kv_scatter", kv_scatter)
    monkeypatch.setattr(K, "kv_gather", kv_gather)
    g = np.load(golden_dir / "hf_session.npz")
    spec = W.HFSpec(**json.loads(str(g["spec"])))
    cfg = PoolConfig(total_blocks=spec.total_blocks, block_size=spec.block_size, num_layers=spec.num_layers,
                     num_kv_heads=spec.num_kv_heads, head_dim=spec.head_dim, dtype=spec.dtype, device="meta")
    kv = torch.zeros((spec.total_blocks, spec.num_layers, 2, spec.num_kv_heads, spec.block_size, spec.head_dim),
                     dtype=getattr(torch, spec.dtype))
    pool = object.__new__(AgentKVPool)
    pool._cfg = cfg
    pool._allocator = OracleSlab(kv, cfg.epoch_interval)
    pool._allocator._status = torch.zeros(8, dtype=torch.int32)
    pool._tree = DualRadixTree(pool._allocator, cfg)
    outs, keys = [], []

    def on_output(e, layer, ok, ov):
        keys.append((e, layer, ok.shape[2]))
        outs.append(np.concatenate([ok.numpy().reshape(-1), ov.numpy().reshape(-1)]))

    caches = W.hf_run(spec, pool, AgentKVCache, torch.from_numpy, on_output)
    np.testing.assert_array_equal(np.asarray(keys), g["out_keys"])
    assert np.concatenate(outs).tobytes() == g["outs"].tobytes()
    tables = np.concatenate([np.asarray(pool.get_block_ids(c.handle), np.int32) for c in caches])
    np.testing.assert_array_equal(tables, g["tables"])
    assert [c.get_seq_length() for c in caches] == g["seen"].tolist()
    assert kv.numpy().tobytes() == g["pool"].tobytes()


def test_react_trace_host_logic_replays_reference(golden_dir, monkeypatch):
    """The ReAct trace (70B geometry, 40,000 blocks, 1,000 steps) through the
    package's pool and tree logic on CPU with the copy_block hook of the
    vLLM adapter: every step's recorded CoW pairs, and at the checkpoints the
    agents' tables, refcounts and free list, as the reference recorded them
    (allocator answered by the oracle, tree kernels by their CPU model)."""
    import torch

    from agentkv_b200 import _native as N
    from agentkv_b200 import device_tree as DT
    from agentkv_b200.pool import AgentKVPool
    from agentkv_b200.radix_tree import DualRadixTree
    from oracle_slab import OracleSlab
    from react_apis import PoolReActAPI
    from tree_kernel_model import TreeKernelModel

    monkeypatch.setattr(N, "lib", TreeKernelModel(N.lib))
    monkeypatch.setattr(DT, "stream_handle", lambda dev: 0)
    g = np.load(golden_dir / "react_70b.npz")
    spec = W.ReActSpec(**json.loads(str(g["spec"])))
    n_, bs, L, H, D, dt = W.LLAMA3_70B_GEOMETRY
    cfg = PoolConfig(total_blocks=n_, block_size=bs, num_layers=L, num_kv_heads=H, head_dim=D, dtype=dt,
                     device="meta")
    slab = OracleSlab(torch.zeros((n_, 1), dtype=torch.uint8), cfg.epoch_interval)
    pairs = []
    slab.copy_block = lambda src, dst: pairs.append((src.block_id, dst.block_id))
    pool = object.__new__(AgentKVPool)
    pool._cfg, pool._allocator = cfg, slab
    pool._tree = DualRadixTree(slab, cfg)
    api = PoolReActAPI(pool)
    root, agents = W.react_setup(api, spec)
    np.testing.assert_array_equal(np.asarray(pool.get_block_ids(root), np.int32), g["root_table"])
    so = g["step_off"]
    for i, actions in enumerate(W.react_trace(spec)):
        pairs.clear()
        W.react_step(api, root, agents, actions)
        np.testing.assert_array_equal(np.asarray(pairs, np.int32).reshape(-1, 2), g["pairs"][so[i]:so[i + 1]],
                                      err_msg=f"step {i}")
        k = f"s{i + 1}"
        if k + "_ref" in g.files:
            tables = np.concatenate([np.asarray(pool.get_block_ids(h), np.int32) for h in agents])
            np.testing.assert_array_equal(tables, g[k + "_tables"], err_msg=k)
            st = slab.o.state()
            np.testing.assert_array_equal(st["ref_counts"], g[k + "_ref"])
            np.testing.assert_array_equal(st["free_list"], g[k + "_free"])


def _cpu_pool(cfg, kv, monkeypatch):
    """An AgentKVPool whose allocator is the oracle (tests/oracle_slab.py)
    and whose tree kernels run as their CPU model, over the CPU tensor kv."""
    import torch  # noqa: F401

    from agentkv_b200 import _native as N
    from agentkv_b200 import device_tree as DT
    from agentkv_b200.pool import AgentKVPool
    from agentkv_b200.radix_tree import DualRadixTree
    from oracle_slab import OracleSlab
    from tree_kernel_model import TreeKernelModel

    if not isinstance(N.lib, TreeKernelModel):
        monkeypatch.setattr(N, "lib", TreeKernelModel(N.lib))
    monkeypatch.setattr(DT, "stream_handle", lambda dev: 0)
    pool = object.__new__(AgentKVPool)
    pool._cfg = cfg
    pool._allocator = OracleSlab(kv, cfg.epoch_interval)
    pool._tree = DualRadixTree(pool._allocator, cfg)
    return pool


def test_quickstart_host_logic_replays_reference(golden_dir, monkeypatch):
    """The quickstart workload through the package's pool logic on CPU:
    children's tables, the root's, match results, refcounts, free list and
    every block's bytes as the reference recorded them."""
    import hashlib

    import torch

    g = json.loads((golden_dir / "quickstart.json").read_text())
    n_, bs, L, H, D, dt = W.QUICKSTART_GEOMETRY
    cfg = PoolConfig(total_blocks=n_, block_size=bs, num_layers=L, num_kv_heads=H, head_dim=D, dtype=dt,
                     device="meta")
    torch.manual_seed(0)
    kv = torch.randn((n_, L, 2, H, bs, D), dtype=torch.float16)
    pool = _cpu_pool(cfg, kv, monkeypatch)
    root = pool.create_root(list(range(32)))
    pool.allocate_block(root)
    kids = [pool.fork(root) for _ in range(3)]
    for c in kids:
        pool.allocate_block(c)
    for c in kids:
        pool.ensure_mutable_block(c, 0)
    pool.commit_prefix(root, 16)
    matches = []
    for q in g["queries"]:
        mh, mlen = pool._tree.match_prefix(q)
        matches.append([-1 if mh is None else mh.shared_node_id, mlen])
    assert [pool.get_block_ids(c) for c in kids] == g["children"]
    assert pool.get_block_ids(root) == g["root"]
    assert matches == g["matches"]
    st = pool._allocator.o.state()
    assert st["ref_counts"].tolist() == g["ref"]
    assert st["free_list"].tolist() == g["free"]
    assert [hashlib.sha256(kv[i].numpy().tobytes()).hexdigest() for i in range(n_)] == g["block_sha256"]


def test_tot_batched_host_logic_replays_reference(golden_dir, monkeypatch):
    """The Tree-of-Thought fan-out on the 60,000-block pool through the
    package's batched pool calls (fork_many, ensure_mutable_batch,
    allocate_blocks, free_many) on CPU: child tables, refcounts and free
    lists after the fan-out and after the frees as the reference recorded
    them."""
    import torch

    g = np.load(golden_dir / "tot_8b.npz")
    spec = W.ToTSpec()
    n_, bs, L, H, D, dt = W.LLAMA3_8B_GEOMETRY
    cfg = PoolConfig(total_blocks=n_, block_size=bs, num_layers=L, num_kv_heads=H, head_dim=D, dtype=dt,
                     device="meta")
    pool = _cpu_pool(cfg, torch.zeros((n_, 1), dtype=torch.uint8), monkeypatch)
    root = pool.create_root(W.tot_root_tokens(spec))
    pool.allocate_blocks(root, spec.root_tokens // 16)
    level, kids = [root], []
    for lvl in range(spec.levels):
        nxt = []
        for parent in level:
            nxt.extend(pool.fork_many(parent, spec.fanout))
        for c in nxt:
            pool.ensure_mutable_batch([(c, len(c.residual_blocks) - 1)])
            pool.allocate_blocks(c, spec.appended_blocks)
        kids.extend(nxt)
        level = nxt
    tables = np.concatenate([np.asarray(pool.get_block_ids(c), np.int32) for c in kids])
    np.testing.assert_array_equal(tables, g["tables"])
    st = pool._allocator.o.state()
    np.testing.assert_array_equal(st["ref_counts"], g["ref_fanout"])
    np.testing.assert_array_equal(st["free_list"], g["free_fanout"])
    pool.free_many(kids)
    st = pool._allocator.o.state()
    np.testing.assert_array_equal(st["ref_counts"], g["ref_freed"])
    np.testing.assert_array_equal(st["free_list"], g["free_freed"])


def test_serving_lifecycle_host_logic_equals_oracle(monkeypatch):
    """The serving-lifecycle schedule through the package's pool logic on CPU
    (oracle allocator, tree kernel model) observes what the oracle's own
    tree observes: hits, block ids, finishes, aborts, counters."""
    import torch

    from serving_pattern import OracleServeAPI, PoolServeAPI, serve

    cfg = PoolConfig(total_blocks=512, block_size=16, num_layers=1, num_kv_heads=1, head_dim=8,
                     dtype="float16", device="meta")
    pool = _cpu_pool(cfg, torch.zeros((512, 1), dtype=torch.uint8), monkeypatch)
    assert serve(PoolServeAPI(pool)) == serve(OracleServeAPI(512, 16))


def test_allocator_error_mapping():
    """SlabAllocator turns the device status codes into the reference's
    exception types with the message parts its tests match
    (tests/test_slab_allocator.py: "exhausted", "not allocated",
    "double-free", "ref_count=1", "exclusively owned", out-of-range ids),
    and validates handles like slab_allocator.py:_validate_handle."""
    from agentkv_b200 import _native as N
    from agentkv_b200.allocator import INVALID_BLOCK, BlockHandle, SlabAllocator

    a = object.__new__(SlabAllocator)
    a._cfg = PoolConfig(total_blocks=8, block_size=4, num_layers=1, num_kv_heads=1, head_dim=4,
                        dtype="float16", device="meta")
    cases = [
        (N.AKV_ERR_EXHAUSTED, "alloc", MemoryError, "exhausted"),
        (N.AKV_ERR_NOT_ALLOCATED, "inc_ref", ValueError, "not allocated"),
        (N.AKV_ERR_DOUBLE_FREE, "dec_ref", ValueError, "double-free"),
        (N.AKV_ERR_NOT_EXCLUSIVE, "copy_block", ValueError, "ref_count=1"),
        (N.AKV_ERR_NOT_EXCLUSIVE, "zero_block", ValueError, "exclusively owned"),
        (N.AKV_ERR_OUT_OF_RANGE, "copy_block", ValueError, "out of range"),
    ]
    for code, op, typ, part in cases:
        e = a._exception(code, 3, 0, op)
        assert type(e) is typ and part in str(e), (code, op, e)
    assert isinstance(a._exception(N.AKV_ERR_TIMEOUT, 0, 0, "copy"), RuntimeError)
    with pytest.raises(TypeError):
        a._validate_handle(3)
    with pytest.raises(ValueError, match="invalid"):
        a._validate_handle(BlockHandle(INVALID_BLOCK))
    with pytest.raises(ValueError, match="out of range"):
        a._validate_handle(BlockHandle(8))
    a._validate_handle(BlockHandle(7))
