"""The product pool (AgentKVPool on a B200) against the reference's fixtures.

* Recorded tree traces (create_root / fork / allocate_block /
  ensure_mutable_block / commit_prefix / free / match_prefix / zero_block,
  with errors) replayed on a CUDA pool seeded with the same contents: every
  result, block table, tree node, refcount, free-list entry and final block
  digest must match.
* The quickstart workload: block tables, CoW pairs, refcounts, match results
  and pool bytes.
* The Tree-of-Thought fan-out on the full 60,000-block pool, through the
  single-op API and through the batched API.
* match_prefix on the stress tree: device results equal the reference's
  (node, length) for every query, and the oracle's comparison counts.
"""

import hashlib
import json

import numpy as np
import pytest
import torch

from agentkv_b200 import AgentKVPool, PoolConfig
from agentkv_b200 import _native as N
from agentkv_b200 import workloads as W
from agentkv_b200.allocator import BlockHandle
from oracle import oracle as O

pytestmark = pytest.mark.gpu

T_CREATE, T_FORK, T_ALLOC, T_COW, T_APPEND, T_COMMIT, T_FREE, T_MATCH, T_ADVANCE, T_ZERO = range(10)


def pool_digests(pool: AgentKVPool, as_int16=False):
    kv = pool._allocator._kv_data
    n = kv.shape[0]
    raw = kv.view(torch.int16) if as_int16 else kv
    host = raw.cpu().numpy()
    return [hashlib.sha256(host[i].tobytes()).hexdigest() for i in range(n)]


def tree_nodes(pool: AgentKVPool) -> dict:
    return {
        str(nid): {"parent": n.parent_id, "edge": n.edge_tokens, "blocks": [b.block_id for b in n.blocks],
                   "children": sorted([int(k), int(v)] for k, v in n.children.items()), "ref": n.ref_count}
        for nid, n in sorted(pool._tree._shared_nodes.items())
    }


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_reference_tree_trace(golden_dir, seed):
    g = json.loads((golden_dir / f"tree_trace_{seed}.json").read_text())
    n, bs = g["n_blocks"], g["block_size"]
    cfg = PoolConfig(total_blocks=n, block_size=bs, num_layers=1, num_kv_heads=2, head_dim=4,
                     dtype="float16", device="cuda", epoch_interval=7)
    pool = AgentKVPool(config=cfg)
    torch.manual_seed(seed)
    pool._allocator._kv_data.copy_(torch.randn(pool._allocator._kv_data.shape, dtype=torch.float32).half())
    live = {}
    states = {step: st for step, st in g["states"]}
    for step, rec in enumerate(g["ops"]):
        op = rec["op"]
        err = None
        try:
            if op == T_CREATE:
                h = pool.create_root(rec["tokens"])
                live[h.handle_id] = h
                assert [h.handle_id, h.shared_node_id, h.shared_match_len] == rec["out"]
            elif op == T_FORK:
                c = pool.fork(live[rec["h"]])
                live[c.handle_id] = c
                assert c.handle_id == rec["out"]
            elif op == T_ALLOC:
                h = live[rec["h"]]
                pool.allocate_block(h)
                assert h.residual_blocks[-1].block_id == rec["out"]
            elif op == T_COW:
                h = live[rec["h"]]
                pool.ensure_mutable_block(h, rec["idx"])
                assert h.residual_blocks[rec["idx"]].block_id == rec["out"]
            elif op == T_APPEND:
                pool.append_tokens(live[rec["h"]], rec["tokens"])
            elif op == T_COMMIT:
                h = live[rec["h"]]
                pool.commit_prefix(h, rec["length"])
                assert [h.shared_node_id, h.shared_match_len] == rec["out"]
            elif op == T_FREE:
                pool.free(live.pop(rec["h"]))
            elif op == T_MATCH:
                mh, mlen = pool._tree.match_prefix(rec["tokens"])
                got = [-1 if mh is None else mh.handle_id, mlen, -1 if mh is None else mh.shared_node_id]
                assert got == rec["out"]
                if mh is not None:
                    live[mh.handle_id] = mh
            elif op == T_ADVANCE:
                pool.maybe_advance_epoch()
            elif op == T_ZERO:
                pool._allocator.zero_block(BlockHandle(rec["block"]))
        except (ValueError, MemoryError) as e:
            err = e
        assert (err is not None) == ("error" in rec), f"step {step}: {rec} -> {err!r}"
        if step in states:
            st = states[step]
            assert {str(k): pool.get_block_ids(h) for k, h in sorted(live.items())} == st["tables"]
            assert {str(k): [h.shared_node_id, h.shared_match_len] for k, h in sorted(live.items())} == st["shared"]
            assert tree_nodes(pool) == st["nodes"]
            assert pool._allocator.ref_counts().tolist() == st["ref"]
            assert pool._allocator.free_list().tolist() == st["free"]
            s = pool.stats()
            for k, v in st["stats"].items():
                assert s[k] == v, (k, s[k], v)
    assert pool_digests(pool) == g["block_sha256"]


def test_quickstart_workload(golden_dir):
    g = json.loads((golden_dir / "quickstart.json").read_text())
    N_, bs, L, H, D, dt = W.QUICKSTART_GEOMETRY
    cfg = PoolConfig(total_blocks=N_, block_size=bs, num_layers=L, num_kv_heads=H, head_dim=D, dtype=dt,
                     device="cuda")
    pool = AgentKVPool(config=cfg)
    torch.manual_seed(0)
    pool._allocator._kv_data.copy_(torch.randn(pool._allocator._kv_data.shape, dtype=torch.float16))
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
    assert pool._allocator.ref_counts().tolist() == g["ref"]
    assert pool._allocator.free_list().tolist() == g["free"]
    assert pool_digests(pool) == g["block_sha256"]
    s = pool.stats()
    for k, v in g["stats"].items():
        assert s[k] == v, k


def _tot_pool():
    N_, bs, L, H, D, dt = W.LLAMA3_8B_GEOMETRY
    cfg = PoolConfig(total_blocks=N_, block_size=bs, num_layers=L, num_kv_heads=H, head_dim=D, dtype=dt,
                     device="meta")
    return AgentKVPool(config=cfg)


def _check_tot(pool, g, kids):
    tables = np.concatenate([np.asarray(pool.get_block_ids(c), np.int32) for c in kids])
    np.testing.assert_array_equal(tables, g["tables"])
    np.testing.assert_array_equal(pool._allocator.ref_counts(), g["ref_fanout"])
    np.testing.assert_array_equal(pool._allocator.free_list(), g["free_fanout"])
    st = json.loads(str(g["stats_fanout"]))
    s = pool.stats()
    for k in ("free_blocks", "allocated_blocks", "peak_allocated", "total_allocs", "epoch", "active_handles"):
        assert s[k] == st[k], k


@pytest.mark.slow
def test_tot_single_op_api(golden_dir):
    g = np.load(golden_dir / "tot_8b.npz")
    spec = W.ToTSpec()
    pool = _tot_pool()
    root = pool.create_root(W.tot_root_tokens(spec))
    for _ in range(spec.root_tokens // 16):
        pool.allocate_block(root)
    level, kids = [root], []
    for lvl in range(spec.levels):
        nxt = []
        for pi, parent in enumerate(level):
            for k in range(spec.fanout):
                c = pool.fork(parent)
                pool.ensure_mutable_block(c, len(c.residual_blocks) - 1)
                pool.append_tokens(c, W.tot_append_tokens(spec, lvl, pi * spec.fanout + k))
                for _ in range(spec.appended_blocks):
                    pool.allocate_block(c)
                nxt.append(c)
        kids.extend(nxt)
        level = nxt
    _check_tot(pool, g, kids)
    for c in kids:
        pool.free(c)
    np.testing.assert_array_equal(pool._allocator.ref_counts(), g["ref_freed"])
    np.testing.assert_array_equal(pool._allocator.free_list(), g["free_freed"])


def test_tot_batched_api(golden_dir):
    """Same fan-out with one launch per batch: fork_many, ensure_mutable_batch,
    allocate_blocks, free_many."""
    g = np.load(golden_dir / "tot_8b.npz")
    spec = W.ToTSpec()
    pool = _tot_pool()
    root = pool.create_root(W.tot_root_tokens(spec))
    pool.allocate_blocks(root, spec.root_tokens // 16)
    level, kids = [root], []
    for lvl in range(spec.levels):
        nxt = []
        for parent in level:
            nxt.extend(pool.fork_many(parent, spec.fanout))
        # CoW and appends keep the reference's per-child order: child c's CoW
        # id, then its appended ids, then child c + 1.
        for c in nxt:
            pool.ensure_mutable_batch([(c, len(c.residual_blocks) - 1)])
            pool.allocate_blocks(c, spec.appended_blocks)
        kids.extend(nxt)
        level = nxt
    _check_tot(pool, g, kids)
    pool.free_many(kids)
    np.testing.assert_array_equal(pool._allocator.ref_counts(), g["ref_freed"])
    np.testing.assert_array_equal(pool._allocator.free_list(), g["free_freed"])


def _build_match_tree(spec, total_blocks):
    prefixes = W.match_prefixes(spec)
    corpus = W.match_sequences(spec, prefixes)
    cfg = PoolConfig(total_blocks=total_blocks, block_size=16, num_layers=1, num_kv_heads=1, head_dim=1,
                     dtype="float16", device="meta")
    pool = AgentKVPool(config=cfg)
    for seq in corpus:
        h = pool.create_root(seq)
        need = -(-len(seq) // 16) - len(pool.get_block_ids(h))
        pool.allocate_blocks(h, need)
        share = (len(seq) // 16) * 16 - h.shared_match_len
        if share > 0:
            pool.commit_prefix(h, share)
    return pool, prefixes, corpus


@pytest.mark.parametrize("name", ["match_small", pytest.param("match_full", marks=pytest.mark.slow)])
def test_match_prefix_stress_tree(golden_dir, name):
    g = np.load(golden_dir / f"{name}.npz")
    spec = W.MatchSpec(**json.loads(str(g["spec"])))
    pool, prefixes, corpus = _build_match_tree(spec, int(g["total_blocks"]))
    assert len(pool._tree._shared_nodes) == int(g["n_nodes"])
    assert pool._tree._next_node_id == int(g["next_node_id"])
    assert pool.free_blocks == int(g["free_blocks"])
    queries = W.match_queries(spec, corpus, prefixes, batch=0, n=len(g["node"]))
    node, mlen, cmp_ = pool.match_prefix_batch(queries, with_compared=True)
    np.testing.assert_array_equal(node, g["node"])
    np.testing.assert_array_equal(mlen, g["len"])
    # single-query path agrees with the batch
    for i, q in enumerate(queries[:16]):
        want = (int(node[i]), int(mlen[i])) if mlen[i] else (-1, 0)
        assert pool._tree._match_prefix_locked(q) == want
    # comparison counts equal the oracle's restatement over the same tree
    otree = _oracle_tree_from(pool)
    flat, q_off = O.pack_queries([q.tolist() for q in queries])
    on, ol, oc = O.match_prefix_csr(otree, flat, q_off, 16)
    np.testing.assert_array_equal(on, node)
    np.testing.assert_array_equal(ol, mlen)
    np.testing.assert_array_equal(oc, cmp_)
    # one hash probe per hop (no unary-chain runs): the same answers
    from agentkv_b200.device_tree import match_batch

    # with one hash probe per hop (no unary-chain runs), with one warp per
    # query, and split into short ranges at every verify width: the same
    # answers and comparison counts
    P, F = N.MATCH_PIPELINED, N.MATCH_PREFETCH
    for runs, split, tpi, chunks in ((False, True, 0, 0), (True, False, 0, 0), (False, False, 0, 4),
                                     (True, True, 32, 1), (True, True, 64, 2), (False, True, 96, 4),
                                     (True, True, 256, 8), (True, True, 512, 16), (True, True, 2048, 8),
                                     (True, False, 0, 4 | P), (False, False, 0, 8 | P | F), (True, True, 64, 2 | P),
                                     (True, True, 128, 8 | F), (True, False, 0, F), (True, False, 0, 16 | F)):
        hn, hl, hc = match_batch(pool._tree._dev_tree, queries, 16, with_compared=True, runs=runs,
                                 split=split, tokens_per_range=tpi, chunks=chunks)
        tag = f"runs={runs} split={split} tokens_per_range={tpi} chunks={chunks}"
        np.testing.assert_array_equal(hn, node, err_msg=tag)
        np.testing.assert_array_equal(hl, mlen, err_msg=tag)
        np.testing.assert_array_equal(hc, cmp_, err_msg=tag)
    # the staged lookup (chase, then windows over the grid) at every window size
    for runs, window in ((True, 0), (False, 0), (True, 256), (True, 1024), (False, 512)):
        hn, hl, hc = match_batch(pool._tree._dev_tree, queries, 16, with_compared=True, runs=runs,
                                 staged=True, window_tokens=window)
        tag = f"staged runs={runs} window={window}"
        np.testing.assert_array_equal(hn, node, err_msg=tag)
        np.testing.assert_array_equal(hl, mlen, err_msg=tag)
        np.testing.assert_array_equal(hc, cmp_, err_msg=tag)


def _oracle_tree_from(pool) -> dict:
    """CSR arrays of the product tree for the oracle's C match."""
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
    return {"child_ptr": child_ptr, "child_key": np.asarray(keys or [0], np.int32),
            "child_id": np.asarray(ids or [0], np.int32), "edge_off": edge_off, "edge_len": edge_len,
            "edge_tokens": np.concatenate(toks) if pos else np.zeros(1, np.int32)}


def test_match_edge_cases():
    cfg = PoolConfig(total_blocks=64, block_size=4, num_layers=1, num_kv_heads=1, head_dim=1,
                     dtype="float16", device="meta")
    pool = AgentKVPool(config=cfg)
    # empty tree, empty query, single token
    assert pool._tree._match_prefix_locked([]) == (-1, 0)
    assert pool._tree._match_prefix_locked([5]) == (-1, 0)
    h = pool.create_root(list(range(12)))
    pool.allocate_blocks(h, 3)
    pool.commit_prefix(h, 8)
    # exact, longer, partial edge (no credit), mismatch at first token
    assert pool._tree._match_prefix_locked(list(range(8)))[1] == 8
    assert pool._tree._match_prefix_locked(list(range(20)))[1] == 8
    assert pool._tree._match_prefix_locked(list(range(7))) == (-1, 0)
    assert pool._tree._match_prefix_locked([1, 2, 3]) == (-1, 0)
    # a non-aligned edge (commit with fewer tokens than blocks) is floored
    h2 = pool.create_root([100, 101, 102])
    pool.allocate_blocks(h2, 2)
    pool.commit_prefix(h2, 8)  # edge holds only 3 tokens
    assert pool._tree._match_prefix_locked([100, 101, 102, 9]) == (-1, 0)
    node, mlen = pool.match_prefix_batch([[100, 101, 102], list(range(9)), []])
    assert mlen.tolist() == [0, 8, 0]
    # split lookups: empty queries, lengths at and across range boundaries
    from agentkv_b200.device_tree import match_batch

    qs = [[], list(range(32)), list(range(12)) + [7] * 52, [100, 101, 102], list(range(8)) + [5] * 56, [0]]
    for tpi in (0, 32, 64):
        node, mlen, cmp_ = match_batch(pool._tree._dev_tree, qs, 4, with_compared=True, split=True,
                                       tokens_per_range=tpi)
        w_node, w_len, w_cmp = match_batch(pool._tree._dev_tree, qs, 4, with_compared=True, split=False)
        assert mlen.tolist() == w_len.tolist() == [0, 8, 8, 0, 8, 0], tpi
        assert cmp_.tolist() == w_cmp.tolist(), tpi
        assert [n if m else -1 for n, m in zip(node, mlen)] == [n if m else -1 for n, m in zip(w_node, w_len)]
    # staged lookups: the same queries, and one whose followed path ends in a
    # partly fitting edge
    for window in (256, 512, 1024):
        node, mlen, cmp_ = match_batch(pool._tree._dev_tree, qs + [list(range(6))], 4, with_compared=True,
                                       staged=True, window_tokens=window)
        w_node, w_len, w_cmp = match_batch(pool._tree._dev_tree, qs + [list(range(6))], 4, with_compared=True)
        assert mlen.tolist() == w_len.tolist() == [0, 8, 8, 0, 8, 0, 0], window
        assert w_cmp[-1] == 6, w_cmp
        assert cmp_.tolist() == w_cmp.tolist(), window
        assert [n if m else -1 for n, m in zip(node, mlen)] == [n if m else -1 for n, m in zip(w_node, w_len)]


def test_split_match_rejects_a_plan_that_disagrees_with_the_order():
    """A range plan that gives a query fewer or more ranges than its length
    needs (here: a plan for two 10-token queries while one is 40 tokens
    long, then a correct one): the split lookup reports it in the tree's
    status, writes no answer for that query, and the next lookup works."""
    import torch

    cfg = PoolConfig(total_blocks=64, block_size=4, num_layers=1, num_kv_heads=1, head_dim=1,
                     dtype="float16", device="meta")
    pool = AgentKVPool(config=cfg)
    h = pool.create_root(list(range(12)))
    pool.allocate_blocks(h, 3)
    pool.commit_prefix(h, 8)
    t = pool._tree._dev_tree
    dev = t.device
    from agentkv_b200.device_tree import split_plan

    tok = torch.arange(50, dtype=torch.int32, device=dev)
    off = torch.tensor([0, 10, 50], dtype=torch.int64, device=dev)  # query 0: 10 tokens, query 1: 40
    order = torch.tensor([1, 0], dtype=torch.int32, device=dev)  # longest first
    node = torch.full((2,), 7, dtype=torch.int32, device=dev)
    mlen = torch.full((2,), 7, dtype=torch.int32, device=dev)
    # a plan for two 10-token queries: query 1 needs two 32-token ranges
    t.match(tok, off, 2, 4, node, mlen, None, order=order, plan=split_plan([10, 10], 32))
    with pytest.raises(RuntimeError, match="invalid argument"):
        t.check()
    assert node[1].item() == 7 and mlen[1].item() == 7  # no answer for the mis-planned query
    assert mlen[0].item() == 8  # the other query is answered
    t.match(tok, off, 2, 4, node, mlen, None, order=order, plan=split_plan([40, 10], 32))
    t.check()
    assert mlen.tolist() == [8, 0]


@pytest.mark.parametrize("mode", ["tree", "levels"])
def test_tot_device_tables(golden_dir, mode):
    """The device-resident fan-out (SlabAllocator.fanout_tree / fanout_level)
    ends in the reference's state: child tables, pairs, refcounts, free list,
    and after freeing every child in creation order the same again."""
    g = np.load(golden_dir / "tot_8b.npz")
    spec = W.ToTSpec()
    pool = _tot_pool()
    a = pool._allocator
    roots = a.alloc_batch(spec.root_tokens // 16)
    if mode == "tree":
        res = a.fanout_tree(roots, [spec.root_tokens // 16], spec.levels, spec.fanout, spec.appended_blocks)
        tables, pairs = res["child_tables"], res["pairs"]
    else:
        tables, pairs = [], []
        t, lens = roots, np.array([spec.root_tokens // 16])
        for _ in range(spec.levels):
            off = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)])).to(a.device)
            r = a.fanout_level(t, off, lens, spec.fanout, spec.appended_blocks)
            tables.append(r["child_tables"])
            pairs.append(r["pairs"])
            t, lens = r["child_tables"], r["child_lens"]
    a.check()
    np.testing.assert_array_equal(torch.cat(tables).cpu().numpy(), g["tables"])
    for lvl in range(3):
        np.testing.assert_array_equal(pairs[lvl].cpu().numpy(), g[f"pairs_l{lvl}"])
    np.testing.assert_array_equal(a.ref_counts(), g["ref_fanout"])
    np.testing.assert_array_equal(a.free_list(), g["free_fanout"])
    st = json.loads(str(g["stats_fanout"]))
    s = a.stats()
    for k in ("free_blocks", "allocated_blocks", "peak_allocated", "total_allocs", "epoch"):
        assert s[k] == st[k], k
    a.dec_ref_batch(torch.cat(tables))
    a.check()
    np.testing.assert_array_equal(a.ref_counts(), g["ref_freed"])
    np.testing.assert_array_equal(a.free_list(), g["free_freed"])
    st = json.loads(str(g["stats_freed"]))
    s = a.stats()
    for k in ("free_blocks", "allocated_blocks", "total_frees", "epoch"):
        assert s[k] == st[k], k


def test_tot_fanout_copies_data():
    """fanout_level with a real pool copies each child's CoW block bit-exactly."""
    cfg = PoolConfig(total_blocks=400, block_size=16, num_layers=2, num_kv_heads=2, head_dim=64,
                     dtype="bfloat16", device="cuda")
    pool = AgentKVPool(config=cfg)
    a = pool._allocator
    a._kv_data.view(torch.int16).random_(-30000, 30000)
    roots = a.alloc_batch(6)
    off = torch.tensor([0, 3, 6], dtype=torch.int64, device=a.device)
    before = a._kv_data.clone()
    r = a.fanout_level(roots, off, [3, 3], 4, 2)
    a.check()
    pairs = r["pairs"].cpu().numpy()
    assert len(pairs) == 8
    for s_, d_ in pairs:
        assert torch.equal(a._kv_data[d_].view(torch.int16), before[s_].view(torch.int16))


def test_match_with_colliding_child_keys():
    """24 root children whose (parent, first token) keys share the low ten
    hash bits, so they sit in one probe chain several 8-slot windows long:
    every inserted sequence is found, and first tokens that join the chain
    without being in the tree are reported absent (the walk runs to the
    chain's empty slot), equal to the oracle's answers."""
    from agentkv_b200.device_tree import tree_hash_np

    toks = np.arange(1, 200000, dtype=np.int64)
    h = tree_hash_np(np.zeros_like(toks), toks)
    same = toks[(h & 1023) == (h[0] & 1023)]
    firsts, absent = same[:24].tolist(), same[24:30].tolist()
    cfg = PoolConfig(total_blocks=512, block_size=4, num_layers=1, num_kv_heads=1, head_dim=4,
                     dtype="float16", device="meta")
    pool = AgentKVPool(config=cfg)
    ot = O.OracleTree(O.OracleAllocator(512), 4)
    rng = np.random.default_rng(5)
    seqs = []
    for f in firsts:
        seq = [int(f)] + rng.integers(0, 50000, size=11).tolist()
        seqs.append(seq)
        for tree, api in ((pool, "pool"), (ot, "oracle")):
            hd = tree.create_root(seq)
            if api == "pool":
                tree.allocate_blocks(hd, 3)
            else:
                for _ in range(3):
                    tree.allocate_block(hd)
            tree.commit_prefix(hd, 12)
    queries = [s + [7, 7, 7] for s in seqs] + [[a] + seqs[0][1:] for a in absent] + [s[:8] for s in seqs[:4]]
    node, mlen = pool.match_prefix_batch(queries)
    want = [ot.match(q)[:2] for q in queries]
    assert [(int(n) if m else -1, int(m)) for n, m in zip(node, mlen)] == \
        [(int(n) if m else -1, int(m)) for n, m in want]
    assert all(int(m) == 12 for m in mlen[:24])
    assert all(int(m) == 0 for m in mlen[24:30])


def test_match_long_unary_chains():
    """A 70-node unary chain (prefixes of one sequence committed one block
    longer each time) with a branch at depth 100: queries cut at every
    depth, diverging at every third position (on an edge's first token and
    inside edges) and running past the chain's end give the oracle's
    (node, length, tokens compared), with the unary-chain runs (up to 32 hops
    per load, across the 32-hop segment boundary) and with one hash probe
    per hop; one warp per query and split into ranges of 32 to 96 tokens
    (stops at range boundaries, ranges past the walk's end)."""
    from agentkv_b200.device_tree import match_batch

    bs = 4
    cfg = PoolConfig(total_blocks=1024, block_size=bs, num_layers=1, num_kv_heads=1, head_dim=4,
                     dtype="float16", device="meta")
    pool = AgentKVPool(config=cfg)
    ot = O.OracleTree(O.OracleAllocator(1024), bs)
    rng = np.random.default_rng(23)
    seq = rng.integers(0, 50000, size=70 * bs).tolist()
    branch = seq[:100] + rng.integers(50000, 60000, size=40).tolist()
    for s in [seq[: bs * k] for k in range(1, 71)] + [branch]:
        for tree, api in ((pool, "pool"), (ot, "oracle")):
            hd = tree.create_root(s)
            need = -(-len(s) // bs)
            if api == "pool":
                tree.allocate_blocks(hd, need - len(tree.get_block_ids(hd)))
            else:
                while len(tree.get_block_ids(hd)) < need:
                    tree.allocate_block(hd)
            tree.commit_prefix(hd, len(s) - hd.shared_match_len)
    queries = [seq[:n] for n in range(0, len(seq) + 1)] + [seq + [1, 2, 3], branch + [9], branch[:103]]
    for p in range(0, len(seq), 3):
        q = list(seq)
        q[p] = 99999
        queries.append(q)
    dev_tree = pool._tree._dev_tree
    want = [ot.match(q) for q in queries]
    for runs, split, tpi in ((True, True, 0), (False, True, 0), (True, False, 0), (False, False, 0),
                             (True, True, 32), (False, True, 32), (True, True, 64), (True, True, 96)):
        node, mlen, cmp_ = match_batch(dev_tree, queries, bs, with_compared=True, runs=runs, split=split,
                                       tokens_per_range=tpi)
        got = [(int(n) if m else -1, int(m), int(c)) for n, m, c in zip(node, mlen, cmp_)]
        assert got == [(int(n) if m else -1, int(m), int(c)) for n, m, c in want], (runs, split, tpi)
    for runs, window in ((True, 256), (False, 256), (True, 512), (True, 1024)):
        node, mlen, cmp_ = match_batch(dev_tree, queries, bs, with_compared=True, runs=runs, staged=True,
                                       window_tokens=window)
        got = [(int(n) if m else -1, int(m), int(c)) for n, m, c in zip(node, mlen, cmp_)]
        assert got == [(int(n) if m else -1, int(m), int(c)) for n, m, c in want], ("staged", runs, window)
    assert dev_tree.d_run_head is not None and int((dev_tree.d_run_head >= 0).sum()) >= 60


def test_match_prefix_many_equals_one_by_one(golden_dir):
    """AgentKVPool.match_prefix_many (one lookup launch) gives the handles,
    shared-node refcounts and allocator state of match_prefix called on each
    query in turn, on the device pool."""
    g = np.load(golden_dir / "match_small.npz")
    spec = W.MatchSpec(**json.loads(str(g["spec"])))
    pools = [_build_match_tree(spec, int(g["total_blocks"]))[0] for _ in range(2)]
    prefixes = W.match_prefixes(spec)
    corpus = W.match_sequences(spec, prefixes)
    queries = W.match_queries(spec, corpus, prefixes, batch=0, n=200)
    a, b = pools
    many = a.match_prefix_many(queries)
    one = [b._tree.match_prefix(q) for q in queries]
    assert sum(1 for h, _ in many if h is not None) > 20
    for (h1, m1), (h2, m2) in zip(many, one):
        assert m1 == m2 and (h1 is None) == (h2 is None)
        if h1 is not None:
            assert (h1.handle_id, h1.shared_node_id) == (h2.handle_id, h2.shared_node_id)
    assert {k: n.ref_count for k, n in a._tree._shared_nodes.items()} == \
        {k: n.ref_count for k, n in b._tree._shared_nodes.items()}
    np.testing.assert_array_equal(a._allocator.free_list(), b._allocator.free_list())
    np.testing.assert_array_equal(a._allocator.ref_counts(), b._allocator.ref_counts())


@pytest.mark.parametrize("name", ["colliding", "long_chain"])
def test_match_scenarios_match_reference(golden_dir, name):
    """The hard lookup shapes of tests/match_scenarios.py on the device pool,
    with the unary-chain runs and with one probe per hop: the reference's
    recorded (node, length) per query, whole and split into 32-token ranges."""
    from agentkv_b200.device_tree import match_batch
    from match_scenarios import SCENARIOS, build

    want = json.loads((golden_dir / "match_scenarios.json").read_text())[name]
    sc = SCENARIOS[name]()
    pool = AgentKVPool(config=PoolConfig(total_blocks=1024, block_size=sc["block_size"], num_layers=1,
                                         num_kv_heads=1, head_dim=4, dtype="float16", device="meta"))
    build(pool, sc, pool.allocate_block)
    for runs, split, tpi in ((True, True, 0), (False, True, 0), (True, False, 0), (False, True, 32),
                             (True, True, 32)):
        node, mlen = match_batch(pool._tree._dev_tree, sc["queries"], sc["block_size"], runs=runs,
                                 split=split, tokens_per_range=tpi)
        assert [[int(n) if m else -1, int(m)] for n, m in zip(node, mlen)] == want, (runs, split, tpi)
    for runs, window in ((True, 256), (False, 512)):
        node, mlen = match_batch(pool._tree._dev_tree, sc["queries"], sc["block_size"], runs=runs, staged=True,
                                 window_tokens=window)
        assert [[int(n) if m else -1, int(m)] for n, m in zip(node, mlen)] == want, ("staged", runs, window)
