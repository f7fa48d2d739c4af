"""The oracle (CPU restatement) against fixtures produced by the reference.

Every fixture under tests/golden/ was recorded by running the reference
implementation (tests/golden/make_golden.py).  These tests replay the same
inputs through the oracle and require identical results: ids, refcounts,
free-list order, reclaimer queues, counters, block tables, tree structure,
match results and block contents.
"""

import hashlib
import json

import numpy as np
import pytest
import torch

from oracle import oracle as O
from agentkv_b200 import workloads as W

A_ALLOC, A_INC, A_DEC, A_ENTER, A_LEAVE, A_ADVANCE = range(6)


def ragged(d, key, i):
    off = d[key + "_off"]
    return d[key][off[i] : off[i + 1]]


@pytest.mark.parametrize("seed", [1, 2, 3, 4])
def test_oracle_allocator_trace(golden_dir, seed):
    d = np.load(golden_dir / f"alloc_trace_{seed}.npz")
    a = O.OracleAllocator(int(d["n_blocks"]), int(d["interval"]))
    for i, (op, arg, want) in enumerate(zip(d["ops"], d["args"], d["results"])):
        if op == A_ALLOC:
            try:
                got = a.alloc()
            except O.OracleError as e:
                got = -e.code
        elif op in (A_INC, A_DEC):
            try:
                got = 0 if op == A_INC else int(a.dec_ref(int(arg)))
                if op == A_INC:
                    a.inc_ref(int(arg))
            except O.OracleError as e:
                got = -e.code
        elif op == A_ENTER:
            got = a.enter_read_section()
        elif op == A_LEAVE:
            a.leave_read_section(int(arg))
            got = 0
        else:
            a.maybe_advance_epoch()
            got = 0
        assert got == want, f"op {i} ({op}, {arg})"
        s = a.state()
        np.testing.assert_array_equal(s["ref_counts"], d["ref"][i], err_msg=f"ref after op {i}")
        np.testing.assert_array_equal(s["free_list"], ragged(d, "free", i), err_msg=f"free after op {i}")
        np.testing.assert_array_equal(s["pending"], ragged(d, "pend_ids", i))
        np.testing.assert_array_equal(s["pending_epochs"], ragged(d, "pend_eps", i))
        np.testing.assert_array_equal(s["deferred"], ragged(d, "deferred", i))
        c = d["ctl"][i]
        assert [s["op_count"], s["epoch"], s["total_allocs"], s["total_frees"], s["peak_allocated"],
                s["epoch_advances"], s["blocks_freed"], len(s["free_list"]), s["allocated_blocks"]] == list(c)


def _pool_bytes(n, shape, dtype, seed_fill):
    return seed_fill


def test_oracle_quickstart(golden_dir):
    g = json.loads((golden_dir / "quickstart.json").read_text())
    N_, bs, L, H, D, dt = W.QUICKSTART_GEOMETRY
    torch.manual_seed(0)
    kv = torch.randn((N_, L, 2, H, bs, D), dtype=torch.float16).numpy()
    pool = kv.view(np.uint8).reshape(N_, -1).copy()
    bpb = pool.shape[1]
    a = O.OracleAllocator(N_)
    pairs = []

    def cp(s, t):
        pairs.append([s, t])
        O.copy_blocks(pool, bpb, np.array([[s, t]], np.int32))

    tree = O.OracleTree(a, bs, copy_cb=cp)
    root = tree.create_root(list(range(32)))
    tree.allocate_block(root)
    kids = [tree.fork(root) for _ in range(3)]
    for c in kids:
        tree.allocate_block(c)
    for c in kids:
        tree.ensure_mutable_block(c, 0)
    tree.commit_prefix(root, 16)
    matches = []
    for q in g["queries"]:
        h, mlen = tree.match_prefix(q)
        matches.append([-1 if h is None else h.shared_node_id, mlen])
    assert [tree.get_block_ids(c) for c in kids] == g["children"]
    assert tree.get_block_ids(root) == g["root"]
    assert pairs == g["pairs"]
    assert matches == g["matches"]
    s = a.state()
    assert s["ref_counts"].tolist() == g["ref"]
    assert s["free_list"].tolist() == g["free"]
    assert [hashlib.sha256(pool[i].tobytes()).hexdigest() for i in range(N_)] == g["block_sha256"]


T_CREATE, T_FORK, T_ALLOC, T_COW, T_APPEND, T_COMMIT, T_FREE, T_MATCH, T_ADVANCE, T_ZERO = range(10)


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_oracle_tree_trace(golden_dir, seed):
    g = json.loads((golden_dir / f"tree_trace_{seed}.json").read_text())
    n, bs = g["n_blocks"], g["block_size"]
    torch.manual_seed(seed)
    kv = torch.randn((n, 1, 2, 2, bs, 4), dtype=torch.float32).half().numpy()
    pool = kv.view(np.uint8).reshape(n, -1).copy()
    bpb = pool.shape[1]
    a = O.OracleAllocator(n, 7)
    tree = O.OracleTree(a, bs, copy_cb=lambda s, t: O.copy_blocks(pool, bpb, np.array([[s, t]], np.int32)))
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
                assert tree.allocate_block(live[rec["h"]]) == rec["out"]
            elif op == T_COW:
                assert tree.ensure_mutable_block(live[rec["h"]], rec["idx"]) == rec["out"]
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
                a.maybe_advance_epoch()
            elif op == T_ZERO:
                b = rec["block"]
                if a.ref_count(b) != 1:
                    raise ValueError("not exclusive")
                O.zero_blocks(pool, bpb, np.array([b], np.int32))
        except (ValueError, O.OracleError) as e:
            err = e
        assert (err is not None) == ("error" in rec), f"step {step}: {rec} -> {err!r}"
        if step in states:
            st = states[step]
            assert {str(k): tree.get_block_ids(h) for k, h in sorted(live.items())} == st["tables"]
            assert {str(k): [h.shared_node_id, h.shared_match_len] for k, h in sorted(live.items())} == st["shared"]
            nodes = {str(nid): {"parent": nd.parent_id, "edge": list(nd.edge), "blocks": list(nd.blocks),
                                "children": sorted([int(k), int(v)] for k, v in nd.children.items()),
                                "ref": nd.ref_count} for nid, nd in sorted(tree.nodes.items())}
            assert nodes == st["nodes"]
            s = a.state()
            assert s["ref_counts"].tolist() == st["ref"]
            assert s["free_list"].tolist() == st["free"]
    assert [hashlib.sha256(pool[i].tobytes()).hexdigest() for i in range(n)] == g["block_sha256"]


def test_oracle_tot_metadata(golden_dir):
    g = np.load(golden_dir / "tot_8b.npz")
    N_, bs = W.LLAMA3_8B_GEOMETRY[:2]
    spec = W.ToTSpec()
    a = O.OracleAllocator(N_)
    pairs = []
    tree = O.OracleTree(a, bs, copy_cb=lambda s, t: pairs.append((s, t)))
    root = tree.create_root(W.tot_root_tokens(spec))
    for _ in range(spec.root_tokens // bs):
        tree.allocate_block(root)
    level, kids = [root], []
    for lvl in range(spec.levels):
        nxt = []
        for parent in level:
            for _ in range(spec.fanout):
                c = tree.fork(parent)
                tree.ensure_mutable_block(c, len(c.residual) - 1)
                for _ in range(spec.appended_blocks):
                    tree.allocate_block(c)
                nxt.append(c)
        kids.extend(nxt)
        level = nxt
    tables = np.concatenate([np.asarray(tree.get_block_ids(c), np.int32) for c in kids])
    np.testing.assert_array_equal(tables, g["tables"])
    np.testing.assert_array_equal(np.asarray(pairs, np.int32),
                                  np.concatenate([g["pairs_l0"], g["pairs_l1"], g["pairs_l2"]]))
    s = a.state()
    np.testing.assert_array_equal(s["ref_counts"], g["ref_fanout"])
    np.testing.assert_array_equal(s["free_list"], g["free_fanout"])
    for c in kids:
        tree.free(c)
    s = a.state()
    np.testing.assert_array_equal(s["ref_counts"], g["ref_freed"])
    np.testing.assert_array_equal(s["free_list"], g["free_freed"])
    st = json.loads(str(g["stats_freed"]))
    assert s["epoch"] == st["epoch"] and s["total_frees"] == st["total_frees"]


def test_oracle_react_trace(golden_dir):
    """The ReAct multi-agent trace (70B geometry, 40,000 blocks, 32 agents,
    1000 steps): every step's CoW pairs, and at the checkpoints the agents'
    block tables, refcounts, free list and counters, equal the reference's."""
    from react_apis import OracleReActAPI

    g = np.load(golden_dir / "react_70b.npz")
    spec = W.ReActSpec(**json.loads(str(g["spec"])))
    N_, bs = W.LLAMA3_70B_GEOMETRY[:2]
    pairs = []
    api = OracleReActAPI(N_, bs, copy_cb=lambda s, t: pairs.append((s, t)))
    root, agents = W.react_setup(api, spec)
    assert not pairs
    np.testing.assert_array_equal(np.asarray(api.get_block_ids(root), np.int32), g["root_table"])
    so = g["step_off"]
    for i, actions in enumerate(W.react_trace(spec)):
        W.react_step(api, root, agents, actions)
        np.testing.assert_array_equal(np.asarray(pairs[so[i]:], np.int32).reshape(-1, 2),
                                      g["pairs"][so[i]:so[i + 1]], err_msg=f"step {i}")
        k = f"s{i + 1}"
        if k + "_ref" in g.files:
            tables = np.concatenate([np.asarray(api.get_block_ids(h), np.int32) for h in agents])
            np.testing.assert_array_equal(tables, g[k + "_tables"])
            s = api.alloc.state()
            np.testing.assert_array_equal(s["ref_counts"], g[k + "_ref"])
            np.testing.assert_array_equal(s["free_list"], g[k + "_free"])
            st = json.loads(str(g[k + "_stats"]))
            assert (s["epoch"], s["total_allocs"], s["total_frees"], s["peak_allocated"]) == \
                (st["epoch"], st["total_allocs"], st["total_frees"], st["peak_allocated"])


def test_oracle_hf_session(golden_dir):
    """The HF cache session (prefill, commit, forks, decode with CoW): every
    update's K/V output, the final block tables and the final pool bytes
    equal the reference's AgentKVCache on a CPU pool."""
    g = np.load(golden_dir / "hf_session.npz")
    spec = W.HFSpec(**json.loads(str(g["spec"])))
    pool = O.OracleKVPool(spec.total_blocks, spec.block_size, spec.num_layers, spec.num_kv_heads,
                          spec.head_dim, spec.dtype)
    outs, keys = [], []

    def on_output(e, layer, ok, ov):
        keys.append((e, layer, ok.shape[2]))
        outs.append(np.concatenate([ok.reshape(-1), ov.reshape(-1)]))

    caches = W.hf_run(spec, pool, O.OracleKVCache, lambda a: a, on_output)
    np.testing.assert_array_equal(np.asarray(keys), g["out_keys"])
    assert np.concatenate(outs).tobytes() == g["outs"].tobytes()
    tables = np.concatenate([np.asarray(pool.get_block_ids(c.handle), np.int32) for c in caches])
    np.testing.assert_array_equal(tables, g["tables"])
    assert [c.get_seq_length() for c in caches] == g["seen"].tolist()
    assert pool.kv.tobytes() == g["pool"].tobytes()


@pytest.mark.parametrize("seed", [1, 2, 7, 13, 17, 42, 137, 999])
def test_oracle_reference_stress_runner(golden_dir, seed):
    """The reference's own stress runner (tests/test_stress.py, its seeds and
    op counts), recorded call by call: the oracle returns every handle id and
    block id (and every pool-exhausted error) the reference returned, and ends
    with its refcounts, free-list order and counters."""
    from stress_replay import replay

    g = np.load(golden_dir / f"stress_{seed}.npz")
    assert int(g["violations"]) == 0
    a = O.OracleAllocator(512)
    tree = O.OracleTree(a, 4)
    replay(g, tree, a.maybe_advance_epoch,
           lambda e: isinstance(e, O.OracleError) and e.code == O.ORC_ERR_EXHAUSTED)
    s = a.state()
    np.testing.assert_array_equal(s["ref_counts"], g["ref"])
    np.testing.assert_array_equal(s["free_list"], g["free"])
    st = json.loads(str(g["stats"]))
    assert (s["epoch"], s["total_allocs"], s["total_frees"], s["peak_allocated"]) == \
        (st["epoch"], st["total_allocs"], st["total_frees"], st["peak_allocated"])


def test_oracle_copy_zero_contents(golden_dir):
    g = json.loads((golden_dir / "copy_zero.json").read_text())
    torch.manual_seed(g["seed"])
    kv = torch.randn((32, 2, 2, 2, 4, 8), dtype=torch.float32).to(torch.bfloat16)
    kv[3].fill_(-1.5)
    kv[4].fill_(float("nan"))
    pool = kv.view(torch.int16).numpy().view(np.uint8).reshape(32, -1).copy()
    bpb = pool.shape[1]
    for op in g["ops"]:
        if op[0] == "copy":
            O.copy_blocks(pool, bpb, np.array([[op[1], op[2]]], np.int32))
        else:
            O.zero_blocks(pool, bpb, np.array([op[1]], np.int32))
    assert [hashlib.sha256(pool[i].tobytes()).hexdigest() for i in range(32)] == g["block_sha256"]
    assert not pool[3].any() and not pool[4].any()  # +0.0 bits, even from -1.5 and NaN


def test_oracle_match_small(golden_dir):
    g = np.load(golden_dir / "match_small.npz")
    spec = W.MatchSpec(**json.loads(str(g["spec"])))
    prefixes = W.match_prefixes(spec)
    corpus = W.match_sequences(spec, prefixes)
    a = O.OracleAllocator(int(g["total_blocks"]))
    tree = O.OracleTree(a, 16)
    for seq in corpus:
        toks = seq.tolist()
        h = tree.create_root(toks)
        need = -(-len(toks) // 16)
        for _ in range(need - len(tree.get_block_ids(h))):
            tree.allocate_block(h)
        share = (len(toks) // 16) * 16 - h.shared_match_len
        if share > 0:
            tree.commit_prefix(h, share)
    assert len(tree.nodes) == int(g["n_nodes"])
    assert tree.next_node == int(g["next_node_id"])
    assert a.free_count == int(g["free_blocks"])
    queries = W.match_queries(spec, corpus, prefixes, batch=0, n=len(g["node"]))
    py = np.asarray([tree.match(q.tolist())[:2] for q in queries], np.int32)
    np.testing.assert_array_equal(py[:, 0], g["node"])
    np.testing.assert_array_equal(py[:, 1], g["len"])
    flat, q_off = O.pack_queries([q.tolist() for q in queries])
    node, mlen, cmp_ = O.match_prefix_csr(O.tree_csr(tree), flat, q_off, 16)
    np.testing.assert_array_equal(node, g["node"])
    np.testing.assert_array_equal(mlen, g["len"])
    py_cmp = np.asarray([tree.match(q.tolist())[2] for q in queries])
    np.testing.assert_array_equal(cmp_, py_cmp)
    # the pure-Python loop over the flattened tree (the CPU baseline's second figure)
    loop = np.asarray(O.match_prefix_py(O.csr_children(O.tree_csr(tree)), [q.tolist() for q in queries], 16))
    np.testing.assert_array_equal(loop[:, 0], g["node"])
    np.testing.assert_array_equal(loop[:, 1], g["len"])
    np.testing.assert_array_equal(loop[:, 2], cmp_)


@pytest.mark.parametrize("name", ["colliding", "long_chain"])
def test_oracle_match_scenarios(golden_dir, name):
    """The oracle's match on the hard tree shapes of tests/match_scenarios.py
    (a long probe chain of colliding keys, a 70-node unary chain with a
    branch) equals the reference's recorded (node, length) per query."""
    from match_scenarios import SCENARIOS, build

    want = json.loads((golden_dir / "match_scenarios.json").read_text())[name]
    sc = SCENARIOS[name]()
    ot = O.OracleTree(O.OracleAllocator(1024), sc["block_size"])
    build(ot, sc, ot.allocate_block)
    assert [list(ot.match(q)[:2]) for q in sc["queries"]] == want
