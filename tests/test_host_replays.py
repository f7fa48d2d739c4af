"""The package's host-side logic replaying the reference's recorded runs on
CPU: the tree logic (agentkv_b200/radix_tree.py), the pool facade and the
HuggingFace cache, with the allocator answered by the oracle
(oracle_slab.py), the tree kernels by their CPU model
(tree_kernel_model.py) and the KV scatter / gather by their contract in
torch indexing.  Every result, error, block table, tree node, refcount,
free-list entry and byte must be the recorded one; the kernels themselves
are the GPU tests' business."""

import json

import numpy as np
import pytest

from agentkv_b200 import workloads as W
from agentkv_b200.config import PoolConfig


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


def _kv_scatter(kv, slots, layer, k, v, status=None):
    """akv_kv_scatter's contract in torch indexing: token i's rows of every
    head to slot slots[i] (block * block_size + position) of `layer`."""
    bs = kv.shape[4]
    for i, slot in enumerate(slots.tolist()):
        kv[slot // bs, layer, 0, :, slot % bs] = k[0, :, i].to(kv.dtype)
        kv[slot // bs, layer, 1, :, slot % bs] = v[0, :, i].to(kv.dtype)


def _kv_gather(kv, table, layer, n_tokens, status=None):
    """akv_kv_gather's contract: the table's blocks of `layer` as contiguous
    [1, heads, tokens, head_dim] K and V, cut to n_tokens."""
    x = kv[table.long(), layer]  # [blocks, 2, H, bs, D]
    nb, _, h, bs, d = x.shape
    k = x[:, 0].permute(1, 0, 2, 3).reshape(1, h, nb * bs, d)[:, :, :n_tokens]
    v = x[:, 1].permute(1, 0, 2, 3).reshape(1, h, nb * bs, d)[:, :, :n_tokens]
    return k.contiguous(), v.contiguous()


def _hf_cpu_pool(spec, monkeypatch):
    import torch

    from agentkv_b200 import kernels as K

    monkeypatch.setattr(K, "kv_scatter", _kv_scatter)
    monkeypatch.setattr(K, "kv_gather", _kv_gather)
    cfg = PoolConfig(total_blocks=spec.total_blocks, block_size=spec.block_size, num_layers=spec.num_layers,
                     num_kv_heads=spec.num_kv_heads, head_dim=spec.head_dim, dtype=spec.dtype, device="meta")
    kv = torch.zeros((spec.total_blocks, spec.num_layers, 2, spec.num_kv_heads, spec.block_size, spec.head_dim),
                     dtype=getattr(torch, spec.dtype))
    pool = _cpu_pool(cfg, kv, monkeypatch)
    pool._allocator._status = torch.zeros(8, dtype=torch.int32)
    return pool, kv


def _hf_session(spec, pool, cache_cls, to_tensor):
    outs, keys = [], []

    def on_output(e, layer, ok, ov):
        ok = ok.numpy() if hasattr(ok, "numpy") else ok
        ov = ov.numpy() if hasattr(ov, "numpy") else ov
        keys.append((e, layer, ok.shape[2]))
        outs.append(np.concatenate([ok.reshape(-1), ov.reshape(-1)]))

    caches = W.hf_run(spec, pool, cache_cls, to_tensor, on_output)
    return caches, keys, np.concatenate(outs)


@pytest.mark.parametrize("append_only", [False, True])
def test_hf_cache_host_logic_replays_reference_session(golden_dir, append_only, monkeypatch):
    """The package's HuggingFace cache logic (agentkv_b200/hf_cache.py: block
    allocation on layer 0, copy-on-write checks in the reference's order,
    slot arithmetic, truncation) replays the reference's recorded session on
    CPU — the pool's allocator answered by the oracle, the tree kernels by
    their CPU model, and the KV scatter / gather by their contract in torch
    indexing — with every K/V output, block table, sequence length and pool
    byte as recorded."""
    import torch

    from agentkv_b200.hf_cache import AgentKVCache

    import functools

    g = np.load(golden_dir / "hf_session.npz")
    spec = W.HFSpec(**json.loads(str(g["spec"])))
    from agentkv_b200 import kernels as K

    pool, kv = _hf_cpu_pool(spec, monkeypatch)
    gathers = []
    monkeypatch.setattr(K, "kv_gather", lambda *a, **k: (gathers.append(1), _kv_gather(*a, **k))[1])
    cls = functools.partial(AgentKVCache, append_only=append_only)
    caches, keys, outs = _hf_session(spec, pool, cls, torch.from_numpy)
    assert all(c.append_only == append_only for c in caches)  # forks keep the mode
    n_updates = len(keys)
    # append_only assembles from the pool once per cache and layer, the default every update
    assert len(gathers) == (len(caches) * spec.num_layers if append_only else n_updates)
    np.testing.assert_array_equal(np.asarray(keys), g["out_keys"])
    assert outs.tobytes() == g["outs"].tobytes()
    tables = np.concatenate([np.asarray(pool.get_block_ids(c.handle), np.int32) for c in caches])
    np.testing.assert_array_equal(tables, g["tables"])
    assert [c.get_seq_length() for c in caches] == g["seen"].tolist()
    assert kv.numpy().tobytes() == g["pool"].tobytes()


@pytest.mark.parametrize("spec", [
    W.HFSpec(total_blocks=512, block_size=16, num_layers=4, num_kv_heads=8, head_dim=128, prompt=200,
             commit=192, forks=3, steps=8, seed=8),
    W.HFSpec(total_blocks=256, block_size=8, num_layers=3, num_kv_heads=2, head_dim=12, prompt=37,
             commit=32, forks=3, steps=12, seed=9),
])
@pytest.mark.parametrize("append_only", [False, True])
def test_hf_cache_host_logic_equals_oracle(spec, append_only, monkeypatch):
    """Larger HF sessions (200- and 37-token prompts, commits, forks decoding
    one and three tokens per step) through the package's cache logic on CPU
    equal the oracle's cache: outputs, tables and pool bytes."""
    import torch

    from agentkv_b200.hf_cache import AgentKVCache
    from oracle import oracle as O

    import functools

    pool, kv = _hf_cpu_pool(spec, monkeypatch)
    cls = functools.partial(AgentKVCache, append_only=append_only)
    caches, keys, outs = _hf_session(spec, pool, cls, torch.from_numpy)
    opool = O.OracleKVPool(spec.total_blocks, spec.block_size, spec.num_layers, spec.num_kv_heads,
                           spec.head_dim, spec.dtype)
    ocaches, okeys, oouts = _hf_session(spec, opool, O.OracleKVCache, lambda a: a)
    assert keys == okeys
    assert outs.tobytes() == oouts.tobytes()
    for c, oc in zip(caches, ocaches):
        assert pool.get_block_ids(c.handle) == opool.get_block_ids(oc.handle)
    assert kv.numpy().tobytes() == opool.kv.tobytes()


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


def test_serving_lifecycle_on_the_oracle(golden_dir):
    """The serving-lifecycle schedule (tests/serving_pattern.py) on the
    oracle: deterministic, with page hits that return the committed blocks,
    misses, aborts, finishes and evictions; the allocated count it reads
    agrees with the oracle's own counter."""
    from serving_pattern import OracleServeAPI, serve

    a = serve(OracleServeAPI(512, 16))
    assert a == serve(OracleServeAPI(512, 16))
    # pinned: the reference pool observed exactly this (tests/golden/serving.json)
    assert json.loads(json.dumps(a)) == json.loads((golden_dir / "serving.json").read_text())["obs"]
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


def test_serving_lifecycle_host_logic_equals_oracle(golden_dir, monkeypatch):
    """The serving-lifecycle schedule through the package's pool logic on CPU
    (oracle allocator, tree kernel model) observes what the oracle's own
    tree observes: hits, block ids, finishes, aborts, counters."""
    import torch

    from serving_pattern import OracleServeAPI, PoolServeAPI, serve

    cfg = PoolConfig(total_blocks=512, block_size=16, num_layers=1, num_kv_heads=1, head_dim=8,
                     dtype="float16", device="meta")
    pool = _cpu_pool(cfg, torch.zeros((512, 1), dtype=torch.uint8), monkeypatch)
    got = serve(PoolServeAPI(pool))
    assert got == serve(OracleServeAPI(512, 16))
    assert json.loads(json.dumps(got)) == json.loads((golden_dir / "serving.json").read_text())["obs"]


def test_match_stress_tree_host_logic_replays_reference(golden_dir, monkeypatch):
    """The match stress tree (600 sequences) built through the pool calls on
    CPU (create_root's lookups, block allocation, commits), then one batched
    lookup: tree size, node-id counter, free count and every query's
    (node, length) as the reference recorded them."""
    import torch

    g = np.load(golden_dir / "match_small.npz")
    spec = W.MatchSpec(**json.loads(str(g["spec"])))
    prefixes = W.match_prefixes(spec)
    corpus = W.match_sequences(spec, prefixes)
    n = int(g["total_blocks"])
    cfg = PoolConfig(total_blocks=n, block_size=16, num_layers=1, num_kv_heads=1, head_dim=1, dtype="float16",
                     device="meta")
    pool = _cpu_pool(cfg, torch.zeros((n, 1), dtype=torch.uint8), monkeypatch)
    for seq in corpus:
        h = pool.create_root(seq)
        pool.allocate_blocks(h, -(-len(seq) // 16) - len(pool.get_block_ids(h)))
        share = (len(seq) // 16) * 16 - h.shared_match_len
        if share > 0:
            pool.commit_prefix(h, share)
    assert len(pool._tree._shared_nodes) == int(g["n_nodes"])
    assert pool._tree._next_node_id == int(g["next_node_id"])
    assert pool.free_blocks == int(g["free_blocks"])
    queries = W.match_queries(spec, corpus, prefixes, batch=0, n=len(g["node"]))
    node, mlen = pool.match_prefix_batch(queries)
    np.testing.assert_array_equal(node, g["node"])
    np.testing.assert_array_equal(mlen, g["len"])


def test_match_prefix_many_equals_one_by_one(golden_dir, monkeypatch):
    """AgentKVPool.match_prefix_many (one lookup launch for the batch) gives
    the handles — ids, shared nodes, lengths, tokens — the shared-node
    refcounts and the allocator / reclaimer state of match_prefix called on
    each query in turn, also while another reader holds a read section and
    freed blocks wait in the pending queue (CPU: oracle allocator, tree
    kernel model)."""
    import torch

    g = np.load(golden_dir / "match_small.npz")
    spec = W.MatchSpec(**json.loads(str(g["spec"])))
    prefixes = W.match_prefixes(spec)
    corpus = W.match_sequences(spec, prefixes)[:200]
    queries = W.match_queries(spec, corpus, prefixes, batch=0, n=120)
    n = int(g["total_blocks"])
    cfg = PoolConfig(total_blocks=n, block_size=16, num_layers=1, num_kv_heads=1, head_dim=1, dtype="float16",
                     device="meta")
    pools = []
    for _ in range(2):
        pool = _cpu_pool(cfg, torch.zeros((n, 1), dtype=torch.uint8), monkeypatch)
        live = []
        for seq in corpus:
            h = pool.create_root(seq)
            pool.allocate_blocks(h, -(-len(seq) // 16) - len(pool.get_block_ids(h)))
            share = (len(seq) // 16) * 16 - h.shared_match_len
            if share > 0:
                pool.commit_prefix(h, share)
            live.append(h)
        reader = pool._allocator.enter_read_section()  # another reader: freed blocks stay pending
        for h in live[::3]:
            pool.free(h)
        pools.append((pool, reader))
    (a, ra), (b, rb) = pools
    assert len(a._allocator.o.state()["pending"]) > 0
    many = a.match_prefix_many(queries)
    one = [b._tree.match_prefix(q) for q in queries]
    assert sum(1 for h, _ in many if h is not None) > 20
    for (h1, m1), (h2, m2) in zip(many, one):
        assert m1 == m2
        if h1 is None:
            assert h2 is None
            continue
        assert (h1.handle_id, h1.shared_node_id, h1.shared_match_len) == (h2.handle_id, h2.shared_node_id,
                                                                          h2.shared_match_len)
        assert list(h1.tokens) == list(h2.tokens)

    def state(pool):
        st = pool._allocator.o.state()
        refs = {nid: nd.ref_count for nid, nd in pool._tree._shared_nodes.items()}
        return (st["ref_counts"].tolist(), st["free_list"].tolist(), st["pending"].tolist(),
                st["deferred"].tolist(), refs, pool._tree._next_handle_id)

    assert state(a) == state(b)
    a._allocator.leave_read_section(ra)
    b._allocator.leave_read_section(rb)
    assert state(a) == state(b)


def test_tree_replica_flow_on_cpu(golden_dir, monkeypatch):
    """The tree-replica flow of the GPU test (owner pool built through the
    pool calls, TreeReplicaSync shares — the whole arrays after a resize,
    else the owner tree's insert commands that the replica applies itself —
    with the owner's runs into a second DeviceTree, lookups on both) run on
    CPU with the stand-ins: the replica's answers equal the reference's
    recorded ones and the owner's comparison counts, and its arrays equal
    the owner's."""
    import torch

    from agentkv_b200.device_tree import DeviceTree, match_batch
    from agentkv_b200.sharded_tree import TreeReplicaSync

    g = np.load(golden_dir / "match_small.npz")
    spec = W.MatchSpec(**json.loads(str(g["spec"])))
    prefixes = W.match_prefixes(spec)
    corpus = W.match_sequences(spec, prefixes)
    n = int(g["total_blocks"])
    cfg = PoolConfig(total_blocks=n, block_size=16, num_layers=1, num_kv_heads=1, head_dim=1, dtype="float16",
                     device="meta")
    pool = _cpu_pool(cfg, torch.zeros((n, 1), dtype=torch.uint8), monkeypatch)
    owner = pool._tree._dev_tree
    sync = TreeReplicaSync(owner)
    replica = DeviceTree(owner.device)
    replica.as_replica()
    kinds, runs_seen = [], 0
    queries = W.match_queries(spec, corpus, prefixes, batch=0, n=len(g["node"]))
    for i, seq in enumerate(corpus):
        h = pool.create_root(seq)
        pool.allocate_blocks(h, -(-len(seq) // 16) - len(pool.get_block_ids(h)))
        share = (len(seq) // 16) * 16 - h.shared_match_len
        if share > 0:
            pool.commit_prefix(h, share)
        if i % 37 == 0 or i == len(corpus) - 1:
            owner.build_runs()
            d = sync.share()
            if d is not None:
                kinds.append("commands" if "commands" in d else ("full" if d["full"] else "rows"))
                replica.apply_shared(d)
                if "run_head" in d:
                    replica.set_runs(d["run_head"], d["runs"])
                    runs_seen += 1
            if i % 111 == 0:
                n0, l0 = match_batch(owner, queries[:64], 16)
                n1, l1 = match_batch(replica, queries[:64], 16)
                np.testing.assert_array_equal(n1, n0)
                np.testing.assert_array_equal(l1, l0)
    assert "full" in kinds and kinds.count("commands") > len(kinds) // 2, kinds
    assert runs_seen > 1 and replica.d_run_head is not None
    node, mlen, cmp_ = match_batch(replica, queries, 16, with_compared=True)
    np.testing.assert_array_equal(node, g["node"])
    np.testing.assert_array_equal(mlen, g["len"])
    _, _, cmp_owner = match_batch(owner, queries, 16, with_compared=True)
    np.testing.assert_array_equal(cmp_, cmp_owner)
    m = owner.n_tokens
    assert torch.equal(replica.d_tokens[:m], owner.d_tokens[:m])
    assert torch.equal(replica.d_slots, owner.d_slots)
    assert torch.equal(replica.d_off, owner.d_off) and torch.equal(replica.d_len, owner.d_len)
    assert sync.share() is None


def test_long_unary_chain_flow_on_cpu(monkeypatch):
    """The long-chain lookup test of the GPU suite on CPU with the stand-ins:
    a 70-node unary chain with a branch at depth 100, queries cut at every
    depth, diverging every third position and running past the end — the
    oracle's (node, length, comparisons) with the runs and without."""
    import torch

    from agentkv_b200.device_tree import match_batch
    from oracle import oracle as O

    bs = 4
    cfg = PoolConfig(total_blocks=1024, block_size=bs, num_layers=1, num_kv_heads=1, head_dim=4,
                     dtype="float16", device="meta")
    pool = _cpu_pool(cfg, torch.zeros((1024, 1), dtype=torch.uint8), monkeypatch)
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
    for runs in (True, False):
        node, mlen, cmp_ = match_batch(dev_tree, queries, bs, with_compared=True, runs=runs)
        got = [(int(n) if m else -1, int(m), int(c)) for n, m, c in zip(node, mlen, cmp_)]
        assert got == [(int(n) if m else -1, int(m), int(c)) for n, m, c in want], runs
    assert int((dev_tree.d_run_head >= 0).sum()) >= 60


def test_block_table_cache_follows_changes(monkeypatch):
    """get_block_ids answers from its per-handle cache only while nothing
    changed: after allocations, copy-on-write, commits (edge splits among
    them), forks and frees it returns the freshly walked table, equal to
    the oracle's, and callers get their own list."""
    import torch

    from oracle import oracle as O

    cfg = PoolConfig(total_blocks=256, block_size=4, num_layers=1, num_kv_heads=1, head_dim=4,
                     dtype="float16", device="meta")
    pool = _cpu_pool(cfg, torch.zeros((256, 1), dtype=torch.uint8), monkeypatch)
    ot = O.OracleTree(O.OracleAllocator(256, cfg.epoch_interval), 4)
    rng = np.random.default_rng(12)
    live = []
    for step in range(300):
        op = int(rng.integers(0, 6))
        if op == 0 or len(live) < 2:
            toks = rng.integers(0, 6, size=int(rng.integers(0, 24))).tolist()
            live.append((pool.create_root(toks), ot.create_root(toks)))
        elif op == 1:
            i = int(rng.integers(0, len(live)))
            live.append((pool.fork(live[i][0]), ot.fork(live[i][1])))
        elif op == 2:
            h, o = live[int(rng.integers(0, len(live)))]
            pool.allocate_block(h)
            ot.allocate_block(o)
        elif op == 3:
            h, o = live[int(rng.integers(0, len(live)))]
            if h.residual_blocks:
                k = int(rng.integers(0, len(h.residual_blocks)))
                pool.ensure_mutable_block(h, k)
                ot.ensure_mutable_block(o, k)
        elif op == 4:
            h, o = live[int(rng.integers(0, len(live)))]
            n = min(len(h.residual_blocks), (len(h.tokens) - h.shared_match_len) // 4)
            if n > 0:
                pool.commit_prefix(h, 4 * n)
                ot.commit_prefix(o, 4 * n)
        else:
            h, o = live.pop(int(rng.integers(0, len(live))))
            pool.free(h)
            ot.free(o)
        for h, o in live:
            a = pool.get_block_ids(h)
            assert a == ot.get_block_ids(o), step
            a.append(-1)  # the caller's list is its own
            assert pool.get_block_ids(h) == ot.get_block_ids(o), step


@pytest.mark.parametrize("name", ["colliding", "long_chain"])
def test_match_scenarios_host_logic(golden_dir, name, monkeypatch):
    """The hard lookup shapes through the package's pool on CPU (tree kernels
    as their CPU model), with the unary-chain runs and with one probe per
    hop: the reference's recorded (node, length) per query."""
    import torch

    from agentkv_b200.device_tree import match_batch
    from match_scenarios import SCENARIOS, build

    want = json.loads((golden_dir / "match_scenarios.json").read_text())[name]
    sc = SCENARIOS[name]()
    cfg = PoolConfig(total_blocks=1024, block_size=sc["block_size"], num_layers=1, num_kv_heads=1, head_dim=4,
                     dtype="float16", device="meta")
    pool = _cpu_pool(cfg, torch.zeros((1024, 1), dtype=torch.uint8), monkeypatch)
    build(pool, sc, pool.allocate_block)
    for runs in (True, False):
        node, mlen = match_batch(pool._tree._dev_tree, sc["queries"], sc["block_size"], runs=runs)
        got = [[int(n) if m else -1, int(m)] for n, m in zip(node, mlen)]
        assert got == want, runs


def replay_tree_trace_with_array_checks(golden_dir, seed, dev, check_each_op=True):
    """Replay the reference's recorded tree trace `seed` through the
    package's DualRadixTree, uploading the tree after every op; returns
    (tree, number of uploads done as commands, number of ops checked).  After
    every upload the device arrays must equal the host mirror's byte for
    byte.  The allocator is the device one when `dev` is a GPU, else the
    oracle stand-in (the caller patches the tree kernels for CPU)."""
    import torch

    from agentkv_b200.radix_tree import DualRadixTree

    g = json.loads((golden_dir / f"tree_trace_{seed}.json").read_text())
    n, bs = g["n_blocks"], g["block_size"]
    if dev.type == "cuda":
        from agentkv_b200 import AgentKVPool

        pool = AgentKVPool(config=PoolConfig(total_blocks=n, block_size=bs, num_layers=1, num_kv_heads=2,
                                             head_dim=4, dtype="float16", device="cuda", epoch_interval=7))
        tree, slab = pool._tree, pool._allocator
    else:
        from oracle_slab import OracleSlab

        kv = torch.zeros((n, 1, 2, 2, bs, 4), dtype=torch.float16)
        slab = OracleSlab(kv, 7)
        tree = DualRadixTree(slab, PoolConfig(total_blocks=n, block_size=bs, num_layers=1, num_kv_heads=2,
                                              head_dim=4, dtype="float16", device="meta", epoch_interval=7))
    T_CREATE, T_FORK, T_ALLOC, T_COW, T_APPEND, T_COMMIT, T_FREE, T_MATCH, T_ADVANCE, T_ZERO = range(10)
    live = {}
    dt = tree._dev_tree
    checked = 0
    for step, rec in enumerate(g["ops"]):
        op = rec["op"]
        try:
            if op == T_CREATE:
                h = tree.create_root(rec["tokens"])
                live[h.handle_id] = h
            elif op == T_FORK:
                c = tree.fork(live[rec["h"]])
                live[c.handle_id] = c
            elif op == T_ALLOC:
                tree.allocate_block(live[rec["h"]])
            elif op == T_COW:
                tree.ensure_mutable_block(live[rec["h"]], rec["idx"])
            elif op == T_APPEND:
                tree.append_tokens(live[rec["h"]], rec["tokens"])
            elif op == T_COMMIT:
                tree.commit_prefix(live[rec["h"]], rec["length"])
            elif op == T_FREE:
                tree.free(live.pop(rec["h"]))
            elif op == T_MATCH:
                mh, _ = tree.match_prefix(rec["tokens"])
                if mh is not None:
                    live[mh.handle_id] = mh
            elif op == T_ADVANCE:
                slab.maybe_advance_epoch()
        except (ValueError, MemoryError):
            pass
        if check_each_op and op in (T_COMMIT, T_FREE, T_CREATE):
            dt.flush()
            k = dt.n_tokens
            assert np.array_equal(dt.d_tokens[:k].cpu().numpy(), dt.h_tokens[:k]), (seed, step, "tokens")
            assert np.array_equal(dt.d_off.cpu().numpy(), dt.h_off), (seed, step, "edge offsets")
            assert np.array_equal(dt.d_len.cpu().numpy(), dt.h_len), (seed, step, "edge lengths")
            assert np.array_equal(dt.d_slots.cpu().numpy(), dt.h_slots), (seed, step, "slots")
            checked += 1
    return tree, dt.command_uploads, checked


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_tree_commands_keep_the_replica_equal_to_the_host_mirror(golden_dir, seed, monkeypatch):
    """The tree changes built by the replica itself (akv_tree_commands: the
    host tree's inserts with their block-aligned split, split == 0 overwrite
    and exact re-commit, and its prunes), here by the kernel's CPU model
    (tree_kernel_model.py): over the reference's recorded tree traces, after
    every commit, free and create the replica's arrays equal the host
    mirror's byte for byte, with most uploads done as commands."""
    import torch

    from agentkv_b200 import _native as N
    from agentkv_b200 import device_tree as DT
    from tree_kernel_model import TreeKernelModel

    model = TreeKernelModel(N.lib)
    monkeypatch.setattr(N, "lib", model)
    monkeypatch.setattr(DT, "stream_handle", lambda dev: 0)
    tree, n_cmd, checked = replay_tree_trace_with_array_checks(golden_dir, seed, torch.device("cpu"))
    assert checked > 50 and n_cmd > 20, (checked, n_cmd)
    assert model.command_calls == n_cmd


def test_tree_commands_under_random_churn(monkeypatch):
    """The same check under random commits and frees that hit every insert
    branch — new leaf, descent, exact re-commit, split off and at block
    boundaries, split == 0 overwrite — and many prunes (tree_churn.py): after
    every step the replica's arrays, changed by akv_tree_commands' CPU
    model, equal the host mirror's."""
    import torch

    from agentkv_b200 import _native as N
    from agentkv_b200 import device_tree as DT
    from agentkv_b200.radix_tree import DualRadixTree
    from oracle_slab import OracleSlab
    from tree_churn import churn
    from tree_kernel_model import TreeKernelModel

    model = TreeKernelModel(N.lib)
    monkeypatch.setattr(N, "lib", model)
    monkeypatch.setattr(DT, "stream_handle", lambda dev: 0)
    kinds = {}
    orig = DT.DeviceTree.apply_commands

    def counting(self, d):
        for c in np.asarray(d["commands"]).reshape(-1, 8):
            kinds[int(c[0])] = kinds.get(int(c[0]), 0) + 1
        orig(self, d)

    monkeypatch.setattr(DT.DeviceTree, "apply_commands", counting)
    for seed in range(3):
        slab = OracleSlab(torch.zeros((400, 1, 2, 1, 4, 2), dtype=torch.float16), 7)
        tree = DualRadixTree(slab, PoolConfig(total_blocks=400, block_size=4, num_layers=1, num_kv_heads=1,
                                              head_dim=2, dtype="float16", device="meta", epoch_interval=7))
        dt = tree._dev_tree

        def check(step):
            dt.flush()
            k = dt.n_tokens
            assert np.array_equal(dt.d_tokens[:k].numpy(), dt.h_tokens[:k]), (seed, step)
            assert np.array_equal(dt.d_off.numpy(), dt.h_off), (seed, step)
            assert np.array_equal(dt.d_len.numpy(), dt.h_len), (seed, step)
            assert np.array_equal(dt.d_slots.numpy(), dt.h_slots), (seed, step)

        churn(tree, np.random.default_rng(seed), 400, check)
        assert tree._next_node_id > 60
    assert kinds.get(1, 0) > 200 and kinds.get(2, 0) > 100, kinds
