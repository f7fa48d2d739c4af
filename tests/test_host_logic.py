"""Host-side logic that needs no GPU: config validation (same rules and
messages as the reference), the device-tree mirror's hash table and arena,
pair validation, the allocator's error mapping, the seeded workload
generators, the bench's byte counts and CPU baselines, and the package's
exported names.  The unary-chain runs and the match path's host side are
in test_host_runs.py; the replays of the reference's recorded runs in
test_host_replays.py."""

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


def test_react_cpu_baseline_plays_the_trace():
    """bench.react_cpu_baseline drives the oracle through the ReAct trace with
    the same call set the parity tests use, and reports steps/s over a
    bounded sample."""
    import bench

    spec = W.ReActSpec(steps=30)
    res = bench.react_cpu_baseline(spec, 1, 60.0)
    assert res["unit"] == "steps/s" and res["value"] > 0 and res["kind"] == "port"
    assert res["sample"].startswith("30 of 30 trace steps")


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


def test_query_packing():
    """pack_queries and QueryStage.pack lay a batch out as the lookup kernel
    reads it (tokens back to back, int64 offsets, longest-first order),
    including empty queries, an empty batch and a stage reused for batches
    larger and smaller than the last."""
    import torch

    from agentkv_b200.device_tree import QueryStage, longest_first, pack_queries

    cpu = torch.device("cpu")
    rng = np.random.default_rng(2)
    stage = QueryStage(cpu)
    for nq in (5, 300, 0, 40, 2000, 3):
        qs = [rng.integers(0, 1000, size=int(rng.integers(0, 90))).astype(np.int32) for _ in range(nq)]
        if nq > 2:
            qs[1] = []  # an empty query (a Python list)
        if nq > 10:
            # every form a caller may hold: lists, other integer dtypes, a
            # strided view, array('i'), a zero-length int32 array
            import array

            qs[3] = [int(x) for x in rng.integers(0, 1000, size=17)]
            qs[4] = rng.integers(0, 1000, size=9).astype(np.int64)
            qs[5] = rng.integers(0, 1000, size=30).astype(np.int32)[::2]
            qs[6] = array.array("i", [int(x) for x in rng.integers(0, 1000, size=11)])
            qs[7] = np.zeros(0, np.int32)
        lens = np.array([len(q) for q in qs], np.int64)
        off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
        flat = np.concatenate([np.asarray(q, np.int32) for q in qs]) if nq else np.zeros(0, np.int32)
        tok, q_off = pack_queries(qs, cpu)
        np.testing.assert_array_equal(q_off.numpy(), off)
        np.testing.assert_array_equal(tok.numpy()[: off[-1]], flat)
        t2, o2, order = stage.pack(qs)
        np.testing.assert_array_equal(o2.numpy(), off)
        np.testing.assert_array_equal(t2.numpy()[: off[-1]], flat)
        want_order = np.argsort(-lens, kind="stable")
        np.testing.assert_array_equal(order.numpy()[:nq], want_order)
        np.testing.assert_array_equal(longest_first(q_off, cpu).numpy(), want_order)


def test_host_helper_reads_token_array_addresses():
    """_akv_pyhost.token_arrays: the address and element count of every item
    that is a C-contiguous 4-byte integer buffer, from `start` on, stopping
    at (and returning the index of) the first item that is not."""
    import array

    from agentkv_b200 import _akv_pyhost as H

    a = np.arange(10, dtype=np.int32)
    b = np.frombuffer(array.array("i", [1, 2, 3]), dtype=np.int32)
    items = [a, b, [1, 2], a.astype(np.int64), a[::2], array.array("i", [5]), np.zeros(0, np.int32), b"abcd"]
    ptrs = np.zeros(len(items), np.uint64)
    lens = np.zeros(len(items), np.int64)
    assert H.token_arrays(items, 0, ptrs, lens) == 2
    assert (int(ptrs[0]), int(lens[0]), int(ptrs[1]), int(lens[1])) == (a.ctypes.data, 10, b.ctypes.data, 3)
    assert H.token_arrays(items, 3, ptrs, lens) == 3
    assert H.token_arrays(items, 4, ptrs, lens) == 4
    assert H.token_arrays(items, 5, ptrs, lens) == 7
    assert lens[5] == 1 and lens[6] == 0
    assert H.token_arrays(items, 8, ptrs, lens) == 8
    with pytest.raises(ValueError):
        H.token_arrays(items, 0, ptrs[:3], lens)
    with pytest.raises(ValueError):
        H.token_arrays(items, 9, ptrs, lens)


def test_run_many_sequencing(monkeypatch):
    """FanoutGraph.run_many's host sequencing, with the CUDA graph, events and
    device context replaced by recording stand-ins: the two instances
    alternate, an instance is read back (its event waited for) before it is
    relaunched, every run's tables come back in run order, and a wrong root
    count is refused before anything is launched."""
    import contextlib

    import torch

    from agentkv_b200 import fanout as F

    log = []

    class Event:
        def __init__(self):
            self.tag = None

        def record(self, stream):
            self.tag = log[-1]

        def synchronize(self):
            log.append(("wait", self.tag))

    monkeypatch.setattr(F.torch.cuda, "device", lambda dev: contextlib.nullcontext())
    monkeypatch.setattr(F.torch.cuda, "current_stream", lambda dev=None: None)
    monkeypatch.setattr(F.torch.cuda, "Event", Event)

    def fake(name):
        g = object.__new__(F.FanoutGraph)
        g.dev = torch.device("cpu")
        g.h_roots = torch.zeros(3, dtype=torch.int32)
        g._h_roots_np = g.h_roots.numpy()
        g.h_tables = torch.zeros(6, dtype=torch.int32)
        g._h_status_np = np.zeros(8, np.int32)
        g.alloc = None

        class Graph:
            def replay(self_inner):
                # the "run": child tables computed from the roots written in
                g.h_tables.numpy()[:] = np.tile(g._h_roots_np, 2) * 10
                log.append(("replay", name, int(g._h_roots_np[0])))

        g.graph = Graph()
        return g

    a, b = fake("a"), fake("b")
    a._twin = b
    roots = [np.array([i, i + 1, i + 2], np.int32) for i in range(5)]
    outs = a.run_many(roots)
    assert [int(o[0]) for o in outs] == [0, 10, 20, 30, 40]
    assert all(np.array_equal(o, np.tile(r, 2) * 10) for o, r in zip(outs, roots))
    replays = [e for e in log if e[0] == "replay"]
    assert [e[1] for e in replays] == ["a", "b", "a", "b", "a"]
    # instance a is waited for (run 0 read back) before its relaunch with run 2
    i_wait = log.index(("wait", ("replay", "a", 0)))
    i_relaunch = log.index(("replay", "a", 2))
    assert i_wait < i_relaunch
    log.clear()
    with pytest.raises(ValueError, match="root ids"):
        a.run_many([np.zeros(2, np.int32)])
    assert not log
    assert a.run_many([]) == []
    # per_replay=2: two instances of 2 fan-outs each alternate over the first
    # 4 runs, the fifth goes through the one-fan-out pair
    def fake2(name):
        g = fake(name)
        g.per_replay = 2
        g.h_roots = torch.zeros(6, dtype=torch.int32)
        g._h_roots_np = g.h_roots.numpy()
        g.h_tables = torch.zeros(12, dtype=torch.int32)

        class Graph:
            def replay(self_inner):
                r = g._h_roots_np.reshape(2, 3)
                g.h_tables.numpy()[:] = np.concatenate([np.tile(x, 2) * 10 for x in r])
                log.append(("replay", name, int(r[0, 0]), int(r[1, 0])))

        g.graph = Graph()
        return g

    a._grouped = {}
    made = []

    def instance(k):
        made.append(k)
        return fake2(f"g{len(made)}")

    a._instance = instance
    log.clear()
    outs = a.run_many(roots, per_replay=2)
    assert made == [2, 2]
    assert all(np.array_equal(o, np.tile(r, 2) * 10) for o, r in zip(outs, roots)) and len(outs) == 5
    replays = [e for e in log if e[0] == "replay"]
    assert replays == [("replay", "g1", 0, 1), ("replay", "g2", 2, 3), ("replay", "a", 4)]
    a.run_many(roots[:4], per_replay=2)  # the grouped instances are kept
    assert made == [2, 2]
    with pytest.raises(ValueError, match="per_replay"):
        a.run_many(roots, per_replay=0)


def _claimed_schedule(n_items: int, grid: int, claim_max: int, rng) -> list:
    """A CPU model of k_copy_bulk's claimed item hand-out (CLAIM > 0): the
    claim size, each CTA's dealt first range, the counter's ranges after
    them (each CTA asks for its next range when it starts the current one)
    and the stop rule, with the CTAs' steps interleaved at random.  Returns
    every item each CTA processes."""
    claim = max(1, min(claim_max, n_items // (4 * grid)))
    dealt = grid * claim
    counter = 0
    done = []
    state = []
    for b in range(grid):
        t = b * claim
        nxt = dealt + counter
        counter += claim
        state.append([t, t + claim, nxt])
    live = [b for b in range(grid) if state[b][0] < n_items]
    while live:
        b = live[rng.integers(len(live))]
        t, end, nxt = state[b]
        done.append(t)
        t += 1
        if t == end and t < n_items:
            t, end = nxt, nxt + claim
            if t < n_items:
                nxt = dealt + counter
                counter += claim
        state[b] = [t, end, nxt]
        if t >= n_items:
            live.remove(b)
    return done


def test_claimed_copy_hands_out_every_item_once():
    """The claimed copy's index arithmetic (k_copy_bulk with CLAIM > 0), on
    the CPU: for batch sizes from one chunk to many claims per CTA, grids
    smaller and larger than the batch (a counted launch may find fewer pairs
    than its grid was sized for) and random interleavings of the CTAs, every
    item is copied exactly once and no CTA runs past the batch."""
    rng = np.random.default_rng(5)
    for n_items in (1, 3, 64, 148, 149, 592, 593, 4096, 9344):
        for grid in (1, 7, 148):
            for claim_max in (1, 4, 8):
                got = _claimed_schedule(n_items, grid, claim_max, rng)
                assert sorted(got) == list(range(n_items)), (n_items, grid, claim_max)
