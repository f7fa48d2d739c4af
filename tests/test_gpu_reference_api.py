"""The reference's unit-test behaviours, run against agentkv_b200 on a GPU.

Each class re-checks what one of the reference's test modules pins
(tests/test_slab_allocator.py, tests/test_radix_tree.py, tests/test_api.py,
tests/test_stress.py, tests/test_vllm_integration.py:96-135) — same
operations, same expected values, same exception types and message
patterns — with the pool on CUDA (this package has no CPU pools) or on meta
for metadata-only checks.
"""

import random

import numpy as np
import pytest

from agentkv_b200 import AgentKVPool, PoolConfig
from agentkv_b200.allocator import INVALID_BLOCK, BlockHandle, SlabAllocator
from agentkv_b200.radix_tree import INVALID_NODE_ID, DualRadixTree

pytestmark = pytest.mark.gpu


def cfg(n=64, bs=4, device="cuda", **kw):
    return PoolConfig(total_blocks=n, block_size=bs, num_layers=2, num_kv_heads=2, head_dim=8,
                      dtype=kw.pop("dtype", "float16"), device=device, **kw)


@pytest.fixture
def alloc():
    return SlabAllocator(cfg())


@pytest.fixture
def tree():
    c = cfg(128)
    a = SlabAllocator(c)
    return DualRadixTree(a, c)


class TestAllocatorLifecycle:
    def test_alloc_and_refcounts(self, alloc):
        h = alloc.alloc()
        assert h.is_valid() and h.block_id >= 0
        assert alloc.ref_count(h) == 1
        alloc.inc_ref(h)
        assert alloc.ref_count(h) == 2
        assert alloc.dec_ref(h) is False
        assert alloc.dec_ref(h) is True

    def test_free_count_returns_after_epoch(self, alloc):
        hs = [alloc.alloc() for _ in range(10)]
        assert alloc.allocated_count == 10
        assert alloc.free_count == 54
        for h in hs:
            alloc.dec_ref(h)
        alloc.maybe_advance_epoch()
        assert alloc.free_count == 64

    def test_exhaustion(self):
        a = SlabAllocator(cfg())
        hs = [a.alloc() for _ in range(64)]
        assert len({h.block_id for h in hs}) == 64
        with pytest.raises(MemoryError, match="exhausted"):
            a.alloc()

    def test_invalid_handle(self, alloc):
        with pytest.raises(ValueError, match="invalid"):
            alloc.ref_count(BlockHandle(INVALID_BLOCK))
        with pytest.raises(ValueError, match="out of range"):
            alloc.ref_count(BlockHandle(64))
        with pytest.raises(TypeError):
            alloc.ref_count(3)

    def test_double_free_and_use_after_free(self, alloc):
        h = alloc.alloc()
        alloc.dec_ref(h)
        with pytest.raises(ValueError, match="double-free|already free"):
            alloc.dec_ref(h)
        with pytest.raises(ValueError, match="not allocated|double-inc|ref_count"):
            alloc.inc_ref(h)
        # the failed ops changed nothing
        assert alloc.ref_count(h) == 0

    def test_copy_and_zero_block(self, alloc):
        src, dst = alloc.alloc(), alloc.alloc()
        alloc.get_block_tensor(src).fill_(1.5)
        alloc.copy_block(src, dst)
        assert bool((alloc.get_block_tensor(dst) == 1.5).all())
        t = alloc.get_block_tensor(dst)
        t.fill_(3.0)
        alloc.zero_block(dst)
        assert bool((t == 0.0).all())

    def test_shared_dst_rejected(self, alloc):
        src, dst = alloc.alloc(), alloc.alloc()
        alloc.inc_ref(dst)
        alloc.get_block_tensor(dst).fill_(2.0)
        with pytest.raises(ValueError, match="ref_count=1"):
            alloc.copy_block(src, dst)
        with pytest.raises(ValueError, match="exclusively owned"):
            alloc.zero_block(dst)
        assert bool((alloc.get_block_tensor(dst) == 2.0).all())

    def test_stats_keys_and_leak_check(self, alloc):
        s = alloc.stats()
        assert {"total_blocks", "free_blocks", "allocated_blocks", "peak_allocated", "total_allocs",
                "total_frees", "pending_reclamation", "epoch", "pool_size_gb"} <= s.keys()
        hs = [alloc.alloc() for _ in range(20)]
        for h in hs[:5]:
            alloc.inc_ref(h)
        for h in hs + hs[:5]:
            alloc.dec_ref(h)
        alloc.maybe_advance_epoch()
        assert alloc.free_count == 64
        assert alloc.stats()["peak_allocated"] == 20

    def test_reader_section_delays_reuse(self, alloc):
        tok = alloc.enter_read_section()
        h = alloc.alloc()
        alloc.dec_ref(h)
        assert alloc._reclaimer.pending_count() == 1
        assert alloc.free_count == 63
        alloc.leave_read_section(tok)
        assert alloc._reclaimer.pending_count() == 0
        alloc.maybe_advance_epoch()
        h2 = alloc.alloc()  # the next op drains the released id to the free list
        assert h2.is_valid()
        assert alloc.free_count == 63

    def test_threads_get_unique_blocks(self):
        import threading

        a = SlabAllocator(cfg())
        got, errs = [], []
        lock = threading.Lock()

        def worker():
            local = []
            try:
                for _ in range(4):
                    local.append(a.alloc().block_id)
            except Exception as e:  # noqa: BLE001
                errs.append(e)
            with lock:
                got.extend(local)

        ts = [threading.Thread(target=worker) for _ in range(8)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        assert not errs and len(got) == 32 and len(set(got)) == 32


class TestTree:
    def test_create_root(self, tree):
        h = tree.create_root([1, 2, 3, 4])
        assert h.tokens == [1, 2, 3, 4] and not h.is_freed
        assert h.shared_node_id == INVALID_NODE_ID and h.shared_match_len == 0
        e = tree.create_root([])
        assert e.tokens == [] and e.shared_match_len == 0

    def test_fork_shares_and_counts(self, tree):
        root = tree.create_root([1, 2, 3, 4])
        bh = tree.allocate_block(root)
        a = tree.fork(root)
        assert bh in a.residual_blocks
        b = tree.fork(a)
        c = tree.fork(b)
        assert tree._alloc.ref_count(bh) == 4
        tree.free(c)
        assert tree._alloc.ref_count(bh) == 3
        child_bh = tree.allocate_block(a)
        assert child_bh not in root.residual_blocks and tree._alloc.ref_count(child_bh) == 1

    def test_fork_tokens_independent(self, tree):
        p = tree.create_root(list(range(8)))
        c = tree.fork(p)
        p.tokens.append(99)
        assert 99 not in c.tokens

    def test_freed_handles(self, tree):
        h = tree.create_root([1, 2])
        tree.free(h)
        assert h.is_freed
        with pytest.raises(ValueError, match="freed|not registered"):
            tree.fork(h)
        with pytest.raises(ValueError, match="not registered|already freed|double-free"):
            tree.free(h)

    def test_free_block(self, tree):
        h1 = tree.create_root([1, 2, 3, 4])
        h2 = tree.create_root([5, 6, 7, 8])
        bh = tree.allocate_block(h1)
        with pytest.raises(ValueError, match="residual block"):
            tree.free_block(h2, bh)
        tree.free_block(h1, bh)
        assert h1.residual_blocks == []

    def test_get_block_ids(self, tree):
        h = tree.create_root([1, 2, 3, 4])
        assert tree.get_block_ids(h) == []
        b1, b2 = tree.allocate_block(h), tree.allocate_block(h)
        assert tree.get_block_ids(h) == [b1.block_id, b2.block_id]
        other = tree.create_root([5, 6, 7, 8])
        tree.allocate_block(other)
        assert set(tree.get_block_ids(h)).isdisjoint(tree.get_block_ids(other))

    def test_commit_prefix_rules(self, tree):
        h = tree.create_root(list(range(8)))
        tree.allocate_block(h)
        tree.allocate_block(h)
        with pytest.raises(ValueError, match="multiple of block_size"):
            tree.commit_prefix(h, 3)
        with pytest.raises(ValueError, match="blocks"):
            tree.commit_prefix(h, 12)
        tree.commit_prefix(h, 4)
        assert len(h.residual_blocks) == 1 and h.shared_node_id != INVALID_NODE_ID
        h2 = tree.create_root(list(range(4)))
        assert h2.shared_match_len == 4

    def test_diverging_commit_splits_edge(self, tree):
        bs = 4
        prefix = list(range(100, 108))

        def request(tokens):
            h = tree.create_root(tokens)
            need = (len(tokens) + bs - 1) // bs
            while len(tree.get_block_ids(h)) < need:
                tree.allocate_block(h)
            share = (len(tokens) // bs) * bs - h.shared_match_len
            if share > 0:
                tree.commit_prefix(h, share)
            return h

        a = request(prefix + list(range(200, 204)))
        b = request(prefix + list(range(300, 304)))
        assert a.shared_match_len == 12 and b.shared_match_len == 12
        assert len(tree.get_block_ids(a)) == 3 and len(tree.get_block_ids(b)) == 3
        c = tree.create_root(prefix + list(range(400, 404)))
        assert c.shared_match_len == len(prefix)
        assert tree.get_block_ids(a)[:2] == tree.get_block_ids(b)[:2]

    def test_pool_exhaustion_through_tree(self):
        c = PoolConfig(total_blocks=4, block_size=4, num_layers=1, num_kv_heads=1, head_dim=4,
                       dtype="float16", device="cuda")
        t = DualRadixTree(SlabAllocator(c), c)
        h = t.create_root([])
        with pytest.raises(MemoryError):
            for _ in range(10):
                t.allocate_block(h)


class TestPoolAPI:
    @pytest.fixture
    def pool(self):
        return AgentKVPool(config=cfg(128))

    def test_quickstart_script(self, pool):
        root = pool.create_root([1, 2, 3, 4])
        a, b = pool.fork(root), pool.fork(root)
        for h in (a, b, root):
            pool.allocate_block(h)
        s = pool.stats()
        assert s["active_handles"] == 3 and s["allocated_blocks"] > 0
        for h in (a, b, root):
            pool.free(h)
        assert pool.stats()["active_handles"] == 0
        assert "AgentKVPool" in repr(pool) and "GiB" in repr(pool)

    def test_capacity_constructor(self):
        p = AgentKVPool(capacity_gb=0.001, block_size=4, num_layers=1, num_kv_heads=1, head_dim=4,
                        dtype="float16", device="cuda")
        assert p.block_size == 4 and p.config.total_blocks >= 1

    def test_fork_keeps_allocated_count(self, pool):
        root = pool.create_root([1, 2, 3, 4])
        pool.allocate_block(root)
        before = pool.allocated_blocks
        child = pool.fork(root)
        assert pool.allocated_blocks == before
        pool.allocate_block(child)
        assert len(set(pool.get_block_ids(child)) - set(pool.get_block_ids(root))) >= 1
        ids = pool.get_block_ids(child)
        assert isinstance(ids, list) and all(isinstance(x, int) for x in ids)
        init = pool.free_blocks
        h = pool.create_root([])
        pool.allocate_block(h)
        assert pool.free_blocks == init - 1

    def test_stats_keys(self, pool):
        s = pool.stats()
        for k in ("total_blocks", "free_blocks", "allocated_blocks", "active_handles", "shared_nodes",
                  "pool_size_gb"):
            assert k in s

    def test_gpu_create_fork_free(self):
        c = PoolConfig(total_blocks=256, block_size=16, num_layers=4, num_kv_heads=4, head_dim=64,
                       dtype="float16", device="cuda")
        pool = AgentKVPool(config=c)
        root = pool.create_root(list(range(16)))
        child = pool.fork(root)
        pool.allocate_block(child)
        assert pool.stats()["allocated_blocks"] == 1
        pool.free(child)
        pool.free(root)


class TestCopyOnWriteRecording:
    """A replaced copy_block on the allocator instance sees every CoW pair as
    plain ints (the vLLM adapter's recording hook)."""

    def test_cow_pairs_are_recorded(self):
        c = PoolConfig(total_blocks=256, block_size=16, num_layers=1, num_kv_heads=1, head_dim=1,
                       dtype="float16", device="meta")
        pool = AgentKVPool(config=c)
        cows = []
        pool._allocator.copy_block = lambda s, d: cows.append((s.block_id, d.block_id))
        tokens = list(range(20))
        parent = pool.create_root(tokens)
        pool.allocate_blocks(parent, 2)
        pool.commit_prefix(parent, 16)
        child = pool.fork(parent)
        shared = parent.residual_blocks[0]
        assert pool._allocator.ref_count(shared) == 2
        pool.append_tokens(parent, [9001])
        pool.ensure_mutable_block(parent, 0)
        assert cows and all(isinstance(x, int) for pair in cows for x in pair)
        assert pool._allocator.ref_count(shared) == 1
        assert parent.residual_blocks[0] != child.residual_blocks[0]
        cows.clear()
        pool.ensure_mutable_block(child, 0)
        assert cows == []


class _Shadow:
    """Ground truth of refcounts for the randomized stress run."""

    def __init__(self, n):
        self.ref = np.zeros(n, np.int64)
        self.agents = {}
        self.violations = []


@pytest.mark.parametrize("seed,n_ops", [(1, 1000), (42, 2000)])
def test_stress_shadow_model(seed, n_ops):
    c = PoolConfig(total_blocks=512, block_size=4, num_layers=2, num_kv_heads=2, head_dim=8,
                   dtype="float16", device="meta")
    a = SlabAllocator(c)
    t = DualRadixTree(a, c)
    rng = random.Random(seed)
    sh = _Shadow(512)
    live = {}
    for _ in range(n_ops):
        alive = list(live)
        if not alive:
            act = "create"
        elif len(alive) >= 32:
            act = rng.choice(["alloc_block", "free_agent"])
        else:
            act = rng.choices(["create", "fork", "alloc_block", "free_agent"], weights=[2, 3, 4, 2])[0]
        try:
            if act == "create":
                h = t.create_root([rng.randint(0, 255) for _ in range(rng.randint(1, 8))])
                live[h.handle_id] = h
                sh.agents[h.handle_id] = []
            elif act == "fork":
                p = live[rng.choice(alive)]
                ch = t.fork(p)
                live[ch.handle_id] = ch
                sh.agents[ch.handle_id] = list(sh.agents[p.handle_id])
                for b in sh.agents[p.handle_id]:
                    sh.ref[b] += 1
            elif act == "alloc_block":
                h = live[rng.choice(alive)]
                b = t.allocate_block(h).block_id
                if sh.ref[b] != 0:
                    sh.violations.append(f"DOUBLE_ALLOC {b}")
                sh.ref[b] = 1
                sh.agents[h.handle_id].append(b)
            else:
                h = live.pop(rng.choice(alive))
                t.free(h)
                for b in sh.agents.pop(h.handle_id):
                    sh.ref[b] -= 1
                for _ in range(3):
                    a.maybe_advance_epoch()
        except MemoryError:
            if live:
                h = live.pop(rng.choice(list(live)))
                t.free(h)
                for b in sh.agents.pop(h.handle_id):
                    sh.ref[b] -= 1
    for h in list(live.values()):
        t.free(h)
    for _ in range(10):
        a.maybe_advance_epoch()
    assert sh.violations == []
    np.testing.assert_array_equal(a.ref_counts()[: 512], np.zeros(512))
    assert a.free_count == 512, "leak"


def test_serving_lifecycle_equals_oracle(golden_dir):
    """The prefix-cache serving lifecycle a serving engine's radix-cache
    adapter drives (tests/serving_pattern.py: lookups adopted as handles,
    appends, page allocations, commits, finishes, aborts, epoch advances)
    observes the same hits, block ids and counters on the device pool as on
    the oracle."""
    from serving_pattern import OracleServeAPI, PoolServeAPI, serve

    pool = AgentKVPool(config=PoolConfig(total_blocks=512, block_size=16, num_layers=1, num_kv_heads=1,
                                         head_dim=8, dtype="float16", device="cuda"))
    got = serve(PoolServeAPI(pool))
    want = serve(OracleServeAPI(512, 16))
    assert got == want
    # and what the reference pool observed (tests/golden/serving.json)
    import json

    assert json.loads(json.dumps(got)) == json.loads((golden_dir / "serving.json").read_text())["obs"]
