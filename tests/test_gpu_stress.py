"""The reference's own stress runner on the device path.

The fixtures hold every call the reference's tests/test_stress.py
StressRunner made (create_root / fork / allocate_block / free /
maybe_advance_epoch over a 512-block pool, with its seeds 1, 2, 7, 13, 17,
42, 137, 999 and op counts) and what each returned.  Replayed through the
device allocator and tree, every handle id, block id and pool-exhausted error
must be the reference's, and the run must end with the reference's
refcounts, free-list order and counters (all blocks free again).
"""

import json

import numpy as np
import pytest

from agentkv_b200.allocator import SlabAllocator
from agentkv_b200.config import PoolConfig
from agentkv_b200.radix_tree import DualRadixTree

from stress_replay import replay, seeds

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("seed", seeds())
def test_reference_stress_runner_replay(golden_dir, seed):
    g = np.load(golden_dir / f"stress_{seed}.npz")
    cfg = PoolConfig(total_blocks=512, block_size=4, num_layers=2, num_kv_heads=2, head_dim=8, dtype="float16",
                     device="cuda")
    alloc = SlabAllocator(cfg)
    tree = DualRadixTree(alloc, cfg)
    replay(g, tree, alloc.maybe_advance_epoch, lambda e: isinstance(e, MemoryError) and "exhausted" in str(e))
    alloc.check()
    np.testing.assert_array_equal(alloc.ref_counts(), g["ref"])
    np.testing.assert_array_equal(alloc.free_list(), g["free"])
    assert alloc.free_count == 512
    st, want = alloc.stats(), json.loads(str(g["stats"]))
    for k in ("free_blocks", "allocated_blocks", "peak_allocated", "total_allocs", "total_frees", "epoch",
              "pending_reclamation"):
        assert st[k] == want[k], k


def test_concurrent_replays_in_threads(golden_dir):
    """Four threads, each replaying another seed on its own allocator and
    tree at the same time (the reference's concurrent stress-runner test):
    every thread still gets exactly the reference's ids and end state."""
    import threading

    errors = []

    def worker(seed):
        try:
            g = np.load(golden_dir / f"stress_{seed}.npz")
            cfg = PoolConfig(total_blocks=512, block_size=4, num_layers=2, num_kv_heads=2, head_dim=8,
                             dtype="float16", device="cuda")
            alloc = SlabAllocator(cfg)
            tree = DualRadixTree(alloc, cfg)
            replay(g, tree, alloc.maybe_advance_epoch,
                   lambda e: isinstance(e, MemoryError) and "exhausted" in str(e))
            alloc.check()
            np.testing.assert_array_equal(alloc.ref_counts(), g["ref"])
            np.testing.assert_array_equal(alloc.free_list(), g["free"])
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append((seed, repr(e)))

    ts = [threading.Thread(target=worker, args=(s,)) for s in (1, 42, 137, 999)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=300)
    assert not any(t.is_alive() for t in ts)
    assert not errors, errors
