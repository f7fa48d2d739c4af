"""akv_decref_batch_noalloc — the dec_ref batch for callers that cannot
allocate device memory where they free blocks (for example a block manager
called from a serving engine's memory-pool hook, or one running after the
engine reserved all free GPU memory up front).  It keeps its work space in a
static device array inside the library instead of caller-provided scratch.

Checked through the C ABI against akv_decref_batch on identical allocator
states, for two calls in a row, with no reader open and with readers open
(the retired ids then wait in the reclaimer's pending queue until the
readers leave): refcounts, free-list order, reclaimer queues, counters and
the retired ids must be identical (integer work: bit-exact).  This file is
collected last so that a failure here leaves every other test already run.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from agentkv_b200 import _native as N
from agentkv_b200.allocator import SlabAllocator
from agentkv_b200.config import PoolConfig

pytestmark = pytest.mark.gpu


def _alloc(n):
    cfg = PoolConfig(total_blocks=n, block_size=16, num_layers=1, num_kv_heads=1, head_dim=1,
                     dtype="float16", device="meta", epoch_interval=7)
    return SlabAllocator(cfg)


def _state(a: SlabAllocator):
    """The allocator's logical state.  The limbo cursors' raw values are left
    out: a per-call dec_ref passes each retirement through the limbo queue
    (the reference's order of steps), a dec_ref batch without readers puts
    it straight on the free list, and both leave the same lists."""
    c = a.ctl()
    deferred, pending, eps = a.limbo()
    return {"ref": a.ref_counts(), "free": a.free_list(), "deferred": deferred,
            "pending": pending, "eps": eps,
            "ctl": np.delete(c, [N.CTL_DONE, N.CTL_LIMBO_HEAD, N.CTL_LIMBO_REL, N.CTL_LIMBO_TAIL])}


def _same(a, b):
    sa, sb = _state(a), _state(b)
    for k in sa:
        np.testing.assert_array_equal(sa[k], sb[k], err_msg=k)


def _compare_two_calls(readers: bool):
    n_blocks = 5000
    rng = np.random.default_rng(2024 + readers)
    a, b = _alloc(n_blocks), _alloc(n_blocks)
    for x in (a, b):
        x.alloc_batch(3000)
    ids = np.arange(n_blocks - 3000, n_blocks, dtype=np.int32)[::-1].copy()
    extra = np.repeat(ids, rng.integers(0, 3, size=len(ids)))
    for x in (a, b):
        x.inc_ref_batch(extra)
    tokens = []
    if readers:
        # Move the epoch on, then open two readers (the epoch stays put while
        # a reader holds it): ids retired now must wait in the pending queue,
        # tagged with their op's epoch, instead of returning to the free list.
        for x in (a, b):
            for _ in range(3):
                x.maybe_advance_epoch()
            tokens.append((x, x.enter_read_section(), x.enter_read_section()))
    a.check()
    b.check()
    _same(a, b)
    refs = a.ref_counts()
    # b's state with its scratch pointers removed: the entry point must not need them.
    # The direct calls change b's device state behind its host mirror.
    with b._lock:
        b._device_op()
    st = N.AkvAllocState.from_buffer_copy(b._state)
    st.scratch_count = None
    st.scratch_last = None
    st.scratch_aux = None
    stream = torch.cuda.current_stream(b.device).cuda_stream
    for call in range(2):
        alive = ids[refs[ids] > 0]
        pick = rng.choice(alive, size=1200, replace=False)
        decs = np.concatenate([np.repeat(pick[:700], refs[pick[:700]]), pick[700:]]).astype(np.int32)
        rng.shuffle(decs)
        out_a = torch.full((len(decs),), -1, dtype=torch.int32, device=a.device)
        out_b = torch.full((len(decs),), -1, dtype=torch.int32, device=b.device)
        a.dec_ref_batch(decs, retired_out=out_a)
        d = torch.from_numpy(decs).to(b.device)
        rc = N.lib.akv_decref_batch_noalloc(C.byref(st), d.data_ptr(), len(decs), b._tick(), out_b.data_ptr(),
                                            b._status.data_ptr(), stream)
        assert rc == N.AKV_OK, N.last_error()
        a.check()
        b.check()
        _same(a, b)
        n_ret = int(a.ctl()[N.CTL_LAST_RETIRED])
        assert n_ret > 0
        np.testing.assert_array_equal(out_a.cpu().numpy(), out_b.cpu().numpy())
        refs = a.ref_counts()
    if readers:
        assert a._reclaimer.pending_count() > 0
        for x, t0, t1 in tokens:
            x.leave_read_section(t0)
            x.leave_read_section(t1)
        a.check()
        b.check()
        _same(a, b)
        assert a._reclaimer.pending_count() == 0


def test_noalloc_decref_matches_decref_batch():
    _compare_two_calls(readers=False)


def test_noalloc_decref_with_open_readers_matches_decref_batch():
    _compare_two_calls(readers=True)
