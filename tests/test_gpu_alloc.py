"""Device free list and refcounts against the reference and the oracle.

* The reference's own recorded op traces (alloc / inc_ref / dec_ref / read
  sections / epoch advances, with errors) replayed through the device
  allocator's single-op API: every result, refcount, free-list entry,
  reclaimer queue and counter must match after every op.
* Random batches through the batched API against the oracle's all-or-nothing
  batches, with repeated ids, retirements, errors and open read sections.
* The fused copy-on-write batch against the oracle, with data.
"""

import numpy as np
import pytest
import torch

from agentkv_b200 import _native as N
from agentkv_b200.allocator import BlockHandle, SlabAllocator
from agentkv_b200.config import PoolConfig
from oracle import oracle as O

pytestmark = pytest.mark.gpu

A_ALLOC, A_INC, A_DEC, A_ENTER, A_LEAVE, A_ADVANCE = range(6)


def make_alloc(n, interval=64, device="meta", bpb_shape=(1, 1, 4, 1)):
    L, H, bs, D = bpb_shape
    cfg = PoolConfig(total_blocks=n, block_size=bs, num_layers=L, num_kv_heads=H, head_dim=D,
                     dtype="float16", device=device, epoch_interval=interval)
    return SlabAllocator(cfg)


def device_state(a: SlabAllocator) -> dict:
    c = a.ctl()
    deferred, pending, pend_eps = a.limbo()
    return {
        "ref": a.ref_counts(),
        "free": a.free_list(),
        "deferred": deferred,
        "pending": pending,
        "pending_epochs": pend_eps,
        "ctl": [int(c[N.CTL_OPS]), int(c[N.CTL_EPOCH]), int(c[N.CTL_ALLOCS]), int(c[N.CTL_FREES]),
                int(c[N.CTL_PEAK]), int(c[N.CTL_ADVANCES]), int(c[N.CTL_RELEASED]),
                int(c[N.CTL_FREE_SIZE]), a.allocated_count],
    }


def assert_same_as_oracle(a: SlabAllocator, o: O.OracleAllocator, where=""):
    d, s = device_state(a), o.state()
    np.testing.assert_array_equal(d["ref"], s["ref_counts"], err_msg=f"ref {where}")
    np.testing.assert_array_equal(d["free"], s["free_list"], err_msg=f"free {where}")
    np.testing.assert_array_equal(d["deferred"], s["deferred"], err_msg=f"deferred {where}")
    np.testing.assert_array_equal(d["pending"], s["pending"], err_msg=f"pending {where}")
    np.testing.assert_array_equal(d["pending_epochs"], s["pending_epochs"], err_msg=f"tags {where}")
    assert d["ctl"] == [s["op_count"], s["epoch"], s["total_allocs"], s["total_frees"], s["peak_allocated"],
                        s["epoch_advances"], s["blocks_freed"], len(s["free_list"]),
                        s["allocated_blocks"]], where


def ragged(d, key, i):
    off = d[key + "_off"]
    return d[key][off[i] : off[i + 1]]


@pytest.mark.parametrize("seed", [1, 2, 3, 4])
def test_reference_trace_single_ops(golden_dir, seed):
    d = np.load(golden_dir / f"alloc_trace_{seed}.npz")
    a = make_alloc(int(d["n_blocks"]), int(d["interval"]))
    for i, (op, arg, want) in enumerate(zip(d["ops"], d["args"], d["results"])):
        arg = int(arg)
        if op == A_ALLOC:
            try:
                got = a.alloc().block_id
            except MemoryError as e:
                assert "exhausted" in str(e)
                got = -3
        elif op == A_INC:
            try:
                a.inc_ref(BlockHandle(arg))
                got = 0
            except ValueError as e:
                assert "not allocated" in str(e) and "ref_count=" in str(e)
                got = -5
        elif op == A_DEC:
            try:
                got = int(a.dec_ref(BlockHandle(arg)))
            except ValueError as e:
                assert "double-free" in str(e)
                got = -4
        elif op == A_ENTER:
            got = a.enter_read_section()
        elif op == A_LEAVE:
            a.leave_read_section(arg)
            got = 0
        else:
            a.maybe_advance_epoch()
            got = 0
        assert got == int(want), f"op {i} ({op}, {arg})"
        ds = device_state(a)
        np.testing.assert_array_equal(ds["ref"], d["ref"][i], err_msg=f"ref after op {i}")
        np.testing.assert_array_equal(ds["free"], ragged(d, "free", i), err_msg=f"free after op {i}")
        np.testing.assert_array_equal(ds["pending"], ragged(d, "pend_ids", i), err_msg=f"pending {i}")
        np.testing.assert_array_equal(ds["pending_epochs"], ragged(d, "pend_eps", i))
        np.testing.assert_array_equal(ds["deferred"], ragged(d, "deferred", i), err_msg=f"deferred {i}")
        assert ds["ctl"] == [int(x) for x in d["ctl"][i]], f"counters after op {i}"


def _random_batch_session(seed, n_blocks, interval, steps, readers):
    rng = np.random.default_rng(seed)
    a = make_alloc(n_blocks, interval)
    o = O.OracleAllocator(n_blocks, interval)
    tokens = []
    for step in range(steps):
        r = rng.random()
        live = np.flatnonzero(o.state()["ref_counts"] > 0).astype(np.int32)
        err_dev = err_orc = None
        if r < 0.3:
            n = int(rng.integers(1, max(2, n_blocks // 3)))
            try:
                want = o.alloc_batch(n)
            except O.OracleError as e:
                err_orc = e.code
            got = a.alloc_batch(n)
            try:
                a.check()
            except MemoryError:
                err_dev = N.AKV_ERR_EXHAUSTED
            if err_orc is None and err_dev is None:
                np.testing.assert_array_equal(got.cpu().numpy(), want)
        elif r < 0.5 and len(live):
            ids = rng.choice(live, size=int(rng.integers(1, 3 * len(live) + 1)))
            if rng.random() < 0.1:
                ids[rng.integers(0, len(ids))] = rng.integers(0, n_blocks)
            try:
                o.inc_ref_batch(ids)
            except O.OracleError as e:
                err_orc = e.code
            a.inc_ref_batch(ids)
            try:
                a.check()
            except ValueError:
                err_dev = N.AKV_ERR_NOT_ALLOCATED
        elif r < 0.8 and len(live):
            refs = o.state()["ref_counts"]
            # mostly exact counts (retire) + some partial, occasionally one too many
            pool = []
            for b in rng.choice(live, size=min(len(live), int(rng.integers(1, len(live) + 1))), replace=False):
                k = int(refs[b]) if rng.random() < 0.6 else int(rng.integers(1, refs[b] + 1))
                pool += [int(b)] * k
            if rng.random() < 0.08:
                pool.append(int(rng.choice(live)))
                pool += [int(rng.choice(live))] * 3
            ids = np.asarray(pool, np.int32)
            rng.shuffle(ids)
            try:
                want_ret = o.dec_ref_batch(ids)
            except O.OracleError as e:
                err_orc = e.code
            out = torch.full((len(ids),), -7, dtype=torch.int32, device=a.device)
            a.dec_ref_batch(ids, retired_out=out)
            try:
                a.check()
            except ValueError:
                err_dev = N.AKV_ERR_DOUBLE_FREE
            if err_orc is None and err_dev is None:
                n_ret = int(a.ctl()[N.CTL_LAST_RETIRED])
                np.testing.assert_array_equal(out[:n_ret].cpu().numpy(), want_ret)
        elif readers and r < 0.87:
            t1 = a.enter_read_section()
            t2 = o.enter_read_section()
            assert t1 == t2
            tokens.append(t1)
        elif readers and r < 0.94 and tokens:
            t = tokens.pop(int(rng.integers(0, len(tokens))))
            a.leave_read_section(t)
            o.leave_read_section(t)
        else:
            a.maybe_advance_epoch()
            o.maybe_advance_epoch()
        assert (err_dev is None) == (err_orc is None), f"step {step}: {err_dev} vs {err_orc}"
        assert_same_as_oracle(a, o, f"step {step}")


@pytest.mark.parametrize("seed", range(6))
def test_random_batches_match_oracle(seed):
    _random_batch_session(seed, n_blocks=[40, 200, 1000, 17, 333, 64][seed],
                          interval=[5, 64, 3, 1, 7, 2][seed], steps=120, readers=False)


@pytest.mark.parametrize("seed", range(4))
def test_random_batches_with_readers_match_oracle(seed):
    _random_batch_session(100 + seed, n_blocks=[40, 120, 64, 9][seed], interval=[4, 9, 2, 3][seed],
                          steps=150, readers=True)


def test_large_decref_batch_ordering():
    """A 150k-id dec_ref batch (many CTAs) retires in sequential order."""
    n = 30_000
    rng = np.random.default_rng(9)
    a = make_alloc(n)
    o = O.OracleAllocator(n)
    got = a.alloc_batch(n)
    want = o.alloc_batch(n)
    np.testing.assert_array_equal(got.cpu().numpy(), want)
    extra = rng.integers(0, 5, size=n)
    incs = np.repeat(np.arange(n, dtype=np.int32), extra)
    rng.shuffle(incs)
    a.inc_ref_batch(incs)
    o.inc_ref_batch(incs)
    decs = np.repeat(np.arange(n, dtype=np.int32), extra + 1)
    rng.shuffle(decs)
    out = torch.empty(len(decs), dtype=torch.int32, device=a.device)
    a.dec_ref_batch(decs, retired_out=out)
    want_ret = o.dec_ref_batch(decs)
    a.check()
    np.testing.assert_array_equal(out[:n].cpu().numpy(), want_ret)
    assert_same_as_oracle(a, o, "after large batch")


@pytest.mark.parametrize("readers", [False, True])
def test_single_cta_and_grid_batches_agree(readers):
    """inc_ref / dec_ref batches of up to 2,048 ids run as one single-CTA
    launch, longer ones over the grid: batches on both sides of that size
    (with repeated ids, a deferred drain, an open read section, and a
    double free on each side) leave the state the oracle's batches leave."""
    n = 6000
    rng = np.random.default_rng(21 + readers)
    a = make_alloc(n, interval=5)
    o = O.OracleAllocator(n, 5)
    np.testing.assert_array_equal(a.alloc_batch(n).cpu().numpy(), o.alloc_batch(n))
    if readers:
        assert a.enter_read_section() == o.enter_read_section()
    for size in (1, 2047, 2048, 2049, 5000):
        live = np.flatnonzero(o.state()["ref_counts"] > 0)
        ids = rng.choice(live, size=size).astype(np.int32)
        a.inc_ref_batch(ids)
        o.inc_ref_batch(ids)
        a.check()
        assert_same_as_oracle(a, o, f"inc {size}")
        refs = o.state()["ref_counts"]
        decs = np.repeat(np.unique(ids), refs[np.unique(ids)]).astype(np.int32)
        rng.shuffle(decs)
        decs = decs[:size]  # `size` ids: blocks listed ref_count times retire, the rest drop a count
        out = torch.full((len(decs),), -7, dtype=torch.int32, device=a.device)
        a.dec_ref_batch(decs, retired_out=out)
        want = o.dec_ref_batch(decs)
        a.check()
        np.testing.assert_array_equal(out[: len(want)].cpu().numpy(), want)
        assert_same_as_oracle(a, o, f"dec {size}")
        a.maybe_advance_epoch()
        o.maybe_advance_epoch()
        # top the pool up again so the next size has live blocks to reference
        free = len(o.state()["free_list"])
        np.testing.assert_array_equal(a.alloc_batch(free).cpu().numpy(), o.alloc_batch(free))
    for size in (100, 3000):  # one id too many: the whole batch is refused
        live = np.flatnonzero(o.state()["ref_counts"] > 0)[:size]
        decs = np.repeat(live, o.state()["ref_counts"][live]).astype(np.int32)
        decs = np.append(decs, live[0])
        with pytest.raises(O.OracleError):
            o.dec_ref_batch(decs)
        a.dec_ref_batch(decs)
        with pytest.raises(ValueError, match="double-free"):
            a.check()
        assert_same_as_oracle(a, o, f"refused dec {size}")


@pytest.mark.parametrize("seed", range(5))
def test_cow_batch_matches_oracle(seed):
    rng = np.random.default_rng(seed)
    n_blocks, shape = 300, (1, 2, 4, 16)
    L, H, bs, D = shape
    a = make_alloc(n_blocks, interval=[3, 64, 5, 2, 11][seed], device="cuda", bpb_shape=shape)
    o = O.OracleAllocator(n_blocks, [3, 64, 5, 2, 11][seed])
    bpb = a.config.bytes_per_block
    g = torch.Generator(device="cpu").manual_seed(seed)
    host = torch.randint(-30000, 30000, (n_blocks, bpb // 2), dtype=torch.int16, generator=g)
    a._kv_data.view(torch.int16).view(n_blocks, -1).copy_(host)
    host = host.numpy().view(np.uint8).reshape(n_blocks, -1).copy()
    ids = a.alloc_batch(120).cpu().numpy()
    o.alloc_batch(120)
    incs = np.repeat(ids, rng.integers(0, 4, size=len(ids)))
    a.inc_ref_batch(incs)
    o.inc_ref_batch(incs)
    for rnd in range(4):
        # distinct slots may hold the same block (forked handles); include
        # contested blocks whose requests outnumber their other holders
        blocks = rng.choice(ids, size=int(rng.integers(1, 80)))
        ob, oc = a.cow_batch(blocks)
        want_b, want_c = o.cow_batch(blocks, host, bpb)
        a.check()
        np.testing.assert_array_equal(ob.cpu().numpy(), want_b, err_msg=f"round {rnd}")
        np.testing.assert_array_equal(oc.cpu().numpy(), want_c)
        assert_same_as_oracle(a, o, f"cow round {rnd}")
        dev_bytes = a._kv_data.view(n_blocks, -1).view(torch.uint8).cpu().numpy()
        np.testing.assert_array_equal(dev_bytes, host)
        ids = np.unique(np.concatenate([ids, want_b]))


def test_cow_batch_exhaustion_is_all_or_nothing():
    a = make_alloc(8)
    ids = a.alloc_batch(6).cpu().numpy()
    a.inc_ref_batch(ids)
    before = device_state(a)
    a.cow_batch(ids)  # needs 6 fresh blocks, only 2 free
    with pytest.raises(MemoryError):
        a.check()
    after = device_state(a)
    for k in ("ref", "free"):
        np.testing.assert_array_equal(before[k], after[k])


@pytest.mark.parametrize("seed", range(3))
def test_cow_many_matches_oracle(seed):
    """ensure_mutable over a batch answered on the host mirror (cow_many),
    the copies enqueued in one launch: the same blocks, copies, allocator
    state and pool bytes as the oracle's batch, with contested blocks."""
    rng = np.random.default_rng(40 + seed)
    n_blocks, shape = 300, (1, 2, 4, 16)
    a = make_alloc(n_blocks, interval=[3, 7, 64][seed], device="cuda", bpb_shape=shape)
    o = O.OracleAllocator(n_blocks, [3, 7, 64][seed])
    bpb = a.config.bytes_per_block
    g = torch.Generator(device="cpu").manual_seed(seed)
    host = torch.randint(-30000, 30000, (n_blocks, bpb // 2), dtype=torch.int16, generator=g)
    a._kv_data.view(torch.int16).view(n_blocks, -1).copy_(host)
    host = host.numpy().view(np.uint8).reshape(n_blocks, -1).copy()
    ids = np.asarray([a.alloc().block_id for _ in range(100)], np.int32)
    o.alloc_batch(100)
    incs = np.repeat(ids, rng.integers(0, 4, size=len(ids)))
    a.inc_ref_batch(incs)
    o.inc_ref_batch(incs)
    for rnd in range(4):
        blocks = rng.choice(ids, size=int(rng.integers(1, 60)))
        ob, oc = a.cow_many(blocks)
        want_b, want_c = o.cow_batch(blocks, host, bpb)
        np.testing.assert_array_equal(ob, want_b, err_msg=f"round {rnd}")
        np.testing.assert_array_equal(oc, want_c)
        a.check()
        assert_same_as_oracle(a, o, f"cow_many round {rnd}")
        dev_bytes = a._kv_data.view(n_blocks, -1).view(torch.uint8).cpu().numpy()
        np.testing.assert_array_equal(dev_bytes, host)
        ids = np.unique(np.concatenate([ids, want_b]))
    # exhaustion: refused at the call, nothing changed
    free = len(o.state()["free_list"])
    shared = np.flatnonzero(o.state()["ref_counts"] > 1)[: free + 1]
    if len(shared) > free:
        before = device_state(a)
        with pytest.raises(MemoryError):
            a.cow_many(shared)
        after = device_state(a)
        for k in ("ref", "free"):
            np.testing.assert_array_equal(before[k], after[k])


def test_cpu_pool_is_rejected():
    with pytest.raises(ValueError, match="CUDA"):
        make_alloc(8, device="cpu")


def test_host_mirror_follows_the_device():
    """The per-call methods are answered by the allocator's host mirror and
    replayed on the device from its op log (akv_alloc_replay); device-side
    batches make the mirror reload from the device.  Over random single
    calls, host-id batches, device-id batches, copy-on-writes, epoch
    advances and read sections, after every step the device arrays (after
    the replay) equal the mirror's and the oracle's, every reader's token is
    the device's epoch at entry, and the replay reports no difference."""
    from agentkv_b200.allocator import BlockHandle

    cfg = PoolConfig(total_blocks=512, block_size=16, num_layers=1, num_kv_heads=1, head_dim=1,
                     dtype="float16", device="meta", epoch_interval=5)
    a = SlabAllocator(cfg)
    o = O.OracleAllocator(512, 5)
    rng = np.random.default_rng(3)
    refs = []  # one entry per reference held
    readers = []
    reloads = 0
    for step in range(400):
        op = int(rng.integers(0, 10))
        if op == 0 or len(refs) < 4:
            b = a.alloc()
            assert b.block_id == int(o.alloc_batch(1)[0]), step
            refs.append(b)
        elif op == 1:
            b = refs[int(rng.integers(len(refs)))]
            a.inc_ref(b)
            o.inc_ref_batch([b.block_id])
            refs.append(b)
        elif op == 2:
            b = refs.pop(int(rng.integers(len(refs))))
            assert a.dec_ref(b) == (len(o.dec_ref_batch([b.block_id])) > 0), step
        elif op == 3:
            got = a.alloc_batch(3).cpu().tolist()
            assert got == o.alloc_batch(3).tolist(), step
            refs += [BlockHandle(int(x)) for x in got]
        elif op == 4:
            drop = [refs.pop(int(rng.integers(len(refs)))) for _ in range(2)]
            a.dec_ref_batch([b.block_id for b in drop])
            o.dec_ref_batch([b.block_id for b in drop])
        elif op == 5:
            a.maybe_advance_epoch()
            o.maybe_advance_epoch()
        elif op == 6 and len(readers) < 3:
            device_epoch = int(a.ctl()[N.CTL_EPOCH])
            readers.append(a.enter_read_section())
            assert readers[-1] == device_epoch == o.enter_read_section(), step
        elif op == 7:
            # a batch of DEVICE ids: runs on the device, the mirror reloads later
            b = refs[int(rng.integers(len(refs)))]
            a.inc_ref_batch(torch.tensor([b.block_id], dtype=torch.int32, device=a.device))
            o.inc_ref_batch([b.block_id])
            refs.append(b)
            reloads += not a._live
        elif op == 8:
            b = refs[int(rng.integers(len(refs)))]
            nb = a.cow_one(b.block_id)
            out, _ = o.cow_batch([b.block_id])
            assert nb == int(out[0]), step
            if nb != b.block_id:
                refs.remove(b)
                refs.append(BlockHandle(nb))
        elif readers:
            t = readers.pop(0)
            a.leave_read_section(t)
            o.leave_read_section(t)
        a.check()
        assert_same_as_oracle(a, o, f"step {step}")
        if a._live:
            ctl, ref, ring, lid, lep = a._mirror.arrays()
            np.testing.assert_array_equal(ref, a.ref_counts(), err_msg=f"mirror refs {step}")
            dev_ctl = a.ctl()
            keep = [i for i in range(N.CTL_WORDS) if i != N.CTL_DONE]
            np.testing.assert_array_equal(ctl[keep], dev_ctl[keep], err_msg=f"mirror ctl {step}")
    assert reloads > 10 and int(a.ctl()[N.CTL_ADVANCES]) > 10
