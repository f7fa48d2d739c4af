"""The allocator's host mirror (akv_mirror_*) against the reference.

* The reference's own recorded op traces (alloc / inc_ref / dec_ref / read
  sections / epoch advances, with errors), replayed through the mirror one
  call at a time: every result, refcount, free-list entry, reclaimer queue
  and counter equals the recording after every op.
* Random batches against the oracle's all-or-nothing batches, with repeated
  ids, retirements, errors and open read sections.
* The op log's records.
Host code only: runs without a GPU."""

import numpy as np
import pytest

from agentkv_b200 import _native as N
from agentkv_b200.mirror import HostMirror, MirrorRefused
from oracle import oracle as O

A_ALLOC, A_INC, A_DEC, A_ENTER, A_LEAVE, A_ADVANCE = range(6)
INT64_MAX = (1 << 63) - 1


class Readers:
    """The reclaimer's reader set, as EpochReclaimer keeps it."""

    def __init__(self, interval):
        self.set = set()
        self.interval = interval

    def tick(self):
        if self.set:
            return N.AkvTick(min(self.set), max(self.set), self.interval, 1)
        return N.AkvTick(0, 0, self.interval, 0)

    def safe(self):
        return min(self.set) if self.set else INT64_MAX


def mirror_state(m: HostMirror) -> dict:
    c = m.ctl()
    deferred, pending, eps = m.limbo()
    allocated = int(c[N.CTL_ALLOCS] - c[N.CTL_FREES])
    return {"ref": m.refs(), "free": m.free_list(), "deferred": deferred, "pending": pending,
            "pending_epochs": eps,
            "ctl": [int(c[N.CTL_OPS]), int(c[N.CTL_EPOCH]), int(c[N.CTL_ALLOCS]), int(c[N.CTL_FREES]),
                    int(c[N.CTL_PEAK]), int(c[N.CTL_ADVANCES]), int(c[N.CTL_RELEASED]),
                    int(c[N.CTL_FREE_SIZE]), allocated]}


def ragged(d, key, i):
    off = d[key + "_off"]
    return d[key][off[i] : off[i + 1]]


@pytest.mark.parametrize("seed", [1, 2, 3, 4])
def test_mirror_follows_reference_traces(golden_dir, seed):
    d = np.load(golden_dir / f"alloc_trace_{seed}.npz")
    m = HostMirror(int(d["n_blocks"]))
    rd = Readers(int(d["interval"]))
    for i, (op, arg, want) in enumerate(zip(d["ops"], d["args"], d["results"])):
        arg = int(arg)
        if op == A_ALLOC:
            try:
                got = int(m.alloc(1, rd.tick())[0])
            except MirrorRefused as e:
                assert e.code == N.AKV_ERR_EXHAUSTED
                got = -3
        elif op == A_INC:
            try:
                m.incref([arg], rd.tick())
                got = 0
            except MirrorRefused as e:
                assert e.code == N.AKV_ERR_NOT_ALLOCATED and e.id == arg
                got = -5
        elif op == A_DEC:
            try:
                got = int(m.decref([arg], rd.tick())[0] > 0)
            except MirrorRefused as e:
                assert e.code == N.AKV_ERR_DOUBLE_FREE and e.id == arg
                got = -4
        elif op == A_ENTER:
            got = m.ctl_word(N.CTL_EPOCH)
            rd.set.add(got)
        elif op == A_LEAVE:
            rd.set.discard(arg)
            m.release(rd.safe())
            got = 0
        else:
            m.advance(rd.tick())
            got = 0
        assert got == int(want), f"op {i} ({op}, {arg})"
        s = mirror_state(m)
        np.testing.assert_array_equal(s["ref"], d["ref"][i], err_msg=f"ref after op {i}")
        np.testing.assert_array_equal(s["free"], ragged(d, "free", i), err_msg=f"free after op {i}")
        np.testing.assert_array_equal(s["pending"], ragged(d, "pend_ids", i), err_msg=f"pending {i}")
        np.testing.assert_array_equal(s["pending_epochs"], ragged(d, "pend_eps", i))
        np.testing.assert_array_equal(s["deferred"], ragged(d, "deferred", i), err_msg=f"deferred {i}")
        assert s["ctl"] == [int(x) for x in d["ctl"][i]], f"counters after op {i}"


def _assert_same(m: HostMirror, o: O.OracleAllocator, where: str) -> None:
    s, t = mirror_state(m), o.state()
    np.testing.assert_array_equal(s["ref"], t["ref_counts"], err_msg=f"ref {where}")
    np.testing.assert_array_equal(s["free"], t["free_list"], err_msg=f"free {where}")
    np.testing.assert_array_equal(s["deferred"], t["deferred"], err_msg=f"deferred {where}")
    np.testing.assert_array_equal(s["pending"], t["pending"], err_msg=f"pending {where}")
    np.testing.assert_array_equal(s["pending_epochs"], t["pending_epochs"], err_msg=f"tags {where}")
    assert s["ctl"] == [t["op_count"], t["epoch"], t["total_allocs"], t["total_frees"], t["peak_allocated"],
                        t["epoch_advances"], t["blocks_freed"], len(t["free_list"]), t["allocated_blocks"]], where


@pytest.mark.parametrize("seed", range(6))
def test_mirror_random_batches_match_oracle(seed):
    n_blocks = [40, 200, 1000, 17, 333, 64][seed]
    interval = [5, 64, 3, 1, 7, 2][seed]
    rng = np.random.default_rng(500 + seed)
    m = HostMirror(n_blocks)
    o = O.OracleAllocator(n_blocks, interval)
    rd = Readers(interval)
    tokens = []
    for step in range(200):
        r = rng.random()
        live = np.flatnonzero(o.state()["ref_counts"] > 0).astype(np.int32)
        err_m = err_o = None
        if r < 0.25:
            n = int(rng.integers(1, max(2, n_blocks // 3)))
            try:
                want = o.alloc_batch(n)
            except O.OracleError as e:
                err_o = e.code
            try:
                got = m.alloc(n, rd.tick())
            except MirrorRefused as e:
                err_m = e.code
            if err_o is None and err_m is None:
                np.testing.assert_array_equal(got, want)
        elif r < 0.45 and len(live):
            ids = rng.choice(live, size=int(rng.integers(1, 3 * len(live) + 1)))
            if rng.random() < 0.1:
                ids[rng.integers(0, len(ids))] = rng.integers(0, n_blocks)
            try:
                o.inc_ref_batch(ids)
            except O.OracleError as e:
                err_o = e.code
            try:
                m.incref(ids, rd.tick())
            except MirrorRefused as e:
                err_m = e.code
        elif r < 0.7 and len(live):
            refs = o.state()["ref_counts"]
            pool = []
            for b in rng.choice(live, size=min(len(live), int(rng.integers(1, len(live) + 1))), replace=False):
                k = int(refs[b]) if rng.random() < 0.6 else int(rng.integers(1, refs[b] + 1))
                pool += [int(b)] * k
            if rng.random() < 0.08:
                pool += [int(rng.choice(live))] * 4
            ids = np.asarray(pool, np.int32)
            rng.shuffle(ids)
            try:
                want_ret = o.dec_ref_batch(ids)
            except O.OracleError as e:
                err_o = e.code
            try:
                _, got_ret = m.decref(ids, rd.tick(), retired=True)
            except MirrorRefused as e:
                err_m = e.code
            if err_o is None and err_m is None:
                np.testing.assert_array_equal(got_ret, want_ret)
        elif r < 0.78 and len(live):
            b = int(rng.choice(live))
            try:
                got = m.cow(b, rd.tick())
            except MirrorRefused as e:
                err_m = e.code
            try:
                out, copied = o.cow_batch([b])
                want = int(out[0])
            except O.OracleError as e:
                err_o = e.code
            if err_o is None and err_m is None:
                assert got == want, (step, b)
        elif r < 0.86:
            t1 = m.ctl_word(N.CTL_EPOCH)
            assert t1 == o.enter_read_section()
            rd.set.add(t1)
            tokens.append(t1)
        elif r < 0.93 and tokens:
            t = tokens.pop(int(rng.integers(0, len(tokens))))
            rd.set.discard(t)  # a set: readers of one epoch share one entry, as in the reference
            o.leave_read_section(t)
            m.release(rd.safe())
        else:
            m.advance(rd.tick())
            o.maybe_advance_epoch()
        assert (err_m is None) == (err_o is None), f"step {step}: {err_m} vs {err_o}"
        _assert_same(m, o, f"step {step}")


def test_mirror_log_records():
    m = HostMirror(16)
    rd = Readers(4)
    ids = m.alloc(3, rd.tick())
    m.incref(ids[:2], rd.tick())
    assert m.cow(int(ids[0]), rd.tick()) != ids[0]
    m.decref(ids[1:], rd.tick())
    rd.set.add(m.ctl_word(N.CTL_EPOCH))
    m.advance(rd.tick())
    m.release(7)
    with pytest.raises(MirrorRefused):
        m.incref([0], rd.tick())  # block 0 is free: refused calls are not logged
    log = np.zeros(m.log_words(), np.int32)
    assert m.take_log(log) == len(log) and m.log_words() == 0
    ops, w = [], 0
    while w < len(log):
        op, n = int(log[w]), int(log[w + 1])
        ops.append((op, log[w + N.LOG_HEADER_WORDS : w + N.LOG_HEADER_WORDS + n].tolist()))
        w += N.LOG_HEADER_WORDS + n
    assert [o for o, _ in ops] == [N.OP_ALLOC, N.OP_INCREF, N.OP_COW, N.OP_DECREF, N.OP_ADVANCE, N.OP_RELEASE]
    assert ops[0][1] == ids.tolist() and ops[1][1] == ids[:2].tolist() and ops[3][1] == ids[1:].tolist()
    assert ops[2][1][0] == ids[0]
    # the release record carries its safe epoch, the advance its reader summary
    rel = log[-N.LOG_HEADER_WORDS:]
    assert int(rel[2]) == 7 and int(rel[3]) == 0
