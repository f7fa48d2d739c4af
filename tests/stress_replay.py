"""Replay of the reference stress runner's recorded calls (fixtures
tests/golden/stress_<seed>.npz, recorded from the reference's own
tests/test_stress.py StressRunner with the seeds and op counts of its tests)
through any tree + allocator with the reference's call set."""

S_CREATE, S_FORK, S_ALLOC, S_FREE, S_ADVANCE = range(5)


def replay(g, tree, advance, is_exhausted) -> None:
    """tree: create_root / fork / allocate_block / free; advance():
    maybe_advance_epoch; is_exhausted(exc) says whether an exception is the
    pool-exhausted error.  Every returned handle id and block id must equal
    the recorded one."""
    live = {}
    ops, toks, t_off = g["ops"], g["tokens"], g["tokens_off"]
    for i, (kind, a, b) in enumerate(ops):
        a, b = int(a), int(b)
        if kind == S_CREATE:
            h = tree.create_root(toks[t_off[i]:t_off[i + 1]].tolist())
            assert h.handle_id == a, (i, h.handle_id, a)
            live[a] = h
        elif kind == S_FORK:
            c = tree.fork(live[a])
            assert c.handle_id == b, (i, c.handle_id, b)
            live[b] = c
        elif kind == S_ALLOC:
            try:
                bid = tree.allocate_block(live[a])
                bid = bid if isinstance(bid, int) else bid.block_id
            except Exception as e:  # noqa: BLE001 - the recorded outcome decides
                if not is_exhausted(e):
                    raise
                bid = -3
            assert bid == b, (i, bid, b)
        elif kind == S_FREE:
            tree.free(live.pop(a))
        elif kind == S_ADVANCE:
            advance()
        else:
            raise ValueError(f"unknown op {kind}")
    assert not live, f"{len(live)} agents left alive"  # the runner frees every agent at the end


def seeds():
    return (1, 2, 7, 13, 17, 42, 137, 999)
