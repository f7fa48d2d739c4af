"""Generate golden fixtures by running the reference AgentKV implementation.

Run where a checkout of the reference exists (it is only read), naming it
with --reference or the AGENTKV_REFERENCE environment variable:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py \
        --reference /root/reference [--skip-full-match]

It imports the reference's own `agentkv` package and records, for seeded
inputs, what the reference's code returns: allocator op traces (ids,
refcounts, free-list order, reclaimer queues, counters), tree op traces
(block tables, tree structure, match results), the quickstart and
Tree-of-Thought workloads, copy/zero contents and match_prefix results on
the stress tree.  The fixtures are what the oracle and the CUDA path are
pinned against; nothing at test time reads the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import random
import sys
import time
from pathlib import Path

import numpy as np

def _reference_root() -> Path:
    """The reference checkout: --reference PATH, else $AGENTKV_REFERENCE."""
    argv = sys.argv[1:]
    for i, a in enumerate(argv):
        if a == "--reference" and i + 1 < len(argv):
            return Path(argv[i + 1])
        if a.startswith("--reference="):
            return Path(a.split("=", 1)[1])
    env = os.environ.get("AGENTKV_REFERENCE")
    if env:
        return Path(env)
    sys.exit("make_golden.py: name the reference checkout with --reference PATH or AGENTKV_REFERENCE")


REF = _reference_root()
if not (REF / "agentkv" / "core" / "radix_tree.py").exists():
    sys.exit(f"make_golden.py: {REF} does not hold the reference's agentkv package")
OUT = Path(__file__).resolve().parent
REPO = OUT.parent.parent
sys.path.insert(0, str(REF))
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

from agentkv.core.config import PoolConfig  # noqa: E402
from agentkv.core.slab_allocator import SlabAllocator, BlockHandle  # noqa: E402
from agentkv.core.radix_tree import DualRadixTree, INVALID_NODE_ID  # noqa: E402
from agentkv.pool import AgentKVPool  # noqa: E402

from agentkv_b200 import workloads as W  # noqa: E402  (seeded generators only)

# opcodes shared with the replaying tests
A_ALLOC, A_INC, A_DEC, A_ENTER, A_LEAVE, A_ADVANCE = range(6)
ERR_EXHAUSTED, ERR_DOUBLE_FREE, ERR_NOT_ALLOCATED = 3, 4, 5


def alloc_snapshot(a: SlabAllocator) -> dict:
    r = a._reclaimer
    return {
        "ref": a._ref_counts.numpy().astype(np.int32).copy(),
        "free": np.asarray(list(a._free_list), np.int32),
        "pend_ids": np.asarray([b for _, b in r._pending], np.int32),
        "pend_eps": np.asarray([e for e, _ in r._pending], np.int64),
        "deferred": np.asarray(list(a._deferred_free), np.int32),
        "ctl": np.asarray(
            [a._op_count, r._epoch, a._alloc_count, a._free_count, a._peak_allocated,
             r._advance_count, r._freed_count, len(a._free_list),
             int((a._ref_counts > 0).sum())], np.int64),
    }


# ── A. allocator traces ──────────────────────────────────────────────────────
def alloc_trace(seed: int, n_blocks: int, interval: int, n_ops: int) -> dict:
    cfg = PoolConfig(total_blocks=n_blocks, block_size=4, num_layers=1, num_kv_heads=1,
                     head_dim=4, dtype="float16", device="meta", epoch_interval=interval)
    a = SlabAllocator(cfg)
    rng = random.Random(seed)
    tokens_open: list[int] = []
    ops, args, results = [], [], []
    snaps = []
    burst = 0
    for _ in range(n_ops):
        live = [i for i in range(n_blocks) if int(a._ref_counts[i]) > 0]
        r = rng.random()
        if burst > 0:
            op = A_ALLOC
            burst -= 1
        elif r < 0.28:
            op = A_ALLOC
        elif r < 0.30:
            op, burst = A_ALLOC, rng.randint(5, 20)
        elif r < 0.45:
            op = A_INC
        elif r < 0.78:
            op = A_DEC
        elif r < 0.85:
            op = A_ENTER
        elif r < 0.92:
            op = A_LEAVE
        else:
            op = A_ADVANCE
        arg = 0
        if op == A_ALLOC:
            try:
                res = a.alloc().block_id
            except MemoryError:
                res = -ERR_EXHAUSTED
        elif op in (A_INC, A_DEC):
            if live and rng.random() < 0.93:
                arg = rng.choice(live)
            else:
                arg = rng.randrange(n_blocks)
            try:
                if op == A_INC:
                    a.inc_ref(BlockHandle(arg))
                    res = 0
                else:
                    res = 1 if a.dec_ref(BlockHandle(arg)) else 0
            except ValueError:
                res = -(ERR_NOT_ALLOCATED if op == A_INC else ERR_DOUBLE_FREE)
        elif op == A_ENTER:
            res = a.enter_read_section()
            tokens_open.append(res)
        elif op == A_LEAVE:
            if tokens_open:
                arg = tokens_open.pop(rng.randrange(len(tokens_open)))
                a.leave_read_section(arg)
                res = 0
            else:
                op, res = A_ADVANCE, 0
                a.maybe_advance_epoch()
        else:
            a.maybe_advance_epoch()
            res = 0
        ops.append(op)
        args.append(arg)
        results.append(res)
        snaps.append(alloc_snapshot(a))
    out = {
        "n_blocks": np.int64(n_blocks), "interval": np.int64(interval),
        "ops": np.asarray(ops, np.int32), "args": np.asarray(args, np.int64),
        "results": np.asarray(results, np.int64),
        "ref": np.stack([s["ref"] for s in snaps]),
        "ctl": np.stack([s["ctl"] for s in snaps]),
    }
    # ragged arrays: concatenated with offsets
    for key in ("free", "pend_ids", "pend_eps", "deferred"):
        vals = [s[key] for s in snaps]
        off = np.zeros(len(vals) + 1, np.int64)
        np.cumsum([len(v) for v in vals], out=off[1:])
        out[key] = np.concatenate(vals) if off[-1] else np.zeros(0, vals[0].dtype)
        out[key + "_off"] = off
    return out


# ── B. tree traces ───────────────────────────────────────────────────────────
T_CREATE, T_FORK, T_ALLOC, T_COW, T_APPEND, T_COMMIT, T_FREE, T_MATCH, T_ADVANCE, T_ZERO = range(10)


def tree_state(pool: AgentKVPool, live: dict) -> dict:
    tree, a = pool._tree, pool._allocator
    nodes = {}
    for nid, n in sorted(tree._shared_nodes.items()):
        nodes[str(nid)] = {
            "parent": n.parent_id, "edge": list(n.edge_tokens), "blocks": [b.block_id for b in n.blocks],
            "children": sorted([int(k), int(v)] for k, v in n.children.items()), "ref": n.ref_count,
        }
    return {
        "tables": {str(h): tree.get_block_ids(hd) for h, hd in sorted(live.items())},
        "shared": {str(h): [hd.shared_node_id, hd.shared_match_len] for h, hd in sorted(live.items())},
        "nodes": nodes,
        "ref": a._ref_counts.tolist(),
        "free": list(a._free_list),
        "stats": pool.stats(),
    }


def tree_trace(seed: int, n_ops: int, n_blocks: int = 96, bs: int = 4) -> dict:
    cfg = PoolConfig(total_blocks=n_blocks, block_size=bs, num_layers=1, num_kv_heads=2,
                     head_dim=4, dtype="float16", device="cpu", epoch_interval=7)
    pool = AgentKVPool(config=cfg)
    torch.manual_seed(seed)
    pool._allocator._kv_data.copy_(torch.randn_like(pool._allocator._kv_data, dtype=torch.float32).half())
    rng = random.Random(seed)
    bases = [[rng.randrange(6) for _ in range(40)] for _ in range(4)]

    def gen_tokens():
        b = rng.choice(bases)
        cut = rng.randint(0, 40)
        tail = [rng.randrange(6) for _ in range(rng.randint(0, 14))]
        return b[:cut] + tail

    live: dict = {}
    ops, states = [], []
    for step in range(n_ops):
        hs = sorted(live)
        r = rng.random()
        op = (T_CREATE if (not hs or r < 0.16) else T_FORK if r < 0.28 else T_ALLOC if r < 0.46
              else T_COW if r < 0.56 else T_APPEND if r < 0.62 else T_COMMIT if r < 0.76
              else T_FREE if r < 0.86 else T_MATCH if r < 0.95 else T_ADVANCE if r < 0.98 else T_ZERO)
        rec = {"op": op}
        try:
            if op == T_CREATE:
                toks = gen_tokens()
                h = pool.create_root(toks)
                live[h.handle_id] = h
                rec.update(tokens=toks, out=[h.handle_id, h.shared_node_id, h.shared_match_len])
            elif op == T_FORK:
                p = live[rng.choice(hs)]
                c = pool.fork(p)
                live[c.handle_id] = c
                rec.update(h=p.handle_id, out=c.handle_id)
            elif op == T_ALLOC:
                h = live[rng.choice(hs)]
                pool.allocate_block(h)
                rec.update(h=h.handle_id, out=h.residual_blocks[-1].block_id)
            elif op == T_COW:
                h = live[rng.choice(hs)]
                if not h.residual_blocks:
                    rec.update(op=T_ADVANCE)
                    pool.maybe_advance_epoch()
                else:
                    idx = rng.randrange(len(h.residual_blocks))
                    pool.ensure_mutable_block(h, idx)
                    rec.update(h=h.handle_id, idx=idx, out=h.residual_blocks[idx].block_id)
            elif op == T_APPEND:
                h = live[rng.choice(hs)]
                toks = [rng.randrange(6) for _ in range(rng.randint(0, 9))]
                pool.append_tokens(h, toks)
                rec.update(h=h.handle_id, tokens=toks)
            elif op == T_COMMIT:
                h = live[rng.choice(hs)]
                k = rng.randint(0, len(h.residual_blocks) + 1)
                length = k * bs if rng.random() < 0.9 else k * bs + 1
                rec.update(h=h.handle_id, length=length)
                pool.commit_prefix(h, length)
                rec.update(out=[h.shared_node_id, h.shared_match_len])
            elif op == T_FREE:
                h = live.pop(rng.choice(hs))
                pool.free(h)
                rec.update(h=h.handle_id)
            elif op == T_MATCH:
                toks = gen_tokens()
                mh, mlen = pool._tree.match_prefix(toks)
                rec.update(tokens=toks, out=[-1 if mh is None else mh.handle_id, mlen,
                                              INVALID_NODE_ID if mh is None else mh.shared_node_id])
                if mh is not None:
                    live[mh.handle_id] = mh
            elif op == T_ADVANCE:
                pool.maybe_advance_epoch()
            elif op == T_ZERO:
                h = live[rng.choice(hs)]
                if h.residual_blocks:
                    b = rng.choice(h.residual_blocks)
                    rec.update(h=h.handle_id, block=b.block_id)
                    pool._allocator.zero_block(b)
                else:
                    rec.update(op=T_ADVANCE)
                    pool.maybe_advance_epoch()
        except (ValueError, MemoryError) as e:
            rec["error"] = type(e).__name__
        ops.append(rec)
        if step % 10 == 9 or step == n_ops - 1:
            states.append([step, tree_state(pool, live)])
    digests = [hashlib.sha256(pool._allocator._kv_data[i].numpy().tobytes()).hexdigest()
               for i in range(n_blocks)]
    return {"seed": seed, "n_blocks": n_blocks, "block_size": bs, "ops": ops, "states": states,
            "block_sha256": digests}


# ── C. quickstart ────────────────────────────────────────────────────────────
def quickstart() -> dict:
    N, bs, L, H, D, dt = W.QUICKSTART_GEOMETRY
    cfg = PoolConfig(total_blocks=N, block_size=bs, num_layers=L, num_kv_heads=H, head_dim=D,
                     dtype=dt, device="cpu")
    pool = AgentKVPool(config=cfg)
    torch.manual_seed(0)
    pool._allocator._kv_data.copy_(torch.randn(pool._allocator._kv_data.shape, dtype=torch.float16))
    pairs = []
    orig = pool._allocator.copy_block

    def rec_copy(src, dst):
        pairs.append([src.block_id, dst.block_id])
        orig(src, dst)

    pool._allocator.copy_block = rec_copy
    root = pool.create_root(list(range(32)))
    pool.allocate_block(root)
    kids = [pool.fork(root) for _ in range(3)]
    for c in kids:
        pool.allocate_block(c)
    for c in kids:
        pool.ensure_mutable_block(c, 0)
    pool.commit_prefix(root, 16)
    matches = []
    for q in W.quickstart_queries():
        mh, mlen = pool._tree.match_prefix(q)
        matches.append([-1 if mh is None else mh.shared_node_id, mlen])
    kv = pool._allocator._kv_data
    return {
        "children": [pool.get_block_ids(c) for c in kids],
        "root": pool.get_block_ids(root),
        "pairs": pairs,
        "ref": pool._allocator._ref_counts.tolist(),
        "free": list(pool._allocator._free_list),
        "matches": matches,
        "queries": W.quickstart_queries(),
        "stats": pool.stats(),
        "block_sha256": [hashlib.sha256(kv[i].numpy().tobytes()).hexdigest() for i in range(N)],
    }


# ── D. Tree-of-Thought fan-out (metadata, full 60,000-block pool) ────────────
def tot() -> dict:
    N, bs, L, H, D, dt = W.LLAMA3_8B_GEOMETRY
    spec = W.ToTSpec()
    cfg = PoolConfig(total_blocks=N, block_size=bs, num_layers=L, num_kv_heads=H, head_dim=D,
                     dtype=dt, device="meta")
    pool = AgentKVPool(config=cfg)
    pairs = []
    orig = pool._allocator.copy_block

    def rec_copy(src, dst):
        pairs.append((src.block_id, dst.block_id))
        orig(src, dst)

    pool._allocator.copy_block = rec_copy
    root = pool.create_root(W.tot_root_tokens(spec))
    for _ in range(spec.root_tokens // bs):
        pool.allocate_block(root)
    level = [root]
    kids_all = []
    level_pairs = []
    for lvl in range(spec.levels):
        nxt = []
        p0 = len(pairs)
        for pi, parent in enumerate(level):
            for k in range(spec.fanout):
                c = pool.fork(parent)
                pool.ensure_mutable_block(c, len(c.residual_blocks) - 1)
                pool.append_tokens(c, W.tot_append_tokens(spec, lvl, pi * spec.fanout + k))
                for _ in range(spec.appended_blocks):
                    pool.allocate_block(c)
                nxt.append(c)
        level_pairs.append(np.asarray(pairs[p0:], np.int32))
        kids_all.extend(nxt)
        level = nxt
    a = pool._allocator
    after_fanout = {
        "tables": [np.asarray(pool.get_block_ids(c), np.int32) for c in kids_all],
        "ref": a._ref_counts.numpy().astype(np.int32).copy(),
        "free": np.asarray(list(a._free_list), np.int32),
        "stats": pool.stats(),
    }
    for c in kids_all:
        pool.free(c)
    after_free = {
        "ref": a._ref_counts.numpy().astype(np.int32).copy(),
        "free": np.asarray(list(a._free_list), np.int32),
        "stats": pool.stats(),
    }
    tables = after_fanout["tables"]
    t_off = np.zeros(len(tables) + 1, np.int64)
    np.cumsum([len(t) for t in tables], out=t_off[1:])
    return {
        "root_table": np.asarray(pool.get_block_ids(root), np.int32),
        "tables": np.concatenate(tables), "tables_off": t_off,
        "pairs_l0": level_pairs[0], "pairs_l1": level_pairs[1], "pairs_l2": level_pairs[2],
        "ref_fanout": after_fanout["ref"], "free_fanout": after_fanout["free"],
        "ref_freed": after_free["ref"], "free_freed": after_free["free"],
        "stats_fanout": np.asarray(json.dumps(after_fanout["stats"])),
        "stats_freed": np.asarray(json.dumps(after_free["stats"])),
    }


# ── D2. ReAct multi-agent trace (metadata, 70B geometry, 40,000 blocks) ─────
class _RefReActAPI:
    """The reference pool's calls as workloads.react_setup / react_step use them."""

    def __init__(self, pool):
        self.p = pool

    def __getattr__(self, name):
        return getattr(self.p, name)

    def allocate_blocks(self, h, n):
        for _ in range(n):
            self.p.allocate_block(h)

    def residual_len(self, h):
        return len(h.residual_blocks)


def react(spec: W.ReActSpec, checkpoints=(200, 1000)) -> dict:
    N, bs, L, H, D, dt = W.LLAMA3_70B_GEOMETRY
    cfg = PoolConfig(total_blocks=N, block_size=bs, num_layers=L, num_kv_heads=H, head_dim=D,
                     dtype=dt, device="meta")
    pool = AgentKVPool(config=cfg)
    pairs = []
    orig = pool._allocator.copy_block

    def rec_copy(src, dst):
        pairs.append((src.block_id, dst.block_id))
        orig(src, dst)

    pool._allocator.copy_block = rec_copy
    api = _RefReActAPI(pool)
    root, agents = W.react_setup(api, spec)
    out = {"setup_pairs": np.asarray(pairs, np.int32).reshape(-1, 2)}
    step_off = [len(pairs)]
    a = pool._allocator
    for i, actions in enumerate(W.react_trace(spec)):
        W.react_step(api, root, agents, actions)
        step_off.append(len(pairs))
        if i + 1 in checkpoints:
            tables = [np.asarray(pool.get_block_ids(h), np.int32) for h in agents]
            t_off = np.zeros(len(tables) + 1, np.int64)
            np.cumsum([len(t) for t in tables], out=t_off[1:])
            k = f"s{i + 1}"
            out[f"{k}_tables"] = np.concatenate(tables)
            out[f"{k}_tables_off"] = t_off
            out[f"{k}_ref"] = a._ref_counts.numpy().astype(np.int32).copy()
            out[f"{k}_free"] = np.asarray(list(a._free_list), np.int32)
            out[f"{k}_stats"] = np.asarray(json.dumps(pool.stats()))
    out["pairs"] = np.asarray(pairs, np.int32).reshape(-1, 2)
    out["step_off"] = np.asarray(step_off, np.int64)
    out["root_table"] = np.asarray(pool.get_block_ids(root), np.int32)
    out["spec"] = np.asarray(json.dumps(spec.__dict__))
    return out


# ── D3. HuggingFace cache session (reference AgentKVCache on a CPU pool) ───
def hf_session(spec: W.HFSpec) -> dict:
    from agentkv.hf_cache import AgentKVCache

    cfg = PoolConfig(total_blocks=spec.total_blocks, block_size=spec.block_size, num_layers=spec.num_layers,
                     num_kv_heads=spec.num_kv_heads, head_dim=spec.head_dim, dtype=spec.dtype, device="cpu")
    pool = AgentKVPool(config=cfg)
    outs, keys = [], []

    def on_output(e, layer, ok, ov):
        keys.append((e, layer, ok.shape[2]))
        outs.append(np.concatenate([ok.numpy().reshape(-1), ov.numpy().reshape(-1)]))

    caches = W.hf_run(spec, pool, AgentKVCache, torch.from_numpy, on_output)
    tables = [np.asarray(pool.get_block_ids(c.handle), np.int32) for c in caches]
    t_off = np.zeros(len(tables) + 1, np.int64)
    np.cumsum([len(t) for t in tables], out=t_off[1:])
    return {
        "out_keys": np.asarray(keys, np.int64), "outs": np.concatenate(outs),
        "tables": np.concatenate(tables), "tables_off": t_off,
        "seen": np.asarray([c.get_seq_length() for c in caches], np.int64),
        "pool": pool._allocator._kv_data.numpy().copy(),
        "spec": np.asarray(json.dumps(spec.__dict__)),
    }


# ── D4. the reference's own stress runner (tests/test_stress.py), recorded ────
S_CREATE, S_FORK, S_ALLOC, S_FREE, S_ADVANCE = range(5)


class _Recorder:
    """Forwards to a pool object and logs the runner-level calls."""

    def __init__(self, obj, log):
        self._obj = obj
        self._log = log

    def __getattr__(self, name):
        attr = getattr(self._obj, name)
        log = self._log
        if name == "create_root":
            def f(tokens):
                h = attr(tokens)
                log.append((S_CREATE, h.handle_id, 0, list(tokens)))
                return h
        elif name == "fork":
            def f(parent):
                c = attr(parent)
                log.append((S_FORK, parent.handle_id, c.handle_id, []))
                return c
        elif name == "allocate_block":
            def f(h):
                try:
                    b = attr(h)
                except MemoryError:
                    log.append((S_ALLOC, h.handle_id, -3, []))
                    raise
                log.append((S_ALLOC, h.handle_id, b.block_id, []))
                return b
        elif name == "free":
            def f(h):
                attr(h)
                log.append((S_FREE, h.handle_id, 0, []))
        elif name == "maybe_advance_epoch":
            def f():
                attr()
                log.append((S_ADVANCE, 0, 0, []))
        else:
            return attr
        return f


def stress(seed: int, n_ops: int) -> dict:
    sys.path.insert(0, str(REF / "tests"))
    import test_stress as TS  # noqa: E402  (the reference's runner, run as is)

    cfg = PoolConfig(total_blocks=512, block_size=4, num_layers=2, num_kv_heads=2, head_dim=8,
                     dtype="float16", device="cpu")
    runner = TS.StressRunner(cfg, n_operations=n_ops, seed=seed)
    log = []
    alloc = runner._alloc
    runner._tree = _Recorder(runner._tree, log)
    runner._alloc = _Recorder(alloc, log)
    violations = runner.run()
    toks = [t for e in log for t in e[3]]
    t_off = np.zeros(len(log) + 1, np.int64)
    np.cumsum([len(e[3]) for e in log], out=t_off[1:])
    return {
        "ops": np.asarray([(e[0], e[1], e[2]) for e in log], np.int64),
        "tokens": np.asarray(toks or [0], np.int32), "tokens_off": t_off,
        "violations": np.asarray(len(violations)),
        "ref": alloc._ref_counts.numpy().astype(np.int32).copy(),
        "free": np.asarray(list(alloc._free_list), np.int32),
        "stats": np.asarray(json.dumps(alloc.stats())),
        "seed": np.asarray(seed), "n_ops": np.asarray(n_ops),
    }


# ── E. copy / zero contents on the CPU path ──────────────────────────────────
def copy_zero() -> dict:
    cfg = PoolConfig(total_blocks=32, block_size=4, num_layers=2, num_kv_heads=2, head_dim=8,
                     dtype="bfloat16", device="cpu")
    a = SlabAllocator(cfg)
    torch.manual_seed(11)
    a._kv_data.copy_(torch.randn(a._kv_data.shape, dtype=torch.float32).to(torch.bfloat16))
    a._kv_data[3].fill_(-1.5)  # negative values: CPU zero gives +0.0, Triton x*0 gives -0.0
    a._kv_data[4].fill_(float("nan"))
    handles = [a.alloc() for _ in range(32)]  # ids 31..0
    by_id = {h.block_id: h for h in handles}
    rng = random.Random(12)
    ops = []
    for _ in range(40):
        if rng.random() < 0.6:
            s, d = rng.sample(range(32), 2)
            a.copy_block(by_id[s], by_id[d])
            ops.append(["copy", s, d])
        else:
            z = rng.randrange(32)
            a.zero_block(by_id[z])
            ops.append(["zero", z])
    a.zero_block(by_id[3])
    a.zero_block(by_id[4])
    ops += [["zero", 3], ["zero", 4]]
    a.inc_ref(by_id[7])
    errs = []
    for fn, args, msg_key in ((a.copy_block, (by_id[1], by_id[7]), "copy"), (a.zero_block, (by_id[7],), "zero")):
        try:
            fn(*args)
        except ValueError as e:
            errs.append([msg_key, str(e)])
    kv = a._kv_data
    return {"ops": ops, "errors": errs,
            "block_sha256": [hashlib.sha256(kv[i].view(torch.int16).numpy().tobytes()).hexdigest() for i in range(32)],
            "seed": 11}


# ── F. match_prefix on the stress tree ───────────────────────────────────────
def match_stress(spec: W.MatchSpec, n_queries: int) -> dict:
    prefixes = W.match_prefixes(spec)
    corpus = W.match_sequences(spec, prefixes)
    total_blocks = sum(-(-len(s) // 16) for s in corpus) + 16
    cfg = PoolConfig(total_blocks=total_blocks, block_size=16, num_layers=1, num_kv_heads=1,
                     head_dim=1, dtype="float16", device="meta")
    pool = AgentKVPool(config=cfg)
    t0 = time.time()
    for seq in corpus:
        toks = seq.tolist()
        h = pool.create_root(toks)
        need = -(-len(toks) // 16)
        have = len(pool.get_block_ids(h))
        for _ in range(need - have):
            pool.allocate_block(h)
        share = (len(toks) // 16) * 16 - h.shared_match_len
        if share > 0:
            pool.commit_prefix(h, share)
    t_build = time.time() - t0
    queries = W.match_queries(spec, corpus, prefixes, batch=0, n=n_queries)
    t0 = time.time()
    res = np.asarray([pool._tree._match_prefix_locked(q.tolist()) for q in queries], np.int32)
    t_match = time.time() - t0
    return {
        "node": res[:, 0].copy(), "len": res[:, 1].copy(),
        "n_nodes": np.int64(len(pool._tree._shared_nodes)),
        "next_node_id": np.int64(pool._tree._next_node_id),
        "free_blocks": np.int64(pool.free_blocks),
        "total_blocks": np.int64(total_blocks),
        "build_s": np.float64(t_build), "match_s": np.float64(t_match),
        "spec": np.asarray(json.dumps(spec.__dict__)),
    }


def serving() -> dict:
    """The serving-lifecycle schedule of tests/serving_pattern.py (the
    SGLang adapter's call pattern) played on the reference pool."""
    sys.path.insert(0, str(OUT.parent))
    from serving_pattern import serve

    pool = AgentKVPool(config=PoolConfig(total_blocks=512, block_size=16, num_layers=1, num_kv_heads=1,
                                         head_dim=8, dtype="float16", device="cpu"))

    class API:
        def __getattr__(self, name):
            return getattr(pool, name)

        def tree_match_prefix(self, tokens):
            return pool._tree.match_prefix(tokens)

        def tree_free(self, h):
            pool._tree.free(h)

        @property
        def free_blocks(self):
            return pool.free_blocks

        @property
        def allocated_blocks(self):
            return pool.allocated_blocks

    return {"obs": json.loads(json.dumps(serve(API())))}


def match_scenarios() -> dict:
    """(node, length) of the reference's _match_prefix_locked on every query
    of tests/match_scenarios.py's hard tree shapes."""
    sys.path.insert(0, str(OUT.parent))
    from match_scenarios import SCENARIOS, build

    out = {}
    for name, make in SCENARIOS.items():
        sc = make()
        pool = AgentKVPool(config=PoolConfig(total_blocks=1024, block_size=sc["block_size"], num_layers=1,
                                             num_kv_heads=1, head_dim=4, dtype="float16", device="cpu"))
        build(pool, sc, pool.allocate_block)
        out[name] = [list(pool._tree._match_prefix_locked(q)) for q in sc["queries"]]
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", help="the reference checkout (read at import time above)")
    ap.add_argument("--skip-full-match", action="store_true")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    todo = set(args.only.split(",")) if args.only else {"alloc", "tree", "quick", "tot", "react", "hf", "stress",
                                                                   "copy", "match", "match_full", "serving",
                                                                   "match_scenarios"}
    if "alloc" in todo:
        for seed, (n, iv, nops) in {1: (48, 5, 700), 2: (32, 3, 700), 3: (64, 64, 900), 4: (16, 2, 500)}.items():
            np.savez_compressed(OUT / f"alloc_trace_{seed}.npz", **alloc_trace(seed, n, iv, nops))
            print("alloc trace", seed)
    if "tree" in todo:
        for seed in (1, 2, 3):
            (OUT / f"tree_trace_{seed}.json").write_text(json.dumps(tree_trace(seed, 400)))
            print("tree trace", seed)
    if "quick" in todo:
        (OUT / "quickstart.json").write_text(json.dumps(quickstart(), indent=0))
        print("quickstart")
    if "tot" in todo:
        np.savez_compressed(OUT / "tot_8b.npz", **tot())
        print("tot")
    if "react" in todo:
        np.savez_compressed(OUT / "react_70b.npz", **react(W.ReActSpec()))
        print("react")
    if "stress" in todo:
        # the seeds and op counts of the reference's stress tests
        for seed, n in ((1, 1000), (2, 10000), (42, 5000), (137, 5000), (999, 5000), (7, 10000), (13, 10000),
                        (17, 10000)):
            d = stress(seed, n)
            np.savez_compressed(OUT / f"stress_{seed}.npz", **d)
            print("stress", seed, len(d["ops"]), int(d["violations"]))
    if "hf" in todo:
        np.savez_compressed(OUT / "hf_session.npz", **hf_session(W.HFSpec()))
        print("hf")
    if "copy" in todo:
        (OUT / "copy_zero.json").write_text(json.dumps(copy_zero(), indent=0))
        print("copy/zero")
    if "match_scenarios" in todo:
        (OUT / "match_scenarios.json").write_text(json.dumps(match_scenarios()))
        print("match scenarios")
    if "serving" in todo:
        (OUT / "serving.json").write_text(json.dumps(serving()))
        print("serving")
    if "match" in todo:
        small = W.MatchSpec(n_sequences=600, n_queries=256)
        np.savez_compressed(OUT / "match_small.npz", **match_stress(small, 256))
        print("match small")
    if "match_full" in todo and not args.skip_full_match:
        d = match_stress(W.MatchSpec(), 4096)
        np.savez_compressed(OUT / "match_full.npz", **d)
        print("match full", d["n_nodes"], d["build_s"], d["match_s"])


if __name__ == "__main__":
    main()
