"""Seeded lookup scenarios with hard tree shapes, shared by the fixture
generator (run on the reference), the oracle and the package:

* colliding — 24 root children whose (parent, first token) keys share the
  low ten bits of the slot hash, so they sit in one probe chain several
  8-slot windows long; queries find each inserted sequence, miss on first
  tokens that join the chain without being in the tree, and cut inside
  edges;
* long_chain — a 70-node unary chain (prefixes of one sequence committed one
  block longer each time) with a branch at depth 100; queries cut at every
  depth, diverge at every third position and run past the end.

A scenario is {"block_size", "inserts" (token lists, each committed whole
after create_root and enough blocks), "queries"}.
"""

from __future__ import annotations

import numpy as np


def colliding() -> dict:
    from agentkv_b200.device_tree import tree_hash_np

    toks = np.arange(1, 200000, dtype=np.int64)
    h = tree_hash_np(np.zeros_like(toks), toks)
    same = toks[(h & 1023) == (h[0] & 1023)]
    firsts, absent = same[:24].tolist(), same[24:30].tolist()
    rng = np.random.default_rng(5)
    seqs = [[int(f)] + rng.integers(0, 50000, size=11).tolist() for f in firsts]
    queries = [s + [7, 7, 7] for s in seqs] + [[int(a)] + seqs[0][1:] for a in absent] + [s[:8] for s in seqs[:4]]
    return {"block_size": 4, "inserts": seqs, "queries": queries}


def long_chain() -> dict:
    bs = 4
    rng = np.random.default_rng(23)
    seq = rng.integers(0, 50000, size=70 * bs).tolist()
    branch = seq[:100] + rng.integers(50000, 60000, size=40).tolist()
    queries = [seq[:n] for n in range(0, len(seq) + 1)] + [seq + [1, 2, 3], branch + [9], branch[:103]]
    for p in range(0, len(seq), 3):
        q = list(seq)
        q[p] = 99999
        queries.append(q)
    return {"block_size": bs, "inserts": [seq[: bs * k] for k in range(1, 71)] + [branch], "queries": queries}


def build(tree, scenario: dict, allocate_one) -> None:
    """Insert the scenario's sequences through the pool-style calls of
    `tree` (create_root, get_block_ids, commit_prefix); allocate_one(handle)
    adds one block to a handle."""
    bs = scenario["block_size"]
    for s in scenario["inserts"]:
        h = tree.create_root(s)
        while len(tree.get_block_ids(h)) < -(-len(s) // bs):
            allocate_one(h)
        tree.commit_prefix(h, len(s) - h.shared_match_len)


SCENARIOS = {"colliding": colliding, "long_chain": long_chain}
