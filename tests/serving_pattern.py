"""A prefix-cache serving lifecycle, driven the way a serving engine's
radix-cache adapter drives the pool (the reference's SGLang adapter,
integrations/sglang/radix_cache.py:107-218): a request first looks up its
shared prefix (DualRadixTree.match_prefix) and adopts the returned handle
when at least one whole page hit, else creates a root; while it runs, its
prompt and generated tokens are appended, blocks are allocated as pages
fill and the page-aligned prefix is committed; a finished request is synced
once more and freed, an aborted one is freed without that; epoch advances
stand for eviction.

serve(api) plays a seeded schedule of interleaved requests through `api` —
the pool's calls plus tree_match_prefix / tree_free (the tree's own
match_prefix and free, which the adapter reaches through pool._tree) and
the free_blocks / allocated_blocks counters — and returns what the engine
observes: hits with their lengths and block ids, misses, evictions, the
counters after every tick.
"""

from __future__ import annotations

import random

VOCAB = 128_256


def serve(api, page: int = 16, ticks: int = 80, seed: int = 21) -> list:
    rng = random.Random(seed)
    prefixes = [[rng.randrange(VOCAB) for _ in range(rng.randrange(1, 5) * page + rng.randrange(page))]
                for _ in range(6)]
    active = {}  # rid -> [handle, tokens, decode steps left, aborts]
    obs = []
    next_rid = 0

    def sync(rid: int) -> None:
        h, tokens = active[rid][0], active[rid][1]
        new = tokens[len(h.tokens):]
        if new:
            api.append_tokens(h, new)
        need = (len(h.tokens) + page - 1) // page
        while len(api.get_block_ids(h)) < need:
            api.allocate_block(h)
        committable = (len(h.tokens) // page) * page - h.shared_match_len
        if committable > 0:
            api.commit_prefix(h, committable)

    for tick in range(ticks):
        if len(active) < 8 and rng.random() < 0.6:
            rid, next_rid = next_rid, next_rid + 1
            tokens = list(rng.choice(prefixes)) + [rng.randrange(VOCAB) for _ in range(rng.randrange(0, 40))]
            h, n = api.tree_match_prefix(tokens)
            hit = (n // page) * page
            if h is not None and hit == 0:
                api.tree_free(h)
                h = None
            if h is None:
                obs.append(("miss", rid))
                h = api.create_root(tokens)
            else:
                obs.append(("hit", rid, hit, list(api.get_block_ids(h)[: hit // page])))
            active[rid] = [h, tokens, rng.randrange(1, 30), rng.random() < 0.15]
            sync(rid)
        for rid in sorted(active):
            entry = active[rid]
            entry[1] = entry[1] + [rng.randrange(VOCAB)]  # one generated token
            entry[2] -= 1
            if entry[2] > 0:
                sync(rid)
                continue
            if entry[3]:
                obs.append(("abort", rid))
            else:
                sync(rid)
                obs.append(("finish", rid, len(entry[0].tokens)))
            api.free(entry[0])
            del active[rid]
        if rng.random() < 0.2:
            before = api.free_blocks
            api.maybe_advance_epoch()
            obs.append(("evict", api.free_blocks - before))
        obs.append(("counts", tick, api.free_blocks, api.allocated_blocks))
    for rid in sorted(active):
        api.free(active[rid][0])
    obs.append(("end", api.free_blocks, api.allocated_blocks))
    return obs


class OracleServeAPI:
    """The oracle's tree and allocator with the call set serve() uses."""

    def __init__(self, n_blocks: int, page: int) -> None:
        from oracle import oracle as O

        self.alloc = O.OracleAllocator(n_blocks)
        self.tree = O.OracleTree(self.alloc, page)
        self.n = n_blocks

    def __getattr__(self, name):
        return getattr(self.tree, name)

    def tree_match_prefix(self, tokens):
        return self.tree.match_prefix(tokens)

    def tree_free(self, h):
        self.tree.free(h)

    def maybe_advance_epoch(self):
        self.alloc.maybe_advance_epoch()

    @property
    def free_blocks(self) -> int:
        return self.alloc.free_count

    @property
    def allocated_blocks(self) -> int:
        st = self.alloc.state()
        return self.n - len(st["free_list"]) - len(st["pending"]) - len(st["deferred"])


class PoolServeAPI:
    """agentkv_b200.AgentKVPool with the call set serve() uses."""

    def __init__(self, pool) -> None:
        self.pool = pool

    def __getattr__(self, name):
        return getattr(self.pool, name)

    def tree_match_prefix(self, tokens):
        return self.pool._tree.match_prefix(tokens)

    def tree_free(self, h):
        self.pool._tree.free(h)
