"""Random commits and frees on a DualRadixTree that reach every branch of
the host insert (new leaf, descent, exact re-commit, block-aligned split,
split == 0 overwrite) and the prune, for the tests that check the
replica's device-built changes (akv_tree_commands) against the host mirror.
Sequences share prefixes from a small pool and diverge at random points,
block size 4, a 12-token vocabulary: splits at and off block boundaries are
frequent."""

from __future__ import annotations

import numpy as np


def churn(tree, rng, steps: int, on_step, bs: int = 4, vocab: int = 12):
    """Drive `tree` for `steps` steps, calling on_step(step) after each."""
    stems = [rng.integers(0, vocab, size=int(rng.integers(4, 40))).tolist() for _ in range(6)]
    live = []
    for step in range(steps):
        r = rng.random()
        if r < 0.55 or len(live) < 3:
            stem = stems[int(rng.integers(len(stems)))]
            cut = int(rng.integers(0, len(stem) + 1))
            toks = stem[:cut] + rng.integers(0, vocab, size=int(rng.integers(0, 30))).tolist()
            if not toks:
                toks = [int(rng.integers(vocab))]
            h = tree.create_root(toks)
            need = -(-len(toks) // bs) - len(h.residual_blocks)
            try:
                for _ in range(max(0, need)):
                    tree.allocate_block(h)
            except MemoryError:
                tree.free(h)
                on_step(step)
                continue
            avail = len(toks) - h.shared_match_len
            n_blocks = min(len(h.residual_blocks), avail // bs)
            if n_blocks > 0 and rng.random() < 0.9:
                tree.commit_prefix(h, bs * int(rng.integers(1, n_blocks + 1)))
            live.append(h)
        elif r < 0.7:
            tree.free(live.pop(int(rng.integers(len(live)))))
        elif r < 0.8:
            # two handles of the same tokens, both created before either
            # commits: the second commit re-commits the same edge exactly or
            # descends through it
            stem = stems[int(rng.integers(len(stems)))]
            toks = stem + rng.integers(0, vocab, size=int(rng.integers(bs, 20))).tolist()
            pair = [tree.create_root(toks) for _ in range(2)]
            try:
                for h in pair:
                    for _ in range(-(-len(toks) // bs) - len(h.residual_blocks)):
                        tree.allocate_block(h)
            except MemoryError:
                for h in pair:
                    tree.free(h)
                on_step(step)
                continue
            avail = (len(toks) - pair[0].shared_match_len) // bs
            if avail > 0:
                k = int(rng.integers(1, avail + 1))
                tree.commit_prefix(pair[0], bs * k)
                tree.commit_prefix(pair[1], bs * (k if rng.random() < 0.5 else int(rng.integers(k, avail + 1))))
            live.extend(pair)
        else:
            h = live[int(rng.integers(len(live)))]
            m, _ = tree.match_prefix(h.tokens[: int(rng.integers(1, len(h.tokens) + 1))])
            if m is not None:
                live.append(m)
        on_step(step)
    for h in live:
        tree.free(h)
    on_step(steps)
