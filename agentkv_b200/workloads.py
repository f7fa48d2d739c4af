"""Seeded synthetic inputs for the five pool workloads of this path.

No public dataset is involved: token ids and pool contents are synthetic,
drawn from seeded generators (``random.Random`` or numpy PCG64, both
reproducible across machines) with the shapes, sizes and distributions of
the workloads they stand for:

* quickstart — a 64-block fp16 pool (L2 H4 D64 bs16): root with tokens 0..31,
  three forked children that each diverge (CoW of the shared block) and eight
  prefix queries;
* Tree-of-Thought fan-out — Llama-3-8B KV geometry (L32 H8 D128 bs16 bf16,
  2 MiB blocks), 60,000 blocks, a 4096-token root forked 8 ways for 3 levels,
  each child copy-on-writes its last inherited block and appends 64 tokens;
* copy / zero sweep — disjoint random (src, dst) pairs from 60,000 blocks,
  batch sizes 1, 8, 64, 512, 4096;
* match_prefix stress — 200 shared prefixes (1024–4096 tokens), sequences
  whose prefix index is Zipf(1.1)-distributed, total lengths 512–8192, vocab
  128,256; 4096-query batches, half extending cached sequences;
* ReAct multi-agent — Llama-3-70B KV geometry (L80 H8 D128 bs16 bf16), a
  16,384-token shared prefix, 32 agents, steps mixing forks, CoW tail copies,
  frees and epoch advances.
"""

from __future__ import annotations

import random
from dataclasses import dataclass
from typing import List, Tuple

import numpy as np

VOCAB = 128_256

# (total_blocks, block_size, num_layers, num_kv_heads, head_dim, dtype)
QUICKSTART_GEOMETRY = (64, 16, 2, 4, 64, "float16")
LLAMA3_8B_GEOMETRY = (60_000, 16, 32, 8, 128, "bfloat16")
LLAMA3_70B_GEOMETRY = (40_000, 16, 80, 8, 128, "bfloat16")

COPY_SWEEP_BATCHES = (1, 8, 64, 512, 4096)


# ── quickstart ───────────────────────────────────────────────────────────────
def quickstart_queries(seed: int = 1, n: int = 8) -> List[List[int]]:
    """Eight queries of length 16–48 sharing 0–32 leading tokens with 0..31."""
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        length = rng.randint(16, 48)
        share = min(rng.randint(0, 32), length)
        q = list(range(share)) + [rng.randrange(VOCAB) for _ in range(length - share)]
        out.append(q)
    return out


# ── Tree-of-Thought fan-out ──────────────────────────────────────────────────
@dataclass(frozen=True)
class ToTSpec:
    root_tokens: int = 4096
    fanout: int = 8
    levels: int = 3
    append_tokens: int = 64
    seed: int = 2

    @property
    def appended_blocks(self) -> int:
        return self.append_tokens // 16

    def children_per_level(self) -> List[int]:
        return [self.fanout ** (lvl + 1) for lvl in range(self.levels)]


def tot_root_tokens(spec: ToTSpec = ToTSpec()) -> List[int]:
    rng = random.Random(spec.seed)
    return [rng.randrange(VOCAB) for _ in range(spec.root_tokens)]


def tot_append_tokens(spec: ToTSpec, level: int, child: int) -> List[int]:
    rng = random.Random(spec.seed * 1_000_003 + level * 10_007 + child)
    return [rng.randrange(VOCAB) for _ in range(spec.append_tokens)]


# ── copy / zero sweep ────────────────────────────────────────────────────────
def copy_sweep_pairs(n: int, total_blocks: int = 60_000, seed: int = 3, rotation: int = 0) -> np.ndarray:
    """n disjoint (src, dst) pairs: the first 2n entries of a seeded
    permutation of the block ids.  `rotation` picks another seed so repeated
    batches touch other blocks."""
    rng = np.random.Generator(np.random.PCG64(seed + 7919 * rotation))
    perm = rng.permutation(total_blocks)[: 2 * n].astype(np.int32)
    return np.stack([perm[:n], perm[n:]], axis=1).copy()


# ── match_prefix stress ──────────────────────────────────────────────────────
@dataclass(frozen=True)
class MatchSpec:
    n_prefixes: int = 200
    prefix_min: int = 1024
    prefix_max: int = 4096
    n_sequences: int = 20_000
    total_min: int = 512
    total_max: int = 8192
    zipf_s: float = 1.1
    n_queries: int = 4096
    seed: int = 4


def _zipf_cdf(n: int, s: float) -> np.ndarray:
    w = 1.0 / np.arange(1, n + 1, dtype=np.float64) ** s
    c = np.cumsum(w)
    return c / c[-1]


def match_prefixes(spec: MatchSpec) -> List[np.ndarray]:
    rng = np.random.Generator(np.random.PCG64(spec.seed))
    lens = rng.integers(spec.prefix_min, spec.prefix_max + 1, size=spec.n_prefixes)
    return [rng.integers(0, VOCAB, size=int(L), dtype=np.int32) for L in lens]


def match_sequences(spec: MatchSpec, prefixes: List[np.ndarray] | None = None,
                    stream: int = 0, count: int | None = None) -> List[np.ndarray]:
    """Sequences = a Zipf-chosen shared prefix (cut to the total length if
    shorter) followed by random tokens up to a total length in
    [total_min, total_max].  `stream` selects an independent generator (0 is
    the inserted corpus, others are fresh query streams)."""
    if prefixes is None:
        prefixes = match_prefixes(spec)
    count = spec.n_sequences if count is None else count
    rng = np.random.Generator(np.random.PCG64(spec.seed * 7_777 + 1 + stream))
    cdf = _zipf_cdf(spec.n_prefixes, spec.zipf_s)
    out = []
    for _ in range(count):
        k = int(np.searchsorted(cdf, rng.random(), side="right"))
        k = min(k, spec.n_prefixes - 1)
        total = int(rng.integers(spec.total_min, spec.total_max + 1))
        p = prefixes[k][:total]
        suffix = rng.integers(0, VOCAB, size=total - len(p), dtype=np.int32)
        out.append(np.concatenate([p, suffix]).astype(np.int32))
    return out


def match_queries(spec: MatchSpec, corpus: List[np.ndarray], prefixes: List[np.ndarray] | None = None,
                  batch: int = 0, n: int | None = None) -> List[np.ndarray]:
    """A query batch: half extend a cached corpus sequence with 16–512 random
    tokens, half are fresh sequences from the generator."""
    n = spec.n_queries if n is None else n
    rng = np.random.Generator(np.random.PCG64(spec.seed * 31_337 + batch))
    fresh = match_sequences(spec, prefixes, stream=1000 + batch, count=n - n // 2)
    out = []
    for i in range(n // 2):
        base = corpus[int(rng.integers(0, len(corpus)))]
        ext = rng.integers(0, VOCAB, size=int(rng.integers(16, 513)), dtype=np.int32)
        out.append(np.concatenate([base, ext]).astype(np.int32))
    out.extend(fresh)
    order = rng.permutation(len(out))
    return [out[i] for i in order]


# ── ReAct multi-agent ────────────────────────────────────────────────────────
@dataclass(frozen=True)
class ReActSpec:
    """A 16,384-token shared prefix committed to the tree, 32 agents forked
    from it, and `steps` rounds in which every agent slot, in slot order,
    takes one action drawn with weights (fork 2, cow 4, free 2, advance 1,
    append 3):

    * fork    — agent s branches: the agent in another slot t (drawn) is freed
                and replaced by fork(agent s), sharing s's residual blocks;
    * cow     — ensure_mutable_block(agent s, -1): the tail block is copied if
                it is shared (after a fork), else nothing moves; an agent with
                no residual block allocates one instead;
    * free    — agent s is freed and restarts as a fork of the prefix root;
    * advance — maybe_advance_epoch();
    * append  — allocate_block(agent s) (16 more tokens).
    """

    prefix_tokens: int = 16_384
    agents: int = 32
    steps: int = 1000
    seed: int = 5
    block_size: int = 16


REACT_FORK, REACT_COW, REACT_FREE, REACT_ADVANCE, REACT_APPEND = range(5)
REACT_WEIGHTS = (2, 4, 2, 1, 3)


def react_prefix(spec: ReActSpec) -> List[int]:
    rng = random.Random(spec.seed)
    return [rng.randrange(VOCAB) for _ in range(spec.prefix_tokens)]


def react_trace(spec: ReActSpec) -> List[List[Tuple[int, int, int]]]:
    """Per step, one (action, slot, target slot) per agent in slot order; the
    target is used by fork only (never the acting slot)."""
    rng = random.Random(spec.seed * 1_000_003 + 1)
    kinds = list(range(5))
    out = []
    for _ in range(spec.steps):
        step = []
        for s in range(spec.agents):
            k = rng.choices(kinds, weights=REACT_WEIGHTS)[0]
            t = rng.randrange(spec.agents - 1)
            step.append((k, s, t if t < s else t + 1))
        out.append(step)
    return out


def react_setup(api, spec: ReActSpec):
    """Commit the shared prefix and fork the agents (each with one private
    block).  `api` offers the pool's calls (create_root, allocate_block,
    allocate_blocks, commit_prefix, fork) plus residual_len(handle)."""
    root = api.create_root(react_prefix(spec))
    api.allocate_blocks(root, spec.prefix_tokens // spec.block_size)
    api.commit_prefix(root, spec.prefix_tokens)
    agents = []
    for _ in range(spec.agents):
        a = api.fork(root)
        api.allocate_block(a)
        agents.append(a)
    return root, agents


def react_step(api, root, agents: list, actions) -> None:
    """Apply one step's actions, in order, through `api` (see ReActSpec)."""
    for kind, s, t in actions:
        if kind == REACT_FORK:
            api.free(agents[t])
            agents[t] = api.fork(agents[s])
        elif kind == REACT_COW:
            if api.residual_len(agents[s]):
                api.ensure_mutable_block(agents[s], -1)
            else:
                api.allocate_block(agents[s])
        elif kind == REACT_FREE:
            api.free(agents[s])
            agents[s] = api.fork(root)
        elif kind == REACT_ADVANCE:
            api.maybe_advance_epoch()
        else:
            api.allocate_block(agents[s])


# ── HuggingFace cache decode script ──────────────────────────────────────────
@dataclass(frozen=True)
class HFSpec:
    """A small HF-cache session: a 10-token prompt prefilled on a root agent,
    8 tokens committed to the shared tree, 3 forks decoding one token per
    step (three tokens at step 2), the root decoding too."""

    total_blocks: int = 64
    block_size: int = 4
    num_layers: int = 2
    num_kv_heads: int = 2
    head_dim: int = 16
    dtype: str = "float16"
    prompt: int = 10
    commit: int = 8
    forks: int = 3
    steps: int = 6
    seed: int = 6


def hf_script(spec: HFSpec) -> List[Tuple[str, int, int]]:
    """Events (kind, agent, n): prefill agent 0 with n tokens, commit n tokens
    of agent 0, fork agent 0 (the new agent gets the next index), update
    agent with n new tokens."""
    ev = [("prefill", 0, spec.prompt), ("commit", 0, spec.commit)]
    ev += [("fork", 0, 0)] * spec.forks
    for step in range(spec.steps):
        for a in range(1, spec.forks + 1):
            ev.append(("update", a, 3 if step == 2 else 1))
        if step % 2 == 0:
            ev.append(("update", 0, 1))
    return ev


def hf_states(spec: HFSpec, event: int, layer: int, n: int) -> Tuple[np.ndarray, np.ndarray]:
    """Seeded K and V states [1, heads, n, head_dim] of one update."""
    rng = np.random.Generator(np.random.PCG64(spec.seed * 1_000_003 + event * 101 + layer))
    shape = (1, spec.num_kv_heads, n, spec.head_dim)
    return (rng.standard_normal(shape).astype(spec.dtype), rng.standard_normal(shape).astype(spec.dtype))


def hf_run(spec: HFSpec, pool, cache_cls, to_tensor, on_output) -> list:
    """Play hf_script through `pool` (the AgentKVPool API) and `cache_cls`
    (the AgentKVCache API); on_output(event, layer, out_k, out_v) sees every
    update's result.  Returns the agents' caches."""
    caches = []
    for e, (kind, a, n) in enumerate(hf_script(spec)):
        if kind == "prefill":
            h = pool.create_root(list(range(100, 100 + n)))
            c = cache_cls(pool, h)
            c._seen_tokens = 0
            caches.append(c)
            kind = "update"
        if kind == "commit":
            pool.commit_prefix(caches[a].handle, n)
        elif kind == "fork":
            caches.append(caches[a].fork())
        elif kind == "update":
            for layer in range(spec.num_layers):
                k, v = hf_states(spec, e, layer, n)
                ok, ov = caches[a].update(to_tensor(k), to_tensor(v), layer)
                on_output(e, layer, ok, ov)
    return caches
