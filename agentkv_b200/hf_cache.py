"""AgentKVCache — a HuggingFace transformers cache whose K/V live in the
AgentKV pool (drop-in for agentkv/hf_cache.py).

Same constructor, attributes and calls as the reference's AgentKVCache
(agentkv/hf_cache.py:29-216): update() allocates blocks on layer 0, makes the
blocks it writes exclusively owned (copy-on-write after a fork), writes the
new tokens' rows and returns the layer's whole K and V.  The data movement is
two launches per layer instead of a Python loop over tokens plus an indexing
gather and a permute: akv_kv_scatter writes every new token's rows,
akv_kv_gather assembles the contiguous [1, heads, tokens, head_dim] outputs
straight from the block tiles.  The copy-on-write checks happen first, in the
reference's order, as one batch: each block a new token starts (and the
first new token's block) is checked before any row lands, which gives the
reference's bytes because a copied block never holds rows of this update.
"""

from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

import numpy as np
import torch

from . import kernels as K
from .pool import AgentKVPool
from .radix_tree import NodeHandle

try:
    from transformers.cache_utils import DynamicCache
except ImportError:  # transformers absent: the class still works on its own
    class DynamicCache:  # type: ignore[no-redef]
        def __init__(self) -> None:
            self.key_cache = []
            self.value_cache = []


class AgentKVCache(DynamicCache):
    def __init__(self, pool: AgentKVPool, handle: NodeHandle) -> None:
        super().__init__()
        self.pool = pool
        self.handle = handle
        self._seen_tokens = len(self.handle.tokens)
        self._next_seen_tokens = self._seen_tokens
        self.key_cache = []
        self.value_cache = []
        self._table: Optional[list] = None
        self._table_dev: Optional[torch.Tensor] = None
        self._table_version = 0  # bumped whenever _table_dev is replaced
        self._slots_key: Optional[tuple] = None  # (first new token, count, table version) of _slots_dev
        self._slots_dev: Optional[torch.Tensor] = None

    def get_seq_length(self, layer_idx: Optional[int] = 0) -> int:
        return self._seen_tokens

    def _device_table(self, ids: list) -> torch.Tensor:
        if self._table != ids:
            self._table = list(ids)
            self._table_dev = torch.tensor(ids, dtype=torch.int32).to(self.pool._allocator._kv_data.device)
            self._table_version += 1
        return self._table_dev

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[Dict[str, Any]] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        if key_states.shape[0] != 1:
            raise ValueError("AgentKVCache requires batch_size=1")
        pool, h = self.pool, self.handle
        bs = pool.block_size
        n_new = key_states.shape[2]
        if layer_idx == 0:
            self._next_seen_tokens = self._seen_tokens + n_new
            required = (self._next_seen_tokens + bs - 1) // bs
            current = len(pool.get_block_ids(h))
            if required > current:
                pool.allocate_blocks(h, required - current)
            if len(h.tokens) < self._next_seen_tokens:
                pool.append_tokens(h, [0] * (self._next_seen_tokens - len(h.tokens)))
        tok = self._seen_tokens + np.arange(n_new, dtype=np.int64)
        blk = tok // bs
        shared = h.shared_match_len // bs
        if n_new and blk[0] < shared:
            raise RuntimeError("Cannot overwrite shared prefix blocks!")
        if layer_idx == 0 and n_new:
            starts = np.flatnonzero((np.arange(n_new) == 0) | (tok % bs == 0))
            pool.ensure_mutable_batch([(h, int(blk[i] - shared)) for i in starts])
        ids = pool.get_block_ids(h)
        kv = pool._allocator._kv_data
        st = pool._allocator._status
        table = self._device_table(ids)
        if n_new:
            # the new tokens' slots are the same for every layer of a step:
            # computed and uploaded once
            key = (self._seen_tokens, n_new, self._table_version)
            if self._slots_key != key:
                slots = np.asarray(ids, np.int64)[blk] * bs + tok % bs
                self._slots_dev = torch.from_numpy(slots.astype(np.int32)).to(kv.device)
                self._slots_key = key
            K.kv_scatter(kv, self._slots_dev, layer_idx, key_states, value_states, status=st)
        out_k, out_v = K.kv_gather(kv, table, layer_idx, self._next_seen_tokens, status=st)
        if layer_idx == pool.config.num_layers - 1:
            self._seen_tokens = self._next_seen_tokens
        return out_k, out_v

    def fork(self) -> "AgentKVCache":
        return AgentKVCache(self.pool, self.pool.fork(self.handle))

    def to_legacy_cache(self) -> Tuple[Tuple[torch.Tensor, torch.Tensor], ...]:
        ids = self.pool.get_block_ids(self.handle)
        kv = self.pool._allocator._kv_data
        out = []
        for layer in range(self.pool.config.num_layers):
            if not ids:
                cfg = self.pool.config
                e = torch.empty(1, cfg.num_kv_heads, 0, cfg.head_dim, device=kv.device, dtype=kv.dtype)
                out.append((e, e.clone()))
            else:
                out.append(K.kv_gather(kv, self._device_table(ids), layer, self._seen_tokens,
                                       status=self.pool._allocator._status))
        return tuple(out)
