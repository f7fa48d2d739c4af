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
    def __init__(self, pool: AgentKVPool, handle: NodeHandle, *, append_only: bool = False) -> None:
        """append_only=True keeps each layer's assembled K/V between updates
        and appends the new tokens' rows to it instead of assembling the
        whole sequence from the pool again: O(new tokens) per update.  The
        bytes are the same as long as the agent's blocks change only through
        this cache's updates (the pool still receives every row, so forks,
        commits and to_legacy_cache see them); a caller that writes into the
        agent's blocks by other means must leave it off (the default).  The
        returned K/V are then views of the held buffers (stride along the
        tokens is the buffer's capacity), which hold a layer's K and V
        besides the pool's copy, as HF's own dynamic cache does."""
        super().__init__()
        self.pool = pool
        self.handle = handle
        self.append_only = append_only
        self._mirror: Dict[int, list] = {}  # layer -> [K buffer, V buffer, tokens held]
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
        if self.append_only:
            out_k, out_v = self._append(layer_idx, key_states, value_states, table)
        else:
            out_k, out_v = K.kv_gather(kv, table, layer_idx, self._next_seen_tokens, status=st)
        if layer_idx == pool.config.num_layers - 1:
            self._seen_tokens = self._next_seen_tokens
        return out_k, out_v

    def _append(self, layer: int, key_states: torch.Tensor, value_states: torch.Tensor,
                table: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """The layer's K/V for append_only: the held buffers plus this update's
        rows when they hold exactly the tokens before it, else assembled from
        the pool (first update, or after a fork made a new cache)."""
        kv = self.pool._allocator._kv_data
        seen, nxt = self._seen_tokens, self._next_seen_tokens
        m = self._mirror.get(layer)
        if m is None or m[2] != seen or m[0].shape[2] < nxt:
            k, v = K.kv_gather(kv, table, layer, nxt, status=self.pool._allocator._status)
            cap = max(nxt + 256, 2 * nxt)  # room for the next updates' rows
            kb = torch.empty((1, k.shape[1], cap, k.shape[3]), dtype=k.dtype, device=k.device)
            vb = torch.empty_like(kb)
            kb[:, :, :nxt].copy_(k)
            vb[:, :, :nxt].copy_(v)
            m = self._mirror[layer] = [kb, vb, nxt]
        else:
            kb, vb = m[0], m[1]
            kb[:, :, seen:nxt].copy_(key_states)
            vb[:, :, seen:nxt].copy_(value_states)
            m[2] = nxt
        return m[0][:, :, :nxt], m[1][:, :, :nxt]

    def fork(self) -> "AgentKVCache":
        return AgentKVCache(self.pool, self.pool.fork(self.handle), append_only=self.append_only)

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
