"""AgentKVPool — the public facade (agentkv/pool.py:29-271), unchanged API.

Thin delegation to DualRadixTree + SlabAllocator, exactly as in the reference,
plus the batched entry points the device path makes cheap
(``allocate_blocks``, ``fork_many``, ``ensure_mutable_batch``, ``free_many``,
``match_prefix_batch``, ``match_prefix_many``).
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

from .allocator import SlabAllocator
from .config import PoolConfig
from .radix_tree import DualRadixTree, NodeHandle


class AgentKVPool:
    """GPU-resident copy-on-write KV-cache block pool for agentic workloads."""

    def __init__(
        self,
        capacity_gb: float = 40.0,
        block_size: int = 16,
        num_layers: int = 32,
        num_kv_heads: int = 8,
        head_dim: int = 128,
        dtype: str = "float16",
        device: str = "cuda",
        *,
        config: Optional[PoolConfig] = None,
    ) -> None:
        if config is not None:
            self._cfg = config
        else:
            self._cfg = PoolConfig.from_capacity_gb(
                capacity_gb=capacity_gb,
                block_size=block_size,
                num_layers=num_layers,
                num_kv_heads=num_kv_heads,
                head_dim=head_dim,
                dtype=dtype,
                device=device,
            )
        self._allocator = SlabAllocator(self._cfg)
        self._tree = DualRadixTree(self._allocator, self._cfg)

    # ── reference API ─────────────────────────────────────────────────────────
    def create_root(self, prompt_tokens: List[int]) -> NodeHandle:
        return self._tree.create_root(prompt_tokens)

    def fork(self, parent: NodeHandle) -> NodeHandle:
        return self._tree.fork(parent)

    def allocate_block(self, handle: NodeHandle) -> None:
        self._tree.allocate_block(handle)

    def ensure_mutable_block(self, handle: NodeHandle, block_idx: int) -> None:
        self._tree.ensure_mutable_block(handle, block_idx)

    def append_tokens(self, handle: NodeHandle, tokens: List[int]) -> None:
        self._tree.append_tokens(handle, tokens)

    def commit_prefix(self, handle: NodeHandle, length: int) -> None:
        self._tree.commit_prefix(handle, length)

    def free(self, handle: NodeHandle) -> None:
        self._tree.free(handle)

    def get_block_ids(self, handle: NodeHandle) -> List[int]:
        return self._tree.get_block_ids(handle)

    def maybe_advance_epoch(self) -> None:
        self._allocator.maybe_advance_epoch()

    def stats(self) -> dict:
        return {**self._allocator.stats(), **self._tree.stats()}

    @property
    def config(self) -> PoolConfig:
        return self._cfg

    @property
    def block_size(self) -> int:
        return self._cfg.block_size

    @property
    def free_blocks(self) -> int:
        return self._allocator.free_count

    @property
    def allocated_blocks(self) -> int:
        return self._allocator.allocated_count

    # ── batched extensions ────────────────────────────────────────────────────
    def allocate_blocks(self, handle: NodeHandle, n: int) -> None:
        self._tree.allocate_blocks(handle, n)

    def fork_many(self, parent: NodeHandle, k: int) -> List[NodeHandle]:
        return self._tree.fork_many(parent, k)

    def ensure_mutable_batch(self, requests: Sequence[Tuple[NodeHandle, int]]) -> List[bool]:
        return self._tree.ensure_mutable_batch(requests)

    def free_many(self, handles: Sequence[NodeHandle]) -> None:
        self._tree.free_many(handles)

    def match_prefix_batch(self, queries: Sequence, *, with_compared: bool = False):
        return self._tree.match_prefix_batch(queries, with_compared=with_compared)

    def match_prefix_many(self, queries: Sequence) -> List[Tuple[Optional[NodeHandle], int]]:
        """The tree's match_prefix on every query (handles included), one lookup launch."""
        return self._tree.match_prefix_many(queries)

    def __repr__(self) -> str:
        s = self.stats()
        return (
            f"AgentKVPool("
            f"total={s['total_blocks']}, "
            f"free={s['free_blocks']}, "
            f"allocated={s['allocated_blocks']}, "
            f"agents={s['active_handles']}, "
            f"pool={self._cfg.total_gb:.2f} GiB"
            f")"
        )
