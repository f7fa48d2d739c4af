"""KV-head sharding of the block pool across the GPUs of one node.

Every block `[L, 2, H, bs, D]` splits by KV head: with `world` ranks, rank r
holds heads [r*H/world, (r+1)*H/world) of every block, as one contiguous
span per block (`[N, L, 2, H/world, bs, D]`).  All ranks use the same global
block ids, so a copy-on-write pair (src, dst) is the same pair on every rank
and each rank copies only its own slice: no KV byte crosses a GPU.

Rank `src` (0) owns the allocator and the tree; after planning a batch it
broadcasts the int32 pair list (8 B per pair) over the process group — NCCL
over NVLink on GPUs — and every rank runs akv_copy_blocks on its slice.
Batches of varying size travel as one fixed-size buffer (`pack_batch`): an
int64 pair count followed by room for `max_pairs` pairs; the copy reads the
count on the device (akv_copy_blocks_counted), so receiving ranks never wait
on the host for it.

Partitioned planning instead splits the block ids: rank r owns the range
[r*B, (r+1)*B) (`partition`) and plans, with an allocator over B blocks, the
agents whose blocks lie there; the ranks all-gather their pair lists
(`gather_pairs`, ids made global by adding each rank's base) and every rank
copies all of them on its slice.  Each rank's allocator work then stays the
same as ranks are added, where a single planner's grows with them.
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import _native as N
from . import kernels as K


def heads_per_rank(num_kv_heads: int, world: int) -> int:
    if world < 1 or num_kv_heads % world:
        raise ValueError(f"{world} ranks do not divide {num_kv_heads} KV heads")
    return num_kv_heads // world


def slice_shape(total_blocks: int, num_layers: int, num_kv_heads: int, block_size: int, head_dim: int,
                world: int) -> tuple:
    return (total_blocks, num_layers, 2, heads_per_rank(num_kv_heads, world), block_size, head_dim)


def head_slice(pool: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rank `rank`'s heads of a full pool tensor [N, L, 2, H, bs, D] (a view)."""
    h = heads_per_rank(pool.shape[3], world)
    return pool[:, :, :, rank * h : (rank + 1) * h]


def partition(total_blocks: int, rank: int, world: int) -> tuple:
    """(base, count): the block ids rank `rank` plans for under partitioned
    planning, [base, base + count)."""
    if world < 1 or not 0 <= rank < world or total_blocks % world:
        raise ValueError(f"{total_blocks} blocks do not split into {world} equal ranges (rank {rank})")
    count = total_blocks // world
    return rank * count, count


class ShardedCopier:
    """Applies rank 0's copy batches to this rank's head slice."""

    def __init__(self, pool_slice: torch.Tensor, group=None, src: int = 0) -> None:
        import torch.distributed as dist

        self.pool = pool_slice
        self.group = group
        self.src = src
        # the status record of this copier's copies alone (the claimed copy
        # variant keeps its work counter there); read with check()
        self.status = torch.zeros(N.STATUS_BYTES // 4, dtype=torch.int32, device=pool_slice.device)
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    def share_pairs(self, pairs: Optional[torch.Tensor], n_pairs: int, out: Optional[torch.Tensor] = None):
        """Rank src passes its (n, 2) int32 pair list, the others receive it."""
        import torch.distributed as dist

        if self.rank == self.src:
            buf = pairs.reshape(-1, 2)
        else:
            buf = out if out is not None else torch.empty((n_pairs, 2), dtype=torch.int32, device=self.pool.device)
        if self.world > 1:
            dist.broadcast(buf, src=self.src, group=self.group)
        return buf

    def gather_pairs(self, pairs: torch.Tensor, base: int, out: torch.Tensor,
                     send: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Partitioned planning: every rank passes its (n, 2) int32 pairs in
        its own ids (0 .. count-1 of its range, the same n on every rank) and
        its range's `base`; `out` ((world * n, 2) int32) receives every
        rank's pairs in rank order with global ids.  `send` ((n, 2) int32) is
        the staging buffer for this rank's shifted pairs (allocated when
        None).  On GPUs: one elementwise add and one NCCL all-gather on the
        current stream, both capturable in a CUDA graph."""
        import torch.distributed as dist

        pairs = pairs.reshape(-1, 2)
        if out.dtype != torch.int32 or pairs.dtype != torch.int32:
            raise ValueError("gather_pairs: pairs and out must be int32")
        if out.shape != (self.world * pairs.shape[0], 2):
            raise ValueError(f"gather_pairs: out is {tuple(out.shape)}, expected "
                             f"({self.world * pairs.shape[0]}, 2)")
        send = torch.add(pairs, base, out=send if send is not None else torch.empty_like(pairs))
        if self.world > 1:
            dist.all_gather_into_tensor(out, send, group=self.group)
        else:
            out.copy_(send)
        return out

    def copy(self, pairs: torch.Tensor, **kw) -> None:
        """Copy (n, 2) pairs on this rank's slice.  Without an explicit
        variant and status the copy uses this copier's own status record and
        the variant kernels.claimed_variant picks."""
        if kw.get("status") is None and self.pool.device.type == "cuda":
            kw["status"] = self.status
            if kw.get("variant", N.VARIANT_AUTO) == N.VARIANT_AUTO:
                kw["variant"] = K.claimed_variant(self.pool)
        K.copy_blocks(self.pool, pairs, **kw)

    def check(self) -> None:
        """Raises for an error the copier's copies recorded (synchronises)."""
        K.raise_for_status(self.status)

    # ── variable-size batches: [int64 count | max_pairs x (src, dst)] ────────
    @staticmethod
    def batch_words(max_pairs: int) -> int:
        return 2 + 2 * max_pairs

    def batch_buffer(self, max_pairs: int) -> torch.Tensor:
        return torch.zeros(self.batch_words(max_pairs), dtype=torch.int32, device=self.pool.device)

    @staticmethod
    def pack_batch(pairs, buf: torch.Tensor) -> torch.Tensor:
        """Write (n, 2) host pairs and their count into `buf` (rank src)."""
        p = np.asarray(pairs, np.int32).reshape(-1, 2)
        cap = (buf.numel() - 2) // 2
        if len(p) > cap:
            raise ValueError(f"pack_batch: {len(p)} pairs exceed the buffer's {cap}")
        host = np.zeros(2 + 2 * len(p), np.int32)
        host[:2].view(np.int64)[0] = len(p)
        host[2:] = p.reshape(-1)
        buf[: host.size].copy_(torch.from_numpy(host))
        return buf

    def share_batch(self, buf: torch.Tensor) -> torch.Tensor:
        """One broadcast of the whole batch buffer from rank src."""
        import torch.distributed as dist

        if self.world > 1:
            dist.broadcast(buf, src=self.src, group=self.group)
        return buf

    @staticmethod
    def batch_count(buf: torch.Tensor) -> torch.Tensor:
        """The int64 count as a one-element tensor view of `buf`."""
        return buf[:2].view(torch.int64)

    @staticmethod
    def batch_pairs(buf: torch.Tensor) -> torch.Tensor:
        return buf[2:].view(-1, 2)

    def copy_batch(self, buf: torch.Tensor, **kw) -> None:
        """Copy the batch's pairs on this rank's slice; the count is read on
        the device."""
        K.copy_blocks_counted(self.pool, self.batch_pairs(buf), self.batch_count(buf), **kw)
