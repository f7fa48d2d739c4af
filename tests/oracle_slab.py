"""The SlabAllocator calls DualRadixTree makes, answered by the oracle's
allocator (the C restatement of the reference's SlabAllocator and
EpochReclaimer) over a CPU pool tensor, so that CPU tests can run the
package's host-side tree logic (agentkv_b200/radix_tree.py) against the
reference's recorded traces.  Test infrastructure only: the package's
allocator is the device one.

Errors are raised at the call, as the reference's single calls raise them:
MemoryError when the pool is exhausted, ValueError otherwise.
"""

from __future__ import annotations

import numpy as np
import torch

from agentkv_b200.allocator import BlockHandle
from oracle import oracle as O


def _raise(e: "O.OracleError"):
    if e.code == O.ORC_ERR_EXHAUSTED:
        raise MemoryError("KV block pool exhausted") from None
    raise ValueError(f"oracle allocator error {e.code}") from None


class OracleSlab:
    def __init__(self, kv: torch.Tensor, epoch_interval: int) -> None:
        self._kv_data = kv  # [N, L, 2, H, bs, D] on the CPU
        self.n = kv.shape[0]
        self.o = O.OracleAllocator(self.n, epoch_interval)
        self.device = torch.device("cpu")

    def _bytes(self) -> np.ndarray:
        return self._kv_data.view(torch.uint8).reshape(self.n, -1).numpy()

    def _valid(self, bh: BlockHandle) -> int:
        b = bh.block_id
        if not 0 <= b < self.n:
            raise ValueError(f"invalid block {b}")
        return b

    def alloc(self) -> BlockHandle:
        try:
            return BlockHandle(self.o.alloc())
        except O.OracleError as e:
            _raise(e)

    def alloc_batch(self, n: int) -> torch.Tensor:
        try:
            return torch.from_numpy(self.o.alloc_batch(n).copy())
        except O.OracleError as e:
            _raise(e)

    def alloc_many(self, n: int) -> list:
        return self.alloc_batch(n).tolist() if n > 0 else []

    def inc_ref_batch(self, ids) -> None:
        try:
            self.o.inc_ref_batch(np.asarray(ids, np.int32))
        except O.OracleError as e:
            _raise(e)

    def dec_ref(self, bh: BlockHandle) -> bool:
        try:
            return self.o.dec_ref(self._valid(bh))
        except O.OracleError as e:
            _raise(e)

    def dec_ref_batch(self, ids) -> None:
        try:
            self.o.dec_ref_batch(np.asarray(ids, np.int32))
        except O.OracleError as e:
            _raise(e)

    def cow_batch(self, ids):
        try:
            out, copied = self.o.cow_batch(np.asarray(ids, np.int32), self._bytes(), self._bytes().shape[1])
        except O.OracleError as e:
            _raise(e)
        return torch.from_numpy(out.copy()), torch.from_numpy(copied.copy())

    def cow_many(self, blocks):
        out, copied = self.cow_batch(blocks)
        return out.numpy(), copied.numpy()

    def cow_one(self, block_id: int) -> int:
        out, _ = self.cow_batch([block_id])
        return int(out[0])

    def ref_count(self, bh: BlockHandle) -> int:
        return self.o.ref_count(self._valid(bh))

    def check(self) -> None:
        pass  # every call above has raised already

    def enter_read_section(self) -> int:
        return self.o.enter_read_section()

    def leave_read_section(self, token: int) -> None:
        self.o.leave_read_section(token)

    def maybe_advance_epoch(self) -> None:
        self.o.maybe_advance_epoch()

    @property
    def free_count(self) -> int:
        return self.o.free_count

    @property
    def allocated_count(self) -> int:
        st = self.o.state()
        return self.n - len(st["free_list"]) - len(st["pending"]) - len(st["deferred"])

    def zero_block(self, bh: BlockHandle) -> None:
        b = self._valid(bh)
        if self.o.ref_count(b) != 1:
            raise ValueError(f"zero_block: block {b} must be exclusively owned")
        O.zero_blocks(self._bytes(), self._bytes().shape[1], np.array([b], np.int32))
