"""EpochReclaimer — host side of the two-epoch safe reclamation.

The reference's EpochReclaimer (agentkv/core/reclamation.py:55-190) keeps the
epoch counter, the set of epochs that hold an open read section, and a FIFO
of retired block ids that may only return to the free list once no reader
that could still see them remains.  Here the retired-id FIFO and the epoch /
op counters are part of the allocator's state (on the device, and in the
allocator's host mirror), and this class keeps what only the host knows — the
reader set:

* ``enter_read_section`` takes the current epoch (the reader's token) and
  adds it to the set — a set, as in the reference, so two readers of one
  epoch share one entry.  The epoch comes from the allocator's host mirror
  when it is current, so this costs no read-back;
* ``leave_read_section`` discards the token and releases every pending id
  older than the oldest remaining reader (all of them when no reader is
  left), ``_try_retire`` in the reference (reclamation.py:147-173);
* ``maybe_advance`` bumps the epoch (unless a reader holds the current epoch)
  followed by the same release.

Both apply to the mirror (and reach the device with its op log) when the
mirror is current, else they are one launch each.

Each allocator batch carries a summary of the reader set (AkvTick) so the
device applies the reference's rules for ids that retire while readers are
open.
"""

from __future__ import annotations

from typing import TYPE_CHECKING, Set

from . import _native as N

if TYPE_CHECKING:  # pragma: no cover
    from .allocator import SlabAllocator

_INT64_MAX = (1 << 63) - 1


class EpochReclaimer:
    def __init__(self, allocator: "SlabAllocator") -> None:
        self._alloc = allocator
        self._active_reader_epochs: Set[int] = set()
        self._tick_cache = None  # (epoch_interval, AkvTick) for the current reader set

    def tick(self, epoch_interval: int) -> N.AkvTick:
        """The reader-set summary every allocator call carries (kept until
        the set changes: callers do not modify it)."""
        c = self._tick_cache
        if c is not None and c[0] == epoch_interval:
            return c[1]
        r = self._active_reader_epochs
        t = N.AkvTick(min(r), max(r), epoch_interval, 1) if r else N.AkvTick(0, 0, epoch_interval, 0)
        self._tick_cache = (epoch_interval, t)
        return t

    def enter_read_section(self) -> int:
        a = self._alloc
        with a._lock:
            token = a.epoch()  # the host's copy when it is current: no wait
            self._active_reader_epochs.add(token)
            self._tick_cache = None
            return token

    def leave_read_section(self, token: int) -> None:
        a = self._alloc
        with a._lock:
            self._active_reader_epochs.discard(token)
            self._tick_cache = None
            safe = min(self._active_reader_epochs) if self._active_reader_epochs else _INT64_MAX
            if a._live:
                a._mirror.release(safe)
                a._maybe_flush()
            else:
                N.check(N.lib.akv_limbo_release(a._state, safe, a._stream()))

    def maybe_advance(self) -> None:
        a = self._alloc
        with a._lock:
            tick = self.tick(a._cfg.epoch_interval)
            if a._live:
                a._mirror.advance(tick)
                a._maybe_flush()
            else:
                N.check(N.lib.akv_epoch_advance(a._state, tick, a._stream()))

    def stats(self) -> dict:
        c = self._alloc.counters()
        return {
            "epoch": int(c[N.CTL_EPOCH]),
            "pending_blocks": int(c[N.CTL_LIMBO_TAIL] - c[N.CTL_LIMBO_REL]),
            "active_readers": len(self._active_reader_epochs),
            "epoch_advances": int(c[N.CTL_ADVANCES]),
            "blocks_freed": int(c[N.CTL_RELEASED]),
        }

    def pending_count(self) -> int:
        c = self._alloc.counters()
        return int(c[N.CTL_LIMBO_TAIL] - c[N.CTL_LIMBO_REL])
