"""HostMirror — the allocator's per-call operations answered on the host.

A thin wrapper of the C ABI's akv_mirror_* functions (akv_mirror.cu): a host
copy of the allocator state that applies the reference's per-call operations
(SlabAllocator.alloc / inc_ref / dec_ref, ensure_mutable_block, the
reclaimer's release and advance: agentkv/core/slab_allocator.py:194-278,
416-437; reclamation.py:88-173) at once, in order, and logs them.  The
SlabAllocator replays the log on the device (akv_alloc_replay) before the
device state is next used, and reloads the mirror from the device after
device-side batches.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional, Tuple

import numpy as np

from . import _native as N


class MirrorRefused(Exception):
    """A per-call operation the allocator state refuses (nothing changed):
    `code` is the AKV_ERR_* the device would have recorded."""

    def __init__(self, status: N.AkvStatus) -> None:
        super().__init__(N.ERROR_NAMES.get(status.code, status.code))
        self.code = int(status.code)
        self.index = int(status.index)
        self.id = int(status.id)
        self.observed = int(status.observed)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class HostMirror:
    def __init__(self, total_blocks: int) -> None:
        self.n = int(total_blocks)
        h = N.lib.akv_mirror_create(self.n)
        if not h:
            raise N.NativeError(N.AKV_ERR_INVALID_ARG, N.last_error())
        self._h = C.c_void_p(h)
        self._err = N.AkvStatus()
        self._err_ptr = C.addressof(self._err)
        self._out = np.zeros(1024, np.int32)
        self._out_ptr = _ptr(self._out)
        self._n_ret = np.zeros(1, np.int32)
        self._ctl = np.zeros(N.CTL_WORDS, np.int64)

    def __del__(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            N.lib.akv_mirror_destroy(h)
            self._h = None

    def _room(self, n: int) -> np.ndarray:
        if n > len(self._out):
            self._out = np.zeros(max(n, 2 * len(self._out)), np.int32)
            self._out_ptr = _ptr(self._out)
        return self._out

    def _done(self, rc: int) -> None:
        if rc == N.AKV_OK:
            return
        if self._err.code == rc:
            raise MirrorRefused(self._err)
        N.check(rc)

    # ── state ────────────────────────────────────────────────────────────────
    def load(self, ref: np.ndarray, ring: np.ndarray, limbo_ids: np.ndarray, limbo_epochs: np.ndarray,
             ctl: np.ndarray) -> None:
        """Take the state from host copies of the device arrays; clears the log."""
        arrs = [np.ascontiguousarray(ref, np.int32), np.ascontiguousarray(ring, np.int32),
                np.ascontiguousarray(limbo_ids, np.int32), np.ascontiguousarray(limbo_epochs, np.int64),
                np.ascontiguousarray(ctl, np.int64)]
        N.check(N.lib.akv_mirror_load(self._h, *[_ptr(a) for a in arrs]))

    def ctl(self) -> np.ndarray:
        N.check(N.lib.akv_mirror_read(self._h, _ptr(self._ctl), None, None, None, None))
        return self._ctl.copy()

    def ctl_word(self, i: int) -> int:
        N.check(N.lib.akv_mirror_read(self._h, _ptr(self._ctl), None, None, None, None))
        return int(self._ctl[i])

    def refs(self) -> np.ndarray:
        out = np.zeros(self.n, np.int32)
        N.check(N.lib.akv_mirror_read(self._h, None, _ptr(out), None, None, None))
        return out

    def arrays(self) -> Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
        """(ctl, refcounts, free ring, limbo ids, limbo epochs), in the device
        arrays' layout."""
        ctl = np.zeros(N.CTL_WORDS, np.int64)
        ref, ring, lid = (np.zeros(self.n, np.int32) for _ in range(3))
        lep = np.zeros(self.n, np.int64)
        N.check(N.lib.akv_mirror_read(self._h, _ptr(ctl), _ptr(ref), _ptr(ring), _ptr(lid), _ptr(lep)))
        return ctl, ref, ring, lid, lep

    def free_list(self) -> np.ndarray:
        ctl, _, ring, _, _ = self.arrays()
        left, size = int(ctl[N.CTL_FREE_LEFT]), int(ctl[N.CTL_FREE_SIZE])
        return ring[(left + np.arange(size)) % self.n]

    def limbo(self) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
        """(deferred ids, pending ids, pending epochs)."""
        ctl, _, _, lid, lep = self.arrays()
        h, r, t = (int(ctl[i]) for i in (N.CTL_LIMBO_HEAD, N.CTL_LIMBO_REL, N.CTL_LIMBO_TAIL))
        d = (h + np.arange(r - h)) % self.n
        p = (r + np.arange(t - r)) % self.n
        return lid[d], lid[p], lep[p]

    def ref(self, block: int) -> int:
        return int(N.lib.akv_mirror_ref(self._h, block))

    # ── operations ───────────────────────────────────────────────────────────
    def alloc(self, n: int, tick: N.AkvTick) -> np.ndarray:
        out = self._room(n)
        self._done(N.lib.akv_mirror_alloc(self._h, n, tick, _ptr(out), self._err_ptr))
        return out[:n].copy()

    def alloc_one(self, tick: N.AkvTick) -> int:
        out = self._out
        self._done(N.lib.akv_mirror_alloc(self._h, 1, tick, self._out_ptr, self._err_ptr))
        return int(out[0])

    def incref(self, ids: np.ndarray, tick: N.AkvTick) -> None:
        ids = np.ascontiguousarray(ids, np.int32)
        self._done(N.lib.akv_mirror_incref(self._h, _ptr(ids), len(ids), tick, self._err_ptr))

    def decref(self, ids: np.ndarray, tick: N.AkvTick, retired: bool = False) -> Tuple[int, Optional[np.ndarray]]:
        """(ids retired, the retired ids in order when asked for)."""
        ids = np.ascontiguousarray(ids, np.int32)
        out = self._room(len(ids)) if retired else None
        self._done(N.lib.akv_mirror_decref(self._h, _ptr(ids), len(ids), tick,
                                           _ptr(out) if retired else None, _ptr(self._n_ret), self._err_ptr))
        k = int(self._n_ret[0])
        return k, (out[:k].copy() if retired else None)

    def cow(self, block: int, tick: N.AkvTick) -> int:
        out = self._room(1)
        self._done(N.lib.akv_mirror_cow(self._h, block, tick, _ptr(out), self._err_ptr))
        return int(out[0])

    def release(self, safe_before_epoch: int) -> None:
        N.check(N.lib.akv_mirror_release(self._h, safe_before_epoch))

    def advance(self, tick: N.AkvTick) -> None:
        N.check(N.lib.akv_mirror_advance(self._h, tick))

    # ── op log ───────────────────────────────────────────────────────────────
    def log_words(self) -> int:
        return int(N.lib.akv_mirror_log_words(self._h))

    def take_log(self, dst: np.ndarray) -> int:
        """Move the log into `dst` (int32, room for log_words()); returns its length."""
        k = self.log_words()
        N.check(N.lib.akv_mirror_take_log(self._h, _ptr(dst) if k else None, len(dst)))
        return k
