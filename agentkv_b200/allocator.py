"""SlabAllocator — KV block pool with a device-resident free list and refcounts.

Same public surface as the reference's SlabAllocator
(agentkv/core/slab_allocator.py:98-447): ``alloc``, ``inc_ref``, ``dec_ref``,
``copy_block``, ``zero_block``, ``get_block_tensor``, ``ref_count``, read
sections, ``maybe_advance_epoch``, ``free_count``, ``allocated_count``,
``stats`` — with the same exceptions and messages.  The state those methods
mutate lives on the GPU:

* ``_kv_data``       the pool tensor [N, L, 2, H, bs, D] (unchanged layout);
* ``_ref_counts``    int32 [N] refcounts;
* ``_free_ring``     the free deque as a ring (pop right, recycled ids left);
* ``_limbo_*``       retired ids waiting for the reclaimer (deferred + pending);
* ``_ctl``           cursors and counters (op count, epoch, stats).

The batched operations are launches of the C ABI (akv_alloc_batch /
akv_incref_batch / akv_decref_batch / akv_cow_batch / akv_limbo_release /
akv_epoch_advance) that reproduce the reference's sequential semantics,
including the order in which ids leave and re-enter the free list; they
return device tensors without waiting, and device-detected errors surface at
``check()``.

The per-call methods (``alloc``, ``inc_ref``, ``dec_ref``, ``cow_one``,
``ref_count``, the read sections, and ``*_batch`` calls with host ids) are
answered by a host mirror of the same state (``HostMirror``, akv_mirror.cu),
which applies each call at once with the same rules and raises the
reference's exceptions at the call, without a device round trip.  The
mirror logs the calls; before anything on the device reads or changes the
allocator state, the log is replayed there in one launch (akv_alloc_replay,
which checks every id the host handed out).  After device-side batches (the
fan-out planners, DeviceAgents, batches of device ids) the mirror is reloaded
from the device at the next per-call method, with one wait.

The pool itself must live on a CUDA device, or on ``meta`` for the
metadata-only pools of the vLLM / SGLang adapters (their free list and
refcounts then live on the current CUDA device).  A CPU pool is rejected:
this package has no CPU implementation of the path.
"""

from __future__ import annotations

import threading
from typing import List, Optional, Tuple

import numpy as np
import torch

from . import _native as N
from .config import PoolConfig, torch_dtype
from .kernels import copy_blocks as _copy_blocks
from .kernels import stream_handle
from .mirror import HostMirror, MirrorRefused
from .reclamation import EpochReclaimer

INVALID_BLOCK: int = -1

_INT64_MAX = (1 << 63) - 1
_LOG_FLUSH_WORDS = 1 << 15  # the op log is replayed on the device once it holds this many words
_MIRROR_MAX_BATCH = 4096  # larger batches of host ids run as device batches (one warp replays the log)


class BlockHandle:
    """Opaque handle to a KV block (agentkv/core/slab_allocator.py:71-95)."""

    __slots__ = ("block_id",)

    def __init__(self, block_id: int) -> None:
        self.block_id = block_id

    def is_valid(self) -> bool:
        return self.block_id != INVALID_BLOCK

    def __repr__(self) -> str:
        return f"BlockHandle(id={self.block_id})"

    def __eq__(self, other: object) -> bool:
        if isinstance(other, BlockHandle):
            return self.block_id == other.block_id
        return NotImplemented

    def __hash__(self) -> int:
        return hash(self.block_id)


def _metadata_device(device: str) -> torch.device:
    dev = torch.device(device)
    if dev.type == "cuda":
        if not torch.cuda.is_available():
            raise RuntimeError("agentkv_b200: a CUDA pool was requested but no CUDA device is visible")
        return torch.device("cuda", dev.index if dev.index is not None else torch.cuda.current_device())
    if dev.type == "meta":
        if not torch.cuda.is_available():
            raise RuntimeError(
                "agentkv_b200: a metadata-only (meta) pool keeps its free list and refcounts "
                "on a CUDA device, and none is visible"
            )
        return torch.device("cuda", torch.cuda.current_device())
    raise ValueError(
        f"agentkv_b200 pools live on a CUDA device (or 'meta' for metadata-only pools); "
        f"got device={device!r}"
    )


class _IdStage:
    """Uploads of host id lists through reused buffers: a pinned host buffer
    and a device buffer of the same size, used in two halves.  A half is
    written again only after the event recorded when it was left has
    completed (its copies are done); the device half is reused in stream
    order, after the kernels that read it (allocator calls share a stream).
    Replaces a fresh pinned tensor and device tensor per call."""

    def __init__(self, device: torch.device, cap: int = 1 << 15) -> None:
        self.device = device
        self._alloc_buffers(cap)

    def _alloc_buffers(self, cap: int) -> None:
        self.cap = cap
        self.h = torch.empty(cap, dtype=torch.int32, pin_memory=True)
        self.h_np = self.h.numpy()
        self.d = torch.empty(cap, dtype=torch.int32, device=self.device)
        self.half = 0
        self.pos = 0
        self.left = [None, None]  # event recorded when each half was last left

    def put(self, ids: np.ndarray) -> torch.Tensor:
        n = len(ids)
        if n == 0:
            return self.d[:0]
        half = self.cap // 2
        if n > half:
            torch.cuda.current_stream(self.device).synchronize()
            self._alloc_buffers(max(4 * n, 2 * self.cap))
            half = self.cap // 2
        if self.pos + n > half:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self.left[self.half] = ev
            self.half ^= 1
            self.pos = 0
            if self.left[self.half] is not None:
                self.left[self.half].synchronize()
        base = self.half * half + self.pos
        self.h_np[base : base + n] = ids
        dst = self.d[base : base + n]
        dst.copy_(self.h[base : base + n], non_blocking=True)
        self.pos += n
        return dst


class SlabAllocator:
    """Fixed-capacity KV block pool; see the module docstring."""

    def __init__(self, config: PoolConfig) -> None:
        if config.epoch_interval <= 0:
            raise ValueError(f"epoch_interval must be > 0, got {config.epoch_interval}")
        self._cfg = config
        self._lock = threading.RLock()
        self._dev = _metadata_device(config.device)
        n = config.total_blocks
        self._kv_data: torch.Tensor = torch.zeros(
            n, config.num_layers, 2, config.num_kv_heads, config.block_size, config.head_dim,
            dtype=torch_dtype(config.dtype), device=config.device,
        )
        dev = self._dev
        i32, i64 = torch.int32, torch.int64
        self._ref_counts = torch.zeros(n, dtype=i32, device=dev)
        self._free_ring = torch.empty(n, dtype=i32, device=dev)
        self._limbo_ids = torch.empty(n, dtype=i32, device=dev)
        self._limbo_epochs = torch.empty(n, dtype=i64, device=dev)
        # ctl and the io words share one allocation, so one copy brings back
        # the status, the small outputs and the counters (op count, epoch,
        # last batch's retirements) after a single call
        self._ctlio = torch.zeros(N.CTL_WORDS + 32, dtype=i64, device=dev)
        self._ctl = self._ctlio[: N.CTL_WORDS]
        self._scratch_count = torch.zeros(n, dtype=i32, device=dev)
        self._scratch_last = torch.zeros(n, dtype=i32, device=dev)
        self._scratch_aux = torch.zeros(N.AUX_WORDS, dtype=i32, device=dev)
        # io: [0:8] AkvStatus, [8:40] small outputs, [40:64] small inputs
        self._io = self._ctlio[N.CTL_WORDS :].view(i32)
        self._status = self._io[0:8]
        self._h_in = torch.zeros(24, dtype=i32, pin_memory=True)
        self._h_in_np = self._h_in.numpy()
        self._h_ctlio = torch.zeros(N.CTL_WORDS + 32, dtype=i64, pin_memory=True)
        self._h_ctlio_np = self._h_ctlio.numpy()
        self._h_io_np = self._h_ctlio_np[N.CTL_WORDS :].view(np.int32)
        self._ids = _IdStage(dev)
        self._ctlio_ptr = self._ctlio.data_ptr()
        self._io_ptr = self._io.data_ptr()
        self._h_ctlio_ptr = self._h_ctlio.data_ptr()
        self._h_in_ptr = self._h_in.data_ptr()
        self._h_ref = torch.zeros(2, dtype=i32, pin_memory=True)
        self._h_ref_np = self._h_ref.numpy()
        # The host mirror: current while _live (the device state is the
        # mirror's minus its unreplayed log); _refused marks a batch the
        # mirror refused, whose error waits in the device status for check().
        self._mirror = HostMirror(n)
        self._live = True
        self._refused = False
        self._calls = 0
        self._log_np = np.zeros(_LOG_FLUSH_WORDS + 4096, np.int32)
        self._log_stage = _IdStage(dev, cap=1 << 17)
        self._h_state: Optional[torch.Tensor] = None  # pinned read-back of the device state
        self._state = N.AkvAllocState(
            self._ref_counts.data_ptr(), self._free_ring.data_ptr(), self._limbo_ids.data_ptr(),
            self._limbo_epochs.data_ptr(), self._ctl.data_ptr(), self._scratch_count.data_ptr(),
            self._scratch_last.data_ptr(), self._scratch_aux.data_ptr(), n, 0,
        )
        self._reclaimer = EpochReclaimer(self)
        with torch.cuda.device(dev):
            # load every kernel and set its attributes on this device now, so
            # that no first launch happens later inside a graph capture
            N.check(N.lib.akv_prepare())
            N.check(N.lib.akv_alloc_init(self._state, self._stream()))

    # ── plumbing ──────────────────────────────────────────────────────────────
    def _stream(self) -> int:
        return stream_handle(self._dev)

    @property
    def device(self) -> torch.device:
        """Device that holds the free list and refcounts."""
        return self._dev

    @property
    def config(self) -> PoolConfig:
        return self._cfg

    def _tick(self) -> N.AkvTick:
        return self._reclaimer.tick(self._cfg.epoch_interval)

    def _sync_io(self, n_out: int = 16) -> np.ndarray:
        """Copy the control words, the status and the first outputs to the
        host in one copy and wait; returns the io words (status, outputs)."""
        hi = N.CTL_WORDS + (8 + n_out + 1) // 2
        off = 8 * N.CTL_OPS
        N.check(N.lib.akv_copy_wait(self._h_ctlio_ptr + off, self._ctlio_ptr + off, 8 * hi - off, 1, 1,
                                    self._stream()))
        return self._h_io_np[: 8 + n_out].copy()

    # ── host mirror plumbing ──────────────────────────────────────────────────
    def _flush(self) -> None:
        """Replay the mirror's op log on the device (one upload, one launch,
        no wait)."""
        k = self._mirror.log_words()
        if k == 0:
            return
        if k > len(self._log_np):
            self._log_np = np.zeros(2 * k, np.int32)
        self._mirror.take_log(self._log_np)
        d = self._log_stage.put(self._log_np[:k])
        N.check(N.lib.akv_alloc_replay(self._state, d.data_ptr(), k, self._status.data_ptr(), self._stream()))

    def _maybe_flush(self) -> None:
        """Replay the log once it has grown large (looked at every 64 calls:
        a call adds at most _MIRROR_MAX_BATCH + 8 words)."""
        self._calls += 1
        if self._calls & 63 == 0 and self._mirror.log_words() >= _LOG_FLUSH_WORDS:
            self._flush()

    def _device_op(self) -> None:
        """Before a device-side operation on the allocator state: the device
        catches up with the mirror's log, and the mirror is stale until it is
        next needed (then reloaded from the device)."""
        self._flush()
        self._live = False

    def _host(self) -> HostMirror:
        """The mirror, current: reloaded from the device (one wait) after
        device-side batches."""
        if not self._live:
            n = self._cfg.total_blocks
            if self._h_state is None:
                self._h_state = torch.empty(3 * n + 2 * (n + N.CTL_WORDS), dtype=torch.int32, pin_memory=True)
            h = self._h_state
            parts = (self._ref_counts, self._free_ring, self._limbo_ids)
            for i, t in enumerate(parts):
                h[i * n : (i + 1) * n].copy_(t, non_blocking=True)
            h64 = h[3 * n :].view(torch.int64)
            h64[:n].copy_(self._limbo_epochs, non_blocking=True)
            h64[n:].copy_(self._ctl, non_blocking=True)
            torch.cuda.current_stream(self._dev).synchronize()
            a = h.numpy()
            a64 = h64.numpy()
            self._mirror.load(a[:n], a[n : 2 * n], a[2 * n : 3 * n], a64[:n], a64[n:])
            self._live = True
        return self._mirror

    def _refuse(self, e: MirrorRefused, op: str, batch: bool) -> Exception:
        """A call the mirror refused.  A per-call method raises it at once;
        a batch posts it to the device status instead (after the log, so the
        calls before it still replay), where the device's own later batches
        see it and do nothing, and check() raises it."""
        exc = self._exception(e.code, e.id, e.observed, op, e.index)
        if batch:
            self._flush()
            self._h_in_np[:8] = 0
            self._h_in_np[:4] = (e.code, e.index, e.id, e.observed)
            N.check(N.lib.akv_copy_wait(self._status.data_ptr(), self._h_in_ptr, N.STATUS_BYTES, 0, 0,
                                        self._stream()))
            torch.cuda.current_stream(self._dev).synchronize()  # the staging words are reused
            self._refused = True
        return exc

    def _pending(self) -> None:
        """A per-call method after a refused batch raises its error, as the
        next waiting call would have."""
        if self._refused:
            self.check()

    def _host_ids(self, ids) -> Optional[np.ndarray]:
        """The ids as a host int32 array, or None when they are device ids."""
        if isinstance(ids, torch.Tensor):
            if ids.device.type != "cpu":
                return None
            return ids.numpy().astype(np.int32, copy=False).reshape(-1)
        return np.asarray(ids, np.int32).reshape(-1)

    def epoch(self) -> int:
        """The reclaimer's current epoch (from the mirror when it is current,
        else read from the device)."""
        with self._lock:
            if self._live:
                return self._mirror.ctl_word(N.CTL_EPOCH)
            return int(self.ctl()[N.CTL_EPOCH])

    def _stage_ids(self, ids) -> int:
        """Put up to 24 ids into the device input slots; returns the pointer."""
        k = len(ids)
        self._h_in_np[:k] = ids
        dst = self._io_ptr + 40 * 4
        N.check(N.lib.akv_copy_wait(dst, self._h_in_ptr, 4 * k, 0, 0, self._stream()))
        return dst

    def _raise_status(self, io: np.ndarray, op: str = "") -> None:
        code = int(io[0])
        if code == 0:
            return
        index, bid, observed = int(io[1]), int(io[2]), int(io[3])
        self._status.zero_()
        raise self._exception(code, bid, observed, op, index)

    def _exception(self, code: int, bid: int, observed: int, op: str, index: int = 0) -> Exception:
        n = self._cfg.total_blocks
        if code == N.AKV_ERR_EXHAUSTED:
            return MemoryError(
                f"AgentKV pool exhausted: all {n} blocks are in use. "
                "Increase PoolConfig.total_blocks or free some agents."
            )
        if code == N.AKV_ERR_NOT_ALLOCATED:
            return ValueError(
                f"inc_ref on block {bid} with ref_count={observed} "
                "(not allocated — double-inc or use-after-free?)"
            )
        if code == N.AKV_ERR_DOUBLE_FREE:
            return ValueError(
                f"dec_ref on block {bid} with ref_count={observed} (already free or double-free?)"
            )
        if code == N.AKV_ERR_NOT_EXCLUSIVE:
            if op == "zero_block":
                return ValueError(
                    f"zero_block: block {bid} must be exclusively owned (ref_count=1, got {observed})"
                )
            return ValueError(
                f"copy_block: dst block {bid} must have ref_count=1 (got {observed}). "
                "Only exclusively-owned blocks may be written."
            )
        if code == N.AKV_ERR_OUT_OF_RANGE:
            return ValueError(f"block_id {bid} out of range [0, {n})")
        return RuntimeError(
            f"agentkv_b200 device error: {N.ERROR_NAMES.get(code, code)} "
            f"(position {index}, id {bid}, observed {observed})"
        )

    def _validate_handle(self, handle: BlockHandle) -> None:
        if not isinstance(handle, BlockHandle):
            raise TypeError(f"Expected BlockHandle, got {type(handle)}")
        if not handle.is_valid():
            raise ValueError("BlockHandle is invalid (block_id == INVALID_BLOCK)")
        if handle.block_id < 0 or handle.block_id >= self._cfg.total_blocks:
            raise ValueError(f"block_id {handle.block_id} out of range [0, {self._cfg.total_blocks})")

    # ── single operations (reference semantics, answered by the host mirror) ──
    def alloc(self) -> BlockHandle:
        """Claim a free block (ref_count 1); MemoryError when exhausted."""
        with self._lock:
            self._pending()
            try:
                bid = self._host().alloc_one(self._tick())
            except MirrorRefused as e:
                raise self._refuse(e, "alloc", False) from None
            self._maybe_flush()
            return BlockHandle(bid)

    def alloc_many(self, n: int) -> List[int]:
        """n alloc() calls: the ids, in the order the calls would return
        them; MemoryError (nothing taken) when fewer than n are free."""
        with self._lock:
            if n <= 0:
                return []
            self._pending()
            try:
                ids = self._host().alloc(n, self._tick())
            except MirrorRefused as e:
                raise self._refuse(e, "alloc", False) from None
            self._maybe_flush()
            return ids.tolist()

    def cow_one(self, block_id: int) -> int:
        """ensure_mutable on one residual block: the block the slot owns
        afterwards (a fresh copy when the block was shared; the data copy is
        enqueued on the device)."""
        with self._lock:
            self._pending()
            try:
                nb = self._host().cow(int(block_id), self._tick())
            except MirrorRefused as e:
                raise self._refuse(e, "ensure_mutable_block", False) from None
            if nb != block_id and self._kv_data.device.type != "meta":
                self._copy_pair(int(block_id), nb)
            self._maybe_flush()
            return nb

    def inc_ref(self, handle: BlockHandle) -> None:
        self._validate_handle(handle)
        with self._lock:
            self._pending()
            try:
                self._host().incref(np.asarray([handle.block_id], np.int32), self._tick())
            except MirrorRefused as e:
                raise self._refuse(e, "inc_ref", False) from None
            self._maybe_flush()

    def dec_ref(self, handle: BlockHandle) -> bool:
        """Decrement; True when the count reached zero (block retired)."""
        self._validate_handle(handle)
        with self._lock:
            self._pending()
            try:
                k, _ = self._host().decref(np.asarray([handle.block_id], np.int32), self._tick())
            except MirrorRefused as e:
                raise self._refuse(e, "dec_ref", False) from None
            self._maybe_flush()
            return k > 0

    def _copy_pair(self, src: int, dst: int) -> None:
        """One block copy on the device (exclusivity checked by the caller on
        the mirror), without waiting."""
        pair = self._ids.put(np.asarray([src, dst], np.int32))  # a staging slot no later call reuses early
        N.check(N.lib.akv_copy_blocks(self._kv_data.data_ptr(), self._cfg.bytes_per_block,
                                      self._cfg.total_blocks, pair.data_ptr(), 1, None, self._status.data_ptr(),
                                      self._stream()))

    def get_block_tensor(self, handle: BlockHandle) -> torch.Tensor:
        self._validate_handle(handle)
        return self._kv_data[handle.block_id]

    def copy_block(self, src: BlockHandle, dst: BlockHandle) -> None:
        """Copy src's KV data into dst, which must be exclusively owned."""
        self._validate_handle(src)
        self._validate_handle(dst)
        with self._lock:
            if self._kv_data.device.type == "meta" or self._live:
                rc = self._read_ref(dst.block_id)
                if rc != 1:
                    raise self._exception(N.AKV_ERR_NOT_EXCLUSIVE, dst.block_id, rc, "copy_block")
                if self._kv_data.device.type != "meta":
                    self._copy_pair(src.block_id, dst.block_id)
                return
            ptr = self._stage_ids([src.block_id, dst.block_id])
            N.check(N.lib.akv_copy_blocks(self._kv_data.data_ptr(), self._cfg.bytes_per_block,
                                          self._cfg.total_blocks, ptr, 1, self._ref_counts.data_ptr(),
                                          self._status.data_ptr(), self._stream()))
            self._raise_status(self._sync_io(0), "copy_block")

    def zero_block(self, handle: BlockHandle) -> None:
        """Write +0.0 over an exclusively owned block."""
        self._validate_handle(handle)
        with self._lock:
            if self._kv_data.device.type == "meta" or self._live:
                rc = self._read_ref(handle.block_id)
                if rc != 1:
                    raise self._exception(N.AKV_ERR_NOT_EXCLUSIVE, handle.block_id, rc, "zero_block")
                if self._kv_data.device.type != "meta":  # checked on the mirror: no device check, no wait
                    ids = self._ids.put(np.asarray([handle.block_id], np.int32))
                    N.check(N.lib.akv_zero_blocks(self._kv_data.data_ptr(), self._cfg.bytes_per_block,
                                                  self._cfg.total_blocks, ids.data_ptr(), 1, None,
                                                  self._status.data_ptr(), self._stream()))
                return
            ptr = self._stage_ids([handle.block_id])
            N.check(N.lib.akv_zero_blocks(self._kv_data.data_ptr(), self._cfg.bytes_per_block,
                                          self._cfg.total_blocks, ptr, 1, self._ref_counts.data_ptr(),
                                          self._status.data_ptr(), self._stream()))
            self._raise_status(self._sync_io(0), "zero_block")

    # ── epoch / reclamation ───────────────────────────────────────────────────
    def enter_read_section(self) -> int:
        return self._reclaimer.enter_read_section()

    def leave_read_section(self, token: int) -> None:
        self._reclaimer.leave_read_section(token)

    def maybe_advance_epoch(self) -> None:
        self._reclaimer.maybe_advance()

    # ── introspection ─────────────────────────────────────────────────────────
    def ref_count(self, handle: BlockHandle) -> int:
        self._validate_handle(handle)
        with self._lock:
            return self._read_ref(handle.block_id)

    def _read_ref(self, block_id: int) -> int:
        """One block's refcount: from the mirror when it is current, else
        one copy and one wait."""
        if self._live:
            return self._mirror.ref(block_id)
        N.check(N.lib.akv_copy_wait(self._h_ref.data_ptr(), self._ref_counts.data_ptr() + 4 * block_id, 4, 1, 1,
                                    self._stream()))
        return int(self._h_ref_np[0])

    def ctl(self) -> np.ndarray:
        """Host copy of the device's control words, after the mirror's log
        (waits)."""
        with self._lock:
            self._flush()
            return self._ctl.cpu().numpy()

    def ref_counts(self) -> np.ndarray:
        """The device's refcounts after the mirror's log (waits)."""
        with self._lock:
            self._flush()
            return self._ref_counts.cpu().numpy()

    def flush(self) -> None:
        """Bring the device arrays up to date with the per-call operations
        answered so far (one launch, no wait)."""
        with self._lock:
            self._flush()

    def counters(self) -> np.ndarray:
        """The control words: the mirror's when it is current (no wait),
        else the device's."""
        with self._lock:
            return self._mirror.ctl() if self._live else self.ctl()

    @property
    def free_count(self) -> int:
        return int(self.counters()[N.CTL_FREE_SIZE])

    @property
    def allocated_count(self) -> int:
        c = self.counters()
        return int(self._cfg.total_blocks - c[N.CTL_FREE_SIZE] - (c[N.CTL_LIMBO_TAIL] - c[N.CTL_LIMBO_HEAD]))

    def stats(self) -> dict:
        c = self.counters()
        n = self._cfg.total_blocks
        return {
            "total_blocks": n,
            "free_blocks": int(c[N.CTL_FREE_SIZE]),
            "allocated_blocks": int(n - c[N.CTL_FREE_SIZE] - (c[N.CTL_LIMBO_TAIL] - c[N.CTL_LIMBO_HEAD])),
            "peak_allocated": int(c[N.CTL_PEAK]),
            "total_allocs": int(c[N.CTL_ALLOCS]),
            "total_frees": int(c[N.CTL_FREES]),
            "pending_reclamation": int(c[N.CTL_LIMBO_TAIL] - c[N.CTL_LIMBO_REL]),
            "epoch": int(c[N.CTL_EPOCH]),
            "pool_size_gb": self._cfg.total_gb,
        }

    def free_list(self) -> np.ndarray:
        """The device's free list left to right (waits)."""
        with self._lock:
            self._flush()
            c = self._ctl.cpu().numpy()
            ring = self._free_ring.cpu().numpy()
        n = self._cfg.total_blocks
        idx = (int(c[N.CTL_FREE_LEFT]) + np.arange(int(c[N.CTL_FREE_SIZE]))) % n
        return ring[idx]

    def limbo(self) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
        """(deferred ids, pending ids, pending epochs) in FIFO order, from the
        device (waits)."""
        with self._lock:
            self._flush()
            c = self._ctl.cpu().numpy()
            ids = self._limbo_ids.cpu().numpy()
            eps = self._limbo_epochs.cpu().numpy()
        n = self._cfg.total_blocks
        h, r, t = (int(c[k]) for k in (N.CTL_LIMBO_HEAD, N.CTL_LIMBO_REL, N.CTL_LIMBO_TAIL))
        d_idx = np.arange(h, r) % n
        p_idx = np.arange(r, t) % n
        return ids[d_idx], ids[p_idx], eps[p_idx]

    # ── batched operations (one launch each, no waiting) ──────────────────────
    def _device_ids(self, ids) -> torch.Tensor:
        if isinstance(ids, torch.Tensor) and ids.device == self._dev and ids.dtype == torch.int32:
            return ids.contiguous()
        if isinstance(ids, torch.Tensor):
            ids = ids.cpu().numpy()
        return self._ids.put(np.asarray(ids, np.int32).reshape(-1))

    def alloc_batch(self, n: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """n alloc() calls; returns the ids (device int32).  Errors surface at
        check()."""
        if out is None:
            out = torch.empty(max(n, 0), dtype=torch.int32, device=self._dev)
        with self._lock:
            if self._live and not self._refused and n <= _MIRROR_MAX_BATCH:
                try:
                    ids = self._mirror.alloc(n, self._tick())
                except MirrorRefused as e:
                    self._refuse(e, "alloc", True)
                    return out
                if n:
                    out[:n].copy_(self._ids.put(ids), non_blocking=True)
                self._maybe_flush()
                return out
            self._device_op()
            N.check(N.lib.akv_alloc_batch(self._state, n, out.data_ptr() if n else None, self._tick(),
                                          self._status.data_ptr(), self._stream()))
        return out

    def inc_ref_batch(self, ids) -> None:
        """n inc_ref() calls (ids may repeat), all or nothing; errors surface
        at check()."""
        host = self._host_ids(ids)
        with self._lock:
            if host is not None and self._live and len(host) <= _MIRROR_MAX_BATCH:
                if self._refused:
                    return  # the device would skip it too: an error is pending
                try:
                    self._mirror.incref(host, self._tick())
                except MirrorRefused as e:
                    self._refuse(e, "inc_ref", True)
                self._maybe_flush()
                return
            t = self._device_ids(ids)
            self._device_op()
            N.check(N.lib.akv_incref_batch(self._state, t.data_ptr(), t.numel(), self._tick(),
                                           self._status.data_ptr(), self._stream()))

    def dec_ref_batch(self, ids, retired_out: Optional[torch.Tensor] = None) -> None:
        """n dec_ref() calls; retired ids (in retirement order) go to
        `retired_out` when given; their count is ctl[LAST_RETIRED].  Errors
        surface at check()."""
        host = self._host_ids(ids)
        with self._lock:
            if host is not None and self._live and len(host) <= _MIRROR_MAX_BATCH:
                if self._refused:
                    return
                try:
                    k, ret = self._mirror.decref(host, self._tick(), retired=retired_out is not None)
                except MirrorRefused as e:
                    self._refuse(e, "dec_ref", True)
                    return
                if retired_out is not None and k:
                    retired_out[:k].copy_(self._ids.put(ret), non_blocking=True)
                self._maybe_flush()
                return
            t = self._device_ids(ids)
            self._device_op()
            N.check(N.lib.akv_decref_batch(self._state, t.data_ptr(), t.numel(), self._tick(),
                                           retired_out.data_ptr() if retired_out is not None else None,
                                           self._status.data_ptr(), self._stream()))

    def cow_batch(self, blocks, out_blocks: Optional[torch.Tensor] = None,
                  out_copied: Optional[torch.Tensor] = None,
                  pairs: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """ensure_mutable over a batch of residual blocks (distinct slots), in
        order: copy-on-write wherever the refcount is > 1.  Returns
        (blocks now owned, 1 where a copy happened)."""
        t = self._device_ids(blocks)
        n = t.numel()
        if out_blocks is None:
            out_blocks = torch.empty(n, dtype=torch.int32, device=self._dev)
        if out_copied is None:
            out_copied = torch.empty(n, dtype=torch.int32, device=self._dev)
        if pairs is None:
            pairs = torch.empty(2 * max(n, 1), dtype=torch.int32, device=self._dev)
        meta = self._kv_data.device.type == "meta"
        with self._lock:
            self._device_op()
            N.check(N.lib.akv_cow_batch(
                self._state, None if meta else self._kv_data.data_ptr(),
                0 if meta else self._cfg.bytes_per_block, t.data_ptr(), n, out_blocks.data_ptr(),
                out_copied.data_ptr(), pairs.data_ptr(), self._tick(), self._status.data_ptr(),
                self._stream()))
        return out_blocks, out_copied

    def cow_many(self, blocks) -> Tuple[np.ndarray, np.ndarray]:
        """ensure_mutable over a batch of residual blocks (distinct slots), in
        order, answered on the host mirror: (blocks now owned, 1 where a copy
        happened) as host arrays, the block copies enqueued in one launch.
        MemoryError, with nothing changed, when the copies would run the pool
        dry."""
        ids = np.asarray(blocks, np.int32).reshape(-1)
        with self._lock:
            self._pending()
            m = self._host()
            # all or nothing: count the copies first (a request copies while
            # its block is still shared after the earlier requests' copies)
            copies, taken = 0, {}
            for x in ids.tolist():
                r = m.ref(x)
                if r == -(1 << 31):
                    raise self._exception(N.AKV_ERR_OUT_OF_RANGE, x, 0, "ensure_mutable_block")
                if r - taken.get(x, 0) > 1:
                    copies += 1
                    taken[x] = taken.get(x, 0) + 1
            c = m.ctl()
            avail = c[N.CTL_FREE_SIZE] + c[N.CTL_LIMBO_REL] - c[N.CTL_LIMBO_HEAD]
            if copies and (c[N.CTL_FREE_SIZE] < 1 or avail < copies):
                raise self._exception(N.AKV_ERR_EXHAUSTED, -1, int(c[N.CTL_FREE_SIZE]), "ensure_mutable_block")
            tick = self._tick()
            out = np.empty(len(ids), np.int32)
            for i, x in enumerate(ids.tolist()):
                out[i] = m.cow(x, tick)
            copied = (out != ids).astype(np.int32)
            if copies and self._kv_data.device.type != "meta":
                pairs = np.stack([ids[copied == 1], out[copied == 1]], axis=1).reshape(-1)
                d = self._ids.put(pairs)
                N.check(N.lib.akv_copy_blocks(self._kv_data.data_ptr(), self._cfg.bytes_per_block,
                                              self._cfg.total_blocks, d.data_ptr(), copies, None,
                                              self._status.data_ptr(), self._stream()))
            self._maybe_flush()
            return out, copied

    def fanout_level(self, parent_tables: torch.Tensor, parent_off: torch.Tensor, parent_lens,
                     fanout: int, append: int, *, pool: Optional[torch.Tensor] = None,
                     copy: bool = True) -> dict:
        """One fork level on device-resident block tables (akv_fanout_plan):
        every parent is forked `fanout` times; each child copy-on-writes its
        last inherited block and appends `append` fresh blocks.  Block ids,
        refcounts and the free list end exactly as after the reference's
        per-child fork / ensure_mutable_block(-1) / allocate_block calls.

        parent_tables / parent_off are device int32 / int64 tensors (tables
        concatenated, offsets[P + 1]); parent_lens the P table lengths on the
        host (all >= 1).  The copies go to `pool` (default: this allocator's
        pool; a head slice of it on a sharded pool), or are skipped with
        copy=False (then `pairs` in the result is what to copy).  Returns the
        device tensors child_tables, child_off, pairs and the launch count."""
        lens = np.asarray(parent_lens, np.int64)
        if (lens < 1).any():
            raise ValueError("fanout_level: every parent needs at least one residual block")
        P, K, A = len(lens), int(fanout), int(append)
        nc = P * K
        total = int(lens.sum())
        dev = self._dev
        with self._lock:
            self._device_op()  # the planner's batches run on the device
        fresh = self.alloc_batch((1 + A) * nc)
        child_tables = torch.empty(K * total + nc * A, dtype=torch.int32, device=dev)
        child_off = torch.empty(nc + 1, dtype=torch.int64, device=dev)
        inc_ids = torch.empty(K * total, dtype=torch.int32, device=dev)
        pairs = torch.empty(2 * nc, dtype=torch.int32, device=dev)
        dec_ids = torch.empty(nc, dtype=torch.int32, device=dev)
        with self._lock:
            N.check(N.lib.akv_fanout_plan(parent_tables.data_ptr(), parent_off.data_ptr(), P, K, A,
                                          fresh.data_ptr(), child_tables.data_ptr(), child_off.data_ptr(),
                                          inc_ids.data_ptr(), pairs.data_ptr(), dec_ids.data_ptr(),
                                          self._stream()))
        self.inc_ref_batch(inc_ids)
        launches = 1 + 1 + 2
        target = pool if pool is not None else self._kv_data
        if copy and target.device.type != "meta":
            _copy_blocks(target, pairs.view(-1, 2), status=self._status)
            launches += 1
        self.dec_ref_batch(dec_ids)
        launches += 4
        return {"child_tables": child_tables, "child_off": child_off, "pairs": pairs.view(-1, 2),
                "child_lens": np.repeat(lens + A, K), "launches": launches}

    def fanout_tree(self, root_tables: torch.Tensor, root_lens, levels: int, fanout: int, append: int,
                    *, level_offsets=None, on_level=None, pairs_out: Optional[torch.Tensor] = None) -> dict:
        """A whole multi-level fan-out (Tree-of-Thought): `levels` levels of
        fanout_level starting from the roots, children of one level being the
        parents of the next, children in (parent, child) order.

        The end state equals the reference's per-child sequence (fork,
        ensure_mutable_block(-1), `append` allocate_block calls, level after
        level): one alloc batch takes every level's ids in the order the
        per-child calls pop them (nothing is freed in between, so one batch
        pops exactly what the levels' batches would), one plan launch per
        level, then one inc_ref batch for all forks and one dec_ref batch for
        all copy-on-write sources.  Every CoW source keeps a refcount >= 1
        throughout, so no id retires and the order of the refcount updates
        cannot change the result.  No copy is made: `pairs[l]` lists level
        l's (src, dst) block copies, ready once `on_level(l)` has been called
        (e.g. to record an event) — copy them on any stream after that point.
        `all_pairs` holds every level's pairs back to back (and, with
        append >= 1, `all_tables` every level's child tables); with append >= 1
        (`independent`) no pair's source is another pair's destination (a
        child's last block, the next level's source, is an appended block),
        so all levels may be copied in one launch.  `pairs_out`, an int32
        (n_pairs, 2) tensor on the allocator's device, becomes all_pairs, so
        that an on_level callback can pass the pairs planned so far on.
        Returns per-level device tensors child_tables / pairs, all_pairs,
        independent and the launch count."""
        K, A = int(fanout), int(append)
        if K < 0 or A < 0 or levels < 0:
            raise ValueError(f"fanout_tree: negative fanout / append / levels ({K}, {A}, {levels})")
        lens = np.asarray(root_lens, np.int64)
        if (lens < 1).any():
            raise ValueError("fanout_tree: every root needs at least one residual block")
        dev = self._dev
        if levels == 0 or K == 0 or len(lens) == 0:  # no child at all: nothing to do
            empty = torch.empty(0, dtype=torch.int32, device=dev)
            for lvl in range(levels):
                if on_level is not None:
                    on_level(lvl)
            return {"child_tables": [empty] * levels, "all_tables": empty, "pairs": [empty.view(0, 2)] * levels,
                    "all_pairs": empty.view(0, 2), "independent": True, "launches": 0}
        shapes, l_ = [], lens
        for _ in range(levels):
            shapes.append((len(l_), int(l_.sum())))
            l_ = np.repeat(l_ + A, K)
        n_fresh = sum((1 + A) * P * K for P, _ in shapes)
        n_pairs = sum(P * K for P, _ in shapes)
        with self._lock:
            self._device_op()  # the planner's batches run on the device
        if pairs_out is not None and (pairs_out.dtype != torch.int32 or pairs_out.device != dev or
                                      tuple(pairs_out.shape) != (n_pairs, 2) or not pairs_out.is_contiguous()):
            raise ValueError(f"fanout_tree: pairs_out must be a contiguous int32 ({n_pairs}, 2) tensor on {dev}")
        fresh_all = self.alloc_batch(n_fresh)
        all_pairs = pairs_out if pairs_out is not None else torch.empty((n_pairs, 2), dtype=torch.int32, device=dev)
        if A >= 1 and 0 < levels <= N.MAX_FANOUT_LEVELS and n_pairs:
            return self._fanout_tree_fused(root_tables, lens, shapes, K, A, fresh_all, all_pairs,
                                           level_offsets, on_level)
        tables = root_tables
        out_tables, out_pairs, incs, decs = [], [], [], []
        launches = 1
        f0 = p0 = 0
        for lvl, (P, total) in enumerate(shapes):
            nc = P * K
            if level_offsets is not None:
                off_d = level_offsets[lvl]
            else:
                off = np.zeros(P + 1, np.int64)
                np.cumsum(lens, out=off[1:])
                off_d = torch.from_numpy(off).to(dev, non_blocking=True)
            fresh = fresh_all[f0 : f0 + (1 + A) * nc]
            pairs = all_pairs[p0 : p0 + nc]
            f0 += (1 + A) * nc
            p0 += nc
            child_tables = torch.empty(K * total + nc * A, dtype=torch.int32, device=dev)
            child_off = torch.empty(nc + 1, dtype=torch.int64, device=dev)
            inc_ids = torch.empty(K * total, dtype=torch.int32, device=dev)
            dec_ids = torch.empty(nc, dtype=torch.int32, device=dev)
            with self._lock:
                N.check(N.lib.akv_fanout_plan(tables.data_ptr(), off_d.data_ptr(), P, K, A, fresh.data_ptr(),
                                              child_tables.data_ptr(), child_off.data_ptr(), inc_ids.data_ptr(),
                                              pairs.data_ptr(), dec_ids.data_ptr(), self._stream()))
            launches += 1
            if on_level is not None:
                on_level(lvl)
            out_tables.append(child_tables)
            out_pairs.append(pairs)
            incs.append(inc_ids)
            decs.append(dec_ids)
            tables = child_tables
            lens = np.repeat(lens + A, K)
        self.inc_ref_batch(torch.cat(incs) if len(incs) > 1 else incs[0])
        self.dec_ref_batch(torch.cat(decs) if len(decs) > 1 else decs[0])
        launches += 2 + 4
        return {"child_tables": out_tables, "pairs": out_pairs, "all_pairs": all_pairs,
                "independent": A >= 1, "launches": launches}

    def _fanout_tree_fused(self, root_tables, lens, shapes, K, A, fresh_all, all_pairs, level_offsets,
                           on_level) -> dict:
        """fanout_tree's levels as one akv_fanout_tree_plan launch (append >= 1)."""
        dev = self._dev
        n_tab = sum(K * total + P * K * A for P, total in shapes)
        n_inc = sum(K * total for _, total in shapes)
        n_kids = all_pairs.shape[0]
        tables = torch.empty(n_tab, dtype=torch.int32, device=dev)
        incs = torch.empty(n_inc, dtype=torch.int32, device=dev)
        decs = torch.empty(n_kids, dtype=torch.int32, device=dev)
        if level_offsets is not None:
            off_d = level_offsets[0]
        else:
            off = np.zeros(len(lens) + 1, np.int64)
            np.cumsum(lens, out=off[1:])
            off_d = torch.from_numpy(off).to(dev, non_blocking=True)
        with self._lock:
            N.check(N.lib.akv_fanout_tree_plan(root_tables.data_ptr(), off_d.data_ptr(), len(lens), int(lens.sum()),
                                               K, A, len(shapes), fresh_all.data_ptr(), tables.data_ptr(),
                                               incs.data_ptr(), all_pairs.data_ptr(), decs.data_ptr(),
                                               self._stream()))
        out_tables, out_pairs = [], []
        t0 = p0 = 0
        for lvl, (P, total) in enumerate(shapes):
            nt, nc = K * total + P * K * A, P * K
            out_tables.append(tables[t0 : t0 + nt])
            out_pairs.append(all_pairs[p0 : p0 + nc])
            t0 += nt
            p0 += nc
            if on_level is not None:
                on_level(lvl)
        self.inc_ref_batch(incs)
        self.dec_ref_batch(decs)
        return {"child_tables": out_tables, "all_tables": tables, "pairs": out_pairs, "all_pairs": all_pairs,
                "independent": True, "launches": 2 + 2 + 4}

    def copy_blocks(self, pairs, *, check_refs: bool = True) -> None:
        """Copy a batch of independent (src, dst) pairs; dsts must be exclusive."""
        if self._kv_data.device.type == "meta":
            return
        if check_refs:
            with self._lock:
                self._flush()  # the device refcounts the kernel checks include the per-call log
        _copy_blocks(self._kv_data, self._device_ids(pairs),
                     ref_counts=self._ref_counts if check_refs else None, status=self._status)

    def check(self) -> None:
        """Wait for queued work (the per-call log replayed first) and raise
        the first device-detected error."""
        with self._lock:
            self._flush()
            self._refused = False
            self._raise_status(self._sync_io(0))
