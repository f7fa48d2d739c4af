"""Device replica of the shared radix tree, and the batched match_prefix call.

The host tree (radix_tree.py) owns the structure; every mutation it makes is
recorded here against a host mirror of four flat arrays and shipped to HBM
as a delta before the next lookup:

* ``tokens``        append-only arena of edge tokens (int32);
* ``edge_off/len``  each node's edge as a range of the arena, indexed by the
                    tree's own node ids (an edge split only narrows ranges,
                    so no token is ever rewritten);
* ``slots``         all nodes' ``children`` dicts as one open-addressing hash
                    table of {parent, first token, child, child's edge length}
                    int32x4 slots,
                    linear probing, parent -1 = empty, -2 = deleted.  The hash
                    is akv_tree_hash (MurmurHash3's 64-bit finalizer over
                    (parent, token)); ``tree_hash`` below is the same function
                    in Python.

A delta is the list of changed slots and node ranges plus the appended token
range; ``flush`` uploads it (akv_tree_apply) on the caller's stream, or the
whole arrays after a resize.  Lookups run the akv_match_prefix kernel: one
warp per query.
"""

from __future__ import annotations

from typing import Optional, Tuple

import numpy as np
import torch

from . import _native as N
from .kernels import stream_handle

_M64 = (1 << 64) - 1
EMPTY = -1
DELETED = -2


def tree_hash(parent: int, token: int) -> int:
    """MurmurHash3 fmix64 of (parent << 32 | token), low 32 bits."""
    k = ((parent & 0xFFFFFFFF) << 32) | (token & 0xFFFFFFFF)
    k ^= k >> 33
    k = (k * 0xFF51AFD7ED558CCD) & _M64
    k ^= k >> 33
    k = (k * 0xC4CEB9FE1A85EC53) & _M64
    k ^= k >> 33
    return k & 0xFFFFFFFF


def tree_hash_np(parent: np.ndarray, token: np.ndarray) -> np.ndarray:
    """Vectorised tree_hash (uint64 arithmetic wraps like the C code)."""
    k = (parent.astype(np.uint64) & np.uint64(0xFFFFFFFF)) << np.uint64(32)
    k |= token.astype(np.int64).astype(np.uint64) & np.uint64(0xFFFFFFFF)
    with np.errstate(over="ignore"):
        k ^= k >> np.uint64(33)
        k *= np.uint64(0xFF51AFD7ED558CCD)
        k ^= k >> np.uint64(33)
        k *= np.uint64(0xC4CEB9FE1A85EC53)
        k ^= k >> np.uint64(33)
    return (k & np.uint64(0xFFFFFFFF)).astype(np.uint32)


class DeviceTree:
    """Host mirror + HBM copy of the shared tree; see the module docstring."""

    def __init__(self, device: torch.device, node_cap: int = 1024, slot_cap: int = 4096,
                 token_cap: int = 1 << 16) -> None:
        self.device = device
        self.h_tokens = np.zeros(token_cap, np.int32)
        self.n_tokens = 0
        self.h_off = np.zeros(node_cap, np.int64)
        self.h_len = np.zeros(node_cap, np.int32)
        self.h_slots = np.full((slot_cap, 4), EMPTY, np.int32)
        self.h_slots[:, 3] = 0
        self.live = 0
        self.dead = 0
        self._slot_of: dict = {}  # (parent, token) -> slot index
        self._dirty_slots: set = set()
        self._dirty_nodes: set = set()
        self._tok_flushed = 0
        self._full = True  # next flush uploads everything
        self.d_tokens = torch.zeros(token_cap, dtype=torch.int32, device=device)
        self.d_off = torch.zeros(node_cap, dtype=torch.int64, device=device)
        self.d_len = torch.zeros(node_cap, dtype=torch.int32, device=device)
        self.d_slots = torch.zeros((slot_cap, 4), dtype=torch.int32, device=device)
        self.status = torch.zeros(N.STATUS_BYTES // 4, dtype=torch.int32, device=device)
        self._view: Optional[N.AkvTreeView] = None

    # ── mutations (host mirror) ──────────────────────────────────────────────
    def append_tokens(self, toks: np.ndarray) -> int:
        toks = np.asarray(toks, np.int32)
        need = self.n_tokens + len(toks)
        if need > len(self.h_tokens):
            cap = max(need, 2 * len(self.h_tokens))
            grown = np.zeros(cap, np.int32)
            grown[: self.n_tokens] = self.h_tokens[: self.n_tokens]
            self.h_tokens = grown
            self._full = True
        off = self.n_tokens
        self.h_tokens[off:need] = toks
        self.n_tokens = need
        return off

    def edge(self, off: int, length: int) -> np.ndarray:
        return self.h_tokens[off : off + length]

    def set_node(self, nid: int, off: int, length: int) -> None:
        if nid >= len(self.h_off):
            cap = max(nid + 1, 2 * len(self.h_off))
            for name in ("h_off", "h_len"):
                old = getattr(self, name)
                new = np.zeros(cap, old.dtype)
                new[: len(old)] = old
                setattr(self, name, new)
            self._full = True
        self.h_off[nid] = off
        self.h_len[nid] = length
        self._dirty_nodes.add(nid)

    def clear_node(self, nid: int) -> None:
        if nid < len(self.h_off):
            self.set_node(nid, 0, 0)

    def _probe(self, parent: int, token: int) -> Tuple[int, int]:
        """(slot holding the key or -1, first reusable slot on the path)."""
        mask = len(self.h_slots) - 1
        i = tree_hash(parent, token) & mask
        free = -1
        slots = self.h_slots
        for _ in range(len(slots)):
            p = slots[i, 0]
            if p == EMPTY:
                return -1, (free if free >= 0 else i)
            if p == DELETED:
                if free < 0:
                    free = i
            elif p == parent and slots[i, 1] == token:
                return i, free
            i = (i + 1) & mask
        return -1, free

    def set_child(self, parent: int, token: int, child: int, child_len: int) -> None:
        """children[parent][token] = child; the slot also carries the child's
        edge length (the device walk chases hops with it)."""
        key = (parent, token)
        s = self._slot_of.get(key)
        if s is None:
            if 2 * (self.live + self.dead + 1) > len(self.h_slots):
                self._rehash(max(len(self.h_slots), 4 * (self.live + 1)))
            _, s = self._probe(parent, token)
            if self.h_slots[s, 0] == DELETED:
                self.dead -= 1
            self.live += 1
            self._slot_of[key] = s
        self.h_slots[s] = (parent, token, child, child_len)
        self._dirty_slots.add(s)

    def del_child(self, parent: int, token: int) -> None:
        s = self._slot_of.pop((parent, token), None)
        if s is None:
            return
        self.h_slots[s] = (DELETED, 0, 0, 0)
        self.live -= 1
        self.dead += 1
        self._dirty_slots.add(s)

    def _rehash(self, min_slots: int) -> None:
        cap = 1
        while cap < 2 * min_slots:
            cap <<= 1
        cap = max(cap, 64)
        entries = [(k, int(self.h_slots[s, 2]), int(self.h_slots[s, 3])) for k, s in self._slot_of.items()]
        self.h_slots = np.full((cap, 4), EMPTY, np.int32)
        self.h_slots[:, 3] = 0
        self._slot_of = {}
        self.live = self.dead = 0
        self._dirty_slots.clear()
        for (p, t), c, ln in entries:
            _, s = self._probe(p, t)
            self.h_slots[s] = (p, t, c, ln)
            self._slot_of[(p, t)] = s
            self.live += 1
        self._full = True

    # ── upload ───────────────────────────────────────────────────────────────
    def flush(self) -> None:
        """Ship pending changes to the device (on the current stream)."""
        dev = self.device
        if self._full:
            if self.d_tokens.numel() < len(self.h_tokens):
                self.d_tokens = torch.zeros(len(self.h_tokens), dtype=torch.int32, device=dev)
            if self.d_off.numel() != len(self.h_off):
                self.d_off = torch.zeros(len(self.h_off), dtype=torch.int64, device=dev)
                self.d_len = torch.zeros(len(self.h_len), dtype=torch.int32, device=dev)
            if self.d_slots.shape[0] != len(self.h_slots):
                self.d_slots = torch.zeros((len(self.h_slots), 4), dtype=torch.int32, device=dev)
            self.d_tokens[: self.n_tokens].copy_(torch.from_numpy(self.h_tokens[: self.n_tokens]))
            self.d_off.copy_(torch.from_numpy(self.h_off))
            self.d_len.copy_(torch.from_numpy(self.h_len))
            self.d_slots.copy_(torch.from_numpy(self.h_slots))
            self._tok_flushed = self.n_tokens
            self._dirty_nodes.clear()
            self._dirty_slots.clear()
            self._full = False
            self._view = None
            return
        if self.n_tokens > self._tok_flushed:
            lo, hi = self._tok_flushed, self.n_tokens
            self.d_tokens[lo:hi].copy_(torch.from_numpy(self.h_tokens[lo:hi]))
            self._tok_flushed = hi
            self._view = None
        if not (self._dirty_nodes or self._dirty_slots):
            return
        su = None
        nu = None
        if self._dirty_slots:
            idx = np.fromiter(self._dirty_slots, np.int64, len(self._dirty_slots))
            su = np.empty((len(idx), 5), np.int32)
            su[:, 0] = idx
            su[:, 1:] = self.h_slots[idx, :4]
        if self._dirty_nodes:
            idx = np.fromiter(self._dirty_nodes, np.int64, len(self._dirty_nodes))
            nu = np.empty((len(idx), 3), np.int64)
            nu[:, 0] = idx
            nu[:, 1] = self.h_off[idx]
            nu[:, 2] = self.h_len[idx]
        su_d = torch.from_numpy(su).to(dev) if su is not None else None
        nu_d = torch.from_numpy(nu).to(dev) if nu is not None else None
        N.check(N.lib.akv_tree_apply(
            self.view(), su_d.data_ptr() if su_d is not None else None, 0 if su is None else len(su),
            nu_d.data_ptr() if nu_d is not None else None, 0 if nu is None else len(nu),
            self.status.data_ptr(), stream_handle(dev)))
        self._dirty_nodes.clear()
        self._dirty_slots.clear()

    def view(self) -> N.AkvTreeView:
        if self._view is None:
            self._view = N.AkvTreeView(
                self.d_tokens.data_ptr(), self.d_off.data_ptr(), self.d_len.data_ptr(),
                self.d_slots.data_ptr(), self._tok_flushed, self.d_off.numel(), self.d_slots.shape[0] - 1)
        return self._view

    # ── lookups ──────────────────────────────────────────────────────────────
    def match(self, tokens: torch.Tensor, q_off: torch.Tensor, nq: int, block_size: int,
              out_node: torch.Tensor, out_len: torch.Tensor, out_cmp: Optional[torch.Tensor],
              chunks: int = 0, order: Optional[torch.Tensor] = None) -> None:
        """Enqueue akv_match_prefix for nq queries packed in `tokens` / `q_off`
        (device int32 / int64 tensors); `order` (device int32) is the launch
        order of the queries, longest first by default in pack_queries."""
        self.flush()
        N.check(N.lib.akv_match_prefix_variant(
            self.view(), tokens.data_ptr(), q_off.data_ptr(), nq, block_size, out_node.data_ptr(),
            out_len.data_ptr(), out_cmp.data_ptr() if out_cmp is not None else None,
            order.data_ptr() if order is not None else None, self.status.data_ptr(), chunks,
            stream_handle(self.device)))

    def check(self) -> None:
        s = self.status.cpu()
        if int(s[0]) != 0:
            self.status.zero_()
            raise RuntimeError(
                f"agentkv_b200 tree replica error: {N.ERROR_NAMES.get(int(s[0]), int(s[0]))} "
                f"(query/update {int(s[1])}, node {int(s[2])})")
