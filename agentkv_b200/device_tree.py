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

Batched lookups also use the unary-chain runs (``build_runs``), derived
from the slots: every maximal chain of single-child nodes stored once as
consecutive int32x4 entries {child, first token, edge length, entries left},
and ``run_head[node]`` the entry of a single-child node's child (-1
otherwise).  The kernel takes up to 32 hops of a chain from one load instead
of one dependent hash probe per hop; the runs are rebuilt from the host
mirror when the tree has changed, and replicas receive the owner's.
"""

from __future__ import annotations

import os
import time
from array import array
from typing import Optional, Sequence, Tuple

import numpy as np
import torch

from . import _native as N
from .kernels import stream_handle

try:
    from . import _akv_pyhost as _pyhost
except ImportError as exc:  # built beside libagentkv_b200.so by _build.build()
    raise ImportError("agentkv_b200: the host helper _akv_pyhost is not built; run "
                      "`python -m agentkv_b200._build`") from exc

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


class _Changes:
    """Changes of the host mirror not yet taken by one consumer (the local
    device upload, or the replicas on other GPUs)."""

    __slots__ = ("slots", "nodes", "tok_from", "full", "cmds", "cmd_tokens", "cmd_len", "cover")

    def __init__(self) -> None:
        self.slots: set = set()
        self.nodes: set = set()
        self.tok_from = 0
        self.full = True
        self.drop_commands()

    def drop_commands(self) -> None:
        """Forget the recorded commands (the rows or the whole arrays cover
        the changes instead); the next change starts a new command list."""
        self.cmds: list = []  # the host tree's inserts and prunes since the last take
        self.cmd_tokens: list = []
        self.cmd_len = 0
        self.cover = True  # every change since the last take came from a command

    def take(self, n_tokens: int) -> None:
        """Everything recorded has been sent to this consumer."""
        self.tok_from = n_tokens
        self.nodes.clear()
        self.slots.clear()
        self.drop_commands()

    def commands_ready(self) -> bool:
        return bool(self.cmds) and self.cover and not self.full


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
        self._local = _Changes()  # for this GPU's arrays
        self._peers: Optional[_Changes] = None  # for replicas (track_peers)
        self._dev_tokens = 0  # tokens on the device
        self._replica = False
        self._runs_dirty = True
        self.runs_version = 0  # bumped by every build_runs that rebuilt
        self._full_ms: Optional[float] = None  # host time of the last full build_runs
        self._patch_ms: Optional[float] = None  # host time of the last incremental one
        self._rent_ms = 0.0  # one-probe-per-hop lookup time since the last change
        self._last_batch_ms = 0.0  # host time of the last batched lookup
        # child structure for the incremental run updates
        self._kids: dict = {}  # parent -> set of first tokens of its children
        self._parent_of: dict = {}  # child -> parent
        self._n_unary = 0  # nodes with exactly one child
        self._runs_touched: set = set()  # nodes whose children changed since the last build
        self._h_run_head: Optional[np.ndarray] = None  # host copy of the runs
        self._h_runs = np.zeros((0, 4), np.int32)
        self._n_entries = 0  # entries in use, live and superseded
        self._node_bound = 0  # 1 + the largest node id in a child link
        self.d_run_head: Optional[torch.Tensor] = None
        self.d_runs: Optional[torch.Tensor] = None
        self.d_tokens = torch.zeros(token_cap, dtype=torch.int32, device=device)
        self.d_off = torch.zeros(node_cap, dtype=torch.int64, device=device)
        self.d_len = torch.zeros(node_cap, dtype=torch.int32, device=device)
        self.d_slots = torch.zeros((slot_cap, 4), dtype=torch.int32, device=device)
        self.status = torch.zeros(N.STATUS_BYTES // 4, dtype=torch.int32, device=device)
        self._view: Optional[N.AkvTreeView] = None
        self._stage: Optional["QueryStage"] = None  # match_batch's reusable buffers
        self._split_scratch: Optional[torch.Tensor] = None  # akv_match_prefix_split's work space
        self._staged_scratch: Optional[torch.Tensor] = None  # akv_match_prefix_staged's work space
        # Changes as commands (akv_tree_commands): the host tree's inserts and
        # prunes since the last upload, applied on the device by the replica
        # itself instead of uploading the rows they changed.  Used when every
        # change since the last upload came from a recorded command and no
        # array was resized or rehashed.
        self.device_commands = True
        self._cmd_scope = False
        self.command_uploads = 0  # uploads done as commands (for tests and figures)

    # ── mutations (host mirror) ──────────────────────────────────────────────
    def append_tokens(self, toks: np.ndarray) -> int:
        if not self._cmd_scope:
            for c in self._trackers():
                c.cover = False
        toks = np.asarray(toks, np.int32)
        need = self.n_tokens + len(toks)
        if need > len(self.h_tokens):
            cap = max(need, 2 * len(self.h_tokens))
            grown = np.zeros(cap, np.int32)
            grown[: self.n_tokens] = self.h_tokens[: self.n_tokens]
            self.h_tokens = grown
            self._mark_full()
        off = self.n_tokens
        self.h_tokens[off:need] = toks
        self.n_tokens = need
        return off

    def edge(self, off: int, length: int) -> np.ndarray:
        return self.h_tokens[off : off + length]

    def set_node(self, nid: int, off: int, length: int) -> None:
        if not self._cmd_scope:
            for c in self._trackers():
                c.cover = False
        if nid >= len(self.h_off):
            cap = max(nid + 1, 2 * len(self.h_off))
            for name in ("h_off", "h_len"):
                old = getattr(self, name)
                new = np.zeros(cap, old.dtype)
                new[: len(old)] = old
                setattr(self, name, new)
            self._mark_full()
        self.h_off[nid] = off
        self.h_len[nid] = length  # edge ranges are not part of the runs
        for c in self._trackers():
            c.nodes.add(nid)

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
        if not self._cmd_scope:
            for c in self._trackers():
                c.cover = False
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
            kids = self._kids.setdefault(parent, set())
            self._n_unary += (len(kids) == 0) - (len(kids) == 1)
            kids.add(token)
        else:
            old = int(self.h_slots[s, 2])
            if old != child and self._parent_of.get(old) == parent:
                del self._parent_of[old]
        self._parent_of[child] = parent
        self._node_bound = max(self._node_bound, parent + 1, child + 1)
        self.h_slots[s] = (parent, token, child, child_len)
        self._changed(parent)
        for c in self._trackers():
            c.slots.add(s)

    def del_child(self, parent: int, token: int) -> None:
        if not self._cmd_scope:
            for c in self._trackers():
                c.cover = False
        s = self._slot_of.pop((parent, token), None)
        if s is None:
            return
        child = int(self.h_slots[s, 2])
        if self._parent_of.get(child) == parent:
            del self._parent_of[child]
        kids = self._kids[parent]
        kids.discard(token)
        self._n_unary += (len(kids) == 1) - (len(kids) == 0)
        if not kids:
            del self._kids[parent]
        self.h_slots[s] = (DELETED, 0, 0, 0)
        self._changed(parent)
        self.live -= 1
        self.dead += 1
        for c in self._trackers():
            c.slots.add(s)

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
        for (p, t), c, ln in entries:
            _, s = self._probe(p, t)
            self.h_slots[s] = (p, t, c, ln)
            self._slot_of[(p, t)] = s
            self.live += 1
        self._mark_full()

    def _changed(self, parent: int) -> None:
        # `parent`'s children changed: the runs through it are stale, and a
        # new stable period of the tree begins
        self._runs_dirty = True
        self._runs_touched.add(parent)
        self._rent_ms = 0.0

    def _trackers(self):
        return (self._local,) if self._peers is None else (self._local, self._peers)

    def _mark_full(self) -> None:
        for c in self._trackers():
            c.full = True
            c.slots.clear()
            c.nodes.clear()
            c.cover = False

    def as_replica(self) -> None:
        """This tree's device arrays come from another GPU's deltas
        (apply_delta): its own (empty) host mirror is never uploaded."""
        self._local.full = False
        self._replica = True

    def track_peers(self) -> None:
        """Also record changes for replicas on other GPUs (take_delta(peers=True));
        the first peer delta is a full one."""
        if self._peers is None:
            self._peers = _Changes()

    # ── changes as commands ──────────────────────────────────────────────────
    def begin_insert(self, parent: int, tokens: np.ndarray, first_new_id: int, block_size: int) -> None:
        """The host tree is about to insert `tokens` under `parent`
        (DualRadixTree._insert_shared_locked); its mirror changes until
        end_command() are this insert's."""
        toks = np.asarray(tokens, np.int32)
        for c in self._trackers():
            c.cmds.append((1, parent, first_new_id, c.cmd_len, len(toks), self.n_tokens, block_size, 0))
            c.cmd_tokens.append(toks)
            c.cmd_len += len(toks)
        self._cmd_scope = True

    def begin_prune(self, parent: int, node: int) -> None:
        """The host tree is about to prune `node` (its parent, or -1 when the
        parent is gone); its mirror changes until end_command() are this
        prune's."""
        for c in self._trackers():
            c.cmds.append((2, parent, node, 0, 0, 0, 0, 0))
        self._cmd_scope = True

    def end_command(self) -> None:
        self._cmd_scope = False

    def take_commands(self, peers: bool = False) -> Optional[dict]:
        """The recorded commands for a consumer when they account for every
        change it has not taken (no other change, no resize or rehash), as
        host arrays {"commands" [n, 8] int64, "payload" int32, "n_tokens",
        "tok_lo"}, and marks them taken; else None (take_delta then)."""
        c = self._peers if peers else self._local
        if c is None or not c.commands_ready():
            return None
        d = {"commands": np.asarray(c.cmds, np.int64).reshape(-1, 8),
             "payload": np.concatenate(c.cmd_tokens) if c.cmd_tokens else np.zeros(0, np.int32),
             "n_tokens": self.n_tokens, "tok_lo": c.tok_from}
        c.take(self.n_tokens)
        return d

    # ── upload ───────────────────────────────────────────────────────────────
    def flush(self) -> None:
        """Ship pending changes to the device (on the current stream): as the
        host tree's commands when they account for every change since the
        last upload, else as the changed rows (or the whole arrays)."""
        if self.device_commands and not self._replica and self.d_tokens.numel() >= self.n_tokens:
            d = self.take_commands()
            if d is not None:
                self.apply_commands(d)
                return
        self._local.drop_commands()
        d = self.take_delta()
        if d is not None:
            self.apply_delta(d)

    def apply_commands(self, d: dict) -> None:
        """Apply the host tree's inserts and prunes to the device arrays
        (akv_tree_commands): from take_commands on this tree or, for a
        replica on another GPU, on the owner's.  The arrays may be host
        (numpy) or device tensors."""
        dev = self.device
        cmds, pay = d["commands"], d["payload"]
        if not isinstance(cmds, torch.Tensor):
            cmds = torch.from_numpy(np.ascontiguousarray(cmds, np.int64))
            pay = torch.from_numpy(np.ascontiguousarray(pay, np.int32))
            if dev.type == "cuda":
                cmds, pay = cmds.pin_memory(), pay.pin_memory()
        cmds = cmds.to(dev, non_blocking=True).reshape(-1, 8)
        pay = pay.to(dev, non_blocking=True).reshape(-1)
        n = cmds.shape[0]
        if n == 0:
            return
        self._dev_tokens = int(d["n_tokens"])
        self._view = None
        self._drop_replica_runs()  # a replica's runs describe the tree before these changes
        N.check(N.lib.akv_tree_commands(self.view(), self.d_tokens.numel(), cmds.data_ptr(), n,
                                        pay.data_ptr() if pay.numel() else None, pay.numel(),
                                        self.status.data_ptr(), stream_handle(dev)))
        self._cmd_keep = (cmds, pay)  # alive until the launch has read them
        self.command_uploads += 1

    def take_delta(self, peers: bool = False) -> Optional[dict]:
        """Changes of the host mirror not yet taken by this consumer (the local
        upload, or with peers=True the replicas), as host arrays; None when
        there are none.  A delta is either full (the whole arrays, after a
        resize or rehash) or incremental (appended tokens, changed slots as
        [slot, parent, token, child, child_len] rows, changed nodes as
        [node, edge_off, edge_len] rows)."""
        c = self._peers if peers else self._local
        if c is None:
            raise RuntimeError("take_delta(peers=True) needs track_peers() first")
        if c.full:
            d = {"full": True, "n_tokens": self.n_tokens, "tokens": self.h_tokens[: self.n_tokens],
                 "token_cap": len(self.h_tokens), "off": self.h_off, "len": self.h_len, "slots": self.h_slots}
            c.full = False
        else:
            lo, hi = c.tok_from, self.n_tokens
            if hi == lo and not (c.nodes or c.slots):
                return None
            su = np.empty((len(c.slots), 5), np.int32)
            if len(su):
                idx = np.fromiter(c.slots, np.int64, len(c.slots))
                su[:, 0] = idx
                su[:, 1:] = self.h_slots[idx, :4]
            nu = np.empty((len(c.nodes), 3), np.int64)
            if len(nu):
                idx = np.fromiter(c.nodes, np.int64, len(c.nodes))
                nu[:, 0] = idx
                nu[:, 1] = self.h_off[idx]
                nu[:, 2] = self.h_len[idx]
            d = {"full": False, "n_tokens": hi, "tok_lo": lo, "tokens": self.h_tokens[lo:hi], "su": su, "nu": nu}
        c.take(self.n_tokens)
        return d

    def apply_shared(self, d: dict) -> None:
        """Apply what TreeReplicaSync.share returned: commands or a delta."""
        if "commands" in d:
            self.apply_commands(d)
        else:
            self.apply_delta(d)

    def apply_delta(self, d: dict) -> None:
        """Bring the device arrays up to date with a delta (from take_delta on
        this tree or, for a replica on another GPU, on the owner's tree).  Its
        arrays may be host (numpy) or device tensors."""
        dev = self.device

        def on_dev(a, dtype):
            if isinstance(a, torch.Tensor):
                return a.to(dev, dtype=dtype)
            return torch.from_numpy(np.ascontiguousarray(a)).to(dev, dtype=dtype)

        if d["full"]:
            cap = int(d["token_cap"])
            if self.d_tokens.numel() < cap:
                self.d_tokens = torch.zeros(cap, dtype=torch.int32, device=dev)
            n = int(d["n_tokens"])
            if n:
                self.d_tokens[:n].copy_(on_dev(d["tokens"], torch.int32))
            self.d_off = on_dev(d["off"], torch.int64).clone()
            self.d_len = on_dev(d["len"], torch.int32).clone()
            self.d_slots = on_dev(d["slots"], torch.int32).reshape(-1, 4).clone()
            self._dev_tokens = n
            self._view = None
            self._drop_replica_runs()
            return
        lo, hi = int(d["tok_lo"]), int(d["n_tokens"])
        if hi > lo:
            self.d_tokens[lo:hi].copy_(on_dev(d["tokens"], torch.int32))
            self._dev_tokens = hi
            self._view = None
        n_su, n_nu = len(d["su"]), len(d["nu"])
        if n_su == 0 and n_nu == 0:
            return
        if n_su:
            self._drop_replica_runs()  # node rows (edge ranges) leave the runs valid
        su_d = on_dev(d["su"], torch.int32) if n_su else None
        nu_d = on_dev(d["nu"], torch.int64) if n_nu else None
        N.check(N.lib.akv_tree_apply(
            self.view(), su_d.data_ptr() if su_d is not None else None, n_su,
            nu_d.data_ptr() if nu_d is not None else None, n_nu,
            self.status.data_ptr(), stream_handle(dev)))

    def view(self, runs: bool = False) -> N.AkvTreeView:
        """The device arrays as an AkvTreeView; with runs=True it also points
        at the unary-chain runs (build_runs must be current)."""
        if self._view is None:
            self._view = N.AkvTreeView(
                self.d_tokens.data_ptr(), self.d_off.data_ptr(), self.d_len.data_ptr(),
                self.d_slots.data_ptr(), self._dev_tokens, self.d_off.numel(), self.d_slots.shape[0] - 1,
                None, None, 0, 0)
        if not runs or self.d_run_head is None:
            return self._view
        v = N.AkvTreeView.from_buffer_copy(self._view)
        v.run_head = self.d_run_head.data_ptr()
        v.run_entries = self.d_runs.data_ptr()
        v.n_runs = self.d_runs.shape[0]
        v.run_nodes = self.d_run_head.numel()
        return v

    # ── unary-chain runs (for the batched lookup) ────────────────────────────
    def _drop_replica_runs(self) -> None:
        # a replica's runs come from its owner; a structural change makes
        # them stale until the owner's next runs arrive (set_runs)
        if self._replica:
            self.d_run_head = self.d_runs = None

    def set_runs(self, run_head: torch.Tensor, runs: torch.Tensor) -> None:
        """A replica takes the owner's runs (device int32 tensors in
        build_runs' layout: a head per node, [n, 4] entries)."""
        self.d_run_head = run_head.to(self.device, torch.int32).reshape(-1)
        self.d_runs = runs.to(self.device, torch.int32).reshape(-1, 4)
        self._runs_dirty = False

    def build_runs(self) -> None:
        """Bring the runs up to date with the host mirror when the tree
        changed since the last build: for every node with exactly one child,
        the chain it starts (its only child, that child's only child, ...
        through the first node without exactly one child), stored per maximal
        chain, each node pointing at its suffix.  After the first build only
        the chains through nodes whose children changed are written again
        (appended; the entries they supersede stay unused until a full build
        compacts them).  A replica without a host mirror has no runs of its
        own (it uses the owner's, set_runs)."""
        if not self._runs_dirty or self._replica:
            return
        t0 = time.perf_counter()
        n = max(len(self.h_off), self._node_bound)
        full = self._next_build_is_full(n)
        if full:
            self._full_runs(n)
        else:
            self._patch_runs(n)
        self._runs_touched.clear()
        runs = self._h_runs[: max(self._n_entries, 1)]  # entry 0 keeps a valid pointer when there are none
        self.d_run_head = torch.from_numpy(self._h_run_head[:n].copy()).to(self.device)
        self.d_runs = torch.from_numpy(runs.copy()).to(self.device)
        self._runs_dirty = False
        self.runs_version += 1
        ms = (time.perf_counter() - t0) * 1e3
        if full:
            self._full_ms = ms
        else:
            self._patch_ms = ms

    def _next_build_is_full(self, n: int) -> bool:
        # a full build the first time, to compact superseded entries, and when
        # so many nodes changed that rewriting their chains would cost more
        superseded = self._n_entries - self._n_unary
        return (self._h_run_head is None or superseded > max(4096, self._n_unary)
                or len(self._runs_touched) > max(64, n // 64))

    def _full_runs(self, n: int) -> None:
        # Array form (no per-node Python): child counts give the unary nodes,
        # list ranking by pointer doubling gives each one's entries left in
        # its chain (rem) and its chain's head, and a head's chain occupies
        # rem[head] consecutive entries from an exclusive scan over the heads.
        m = len(self._slot_of)
        rows = self.h_slots[np.fromiter(self._slot_of.values(), np.int64, m)].astype(np.int64)
        par, tok, ch, ln = rows[:, 0], rows[:, 1], rows[:, 2], rows[:, 3]
        unary = np.bincount(par, minlength=n) == 1
        sel = unary[par]  # the slot rows of the unary nodes' only children
        nxt = np.full(n, -1, np.int64)
        ntok = np.zeros(n, np.int64)
        nlen = np.zeros(n, np.int64)
        nxt[par[sel]], ntok[par[sel]], nlen[par[sel]] = ch[sel], tok[sel], ln[sel]
        parent_of = np.full(n, -1, np.int64)
        parent_of[ch] = par
        us = np.flatnonzero(unary)
        # succ: the chain's next unary node (-1 at its end); pred: its previous one
        succ = np.full(n, -1, np.int64)
        succ[us] = np.where(unary[nxt[us]], nxt[us], -1)
        pred = np.full(n, -1, np.int64)
        pu = parent_of[us]
        pred[us] = np.where((pu >= 0) & unary[np.maximum(pu, 0)], pu, -1)
        rem = unary.astype(np.int64)
        jump = succ.copy()
        for _ in range(64):
            live = np.flatnonzero(jump >= 0)
            if len(live) == 0:
                break
            rem[live] += rem[jump[live]]
            jump[live] = jump[jump[live]]
        else:
            raise RuntimeError("DeviceTree.build_runs: the child links form a cycle")
        root = np.where(pred >= 0, pred, np.arange(n))
        for _ in range(64):
            nr = root[root]
            if np.array_equal(nr, root):
                break
            root = nr
        else:
            raise RuntimeError("DeviceTree.build_runs: the child links form a cycle")
        heads = np.flatnonzero(unary & (pred < 0))
        base = np.zeros(n, np.int64)
        base[heads] = np.cumsum(rem[heads]) - rem[heads]
        pos = base[root[us]] + rem[root[us]] - rem[us]
        head = np.full(n, -1, np.int32)
        head[us] = pos
        cap = max(16, 2 * len(us))
        self._h_runs = np.zeros((cap, 4), np.int32)
        self._h_runs[pos] = np.stack([nxt[us], ntok[us], nlen[us], rem[us]], axis=1)
        self._h_run_head = head
        self._n_entries = len(us)

    def _patch_runs(self, n: int) -> None:
        # Rewrite every chain that runs through a node whose children changed
        # (the chain entering it, through its parent, and the one leaving it);
        # chains split off below a change keep their entries, which are
        # suffixes of the old chain ending where they still end.
        kids, parent_of = self._kids, self._parent_of
        if len(self._h_run_head) < n:
            grown = np.full(max(n, 2 * len(self._h_run_head)), -1, np.int32)
            grown[: len(self._h_run_head)] = self._h_run_head
            self._h_run_head = grown
        head = self._h_run_head
        limit = len(parent_of) + 1

        def unary(u) -> bool:
            k = kids.get(u)
            return k is not None and len(k) == 1

        starts = set()
        for p in self._runs_touched:
            if not unary(p) and p < len(head):
                head[p] = -1
            for q in (p, parent_of.get(p)):
                if q is None or not unary(q):
                    continue
                steps = 0
                while parent_of.get(q) is not None and unary(parent_of[q]):
                    q = parent_of[q]
                    steps += 1
                    if steps > limit:
                        raise RuntimeError("DeviceTree.build_runs: the child links form a cycle")
                starts.add(q)
        for u in starts:
            chain = []
            while unary(u):
                (t,) = kids[u]
                s = self._slot_of[(u, t)]
                c = int(self.h_slots[s, 2])
                chain.append((u, c, t, int(self.h_slots[s, 3])))
                u = c
                if len(chain) > limit:
                    raise RuntimeError("DeviceTree.build_runs: the child links form a cycle")
            m, base = len(chain), self._n_entries
            if base + m > len(self._h_runs):
                grown = np.zeros((max(2 * len(self._h_runs), base + m, 16), 4), np.int32)
                grown[:base] = self._h_runs[:base]
                self._h_runs = grown
            for k, (v, c, t, ln) in enumerate(chain):
                self._h_runs[base + k] = (c, t, ln, m - k)
                head[v] = base + k
            self._n_entries = base + m

    def want_runs(self) -> bool:
        """Whether a batched lookup should use the unary-chain runs: yes when
        they are current; on a replica only when the owner's have arrived.
        With stale runs the rule is ski rental: rebuild once the
        one-probe-per-hop lookups since the tree last changed, counting the
        coming one at the last batch's time, have cost as much as the
        rebuild would — the last build of the kind the next one will be (an
        incremental one costs tens of microseconds, so a tree that changes
        between batches normally rebuilds every time; a full one, needed
        after many changes or to compact, is paid for by renting first).  A
        tree whose runs were never built builds them."""
        if self._replica:
            return self.d_run_head is not None
        if not self._runs_dirty or self._full_ms is None:
            return True
        if self._next_build_is_full(max(len(self.h_off), self._node_bound)):
            cost = self._full_ms
        else:
            cost = self._patch_ms or 0.0  # no incremental build yet: try one
        return self._rent_ms + self._last_batch_ms >= cost

    def note_lookup(self, ms: float, runs: bool) -> None:
        """Record a batched lookup's host time and whether it used the runs."""
        self._last_batch_ms = ms
        if not runs:
            self._rent_ms += ms

    # ── lookups ──────────────────────────────────────────────────────────────
    def match(self, tokens: torch.Tensor, q_off: torch.Tensor, nq: int, block_size: int,
              out_node: torch.Tensor, out_len: torch.Tensor, out_cmp: Optional[torch.Tensor],
              chunks: int = 0, order: Optional[torch.Tensor] = None, runs: bool = False,
              plan: Optional["SplitPlan"] = None, status: Optional[torch.Tensor] = None,
              staged: bool = False, window_tokens: int = 0, n_tokens: Optional[int] = None) -> None:
        """Enqueue a match_prefix lookup of nq queries packed in `tokens` /
        `q_off` (device int32 / int64 tensors); `order` (device int32) is the
        launch order of the queries, longest first by default in
        pack_queries.  With runs=True unary chains are followed a run at a
        time (the runs are rebuilt first if the tree changed: worth it for
        batches, not for the single lookups of create_root).

        With a `plan` (split_plan of the queries' lengths in `order`) the
        lookup is akv_match_prefix_split: every query's positions in ranges
        of plan.tokens_per_range tokens, one warp per range, so a long query
        does not hold the batch; its scratch is this tree's.  Without it,
        akv_match_prefix_variant (one warp per query).  The answers are the
        same.  With staged=True the lookup is akv_match_prefix_staged: one
        warp per query follows the tree by first tokens, then one warp per
        window_tokens-token window (0 = the library's default) compares the
        followed path; n_tokens is the packing's token count (default
        tokens.numel()).  `status` (8 int32 on the device) replaces the
        tree's status record for this lookup."""
        self.flush()
        if runs:
            self.build_runs()
        st = (status if status is not None else self.status).data_ptr()
        out_c = out_cmp.data_ptr() if out_cmp is not None else None
        ordp = order.data_ptr() if order is not None else None
        if staged:
            if plan is not None:
                raise ValueError("match_prefix: a lookup is either split or staged")
            nt = tokens.numel() if n_tokens is None else int(n_tokens)
            need = int(N.lib.akv_match_staged_scratch_bytes(nq, nt, window_tokens))
            if need < 0:
                raise ValueError(f"match_prefix: no staged lookup of {nq} queries, {nt} tokens, "
                                 f"window {window_tokens}")
            if self._staged_scratch is None or self._staged_scratch.numel() < need:
                cap = max(need, 2 * (self._staged_scratch.numel() if self._staged_scratch is not None else 0))
                self._staged_scratch = torch.empty(cap, dtype=torch.uint8, device=self.device)
            sc = self._staged_scratch
            N.check(N.lib.akv_match_prefix_staged(
                self.view(runs), tokens.data_ptr(), q_off.data_ptr(), nq, nt, block_size, out_node.data_ptr(),
                out_len.data_ptr(), out_c, ordp, window_tokens, sc.data_ptr(), sc.numel(), st,
                stream_handle(self.device)))
            return
        if plan is None:
            N.check(N.lib.akv_match_prefix_variant(
                self.view(runs), tokens.data_ptr(), q_off.data_ptr(), nq, block_size, out_node.data_ptr(),
                out_len.data_ptr(), out_c, ordp, st, chunks, stream_handle(self.device)))
            return
        if order is None:
            raise ValueError("match_prefix: a split lookup needs the longest-first order")
        need = plan.scratch_bytes(nq)
        if self._split_scratch is None or self._split_scratch.numel() < need:
            cap = max(need, 2 * (self._split_scratch.numel() if self._split_scratch is not None else 0), 1 << 16)
            self._split_scratch = torch.empty(cap, dtype=torch.uint8, device=self.device)
        sc = self._split_scratch
        N.check(N.lib.akv_match_prefix_split(
            self.view(runs), tokens.data_ptr(), q_off.data_ptr(), nq, block_size, out_node.data_ptr(),
            out_len.data_ptr(), out_c, ordp, plan.starts_ptr, plan.n_ranges, plan.tokens_per_range,
            sc.data_ptr(), sc.numel(), chunks, st, stream_handle(self.device)))

    def check(self) -> None:
        s = self.status.cpu()
        if int(s[0]) != 0:
            self.status.zero_()
            raise RuntimeError(
                f"agentkv_b200 tree replica error: {N.ERROR_NAMES.get(int(s[0]), int(s[0]))} "
                f"(query/update {int(s[1])}, node {int(s[2])})")


# ── split lookups ────────────────────────────────────────────────────────────
class SplitPlan:
    """Range plan of a split lookup (akv_match_prefix_split): range j of a
    query covers its positions [j R, (j + 1) R); with the queries launched
    longest first, range j exists for the first n_j ranks, and starts[j] is
    the first warp of range j.  Computed on the host from the lengths."""

    __slots__ = ("starts", "n_ranges", "tokens_per_range", "_c_starts")

    def __init__(self, starts: np.ndarray, tokens_per_range: int) -> None:
        self.starts = np.ascontiguousarray(starts, np.int64)
        self.n_ranges = len(self.starts) - 1
        self.tokens_per_range = int(tokens_per_range)
        self._c_starts = self.starts  # kept alive for the pointer below

    @property
    def starts_ptr(self) -> int:
        return self._c_starts.ctypes.data

    @property
    def n_items(self) -> int:
        return int(self.starts[-1])

    def scratch_bytes(self, nq: int) -> int:
        b = 16 * self.n_items + 4 * nq
        return (b + 255) // 256 * 256


SPLIT_DEFAULT_TOKENS = 1024  # the library's default range


def split_plan(lengths_in_order, tokens_per_range: int = 0) -> SplitPlan:
    """The range plan for queries of these lengths, given in launch order
    (longest first).  Ranges are tokens_per_range tokens (0 = 1024), longer
    (a multiple of 32) where the longest query would need more than
    MATCH_MAX_RANGES of them."""
    lens = np.asarray(lengths_in_order, np.int64)
    if len(lens) and np.any(np.diff(lens) > 0):
        raise ValueError("split_plan: lengths must be in longest-first order")
    R = int(tokens_per_range) or SPLIT_DEFAULT_TOKENS
    if R < 32 or R % 32:
        raise ValueError(f"split_plan: tokens_per_range={tokens_per_range} is not a multiple of 32")
    lmax = int(lens[0]) if len(lens) else 0
    if -(-lmax // R) > N.MATCH_MAX_RANGES:
        R = -(-lmax // N.MATCH_MAX_RANGES)
        R = -(-R // 32) * 32
    k = max(1, -(-lmax // R))
    # n_j = queries longer than j R (every query for j = 0)
    desc = -lens  # ascending
    n = [len(lens)] + [int(np.searchsorted(desc, -j * R, side="left")) for j in range(1, k)]
    starts = np.zeros(k + 1, np.int64)
    np.cumsum(n, out=starts[1:])
    return SplitPlan(starts, R)


# ── batched lookups on any tree replica ───────────────────────────────────────
def pack_queries(queries: Sequence, device: torch.device) -> Tuple[torch.Tensor, torch.Tensor]:
    """Concatenate token sequences into device (tokens int32, offsets int64)."""
    lens = np.fromiter((len(q) for q in queries), np.int64, len(queries))
    q_off = np.zeros(len(queries) + 1, np.int64)
    np.cumsum(lens, out=q_off[1:])
    flat = np.zeros(max(int(q_off[-1]), 1), np.int32)
    if int(q_off[-1]):
        np.concatenate([np.asarray(q, np.int32) for q in queries], out=flat[: int(q_off[-1])])
    return _upload(flat, device), _upload(q_off, device)


_GATHER_THREADS = max(1, min(8, os.cpu_count() or 1))


def _i32(q) -> np.ndarray:
    """A query as a contiguous int32 array (lists via array('i'), about twice
    as fast as numpy's conversion)."""
    if isinstance(q, list):
        return np.frombuffer(array("i", q), dtype=np.int32)
    return np.ascontiguousarray(q, dtype=np.int32).reshape(-1)


class QueryStage:
    """Reusable buffers for packing lookup batches: host buffers (pinned on a
    GPU, so the uploads are asynchronous) and device buffers that grow with
    the largest batch seen.  Fresh host memory is not free — first-touch page
    faults on a new 70 MB token buffer cost more than the lookup itself — so
    after the first batches nothing is allocated.  A batch's buffers are
    reused by the next pack(): the caller finishes the lookup (reads its
    results) first, as match_batch does."""

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self._tok_cap = self._q_cap = 0
        self.total = 0
        self.lens_in_order = np.zeros(0, np.int64)

    def _grow(self, total: int, nq: int) -> None:
        pin = self.device.type == "cuda"
        if total > self._tok_cap:
            # with headroom: batches of one workload vary in size, and a
            # regrown pinned buffer costs tens of milliseconds
            cap = max(total + total // 4, self._tok_cap + self._tok_cap // 2, 1 << 16)
            self.h_tok = torch.empty(cap, dtype=torch.int32, pin_memory=pin)
            self.d_tok = torch.empty(cap, dtype=torch.int32, device=self.device)
            self._tok_cap = cap
        if nq + 1 > self._q_cap:
            cap = max(nq + 1, self._q_cap + self._q_cap // 2, 1024)
            self.h_off = torch.empty(cap, dtype=torch.int64, pin_memory=pin)
            self.h_ord = torch.empty(cap, dtype=torch.int32, pin_memory=pin)
            self.d_off = torch.empty(cap, dtype=torch.int64, device=self.device)
            self.d_ord = torch.empty(cap, dtype=torch.int32, device=self.device)
            self._q_cap = cap

    def pack(self, queries: Sequence) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(tokens int32, offsets int64, longest-first order int32) on the
        device, enqueued on the current stream."""
        nq = len(queries)
        # Every query's address and length: int32 buffers (numpy arrays,
        # array('i')) are read in one C loop; anything else (lists, other
        # dtypes) is converted here and kept alive until the gather is done.
        ptrs = np.empty(nq, np.uint64)
        lens = np.empty(nq, np.int64)
        converted = []
        i = 0
        while i < nq:
            i = _pyhost.token_arrays(queries, i, ptrs, lens)
            if i < nq:
                a = _i32(queries[i])
                converted.append(a)
                ptrs[i] = a.ctypes.data if a.size else 0
                lens[i] = a.size
                i += 1
        total = int(lens.sum())
        self._grow(total, nq)
        off = self.h_off.numpy()[: nq + 1]
        off[0] = 0
        np.cumsum(lens, out=off[1:])
        # One C call gathers the queries into the pinned buffer with several
        # host threads and enqueues the upload (a single-threaded
        # np.concatenate of a 73 MB batch took 14 ms on the GPU hosts).
        if total:
            cuda = self.device.type == "cuda"
            N.check(N.lib.akv_gather_upload(ptrs.ctypes.data, lens.ctypes.data, nq, self.h_tok.data_ptr(),
                                            self.d_tok.data_ptr() if cuda else None, _GATHER_THREADS,
                                            stream_handle(self.device) if cuda else None))
            if not cuda:
                self.d_tok[:total].copy_(self.h_tok[:total])
        order = np.argsort(-lens, kind="stable")
        self.h_ord.numpy()[:nq] = order
        self.lens_in_order = lens[order]
        self.d_off[: nq + 1].copy_(self.h_off[: nq + 1], non_blocking=True)
        self.d_ord[:nq].copy_(self.h_ord[:nq], non_blocking=True)
        self.total = total
        return self.d_tok[: max(total, 1)], self.d_off[: nq + 1], self.d_ord[: max(nq, 1)]


class SingleLookup:
    """One query's lookup with one upload and one read-back: the query's
    offsets and tokens go up from one pinned buffer in one copy, and the
    answer comes back with its own status record in one copy.  For the
    single lookups of create_root and match_prefix."""

    def __init__(self, tree: "DeviceTree") -> None:
        self.tree = tree
        dev = tree.device
        self.io = torch.zeros(16, dtype=torch.int32, device=dev)  # status [0:8], node [8], length [9]
        self.h_io = torch.zeros(16, dtype=torch.int32, pin_memory=dev.type == "cuda")
        self.h_io_np = self.h_io.numpy()
        self._cap = 0

    def _grow(self, n: int) -> None:
        cap = max(4 + n, 2 * self._cap, 4096)
        pin = self.tree.device.type == "cuda"
        self.h = torch.zeros(cap, dtype=torch.int32, pin_memory=pin)
        self.h_np = self.h.numpy()
        self.d = torch.zeros(cap, dtype=torch.int32, device=self.tree.device)
        self._cap = cap

    def run(self, tokens: np.ndarray, block_size: int, chunks: int = 0) -> Tuple[int, int]:
        n = len(tokens)
        if 4 + n > self._cap:
            self._grow(n)
        self.h_np[:4].view(np.int64)[:] = (0, n)  # q_off = [0, n]
        self.h_np[4 : 4 + n] = tokens
        cuda = self.tree.device.type == "cuda"
        stream = stream_handle(self.tree.device) if cuda else 0
        if cuda:
            N.check(N.lib.akv_copy_wait(self.d.data_ptr(), self.h.data_ptr(), 4 * (4 + n), 0, 0, stream))
        else:
            self.d[: 4 + n].copy_(self.h[: 4 + n])
        self.tree.match(self.d[4:], self.d[:4].view(torch.int64), 1, block_size, self.io[8:9], self.io[9:10],
                        None, chunks=chunks, status=self.io[0:8])
        if cuda:
            N.check(N.lib.akv_copy_wait(self.h_io.data_ptr(), self.io.data_ptr(), 4 * 16, 1, 1, stream))
        else:
            self.h_io.copy_(self.io)
        io = self.h_io_np
        if int(io[0]) != 0:
            code, index, node = int(io[0]), int(io[1]), int(io[2])
            self.io[0:8].zero_()
            raise RuntimeError(f"agentkv_b200 tree replica error: {N.ERROR_NAMES.get(code, code)} "
                               f"(query/update {index}, node {node})")
        return int(io[8]), int(io[9])


def _upload(a: np.ndarray, device: torch.device) -> torch.Tensor:
    # through pinned memory (an asynchronous copy) when the target is a GPU
    t = torch.from_numpy(a)
    if device.type == "cuda":
        t = t.pin_memory()
    return t.to(device, non_blocking=True)


def longest_first(q_off, device: torch.device) -> torch.Tensor:
    """Launch order for akv_match_prefix: query indices by decreasing length
    (stable), so the longest walks start first and spread over the SMs."""
    q_off = np.asarray(q_off.cpu() if isinstance(q_off, torch.Tensor) else q_off, np.int64)
    order = np.argsort(-np.diff(q_off), kind="stable").astype(np.int32)
    return _upload(order, device)


def match_batch(tree: DeviceTree, queries: Sequence, block_size: int, *, with_compared: bool = False,
                runs: Optional[bool] = None, tokens_per_range: int = 0, split: bool = False,
                chunks: int = 0, staged: bool = False, window_tokens: int = 0):
    """Longest shared prefix of many queries in one akv_match_prefix launch on
    `tree` (the owner's replica or another GPU's): (node ids, match lengths
    [, tokens compared]) as numpy arrays, each equal to the reference's
    _match_prefix_locked (agentkv/core/radix_tree.py:513-570) on that query.
    runs=True follows the unary-chain runs (rebuilt first when stale),
    runs=False takes one hash probe per hop, None lets the tree decide
    (DeviceTree.want_runs); the answers are the same.  The lookup splits
    long queries into ranges of tokens_per_range tokens (0 = the library's
    default; see DeviceTree.match) when split=True; by default one warp
    walks each query (measured faster on the match stress workload).
    chunks: 32-token chunks compared per verify step (0 = the kernel's
    default), optionally with N.MATCH_PIPELINED / N.MATCH_PREFETCH.
    staged=True: the two-launch lookup (DeviceTree.match) with windows of
    window_tokens tokens."""
    t0 = time.perf_counter()
    if runs is None:
        runs = tree.want_runs()
    dev = tree.device
    nq = len(queries)
    if tree._stage is None:
        tree._stage = QueryStage(dev)
    tok, q_off, order = tree._stage.pack(queries)
    node = torch.empty(max(nq, 1), dtype=torch.int32, device=dev)
    mlen = torch.empty(max(nq, 1), dtype=torch.int32, device=dev)
    cmp_ = torch.empty(max(nq, 1), dtype=torch.int64, device=dev) if with_compared else None
    plan = split_plan(tree._stage.lens_in_order, tokens_per_range) if (split and nq) else None
    tree.match(tok, q_off, nq, block_size, node, mlen, cmp_, order=order, runs=runs, chunks=chunks, plan=plan,
               staged=staged, window_tokens=window_tokens, n_tokens=tree._stage.total)
    tree.check()
    res = (node[:nq].cpu().numpy(), mlen[:nq].cpu().numpy())
    if with_compared:
        res = res + (cmp_[:nq].cpu().numpy(),)
    tree.note_lookup((time.perf_counter() - t0) * 1e3, runs)
    return res
