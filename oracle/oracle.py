"""Oracle for the AgentKV hot path — TEST INFRASTRUCTURE ONLY.

A CPU restatement of the reference's algorithms, used by ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` to check
results and to time the reference algorithm on the host.  The
``agentkv_b200`` package never imports it.

* ``OracleAllocator`` wraps the C restatement of SlabAllocator +
  EpochReclaimer (``akv_oracle.c``; agentkv/core/slab_allocator.py:155-437,
  agentkv/core/reclamation.py:87-173).
* ``OracleTree`` restates DualRadixTree's tree logic in plain Python
  (agentkv/core/radix_tree.py:185-717): create_root / fork / allocate_block /
  ensure_mutable_block / commit_prefix / free / match_prefix /
  get_block_ids and the edge-split insert with its quirks.
* ``tree_csr`` flattens an OracleTree into sorted-children CSR arrays and
  ``match_prefix_csr`` runs the C restatement of _match_prefix_locked
  (radix_tree.py:513-570) over them.

Parity of this oracle is pinned against fixtures generated from the reference
itself (tests/golden/make_golden.py).
"""

from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path
from typing import Dict, List, Optional, Tuple

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "libakv_oracle.so"

ORC_OK = 0
ORC_ERR_OUT_OF_RANGE = 2
ORC_ERR_EXHAUSTED = 3
ORC_ERR_DOUBLE_FREE = 4
ORC_ERR_NOT_ALLOCATED = 5

ROOT_NODE_ID = 0
INVALID_NODE_ID = -1


def build(force: bool = False) -> Path:
    """Compile akv_oracle.c with the Makefile beside it."""
    src = ORACLE_DIR / "akv_oracle.c"
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "-B" if force else "all"], check=True)
    return LIB_PATH


def _load() -> C.CDLL:
    build()
    lib = C.CDLL(str(LIB_PATH))
    P, I32, I64 = C.c_void_p, C.c_int32, C.c_int64
    sig = {
        "orc_copy_blocks": (None, [P, I64, P, I32]),
        "orc_copy_blocks_mt": (None, [P, I64, P, I32, C.c_int]),
        "orc_zero_blocks": (None, [P, I64, P, I32]),
        "orc_zero_blocks_mt": (None, [P, I64, P, I32, C.c_int]),
        "orc_alloc_new": (P, [I32, I32]),
        "orc_alloc_delete": (None, [P]),
        "orc_alloc_clone": (P, [P]),
        "orc_alloc_one": (I32, [P]),
        "orc_incref": (C.c_int, [P, I32]),
        "orc_decref": (C.c_int, [P, I32, P]),
        "orc_enter_read": (I64, [P]),
        "orc_leave_read": (None, [P, I64]),
        "orc_maybe_advance": (None, [P]),
        "orc_alloc_state": (None, [P, P, P, P]),
        "orc_ref_count": (C.c_int32, [P, C.c_int32]),
        "orc_alloc_limbo": (None, [P, P, P, P]),
        "orc_alloc_seq": (I32, [P, I32, P]),
        "orc_incref_seq": (I32, [P, P, I32]),
        "orc_decref_seq": (I32, [P, P, I32]),
        "orc_alloc_batch": (C.c_int, [P, I32, P, P]),
        "orc_incref_batch": (C.c_int, [P, P, I32, P]),
        "orc_decref_batch": (C.c_int, [P, P, I32, P, P, P]),
        "orc_cow_batch": (C.c_int, [P, P, I64, P, I32, P, P, P]),
        "orc_match_prefix": (None, [P, P, P, P, P, P, P, P, I32, I32, P, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# ── block movement ───────────────────────────────────────────────────────────
def copy_blocks(pool: np.ndarray, bytes_per_block: int, pairs: np.ndarray, threads: int = 1) -> None:
    """Sequential dst.copy_(src) per (src, dst) pair on a host byte pool."""
    pairs = np.ascontiguousarray(pairs, dtype=np.int32).reshape(-1, 2)
    if threads > 1:
        lib.orc_copy_blocks_mt(_ptr(pool), bytes_per_block, _ptr(pairs), len(pairs), threads)
    else:
        lib.orc_copy_blocks(_ptr(pool), bytes_per_block, _ptr(pairs), len(pairs))


def zero_blocks(pool: np.ndarray, bytes_per_block: int, ids: np.ndarray, threads: int = 1) -> None:
    """block.zero_() per id: +0.0 in every element."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    if threads > 1:
        lib.orc_zero_blocks_mt(_ptr(pool), bytes_per_block, _ptr(ids), len(ids), threads)
    else:
        lib.orc_zero_blocks(_ptr(pool), bytes_per_block, _ptr(ids), len(ids))


# ── allocator ────────────────────────────────────────────────────────────────
class OracleError(Exception):
    def __init__(self, code: int, index: int = 0) -> None:
        super().__init__(code, index)
        self.code = code
        self.index = index


class OracleAllocator:
    """SlabAllocator + EpochReclaimer restated in C; ids are plain ints."""

    def __init__(self, total_blocks: int, epoch_interval: int = 64) -> None:
        self.n = total_blocks
        self._h = lib.orc_alloc_new(total_blocks, epoch_interval)

    def __del__(self) -> None:
        h, self._h = getattr(self, "_h", None), None
        if h:
            lib.orc_alloc_delete(h)

    # single ops, reference semantics (error = nothing changed)
    def alloc(self) -> int:
        r = lib.orc_alloc_one(self._h)
        if r < 0:
            raise OracleError(-r)
        return int(r)

    def inc_ref(self, bid: int) -> None:
        rc = lib.orc_incref(self._h, bid)
        if rc:
            raise OracleError(rc)

    def dec_ref(self, bid: int) -> bool:
        r = C.c_int32(0)
        rc = lib.orc_decref(self._h, bid, C.addressof(r))
        if rc:
            raise OracleError(rc)
        return bool(r.value)

    def enter_read_section(self) -> int:
        return int(lib.orc_enter_read(self._h))

    def leave_read_section(self, token: int) -> None:
        lib.orc_leave_read(self._h, token)

    def maybe_advance_epoch(self) -> None:
        lib.orc_maybe_advance(self._h)

    # sequential runs: the reference's single calls in a loop (no rollback)
    def alloc_seq(self, n: int) -> np.ndarray:
        out = np.zeros(max(n, 1), np.int32)
        done = lib.orc_alloc_seq(self._h, n, _ptr(out))
        if done != n:
            raise OracleError(ORC_ERR_EXHAUSTED, done)
        return out[:n]

    def inc_ref_seq(self, ids: np.ndarray) -> None:
        ids = np.ascontiguousarray(ids, np.int32)
        done = lib.orc_incref_seq(self._h, _ptr(ids), len(ids))
        if done != len(ids):
            raise OracleError(ORC_ERR_NOT_ALLOCATED, done)

    def dec_ref_seq(self, ids: np.ndarray) -> None:
        ids = np.ascontiguousarray(ids, np.int32)
        done = lib.orc_decref_seq(self._h, _ptr(ids), len(ids))
        if done != len(ids):
            raise OracleError(ORC_ERR_DOUBLE_FREE, done)

    # all-or-nothing batches
    def alloc_batch(self, n: int) -> np.ndarray:
        out = np.zeros(max(n, 1), np.int32)
        fi = C.c_int32(0)
        rc = lib.orc_alloc_batch(self._h, n, _ptr(out), C.addressof(fi))
        if rc:
            raise OracleError(rc, fi.value)
        return out[:n]

    def inc_ref_batch(self, ids) -> None:
        ids = np.ascontiguousarray(ids, np.int32)
        fi = C.c_int32(0)
        rc = lib.orc_incref_batch(self._h, _ptr(ids), len(ids), C.addressof(fi))
        if rc:
            raise OracleError(rc, fi.value)

    def dec_ref_batch(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.zeros(max(len(ids), 1), np.int32)
        nr, fi = C.c_int32(0), C.c_int32(0)
        rc = lib.orc_decref_batch(self._h, _ptr(ids), len(ids), _ptr(out), C.addressof(nr), C.addressof(fi))
        if rc:
            raise OracleError(rc, fi.value)
        return out[: nr.value]

    def cow_batch(self, blocks, pool: Optional[np.ndarray] = None, bytes_per_block: int = 0):
        blocks = np.ascontiguousarray(blocks, np.int32)
        n = len(blocks)
        ob = np.zeros(max(n, 1), np.int32)
        oc = np.zeros(max(n, 1), np.int32)
        fi = C.c_int32(0)
        rc = lib.orc_cow_batch(
            self._h, _ptr(pool) if pool is not None else None, bytes_per_block, _ptr(blocks), n,
            _ptr(ob), _ptr(oc), C.addressof(fi),
        )
        if rc:
            raise OracleError(rc, fi.value)
        return ob[:n], oc[:n]

    # state
    def state(self) -> dict:
        ref = np.zeros(self.n, np.int32)
        free = np.zeros(self.n, np.int32)
        ctl = np.zeros(16, np.int64)
        lib.orc_alloc_state(self._h, _ptr(ref), _ptr(free), _ptr(ctl))
        pend = np.zeros(self.n, np.int32)
        pend_ep = np.zeros(self.n, np.int64)
        defer = np.zeros(self.n, np.int32)
        lib.orc_alloc_limbo(self._h, _ptr(pend), _ptr(pend_ep), _ptr(defer))
        return {
            "ref_counts": ref,
            "free_list": free[: ctl[0]].copy(),
            "pending": pend[: ctl[1]].copy(),
            "pending_epochs": pend_ep[: ctl[1]].copy(),
            "deferred": defer[: ctl[2]].copy(),
            "op_count": int(ctl[3]),
            "epoch": int(ctl[4]),
            "total_allocs": int(ctl[5]),
            "total_frees": int(ctl[6]),
            "peak_allocated": int(ctl[7]),
            "epoch_advances": int(ctl[8]),
            "blocks_freed": int(ctl[9]),
            "allocated_blocks": int(ctl[10]),
        }

    def ref_count(self, bid: int) -> int:
        return int(lib.orc_ref_count(self._h, bid))

    @property
    def free_count(self) -> int:
        ctl = np.zeros(16, np.int64)
        lib.orc_alloc_state(self._h, None, None, _ptr(ctl))
        return int(ctl[0])


# ── tree ─────────────────────────────────────────────────────────────────────
class _Node:
    __slots__ = ("node_id", "parent_id", "edge", "blocks", "children", "ref_count")

    def __init__(self, node_id, parent_id, edge, blocks, ref_count=0):
        self.node_id = node_id
        self.parent_id = parent_id
        self.edge = edge
        self.blocks = blocks
        self.children: Dict[int, int] = {}
        self.ref_count = ref_count


class _Handle:
    __slots__ = ("handle_id", "shared_node_id", "shared_match_len", "residual", "tokens", "freed")

    def __init__(self, hid, node, mlen, residual, tokens):
        self.handle_id = hid
        self.shared_node_id = node
        self.shared_match_len = mlen
        self.residual: List[int] = residual
        self.tokens: List[int] = tokens
        self.freed = False


class OracleTree:
    """DualRadixTree restated over OracleAllocator (radix_tree.py:138-717)."""

    def __init__(self, alloc: OracleAllocator, block_size: int, copy_cb=None) -> None:
        self.alloc = alloc
        self.bs = block_size
        self.nodes: Dict[int, _Node] = {ROOT_NODE_ID: _Node(ROOT_NODE_ID, INVALID_NODE_ID, [], [])}
        self.next_node = 1
        self.handles: Dict[int, _Handle] = {}
        self.next_handle = 0
        # Called as copy_cb(src, dst) for each CoW copy (the data movement).
        self.copy_cb = copy_cb

    # radix_tree.py:185-220
    def create_root(self, tokens: List[int]) -> _Handle:
        node, mlen = self.match(tokens)[:2]
        h = _Handle(self.next_handle, node, mlen, [], list(tokens))
        self.next_handle += 1
        if node != INVALID_NODE_ID:
            self._inc_shared(node)
        self.handles[h.handle_id] = h
        return h

    # radix_tree.py:222-264
    def fork(self, parent: _Handle) -> _Handle:
        self._check(parent)
        for b in parent.residual:
            self.alloc.inc_ref(b)
        if parent.shared_node_id != INVALID_NODE_ID:
            self._inc_shared(parent.shared_node_id)
        c = _Handle(self.next_handle, parent.shared_node_id, parent.shared_match_len,
                    list(parent.residual), list(parent.tokens))
        self.next_handle += 1
        self.handles[c.handle_id] = c
        return c

    # radix_tree.py:266-284
    def allocate_block(self, h: _Handle) -> int:
        self._check(h)
        b = self.alloc.alloc()
        h.residual.append(b)
        return b

    # radix_tree.py:286-314
    def ensure_mutable_block(self, h: _Handle, idx: int) -> int:
        self._check(h)
        b = h.residual[idx]
        if self.alloc.ref_count(b) > 1:
            nb = self.alloc.alloc()
            if self.copy_cb is not None:
                self.copy_cb(b, nb)
            self.alloc.dec_ref(b)
            h.residual[idx] = nb
            return nb
        return b

    # radix_tree.py:336-349
    def append_tokens(self, h: _Handle, toks: List[int]) -> None:
        self._check(h)
        h.tokens.extend(toks)

    # radix_tree.py:351-377
    def free(self, h: _Handle) -> None:
        self._check(h)
        for b in h.residual:
            self.alloc.dec_ref(b)
        h.residual.clear()
        if h.shared_node_id != INVALID_NODE_ID:
            self._dec_shared(h.shared_node_id)
        h.freed = True
        del self.handles[h.handle_id]

    # radix_tree.py:379-416 (returns the handle or None, and the length)
    def match_prefix(self, tokens: List[int]) -> Tuple[Optional[_Handle], int]:
        tok = self.alloc.enter_read_section()
        try:
            node, mlen = self.match(tokens)[:2]
            if node == INVALID_NODE_ID or mlen == 0:
                return None, 0
            self._inc_shared(node)
            h = _Handle(self.next_handle, node, mlen, [], list(tokens[:mlen]))
            self.next_handle += 1
            self.handles[h.handle_id] = h
            return h, mlen
        finally:
            self.alloc.leave_read_section(tok)

    # radix_tree.py:418-468
    def commit_prefix(self, h: _Handle, length: int) -> None:
        self._check(h)
        if length % self.bs != 0:
            raise ValueError("length must be a multiple of block_size")
        nb = length // self.bs
        if nb > len(h.residual):
            raise ValueError("requested more blocks than the agent has")
        ptoks = h.tokens[h.shared_match_len:][:length]
        pblocks = h.residual[:nb]
        parent = h.shared_node_id if h.shared_node_id != INVALID_NODE_ID else ROOT_NODE_ID
        new_id = self._insert(parent, ptoks, pblocks)
        h.residual = h.residual[nb:]
        h.shared_node_id = new_id
        h.shared_match_len += length
        self._inc_shared(new_id)

    # radix_tree.py:470-496
    def get_block_ids(self, h: _Handle) -> List[int]:
        self._check(h)
        ids: List[int] = []
        if h.shared_node_id != INVALID_NODE_ID:
            chain = []
            nid = h.shared_node_id
            while nid != INVALID_NODE_ID and nid in self.nodes:
                chain.append(self.nodes[nid])
                nid = self.nodes[nid].parent_id
                if nid == ROOT_NODE_ID:
                    break
            for node in reversed(chain):
                ids.extend(node.blocks)
        ids.extend(h.residual)
        return ids

    # radix_tree.py:513-570, with the comparison count
    def match(self, tokens: List[int]) -> Tuple[int, int, int]:
        cur, matched, compared = ROOT_NODE_ID, 0, 0
        n = len(tokens)
        while matched < n:
            node = self.nodes[cur]
            child_id = node.children.get(tokens[matched])
            if child_id is None:
                break
            edge = self.nodes[child_id].edge
            em = 0
            for i, et in enumerate(edge):
                if matched + i >= n:
                    break
                compared += 1
                if tokens[matched + i] != et:
                    break
                em += 1
            if em == 0 or em < len(edge):
                break
            matched += em
            cur = child_id
        matched = (matched // self.bs) * self.bs
        if matched == 0:
            return INVALID_NODE_ID, 0, compared
        return cur, matched, compared

    # radix_tree.py:572-686
    def _insert(self, parent_id: int, tokens: List[int], blocks: List[int]) -> int:
        if not tokens:
            return parent_id
        parent = self.nodes[parent_id]
        first = tokens[0]
        if first not in parent.children:
            nid = self._new_node(parent_id, list(tokens), list(blocks), 0)
            parent.children[first] = nid
            return nid
        cid = parent.children[first]
        child = self.nodes[cid]
        edge = child.edge
        m = min(len(edge), len(tokens))
        common = 0
        while common < m and edge[common] == tokens[common]:
            common += 1
        if common == len(edge) and common == len(tokens):
            child.blocks = list(blocks)  # exact re-commit: no dec_ref of the old blocks
            return cid
        if common == len(edge):
            return self._insert(cid, tokens[common:], blocks[common // self.bs:])
        split = (common // self.bs) * self.bs
        if split == 0:
            nid = self._new_node(parent_id, list(tokens), list(blocks), 0)
            parent.children[first] = nid  # overwrites (orphans) the old sibling
            return nid
        sb = split // self.bs
        mid = self._new_node(parent_id, list(edge[:split]), list(child.blocks[:sb]), child.ref_count)
        child.parent_id = mid
        child.edge = list(edge[split:])
        child.blocks = list(child.blocks[sb:])
        self.nodes[mid].children[child.edge[0]] = cid
        parent.children[first] = mid
        if split == len(tokens):
            return mid
        nid = self._new_node(mid, list(tokens[split:]), list(blocks[sb:]), 0)
        self.nodes[mid].children[tokens[split]] = nid
        return nid

    def _new_node(self, parent_id, edge, blocks, ref_count) -> int:
        nid = self.next_node
        self.next_node += 1
        self.nodes[nid] = _Node(nid, parent_id, edge, blocks, ref_count)
        return nid

    # radix_tree.py:688-693
    def _inc_shared(self, nid: int) -> None:
        while nid != INVALID_NODE_ID and nid in self.nodes:
            self.nodes[nid].ref_count += 1
            nid = self.nodes[nid].parent_id

    # radix_tree.py:695-717
    def _dec_shared(self, nid: int) -> None:
        while nid != INVALID_NODE_ID and nid in self.nodes:
            node = self.nodes[nid]
            node.ref_count -= 1
            if node.ref_count <= 0 and nid != ROOT_NODE_ID and not node.children:
                for b in node.blocks:
                    self.alloc.dec_ref(b)
                pid = node.parent_id
                if pid in self.nodes:
                    p = self.nodes[pid]
                    p.children = {k: v for k, v in p.children.items() if v != nid}
                del self.nodes[nid]
                nid = pid
            else:
                nid = self.nodes[nid].parent_id

    def _check(self, h: _Handle) -> None:
        if h.handle_id not in self.handles or h.freed:
            raise ValueError(f"NodeHandle {h.handle_id} is not registered")


# ── CSR flattening + C match ─────────────────────────────────────────────────
def tree_csr(tree: OracleTree) -> dict:
    """Sorted-children CSR over node ids 0..max_id (absent ids have no
    children and an empty edge)."""
    max_id = max(tree.nodes) if tree.nodes else 0
    n = max_id + 1
    child_ptr = np.zeros(n + 1, np.int64)
    keys: List[int] = []
    ids: List[int] = []
    edge_off = np.zeros(n, np.int64)
    edge_len = np.zeros(n, np.int32)
    toks: List[np.ndarray] = []
    pos = 0
    for nid in range(n):
        node = tree.nodes.get(nid)
        if node is not None:
            for k in sorted(node.children):
                keys.append(k)
                ids.append(node.children[k])
            edge_off[nid] = pos
            edge_len[nid] = len(node.edge)
            toks.append(np.asarray(node.edge, np.int32))
            pos += len(node.edge)
        child_ptr[nid + 1] = len(keys)
    return {
        "child_ptr": child_ptr,
        "child_key": np.asarray(keys, np.int32) if keys else np.zeros(1, np.int32),
        "child_id": np.asarray(ids, np.int32) if ids else np.zeros(1, np.int32),
        "edge_off": edge_off,
        "edge_len": edge_len,
        "edge_tokens": np.concatenate(toks) if pos else np.zeros(1, np.int32),
    }


def pack_queries(queries: List[List[int]]) -> Tuple[np.ndarray, np.ndarray]:
    lens = np.array([len(q) for q in queries], np.int64)
    q_off = np.zeros(len(queries) + 1, np.int64)
    np.cumsum(lens, out=q_off[1:])
    flat = np.concatenate([np.asarray(q, np.int32) for q in queries]) if q_off[-1] else np.zeros(1, np.int32)
    return flat, q_off


def match_prefix_csr(csr: dict, tokens: np.ndarray, q_off: np.ndarray, block_size: int):
    """(node, len, compared) per query, restating _match_prefix_locked."""
    nq = len(q_off) - 1
    node = np.zeros(max(nq, 1), np.int32)
    mlen = np.zeros(max(nq, 1), np.int32)
    cmp_ = np.zeros(max(nq, 1), np.int64)
    tokens = np.ascontiguousarray(tokens, np.int32)
    q_off = np.ascontiguousarray(q_off, np.int64)
    lib.orc_match_prefix(
        _ptr(csr["child_ptr"]), _ptr(csr["child_key"]), _ptr(csr["child_id"]), _ptr(csr["edge_off"]),
        _ptr(csr["edge_len"]), _ptr(csr["edge_tokens"]), _ptr(tokens), _ptr(q_off), nq, block_size,
        _ptr(node), _ptr(mlen), _ptr(cmp_),
    )
    return node[:nq], mlen[:nq], cmp_[:nq]


class _Edges:
    """Node edges as Python lists, converted from the CSR arena when first
    walked (a large tree's arena as Python ints would take gigabytes)."""

    def __init__(self, csr: dict) -> None:
        self._off, self._len, self._tok = csr["edge_off"], csr["edge_len"], csr["edge_tokens"]
        self._lists: dict = {}

    def __getitem__(self, u: int) -> list:
        e = self._lists.get(u)
        if e is None:
            o = int(self._off[u])
            e = self._lists[u] = self._tok[o:o + int(self._len[u])].tolist()
        return e


def csr_children(csr: dict) -> list:
    """Per node, its children as a dict first token -> child id, and its edge
    as a Python list: the shapes the reference's loop walks
    (radix_tree.py:82-103)."""
    ptr, keys, ids = csr["child_ptr"], csr["child_key"], csr["child_id"]
    kids = [dict(zip(keys[ptr[u]:ptr[u + 1]].tolist(), ids[ptr[u]:ptr[u + 1]].tolist()))
            for u in range(len(ptr) - 1)]
    return [kids, _Edges(csr)]


def match_prefix_py(tree: list, queries, block_size: int):
    """(node, len, compared) per query by the reference's own loop in pure
    Python (radix_tree.py:513-570: child by first token, compare the edge token
    by token, stop at a mismatch or a partial edge, floor to the block size),
    over csr_children's tree — what the reference's CPU path costs per query."""
    kids, edges = tree
    out = []
    for q in queries:
        n = len(q)
        cur, matched, compared = 0, 0, 0
        while matched < n:
            child = kids[cur].get(q[matched])
            if child is None:
                break
            edge = edges[child]
            em = 0
            for i, et in enumerate(edge):
                if matched + i >= n:
                    break
                compared += 1
                if q[matched + i] != et:
                    break
                em += 1
            if em == 0 or em < len(edge):
                break
            matched += em
            cur = child
        m = (matched // block_size) * block_size
        out.append((cur if m else INVALID_NODE_ID, m, compared))
    return out


# ── HuggingFace cache (agentkv/hf_cache.py) ──────────────────────────────────
class OracleKVPool:
    """A pool's calls the HF cache uses — OracleTree over OracleAllocator plus
    a host array [N, L, 2, H, bs, D] standing for _kv_data (zero-filled, as
    slab_allocator.py:155-164 creates it); CoW copies move its rows."""

    def __init__(self, total_blocks, block_size, num_layers, num_kv_heads, head_dim, dtype) -> None:
        self.kv = np.zeros((total_blocks, num_layers, 2, num_kv_heads, block_size, head_dim), dtype)
        self.alloc = OracleAllocator(total_blocks)
        self.tree = OracleTree(self.alloc, block_size, copy_cb=self._copy)
        self.block_size = block_size
        self.num_layers = num_layers

    def _copy(self, src: int, dst: int) -> None:
        self.kv[dst] = self.kv[src]

    def __getattr__(self, name):
        return getattr(self.tree, name)


class OracleKVCache:
    """AgentKVCache restated (agentkv/hf_cache.py:38-185) on OracleKVPool."""

    def __init__(self, pool: OracleKVPool, handle: _Handle) -> None:
        self.pool = pool
        self.handle = handle
        self._seen_tokens = len(handle.tokens)
        self._next_seen_tokens = self._seen_tokens

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self._seen_tokens

    # hf_cache.py:57-160
    def update(self, key_states: np.ndarray, value_states: np.ndarray, layer_idx: int):
        if key_states.shape[0] != 1:
            raise ValueError("AgentKVCache requires batch_size=1")
        p, h, bs = self.pool, self.handle, self.pool.block_size
        n_new = key_states.shape[2]
        if layer_idx == 0:
            self._next_seen_tokens = self._seen_tokens + n_new
            required = (self._next_seen_tokens + bs - 1) // bs
            while len(p.tree.get_block_ids(h)) < required:
                p.tree.allocate_block(h)
            if len(h.tokens) < self._next_seen_tokens:
                p.tree.append_tokens(h, [0] * (self._next_seen_tokens - len(h.tokens)))
        for i in range(n_new):
            tok = self._seen_tokens + i
            blk, pos = tok // bs, tok % bs
            ridx = blk - h.shared_match_len // bs
            if ridx < 0:
                raise RuntimeError("Cannot overwrite shared prefix blocks!")
            if layer_idx == 0 and (i == 0 or pos == 0):
                p.tree.ensure_mutable_block(h, ridx)
            b = p.tree.get_block_ids(h)[blk]
            p.kv[b, layer_idx, 0, :, pos, :] = key_states[0, :, i, :]
            p.kv[b, layer_idx, 1, :, pos, :] = value_states[0, :, i, :]
        ids = p.tree.get_block_ids(h)
        data = p.kv[ids, layer_idx]  # [nb, 2, H, bs, D]
        H, D = data.shape[2], data.shape[4]
        out_k = data[:, 0].transpose(1, 0, 2, 3).reshape(1, H, -1, D)[:, :, : self._next_seen_tokens]
        out_v = data[:, 1].transpose(1, 0, 2, 3).reshape(1, H, -1, D)[:, :, : self._next_seen_tokens]
        if layer_idx == p.num_layers - 1:
            self._seen_tokens = self._next_seen_tokens
        return out_k, out_v

    # hf_cache.py:162-170
    def fork(self) -> "OracleKVCache":
        return OracleKVCache(self.pool, self.pool.tree.fork(self.handle))
