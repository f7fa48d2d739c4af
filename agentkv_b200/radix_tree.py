"""DualRadixTree — the copy-on-write radix tree over the device block pool.

Same API, handle types and semantics as the reference's DualRadixTree
(agentkv/core/radix_tree.py:138-746): create_root / fork / allocate_block /
ensure_mutable_block / free_block / append_tokens / free / match_prefix /
commit_prefix / get_block_ids / stats, including the reference's quirks
(a partially matched edge earns no credit, the match is floored to the block
size, an insert that diverges inside the first block overwrites the sibling
with the same first token, an exact re-commit replaces the node's blocks).

What moved to the GPU:
* every refcount change reaches the device allocator as one batch per tree
  operation (fork inc_refs all inherited blocks, free dec_refs the residual
  blocks and any pruned node blocks): answered at the call by the
  allocator's host mirror and replayed on the device from its op log, or
  launched directly on the device for batches of device ids;
* copy-on-write decides on the mirror (refcount test, alloc, dec_ref) and
  enqueues the block copies in one launch — unless the allocator's copy_block
  was replaced on the instance (the vLLM adapter records CoW pairs that way),
  in which case the reference's per-step sequence runs and calls that
  replacement;
* _match_prefix_locked is the akv_match_prefix kernel over the tree's device
  replica (device_tree.py), which every structural change keeps current.

Batched extensions for schedulers: ``allocate_blocks``, ``fork_many``,
``ensure_mutable_batch``, ``free_many`` and ``match_prefix_batch``.
"""

from __future__ import annotations

import threading
from array import array
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _native as N
from .allocator import BlockHandle, SlabAllocator
from .config import PoolConfig
from .device_tree import (DeviceTree, QueryStage, SingleLookup, longest_first, match_batch,  # noqa: F401
                          pack_queries, split_plan)

ROOT_NODE_ID: int = 0
INVALID_NODE_ID: int = -1


class SharedNode:
    """A node of the shared tree (radix_tree.py:81-103).  Its edge is a range
    of the device replica's token arena."""

    __slots__ = ("node_id", "parent_id", "edge_off", "edge_len", "blocks", "children", "ref_count",
                 "_arena")

    def __init__(self, node_id: int, parent_id: int, arena: DeviceTree, edge_off: int = 0,
                 edge_len: int = 0, blocks: Optional[List[BlockHandle]] = None, ref_count: int = 0):
        self.node_id = node_id
        self.parent_id = parent_id
        self._arena = arena
        self.edge_off = edge_off
        self.edge_len = edge_len
        self.blocks: List[BlockHandle] = blocks if blocks is not None else []
        self.children: Dict[int, int] = {}
        self.ref_count = ref_count

    @property
    def edge(self) -> np.ndarray:
        return self._arena.edge(self.edge_off, self.edge_len)

    @property
    def edge_tokens(self) -> List[int]:
        return self.edge.tolist()

    def __repr__(self) -> str:
        return (f"SharedNode(id={self.node_id}, parent={self.parent_id}, edge_len={self.edge_len}, "
                f"blocks={len(self.blocks)}, children={len(self.children)}, ref={self.ref_count})")


@dataclass
class NodeHandle:
    """Per-agent state (radix_tree.py:108-133)."""

    handle_id: int
    shared_node_id: int
    shared_match_len: int
    residual_blocks: List[BlockHandle] = field(default_factory=list)
    tokens: List[int] = field(default_factory=list)
    ref_count: int = 1
    is_freed: bool = False

    def __repr__(self) -> str:
        return (
            f"NodeHandle(id={self.handle_id}, shared_node={self.shared_node_id}, "
            f"shared_len={self.shared_match_len}, residual_blocks={len(self.residual_blocks)}, "
            f"tokens={len(self.tokens)})"
        )


def _as_i32(tokens) -> np.ndarray:
    if isinstance(tokens, list):
        # array('i') converts a list of ints about twice as fast as numpy
        return np.frombuffer(array("i", tokens), dtype=np.int32)
    return np.asarray(tokens, dtype=np.int32).reshape(-1)


def _lcp(a: np.ndarray, b: np.ndarray) -> int:
    m = min(len(a), len(b))
    if m == 0:
        return 0
    neq = np.flatnonzero(a[:m] != b[:m])
    return int(neq[0]) if len(neq) else m


class DualRadixTree:
    """Copy-on-write radix tree KV cache manager; see the module docstring."""

    def __init__(self, allocator: SlabAllocator, config: PoolConfig) -> None:
        self._alloc = allocator
        self._cfg = config
        self._lock = threading.RLock()
        self._dev_tree = DeviceTree(allocator.device)
        self._shared_nodes: Dict[int, SharedNode] = {
            ROOT_NODE_ID: SharedNode(ROOT_NODE_ID, INVALID_NODE_ID, self._dev_tree)
        }
        self._dev_tree.set_node(ROOT_NODE_ID, 0, 0)
        self._next_node_id: int = 1
        self._handles: Dict[int, NodeHandle] = {}
        self._next_handle_id: int = 0
        # get_block_ids results per handle, valid while nothing changed:
        # every mutating call bumps _version
        self._version = 0
        self._ids_cache: Dict[int, Tuple[tuple, List[int]]] = {}
        dev = allocator.device
        self._one = SingleLookup(self._dev_tree)  # single lookups (create_root, match_prefix)

    # ── create / fork / allocate ──────────────────────────────────────────────
    def create_root(self, tokens: List[int]) -> NodeHandle:
        with self._lock:
            self._version += 1
            shared_node_id, match_len = self._match_prefix_locked(tokens)
            handle = NodeHandle(
                handle_id=self._next_handle_id,
                shared_node_id=shared_node_id,
                shared_match_len=match_len,
                residual_blocks=[],
                tokens=list(tokens),
                ref_count=1,
            )
            self._next_handle_id += 1
            if shared_node_id != INVALID_NODE_ID:
                self._inc_shared_ref_locked(shared_node_id)
            self._handles[handle.handle_id] = handle
            return handle

    def fork(self, parent: NodeHandle) -> NodeHandle:
        with self._lock:
            self._version += 1
            self._validate_handle_locked(parent)
            if parent.residual_blocks:
                self._alloc.inc_ref_batch([b.block_id for b in parent.residual_blocks])
            if parent.shared_node_id != INVALID_NODE_ID:
                self._inc_shared_ref_locked(parent.shared_node_id)
            child = NodeHandle(
                handle_id=self._next_handle_id,
                shared_node_id=parent.shared_node_id,
                shared_match_len=parent.shared_match_len,
                residual_blocks=list(parent.residual_blocks),
                tokens=list(parent.tokens),
                ref_count=1,
            )
            self._next_handle_id += 1
            self._handles[child.handle_id] = child
            return child

    def fork_many(self, parent: NodeHandle, k: int) -> List[NodeHandle]:
        """k forks of one parent with a single inc_ref launch."""
        with self._lock:
            self._version += 1
            self._validate_handle_locked(parent)
            if parent.residual_blocks and k > 0:
                ids = np.tile(np.fromiter((b.block_id for b in parent.residual_blocks), np.int32), k)
                self._alloc.inc_ref_batch(ids)
            kids = []
            for _ in range(k):
                if parent.shared_node_id != INVALID_NODE_ID:
                    self._inc_shared_ref_locked(parent.shared_node_id)
                c = NodeHandle(self._next_handle_id, parent.shared_node_id, parent.shared_match_len,
                               list(parent.residual_blocks), list(parent.tokens), 1)
                self._next_handle_id += 1
                self._handles[c.handle_id] = c
                kids.append(c)
            return kids

    def allocate_block(self, handle: NodeHandle) -> BlockHandle:
        with self._lock:
            self._version += 1
            self._validate_handle_locked(handle)
            bh = self._alloc.alloc()
            handle.residual_blocks.append(bh)
            return bh

    def allocate_blocks(self, handle: NodeHandle, n: int) -> List[BlockHandle]:
        """n allocate_block() calls in one launch (one wait for the ids)."""
        with self._lock:
            self._version += 1
            self._validate_handle_locked(handle)
            if n <= 0:
                return []
            new = [BlockHandle(int(b)) for b in self._alloc.alloc_many(n)]  # one wait
            handle.residual_blocks.extend(new)
            return new

    # ── copy-on-write ─────────────────────────────────────────────────────────
    def ensure_mutable_block(self, handle: NodeHandle, block_idx: int) -> BlockHandle:
        with self._lock:
            self._version += 1
            self._validate_handle_locked(handle)
            bh = handle.residual_blocks[block_idx]
            if "copy_block" in self._alloc.__dict__:
                # copy_block was replaced on the instance: run the reference's
                # steps so the replacement sees every (src, dst) pair.
                if self._alloc.ref_count(bh) > 1:
                    new_bh = self._alloc.alloc()
                    self._alloc.copy_block(bh, new_bh)
                    self._alloc.dec_ref(bh)
                    handle.residual_blocks[block_idx] = new_bh
                    return new_bh
                return bh
            nb = self._alloc.cow_one(bh.block_id)  # one wait: status and the owned block
            if nb != bh.block_id:
                bh = BlockHandle(nb)
                handle.residual_blocks[block_idx] = bh
            return bh

    def ensure_mutable_batch(self, requests: Sequence[Tuple[NodeHandle, int]]) -> List[bool]:
        """ensure_mutable_block for many (handle, index) slots, applied in
        order with one launch; returns which requests copied."""
        with self._lock:
            self._version += 1
            if not requests:
                return []
            seen = set()
            for h, i in requests:
                self._validate_handle_locked(h)
                key = (h.handle_id, i if i >= 0 else len(h.residual_blocks) + i)
                if key in seen:
                    raise ValueError("ensure_mutable_batch: a (handle, index) slot appears twice")
                seen.add(key)
            if "copy_block" in self._alloc.__dict__:
                return [self.ensure_mutable_block(h, i).block_id != b
                        for (h, i), b in zip(requests, [h.residual_blocks[i].block_id for h, i in requests])]
            blocks = np.fromiter((h.residual_blocks[i].block_id for h, i in requests), np.int32, len(requests))
            out_h, cp_h = self._alloc.cow_many(blocks)  # answered at the call, the copies enqueued
            for (h, i), nb, c in zip(requests, out_h, cp_h):
                if c:
                    h.residual_blocks[i] = BlockHandle(int(nb))
            return [bool(c) for c in cp_h]

    # ── frees / tokens ────────────────────────────────────────────────────────
    def free_block(self, handle: NodeHandle, block: BlockHandle) -> None:
        with self._lock:
            self._version += 1
            self._validate_handle_locked(handle)
            if block not in handle.residual_blocks:
                raise ValueError(
                    f"block {block} is not a residual block of handle {handle.handle_id}"
                )
            handle.residual_blocks.remove(block)
            self._alloc.dec_ref(block)

    def append_tokens(self, handle: NodeHandle, new_tokens: List[int]) -> None:
        with self._lock:
            self._validate_handle_locked(handle)
            handle.tokens.extend(new_tokens)

    def free(self, handle: NodeHandle) -> None:
        with self._lock:
            self._version += 1
            self._validate_handle_locked(handle)
            if handle.is_freed:
                raise ValueError(f"double-free of handle {handle.handle_id}")
            decs = [b.block_id for b in handle.residual_blocks]
            handle.residual_blocks.clear()
            if handle.shared_node_id != INVALID_NODE_ID:
                self._dec_shared_ref_locked(handle.shared_node_id, decs)
            if decs:
                self._alloc.dec_ref_batch(np.asarray(decs, np.int32))
            handle.is_freed = True
            del self._handles[handle.handle_id]
            self._ids_cache.pop(handle.handle_id, None)

    def free_many(self, handles: Sequence[NodeHandle]) -> None:
        """free() of several handles, in order, with one dec_ref launch."""
        with self._lock:
            self._version += 1
            decs: List[int] = []
            for h in handles:
                self._validate_handle_locked(h)
                if h.is_freed:
                    raise ValueError(f"double-free of handle {h.handle_id}")
            for h in handles:
                decs.extend(b.block_id for b in h.residual_blocks)
                h.residual_blocks.clear()
                if h.shared_node_id != INVALID_NODE_ID:
                    self._dec_shared_ref_locked(h.shared_node_id, decs)
                h.is_freed = True
                del self._handles[h.handle_id]
                self._ids_cache.pop(h.handle_id, None)
            if decs:
                self._alloc.dec_ref_batch(np.asarray(decs, np.int32))

    # ── match / commit ────────────────────────────────────────────────────────
    def match_prefix(self, tokens: List[int]) -> Tuple[Optional[NodeHandle], int]:
        epoch_token = self._alloc.enter_read_section()
        try:
            with self._lock:
                self._version += 1
                node_id, match_len = self._match_prefix_locked(tokens)
                if node_id == INVALID_NODE_ID or match_len == 0:
                    return None, 0
                self._inc_shared_ref_locked(node_id)
                h = NodeHandle(
                    handle_id=self._next_handle_id,
                    shared_node_id=node_id,
                    shared_match_len=match_len,
                    tokens=list(tokens[:match_len]),
                )
                self._next_handle_id += 1
                self._handles[h.handle_id] = h
                return h, match_len
        finally:
            self._alloc.leave_read_section(epoch_token)

    def match_prefix_many(self, queries: Sequence) -> List[Tuple[Optional[NodeHandle], int]]:
        """match_prefix on each query in order, with the lookups of all of
        them in one launch: the same (handle, length) pairs, handle ids,
        shared-node refcounts and reclaimer state as the calls one by one.
        One read section spans the batch; the calls' sections would each
        have released the same pending blocks, in the same order, with
        nothing else happening in between."""
        epoch_token = self._alloc.enter_read_section()
        try:
            with self._lock:
                self._version += 1
                node, mlen = match_batch(self._dev_tree, queries, self._cfg.block_size)
                out: List[Tuple[Optional[NodeHandle], int]] = []
                for q, nid, m in zip(queries, node.tolist(), mlen.tolist()):
                    if nid == INVALID_NODE_ID or m == 0:
                        out.append((None, 0))
                        continue
                    self._inc_shared_ref_locked(nid)
                    h = NodeHandle(handle_id=self._next_handle_id, shared_node_id=nid, shared_match_len=m,
                                   tokens=list(q[:m]))
                    self._next_handle_id += 1
                    self._handles[h.handle_id] = h
                    out.append((h, m))
                return out
        finally:
            self._alloc.leave_read_section(epoch_token)

    def match_prefix_batch(self, queries: Sequence, *, with_compared: bool = False):
        """Longest shared prefix of many queries in one launch, without
        creating handles: (node ids, match lengths[, tokens compared]) as numpy
        arrays.  Each result equals _match_prefix_locked on that query."""
        with self._lock:
            return match_batch(self._dev_tree, queries, self._cfg.block_size, with_compared=with_compared)

    def commit_prefix(self, handle: NodeHandle, length: int) -> None:
        with self._lock:
            self._version += 1
            self._validate_handle_locked(handle)
            bs = self._cfg.block_size
            if length % bs != 0:
                raise ValueError(
                    f"commit_prefix: length={length} must be a multiple of block_size={bs}"
                )
            n_blocks = length // bs
            if n_blocks > len(handle.residual_blocks):
                raise ValueError(
                    f"commit_prefix: requested {n_blocks} blocks but agent only "
                    f"has {len(handle.residual_blocks)} residual blocks"
                )
            promote = _as_i32(handle.tokens[handle.shared_match_len:][:length])
            promote_blocks = handle.residual_blocks[:n_blocks]
            parent = handle.shared_node_id if handle.shared_node_id != INVALID_NODE_ID else ROOT_NODE_ID
            # the replica applies the same insert itself (akv_tree_commands)
            self._dev_tree.begin_insert(parent, promote, self._next_node_id, bs)
            try:
                new_node_id = self._insert_shared_locked(parent, promote, promote_blocks)
            finally:
                self._dev_tree.end_command()
            handle.residual_blocks = handle.residual_blocks[n_blocks:]
            handle.shared_node_id = new_node_id
            handle.shared_match_len += length
            self._inc_shared_ref_locked(new_node_id)

    def get_block_ids(self, handle: NodeHandle) -> List[int]:
        with self._lock:
            self._validate_handle_locked(handle)
            # the walk up the shared chain is repeated only after a change
            # (a model layer's update asks once per layer)
            key = (self._version, handle.shared_node_id, id(handle.residual_blocks), len(handle.residual_blocks))
            hit = self._ids_cache.get(handle.handle_id)
            if hit is not None and hit[0] == key:
                return list(hit[1])
            ids: List[int] = []
            if handle.shared_node_id != INVALID_NODE_ID:
                for node in self._collect_shared_chain_locked(handle.shared_node_id):
                    ids.extend(bh.block_id for bh in node.blocks)
            ids.extend(bh.block_id for bh in handle.residual_blocks)
            self._ids_cache[handle.handle_id] = (key, ids)
            return list(ids)

    def stats(self) -> dict:
        with self._lock:
            return {
                "active_handles": len(self._handles),
                "shared_nodes": len(self._shared_nodes),
                "shared_blocks": sum(len(n.blocks) for n in self._shared_nodes.values()),
            }

    # ── internals ─────────────────────────────────────────────────────────────
    def _match_prefix_locked(self, tokens) -> Tuple[int, int]:
        """(node_id, match_len) of the longest block-aligned shared prefix,
        computed by the akv_match_prefix kernel on the device replica."""
        t = _as_i32(tokens)
        if len(t) == 0:
            return INVALID_NODE_ID, 0
        # one upload (offsets and tokens) and one read-back (status and
        # answer); the kernel asks L2 for the query's tokens first
        node, mlen = self._one.run(t, self._cfg.block_size, chunks=N.MATCH_PREFETCH)
        if mlen == 0:
            return INVALID_NODE_ID, 0
        return node, mlen

    def _new_node(self, parent_id: int, off: int, length: int, blocks: List[BlockHandle],
                  ref_count: int) -> SharedNode:
        nid = self._next_node_id
        self._next_node_id += 1
        node = SharedNode(nid, parent_id, self._dev_tree, off, length, list(blocks), ref_count)
        self._shared_nodes[nid] = node
        self._dev_tree.set_node(nid, off, length)
        return node

    def _set_child(self, parent: SharedNode, token: int, child_id: int) -> None:
        parent.children[token] = child_id
        self._dev_tree.set_child(parent.node_id, token, child_id, self._shared_nodes[child_id].edge_len)

    def _insert_shared_locked(self, parent_id: int, tokens: np.ndarray, blocks: List[BlockHandle]) -> int:
        """Insert under parent, splitting an edge on a block boundary
        (radix_tree.py:572-686)."""
        if len(tokens) == 0:
            return parent_id
        bs = self._cfg.block_size
        parent = self._shared_nodes[parent_id]
        first = int(tokens[0])
        if first not in parent.children:
            off = self._dev_tree.append_tokens(tokens)
            node = self._new_node(parent_id, off, len(tokens), blocks, 0)
            self._set_child(parent, first, node.node_id)
            return node.node_id
        child_id = parent.children[first]
        child = self._shared_nodes[child_id]
        common = _lcp(child.edge, tokens)
        if common == child.edge_len and common == len(tokens):
            child.blocks = list(blocks)
            return child_id
        if common == child.edge_len:
            return self._insert_shared_locked(child_id, tokens[common:], blocks[common // bs:])
        split = (common // bs) * bs
        if split == 0:
            off = self._dev_tree.append_tokens(tokens)
            node = self._new_node(parent_id, off, len(tokens), blocks, 0)
            self._set_child(parent, first, node.node_id)
            return node.node_id
        split_blocks = split // bs
        mid = self._new_node(parent_id, child.edge_off, split, child.blocks[:split_blocks], child.ref_count)
        child.parent_id = mid.node_id
        child.edge_off += split
        child.edge_len -= split
        child.blocks = list(child.blocks[split_blocks:])
        self._dev_tree.set_node(child_id, child.edge_off, child.edge_len)
        self._set_child(mid, int(self._dev_tree.h_tokens[child.edge_off]), child_id)
        self._set_child(parent, first, mid.node_id)
        if split == len(tokens):
            return mid.node_id
        rest = tokens[split:]
        off = self._dev_tree.append_tokens(rest)
        node = self._new_node(mid.node_id, off, len(rest), blocks[split_blocks:], 0)
        self._set_child(mid, int(rest[0]), node.node_id)
        return node.node_id

    def _inc_shared_ref_locked(self, node_id: int) -> None:
        nid = node_id
        while nid != INVALID_NODE_ID and nid in self._shared_nodes:
            self._shared_nodes[nid].ref_count += 1
            nid = self._shared_nodes[nid].parent_id

    def _dec_shared_ref_locked(self, node_id: int, decs: Optional[List[int]] = None) -> None:
        """Decrement up the chain and prune childless nodes at zero
        (radix_tree.py:695-717).  Blocks of pruned nodes are appended to
        `decs` (dec_ref'd by the caller in that order) or dec_ref'd now."""
        own = decs is None
        if own:
            decs = []
        nid = node_id
        while nid != INVALID_NODE_ID and nid in self._shared_nodes:
            node = self._shared_nodes[nid]
            node.ref_count -= 1
            if node.ref_count <= 0 and nid != ROOT_NODE_ID and not node.children:
                decs.extend(b.block_id for b in node.blocks)
                parent_id = node.parent_id
                self._dev_tree.begin_prune(parent_id if parent_id in self._shared_nodes else -1, nid)
                if parent_id in self._shared_nodes:
                    parent = self._shared_nodes[parent_id]
                    for k in [k for k, v in parent.children.items() if v == nid]:
                        del parent.children[k]
                        self._dev_tree.del_child(parent_id, k)
                del self._shared_nodes[nid]
                self._dev_tree.clear_node(nid)
                self._dev_tree.end_command()
                nid = parent_id
            else:
                nid = self._shared_nodes[nid].parent_id
        if own and decs:
            self._alloc.dec_ref_batch(np.asarray(decs, np.int32))

    def _collect_shared_chain_locked(self, node_id: int) -> List[SharedNode]:
        chain: List[SharedNode] = []
        nid = node_id
        while nid != INVALID_NODE_ID and nid in self._shared_nodes:
            node = self._shared_nodes[nid]
            chain.append(node)
            nid = node.parent_id
            if nid == ROOT_NODE_ID:
                break
        chain.reverse()
        return chain

    def _validate_handle_locked(self, handle: NodeHandle) -> None:
        if handle.handle_id not in self._handles:
            raise ValueError(
                f"NodeHandle {handle.handle_id} is not registered (was it already freed?)"
            )
        if handle.is_freed:
            raise ValueError(f"NodeHandle {handle.handle_id} has already been freed")


CoWRadixTree = DualRadixTree
