"""DeviceAgents — many agents stepped on the device, one launch per batch.

The reference's multi-agent consumers drive the pool one call at a time:
per step and agent slot, fork an agent into another slot (free the slot's
agent, then fork), copy-on-write the tail block (ensure_mutable_block(h,
-1)), free an agent and restart it from the shared root, advance the epoch,
or append a block (DualRadixTree.free / fork / ensure_mutable_block /
allocate_block, agentkv/core/radix_tree.py:222-377; EpochReclaimer.
maybe_advance, reclamation.py:129-143).  Each such call that returns a block
id costs a device round trip here.  DeviceAgents keeps the agents' residual
block tables in device memory and applies whole batches of those steps with
one akv_agent_steps launch, op by op with the reference's allocator
semantics, and returns each step's copy-on-write pairs on the device in the
counted-copy format (ShardedCopier.copy_batch / kernels.copy_blocks_counted
copy them; rank 0 can broadcast them to a head-sharded pool as one buffer).

Host bookkeeping follows the calls exactly: every fork takes the tree's next
handle id, in action order; a freed handle leaves the tree's registry.  The
NodeHandle objects of the slots' current agents are built by sync() (their
residual tables come back from the device); until then the handles given to
the constructor must not be used with the pool's per-call API.

All agents and the root must share one shared-tree node (as agents forked
from a committed root do): a free then drops, and the fork that follows
takes, one reference on that node's chain, so the shared tree is unchanged
by a step and no prune can happen inside a batch.
"""

from __future__ import annotations

from typing import List, Optional, Sequence

import numpy as np
import torch

from . import _native as N
from .allocator import BlockHandle
from .kernels import stream_handle
from .radix_tree import INVALID_NODE_ID, NodeHandle

FORK, COW, FREE, ADVANCE, APPEND = range(5)


class DeviceAgents:
    def __init__(self, pool, root: NodeHandle, agents: Sequence[NodeHandle], capacity: int = 0) -> None:
        tree = getattr(pool, "_tree", pool)
        self.tree = tree
        self.alloc = tree._alloc
        self.device = self.alloc.device
        with tree._lock:
            tree._validate_handle_locked(root)
            for h in agents:
                tree._validate_handle_locked(h)
                if h.shared_node_id != root.shared_node_id or h.shared_match_len != root.shared_match_len:
                    raise ValueError("DeviceAgents: every agent must share the root's shared-tree node")
            lens = [len(h.residual_blocks) for h in agents]
            cap = capacity or max(1024, 4 * max(lens + [len(root.residual_blocks), 1]))
            if max(lens + [len(root.residual_blocks)]) > cap:
                raise ValueError(f"DeviceAgents: capacity {cap} is below an agent's {max(lens)} blocks")
            self.cap = cap
            self.n = len(agents)
            tab = np.zeros((self.n, cap), np.int32)
            for i, h in enumerate(agents):
                tab[i, : lens[i]] = [b.block_id for b in h.residual_blocks]
            self.tables = torch.from_numpy(tab).to(self.device)
            self.lens = torch.tensor(lens, dtype=torch.int32, device=self.device)
            rt = np.asarray([b.block_id for b in root.residual_blocks] or [0], np.int32)
            self.root_table = torch.from_numpy(rt).to(self.device)
            self.root_len = len(root.residual_blocks)
        self.root = root
        self._originals = {h.handle_id: h for h in agents}
        self._slot_id = [h.handle_id for h in agents]  # handle id of each slot's current agent
        self._slot_tokens = [h.tokens for h in agents]  # the token list each slot's agent was forked with
        self._pairs_buf: Optional[torch.Tensor] = None
        self._keep = None

    def steps(self, step_actions: Sequence, pairs_cap: int = 0) -> torch.Tensor:
        """Apply steps (each an array of (kind, slot, target) actions: FORK,
        COW, FREE, ADVANCE, APPEND) in one launch; returns the device int32
        buffer [steps, 2 + 2 * pairs_cap] of each step's copy-on-write pairs
        (an int64 count, then the pairs), valid until the next call.
        pairs_cap defaults to the largest step's action count.  Errors (an
        exhausted pool, ...) are raised by check()."""
        acts = [np.asarray(a, np.int32).reshape(-1, 3) for a in step_actions]
        n_steps = len(acts)
        off = np.zeros(n_steps + 1, np.int32)
        np.cumsum([len(a) for a in acts], out=off[1:])
        cap = pairs_cap or max([len(a) for a in acts] + [1])
        flat = np.concatenate(acts) if acts else np.zeros((0, 3), np.int32)
        tree = self.tree
        with tree._lock:
            # host bookkeeping of the calls: a freed agent leaves the registry,
            # each fork takes the next handle id
            for kind, s, t in flat:
                if kind == FORK:
                    self._retire_slot(t)
                    self._slot_id[t] = tree._next_handle_id
                    self._slot_tokens[t] = self._slot_tokens[s]
                    tree._next_handle_id += 1
                elif kind == FREE:
                    self._retire_slot(s)
                    self._slot_id[s] = tree._next_handle_id
                    self._slot_tokens[s] = self.root.tokens
                    tree._next_handle_id += 1
            tree._version += 1
            words = n_steps * (2 + 2 * cap)
            if self._pairs_buf is None or self._pairs_buf.numel() < words:
                self._pairs_buf = torch.zeros(max(words, 1024), dtype=torch.int32, device=self.device)
            up = np.concatenate([off, flat.reshape(-1)]).astype(np.int32)
            dev_up = self.alloc._ids.put(up)
            self._keep = dev_up
            a = self.alloc
            with a._lock:
                a._device_op()  # the per-call log first; the mirror is reloaded when next needed
                N.check(N.lib.akv_agent_steps(
                    a._state, a._tick(), self.tables.data_ptr(), self.lens.data_ptr(), self.n, self.cap,
                    self.root_table.data_ptr(), self.root_len, dev_up.data_ptr() + 4 * (n_steps + 1),
                    dev_up.data_ptr(), n_steps, self._pairs_buf.data_ptr(), cap, a._status.data_ptr(),
                    stream_handle(self.device)))
        return self._pairs_buf[:words].view(n_steps, 2 + 2 * cap)

    def _retire_slot(self, slot: int) -> None:
        h = self._originals.pop(self._slot_id[slot], None)
        if h is not None:  # a handle from the constructor: it is freed now
            h.is_freed = True
            h.residual_blocks = []
            self.tree._handles.pop(h.handle_id, None)
            self.tree._ids_cache.pop(h.handle_id, None)

    def check(self) -> None:
        """Wait for the queued steps and raise the first error, as the
        reference's failing call would."""
        self.alloc.check()

    def sync(self) -> List[NodeHandle]:
        """The slots' current agents as NodeHandles, registered with the tree
        (their residual tables read back from the device).  Waits."""
        self.check()
        tab = self.tables.cpu().numpy()
        lens = self.lens.cpu().numpy()
        tree = self.tree
        out = []
        with tree._lock:
            for i in range(self.n):
                hid = self._slot_id[i]
                h = self._originals.get(hid)
                blocks = [BlockHandle(int(b)) for b in tab[i, : lens[i]]]
                if h is None:
                    h = NodeHandle(hid, self.root.shared_node_id, self.root.shared_match_len, blocks,
                                   list(self._slot_tokens[i]))
                    tree._handles[hid] = h
                    self._originals[hid] = h
                else:
                    h.residual_blocks = blocks
                out.append(h)
            tree._version += 1
        return out

    @staticmethod
    def pairs_of(buf: torch.Tensor, step: int) -> np.ndarray:
        """Step `step`'s pairs from a steps() buffer, on the host (waits)."""
        row = buf[step].cpu().numpy()
        n = int(row[:2].view(np.int64)[0])
        return row[2 : 2 + 2 * n].reshape(-1, 2)


__all__ = ["DeviceAgents", "FORK", "COW", "FREE", "ADVANCE", "APPEND", "INVALID_NODE_ID"]
