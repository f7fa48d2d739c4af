"""CPU model of the two tree kernels — akv_tree_apply and
akv_match_prefix_variant — reading the same AkvTreeView arrays from host
memory, so that CPU tests can run the host-side orchestration of the device
tree (deltas, replicas, unary-chain runs, their rebuild policy) on CPU
DeviceTrees.  Test infrastructure only: the package's lookups run the CUDA
kernels and nothing else.

The match model follows the kernel's contract: hop by hop from the root; at
a node with a run it takes hops from consecutive run entries (as the kernel
does), elsewhere from the slot table's linear probe; every hop's edge tokens
are compared the way the reference loop (agentkv/core/radix_tree.py:
513-570) compares them, counting comparisons; the match is floored to the
block size, (-1, 0) when nothing is credited.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from agentkv_b200.device_tree import DELETED, EMPTY, tree_hash


def _arr(ptr: int, ctype, shape) -> np.ndarray:
    n = int(np.prod(shape))
    if n == 0:
        return np.zeros(shape, np.dtype(ctype))
    return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(ctype)), shape=(n,)).reshape(shape)


class TreeKernelModel:
    """Stands in for the native library object: the two tree calls are
    modelled, everything else is the real library's."""

    def __init__(self, real) -> None:
        self._real = real
        self.match_calls = 0
        self.run_hops = 0

    def __getattr__(self, name):
        return getattr(self._real, name)

    def akv_tree_apply(self, view, su, n_su, nu, n_nu, status, stream) -> int:
        slots = _arr(view.slots, C.c_int32, (view.slot_mask + 1, 4))
        off = _arr(view.node_edge_off, C.c_int64, (view.n_nodes,))
        ln = _arr(view.node_edge_len, C.c_int32, (view.n_nodes,))
        for r in _arr(su, C.c_int32, (n_su, 5)) if n_su else ():
            slots[r[0]] = r[1:]
        for r in _arr(nu, C.c_int64, (n_nu, 3)) if n_nu else ():
            off[r[0]] = r[1]
            ln[r[0]] = r[2]
        return 0

    def akv_match_prefix_variant(self, view, tokens, q_off, nq, block_size, out_node, out_len, out_cmp,
                                 order, status, chunks, stream) -> int:
        self.match_calls += 1
        slots = _arr(view.slots, C.c_int32, (view.slot_mask + 1, 4))
        off = _arr(view.node_edge_off, C.c_int64, (view.n_nodes,))
        elen = _arr(view.node_edge_len, C.c_int32, (view.n_nodes,))
        arena = _arr(view.tokens, C.c_int32, (view.n_tokens,))
        qo = _arr(q_off, C.c_int64, (nq + 1,))
        q_all = _arr(tokens, C.c_int32, (int(qo[-1]),))
        o_node = _arr(out_node, C.c_int32, (nq,))
        o_len = _arr(out_len, C.c_int32, (nq,))
        o_cmp = _arr(out_cmp, C.c_int64, (nq,)) if out_cmp else None
        runs = view.run_head is not None and view.run_head != 0
        if runs:
            head = _arr(view.run_head, C.c_int32, (view.run_nodes,))
            ent = _arr(view.run_entries, C.c_int32, (view.n_runs, 4))
        mask = view.slot_mask

        def probe(node, t):
            i = tree_hash(node, t) & mask
            for _ in range(mask + 1):
                p = slots[i, 0]
                if p == EMPTY:
                    return -1, 0
                if p != DELETED and p == node and slots[i, 1] == t:
                    return int(slots[i, 2]), int(slots[i, 3])
                i = (i + 1) & mask
            return -1, 0

        for q in range(nq):
            Q = q_all[qo[q]:qo[q + 1]]
            L = len(Q)
            cur, d, compared = 0, 0, 0
            node = 0
            pending = []  # run entries still to use, in order
            while d < L:
                if not pending and runs and node < view.run_nodes and head[node] >= 0:
                    rp = int(head[node])
                    rem = int(ent[rp, 3])
                    assert rem >= 1 and rp + rem <= view.n_runs, (node, rp, rem)
                    pending = [tuple(int(x) for x in ent[rp + k]) for k in range(rem)]
                if pending:
                    c, t, cl, _ = pending.pop(0)
                    self.run_hops += 1
                    child, clen = (c, cl) if int(Q[d]) == t else (-1, 0)
                else:
                    child, clen = probe(node, int(Q[d]))
                if child < 0:
                    break
                assert int(elen[child]) == clen, (child, int(elen[child]), clen)
                lim = min(clen, L - d)
                e = arena[off[child]:off[child] + lim]
                ne = np.flatnonzero(Q[d:d + lim] != e)
                em = int(ne[0]) if len(ne) else lim
                compared += em + (1 if em < lim else 0)
                if em == 0 or em < clen:
                    break
                d += em
                node = cur = child
            m = (d // block_size) * block_size
            o_node[q] = cur if m else -1
            o_len[q] = m
            if o_cmp is not None:
                o_cmp[q] = compared
        return 0
