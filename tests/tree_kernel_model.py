"""CPU model of the tree kernels — akv_tree_apply, akv_tree_commands,
akv_match_prefix_variant and akv_match_prefix_split — reading the same
AkvTreeView arrays from host memory, so that CPU tests can run the host-side orchestration of the device
tree (deltas, replicas, unary-chain runs, their rebuild policy) on CPU
DeviceTrees.  Test infrastructure only: the package's lookups run the CUDA
kernels and nothing else.

The match model follows the kernel's contract: hop by hop from the root; at
a node with a run it takes hops from consecutive run entries (as the kernel
does), elsewhere from the slot table's linear probe; every hop's edge tokens
are compared the way the reference loop (agentkv/core/radix_tree.py:
513-570) compares them, counting comparisons; the match is floored to the
block size, (-1, 0) when nothing is credited.  The split model restates the
range decomposition: each range [a, b) of a query's positions walks the
same hops, compares only its own positions and reports its first stop as a
key (2 x position + mismatch); the smallest key over a query's ranges gives
the answer.
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

    def _walker(self, view):
        """next_hop(node, token, pending) for the view: run entries where the
        node has a run, else the slot table's linear probe."""
        slots = _arr(view.slots, C.c_int32, (view.slot_mask + 1, 4))
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

        def next_hop(node, t, pending):
            if not pending and runs and node < view.run_nodes and head[node] >= 0:
                rp = int(head[node])
                rem = int(ent[rp, 3])
                assert rem >= 1 and rp + rem <= view.n_runs, (node, rp, rem)
                pending.extend(tuple(int(x) for x in ent[rp + k]) for k in range(rem))
            if pending:
                c, tok, cl, _ = pending.pop(0)
                self.run_hops += 1
                return (c, cl) if t == tok else (-1, 0)
            return probe(node, t)

        return next_hop

    def _arrays(self, view, tokens, q_off, nq):
        off = _arr(view.node_edge_off, C.c_int64, (view.n_nodes,))
        elen = _arr(view.node_edge_len, C.c_int32, (view.n_nodes,))
        arena = _arr(view.tokens, C.c_int32, (view.n_tokens,))
        qo = _arr(q_off, C.c_int64, (nq + 1,))
        q_all = _arr(tokens, C.c_int32, (int(qo[-1]),))
        return off, elen, arena, qo, q_all

    def akv_tree_commands(self, view, token_cap, cmds, n_cmds, payload, payload_len, status, stream) -> int:
        """The device-side inserts and prunes, restated on the host arrays:
        the same walk, split rules, arena appends and slot claims as the
        kernel (and, by design, as the host mirror)."""
        self.command_calls = getattr(self, "command_calls", 0) + 1
        slots = _arr(view.slots, C.c_int32, (view.slot_mask + 1, 4))
        off = _arr(view.node_edge_off, C.c_int64, (view.n_nodes,))
        ln = _arr(view.node_edge_len, C.c_int32, (view.n_nodes,))
        arena = _arr(view.tokens, C.c_int32, (token_cap,))
        cm = _arr(cmds, C.c_int64, (n_cmds, 8))
        pay = _arr(payload, C.c_int32, (payload_len,))
        mask = view.slot_mask

        def probe(parent, token):
            i = tree_hash(parent, token) & mask
            free = -1
            for _ in range(mask + 1):
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

        def set_child(parent, token, child, clen):
            found, free = probe(parent, token)
            s_ = found if found >= 0 else free
            assert s_ >= 0, "slot table full"
            slots[s_] = (parent, token, child, clen)

        for kind, parent, a2, src, n, ar, bs, _ in (tuple(int(x) for x in r) for r in cm):
            if kind == 2:
                nid = a2
                if parent >= 0 and ln[nid] > 0:
                    found, _f = probe(parent, int(arena[off[nid]]))
                    if found >= 0 and slots[found, 2] == nid:
                        slots[found] = (DELETED, 0, 0, 0)
                off[nid], ln[nid] = 0, 0
                continue
            assert kind == 1, kind
            toks = pay[src:src + n]
            node, nxt, pos = parent, a2, 0

            def append(p0):
                nonlocal ar
                m = n - p0
                assert ar + m <= token_cap
                arena[ar:ar + m] = toks[p0:]
                ar += m
                return ar - m

            while pos < n:
                first = int(toks[pos])
                found, _f = probe(node, first)
                if found < 0:
                    o = append(pos)
                    off[nxt], ln[nxt] = o, n - pos
                    set_child(node, first, nxt, n - pos)
                    break
                child = int(slots[found, 2])
                co, cl = int(off[child]), int(ln[child])
                lim = min(cl, n - pos)
                ne = np.flatnonzero(arena[co:co + lim] != toks[pos:pos + lim])
                common = int(ne[0]) if len(ne) else lim
                if common == cl and common == n - pos:
                    break
                if common == cl:
                    node, pos = child, pos + common
                    continue
                split = (common // bs) * bs
                if split == 0:
                    o = append(pos)
                    off[nxt], ln[nxt] = o, n - pos
                    set_child(node, first, nxt, n - pos)
                    break
                mid = nxt
                nxt += 1
                off[mid], ln[mid] = co, split
                off[child], ln[child] = co + split, cl - split
                set_child(mid, int(arena[co + split]), child, cl - split)
                set_child(node, first, mid, split)
                if split == n - pos:
                    break
                o = append(pos + split)
                off[nxt], ln[nxt] = o, n - pos - split
                set_child(mid, int(toks[pos + split]), nxt, n - pos - split)
                break
        return 0

    def akv_match_prefix_variant(self, view, tokens, q_off, nq, block_size, out_node, out_len, out_cmp,
                                 order, status, chunks, stream) -> int:
        self.match_calls += 1
        next_hop = self._walker(view)
        off, elen, arena, qo, q_all = self._arrays(view, tokens, q_off, nq)
        o_node = _arr(out_node, C.c_int32, (nq,))
        o_len = _arr(out_len, C.c_int32, (nq,))
        o_cmp = _arr(out_cmp, C.c_int64, (nq,)) if out_cmp else None
        for q in range(nq):
            Q = q_all[qo[q]:qo[q + 1]]
            L = len(Q)
            cur, d, compared = 0, 0, 0
            node = 0
            pending = []  # run entries still to use, in order
            while d < L:
                child, clen = next_hop(node, int(Q[d]), pending)
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

    def akv_match_prefix_split(self, view, tokens, q_off, nq, block_size, out_node, out_len, out_cmp, order,
                               range_starts, n_ranges, tokens_per_range, scratch, scratch_bytes, chunks,
                               status, stream) -> int:
        self.match_calls += 1
        R = tokens_per_range or 1024
        starts = _arr(range_starts, C.c_int64, (n_ranges + 1,)).copy()
        assert starts[0] == 0 and starts[1] == nq, starts
        need = 16 * int(starts[-1]) + 4 * nq
        assert scratch_bytes >= need, (need, scratch_bytes)
        next_hop = self._walker(view)
        off, elen, arena, qo, q_all = self._arrays(view, tokens, q_off, nq)
        ordr = _arr(order, C.c_int32, (nq,))
        o_node = _arr(out_node, C.c_int32, (nq,))
        o_len = _arr(out_len, C.c_int32, (nq,))
        o_cmp = _arr(out_cmp, C.c_int64, (nq,)) if out_cmp else None
        self.split_ranges = getattr(self, "split_ranges", 0)
        n_j = np.diff(starts)

        def range_stop(Q, a, b):
            """(key, matched, node) of the first stop range [a, b) sees, or
            None when the walk passes b without one."""
            L = len(Q)
            cur, d, pending = 0, 0, []
            while True:
                if d >= L:
                    return 2 * d, d, cur
                if d >= b:
                    return None
                child, clen = next_hop(cur, int(Q[d]), pending)
                if child < 0 or clen == 0:
                    return 2 * d, d, cur
                assert int(elen[child]) == clen, (child, int(elen[child]), clen)
                lim = min(clen, L - d)
                lo, hi = max(a, d), min(b, d + lim)
                if lo < hi:
                    ne = np.flatnonzero(Q[lo:hi] != arena[off[child] + lo - d:off[child] + hi - d])
                    if len(ne):
                        return 2 * (lo + int(ne[0])) + 1, d, cur
                if lim < clen:  # the edge runs past the query's end
                    return 2 * L, d, cur
                d += clen
                cur = child

        for r in range(nq):
            q = int(ordr[r])
            Q = q_all[qo[q]:qo[q + 1]]
            k = max(1, -(-len(Q) // R))
            # the plan gives rank r exactly ranges 0 .. k-1
            assert k <= n_ranges and r < n_j[k - 1] and (k == n_ranges or r >= n_j[k]), (r, k, n_j)
            stops = [range_stop(Q, j * R, min((j + 1) * R, len(Q))) for j in range(k)]
            self.split_ranges += k
            key, matched, node = min(s for s in stops if s is not None)
            m = (matched // block_size) * block_size
            o_node[q] = node if m else -1
            o_len[q] = m
            if o_cmp is not None:
                o_cmp[q] = (key >> 1) + (key & 1)
        return 0

    def akv_match_prefix_staged(self, view, tokens, q_off, nq, n_tokens, block_size, out_node, out_len, out_cmp,
                                order, window_tokens, scratch, scratch_bytes, status, stream) -> int:
        """The staged lookup as its two kernels do it: the chase follows
        first tokens only and records hops; the windows of the chased span
        report their first mismatch (position, hop); the smallest over the
        windows, or else the last hop, decides the answer (staged_finish)."""
        self.match_calls += 1
        W = window_tokens or 512
        need = self._real.akv_match_staged_scratch_bytes(nq, n_tokens, window_tokens)
        assert 0 <= need <= scratch_bytes, (need, scratch_bytes)
        next_hop = self._walker(view)
        off, elen, arena, qo, q_all = self._arrays(view, tokens, q_off, nq)
        assert int(qo[-1]) <= n_tokens
        o_node = _arr(out_node, C.c_int32, (nq,))
        o_len = _arr(out_len, C.c_int32, (nq,))
        o_cmp = _arr(out_cmp, C.c_int64, (nq,)) if out_cmp else None
        self.staged_windows = getattr(self, "staged_windows", 0)
        for q in range(nq):
            Q = q_all[qo[q]:qo[q + 1]]
            L = len(Q)
            hops, node, d, pending = [], 0, 0, []  # (child, edge length, depth)
            while d < L:
                child, clen = next_hop(node, int(Q[d]), pending)
                if child < 0:
                    break
                assert int(elen[child]) == clen, (child, int(elen[child]), clen)
                hops.append((child, clen, d))
                if clen == 0 or d + clen > L:
                    break
                d += clen
                node = child
            lims = [min(c, L - dd) for _, c, dd in hops]
            D = hops[-1][2] + lims[-1] if hops else 0
            starts = [dd for _, _, dd in hops]
            stop = None
            for k in range(-(-D // W)):  # every window on its own, as the verify warps take them
                self.staged_windows += 1
                lo, hi = k * W, min((k + 1) * W, D)
                h = int(np.searchsorted(starts, lo, side="right")) - 1
                p = lo
                while p < hi:
                    child, _, dd = hops[h]
                    e = min(hi, dd + lims[h])
                    ne = np.flatnonzero(Q[p:e] != arena[off[child] + p - dd:off[child] + e - dd])
                    if len(ne):
                        cand = (p + int(ne[0]), h)
                        stop = cand if stop is None else min(stop, cand)
                        break
                    p = e
                    h += 1
            if stop is not None:
                P, h = stop
                key, matched, nd = 2 * P + 1, hops[h][2], hops[h - 1][0] if h > 0 else 0
            elif not hops:
                key, matched, nd = 0, 0, 0
            else:
                child, clen, dd = hops[-1]
                if lims[-1] < clen or clen == 0:
                    key, matched, nd = 2 * (dd + lims[-1]), dd, hops[-2][0] if len(hops) > 1 else 0
                else:
                    key, matched, nd = 2 * (dd + clen), dd + clen, child
            m = (matched // block_size) * block_size
            o_node[q] = nd if m else -1
            o_len[q] = m
            if o_cmp is not None:
                o_cmp[q] = (key >> 1) + (key & 1)
        return 0
