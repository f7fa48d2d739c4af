"""The C-ABI library loads, exports exactly what include/agentkv_b200.h
declares, and its structs have the layout the Python binding assumes.  No
call here touches a GPU: only argument validation paths that return before
any CUDA call, and the pure host function akv_tree_hash."""

import ctypes as C
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from agentkv_b200 import _native as N
from agentkv_b200.device_tree import tree_hash, tree_hash_np

REPO = Path(__file__).resolve().parent.parent
HEADERS = sorted((REPO / "include").glob("*.h"))


def declared_symbols():
    names = set()
    for h in HEADERS:
        for m in re.finditer(r"^AKV_API\s+\w+\s*\**\s*(akv_\w+)\s*\(", h.read_text(), re.M):
            names.add(m.group(1))
    return names


def exported_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", str(N.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_library_exports_every_declared_symbol():
    decl = declared_symbols()
    assert len(decl) >= 18
    assert exported_symbols() == decl
    for name in decl:
        assert hasattr(N.lib, name)
        assert name in N.SIGNATURES


def test_struct_layouts_match_header(tmp_path):
    src = tmp_path / "probe.c"
    src.write_text(r"""
#include <stdio.h>
#include <stddef.h>
#include "agentkv_b200.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu %zu %zu\n", sizeof(AkvStatus), sizeof(AkvAllocState),
         sizeof(AkvTick), sizeof(AkvTreeView), offsetof(AkvAllocState, total_blocks),
         offsetof(AkvTick, epoch_interval), offsetof(AkvTreeView, n_tokens),
         offsetof(AkvTreeView, slot_mask));
  printf("%d %d %d\n", AKV_CTL_WORDS, AKV_AUX_WORDS, AKV_CTL_RELEASED);
  return 0;
}
""")
    exe = tmp_path / "probe"
    subprocess.run(["gcc", f"-I{REPO / 'include'}", str(src), "-o", str(exe)], check=True)
    lines = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    c_vals = [int(x) for x in lines[0].split()]
    py_vals = [C.sizeof(N.AkvStatus), C.sizeof(N.AkvAllocState), C.sizeof(N.AkvTick),
               C.sizeof(N.AkvTreeView), N.AkvAllocState.total_blocks.offset,
               N.AkvTick.epoch_interval.offset, N.AkvTreeView.n_tokens.offset,
               N.AkvTreeView.slot_mask.offset]
    assert c_vals == py_vals
    assert [int(x) for x in lines[1].split()] == [N.CTL_WORDS, N.AUX_WORDS, N.CTL_RELEASED]


def test_version_and_last_error():
    assert N.version() >= (0, 3)
    # Rejected on the host before any CUDA call.
    rc = N.lib.akv_copy_blocks(None, 64, 4, None, -1, None, None, None)
    assert rc == N.AKV_ERR_INVALID_ARG
    assert "n_pairs" in N.last_error()
    rc = N.lib.akv_zero_blocks(None, 64, 4, None, 3, None, None, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "NULL" in N.last_error()
    with pytest.raises(N.NativeError):
        N.check(N.AKV_ERR_INVALID_ARG)


def test_empty_batches_are_noops_without_gpu():
    assert N.lib.akv_copy_blocks(None, 64, 4, None, 0, None, None, None) == N.AKV_OK
    assert N.lib.akv_zero_blocks(None, 64, 4, None, 0, None, None, None) == N.AKV_OK


def test_match_prefix_rejects_bad_tree_view():
    v = N.AkvTreeView(None, None, None, None, 0, 0, 0, None, None, 0, 0)
    rc = N.lib.akv_match_prefix(C.byref(v), None, None, 1, 16, None, None, None, None, None)
    assert rc == N.AKV_ERR_INVALID_ARG


def test_tree_hash_python_equals_c():
    rng = np.random.default_rng(0)
    parents = rng.integers(-5, 2**31 - 1, size=2000)
    tokens = rng.integers(-(2**31), 2**31 - 1, size=2000)
    c = np.array([N.lib.akv_tree_hash(int(p), int(t)) for p, t in zip(parents, tokens)], np.uint32)
    assert all(tree_hash(int(p), int(t)) == int(h) for p, t, h in zip(parents[:200], tokens[:200], c[:200]))
    np.testing.assert_array_equal(tree_hash_np(parents, tokens), c)


def test_host_argument_checks_of_tuning_entry_points():
    """Arguments the library refuses on the host, before any CUDA call: copy
    variants past 18, the dynamically claiming variants 14-18 without a
    status record (their work counter lives there), layer-copy variants past
    4 and unaligned layer spans,
    match widths outside {1,2,4,8,16}, run arrays without their entries,
    fan-out plans deeper than AKV_MAX_FANOUT_LEVELS or without appended
    blocks.  (Pointers are dummies: nothing is dereferenced.)"""
    P = 16  # a dummy non-NULL pointer
    rc = N.lib.akv_copy_blocks_variant(P, 64, 4, P, 1, None, None, 19, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "unknown variant 19" in N.last_error()
    for v in (14, 15, 16, 17, 18):
        rc = N.lib.akv_copy_blocks_variant(P, 64, 4, P, 1, None, None, v, None)
        assert rc == N.AKV_ERR_INVALID_ARG and "NULL status" in N.last_error()
    rc = N.lib.akv_copy_blocks_layers(P, 2, 4096, 4096, 8, P, 1, None, None, 5, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "variant 5" in N.last_error()
    rc = N.lib.akv_copy_blocks_layers(P, 2, 4100, 4100, 8, P, 1, None, None, 0, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "multiples of 16" in N.last_error()
    assert N.lib.akv_copy_blocks_layers(P, 0, 4096, 4096, 8, P, 1, None, None, 0, None) == N.AKV_OK

    v = N.AkvTreeView(P, P, P, P, 8, 4, 31, None, None, 0, 0)
    rc = N.lib.akv_match_prefix_variant(C.byref(v), P, P, 1, 16, P, P, None, None, None, 3, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "chunks=3" in N.last_error()
    v_runs = N.AkvTreeView(P, P, P, P, 8, 4, 31, P, None, 0, 4)
    rc = N.lib.akv_match_prefix_variant(C.byref(v_runs), P, P, 1, 16, P, P, None, None, None, 0, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "run_head" in N.last_error()
    v_mask = N.AkvTreeView(P, P, P, P, 8, 4, 30, None, None, 0, 0)
    rc = N.lib.akv_match_prefix_variant(C.byref(v_mask), P, P, 1, 16, P, P, None, None, None, 0, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "power of two" in N.last_error()

    rc = N.lib.akv_fanout_tree_plan(P, P, 1, 4, 2, 1, N.MAX_FANOUT_LEVELS + 1, P, P, P, P, P, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "levels" in N.last_error()
    rc = N.lib.akv_fanout_tree_plan(P, P, 1, 4, 2, 0, 2, P, P, P, P, P, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "append" in N.last_error()


def test_host_argument_checks_of_kv_io():
    """akv_kv_gather / akv_kv_scatter refuse on the host: NULL buffers, a
    layer past the model, more tokens than the table's blocks hold; an empty
    gather is a no-op.  (Dummy pointers: nothing is dereferenced.)"""
    P = 16
    rc = N.lib.akv_kv_gather(None, 8, 2, 2, 16, 256, 0, P, 1, 4, P, P, None, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "NULL" in N.last_error()
    rc = N.lib.akv_kv_gather(P, 8, 2, 2, 16, 256, 2, P, 1, 4, P, P, None, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "layer 2 of 2" in N.last_error()
    rc = N.lib.akv_kv_gather(P, 8, 2, 2, 16, 256, 0, P, 1, 17, P, P, None, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "17 tokens exceed 1 blocks of 16" in N.last_error()
    assert N.lib.akv_kv_gather(P, 8, 2, 2, 16, 256, 0, P, 1, 0, P, P, None, None) == N.AKV_OK
    rc = N.lib.akv_kv_scatter(P, 8, 2, 2, 16, 256, 5, P, 1, P, P, 256, 512, None, None)
    assert rc == N.AKV_ERR_INVALID_ARG


def test_host_argument_checks_of_noalloc_decref():
    """akv_decref_batch_noalloc refuses on the host, before any CUDA call:
    an incomplete state, a pool larger than its static scratch covers, a bad
    tick, a NULL status or ids, a negative count; an empty batch is a no-op.
    (Dummy pointers: nothing is dereferenced.)"""
    P = 16
    tick = N.AkvTick(0, 0, 64, 0)

    def state(n_blocks, ref=P):
        return N.AkvAllocState(ref, P, P, P, P, None, None, None, n_blocks, 0)

    f = N.lib.akv_decref_batch_noalloc
    rc = f(C.byref(state(64, ref=None)), P, 1, C.byref(tick), None, P, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "incomplete" in N.last_error()
    big = state(N.NOALLOC_MAX_BLOCKS + 1)
    rc = f(C.byref(big), P, 1, C.byref(tick), None, P, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "exceeds" in N.last_error()
    assert str(N.NOALLOC_MAX_BLOCKS) in N.last_error()
    ok = state(N.NOALLOC_MAX_BLOCKS)
    rc = f(C.byref(ok), P, 1, C.byref(N.AkvTick(0, 0, 0, 0)), None, P, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "tick" in N.last_error()
    rc = f(C.byref(ok), P, 1, C.byref(tick), None, None, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "status" in N.last_error()
    rc = f(C.byref(ok), P, -1, C.byref(tick), None, P, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "n=-1" in N.last_error()
    rc = f(C.byref(ok), None, 3, C.byref(tick), None, P, None)
    assert rc == N.AKV_ERR_INVALID_ARG and "ids is NULL" in N.last_error()
    # an empty batch returns before the scratch lookup (no CUDA call); an
    # oversized pool is refused even then
    assert f(C.byref(ok), None, 0, C.byref(tick), None, P, None) == N.AKV_OK
    assert f(C.byref(big), None, 0, C.byref(tick), None, P, None) == N.AKV_ERR_INVALID_ARG


def test_split_plan_python_equals_c():
    """The range plan of a split lookup: the package's split_plan and the
    library's host function akv_match_split_plan agree (queries longest
    first; range j holds the queries longer than j x R, all of them for
    j = 0), including empty queries, lengths on range boundaries and the
    longer ranges taken when the longest query would need more than
    AKV_MATCH_MAX_RANGES."""
    from agentkv_b200.device_tree import split_plan

    rng = np.random.default_rng(5)
    cases = [[0], [32, 32, 0], [8192, 4096, 4095, 33, 32, 31, 0], [64 * 1024 + 1, 5]]
    cases += [sorted(rng.integers(0, 9000, size=int(rng.integers(1, 300))).tolist(), reverse=True)
              for _ in range(20)]
    for lens in cases:
        for R in (0, 32, 1024, 2048):
            plan = split_plan(lens, R)
            L = np.asarray(lens, np.int64)
            starts = np.zeros(N.MATCH_MAX_RANGES + 1, np.int64)
            n = C.c_int32(-1)
            rc = N.lib.akv_match_split_plan(L.ctypes.data, len(L), plan.tokens_per_range, starts.ctypes.data,
                                            C.byref(n))
            assert rc == N.AKV_OK, N.last_error()
            assert n.value == plan.n_ranges
            np.testing.assert_array_equal(starts[: n.value + 1], plan.starts)
            k = np.maximum(1, -(-L // plan.tokens_per_range))
            assert plan.n_items == int(k.sum()) and plan.n_ranges <= N.MATCH_MAX_RANGES
    L = np.asarray([1, 2], np.int64)
    rc = N.lib.akv_match_split_plan(L.ctypes.data, 2, 32, np.zeros(4, np.int64).ctypes.data, C.byref(C.c_int32()))
    assert rc == N.AKV_ERR_INVALID_ARG and "longest first" in N.last_error()


def test_host_argument_checks_of_split_match():
    """akv_match_prefix_split refuses on the host: a missing order or range
    plan, a plan whose first range is not every query, ranges that grow,
    too little scratch, a range length that is not a multiple of 32, an
    unknown verify width.  (Dummy device pointers: nothing is dereferenced.)"""
    P = 16
    v = N.AkvTreeView(P, P, P, P, 8, 4, 31, None, None, 0, 0)
    good = np.array([0, 3, 5], np.int64)
    f = N.lib.akv_match_prefix_split

    def call(order=P, starts=good, n_ranges=2, R=32, scratch=256, bytes_=1 << 20, chunks=0):
        sp = starts.ctypes.data if starts is not None else None
        return f(C.byref(v), P, P, 3, 16, P, P, None, order, sp, n_ranges, R, scratch, bytes_, chunks, None, None)

    assert call(order=None) == N.AKV_ERR_INVALID_ARG and "required" in N.last_error()
    assert call(starts=None) == N.AKV_ERR_INVALID_ARG
    assert call(starts=np.array([0, 2, 3], np.int64)) == N.AKV_ERR_INVALID_ARG and "begin" in N.last_error()
    assert call(starts=np.array([0, 3, 7], np.int64)) == N.AKV_ERR_INVALID_ARG and "holds" in N.last_error()
    assert call(n_ranges=0) == N.AKV_ERR_INVALID_ARG
    assert call(n_ranges=N.MATCH_MAX_RANGES + 1) == N.AKV_ERR_INVALID_ARG
    assert call(bytes_=64) == N.AKV_ERR_INVALID_ARG and "needed" in N.last_error()
    assert call(scratch=None) == N.AKV_ERR_INVALID_ARG
    assert call(scratch=264) == N.AKV_ERR_INVALID_ARG and "aligned" in N.last_error()
    assert call(R=48) == N.AKV_ERR_INVALID_ARG and "multiple of 32" in N.last_error()
    assert call(chunks=3) == N.AKV_ERR_INVALID_ARG and "verify width" in N.last_error()
    assert call(chunks=16 | N.MATCH_PIPELINED) == N.AKV_ERR_INVALID_ARG
    assert N.lib.akv_match_scratch_bytes(3, 100, 48) == -1
    assert N.lib.akv_match_scratch_bytes(4096, 18_000_000, 0) == \
        (16 * (4096 + 18_000_000 // 1024) + 4 * 4096 + 255) // 256 * 256


def test_host_argument_checks_of_agent_steps():
    """akv_agent_steps refuses on the host: an incomplete allocator state, a
    bad tick, a NULL status, bad sizes (no agents, a root table longer than
    the capacity, a negative step count), NULL arrays; zero steps is a
    no-op.  (Dummy pointers: nothing is dereferenced.)"""
    P = 16
    tick = N.AkvTick(0, 0, 64, 0)
    ok = N.AkvAllocState(P, P, P, P, P, None, None, None, 64, 0)
    f = N.lib.akv_agent_steps

    def call(st=ok, tk=tick, n_agents=4, cap=8, root_len=2, n_steps=1, status=P, actions=P):
        return f(C.byref(st), C.byref(tk), P, P, n_agents, cap, P, root_len, actions, P, n_steps, P, 4, status, None)

    assert call(st=N.AkvAllocState(None, P, P, P, P, None, None, None, 64, 0)) == N.AKV_ERR_INVALID_ARG
    assert "incomplete" in N.last_error()
    assert call(tk=N.AkvTick(0, 0, 0, 0)) == N.AKV_ERR_INVALID_ARG and "tick" in N.last_error()
    assert call(status=None) == N.AKV_ERR_INVALID_ARG and "status" in N.last_error()
    assert call(n_agents=0) == N.AKV_ERR_INVALID_ARG
    assert call(root_len=9) == N.AKV_ERR_INVALID_ARG
    assert call(n_steps=-1) == N.AKV_ERR_INVALID_ARG
    assert call(actions=None) == N.AKV_ERR_INVALID_ARG and "NULL" in N.last_error()
    assert call(n_steps=0, actions=None) == N.AKV_OK
