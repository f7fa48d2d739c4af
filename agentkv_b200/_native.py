"""ctypes binding of ``libagentkv_b200.so`` (the C ABI in include/agentkv_b200.h).

The library is the only implementation of the block-movement, allocator and
match_prefix paths: there is no Python or CPU fallback.  Importing this module
fails loudly when the library is missing; build it with
``python -m agentkv_b200._build`` (``__graft_entry__.build()`` does it too).
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libagentkv_b200.so"

# ── status codes (enum in agentkv_b200.h) ────────────────────────────────────
AKV_OK = 0
AKV_ERR_INVALID_ARG = 1
AKV_ERR_OUT_OF_RANGE = 2
AKV_ERR_EXHAUSTED = 3
AKV_ERR_DOUBLE_FREE = 4
AKV_ERR_NOT_ALLOCATED = 5
AKV_ERR_NOT_EXCLUSIVE = 6
AKV_ERR_DEPENDENT_PAIRS = 7
AKV_ERR_CUDA = 8
AKV_ERR_TIMEOUT = 9
AKV_ERR_TREE = 10
AKV_ERR_MIRROR = 11

ERROR_NAMES = {
    AKV_OK: "ok",
    AKV_ERR_INVALID_ARG: "invalid argument",
    AKV_ERR_OUT_OF_RANGE: "block id out of range",
    AKV_ERR_EXHAUSTED: "pool exhausted",
    AKV_ERR_DOUBLE_FREE: "double free",
    AKV_ERR_NOT_ALLOCATED: "not allocated",
    AKV_ERR_NOT_EXCLUSIVE: "destination not exclusively owned",
    AKV_ERR_DEPENDENT_PAIRS: "dependent copy pairs",
    AKV_ERR_CUDA: "CUDA error",
    AKV_ERR_TIMEOUT: "device wait timed out",
    AKV_ERR_TREE: "malformed tree replica",
    AKV_ERR_MIRROR: "replayed per-call log disagrees with the device state",
}

# ── ctl word indices ─────────────────────────────────────────────────────────
CTL_FREE_LEFT = 0
CTL_FREE_SIZE = 1
CTL_LIMBO_HEAD = 2
CTL_LIMBO_REL = 3
CTL_LIMBO_TAIL = 4
CTL_OPS = 5
CTL_EPOCH = 6
CTL_ALLOCS = 7
CTL_FREES = 8
CTL_PEAK = 9
CTL_LAST_RETIRED = 10
CTL_LAST_COPIED = 11
CTL_DONE = 12
CTL_ADVANCES = 13
CTL_RELEASED = 14
CTL_WORDS = 16
AUX_WORDS = 2048
LOG_HEADER_WORDS = 8
OP_ALLOC, OP_INCREF, OP_DECREF, OP_COW, OP_RELEASE, OP_ADVANCE = range(1, 7)
NOALLOC_MAX_BLOCKS = 262144
MAX_FANOUT_LEVELS = 16  # AKV_MAX_FANOUT_LEVELS
MATCH_PIPELINED = 0x100  # AKV_MATCH_PIPELINED
MATCH_PREFETCH = 0x200  # AKV_MATCH_PREFETCH
MATCH_MAX_RANGES = 64  # AKV_MATCH_MAX_RANGES

# Copy kernel variants (akv_copy_blocks_variant).
VARIANT_AUTO = 0
VARIANT_VEC = 1
VARIANT_BULK = 2
# bulk copies whose items are claimed from a counter in the status record
# (16 KiB x 12 / 32 KiB x 6 per SM); the status record must not be shared by
# launches that overlap on the GPU
VARIANT_CLAIMED_16K = 14
VARIANT_CLAIMED_32K = 15


class AkvStatus(C.Structure):
    _fields_ = [
        ("code", C.c_int32),
        ("index", C.c_int32),
        ("id", C.c_int32),
        ("observed", C.c_int32),
        ("aux", C.c_int64),
        ("_reserved", C.c_int64),
    ]


STATUS_BYTES = C.sizeof(AkvStatus)  # 32


class AkvAllocState(C.Structure):
    _fields_ = [
        ("ref_counts", C.c_void_p),
        ("free_ring", C.c_void_p),
        ("limbo_ids", C.c_void_p),
        ("limbo_epochs", C.c_void_p),
        ("ctl", C.c_void_p),
        ("scratch_count", C.c_void_p),
        ("scratch_last", C.c_void_p),
        ("scratch_aux", C.c_void_p),
        ("total_blocks", C.c_int32),
        ("_pad", C.c_int32),
    ]


class AkvTick(C.Structure):
    _fields_ = [
        ("readers_min", C.c_int64),
        ("readers_max", C.c_int64),
        ("epoch_interval", C.c_int32),
        ("readers_active", C.c_int32),
    ]


class AkvTreeView(C.Structure):
    _fields_ = [
        ("tokens", C.c_void_p),
        ("node_edge_off", C.c_void_p),
        ("node_edge_len", C.c_void_p),
        ("slots", C.c_void_p),
        ("n_tokens", C.c_int64),
        ("n_nodes", C.c_int32),
        ("slot_mask", C.c_int32),
        ("run_head", C.c_void_p),
        ("run_entries", C.c_void_p),
        ("n_runs", C.c_int32),
        ("run_nodes", C.c_int32),
    ]


_P = C.c_void_p
_I32 = C.c_int32
_I64 = C.c_int64

# name -> (restype, argtypes)
SIGNATURES = {
    "akv_version": (C.c_int, []),
    "akv_last_error": (C.c_int, [C.c_char_p, C.c_int]),
    "akv_status_clear": (C.c_int, [_P, _P]),
    "akv_agent_steps": (C.c_int, [C.POINTER(AkvAllocState), C.POINTER(AkvTick), _P, _P, _I32, _I32, _P, _I32, _P, _P,
                                  _I32, _P, _I32, _P, _P]),
    "akv_copy_wait": (C.c_int, [_P, _P, _I64, _I32, _I32, _P]),
    "akv_prepare": (C.c_int, []),
    "akv_copy_blocks": (C.c_int, [_P, _I64, _I32, _P, _I32, _P, _P, _P]),
    "akv_copy_blocks_variant": (C.c_int, [_P, _I64, _I32, _P, _I32, _P, _P, _I32, _P]),
    "akv_copy_blocks_counted": (C.c_int, [_P, _I64, _I32, _P, _I32, _P, _P, _P, _P]),
    "akv_kv_gather": (C.c_int, [_P, _I32, _I32, _I32, _I32, _I64, _I32, _P, _I32, _I64, _P, _P, _P, _P]),
    "akv_kv_scatter": (C.c_int, [_P, _I32, _I32, _I32, _I32, _I64, _I32, _P, _I32, _P, _P, _I64, _I64, _P, _P]),
    "akv_copy_blocks_layers": (C.c_int, [_P, _I32, _I64, _I64, _I32, _P, _I32, _P, _P, _I32, _P]),
    "akv_zero_blocks": (C.c_int, [_P, _I64, _I32, _P, _I32, _P, _P, _P]),
    "akv_zero_blocks_variant": (C.c_int, [_P, _I64, _I32, _P, _I32, _P, _P, _I32, _P]),
    "akv_check_pairs": (C.c_int, [_P, _I32, _I32, _P, _P, _P]),
    "akv_alloc_init": (C.c_int, [C.POINTER(AkvAllocState), _P]),
    "akv_alloc_batch": (C.c_int, [C.POINTER(AkvAllocState), _I32, _P, C.POINTER(AkvTick), _P, _P]),
    "akv_incref_batch": (C.c_int, [C.POINTER(AkvAllocState), _P, _I32, C.POINTER(AkvTick), _P, _P]),
    "akv_decref_batch": (
        C.c_int,
        [C.POINTER(AkvAllocState), _P, _I32, C.POINTER(AkvTick), _P, _P, _P],
    ),
    "akv_decref_batch_noalloc": (
        C.c_int,
        [C.POINTER(AkvAllocState), _P, _I32, C.POINTER(AkvTick), _P, _P, _P],
    ),
    "akv_limbo_release": (C.c_int, [C.POINTER(AkvAllocState), _I64, _P]),
    "akv_epoch_advance": (C.c_int, [C.POINTER(AkvAllocState), C.POINTER(AkvTick), _P]),
    "akv_cow_batch": (
        C.c_int,
        [C.POINTER(AkvAllocState), _P, _I64, _P, _I32, _P, _P, _P, C.POINTER(AkvTick), _P, _P],
    ),
    "akv_fanout_plan": (C.c_int, [_P, _P, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P]),
    "akv_fanout_tree_plan": (C.c_int, [_P, _P, _I32, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P]),
    "akv_tree_hash": (C.c_uint32, [_I32, _I32]),
    "akv_tree_apply": (C.c_int, [C.POINTER(AkvTreeView), _P, _I32, _P, _I32, _P, _P]),
    "akv_tree_commands": (C.c_int, [C.POINTER(AkvTreeView), _I64, _P, _I32, _P, _I64, _P, _P]),
    "akv_match_prefix": (
        C.c_int,
        [C.POINTER(AkvTreeView), _P, _P, _I32, _I32, _P, _P, _P, _P, _P],
    ),
    "akv_match_prefix_variant": (
        C.c_int,
        [C.POINTER(AkvTreeView), _P, _P, _I32, _I32, _P, _P, _P, _P, _P, _I32, _P],
    ),
    "akv_match_scratch_bytes": (C.c_int64, [_I32, _I64, _I32]),
    "akv_match_split_plan": (C.c_int, [_P, _I32, _I32, _P, _P]),
    "akv_match_prefix_split": (
        C.c_int,
        [C.POINTER(AkvTreeView), _P, _P, _I32, _I32, _P, _P, _P, _P, _P, _I32, _I32, _P, _I64, _I32, _P, _P],
    ),
    "akv_gather_upload": (C.c_int, [_P, _P, _I32, _P, _P, _I32, _P]),
    "akv_mirror_create": (C.c_void_p, [_I32]),
    "akv_mirror_destroy": (None, [_P]),
    "akv_mirror_load": (C.c_int, [_P, _P, _P, _P, _P, _P]),
    "akv_mirror_alloc": (C.c_int, [_P, _I32, C.POINTER(AkvTick), _P, _P]),
    "akv_mirror_incref": (C.c_int, [_P, _P, _I32, C.POINTER(AkvTick), _P]),
    "akv_mirror_decref": (C.c_int, [_P, _P, _I32, C.POINTER(AkvTick), _P, _P, _P]),
    "akv_mirror_cow": (C.c_int, [_P, _I32, C.POINTER(AkvTick), _P, _P]),
    "akv_mirror_release": (C.c_int, [_P, _I64]),
    "akv_mirror_advance": (C.c_int, [_P, C.POINTER(AkvTick)]),
    "akv_mirror_read": (C.c_int, [_P, _P, _P, _P, _P, _P]),
    "akv_mirror_ref": (C.c_int32, [_P, _I32]),
    "akv_mirror_log_words": (C.c_int64, [_P]),
    "akv_mirror_take_log": (C.c_int, [_P, _P, _I64]),
    "akv_alloc_replay": (C.c_int, [C.POINTER(AkvAllocState), _P, _I64, _P, _P]),
    "akv_match_staged_scratch_bytes": (C.c_int64, [_I32, _I64, _I32]),
    "akv_match_prefix_staged": (
        C.c_int,
        [C.POINTER(AkvTreeView), _P, _P, _I32, _I64, _I32, _P, _P, _P, _P, _I32, _P, _I64, _P, _P],
    ),
}


class NativeError(RuntimeError):
    """A host-side failure reported by the C ABI (nothing was enqueued)."""

    def __init__(self, code: int, message: str) -> None:
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {message}")
        self.code = code


def _load() -> C.CDLL:
    if not _LIB_PATH.exists():
        raise ImportError(
            f"agentkv_b200 native library not found at {_LIB_PATH}. "
            "Build it with `python -m agentkv_b200._build` (needs nvcc); "
            "agentkv_b200 has no CPU fallback."
        )
    lib = C.CDLL(str(_LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()
LIB_PATH = _LIB_PATH


def last_error() -> str:
    buf = C.create_string_buffer(512)
    lib.akv_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    """Raise NativeError for a non-zero host status."""
    if rc != AKV_OK:
        raise NativeError(rc, last_error())


def version() -> tuple[int, int]:
    v = lib.akv_version()
    return v >> 16, v & 0xFFFF
