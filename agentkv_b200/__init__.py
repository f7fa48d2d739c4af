"""agentkv_b200 — B200-native block-movement and prefix-lookup path for AgentKV.

Public API mirrors the reference package `agentkv`:
  AgentKVPool, DualRadixTree / CoWRadixTree, SlabAllocator, PoolConfig,
  AgentKVCache (the HuggingFace cache), BlockHandle, NodeHandle;
  kernels.copy_block / kernels.zero_block are the
  drop-ins for agentkv.core.triton_kernels.  FanoutGraph replays a whole
  Tree-of-Thought fan-out (forks, copy-on-write copies, appends, frees) as
  one CUDA graph.

The hot path (block copy / zero, free list and refcounts, match_prefix) runs
as sm_100a CUDA kernels in libagentkv_b200.so behind a C ABI
(include/agentkv_b200.h).  Submodules load lazily, so the seeded workload
generators (`agentkv_b200.workloads`) import without the native library.
"""

from __future__ import annotations

import importlib

__version__ = "0.3.0"

_EXPORTS = {
    "AgentKVPool": "pool",
    "PoolConfig": "config",
    "SlabAllocator": "allocator",
    "BlockHandle": "allocator",
    "INVALID_BLOCK": "allocator",
    "DualRadixTree": "radix_tree",
    "CoWRadixTree": "radix_tree",
    "NodeHandle": "radix_tree",
    "SharedNode": "radix_tree",
    "ROOT_NODE_ID": "radix_tree",
    "INVALID_NODE_ID": "radix_tree",
    "FanoutGraph": "fanout",
    "AgentKVCache": "hf_cache",
}

__all__ = ["__version__", *_EXPORTS]


def __getattr__(name: str):
    mod = _EXPORTS.get(name)
    if mod is None:
        raise AttributeError(f"module 'agentkv_b200' has no attribute {name!r}")
    return getattr(importlib.import_module(f"agentkv_b200.{mod}"), name)
