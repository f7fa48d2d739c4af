"""Run code written against the reference package on this one.

The reference's consumers import more than the top-level names: the vLLM
and SGLang adapters do ``from agentkv.core.radix_tree import NodeHandle``
(integrations/vllm/block_manager.py:7, integrations/sglang/radix_cache.py:
63), the HF cache lives at ``agentkv.hf_cache`` and the kernels at
``agentkv.core.triton_kernels``.  ``install()`` registers this package under
the reference's module names, so such code runs unchanged:

    from agentkv_b200 import compat
    compat.install()                  # before importing the consumer
    from integrations.vllm.block_manager import AgentKVBlockManager

Module map (reference -> here): agentkv -> agentkv_b200, agentkv.pool ->
pool, agentkv.hf_cache -> hf_cache, agentkv.core.config -> config,
agentkv.core.radix_tree -> radix_tree, agentkv.core.slab_allocator ->
allocator, agentkv.core.reclamation -> reclamation,
agentkv.core.triton_kernels -> kernels; agentkv.core re-exports
CoWRadixTree, NodeHandle, SlabAllocator and BlockHandle as the reference's
agentkv/core/__init__.py does.
"""

from __future__ import annotations

import sys
import types

_SUBMODULES = {
    "pool": "pool",
    "hf_cache": "hf_cache",
    "core.config": "config",
    "core.radix_tree": "radix_tree",
    "core.slab_allocator": "allocator",
    "core.reclamation": "reclamation",
    "core.triton_kernels": "kernels",
}


def install(name: str = "agentkv") -> types.ModuleType:
    """Register this package as `name` (and its submodules under the
    reference's names) in sys.modules; returns the package.  Idempotent."""
    import importlib

    pkg = importlib.import_module("agentkv_b200")
    sys.modules[name] = pkg
    core = types.ModuleType(f"{name}.core", "agentkv_b200's modules under the reference's agentkv.core names")
    core.__path__ = []  # a package, so that its submodules import
    sys.modules[f"{name}.core"] = core
    for ref_name, here in _SUBMODULES.items():
        mod = importlib.import_module(f"agentkv_b200.{here}")
        sys.modules[f"{name}.{ref_name}"] = mod
        parent, _, leaf = ref_name.rpartition(".")
        setattr(core if parent == "core" else pkg, leaf, mod)
    from .allocator import BlockHandle, SlabAllocator
    from .radix_tree import CoWRadixTree, NodeHandle

    core.CoWRadixTree, core.NodeHandle = CoWRadixTree, NodeHandle
    core.SlabAllocator, core.BlockHandle = SlabAllocator, BlockHandle
    setattr(pkg, "core", core)
    return pkg
