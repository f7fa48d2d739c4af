"""pytest plugin that runs the reference's own adapter tests on this package.

Loaded with ``-p reference_alias_plugin`` by tests/test_reference_adapters.py
in a child pytest over the reference checkout's unmodified test files.  It
registers agentkv_b200 under the reference's module names
(agentkv_b200.compat.install) before the tests import the adapters, so the
adapters' ``from agentkv import AgentKVPool`` and ``from
agentkv.core.radix_tree import NodeHandle`` resolve here.  With no GPU, the
device parts are stood in for by the test stand-ins used elsewhere in this
suite: the allocator by the oracle's allocator (oracle_slab.py) and the two
tree kernels by their CPU model (tree_kernel_model.py); everything else —
AgentKVPool, DualRadixTree's handles, shared nodes, inserts, splits, the
copy_block hook dispatch — is the package's own code.
"""

from __future__ import annotations

import torch

from agentkv_b200 import _native as N
from agentkv_b200 import compat
from agentkv_b200 import device_tree as DT
from agentkv_b200 import pool as P
from agentkv_b200 import radix_tree as RT
from oracle_slab import OracleSlab
from tree_kernel_model import TreeKernelModel


class CpuSlab(OracleSlab):
    """OracleSlab built from a PoolConfig, as AgentKVPool builds its allocator."""

    built = 0

    def __init__(self, cfg) -> None:
        CpuSlab.built += 1
        dev = "meta" if cfg.device == "meta" else "cpu"
        kv = torch.empty((cfg.total_blocks, cfg.num_layers, 2, cfg.num_kv_heads, cfg.block_size, cfg.head_dim),
                         dtype=torch.float16, device=dev)
        super().__init__(kv, cfg.epoch_interval)
        self._cfg = cfg

    def copy_block(self, src, dst) -> None:
        b = self._valid(dst)
        if self.o.ref_count(b) != 1:
            raise ValueError(f"copy_block: dst block {b} must have ref_count=1")
        if self._kv_data.device.type != "meta":
            self._kv_data[b].copy_(self._kv_data[self._valid(src)])

    def stats(self) -> dict:
        st = self.o.state()
        return {"total_blocks": self.n, "free_blocks": len(st["free_list"]),
                "allocated_blocks": self.allocated_count}


def pytest_configure(config) -> None:
    compat.install()
    N.lib = TreeKernelModel(N.lib)
    DT.stream_handle = lambda dev: 0
    P.SlabAllocator = CpuSlab
    RT.SlabAllocator = CpuSlab


def pytest_sessionfinish(session, exitstatus) -> None:
    """Evidence for the parent test that the adapters ran on this package:
    the pools they built and the lookups this package's tree made."""
    import sys

    import agentkv_b200

    print(f"\nagentkv_b200 alias: aliased={sys.modules['agentkv'] is agentkv_b200} "
          f"pools={CpuSlab.built} lookups={N.lib.match_calls}")
