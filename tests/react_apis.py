"""Adapters that give the oracle and the product pool the call set the
ReAct workload driver (agentkv_b200.workloads.react_setup / react_step) uses:
the pool's own calls plus residual_len(handle)."""

from oracle import oracle as O


class OracleReActAPI:
    """OracleTree + OracleAllocator (CPU restatement of the reference)."""

    def __init__(self, n_blocks: int, block_size: int, epoch_interval: int = 64, copy_cb=None):
        self.alloc = O.OracleAllocator(n_blocks, epoch_interval)
        self.tree = O.OracleTree(self.alloc, block_size, copy_cb=copy_cb)

    def __getattr__(self, name):
        return getattr(self.tree, name)

    def allocate_blocks(self, h, n):
        for _ in range(n):
            self.tree.allocate_block(h)

    def maybe_advance_epoch(self):
        self.alloc.maybe_advance_epoch()

    @staticmethod
    def residual_len(h):
        return len(h.residual)


class PoolReActAPI:
    """agentkv_b200.AgentKVPool (the device path)."""

    def __init__(self, pool):
        self.pool = pool

    def __getattr__(self, name):
        return getattr(self.pool, name)

    @staticmethod
    def residual_len(h):
        return len(h.residual_blocks)
