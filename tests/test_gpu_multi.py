"""Two GPUs, NCCL: the KV-head sharded fan-out (needs >= 2 visible GPUs).

Rank 0 plans a Tree-of-Thought fan-out on its allocator and broadcasts each
level's pair list; every rank copies its head slice.  Each rank's slice must
equal the corresponding slice of a single-GPU copy of the same pool, and both
ranks must have received the same pairs as rank 0 planned.
"""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, q):
    import datetime

    import torch.distributed as dist

    from agentkv_b200 import kernels as K
    from agentkv_b200 import sharded as S
    from agentkv_b200.allocator import SlabAllocator
    from agentkv_b200.config import PoolConfig

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        n, L, H, bs, D = 400, 2, 8, 16, 32
        g = torch.Generator(device="cpu").manual_seed(77)
        full = torch.randint(-30000, 30000, (n, L, 2, H, bs, D), dtype=torch.int16, generator=g)
        mine = S.head_slice(full, rank, WORLD).contiguous().to(dev)
        copier = S.ShardedCopier(mine)
        lens = [4, 4]
        planned = []
        if rank == 0:
            a = SlabAllocator(PoolConfig(total_blocks=n, block_size=bs, num_layers=L, num_kv_heads=H,
                                         head_dim=D, dtype="float16", device="meta"))
            roots = a.alloc_batch(8)
            res = a.fanout_tree(roots, lens, 2, 3, 1)
            a.check()
        shapes = [len(lens) * 3, len(lens) * 9]
        got = []
        for lvl, npairs in enumerate(shapes):
            p = res["pairs"][lvl] if rank == 0 else None
            p = copier.share_pairs(p, npairs)
            copier.copy(p)
            got.append(p.cpu())
        torch.cuda.synchronize()
        # single-GPU reference on the full pool
        ref = full.to(dev)
        for p in got:
            K.copy_blocks(ref, p.to(dev))
        want = S.head_slice(ref, rank, WORLD).contiguous()
        ok = bool(torch.equal(mine, want))
        allp = torch.cat([x.view(-1) for x in got]).to(dev)
        gathered = [torch.empty_like(allp) for _ in range(WORLD)]
        dist.all_gather(gathered, allp)
        same = all(torch.equal(gathered[0], x) for x in gathered)
        q.put((rank, ok, same))
    finally:
        dist.destroy_process_group()


def test_sharded_fanout_two_gpus():
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(WORLD))
    assert all(ok for _, ok, _ in res), res
    assert all(same for _, _, same in res), res
