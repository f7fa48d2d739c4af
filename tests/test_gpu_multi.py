"""Two GPUs, NCCL: the KV-head sharded pool (needs >= 2 visible GPUs).

* Rank 0 plans a Tree-of-Thought fan-out on its allocator and broadcasts each
  level's pair list; every rank copies its head slice.  Each rank's slice must
  equal the corresponding slice of a single-GPU copy of the same pool, and
  both ranks must have received the same pairs as rank 0 planned.
* The ReAct multi-agent trace (70B geometry, 1000 steps): rank 0 runs the
  pool calls on a metadata-only pool and records each step's CoW pairs; each
  step's batch (count + pairs) goes to every rank in one broadcast and each
  rank copies its head slice with the count read on the device.  Every slice
  must equal the same heads of the oracle's pool after the reference's
  recorded pairs.
* Partitioned planning: each rank plans a fan-out in its own range of block
  ids, the ranks all-gather the pair lists and every slice takes all of them
  (checked against the oracle's copy of the full pool).
* match_prefix over replicas: rank 0 builds the stress tree through the pool
  API and broadcasts its deltas as it grows; each rank matches its
  contiguous range of the reference's recorded queries on its own replica;
  the gathered results equal the reference's.
"""

import os
import socket

import time

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
    holder = {"fg": None}
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


def _partition_worker(rank, port, q):
    """Partitioned planning: each rank runs a Tree-of-Thought fan-out on an
    allocator over its own range of block ids, the ranks all-gather the pair
    lists, and each rank copies every rank's pairs on its head slice."""
    import datetime

    import torch.distributed as dist

    from agentkv_b200 import sharded as S
    from agentkv_b200.allocator import SlabAllocator
    from agentkv_b200.config import PoolConfig
    from oracle import oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    holder = {"fg": None}
    try:
        n, L, H, bs, D = 400, 2, 8, 16, 32
        g = torch.Generator(device="cpu").manual_seed(78)
        full = torch.randint(-30000, 30000, (n, L, 2, H, bs, D), dtype=torch.int16, generator=g)
        mine = S.head_slice(full, rank, WORLD).contiguous().to(dev)
        copier = S.ShardedCopier(mine)
        base, count = S.partition(n, rank, WORLD)
        a = SlabAllocator(PoolConfig(total_blocks=count, block_size=bs, num_layers=L, num_kv_heads=H,
                                     head_dim=D, dtype="float16", device="meta"))
        roots = a.alloc_batch(6)
        res = a.fanout_tree(roots, [3, 3], 2, 3, 1)
        local = res["all_pairs"]
        out = torch.empty((WORLD * local.shape[0], 2), dtype=torch.int32, device=dev)
        got = copier.gather_pairs(local, base, out)
        copier.copy(got)
        a.check()
        torch.cuda.synchronize()
        everyone = [torch.empty_like(local) for _ in range(WORLD)]
        dist.all_gather(everyone, local + base)
        pairs_ok = bool(torch.equal(got, torch.cat(everyone)))
        host = full.numpy().view(np.uint8).reshape(n, -1).copy()
        O.copy_blocks(host, host.shape[1], got.cpu().numpy())
        # the same through a recorded FanoutGraph (gather inside the graph), replayed
        # three times with every child freed after its copy
        from agentkv_b200.fanout import FanoutGraph

        fg = holder["fg"] = FanoutGraph(a, [3, 3], 2, 3, 1, pool=mine, free_children=True, copier=copier,
                                        id_base=base)
        roots_np = roots.cpu().numpy()
        for _ in range(3):
            fg.run(roots_np)
            res_r, _, _, _, gathered_r = fg._keep[0]  # the replay's one fan-out
            gathered = gathered_r.cpu()
            everyone = [torch.empty_like(local) for _ in range(WORLD)]
            dist.all_gather(everyone, res_r["all_pairs"] + base)
            pairs_ok &= bool(torch.equal(gathered, torch.cat(everyone).cpu()))
            O.copy_blocks(host, host.shape[1], gathered.numpy())
        torch.cuda.synchronize()
        fg = holder["fg"] = None
        want = S.head_slice(torch.from_numpy(host.view(np.int16).reshape(full.shape)), rank, WORLD)
        q.put((rank, bool(torch.equal(mine.cpu(), want)), pairs_ok))
    finally:
        # a graph that holds NCCL calls must go before the process group, on
        # an error too, or destroy_process_group waits for good
        fg = holder["fg"] = None
        import gc

        gc.collect()
        dist.destroy_process_group()


def _react_worker(rank, port, q, golden):
    import datetime
    import json

    import torch.distributed as dist

    from agentkv_b200 import AgentKVPool, PoolConfig
    from agentkv_b200 import sharded as S
    from agentkv_b200 import workloads as W
    from oracle import oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        g = np.load(golden)
        spec = W.ReActSpec(**json.loads(str(g["spec"])))
        N_, bs, L, H, D, dt = W.LLAMA3_70B_GEOMETRY
        gen = torch.Generator(device="cpu").manual_seed(21)
        full = torch.randint(-30000, 30000, (N_, 1, 2, 2, bs, 32), dtype=torch.int16, generator=gen)
        mine = S.head_slice(full, rank, WORLD).contiguous().to(dev)
        copier = S.ShardedCopier(mine)
        buf = copier.batch_buffer(spec.agents)
        trace = W.react_trace(spec)
        pairs_ok = True
        if rank == 0:
            meta = AgentKVPool(config=PoolConfig(total_blocks=N_, block_size=bs, num_layers=L, num_kv_heads=H,
                                                 head_dim=D, dtype=dt, device="meta"))
            rec = []
            orig = meta._allocator.copy_block

            def record(src, dst):
                rec.append((src.block_id, dst.block_id))
                orig(src, dst)

            meta._allocator.copy_block = record

            class Api:
                def __getattr__(self, name):
                    return getattr(meta, name)

                @staticmethod
                def residual_len(h):
                    return len(h.residual_blocks)

            api = Api()
            root, agents = W.react_setup(api, spec)
        so = g["step_off"]
        for i, actions in enumerate(trace):
            if rank == 0:
                rec.clear()
                W.react_step(api, root, agents, actions)
                got = np.asarray(rec, np.int32).reshape(-1, 2)
                pairs_ok &= np.array_equal(got, g["pairs"][so[i]:so[i + 1]])
                copier.pack_batch(got, buf)
            copier.share_batch(buf)
            copier.copy_batch(buf)
        torch.cuda.synchronize()
        host = full.numpy().view(np.uint8).reshape(N_, -1).copy()
        O.copy_blocks(host, host.shape[1], g["pairs"])
        want = S.head_slice(torch.from_numpy(host.view(np.int16).reshape(full.shape)), rank, WORLD)
        ok = bool(torch.equal(mine.cpu(), want.contiguous()))
        q.put((rank, ok, bool(pairs_ok)))
    finally:
        dist.destroy_process_group()


def _match_worker(rank, port, q, golden):
    import datetime
    import json

    import torch.distributed as dist

    from agentkv_b200 import AgentKVPool, PoolConfig
    from agentkv_b200 import workloads as W
    from agentkv_b200.device_tree import DeviceTree
    from agentkv_b200.sharded_tree import TreeReplicaSync, match_split

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        g = np.load(golden)
        spec = W.MatchSpec(**json.loads(str(g["spec"])))
        prefixes = W.match_prefixes(spec)
        corpus = W.match_sequences(spec, prefixes)
        if rank == 0:
            pool = AgentKVPool(config=PoolConfig(total_blocks=int(g["total_blocks"]), block_size=16,
                                                 num_layers=1, num_kv_heads=1, head_dim=1, dtype="float16",
                                                 device="meta"))
            tree = pool._tree._dev_tree
        else:
            tree = DeviceTree(dev)
        sync = TreeReplicaSync(tree)
        for i, seq in enumerate(corpus):
            if rank == 0:
                h = pool.create_root(seq)
                pool.allocate_blocks(h, -(-len(seq) // 16) - len(pool.get_block_ids(h)))
                share = (len(seq) // 16) * 16 - h.shared_match_len
                if share > 0:
                    pool.commit_prefix(h, share)
            if i % 50 == 49 or i == len(corpus) - 1:
                sync.sync()
        queries = W.match_queries(spec, corpus, prefixes, batch=0, n=len(g["node"]))
        node, mlen = match_split(sync, queries, 16)
        ok = bool(np.array_equal(node, g["node"]) and np.array_equal(mlen, g["len"]))
        q.put((rank, ok, True))
    finally:
        dist.destroy_process_group()


def test_match_split_over_replicas_two_gpus(golden_dir):
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    res = _spawn(_match_worker, (str(golden_dir / "match_small.npz"),))
    assert all(ok for _, ok, _ in res), res


def _spawn(target, extra=()):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=target, args=(r, port, q, *extra)) for r in range(WORLD)]
    for p in procs:
        p.start()
    deadline = time.monotonic() + 180
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.monotonic()))
    codes = [p.exitcode for p in procs]
    for p in procs:  # a rank still running at the deadline is ended, not left behind
        if p.exitcode is None:
            p.kill()
            p.join(timeout=30)
    assert all(c == 0 for c in codes), codes
    return sorted(q.get(timeout=5) for _ in range(WORLD))


def test_sharded_react_two_gpus(golden_dir):
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    res = _spawn(_react_worker, (str(golden_dir / "react_70b.npz"),))
    assert all(ok for _, ok, _ in res), res
    assert all(pairs_ok for _, _, pairs_ok in res), res


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


def test_partitioned_planning_two_gpus():
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    res = _spawn(_partition_worker)
    assert all(ok for _, ok, _ in res), res
    assert all(pairs_ok for _, _, pairs_ok in res), res
