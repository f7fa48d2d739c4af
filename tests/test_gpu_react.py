"""The ReAct multi-agent workload (Llama-3-70B geometry, 40,000 blocks, a
16,384-token shared prefix, 32 agents, 1000 steps of forks, CoW tail copies,
frees, appends and epoch advances) on the device pool.

* Through AgentKVPool's per-call API on a CUDA pool: at the checkpoints the
  agents' block tables equal the reference's recorded ones, and the device
  free list, refcounts, reclaimer queues and counters equal the oracle's
  after the same calls; at the end every block's bytes equal the oracle's.
* The vLLM-adapter pattern (copy_block replaced on the instance to record
  pairs, a metadata-only pool): each step's recorded pairs equal the
  reference's, and applying them step by step as variable-size batches
  (count + pairs in one buffer, count read on the device) gives the oracle's
  bytes.
"""

import json

import numpy as np
import pytest
import torch

from agentkv_b200 import AgentKVPool, PoolConfig
from agentkv_b200 import workloads as W
from agentkv_b200.sharded import ShardedCopier
from oracle import oracle as O

from react_apis import OracleReActAPI, PoolReActAPI
from test_gpu_alloc import assert_same_as_oracle

pytestmark = pytest.mark.gpu

N_BLOCKS, BS = W.LLAMA3_70B_GEOMETRY[:2]


def _golden(golden_dir):
    g = np.load(golden_dir / "react_70b.npz")
    return g, W.ReActSpec(**json.loads(str(g["spec"])))


def _seeded_bytes(kv: torch.Tensor, seed: int) -> np.ndarray:
    gen = torch.Generator(device=kv.device).manual_seed(seed)
    kv.view(torch.int16).random_(-30000, 30000, generator=gen)
    return kv.view(torch.uint8).reshape(kv.shape[0], -1).cpu().numpy().copy()


def test_react_trace_device_pool(golden_dir):
    g, spec = _golden(golden_dir)
    # 4 KiB blocks (1 layer, 2 heads, head_dim 32): the bytes are checked on
    # every block; the metadata does not depend on the block geometry.
    cfg = PoolConfig(total_blocks=N_BLOCKS, block_size=BS, num_layers=1, num_kv_heads=2, head_dim=32,
                     dtype="bfloat16", device="cuda")
    pool = AgentKVPool(config=cfg)
    kv = pool._allocator._kv_data
    host = _seeded_bytes(kv, 11)
    bpb = host.shape[1]
    api = PoolReActAPI(pool)
    oapi = OracleReActAPI(N_BLOCKS, BS, cfg.epoch_interval,
                          copy_cb=lambda s, d: O.copy_blocks(host, bpb, np.array([[s, d]], np.int32)))
    root, agents = W.react_setup(api, spec)
    oroot, oagents = W.react_setup(oapi, spec)
    np.testing.assert_array_equal(np.asarray(pool.get_block_ids(root), np.int32), g["root_table"])
    for i, actions in enumerate(W.react_trace(spec)):
        W.react_step(api, root, agents, actions)
        W.react_step(oapi, oroot, oagents, actions)
        k = f"s{i + 1}"
        if k + "_ref" in g.files:
            tables = np.concatenate([np.asarray(pool.get_block_ids(h), np.int32) for h in agents])
            np.testing.assert_array_equal(tables, g[k + "_tables"], err_msg=k)
            np.testing.assert_array_equal(pool._allocator.ref_counts(), g[k + "_ref"])
            np.testing.assert_array_equal(pool._allocator.free_list(), g[k + "_free"])
            assert_same_as_oracle(pool._allocator, oapi.alloc, k)
            st, want = pool.stats(), json.loads(str(g[k + "_stats"]))
            for key in ("free_blocks", "allocated_blocks", "peak_allocated", "total_allocs", "total_frees",
                        "epoch", "active_handles", "shared_nodes", "shared_blocks"):
                assert st[key] == want[key], (k, key)
    torch.cuda.synchronize()
    dev = kv.view(torch.uint8).reshape(N_BLOCKS, -1).cpu().numpy()
    assert np.array_equal(dev, host)


def test_react_recorded_pairs_as_counted_batches(golden_dir):
    g, spec = _golden(golden_dir)
    N_, bs, L, H, D, dt = W.LLAMA3_70B_GEOMETRY
    meta = AgentKVPool(config=PoolConfig(total_blocks=N_, block_size=bs, num_layers=L, num_kv_heads=H,
                                         head_dim=D, dtype=dt, device="meta"))
    step_pairs = []
    orig = meta._allocator.copy_block

    def record(src, dst):
        step_pairs.append((src.block_id, dst.block_id))
        orig(src, dst)

    meta._allocator.copy_block = record
    api = PoolReActAPI(meta)
    root, agents = W.react_setup(api, spec)
    assert not step_pairs

    # a 2 KiB-per-block slice stands for one rank's heads of every block
    dev = torch.device("cuda", 0)
    slice_pool = torch.empty((N_, 1, 2, 1, bs, 32), dtype=torch.bfloat16, device=dev)
    host = _seeded_bytes(slice_pool, 12)
    copier = ShardedCopier(slice_pool)
    buf = copier.batch_buffer(spec.agents)
    so = g["step_off"]
    for i, actions in enumerate(W.react_trace(spec)):
        step_pairs.clear()
        W.react_step(api, root, agents, actions)
        got = np.asarray(step_pairs, np.int32).reshape(-1, 2)
        want = g["pairs"][so[i]:so[i + 1]]
        np.testing.assert_array_equal(got, want, err_msg=f"step {i}")
        copier.pack_batch(got, buf)
        copier.share_batch(buf)
        copier.copy_batch(buf)
        O.copy_blocks(host, host.shape[1], want)
    torch.cuda.synchronize()
    assert np.array_equal(slice_pool.view(torch.uint8).reshape(N_, -1).cpu().numpy(), host)
    k = f"s{spec.steps}"
    tables = np.concatenate([np.asarray(meta.get_block_ids(h), np.int32) for h in agents])
    np.testing.assert_array_equal(tables, g[k + "_tables"])
    np.testing.assert_array_equal(meta._allocator.free_list(), g[k + "_free"])


def test_counted_copy_caps_and_empty():
    dev = torch.device("cuda", 0)
    pool = torch.empty((64, 1024), dtype=torch.uint8, device=dev)
    host = _seeded_bytes(pool, 13)
    copier = ShardedCopier(pool)
    buf = copier.batch_buffer(8)
    for pairs in ([], [[1, 2]], [[3, 4], [5, 6], [7, 8]]):
        copier.pack_batch(pairs, buf)
        copier.copy_batch(buf)
        O.copy_blocks(host, 1024, np.asarray(pairs, np.int32).reshape(-1, 2))
        torch.cuda.synchronize()
        assert np.array_equal(pool.cpu().numpy(), host)
    # a count above the buffer's capacity copies the capacity only
    copier.pack_batch([[10 + j, 30 + j] for j in range(8)], buf)
    copier.batch_count(buf).fill_(1000)
    copier.copy_batch(buf)
    O.copy_blocks(host, 1024, np.array([[10 + j, 30 + j] for j in range(8)], np.int32))
    torch.cuda.synchronize()
    assert np.array_equal(pool.cpu().numpy(), host)
    with pytest.raises(ValueError):
        copier.pack_batch([[0, 1]] * 9, buf)


@pytest.mark.parametrize("per_launch", [1, 10])
def test_react_trace_device_agents(golden_dir, per_launch):
    """The same trace through DeviceAgents: the agents' block tables on the
    device, `per_launch` steps applied by one akv_agent_steps launch.  Each
    step's copy-on-write pairs (read from the launch's pair buffer) equal the
    reference's recorded ones; copying them step by step with the counted
    copy gives the oracle's bytes; at the checkpoints the tables (after
    sync()), refcounts, free list, counters and stats equal the recorded
    ones."""
    from agentkv_b200.agents import DeviceAgents

    g, spec = _golden(golden_dir)
    N_, bs, L, H, D, dt = W.LLAMA3_70B_GEOMETRY
    meta = AgentKVPool(config=PoolConfig(total_blocks=N_, block_size=bs, num_layers=L, num_kv_heads=H,
                                         head_dim=D, dtype=dt, device="meta"))
    api = PoolReActAPI(meta)
    root, agents = W.react_setup(api, spec)
    dev_agents = DeviceAgents(meta, root, agents)
    dev = torch.device("cuda", 0)
    slice_pool = torch.empty((N_, 1, 2, 1, bs, 32), dtype=torch.bfloat16, device=dev)
    host = _seeded_bytes(slice_pool, 14)
    copier = ShardedCopier(slice_pool)
    so = g["step_off"]
    trace = W.react_trace(spec)
    for i0 in range(0, spec.steps, per_launch):
        chunk = trace[i0:i0 + per_launch]
        buf = dev_agents.steps(chunk, pairs_cap=spec.agents)
        for j in range(len(chunk)):
            i = i0 + j
            copier.copy_batch(buf[j])
            want = g["pairs"][so[i]:so[i + 1]]
            np.testing.assert_array_equal(DeviceAgents.pairs_of(buf, j), want, err_msg=f"step {i}")
            O.copy_blocks(host, host.shape[1], want)
        dev_agents.check()
        for j in range(len(chunk)):
            k = f"s{i0 + j + 1}"
            if k + "_ref" in g.files:
                assert j == len(chunk) - 1, "checkpoints fall on launch boundaries"
                handles = dev_agents.sync()
                tables = np.concatenate([np.asarray(meta.get_block_ids(h), np.int32) for h in handles])
                np.testing.assert_array_equal(tables, g[k + "_tables"], err_msg=k)
                np.testing.assert_array_equal(meta._allocator.ref_counts(), g[k + "_ref"])
                np.testing.assert_array_equal(meta._allocator.free_list(), g[k + "_free"])
                st, want = meta.stats(), json.loads(str(g[k + "_stats"]))
                for key in ("free_blocks", "allocated_blocks", "peak_allocated", "total_allocs", "total_frees",
                            "epoch", "active_handles", "shared_nodes", "shared_blocks"):
                    assert st[key] == want[key], (k, key)
    torch.cuda.synchronize()
    assert np.array_equal(slice_pool.view(torch.uint8).reshape(N_, -1).cpu().numpy(), host)
