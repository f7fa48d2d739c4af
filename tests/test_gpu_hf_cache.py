"""AgentKVCache (the HuggingFace cache on the pool) against the reference's
recorded session and the oracle: every update's K/V output, the block
tables and the pool bytes, bit for bit; plus the gather/scatter kernels on
their own (partial last blocks, strided states, bad ids)."""

import json

import numpy as np
import pytest
import torch

from agentkv_b200 import AgentKVPool, PoolConfig
from agentkv_b200 import _native as N
from agentkv_b200 import kernels as K
from agentkv_b200 import workloads as W
from agentkv_b200.hf_cache import AgentKVCache
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _pool(spec):
    return AgentKVPool(config=PoolConfig(total_blocks=spec.total_blocks, block_size=spec.block_size,
                                         num_layers=spec.num_layers, num_kv_heads=spec.num_kv_heads,
                                         head_dim=spec.head_dim, dtype=spec.dtype, device="cuda"))


def _session(spec, pool, cache_cls, to_tensor):
    outs, keys = [], []

    def on_output(e, layer, ok, ov):
        ok = ok.cpu().numpy() if isinstance(ok, torch.Tensor) else ok
        ov = ov.cpu().numpy() if isinstance(ov, torch.Tensor) else ov
        keys.append((e, layer, ok.shape[2]))
        outs.append(np.concatenate([ok.reshape(-1), ov.reshape(-1)]))

    caches = W.hf_run(spec, pool, cache_cls, to_tensor, on_output)
    return caches, keys, np.concatenate(outs)


@pytest.mark.parametrize("append_only", [False, True])
def test_hf_session_matches_reference(golden_dir, append_only):
    import functools

    g = np.load(golden_dir / "hf_session.npz")
    spec = W.HFSpec(**json.loads(str(g["spec"])))
    pool = _pool(spec)
    cls = functools.partial(AgentKVCache, append_only=append_only)
    caches, keys, outs = _session(spec, pool, cls, lambda a: torch.from_numpy(a).to(DEV))
    np.testing.assert_array_equal(np.asarray(keys), g["out_keys"])
    assert outs.tobytes() == g["outs"].tobytes()
    tables = np.concatenate([np.asarray(pool.get_block_ids(c.handle), np.int32) for c in caches])
    np.testing.assert_array_equal(tables, g["tables"])
    assert [c.get_seq_length() for c in caches] == g["seen"].tolist()
    assert pool._allocator._kv_data.cpu().numpy().tobytes() == g["pool"].tobytes()
    legacy = caches[1].to_legacy_cache()
    assert len(legacy) == spec.num_layers and legacy[0][0].shape[2] == caches[1].get_seq_length()


@pytest.mark.parametrize("spec", [
    W.HFSpec(total_blocks=512, block_size=16, num_layers=4, num_kv_heads=8, head_dim=128, prompt=200,
             commit=192, forks=3, steps=8, seed=8),
    W.HFSpec(total_blocks=256, block_size=8, num_layers=3, num_kv_heads=2, head_dim=12, prompt=37,
             commit=32, forks=3, steps=12, seed=9),
])
def test_hf_session_matches_oracle(spec):
    pool = _pool(spec)
    caches, keys, outs = _session(spec, pool, AgentKVCache, lambda a: torch.from_numpy(a).to(DEV))
    opool = O.OracleKVPool(spec.total_blocks, spec.block_size, spec.num_layers, spec.num_kv_heads,
                           spec.head_dim, spec.dtype)
    ocaches, okeys, oouts = _session(spec, opool, O.OracleKVCache, lambda a: a)
    assert keys == okeys
    assert outs.tobytes() == oouts.tobytes()
    for c, oc in zip(caches, ocaches):
        assert pool.get_block_ids(c.handle) == opool.get_block_ids(oc.handle)
    assert pool._allocator._kv_data.cpu().numpy().tobytes() == opool.kv.tobytes()


def test_reference_fork_and_cow_flow():
    """The reference's own fork/CoW test flow (tests/test_hf_cache.py), on a
    CUDA pool."""
    pool = AgentKVPool(config=PoolConfig(total_blocks=16, block_size=4, num_layers=2, num_kv_heads=2,
                                         head_dim=16, dtype="float32", device="cuda"))
    root = pool.create_root([101, 102, 103, 104])
    cache = AgentKVCache(pool, root)
    cache._seen_tokens = 0
    ones = torch.ones(1, 2, 4, 16, device=DEV)
    cache.update(ones, ones, 0)
    cache.update(ones, ones, 1)
    pool.commit_prefix(root, 4)
    c1, c2 = cache.fork(), cache.fork()
    assert c1.get_seq_length() == c2.get_seq_length() == 4
    two = torch.full((1, 2, 1, 16), 2.0, device=DEV)
    k0, _ = c1.update(two, two, 0)
    c1.update(two, two, 1)
    assert c1.get_seq_length() == 5 and c2.get_seq_length() == 4
    assert torch.equal(k0[:, :, :4], torch.ones(1, 2, 4, 16, device=DEV))
    assert torch.equal(k0[:, :, 4:], two)
    legacy = c1.to_legacy_cache()
    assert len(legacy) == 2 and legacy[0][0].shape == (1, 2, 5, 16)
    with pytest.raises(ValueError):
        c1.update(torch.ones(2, 2, 1, 16, device=DEV), torch.ones(2, 2, 1, 16, device=DEV), 0)


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 12), (torch.float32, 7),
                                     (torch.bfloat16, 256)])  # the last: 8 KiB tiles, the general kernel
def test_gather_scatter_kernels(dtype, D):
    n, L, H, bs = 40, 3, 4, 16
    pool = torch.zeros((n, L, 2, H, bs, D), dtype=dtype, device=DEV)
    pool.view(-1).copy_(torch.randn(pool.numel(), device=DEV).to(dtype))
    host = pool.cpu().clone()
    rng = np.random.default_rng(3)
    ids = rng.permutation(n)[:7].astype(np.int32)
    for layer in range(L):
        for n_tok in (1, 16, 17, 100, 112):
            k, v = K.kv_gather(pool, torch.from_numpy(ids), layer, n_tok)
            data = host[torch.from_numpy(ids).long(), layer]
            want_k = data[:, 0].permute(1, 0, 2, 3).reshape(1, H, -1, D)[:, :, :n_tok]
            want_v = data[:, 1].permute(1, 0, 2, 3).reshape(1, H, -1, D)[:, :, :n_tok]
            assert torch.equal(k.cpu(), want_k) and torch.equal(v.cpu(), want_v)
    # scatter from strided states ([1, n, H, D] transposed to [1, H, n, D])
    new = torch.randn(1, 5, H, D, device=DEV).to(dtype).transpose(1, 2)
    newv = torch.randn(1, 5, H, D, device=DEV).to(dtype).transpose(1, 2)
    slots = np.array([3 * bs + 0, 3 * bs + 1, 9 * bs + 15, 20 * bs + 7, 39 * bs + 2], np.int32)
    K.kv_scatter(pool, torch.from_numpy(slots), 1, new, newv)
    for i, sl in enumerate(slots):
        host[sl // bs, 1, 0, :, sl % bs, :] = new[0, :, i, :].cpu()
        host[sl // bs, 1, 1, :, sl % bs, :] = newv[0, :, i, :].cpu()
    torch.cuda.synchronize()
    assert torch.equal(pool.cpu(), host)
    # bad ids / slots are reported, the rest still moves
    st = torch.zeros(8, dtype=torch.int32, device=DEV)
    K.kv_gather(pool, torch.tensor([1, 99], dtype=torch.int32), 0, 20, status=st)
    assert K.read_status(st)[:3] == (N.AKV_ERR_OUT_OF_RANGE, 1, 99)
    st.zero_()
    K.kv_scatter(pool, torch.tensor([-1], dtype=torch.int32), 0, new[:, :, :1], newv[:, :, :1], status=st)
    assert K.read_status(st)[0] == N.AKV_ERR_OUT_OF_RANGE
    with pytest.raises(N.NativeError):
        K.kv_gather(pool, torch.from_numpy(ids), 0, 7 * bs + 1)


@pytest.mark.parametrize("graph", [False, True])
def test_chained_scatter_gather_see_each_other(graph):
    """A decode step's chain of short launches, as the layers issue them:
    scatter a new row, gather the layer (which must read that row), scatter
    the next token's row into the block the gather just read, gather
    again ...  The scatters and gathers may be scheduled before the launch
    ahead of them ends (programmatic dependent launch); each must still see
    every write before it.  Eagerly and replayed from a CUDA graph, the
    gathered K/V equal a host model of the same writes."""
    n, L, H, bs, D = 64, 4, 8, 16, 128
    pool = torch.zeros((n, L, 2, H, bs, D), dtype=torch.bfloat16, device=DEV)
    pool.view(-1).copy_(torch.randn(pool.numel(), device=DEV).to(torch.bfloat16))
    host = pool.cpu().clone()
    rng = np.random.default_rng(11)
    ids = torch.from_numpy(rng.permutation(n)[:8].astype(np.int32)).to(DEV)
    ids_host = ids.cpu().long()
    n_steps = 6
    first = 100  # the sequence holds `first + s` tokens before step s's row
    rows_k = torch.randn(n_steps, L, 1, H, 1, D, device=DEV).to(torch.bfloat16)
    rows_v = torch.randn(n_steps, L, 1, H, 1, D, device=DEV).to(torch.bfloat16)
    slots = [torch.tensor([int(ids_host[(first + s) // bs]) * bs + (first + s) % bs], dtype=torch.int32,
                          device=DEV) for s in range(n_steps)]
    outs = []

    def chain():
        outs.clear()
        for s in range(n_steps):
            for layer in range(L):
                K.kv_scatter(pool, slots[s], layer, rows_k[s, layer], rows_v[s, layer])
                outs.append(K.kv_gather(pool, ids, layer, first + s + 1))

    if graph:
        pool_before = pool.clone()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            chain()
        pool.copy_(pool_before)  # capturing ran nothing, but start from the same bytes regardless
        g.replay()
    else:
        chain()
    torch.cuda.synchronize()
    i = 0
    for s in range(n_steps):
        pos = first + s
        b = int(ids_host[pos // bs])
        for layer in range(L):
            host[b, layer, 0, :, pos % bs, :] = rows_k[s, layer, 0, :, 0, :].cpu()
            host[b, layer, 1, :, pos % bs, :] = rows_v[s, layer, 0, :, 0, :].cpu()
            data = host[ids_host, layer]
            want_k = data[:, 0].permute(1, 0, 2, 3).reshape(1, H, -1, D)[:, :, :pos + 1]
            want_v = data[:, 1].permute(1, 0, 2, 3).reshape(1, H, -1, D)[:, :, :pos + 1]
            k, v = outs[i]
            i += 1
            assert torch.equal(k.cpu(), want_k) and torch.equal(v.cpu(), want_v), (s, layer)
    assert torch.equal(pool.cpu(), host)
