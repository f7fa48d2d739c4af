"""Block copies across a serving engine's per-layer KV caches (the vLLM
consumer of the reference's recorded CoW pairs) against the oracle: every
layer's K and V cache must equal the oracle's sequential copy, bit for bit,
in both of vLLM's cache layouts."""

import numpy as np
import pytest
import torch

from agentkv_b200 import _native as N
from agentkv_b200 import kernels as K
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _rand(shape, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    t = torch.empty(shape, dtype=dtype, device=DEV)
    t.view(torch.int16).random_(-30000, 30000, generator=g)
    return t


def _host_blocks(t):
    return t.view(torch.uint8).reshape(t.shape[0], -1).cpu().numpy().copy()


def _pairs(n_blocks, n, seed):
    perm = np.random.default_rng(seed).permutation(n_blocks)[: 2 * n].astype(np.int32)
    return np.stack([perm[:n], perm[n:]], 1).copy()


@pytest.mark.parametrize("variant", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("n_layers,n_blocks,bs,H,D", [(4, 64, 16, 2, 64), (32, 40, 16, 8, 128), (3, 17, 8, 1, 8)])
def test_flash_layout_kv_caches(n_layers, n_blocks, bs, H, D, variant):
    """vLLM's flash-attention layout: one [2, N, bs, H, D] tensor per layer."""
    kv = [_rand((2, n_blocks, bs, H, D), torch.bfloat16, 100 + i) for i in range(n_layers)]
    keys, values = [t[0] for t in kv], [t[1] for t in kv]
    host = [_host_blocks(t) for t in keys + values]
    for n in (1, 5, n_blocks // 2):
        pairs = _pairs(n_blocks, n, n)
        for h in host:
            O.copy_blocks(h, h.shape[1], pairs)
        K.copy_blocks_vllm(keys, values, torch.from_numpy(pairs).long(), variant=variant)
        torch.cuda.synchronize()
        for c, h in zip(keys + values, host):
            assert np.array_equal(_host_blocks(c), h), n
    assert K.read_status(K._status_buffer(DEV))[0] == 0


def test_paged_layout_key_value_lists():
    """vLLM's paged-attention layout: key caches [N, H, D/x, bs, x] and value
    caches [N, H, D, bs] as separate per-layer lists."""
    n_layers, n_blocks, H, D, bs, x = 3, 50, 4, 64, 16, 8
    keys = [_rand((n_blocks, H, D // x, bs, x), torch.float16, 200 + i) for i in range(n_layers)]
    values = [_rand((n_blocks, H, D, bs), torch.float16, 300 + i) for i in range(n_layers)]
    host = [_host_blocks(t) for t in keys + values]
    pairs = _pairs(n_blocks, 20, 7)
    for h in host:
        O.copy_blocks(h, h.shape[1], pairs)
    K.copy_blocks_vllm(keys, values, pairs.tolist())
    torch.cuda.synchronize()
    for c, h in zip(keys + values, host):
        assert np.array_equal(_host_blocks(c), h)


def test_layers_errors():
    kv = [_rand((2, 32, 16, 2, 64), torch.bfloat16, 400 + i) for i in range(2)]
    caches = [t[0] for t in kv] + [t[1] for t in kv]
    before = [_host_blocks(c) for c in caches]
    st = torch.zeros(8, dtype=torch.int32, device=DEV)
    K.copy_blocks_layers(caches, torch.tensor([[1, 2], [3, 99]]), status=st)
    code, idx, bid, _, _ = K.read_status(st)
    assert (code, idx, bid) == (N.AKV_ERR_OUT_OF_RANGE, 1, 99)
    for h in before:
        O.copy_blocks(h, h.shape[1], np.array([[1, 2]], np.int32))
    for c, h in zip(caches, before):
        assert np.array_equal(_host_blocks(c), h)
    # mismatched caches are rejected on the host, before any launch
    with pytest.raises(ValueError):
        K.copy_blocks_layers(caches + [_rand((16, 16, 2, 64), torch.bfloat16, 9)], [[0, 1]])
    with pytest.raises(ValueError):
        K.copy_blocks_layers([_rand((32, 3, 2), torch.bfloat16, 9)], [[0, 1]])  # 12-byte blocks
