"""Block copy / zero on the GPU against the oracle: bit-exact.

Small pools are compared byte for byte with the oracle's sequential
dst.copy_(src) / block.zero_() applied to a host copy of the same pool.  At
the full 60,000-block Llama-3-8B size the check is size-independent: after a
batch every dst equals its src (compared by torch), every zeroed block is
all-zero bits.
"""

import numpy as np
import pytest
import torch

from agentkv_b200 import _native as N
from agentkv_b200 import kernels as K
from agentkv_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)

# (total_blocks, bytes_per_block): the quickstart block, an odd 12-byte block,
# a 4-byte metadata-pool block, a 2 MiB Llama-3-8B block.
GEOMETRIES = [(64, 65536), (97, 12), (50, 4), (96, 2 * 1024 * 1024), (40, 1040)]


def random_pool(n, bpb, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    host = torch.randint(0, 256, (n, bpb), dtype=torch.uint8, generator=g)
    return host.numpy().copy(), host.to(DEV)


def random_pairs(n_blocks, n, seed):
    rng = np.random.default_rng(seed)
    perm = rng.permutation(n_blocks)[: 2 * n].astype(np.int32)
    return np.stack([perm[:n], perm[n:]], 1).copy()


@pytest.mark.parametrize("variant", [N.VARIANT_VEC, N.VARIANT_BULK, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 17, 18])
@pytest.mark.parametrize("n_blocks,bpb", GEOMETRIES)
def test_copy_blocks_bitexact(n_blocks, bpb, variant):
    host, pool = random_pool(n_blocks, bpb, seed=n_blocks + bpb)
    for n in (1, 3, n_blocks // 2):
        pairs = random_pairs(n_blocks, n, seed=n)
        O.copy_blocks(host, bpb, pairs)
        K.copy_blocks(pool, torch.from_numpy(pairs), variant=variant, check=True)
        torch.cuda.synchronize()
        assert np.array_equal(pool.cpu().numpy(), host), f"n={n}"


@pytest.mark.parametrize("variant", [14, 15, 16, 17, 18])
def test_dynamic_claims_counter_returns_to_zero(variant):
    """Variants 14-18 take their items from a counter in the status record's
    last word: after every launch — a clean one, one that meets a pair it
    must skip, one that starts with an error already recorded — the counter
    is zero again, and the bytes equal the oracle's (skipped pairs left
    alone, as the static shapes do)."""
    n_blocks, bpb = 64, 65536
    host, pool = random_pool(n_blocks, bpb, seed=5)
    st = torch.zeros(N.STATUS_BYTES // 4, dtype=torch.int32, device=DEV)

    def counter():
        return int(st.cpu().numpy().view(np.int64)[3])

    for n in (1, 7, 32):
        pairs = random_pairs(n_blocks, n, seed=100 + n)
        O.copy_blocks(host, bpb, pairs)
        K.copy_blocks(pool, torch.from_numpy(pairs), variant=variant, status=st)
        torch.cuda.synchronize()
        assert counter() == 0 and int(st[0]) == 0
        assert np.array_equal(pool.cpu().numpy(), host), f"n={n}"
    # a destination that is not exclusively owned: skipped and reported
    pairs = random_pairs(n_blocks, 16, seed=7)
    refs = torch.ones(n_blocks, dtype=torch.int32, device=DEV)
    refs[int(pairs[5, 1])] = 2
    O.copy_blocks(host, bpb, np.delete(pairs, 5, axis=0))
    K.copy_blocks(pool, torch.from_numpy(pairs), variant=variant, status=st, ref_counts=refs)
    torch.cuda.synchronize()
    assert int(st[0]) == N.AKV_ERR_NOT_EXCLUSIVE and counter() == 0
    assert np.array_equal(pool.cpu().numpy(), host)
    # an error already recorded: nothing is copied, the counter stays zero
    K.copy_blocks(pool, torch.from_numpy(random_pairs(n_blocks, 16, seed=8)), variant=variant, status=st)
    torch.cuda.synchronize()
    assert counter() == 0
    assert np.array_equal(pool.cpu().numpy(), host)


@pytest.mark.parametrize("variant", [N.VARIANT_VEC, N.VARIANT_BULK])
@pytest.mark.parametrize("n_blocks,bpb", GEOMETRIES)
def test_zero_blocks_bitexact(n_blocks, bpb, variant):
    host, pool = random_pool(n_blocks, bpb, seed=7 * n_blocks + bpb)
    rng = np.random.default_rng(bpb)
    for n in (1, 5, n_blocks // 3):
        ids = rng.choice(n_blocks, size=n, replace=False).astype(np.int32)
        O.zero_blocks(host, bpb, ids)
        K.zero_blocks(pool, torch.from_numpy(ids), variant=variant, check=True)
        assert np.array_equal(pool.cpu().numpy(), host), f"n={n}"


def test_zero_writes_positive_zero_bits():
    """+0.0 everywhere, also over negative values and NaN (the reference's CPU
    path; its Triton path would leave -0.0 / NaN)."""
    pool = torch.empty((8, 2, 2, 4, 16, 8), dtype=torch.bfloat16, device=DEV)
    pool[0].fill_(-1.5)
    pool[1].fill_(float("nan"))
    pool[2].fill_(float("-inf"))
    pool[3:].normal_()
    K.zero_blocks(pool, torch.tensor([0, 1, 2, 5]), check=True)
    bits = pool.view(torch.int16)
    for b in (0, 1, 2, 5):
        assert int(torch.count_nonzero(bits[b])) == 0
    assert int(torch.count_nonzero(bits[3])) > 0


def test_dropin_copy_block_and_zero_block():
    """kernels.copy_block / zero_block keep triton_kernels' signatures: two
    block views of one pool go through the library's copy, any other two
    tensors of one shape are copied as the reference copies them."""
    pool = torch.randn((16, 2, 2, 4, 16, 64), dtype=torch.float16, device=DEV)
    ref = pool.clone()
    K.copy_block(pool[3], pool[9])
    ref[9] = ref[3]
    K.copy_block(pool[12], pool[1])
    ref[1] = ref[12]
    K.zero_block(pool[5])
    ref[5] = 0
    torch.cuda.synchronize()
    assert torch.equal(pool.view(torch.int16), ref.view(torch.int16))
    with pytest.raises(AssertionError):
        K.copy_block(pool[0], pool[1, 0])
    with pytest.raises(ValueError):
        K.copy_block(pool[0].cpu(), pool[1].cpu())
    # any two CUDA tensors of one shape, as the reference's copy_block takes:
    # a block of another tensor, a strided view, a different dtype
    other = torch.randn((2, 2, 4, 16, 64), dtype=torch.float16, device=DEV)
    K.copy_block(other, pool[7])
    ref[7] = other
    strided = torch.randn((2, 2, 4, 64, 16), dtype=torch.float16, device=DEV).transpose(-1, -2)
    K.copy_block(strided, pool[8])
    ref[8] = strided
    wide = torch.randn((2, 2, 4, 16, 64), dtype=torch.float32, device=DEV)
    K.copy_block(wide, pool[10])
    ref[10] = wide.to(torch.float16)
    torch.cuda.synchronize()
    assert torch.equal(pool.view(torch.int16), ref.view(torch.int16))


def test_meta_blocks_are_noops():
    pool = torch.empty((4, 8), device="meta")
    K.copy_block(pool[0], pool[1])
    K.zero_block(pool[2])
    K.copy_blocks(pool, [[0, 1]])


def test_out_of_range_and_not_exclusive_are_reported():
    host, pool = random_pool(32, 256, 3)
    st = torch.zeros(8, dtype=torch.int32, device=DEV)
    K.copy_blocks(pool, torch.tensor([[1, 2], [5, 40]]), status=st)
    code, idx, bid, observed, _ = K.read_status(st)
    assert (code, idx, bid) == (N.AKV_ERR_OUT_OF_RANGE, 1, 40)
    # The valid pair was copied, the bad one skipped.
    O.copy_blocks(host, 256, np.array([[1, 2]], np.int32))
    assert np.array_equal(pool.cpu().numpy(), host)
    # Sticky: while the status holds an error nothing else runs.
    K.copy_blocks(pool, torch.tensor([[3, 4]]), status=st)
    assert np.array_equal(pool.cpu().numpy(), host)
    st.zero_()
    refs = torch.ones(32, dtype=torch.int32, device=DEV)
    refs[4] = 2
    K.copy_blocks(pool, torch.tensor([[3, 4]]), ref_counts=refs, status=st)
    code, idx, bid, observed, _ = K.read_status(st)
    assert (code, bid, observed) == (N.AKV_ERR_NOT_EXCLUSIVE, 4, 2)
    assert np.array_equal(pool.cpu().numpy(), host)
    with pytest.raises(K.BlockOpError):
        K.raise_for_status(st)
    assert K.read_status(st)[0] == 0


@pytest.mark.parametrize("pairs,bad", [
    ([[0, 1], [2, 3], [4, 5]], False),
    ([[0, 1], [2, 1]], True),          # dst twice
    ([[0, 1], [1, 2]], True),          # dst read by another pair
    ([[7, 7], [3, 4]], False),         # self pair is a no-op
])
def test_check_pairs_on_device(pairs, bad):
    mark = torch.zeros(16, dtype=torch.int32, device=DEV)
    st = torch.zeros(8, dtype=torch.int32, device=DEV)
    K.check_pairs_on_device(torch.tensor(pairs, dtype=torch.int32, device=DEV), 16, mark, st)
    code = K.read_status(st)[0]
    assert (code == N.AKV_ERR_DEPENDENT_PAIRS) == bad
    assert int(mark.abs().sum()) == 0


@pytest.mark.slow
def test_full_size_sweep_property():
    """Copy / zero sweep on the full 60,000-block Llama-3-8B pool (126 GB):
    after each batch every dst equals its src; zeroed blocks are all-zero."""
    n_blocks, bs, L, H, D, _ = W.LLAMA3_8B_GEOMETRY
    torch.cuda.synchronize()
    torch.cuda.empty_cache()  # blocks cached by earlier tests
    free, _ = torch.cuda.mem_get_info()
    if free < 130e9:
        pytest.skip(f"needs ~130 GB of free device memory, {free / 1e9:.0f} GB free")
    pool = torch.empty((n_blocks, L, 2, H, bs, D), dtype=torch.bfloat16, device=DEV)
    flat = pool.view(n_blocks, -1)
    for i in range(0, n_blocks, 4096):
        flat[i : i + 4096].view(torch.int16).random_(-32768, 32767)
    for variant in (N.VARIANT_VEC, N.VARIANT_BULK):
        for n in W.COPY_SWEEP_BATCHES:
            pairs = torch.from_numpy(W.copy_sweep_pairs(n, n_blocks, rotation=variant)).to(DEV)
            K.copy_blocks(pool, pairs, variant=variant, check=True)
            for c in range(0, n, 256):  # compare 256 pairs (1 GiB) at a time
                p = pairs[c : c + 256].long()
                assert torch.equal(flat[p[:, 0]].view(torch.int16), flat[p[:, 1]].view(torch.int16)), f"n={n}"
            K.zero_blocks(pool, pairs[:, 1], variant=variant, check=True)
            for c in range(0, n, 256):
                p = pairs[c : c + 256, 1].long()
                assert int(torch.count_nonzero(flat[p].view(torch.int16))) == 0, f"n={n}"
    del pool, flat
    torch.cuda.empty_cache()
