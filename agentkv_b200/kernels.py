"""Block-movement entry points: the drop-in for agentkv/core/triton_kernels.py.

``copy_block(src, dst)`` and ``zero_block(block)`` keep the reference's
signatures (triton_kernels.py:171, :206) and are what SlabAllocator calls;
``copy_blocks`` / ``zero_blocks`` take a whole batch of block ids in one
launch.  Every call goes to the sm_100a kernels of libagentkv_b200.so through
its C ABI; there is no Triton, no multi-backend dispatch and no CPU path.
A CPU tensor is rejected.  A ``meta`` tensor (the metadata-only pools the
vLLM / SGLang adapters build) holds no bytes, so there is nothing to move and
the call returns.

Semantics: copy is byte-identical.  zero writes +0.0 (all bits clear) like the
reference's CPU path ``block.zero_()``; the reference's Triton kernel stores
``x * 0`` instead (-0.0 for negative inputs, NaN for NaN/Inf).
"""

from __future__ import annotations

import weakref
from typing import Optional, Sequence, Tuple

import torch

from . import _native as N

_STATUS: dict = {}


def _status_buffer(device: torch.device) -> torch.Tensor:
    """A scratch AkvStatus for calls that do not pass their own: one per
    device and current stream, so launches on different streams never share
    one (the block copy keeps its work counter in it)."""
    key = (device.type, device.index, stream_handle(device) if device.type == "cuda" else 0)
    buf = _STATUS.get(key)
    if buf is None:
        buf = torch.zeros(N.STATUS_BYTES // 4, dtype=torch.int32, device=device)
        _STATUS[key] = buf
    return buf


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device) -> int:
    """The device's current CUDA stream as a raw handle (the cheap accessor
    when torch has it: this runs on every launch)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if _RAW_STREAM is not None:
        return _RAW_STREAM(idx)
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, what: str) -> bool:
    """True for a CUDA tensor, False for meta (nothing to do); raises otherwise."""
    if t.device.type == "cuda":
        return True
    if t.device.type == "meta":
        return False
    raise ValueError(
        f"{what}: agentkv_b200 moves KV blocks with its CUDA kernels only; "
        f"got a {t.device.type} tensor"
    )


def read_status(status: torch.Tensor) -> tuple:
    """(code, index, id, observed, aux) of a device AkvStatus; synchronises."""
    s = status.cpu()
    aux = int(s[4].item()) | (int(s[5].item()) << 32)
    return int(s[0]), int(s[1]), int(s[2]), int(s[3]), aux


def raise_for_status(status: torch.Tensor, clear: bool = True) -> None:
    code, index, bid, observed, aux = read_status(status)
    if code == 0:
        return
    if clear:
        status.zero_()
    raise BlockOpError(code, index, bid, observed, aux)


class BlockOpError(RuntimeError):
    """A device-detected failure of a batched block operation."""

    def __init__(self, code: int, index: int, block_id: int, observed: int, aux: int = 0) -> None:
        self.code, self.index, self.block_id, self.observed, self.aux = code, index, block_id, observed, aux
        super().__init__(
            f"{N.ERROR_NAMES.get(code, code)} at batch position {index}: "
            f"block {block_id} (observed {observed})"
        )


# ── drop-ins for triton_kernels.copy_block / zero_block ──────────────────────
def copy_block(src: torch.Tensor, dst: torch.Tensor) -> None:
    """Copy one KV block (triton_kernels.py:171-203).  Two contiguous CUDA
    blocks of one dtype that lie a whole number of blocks apart — two block
    views of one pool tensor, as SlabAllocator passes them — are copied by
    akv_copy_blocks.  Any other pair of tensors of one shape is copied with
    dst.copy_(src), the reference's own path for tensors its kernel does not
    take (triton_kernels.py:184-196)."""
    assert src.shape == dst.shape, f"Shape mismatch: {src.shape} vs {dst.shape}"
    if not _require_cuda(src, "copy_block"):
        return
    nbytes = src.numel() * src.element_size()
    if nbytes == 0:
        return
    a, b = src.data_ptr(), dst.data_ptr()
    base = min(a, b)
    one_pool = (src.is_contiguous() and dst.is_contiguous() and src.dtype == dst.dtype
                and src.device == dst.device and (max(a, b) - base) % nbytes == 0
                and (max(a, b) - base) // nbytes < (1 << 31) - 1)
    if not one_pool:
        dst.copy_(src)
        return
    pairs = torch.tensor([[(a - base) // nbytes, (b - base) // nbytes]], dtype=torch.int32, device=src.device)
    total = (max(a, b) - base) // nbytes + 1
    N.check(
        N.lib.akv_copy_blocks(base, nbytes, total, pairs.data_ptr(), 1, None, None, stream_handle(src.device))
    )


def zero_block(block: torch.Tensor) -> None:
    """Zero one KV block with +0.0 (triton_kernels.py:206-229)."""
    if not _require_cuda(block, "zero_block"):
        return
    if not block.is_contiguous():
        raise ValueError("zero_block: block must be contiguous")
    nbytes = block.numel() * block.element_size()
    if nbytes == 0:
        return
    ids = torch.zeros(1, dtype=torch.int32, device=block.device)
    N.check(N.lib.akv_zero_blocks(block.data_ptr(), nbytes, 1, ids.data_ptr(), 1, None, None,
                                  stream_handle(block.device)))


# ── batched block movement ───────────────────────────────────────────────────
def claimed_variant(pool: torch.Tensor) -> int:
    """The automatic copy variant of copy_blocks, whose status record belongs
    to one stream (no other launch with that record overlaps its copies on
    the GPU): the bulk copy of 32 KiB x 6 chunks per SM whose items are
    claimed 128 KiB at a time from a counter in that record.  On seeded
    disjoint pairs of 2 MiB blocks it copied 512 / 4,096 pairs in 0.324 /
    2.533 ms against 0.346 / 2.750 ms for the statically dealt 16 KiB x 12
    copy the library's own automatic choice makes.  Measured on Tree-of-Thought steps
    (8 children per source, the allocator's kernels of the next fan-out on a
    side stream): the copy launch in the step took 0.2245 / 0.226 / 0.235 /
    0.235 ms for whole 2 MiB blocks and 1 MiB / 512 KiB / 256 KiB head slices,
    against 0.2316 / 0.263 / 0.272 / 0.250 ms for the statically dealt copy
    the automatic choice makes.  Pools whose blocks are not 16-byte aligned
    keep the automatic choice (vector copies)."""
    total, bpb = _pool_geometry(pool)
    aligned = pool.data_ptr() % 16 == 0 and bpb % 16 == 0
    return N.VARIANT_CLAIMED_32K if aligned else N.VARIANT_AUTO


def _pool_geometry(pool: torch.Tensor) -> tuple:
    if pool.dim() < 1 or not pool.is_contiguous():
        raise ValueError("pool must be a contiguous tensor whose first dim indexes blocks")
    total = pool.shape[0]
    bpb = (pool.numel() // max(total, 1)) * pool.element_size()
    return total, bpb


def _as_device_i32(x, device: torch.device) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        if x.dtype != torch.int32:
            x = x.to(torch.int32)
        if x.device != device:
            x = x.to(device, non_blocking=True)
        return x.contiguous()
    return torch.as_tensor(x, dtype=torch.int32).to(device, non_blocking=True)


def copy_blocks(
    pool: torch.Tensor,
    pairs,
    *,
    ref_counts: Optional[torch.Tensor] = None,
    status: Optional[torch.Tensor] = None,
    variant: int = N.VARIANT_AUTO,
    check: bool = False,
    validate: bool = False,
) -> None:
    """Copy a batch of (src, dst) block pairs of `pool` in one launch.

    The pairs must be independent (no dst repeated, no dst used as another
    pair's src); `validate=True` checks that on the host before launching.
    With `ref_counts` every dst must have refcount 1.  Device-detected errors
    land in `status` (by default a buffer of this device and stream) and
    raise on `check=True` (which synchronises).  The automatic variant is
    the claimed bulk copy (claimed_variant), which keeps a work counter in
    the status record: a record passed in must not be in use by another
    launch that overlaps this one on the GPU (one record per stream).
    """
    if not _require_cuda(pool, "copy_blocks"):
        return
    total, bpb = _pool_geometry(pool)
    pairs_t = _as_device_i32(pairs, pool.device).reshape(-1, 2)
    n = pairs_t.shape[0]
    if n == 0:
        return
    if validate:
        validate_pairs(pairs_t.cpu().numpy(), total)
    st = status if status is not None else _status_buffer(pool.device)
    if variant == N.VARIANT_AUTO:
        variant = claimed_variant(pool)
    N.check(
        N.lib.akv_copy_blocks_variant(
            pool.data_ptr(), bpb, total, pairs_t.data_ptr(), n,
            ref_counts.data_ptr() if ref_counts is not None else None, st.data_ptr(), int(variant),
            stream_handle(pool.device),
        )
    )
    if check:
        raise_for_status(st)


def copy_blocks_counted(
    pool: torch.Tensor,
    pairs: torch.Tensor,
    count: torch.Tensor,
    *,
    ref_counts: Optional[torch.Tensor] = None,
    status: Optional[torch.Tensor] = None,
) -> None:
    """copy_blocks where the number of valid pairs lives on the device:
    `pairs` is a device int32 [n_max, 2] buffer, `count` a device int64
    tensor whose first element says how many of its rows to copy (capped at
    n_max; read by the kernel, never by the host)."""
    if not _require_cuda(pool, "copy_blocks_counted"):
        return
    total, bpb = _pool_geometry(pool)
    if pairs.dtype != torch.int32 or pairs.device != pool.device or not pairs.is_contiguous():
        raise ValueError("copy_blocks_counted: pairs must be a contiguous int32 tensor on the pool's device")
    if count.dtype != torch.int64 or count.device != pool.device or count.numel() < 1:
        raise ValueError("copy_blocks_counted: count must be an int64 tensor on the pool's device")
    n_max = pairs.numel() // 2
    st = status if status is not None else _status_buffer(pool.device)
    N.check(
        N.lib.akv_copy_blocks_counted(
            pool.data_ptr(), bpb, total, pairs.data_ptr(), n_max, count.data_ptr(),
            ref_counts.data_ptr() if ref_counts is not None else None, st.data_ptr(),
            stream_handle(pool.device),
        )
    )


_CACHE_TABLES: dict = {}


def _cache_table(caches: Sequence[torch.Tensor]) -> Tuple[torch.Tensor, int, int, int]:
    """Device table of the caches' base addresses plus (num_blocks,
    block_bytes, block_stride), validated once per set of cache tensors (the
    same tensor objects, in the same order, reuse the table)."""
    if not caches:
        raise ValueError("copy_blocks_layers: no caches")
    key = tuple(map(id, caches))
    hit = _CACHE_TABLES.get(key)
    if hit is not None and all(r() is c for r, c in zip(hit[0], caches)):
        return hit[1]
    # new tensor objects over the same memory (an engine slicing K and V out
    # of per-layer tensors on every call): reuse the table by address
    akey = tuple((c.data_ptr(), c.stride(0), c.shape[0], c.numel(), c.element_size()) for c in caches)
    hit = _CACHE_TABLES.get(akey)
    if hit is not None:
        return hit[1]
    dev = caches[0].device
    n = caches[0].shape[0]
    esz = caches[0].element_size()
    block_bytes = (caches[0].numel() // max(n, 1)) * esz
    stride = caches[0].stride(0) * esz
    for c in caches:
        if c.device != dev:
            raise ValueError("copy_blocks_layers: caches on different devices")
        if c.shape[0] != n or (c.numel() // max(n, 1)) * c.element_size() != block_bytes:
            raise ValueError("copy_blocks_layers: caches differ in block count or block size")
        if c.stride(0) * c.element_size() != stride or not c[0].is_contiguous():
            raise ValueError("copy_blocks_layers: every cache must hold each block as one span, "
                             "all with the same block stride")
        if c.data_ptr() % 16:
            raise ValueError("copy_blocks_layers: cache base not 16-byte aligned")
    if block_bytes % 16 or stride % 16 or stride < block_bytes:
        raise ValueError(f"copy_blocks_layers: block bytes {block_bytes} / stride {stride} must be "
                         "multiples of 16 with stride >= bytes")
    table = torch.tensor([c.data_ptr() for c in caches], dtype=torch.int64).to(dev)
    if len(_CACHE_TABLES) >= 32:
        _CACHE_TABLES.clear()
    res = (table, n, block_bytes, stride)
    _CACHE_TABLES[key] = ([weakref.ref(c) for c in caches], res)
    _CACHE_TABLES[akey] = (None, res)
    return res


def copy_blocks_layers(caches: Sequence[torch.Tensor], pairs, *, status: Optional[torch.Tensor] = None,
                       variant: int = 0, check: bool = False) -> None:
    """Copy every (src, dst) block pair in each of `caches` (tensors whose
    first dim indexes blocks, e.g. one K and one V cache per layer) in one
    launch; pairs must be independent."""
    if caches and caches[0].device.type == "meta":
        return
    if not caches or not _require_cuda(caches[0], "copy_blocks_layers"):
        return
    table, n_blocks, block_bytes, stride = _cache_table(caches)
    dev = caches[0].device
    pairs_t = _as_device_i32(pairs, dev).reshape(-1, 2)
    if pairs_t.shape[0] == 0:
        return
    st = status if status is not None else _status_buffer(dev)
    N.check(N.lib.akv_copy_blocks_layers(
        table.data_ptr(), len(caches), block_bytes, stride, n_blocks, pairs_t.data_ptr(), pairs_t.shape[0],
        None, st.data_ptr(), int(variant), stream_handle(dev)))
    if check:
        raise_for_status(st)


def copy_blocks_vllm(key_caches: Sequence[torch.Tensor], value_caches: Sequence[torch.Tensor],
                     block_mapping, *, variant: int = 0) -> None:
    """Drop-in for vLLM's `copy_blocks(key_caches, value_caches,
    block_mapping)`: the blocks_to_copy pairs that the reference's vLLM
    adapter returns from append_slots (integrations/vllm/block_manager.py:
    134-167), applied to every layer's K and V cache in one launch."""
    copy_blocks_layers(list(key_caches) + list(value_caches), block_mapping, variant=variant)


def _kv_geometry(pool: torch.Tensor) -> Tuple[int, int, int, int, int, int]:
    """(total_blocks, layers, heads, block_size, head_dim, row_bytes) of a
    contiguous [N, L, 2, H, bs, D] pool."""
    if pool.dim() != 6 or pool.shape[2] != 2 or not pool.is_contiguous():
        raise ValueError("kv pool must be a contiguous [blocks, layers, 2, heads, block_size, head_dim] tensor")
    n, L, _, H, bs, D = pool.shape
    return n, L, H, bs, D, D * pool.element_size()


def kv_gather(pool: torch.Tensor, block_ids, layer: int, n_tokens: int, *,
              status: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Layer `layer`'s K and V of a sequence stored in blocks `block_ids`, as
    two contiguous [1, heads, n_tokens, head_dim] tensors, in one launch."""
    n, L, H, bs, D, row = _kv_geometry(pool)
    dev = pool.device
    ids = _as_device_i32(block_ids, dev).reshape(-1)
    out = torch.empty((2, 1, H, n_tokens, D), dtype=pool.dtype, device=dev)  # one allocation for K and V
    out_k, out_v = out[0], out[1]
    if n_tokens == 0 or not _require_cuda(pool, "kv_gather"):
        return out_k, out_v
    st = status if status is not None else _status_buffer(dev)
    N.check(N.lib.akv_kv_gather(pool.data_ptr(), n, L, H, bs, row, int(layer), ids.data_ptr(), ids.numel(),
                                int(n_tokens), out_k.data_ptr(), out_v.data_ptr(), st.data_ptr(),
                                stream_handle(dev)))
    return out_k, out_v


def kv_scatter(pool: torch.Tensor, slots, layer: int, key_states: torch.Tensor, value_states: torch.Tensor, *,
               status: Optional[torch.Tensor] = None) -> None:
    """Write new tokens' K and V rows ([1, heads, n, head_dim] states, head_dim
    contiguous) of layer `layer` to pool slots (block * block_size + position)
    in one launch."""
    n, L, H, bs, D, row = _kv_geometry(pool)
    if not _require_cuda(pool, "kv_scatter"):
        return
    dev = pool.device
    # states in another dtype or on another device are converted, as the
    # reference's indexed assignment into the pool converts them
    k = key_states[0].to(device=dev, dtype=pool.dtype)
    v = value_states[0].to(device=dev, dtype=pool.dtype)
    for t in (k, v):
        if t.shape != (H, k.shape[1], D):
            raise ValueError(f"kv_scatter: states must be [1, {H}, n, {D}], got {tuple(t.shape)}")
    if k.stride() != v.stride() or k.stride(2) != 1:
        k, v = k.contiguous(), v.contiguous()
    s = _as_device_i32(slots, dev).reshape(-1)
    if s.numel() != k.shape[1]:
        raise ValueError("kv_scatter: one slot per new token")
    esz = pool.element_size()
    st = status if status is not None else _status_buffer(dev)
    N.check(N.lib.akv_kv_scatter(pool.data_ptr(), n, L, H, bs, row, int(layer), s.data_ptr(), s.numel(),
                                 k.data_ptr(), v.data_ptr(), k.stride(0) * esz, k.stride(1) * esz,
                                 st.data_ptr(), stream_handle(dev)))


def zero_blocks(
    pool: torch.Tensor,
    ids,
    *,
    ref_counts: Optional[torch.Tensor] = None,
    status: Optional[torch.Tensor] = None,
    variant: int = N.VARIANT_AUTO,
    check: bool = False,
) -> None:
    """Write +0.0 over a batch of blocks of `pool` in one launch."""
    if not _require_cuda(pool, "zero_blocks"):
        return
    total, bpb = _pool_geometry(pool)
    ids_t = _as_device_i32(ids, pool.device).reshape(-1)
    n = ids_t.shape[0]
    if n == 0:
        return
    st = status if status is not None else _status_buffer(pool.device)
    N.check(
        N.lib.akv_zero_blocks_variant(
            pool.data_ptr(), bpb, total, ids_t.data_ptr(), n,
            ref_counts.data_ptr() if ref_counts is not None else None, st.data_ptr(), int(variant),
            stream_handle(pool.device),
        )
    )
    if check:
        raise_for_status(st)


def check_pairs_on_device(pairs: torch.Tensor, total_blocks: int, mark: torch.Tensor,
                          status: torch.Tensor) -> None:
    """Enqueue the device-side independence check (akv_check_pairs)."""
    pairs = pairs.reshape(-1, 2)
    N.check(N.lib.akv_check_pairs(pairs.data_ptr(), pairs.shape[0], total_blocks, mark.data_ptr(),
                                  status.data_ptr(), stream_handle(pairs.device)))


def validate_pairs(pairs, total_blocks: int) -> None:
    """Host check that a pair batch is in range and independent."""
    import numpy as np

    p = np.asarray(pairs, dtype=np.int64).reshape(-1, 2)
    if p.size == 0:
        return
    if p.min() < 0 or p.max() >= total_blocks:
        raise ValueError(f"copy_blocks: block id out of range [0, {total_blocks})")
    src, dst = p[:, 0], p[:, 1]
    if len(np.unique(dst)) != len(dst):
        raise ValueError("copy_blocks: a dst block appears twice in the batch")
    moving = src != dst
    if np.intersect1d(src[moving], dst).size:
        raise ValueError("copy_blocks: a dst block is also read as another pair's src")


def is_native_available() -> bool:
    return N.LIB_PATH.exists() and torch.cuda.is_available()


def is_triton_available() -> bool:
    """triton_kernels.is_triton_available (triton_kernels.py:232): whether
    block moves run as Triton kernels — never here (they run as this
    library's CUDA kernels; see is_native_available)."""
    return False


def kernel_info() -> dict:
    gpu = torch.cuda.get_device_name(0) if torch.cuda.is_available() else "N/A"
    cap = torch.cuda.get_device_capability(0) if torch.cuda.is_available() else None
    major, minor = N.version()
    return {
        "library": str(N.LIB_PATH),
        "library_version": f"{major}.{minor}",
        "cuda_available": torch.cuda.is_available(),
        "gpu_name": gpu,
        "gpu_arch": f"sm_{cap[0]}{cap[1]}" if cap else "cpu",
        "kernels": "sm_100a: vectorised / bulk-async block copy, write-only zero, "
        "device free list + refcounts, warp-per-query match_prefix",
        "fallback": None,
    }
