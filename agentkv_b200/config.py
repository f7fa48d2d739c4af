"""PoolConfig — pool geometry and validation.

Same fields, defaults, validation and error messages as the reference's
PoolConfig (agentkv/core/config.py:21-224), so a config built for the
reference builds the same pool here.  ``bytes_per_block`` is
``num_layers * 2 * num_kv_heads * block_size * head_dim * bytes_per_element``
(agentkv/core/config.py:92-98): one block is one contiguous span of the pool
tensor ``[total_blocks, num_layers, 2, num_kv_heads, block_size, head_dim]``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Literal

_DTYPE_BYTES = {"float16": 2, "bfloat16": 2, "float32": 4}


@dataclass
class PoolConfig:
    """Configuration of an AgentKV block pool (see the module docstring)."""

    total_blocks: int = 4096
    block_size: int = 16
    num_layers: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    dtype: Literal["float16", "bfloat16", "float32"] = "float16"
    device: str = "cuda"
    max_agents: int = 1024
    epoch_interval: int = 64

    bytes_per_element: int = field(init=False, repr=False)
    bytes_per_block: int = field(init=False, repr=False)

    def __post_init__(self) -> None:
        if self.dtype not in _DTYPE_BYTES:
            raise ValueError(f"dtype must be one of {list(_DTYPE_BYTES)}, got '{self.dtype}'")
        self.bytes_per_element = _DTYPE_BYTES[self.dtype]
        if self.block_size <= 0 or (self.block_size & (self.block_size - 1)) != 0:
            raise ValueError(f"block_size must be a positive power of 2, got {self.block_size}")
        if self.total_blocks <= 0:
            raise ValueError(f"total_blocks must be > 0, got {self.total_blocks}")
        if self.max_agents <= 0:
            raise ValueError(f"max_agents must be > 0, got {self.max_agents}")
        elements = self.num_layers * 2 * self.num_kv_heads * self.block_size * self.head_dim
        self.bytes_per_block = elements * self.bytes_per_element

    @property
    def total_bytes(self) -> int:
        return self.total_blocks * self.bytes_per_block

    @property
    def total_gb(self) -> float:
        return self.total_bytes / (1024**3)

    @classmethod
    def from_capacity_gb(
        cls,
        capacity_gb: float,
        block_size: int = 16,
        num_layers: int = 32,
        num_kv_heads: int = 8,
        head_dim: int = 128,
        dtype: str = "float16",
        device: str = "cuda",
        **kwargs,
    ) -> "PoolConfig":
        """Largest power-of-two block count whose pool fits in capacity_gb GiB."""
        bytes_per_elem = _DTYPE_BYTES[dtype]
        bytes_per_block = num_layers * 2 * num_kv_heads * block_size * head_dim * bytes_per_elem
        raw_blocks = int(capacity_gb * (1024**3)) // bytes_per_block
        if raw_blocks <= 0:
            raise ValueError(
                f"capacity_gb={capacity_gb} is too small for the given block geometry"
            )
        total_blocks = 2 ** math.floor(math.log2(raw_blocks))
        return cls(
            total_blocks=total_blocks,
            block_size=block_size,
            num_layers=num_layers,
            num_kv_heads=num_kv_heads,
            head_dim=head_dim,
            dtype=dtype,
            device=device,
            **kwargs,
        )

    @classmethod
    def max_for_device(
        cls,
        fraction: float = 0.7,
        block_size: int = 16,
        num_layers: int = 32,
        num_kv_heads: int = 8,
        head_dim: int = 128,
        dtype: str = "float16",
        device: str = "cuda",
        **kwargs,
    ) -> "PoolConfig":
        """Pool sized to `fraction` of the device's currently free memory."""
        import torch

        if not torch.cuda.is_available():
            raise RuntimeError(
                "max_for_device() requires a CUDA GPU. "
                "Use PoolConfig(total_blocks=...) for CPU pools."
            )
        free_bytes, _ = torch.cuda.mem_get_info(device if device != "cpu" else 0)
        return cls.from_capacity_gb(
            capacity_gb=free_bytes * fraction / (1024**3),
            block_size=block_size,
            num_layers=num_layers,
            num_kv_heads=num_kv_heads,
            head_dim=head_dim,
            dtype=dtype,
            device=device,
            **kwargs,
        )

    def __repr__(self) -> str:
        return (
            f"PoolConfig("
            f"total_blocks={self.total_blocks}, "
            f"block_size={self.block_size}, "
            f"layers={self.num_layers}, "
            f"kv_heads={self.num_kv_heads}, "
            f"head_dim={self.head_dim}, "
            f"dtype={self.dtype}, "
            f"device={self.device}, "
            f"pool_size={self.total_gb:.2f} GiB"
            f")"
        )


def torch_dtype(name: str):
    import torch

    table = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}
    if name not in table:
        raise ValueError(f"Unknown dtype '{name}'")
    return table[name]
