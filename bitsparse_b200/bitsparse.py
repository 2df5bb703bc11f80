"""The tile-wise bitmask sparse format: BitsparseTensor and TensorBuffer.

Same classes, fields and constructor signatures as lib_sparse/bitsparse.py
(Maxzhu123/bitsparse), so code written against the reference's format
objects runs unchanged.
"""
from __future__ import annotations

import torch
from torch import Tensor

from .fp8 import is_fp8
from .src.bitpacking import packed_nbytes


def pack_codec(dtype) -> int:
    """Packed-bitstream codec of a storage dtype (lib_sparse/bitsparse.py:8-18):
    0 = bf16 (15 bits/value), 1 = e4m3fn, 2 = e5m2 (7 bits/value)."""
    if dtype == torch.float8_e4m3fn:
        return 1
    if dtype == torch.float8_e5m2:
        return 2
    return 0


def bits_per_value(dtype) -> int:
    """Bits each value occupies in the packed stream (lib_sparse/bitsparse.py:21-23)."""
    return 7 if pack_codec(dtype) else 15


class BitsparseTensor:
    """Tile-wise bitmask sparse tensor of a dense [M, N] matrix
    (lib_sparse/bitsparse.py:26-87).

    vals        positive entries in (tile, row, col) order, storage dtype; with
                ``pack_sbit`` a uint8 15/7-bit stream.
    bitmask     uint8[T*512], one bit per element, LSB first, row-major in tile.
    prefix      uint32[T+1], prefix[t] = logical offset of tile t's values.
    vals_offset int64 tensor: logical index of this tensor's first value in
                ``vals`` (0 unless ``vals`` is a shared TensorBuffer arena).
    scale       fp32 0-dim per-tensor FP8 scale, or None.
    tile_scales fp32[T] per-tile FP8 scales (the per-tile scale mode, an
                extension of the reference's per-tensor format), or None.
    """

    def __init__(self, vals, bitmask, prefix, shape, dtype,
                 grid_m, grid_n, BLOCK_M, BLOCK_N,
                 scale=None, vals_offset=None, pack_sbit=False, tile_scales=None):
        self.vals = vals
        self.bitmask = bitmask
        self.prefix = prefix
        if vals_offset is None:
            vals_offset = torch.tensor(0, device=vals.device, dtype=torch.int64)
        self.vals_offset = vals_offset
        self.pack_sbit = pack_sbit
        self.dtype = dtype
        self.scale = scale
        self.tile_scales = tile_scales
        self.grid_m = grid_m
        self.grid_n = grid_n
        self.BLOCK_M = BLOCK_M
        self.BLOCK_N = BLOCK_N
        self.shape = shape

    @property
    def fp8(self) -> bool:
        """True when values are stored as FP8 (e4m3fn or e5m2)."""
        return is_fp8(self.dtype)

    def __repr__(self):
        return (f"BitsparseTensor(shape={list(self.shape)}, "
                f"nnz={self.nnz()}, sparsity={self.sparsity_ratio():.2f}, "
                f"pack_sbit={self.pack_sbit})")

    def nnz(self):
        """Total nonzeros (the last prefix entry, as a 0-dim tensor)."""
        return self.prefix[-1].to(torch.int64)

    def vram_size(self):
        """Bytes held by this tensor's values, bitmask and prefix (syncs)."""
        nnz = int(self.prefix[-1].item())
        if self.pack_sbit:
            val_size = packed_nbytes(nnz, bits_per_value(self.dtype))
        else:
            val_size = nnz * self.vals.element_size()
        bitmask_size = self.bitmask.element_size() * self.bitmask.nelement()
        prefix_size = self.prefix.element_size() * self.prefix.nelement()
        return val_size + bitmask_size + prefix_size

    def sparsity_ratio(self):
        return 1 - self.nnz() / (self.shape[0] * self.shape[1])


class TensorBuffer:
    """Preallocated value arena shared by several BitsparseTensors
    (lib_sparse/bitsparse.py:90-117).  ``offset`` is a device int64[1]
    running logical offset; compressing into the buffer advances it on the
    device without a host sync."""

    def __init__(self, size: int, device="cuda", dtype=torch.bfloat16,
                 pack_sbit: bool = False):
        """size: storage bytes; dtype: logical dtype of stored values."""
        self.size = size
        self.device = device
        self.dtype = dtype
        self.pack_sbit = pack_sbit
        if pack_sbit:
            storage_size = (self.size + 3) // 4 * 4 + 4
            self.vals = torch.zeros(storage_size, device=self.device, dtype=torch.uint8)
        else:
            elt = torch.empty((), dtype=dtype).element_size()
            if self.size % elt != 0:
                raise ValueError("raw TensorBuffer size must be a multiple of dtype size")
            self.vals = torch.zeros(self.size // elt, device=self.device, dtype=self.dtype)
        self.offset = torch.zeros(1, device=self.device, dtype=torch.int64)

    def reset_buffer(self):
        """Restart filling from offset 0 (once per training step)."""
        self.offset = torch.zeros(1, device=self.device, dtype=torch.int64)


def tile_grid(M: int, N: int, BLOCK_M: int, BLOCK_N: int) -> tuple[int, int, int, int, int]:
    """(grid_m, grid_n, num_tiles, TILE_NUMEL, TILE_BYTES) (lib_sparse/bitsparse.py:120-127)."""
    TILE_NUMEL = BLOCK_M * BLOCK_N
    TILE_BYTES = TILE_NUMEL // 8
    grid_m = (M + BLOCK_M - 1) // BLOCK_M
    grid_n = (N + BLOCK_N - 1) // BLOCK_N
    num_tiles = grid_m * grid_n
    return grid_m, grid_n, num_tiles, TILE_NUMEL, TILE_BYTES
