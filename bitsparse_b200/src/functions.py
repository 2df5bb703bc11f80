"""dense_to_tilesparse: the compression entry point (lib_sparse/src/functions.py).

The reference runs tile_pack, a torch.cumsum scan and compact_vals (three
launches, two reads of the dense tensor).  Here one fused kernel does all
of it; ``_prepare_tiles`` is kept for callers of the reference's two-step
API.
"""
from __future__ import annotations

from typing import NamedTuple

import torch
from torch import Tensor

from ..bitsparse import BitsparseTensor, TensorBuffer, tile_grid
from ..config import BLOCK_M, BLOCK_N
from ..fp8 import is_fp8
from .operators import compress, tile_pack


class _PreparedTiles(NamedTuple):
    M: int
    N: int
    grid_m: int
    grid_n: int
    num_tiles: int
    tile_numel: int
    bitmasks: Tensor
    prefix: Tensor


def _prepare_tiles(dense: Tensor) -> _PreparedTiles:
    """Bitmasks + uint32 prefix of per-tile counts (lib_sparse/src/functions.py:23-45)."""
    if dense.dtype != torch.bfloat16 and not is_fp8(dense.dtype):
        raise TypeError("BitsparseTensor supports bfloat16 and FP8 (e4m3fn/e5m2) values")
    M, N = dense.shape
    grid_m, grid_n, num_tiles, TILE_NUMEL, TILE_BYTES = tile_grid(M, N, BLOCK_M, BLOCK_N)
    tile_counts = torch.empty(num_tiles, device=dense.device, dtype=torch.int32)
    tile_bitmasks = torch.empty(num_tiles * TILE_BYTES, device=dense.device, dtype=torch.uint8)
    tile_pack(dense, tile_counts, tile_bitmasks,
              M, N, grid_m, grid_n, BLOCK_M, BLOCK_N, TILE_NUMEL, TILE_BYTES)
    tile_prefix = torch.zeros(num_tiles + 1, device=dense.device, dtype=torch.uint32)
    torch.cumsum(tile_counts, 0, out=tile_prefix.view(torch.int32)[1:])
    return _PreparedTiles(M, N, grid_m, grid_n, num_tiles, TILE_NUMEL,
                          tile_bitmasks, tile_prefix)


def dense_to_tilesparse(
    dense: Tensor, scale: Tensor | None,
    sparse_data: TensorBuffer | None = None,
    pack_sbit: bool = False,
) -> BitsparseTensor:
    """Convert a 2-D bf16 / fp8 tensor into a BitsparseTensor
    (lib_sparse/src/functions.py:55-99).

    ``scale`` is stored as metadata (the FP8 per-tensor scale the values
    were quantised with).  With ``sparse_data`` the values go into the shared
    TensorBuffer at its running offset (8-aligned when ``pack_sbit``) and the
    offset advances on the device; otherwise the values get their own
    exactly sized storage.
    """
    if dense.dtype != torch.bfloat16 and not is_fp8(dense.dtype):
        raise TypeError("BitsparseTensor supports bfloat16 and FP8 (e4m3fn/e5m2) values")
    return compress(dense, scale=scale, sparse_data=sparse_data, pack_sbit=pack_sbit)


def relu_to_tilesparse_fp8(h: Tensor, sparse_data: TensorBuffer | None = None,
                           pack_sbit: bool = False) -> tuple[Tensor, BitsparseTensor]:
    """``to_fp8`` followed by ``dense_to_tilesparse`` in two kernels.

    Equivalent to the reference's ``h_fp8, scale = to_fp8(h)`` then
    ``dense_to_tilesparse(h_fp8, scale, ...)`` (lib_sparse/layers.py:32-37):
    an amax pass produces the scale, then one fused pass quantises, writes
    the dense e4m3 tensor (needed by the FP8 GEMM) and compresses it.
    """
    from ..fp8 import fp8_scale

    scale = fp8_scale(h)
    h_fp8 = torch.empty(h.shape, device=h.device, dtype=torch.float8_e4m3fn)
    sp = compress(h, scale=scale, sparse_data=sparse_data, pack_sbit=pack_sbit,
                  quant_scale=scale, quant_out=h_fp8)
    return h_fp8, sp
