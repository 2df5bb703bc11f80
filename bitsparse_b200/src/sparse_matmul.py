"""Dense x BitsparseTensor GEMMs (lib_sparse/src/sparse_matmul.py).

``AspB`` / ``AspRelu2B`` compute ``A @ B`` / ``A @ (k * B^2)`` with B stored
sparse: B is reconstructed by the CUDA unpack kernel, then multiplied; or,
with ``FUSED_DW`` (bf16 raw storage, A the transpose of a row-major operand
as the layers' ``grad_output.T``), one tcgen05 GEMM expands B's compressed
tiles straight into its shared-memory operand (``matmul_unpack_dw``).
``row_batch > 0`` unpacks tile-aligned row batches and accumulates, trading
time for peak memory, as in the reference.
"""
from __future__ import annotations

import os

import torch
from torch import Tensor

from ..bitsparse import BitsparseTensor
from ..fp8 import matmul
from .operators import matmul_unpack_dw, unpack_batch_, unpack_relu2_batch_


# The fused reconstruct + tcgen05 weight-gradient GEMM (matmul_unpack_dw) is
# opt-in: it never writes the dense activation, but on B200 its per-tile
# expansion on the CUDA cores cannot keep pace with the tensor cores, and
# unpack + cuBLAS is faster at every measured shape.  BS_DW_FUSED=1 selects it.
FUSED_DW = os.environ.get("BS_DW_FUSED", "0") == "1"


def _row_batches(grid_m: int, BLOCK_M: int, N: int, row_batch: int):
    row_tiles = max(1, row_batch // BLOCK_M)
    for first_tile in range(0, grid_m, row_tiles):
        start = first_tile * BLOCK_M
        end = min(start + row_tiles * BLOCK_M, N)
        rows = end - start
        yield first_tile, start, end, rows, (rows + BLOCK_M - 1) // BLOCK_M


def AspB(A: Tensor, B_sparse: BitsparseTensor, A_scale: Tensor | None = None,
         row_batch: int = 0) -> Tensor:
    """A[M, N] @ sparse B[N, K] -> [M, K] (lib_sparse/src/sparse_matmul.py:9-47)."""
    BLOCK_M = B_sparse.BLOCK_M
    grid_m, grid_n = B_sparse.grid_m, B_sparse.grid_n
    N, K = B_sparse.shape
    M = A.shape[0]
    if row_batch <= 0:
        if FUSED_DW and not B_sparse.fp8:  # reconstruct fused into the tcgen05 GEMM
            out = matmul_unpack_dw(A, B_sparse)
            if out is not None:
                return out
        dense = torch.empty(N, K, device=A.device, dtype=B_sparse.dtype)
        unpack_batch_(B_sparse, dense, 0, grid_n, K, N, grid_m * grid_n)
        return matmul(A, dense, B_sparse.fp8, a_scale=A_scale, b_scale=B_sparse.scale)
    out = torch.zeros(M, K, device=A.device, dtype=A.dtype)
    for first, start, end, rows, nrt in _row_batches(grid_m, BLOCK_M, N, row_batch):
        dense_batch = torch.empty(rows, K, device=A.device, dtype=B_sparse.dtype)
        unpack_batch_(B_sparse, dense_batch, first, grid_n, K, rows, nrt * grid_n)
        out.addmm_(A[:, start:end], dense_batch)
    return out


def spAB(A_sparse: BitsparseTensor, B: Tensor, out: Tensor | None = None,
         row_batch: int = 0) -> Tensor:
    """sparse A[M, N] @ B[N, K] -> [M, K] (lib_sparse/src/sparse_matmul.py:50-88)."""
    BLOCK_M = A_sparse.BLOCK_M
    grid_m, grid_n = A_sparse.grid_m, A_sparse.grid_n
    M, N = A_sparse.shape
    K = B.shape[1]
    if row_batch <= 0:
        dense = torch.empty(M, N, device=B.device, dtype=A_sparse.dtype)
        unpack_batch_(A_sparse, dense, 0, grid_n, N, M, grid_m * grid_n)
        return matmul(dense, B, A_sparse.fp8, a_scale=A_sparse.scale)
    out = torch.zeros(M, K, device=B.device, dtype=B.dtype) if out is None else out
    for first, start, end, rows, nrt in _row_batches(grid_m, BLOCK_M, M, row_batch):
        dense_batch = torch.empty(rows, N, device=B.device, dtype=A_sparse.dtype)
        unpack_batch_(A_sparse, dense_batch, first, grid_n, N, rows, nrt * grid_n)
        torch.mm(dense_batch, B, out=out[start:end])
    return out


def _relu2_fp8_colmajor(sp: BitsparseTensor) -> tuple[Tensor, Tensor]:
    """to_fp8(unpack_relu2(sp)) transposed ([N, M] row-major) and its scale,
    in one pass over the compressed tensor (bs_unpack_relu2_fp8t)."""
    from .. import _lib, _runtime as R
    from ..config import RELU2_SCALE
    from ..fp8 import fp8_flags
    M, N = sp.shape
    dev = sp.bitmask.device
    bT = torch.empty(N, M, device=dev, dtype=torch.float8_e4m3fn)
    qs = torch.empty((), device=dev, dtype=torch.float32)
    scale = None if sp.scale is None else sp.scale.to(device=dev, dtype=torch.float32)
    _lib.call("bs_unpack_relu2_fp8t", sp.vals.data_ptr(), sp.bitmask.data_ptr(),
              sp.prefix.data_ptr(), sp.vals_offset.data_ptr(), R.dtype_code(sp.dtype), M, N,
              R.ptr(scale), float(RELU2_SCALE), R.amax_scratch(dev).data_ptr(), qs.data_ptr(),
              bT.data_ptr(), M, fp8_flags(), R.stream_handle(dev))
    return bT, qs


def AspRelu2B(A: Tensor, B_sparse: BitsparseTensor, A_scale: Tensor | None = None,
              row_batch: int = 0) -> Tensor:
    """A @ (k * B^2) with sparse B = relu(preact) (lib_sparse/src/sparse_matmul.py:91-132).

    The squared reconstruction is bf16 (squaring overflows FP8 storage); in
    FP8 mode it is re-quantised by the FP8 matmul."""
    BLOCK_M = B_sparse.BLOCK_M
    grid_m, grid_n = B_sparse.grid_m, B_sparse.grid_n
    N, K = B_sparse.shape
    M = A.shape[0]
    if row_batch <= 0:
        if (B_sparse.fp8 and not B_sparse.pack_sbit and A_scale is not None
                and A.dtype == B_sparse.dtype == torch.float8_e4m3fn):
            # the fp8 operand straight from the compressed form: reconstruct,
            # to_fp8 and the column-major copy in one kernel
            from ..fp8 import _row_major_fp8, _scaled_mm
            bT, b_scale = _relu2_fp8_colmajor(B_sparse)
            return _scaled_mm(_row_major_fp8(A), bT.T, A_scale, b_scale,
                              output_dtype=torch.bfloat16)
        if FUSED_DW and not B_sparse.fp8:
            out = matmul_unpack_dw(A, B_sparse, relu2=True)
            if out is not None:
                return out
        dense = torch.empty(N, K, device=A.device, dtype=torch.bfloat16)
        unpack_relu2_batch_(B_sparse, dense, 0, grid_n, K, N, grid_m * grid_n)
        return matmul(A, dense, B_sparse.fp8, a_scale=A_scale)
    out = torch.zeros(M, K, device=A.device, dtype=A.dtype)
    for first, start, end, rows, nrt in _row_batches(grid_m, BLOCK_M, N, row_batch):
        dense_batch = torch.empty(rows, K, device=A.device, dtype=torch.bfloat16)
        unpack_relu2_batch_(B_sparse, dense_batch, first, grid_n, K, rows, nrt * grid_n)
        out.addmm_(A[:, start:end], dense_batch)
    return out
