"""Operator boundary: the reference's triton_operators API on CUDA kernels.

Same function names, arguments, in-place semantics and return values as
lib_sparse/src/triton_operators.py (Maxzhu123/bitsparse); every function
is a thin launcher of a C-ABI entry point of libbitsparse_b200.so.  All
work is enqueued on the current CUDA stream.  There is no CPU path: CPU
tensors are rejected.

Plus the fused single-pass compressor ``compress`` used by
``dense_to_tilesparse``.
"""
from __future__ import annotations

import os

import torch
from torch import Tensor

from .. import _lib
from .. import _runtime as R
from ..bitsparse import BitsparseTensor, bits_per_value, tile_grid
from ..config import BLOCK_M as _BM, BLOCK_N as _BN, RELU2_SCALE
from ..fp8 import is_fp8
from .bitpacking import packed_storage_nbytes

if RELU2_SCALE != 1:  # the kernels take k as a parameter fixed to 1.0 below
    raise NotImplementedError("RELU2_SCALE other than 1 is not wired to the kernels")


def _check_tiles(BLOCK_M: int, BLOCK_N: int) -> None:
    if (BLOCK_M, BLOCK_N) != (64, 64):
        raise ValueError("bitsparse_b200 kernels are built for 64x64 tiles")


def _row_major(t: Tensor, name: str) -> tuple[Tensor, int]:
    """(tensor, row stride in elements) for a 2-D tensor with unit column stride."""
    R.require_cuda(t, name)
    if t.dim() != 2:
        raise ValueError(f"{name} must be 2-D")
    if t.stride(1) != 1 or t.stride(0) < t.shape[1]:
        t = t.contiguous()
    return t, max(t.stride(0), t.shape[1])


def _ld(t: Tensor) -> int:
    """Row stride of a 2-D tensor for the C ABI (a single row's stride is
    arbitrary in torch; the kernels want at least the row length)."""
    return t.stride(0) if t.shape[0] > 1 else t.shape[1]


def _stream(t: Tensor) -> int:
    return R.stream_handle(t.device)


# ---------------------------------------------------------------------------
# Compression
# ---------------------------------------------------------------------------
def tile_pack(
    dense: Tensor, tile_counts: Tensor, tile_bitmasks: Tensor,
    M: int, N: int, grid_m: int, grid_n: int,
    BLOCK_M: int, BLOCK_N: int, TILE_NUMEL: int, TILE_BYTES: int,
) -> None:
    """Bitmask + per-tile nonzero counts, in place (triton_operators.py:21-33)."""
    _check_tiles(BLOCK_M, BLOCK_N)
    dense, ld = _row_major(dense, "dense")
    _lib.call("bs_tile_pack", dense.data_ptr(), R.dtype_code(dense.dtype), M, N, ld,
              tile_counts.data_ptr(), tile_bitmasks.data_ptr(), _stream(dense))


def compact_vals(
    dense: Tensor, tile_bitmasks: Tensor, tile_prefix: Tensor,
    vals: Tensor | None, vals_offset: Tensor | None,
    M: int, N: int, grid_n: int, num_tiles: int,
    BLOCK_M: int, BLOCK_N: int, TILE_NUMEL: int, pack_sbit: bool,
) -> tuple[Tensor, Tensor]:
    """Compact positives into standalone or preallocated storage
    (triton_operators.py:36-115).  Standalone storage syncs once for nnz,
    as the reference does (triton_operators.py:50)."""
    _check_tiles(BLOCK_M, BLOCK_N)
    dense, ld = _row_major(dense, "dense")
    dt = dense.dtype
    if vals is None:
        nnz = int(tile_prefix[-1].item())
        if pack_sbit:
            vals = torch.zeros(packed_storage_nbytes(nnz, bits_per_value(dt)),
                               device=dense.device, dtype=torch.uint8)
        else:
            vals = torch.empty(nnz, device=dense.device, dtype=dt)
        vals_offset = torch.zeros((), device=dense.device, dtype=torch.int64)
    cap = vals.numel() * (vals.element_size() if pack_sbit else 1)
    _lib.call("bs_compact_vals", dense.data_ptr(), R.dtype_code(dt), M, N, ld,
              tile_prefix.data_ptr(), vals.data_ptr(), cap, int(pack_sbit),
              R.ptr(vals_offset), R.status_word(dense.device).data_ptr(), _stream(dense))
    return vals, vals_offset


# Standalone compress in the reference's order (count, sync, allocate
# exactly, compact): no dense-sized transient, two reads of the input, 3%
# slower than the one-pass form at 8192 x 3072 (95.6 vs 92.6 us).  Default;
# BS_COMPRESS_EXACT=0 selects the one-pass form with a worst-case scratch.
EXACT_STANDALONE = os.environ.get("BS_COMPRESS_EXACT", "1") == "1"


def compress(dense: Tensor, scale: Tensor | None = None, sparse_data=None,
             pack_sbit: bool = False, quant_scale: Tensor | None = None,
             quant_out: Tensor | None = None) -> BitsparseTensor:
    """Fused single-pass compression of a 2-D dense tensor.

    One kernel writes the bitmask, the prefix and the values (and advances a
    TensorBuffer's offset on the device).  With ``quant_scale`` (fp32 0-dim
    device tensor) a bf16 / fp32 input is quantised to e4m3fn in the same
    pass, exactly as ``to_fp8`` would, and ``quant_out`` (optional, e4m3
    [M, N]) receives the dense quantised tensor.

    Standalone storage (``sparse_data is None``), inputs that are not
    quantised: the reference's order (triton_operators.py:21-57) -- bitmask
    and tile counts, the prefix, one host sync for the total, an exactly
    sized allocation, then the compaction (two reads of the dense input, no
    dense-sized transient; ``EXACT_STANDALONE``).  Quantising inputs, or
    ``BS_COMPRESS_EXACT=0``: the one-pass kernel compacts into a worst-case
    scratch tensor, the total is read back (one sync) and copied into an
    exactly sized tensor.  With a TensorBuffer there is no sync.
    """
    dense, ld = _row_major(dense, "dense")
    M, N = dense.shape
    grid_m, grid_n, T, _, TB = tile_grid(M, N, _BM, _BN)
    dev = dense.device
    stored = torch.float8_e4m3fn if quant_scale is not None else dense.dtype
    if quant_scale is None and stored not in (torch.bfloat16,) and not is_fp8(stored):
        raise TypeError("BitsparseTensor supports bfloat16 and FP8 (e4m3fn/e5m2) values")
    bits = bits_per_value(stored)
    bitmask = torch.empty(T * TB, device=dev, dtype=torch.uint8)
    prefix = torch.empty(T + 1, device=dev, dtype=torch.uint32)
    st = _stream(dense)
    ws = R.workspace(dev, T, st)
    status = R.status_word(dev)
    qs = R.ptr(quant_scale)
    qo = R.ptr(quant_out)
    dcode = R.dtype_code(dense.dtype)
    if quant_scale is not None:  # to_fp8's arithmetic: eager or compiled
        from ..fp8 import fp8_flags
        dcode |= fp8_flags()
    if quant_out is not None and (quant_out.dtype != torch.float8_e4m3fn
                                  or not quant_out.is_contiguous()
                                  or tuple(quant_out.shape) != (M, N)):
        raise ValueError("quant_out must be a contiguous float8_e4m3fn [M, N] tensor")
    if sparse_data is None and T and quant_scale is None and EXACT_STANDALONE:
        counts = torch.empty(T, device=dev, dtype=torch.int32)
        tile_pack(dense, counts, bitmask, M, N, grid_m, grid_n, _BM, _BN, _BM * _BN,
                  _BM * _BN // 8)
        prefix[:1].zero_()
        torch.cumsum(counts, 0, dtype=torch.int32, out=prefix[1:].view(torch.int32))
        vals, vals_offset = compact_vals(dense, bitmask, prefix, None, None, M, N, grid_n, T,
                                         _BM, _BN, _BM * _BN, pack_sbit)
    elif sparse_data is None:
        if T == 0:
            prefix.zero_()
            vals = torch.empty(packed_storage_nbytes(0, bits) if pack_sbit else 0,
                               device=dev, dtype=torch.uint8 if pack_sbit else stored)
            if pack_sbit:
                vals.zero_()
            vals_offset = torch.zeros((), device=dev, dtype=torch.int64)
        else:
            if pack_sbit:
                tmp = torch.empty(packed_storage_nbytes(M * N, bits), device=dev,
                                  dtype=torch.uint8)
                cap = tmp.numel()
            else:
                tmp = torch.empty(M * N, device=dev, dtype=stored)
                cap = M * N
            nnz_t = torch.empty((), device=dev, dtype=torch.int64)
            _lib.call("bs_compress", dense.data_ptr(), dcode, M, N, ld,
                      qs, qo, bitmask.data_ptr(), prefix.data_ptr(), tmp.data_ptr(), cap,
                      int(pack_sbit), None, None, nnz_t.data_ptr(), ws.data_ptr(),
                      ws.numel(), status.data_ptr(), st)
            nnz = int(nnz_t.item())  # host sync (triton_operators.py:50)
            size = packed_storage_nbytes(nnz, bits) if pack_sbit else nnz
            vals = tmp[:size].clone()
            vals_offset = torch.zeros((), device=dev, dtype=torch.int64)
    else:
        vals = sparse_data.vals
        if pack_sbit != bool(sparse_data.pack_sbit):
            raise ValueError("pack_sbit must match the TensorBuffer's pack_sbit")
        if not pack_sbit and vals.dtype != stored:
            raise TypeError(f"TensorBuffer holds {vals.dtype}, values are {stored}")
        R.require_cuda(vals, "TensorBuffer.vals")
        cap = vals.numel()
        vals_offset = torch.empty(1, device=dev, dtype=torch.int64)
        if T == 0:
            prefix.zero_()
            off = sparse_data.offset
            vals_offset.copy_((off + 7) // 8 * 8 if pack_sbit else off)
        else:
            _lib.call("bs_compress", dense.data_ptr(), dcode, M, N, ld,
                      qs, qo, bitmask.data_ptr(), prefix.data_ptr(), vals.data_ptr(), cap,
                      int(pack_sbit), sparse_data.offset.data_ptr(), vals_offset.data_ptr(),
                      None, ws.data_ptr(), ws.numel(), status.data_ptr(), st)
    return BitsparseTensor(vals, bitmask, prefix, dense.shape, stored,
                           grid_m, grid_n, _BM, _BN, scale=scale,
                           vals_offset=vals_offset, pack_sbit=pack_sbit)


# ---------------------------------------------------------------------------
# Reconstruction and gradient masks
# ---------------------------------------------------------------------------
def _unpack(sparse: BitsparseTensor, output: Tensor, first_m_tile: int, grid_n: int, K: int,
            batch_rows: int, num_tiles_in_batch: int, relu2: bool) -> Tensor:
    _check_tiles(sparse.BLOCK_M, sparse.BLOCK_N)
    R.require_cuda(output, "output")
    want = torch.bfloat16 if relu2 else sparse.dtype
    if output.dtype != want:
        raise TypeError(f"output must be {want}, got {output.dtype}")
    if output.dim() != 2 or output.stride(1) != 1:
        raise ValueError("output must be a 2-D tensor with unit column stride")
    if output.shape[0] < batch_rows or output.shape[1] < K:
        raise ValueError("output is smaller than [batch_rows, K]")
    scale = sparse.scale if relu2 else None
    if scale is not None:
        scale = scale.to(device=output.device, dtype=torch.float32)
    _lib.call("bs_unpack", sparse.vals.data_ptr(), sparse.bitmask.data_ptr(),
              sparse.prefix.data_ptr(), sparse.vals_offset.data_ptr(),
              R.dtype_code(sparse.dtype), int(sparse.pack_sbit), output.data_ptr(),
              _ld(output), first_m_tile, grid_n, K, batch_rows, num_tiles_in_batch,
              int(relu2), R.ptr(scale), _stream(output))
    return output


def unpack_batch_(
    sparse: BitsparseTensor, output: Tensor,
    first_m_tile: int, grid_n: int, K: int, batch_rows: int,
    num_tiles_in_batch: int,
) -> Tensor:
    """Unpack a slice of tiles into a dense [batch_rows, K] slice, in place
    (triton_operators.py:118-138).  ``output`` has the stored dtype."""
    return _unpack(sparse, output, first_m_tile, grid_n, K, batch_rows,
                   num_tiles_in_batch, relu2=False)


def unpack_relu2_batch_(
    sparse: BitsparseTensor, output: Tensor,
    first_m_tile: int, grid_n: int, K: int, batch_rows: int,
    num_tiles_in_batch: int,
) -> Tensor:
    """Unpack stored r = relu(a) as bf16 k * r^2 (times scale^2 when the
    tensor has an FP8 scale), in place (triton_operators.py:141-162)."""
    return _unpack(sparse, output, first_m_tile, grid_n, K, batch_rows,
                   num_tiles_in_batch, relu2=True)


def mask_with_bitmask_(grad: Tensor, sparse: BitsparseTensor) -> Tensor:
    """grad <- grad * bitmask, in place (triton_operators.py:165-175)."""
    _check_tiles(sparse.BLOCK_M, sparse.BLOCK_N)
    R.require_cuda(grad, "grad")
    M, N = sparse.shape
    if tuple(grad.shape) != (M, N) or grad.stride(1) != 1:
        raise ValueError("grad must be [M, N] with unit column stride")
    _lib.call("bs_mask_with_bitmask", grad.data_ptr(), R.dtype_code(grad.dtype), M, N,
              _ld(grad), sparse.bitmask.data_ptr(), _stream(grad))
    return grad


def relu2_grad_sparse_(grad: Tensor, sparse_z: BitsparseTensor) -> Tensor:
    """grad <- grad * 2 k r under the mask, then * scale, in place
    (triton_operators.py:178-202)."""
    _check_tiles(sparse_z.BLOCK_M, sparse_z.BLOCK_N)
    R.require_cuda(grad, "grad")
    M, N = sparse_z.shape
    if tuple(grad.shape) != (M, N) or grad.stride(1) != 1:
        raise ValueError("grad must be [M, N] with unit column stride")
    scale = sparse_z.scale
    if scale is not None:
        scale = scale.to(device=grad.device, dtype=torch.float32)
    _lib.call("bs_relu2_grad", grad.data_ptr(), R.dtype_code(grad.dtype), M, N,
              _ld(grad), sparse_z.vals.data_ptr(), sparse_z.bitmask.data_ptr(),
              sparse_z.prefix.data_ptr(), sparse_z.vals_offset.data_ptr(),
              R.dtype_code(sparse_z.dtype), int(sparse_z.pack_sbit), R.ptr(scale),
              _stream(grad))
    return grad


# ---------------------------------------------------------------------------
# Tensor-core GEMM with the ReLU mask in its epilogue
# ---------------------------------------------------------------------------
def matmul_relu_mask(a: Tensor, b: Tensor, sparse: BitsparseTensor | None = None) -> Tensor:
    """bf16 ``a [M, K] @ b [K, N]`` on the tcgen05 tensor cores (fp32
    accumulation, bf16 result); with ``sparse`` (a bitsparse [M, N] tensor)
    the elements whose bitmask bit is clear are written as 0.

    ``matmul_relu_mask(grad_y, W2, h)`` equals ``mask_with_bitmask_(grad_y @
    W2, h)`` (lib_sparse/layers.py:38-51) up to the accumulation order of the
    GEMM, without the dense ``grad_y @ W2`` reaching memory.
    """
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("matmul_relu_mask takes bfloat16 operands")
    a, lda = _row_major(a, "a")
    b, ldb = _row_major(b, "b")
    M, K = a.shape
    K2, N = b.shape
    if K != K2:
        raise ValueError(f"inner dimensions differ: {K} vs {K2}")
    mask = 0
    if sparse is not None:
        if tuple(sparse.shape) != (M, N):
            raise ValueError(f"mask shape {tuple(sparse.shape)} != output shape {(M, N)}")
        _check_tiles(sparse.BLOCK_M, sparse.BLOCK_N)
        mask = sparse.bitmask.data_ptr()
    out = torch.empty((M, N), device=a.device, dtype=torch.bfloat16)
    status = R.status_word(a.device)
    _lib.call("bs_gemm_bf16_mask", a.data_ptr(), lda, b.data_ptr(), ldb, out.data_ptr(), N,
              M, N, K, mask or None, status.data_ptr(), _stream(a))
    return out


def matmul_relu2_grad(a: Tensor, b: Tensor, sparse: BitsparseTensor) -> Tensor | None:
    """``relu2_grad_sparse_(a @ b, sparse)`` for bf16 storage in one tcgen05
    GEMM: the ReLU^2 gradient ``grad * (2 k r)`` (r the stored activation)
    is applied in the epilogue, so the dense ``a @ b`` never reaches memory
    (lib_sparse/layers.py:146-147).  Same roundings as the two-step form.
    Returns ``None`` when this path does not apply (FP8 or packed storage, a
    value base not 16-byte aligned, operands TMA cannot read), and the
    caller uses the two steps."""
    if (sparse.dtype != torch.bfloat16 or sparse.pack_sbit or sparse.scale is not None
            or a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16):
        return None
    if a.dim() != 2 or b.dim() != 2 or a.stride(1) != 1 or b.stride(1) != 1:
        return None
    M, K = a.shape
    K2, N = b.shape
    if K != K2 or tuple(sparse.shape) != (M, N) or sparse.vals.data_ptr() % 16:
        return None
    if (sparse.BLOCK_M, sparse.BLOCK_N) != (_BM, _BN):
        return None
    out = torch.empty((M, N), device=a.device, dtype=torch.bfloat16)
    rc = _lib.load().bs_gemm_bf16_relu2(
        a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), out.data_ptr(), N, M, N, K,
        sparse.vals.data_ptr(), sparse.bitmask.data_ptr(), sparse.prefix.data_ptr(),
        sparse.vals_offset.data_ptr(), float(RELU2_SCALE), R.status_word(a.device).data_ptr(),
        _stream(a))
    if rc == _lib.BS_ERR_ALIGN:
        return None
    _lib.check(rc, "bs_gemm_bf16_relu2")
    return out


def matmul_unpack_dw(a: Tensor, sparse: BitsparseTensor, relu2: bool = False) -> Tensor | None:
    """``a @ unpack(sparse)`` (AspB) or ``a @ (k * unpack(sparse)^2)``
    (AspRelu2B) in one tcgen05 GEMM that expands each compressed tile of
    ``sparse`` straight into its shared-memory operand
    (lib_sparse/src/sparse_matmul.py:9-47, :91-132): the FFN's weight
    gradient ``grad_output.T @ h`` without the dense h.  ``a`` [D, T] must
    be the transpose of a row-major bf16 [T, D] (the layers pass
    ``grad_output.T``).  Returns ``None`` when the path does not apply (FP8
    or packed storage, a scaled tensor, k != 1 for ReLU^2, D < 256, layouts
    TMA cannot read), and the caller unpacks and multiplies."""
    if (sparse.dtype != torch.bfloat16 or sparse.pack_sbit or sparse.scale is not None
            or a.dtype != torch.bfloat16 or a.dim() != 2 or not a.is_cuda):
        return None
    if relu2 and RELU2_SCALE != 1:
        return None
    D, T = a.shape
    if tuple(sparse.shape)[0] != T or (sparse.BLOCK_M, sparse.BLOCK_N) != (_BM, _BN):
        return None
    if D < 256 or a.stride(0) != 1 or a.stride(1) < D or a.data_ptr() % 16 or (a.stride(1) * 2) % 16:
        return None
    if sparse.vals.data_ptr() % 16 or sparse.bitmask.data_ptr() % 16:
        return None
    H = sparse.shape[1]
    out = torch.empty((D, H), device=a.device, dtype=torch.bfloat16)
    lib = _lib.load()
    with torch.cuda.device(a.device):
        wsb = int(lib.bs_gemm_unpack_dw_workspace_bytes(T, D, H))
    ws = torch.empty(wsb // 4 + 4, device=a.device, dtype=torch.float32) if wsb else None
    rc = lib.bs_gemm_unpack_dw(
        a.data_ptr(), a.stride(1), T, D, sparse.vals.data_ptr(), sparse.bitmask.data_ptr(),
        sparse.prefix.data_ptr(), sparse.vals_offset.data_ptr(), H, int(relu2),
        float(RELU2_SCALE), out.data_ptr(), H, R.ptr(ws), wsb, R.status_word(a.device).data_ptr(),
        _stream(a))
    if rc == _lib.BS_ERR_ALIGN:
        return None
    _lib.check(rc, "bs_gemm_unpack_dw")
    return out


def matmul_fp8_relu2_grad(a: Tensor, bt: Tensor, a_scale: Tensor, b_scale: Tensor,
                          sparse: BitsparseTensor) -> Tensor | None:
    """``relu2_grad_sparse_(scaled_mm(a, bt.T), sparse)`` for e4m3 storage in
    one tcgen05 FP8 GEMM (``kind::f8f6f4``): the ReLU^2 gradient ``grad * (2
    k r)`` and the ``grad *= scale`` of the stored tensor's scale applied in
    the epilogue (lib_sparse/layers.py:146-147 with the FP8 matmul of
    lib_sparse/fp8.py:52-115), with the same roundings as the separate
    steps on this library's FP8 GEMM.  ``a`` [M, K], ``bt`` [N, K] e4m3 with
    unit column stride.  ``None`` when the path does not apply (packed or
    non-e4m3 storage, alignment), and the caller uses the two steps."""
    if (sparse.dtype != torch.float8_e4m3fn or sparse.pack_sbit
            or a.dtype != torch.float8_e4m3fn or bt.dtype != torch.float8_e4m3fn):
        return None
    if a.dim() != 2 or bt.dim() != 2 or a.stride(1) != 1 or bt.stride(1) != 1:
        return None
    M, K = a.shape
    N = bt.shape[0]
    lda = a.stride(0) if M > 1 else K
    ldb = bt.stride(0) if N > 1 else K
    if (bt.shape[1] != K or tuple(sparse.shape) != (M, N) or sparse.vals.data_ptr() % 16
            or a.data_ptr() % 16 or bt.data_ptr() % 16 or lda % 16 or ldb % 16):
        return None
    if (sparse.BLOCK_M, sparse.BLOCK_N) != (_BM, _BN):
        return None
    out = torch.empty((M, N), device=a.device, dtype=torch.bfloat16)
    sa = a_scale.reshape(()).to(torch.float32)
    sb = b_scale.reshape(()).to(torch.float32)
    hs = None if sparse.scale is None else sparse.scale.reshape(()).to(torch.float32)
    rc = _lib.load().bs_gemm_fp8_relu2(
        a.data_ptr(), lda, bt.data_ptr(), ldb, out.data_ptr(), N, M, N, K, sa.data_ptr(),
        sb.data_ptr(), sparse.vals.data_ptr(), sparse.bitmask.data_ptr(),
        sparse.prefix.data_ptr(), sparse.vals_offset.data_ptr(), float(RELU2_SCALE),
        R.ptr(hs), R.status_word(a.device).data_ptr(), _stream(a))
    if rc == _lib.BS_ERR_ALIGN:
        return None
    _lib.check(rc, "bs_gemm_fp8_relu2")
    return out


def _fused_compress(fn, name: str, head: tuple, dev, stream: int, stored, M: int, N: int,
                    T: int, bitmask: Tensor, prefix: Tensor, sparse_data, pack_sbit: bool,
                    flags: tuple = ()):
    """Run a fused compress entry point ``fn(*head, bitmask, prefix, vals,
    capacity, pack_sbit, arena_offset, vals_offset_out, nnz_out, workspace,
    workspace_bytes, status, stream)`` (``head``: its leading arguments,
    already plain ints) in either storage mode.  Returns (vals, vals_offset),
    or None when the entry point reports BS_ERR_ALIGN (the one-pass kernel
    cannot read the tensors)."""
    ws = R.workspace(dev, T, stream)
    status = R.status_word(dev)
    if sparse_data is None:
        bits = bits_per_value(stored)
        if pack_sbit:
            tmp = torch.empty(packed_storage_nbytes(M * N, bits), device=dev, dtype=torch.uint8)
        else:
            tmp = torch.empty(M * N, device=dev, dtype=stored)
        nnz_t = torch.empty((), device=dev, dtype=torch.int64)
        rc = fn(*head, bitmask.data_ptr(), prefix.data_ptr(), tmp.data_ptr(), tmp.numel(),
                int(pack_sbit), None, None, nnz_t.data_ptr(), ws.data_ptr(), ws.numel(),
                *flags, status.data_ptr(), stream)
        if rc == _lib.BS_ERR_ALIGN:
            return None
        _lib.check(rc, name)
        nnz = int(nnz_t.item())  # host sync (triton_operators.py:50)
        size = packed_storage_nbytes(nnz, bits) if pack_sbit else nnz
        return tmp[:size].clone(), torch.zeros((), device=dev, dtype=torch.int64)
    vals = sparse_data.vals
    if pack_sbit != bool(sparse_data.pack_sbit):
        raise ValueError("pack_sbit must match the TensorBuffer's pack_sbit")
    if not pack_sbit and vals.dtype != stored:
        raise TypeError(f"TensorBuffer holds {vals.dtype}, values are {stored}")
    vals_offset = torch.empty(1, device=dev, dtype=torch.int64)
    rc = fn(*head, bitmask.data_ptr(), prefix.data_ptr(), vals.data_ptr(), vals.numel(),
            int(pack_sbit), sparse_data.offset.data_ptr(), vals_offset.data_ptr(), None,
            ws.data_ptr(), ws.numel(), *flags, status.data_ptr(), stream)
    if rc == _lib.BS_ERR_ALIGN:
        return None
    _lib.check(rc, name)
    return vals, vals_offset


def _fused_exact(fn, name: str, head: tuple, dev, stream: int, dense_vals: Tensor, M: int,
                 N: int, grid_n: int, T: int, bitmask: Tensor, prefix: Tensor, pack_sbit: bool,
                 flags: tuple = ()):
    """Standalone storage of a fused compress in the reference's order: the
    fused kernel with no value storage (bitmask, prefix, the dense side
    output and the total), one host sync for the total, an exactly sized
    allocation, then ``bs_compact_vals`` from ``dense_vals`` -- the dense
    side output, which holds exactly the values being stored.  No
    dense-sized transient.  Returns (vals, vals_offset) or None (alignment)."""
    ws = R.workspace(dev, T, stream)
    status = R.status_word(dev)
    nnz_t = torch.empty((), device=dev, dtype=torch.int64)
    rc = fn(*head, bitmask.data_ptr(), prefix.data_ptr(), None, 0, int(pack_sbit), None, None,
            nnz_t.data_ptr(), ws.data_ptr(), ws.numel(), *flags, status.data_ptr(), stream)
    if rc == _lib.BS_ERR_ALIGN:
        return None
    _lib.check(rc, name)
    nnz = int(nnz_t.item())  # host sync (triton_operators.py:50)
    if pack_sbit:
        vals = torch.zeros(packed_storage_nbytes(nnz, bits_per_value(dense_vals.dtype)),
                           device=dev, dtype=torch.uint8)
    else:
        vals = torch.empty(nnz, device=dev, dtype=dense_vals.dtype)
    vals_offset = torch.zeros((), device=dev, dtype=torch.int64)
    return compact_vals(dense_vals, bitmask, prefix, vals, vals_offset, M, N, grid_n, T,
                        _BM, _BN, _BM * _BN, pack_sbit)


def compress_bias_relu(z: Tensor, bias: Tensor, sparse_data=None, pack_sbit: bool = False):
    """Fused ``h = relu(z + bias)`` + compress of h in one pass over z (bf16).

    Returns ``(h, BitsparseTensor)`` -- h dense (the FFN's second GEMM needs
    it), the compressed form equal to ``compress(h, ...)`` -- or ``None``
    when the one-pass kernel cannot read these tensors (alignment), in which
    case the caller runs the steps separately.  Same storage modes as
    ``compress`` (standalone, or a TensorBuffer arena).
    """
    if z.dtype != torch.bfloat16 or bias.dtype != torch.bfloat16:
        return None
    if not z.is_cuda:
        R.require_cuda(z, "z")
    if z.dim() != 2:
        raise ValueError("z must be 2-D")
    M, N = z.shape
    if z.stride(1) != 1 or z.stride(0) < N:
        z = z.contiguous()
    ld = max(z.stride(0), N)
    if not bias.is_contiguous():
        bias = bias.contiguous()
    if bias.numel() != N:
        raise ValueError(f"bias has {bias.numel()} elements, z has {N} columns")
    grid_m, grid_n = (M + _BM - 1) // _BM, (N + _BN - 1) // _BN
    T = grid_m * grid_n
    if T == 0:
        return None
    dev = z.device
    h = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
    bitmask = torch.empty(T * (_BM * _BN // 8), device=dev, dtype=torch.uint8)
    prefix = torch.empty(T + 1, device=dev, dtype=torch.uint32)
    st = R.stream_handle(dev)
    head = (z.data_ptr(), M, N, ld, bias.data_ptr(), h.data_ptr(), N)
    fn = _lib.load().bs_compress_bias_relu
    if sparse_data is None and EXACT_STANDALONE:
        out = _fused_exact(fn, "bs_compress_bias_relu", head, dev, st, h, M, N, grid_n, T,
                           bitmask, prefix, pack_sbit)
    else:
        out = _fused_compress(fn, "bs_compress_bias_relu", head, dev, st, torch.bfloat16, M, N,
                              T, bitmask, prefix, sparse_data, pack_sbit)
    if out is None:
        return None
    vals, vals_offset = out
    return h, BitsparseTensor(vals, bitmask, prefix, (M, N), torch.bfloat16, grid_m, grid_n,
                              _BM, _BN, vals_offset=vals_offset, pack_sbit=pack_sbit)


def compress_bias_relu_fp8(z: Tensor, bias: Tensor, sparse_data=None, pack_sbit: bool = False,
                           square: bool = False):
    """FP8 form of ``compress_bias_relu``: h = relu(z + bias) is stored as
    ``to_fp8(h)`` (lib_sparse/layers.py:32-37, 112-117) and compressed, in two
    passes over z (the amax of h, then quantise + compress).

    Returns ``(side, side_scale, BitsparseTensor)``: ``side`` is the dense
    e4m3 operand of the FFN's second GEMM -- ``to_fp8(h)`` or, with
    ``square``, ``to_fp8(h * h)`` (Relu2Linear, RELU2_SCALE = 1) -- or
    ``None`` when the one-pass kernel cannot read the tensors.
    """
    from ..config import RELU2_SCALE
    from ..fp8 import fp8_flags
    if z.dtype != torch.bfloat16 or bias.dtype != torch.bfloat16:
        return None
    if square and RELU2_SCALE != 1:
        return None  # the fused square assumes k = 1 (config.py)
    z, ld = _row_major(z, "z")
    M, N = z.shape
    bias = bias.contiguous()
    if bias.numel() != N:
        raise ValueError(f"bias has {bias.numel()} elements, z has {N} columns")
    grid_m, grid_n, T, _, TB = tile_grid(M, N, _BM, _BN)
    if T == 0 or z.data_ptr() % 16 or bias.data_ptr() % 16:
        return None
    dev = z.device
    lib = _lib.load()
    st = _stream(z)
    scale_h = torch.empty((), device=dev, dtype=torch.float32)
    scale_s = torch.empty((), device=dev, dtype=torch.float32) if square else None
    _lib.check(lib.bs_fp8_scales_bias_relu(z.data_ptr(), M, N, ld, bias.data_ptr(),
                                           R.amax_scratch(dev).data_ptr(), scale_h.data_ptr(),
                                           R.ptr(scale_s), fp8_flags(), st),
               "bs_fp8_scales_bias_relu")
    side = torch.empty((M, N), device=dev, dtype=torch.float8_e4m3fn)
    bitmask = torch.empty(T * TB, device=dev, dtype=torch.uint8)
    prefix = torch.empty(T + 1, device=dev, dtype=torch.uint32)
    head = (z.data_ptr(), M, N, ld, bias.data_ptr(), scale_h.data_ptr(), R.ptr(scale_s),
            side.data_ptr())
    fn = lib.bs_compress_bias_relu_fp8
    if sparse_data is None and EXACT_STANDALONE and not square:
        # side = to_fp8(h): exactly the stored codes
        out = _fused_exact(fn, "bs_compress_bias_relu_fp8", head, dev, st, side, M, N,
                           grid_n, T, bitmask, prefix, pack_sbit, flags=(fp8_flags(),))
    else:
        out = _fused_compress(fn, "bs_compress_bias_relu_fp8", head, dev, st,
                              torch.float8_e4m3fn, M, N, T, bitmask, prefix, sparse_data,
                              pack_sbit, flags=(fp8_flags(),))
    if out is None:
        return None
    vals, vals_offset = out
    sp = BitsparseTensor(vals, bitmask, prefix, (M, N), torch.float8_e4m3fn, grid_m, grid_n,
                         _BM, _BN, scale=scale_h, vals_offset=vals_offset, pack_sbit=pack_sbit)
    return side, (scale_s if square else scale_h), sp


# ---------------------------------------------------------------------------
# Per-tile FP8 scale mode (an extension: the reference's to_fp8 is per tensor)
# ---------------------------------------------------------------------------
def compress_fp8_tile_scaled(dense: Tensor, sparse_data=None,
                             pack_sbit: bool = False) -> BitsparseTensor:
    """Compress a bf16 [M, N] tensor to e4m3 with one scale per 64 x 64 tile,
    in one pass (bs_compress_fp8_tile_scaled): scale_t = amax_t / 448, code =
    e4m3(x * (448 / amax_t)), the positive codes stored as usual.  The
    returned tensor's ``tile_scales`` (fp32 [T]) go with it; its ``scale`` is
    None.  The input must be TMA-readable (16-byte aligned base, row stride
    a multiple of 8 elements)."""
    if dense.dtype != torch.bfloat16:
        raise TypeError("the per-tile scale mode takes bfloat16 input")
    dense, ld = _row_major(dense, "dense")
    M, N = dense.shape
    grid_m, grid_n, T, _, TB = tile_grid(M, N, _BM, _BN)
    dev = dense.device
    stored = torch.float8_e4m3fn
    bitmask = torch.empty(T * TB, device=dev, dtype=torch.uint8)
    prefix = torch.empty(T + 1, device=dev, dtype=torch.uint32)
    tile_scales = torch.empty(T, device=dev, dtype=torch.float32)
    if T == 0:
        prefix.zero_()
        vals = torch.empty(packed_storage_nbytes(0, 7) if pack_sbit else 0, device=dev,
                           dtype=torch.uint8 if pack_sbit else stored)
        return BitsparseTensor(vals, bitmask, prefix, (M, N), stored, grid_m, grid_n, _BM, _BN,
                               pack_sbit=pack_sbit, tile_scales=tile_scales)
    lib = _lib.load()
    out = _fused_compress(lib.bs_compress_fp8_tile_scaled, "bs_compress_fp8_tile_scaled",
                          (dense.data_ptr(), M, N, ld, tile_scales.data_ptr()), dev,
                          _stream(dense), stored, M, N, T, bitmask, prefix, sparse_data, pack_sbit)
    if out is None:
        raise ValueError("the per-tile scale mode needs a 16-byte aligned base and row stride")
    vals, vals_offset = out
    return BitsparseTensor(vals, bitmask, prefix, (M, N), stored, grid_m, grid_n, _BM, _BN,
                           vals_offset=vals_offset, pack_sbit=pack_sbit, tile_scales=tile_scales)


def unpack_tile_scaled_(sparse: BitsparseTensor, output: Tensor, first_m_tile: int = 0,
                        grid_n: int | None = None, K: int | None = None,
                        batch_rows: int | None = None,
                        num_tiles_in_batch: int | None = None) -> Tensor:
    """bf16 ``output`` = the dequantised tensor of a per-tile-scaled e4m3
    BitsparseTensor: bf16(value(code) * tile_scale), zeros elsewhere
    (bs_unpack_tile_scaled; whole tensor by default, or a tile-row batch as
    ``unpack_batch_`` takes it)."""
    if sparse.tile_scales is None or sparse.dtype != torch.float8_e4m3fn:
        raise ValueError("not a per-tile-scaled e4m3 BitsparseTensor")
    if output.dtype != torch.bfloat16:
        raise TypeError("the dequantised output is bfloat16")
    M, N = sparse.shape
    grid_n = sparse.grid_n if grid_n is None else grid_n
    K = N if K is None else K
    batch_rows = M if batch_rows is None else batch_rows
    if num_tiles_in_batch is None:
        num_tiles_in_batch = sparse.grid_m * sparse.grid_n
    _lib.call("bs_unpack_tile_scaled", sparse.vals.data_ptr(), sparse.bitmask.data_ptr(),
              sparse.prefix.data_ptr(), sparse.vals_offset.data_ptr(), int(sparse.pack_sbit),
              sparse.tile_scales.data_ptr(), output.data_ptr(), output.stride(0), first_m_tile,
              grid_n, K, batch_rows, num_tiles_in_batch, _stream(output))
    return output
