"""FP8 helpers: per-tensor e4m3 quantiser and the FP8 matmul autograd op.

Mirrors lib_sparse/fp8.py (Maxzhu123/bitsparse).  ``to_fp8`` runs on this
library's CUDA kernels (amax -> scale, then quantise) with the arithmetic of
``FP8_SEMANTICS``.  The FP8 GEMMs are cuBLASLt through ``F.scaled_mm``, as in
the reference, or this library's tcgen05 kernels (``FP8_GEMM``).

Two deliberate differences from the reference, both bug fixes:

* ``matmul`` passes the scales positionally: the reference's keyword call
  (lib_sparse/fp8.py:120) is rejected by ``autograd.Function.apply`` on
  current PyTorch because ``MatmulFp8`` defines no ``setup_context``;
* operand B is made column-major whenever it is not (cuBLASLt's FP8 layout
  rule on B200, compute capability 10.0); the reference only does this for
  capability < 12 (lib_sparse/fp8.py:15-17), which includes B200 anyway.
"""
from __future__ import annotations

import os

import torch
from torch import Tensor
from torch.autograd import Function
from torch.nn import functional as F

from .config import CACHE_FP8_MATMUl

# to_fp8's arithmetic (lib_sparse/fp8.py:123-129), which decides the FP8
# bytes: "compiled" -- the reference's @torch.compile'd to_fp8 as it runs on
# a GPU (scale = amax * (1/448) in fp32, q = e4m3(x / scale) with Triton's
# fp32 division), the default;
# "eager" -- eager PyTorch's (bf16 input: the scale and the quotient rounded
# to bf16), which the reference's CPU golden fixtures hold.
# BS_FP8_SEMANTICS in the environment overrides the default.
FP8_SEMANTICS = os.environ.get("BS_FP8_SEMANTICS", "compiled")


class fp8_semantics:
    """Context manager: ``with fp8_semantics("eager"): ...`` runs to_fp8's
    quantisation with that arithmetic and restores the previous one."""

    def __init__(self, mode: str):
        self.mode = mode

    def __enter__(self):
        global FP8_SEMANTICS
        self.prev, FP8_SEMANTICS = FP8_SEMANTICS, self.mode
        return self

    def __exit__(self, *a):
        global FP8_SEMANTICS
        FP8_SEMANTICS = self.prev


def fp8_flags() -> int:
    """The C ABI flag of the current FP8_SEMANTICS."""
    from . import _lib
    if FP8_SEMANTICS not in ("compiled", "eager"):
        raise ValueError(f"FP8_SEMANTICS must be 'compiled' or 'eager', not {FP8_SEMANTICS!r}")
    return _lib.BS_FP8_COMPILED if FP8_SEMANTICS == "compiled" else 0


_FP8_DTYPES = (torch.float8_e4m3fn, torch.float8_e5m2)
_FP8_DTYPE = torch.float8_e4m3fn
_FP8_MAX = torch.finfo(_FP8_DTYPE).max


def is_fp8(dtype) -> bool:
    """True for the supported 8-bit float storage dtypes (e4m3fn, e5m2)."""
    return dtype in _FP8_DTYPES


def _dense_layout(x: Tensor) -> tuple[Tensor, bool]:
    """(a contiguous tensor with x's elements, whether it is x transposed).

    A 2-D tensor whose transpose is contiguous (e.g. ``W.T``) is processed as
    that transpose, so no transposed copy is made; the result is transposed
    back as a view, keeping x's layout."""
    if x.is_contiguous():
        t, tr = x, False
    elif x.dim() == 2 and x.T.is_contiguous():
        t, tr = x.T, True
    else:
        return x.contiguous(), False
    if t.data_ptr() % 16:  # a view at an odd offset: the kernels read 16-byte vectors
        t = t.clone(memory_format=torch.contiguous_format)
    return t, tr


@torch.no_grad()
def fp8_scale(x: Tensor) -> Tensor:
    """Per-tensor scale of to_fp8: max(amax(|x|) / 448, 1e-9), fp32 0-dim.

    In eager semantics amax / 448 is rounded to bf16 for bf16 input (eager
    PyTorch on lib_sparse/fp8.py:126); in compiled semantics it stays fp32."""
    from . import _lib, _runtime as R

    R.require_cuda(x, "x")
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("to_fp8 takes bfloat16 or float32 input")
    x, _ = _dense_layout(x)  # the amax does not depend on the layout
    scale = torch.empty((), dtype=torch.float32, device=x.device)
    _lib.call("bs_fp8_scale", x.data_ptr(), R.dtype_code(x.dtype) | fp8_flags(), x.numel(),
              R.amax_scratch(x.device).data_ptr(), scale.data_ptr(),
              R.stream_handle(x.device))
    return scale


@torch.no_grad()
def quantize_e4m3(x: Tensor, scale: Tensor) -> Tensor:
    """to_fp8's quantiser, elementwise: e4m3fn(bf16(x / scale)) for bf16 input
    in eager semantics, e4m3fn(x / scale) with Triton's fp32 division in
    compiled semantics."""
    from . import _lib, _runtime as R

    xc, transposed = _dense_layout(x)
    q = torch.empty(xc.shape, dtype=_FP8_DTYPE, device=x.device)
    _lib.call("bs_quantize_e4m3", xc.data_ptr(), R.dtype_code(xc.dtype) | fp8_flags(), xc.numel(),
              scale.data_ptr(), q.data_ptr(), R.stream_handle(x.device))
    return q.T if transposed else q


def estimate_exact(scale: Tensor) -> bool:
    """Whether the quantisers take the plain estimate x * (1/scale) at this
    scale in the current semantics (an exhaustive check over the bf16 codes
    that can reach an e4m3 rounding boundary; bs_fp8_estimate_exact).  They
    divide where it is False; the codes are the same either way."""
    from . import _lib, _runtime as R

    R.require_cuda(scale, "scale")
    out = torch.empty(1, dtype=torch.int32, device=scale.device)
    _lib.call("bs_fp8_estimate_exact", scale.data_ptr(), fp8_flags(), out.data_ptr(),
              R.stream_handle(scale.device))
    return bool(out.item())


@torch.no_grad()
def to_fp8(x: Tensor) -> tuple[Tensor, Tensor]:
    """(x_fp8, scale): per-tensor e4m3fn quantisation (lib_sparse/fp8.py:123-129)."""
    scale = fp8_scale(x)
    return quantize_e4m3(x, scale), scale


@torch.no_grad()
def quantize_e4m3_layouts(x: Tensor, scale: Tensor, row: bool = True,
                          col: bool = False) -> tuple[Tensor | None, Tensor | None]:
    """e4m3fn(x / scale) of a 2-D bf16 tensor in the layouts asked for:
    ``row`` -> a row-major (unit column stride) tensor, ``col`` -> a
    column-major one (unit row stride, the order cuBLASLt's fp8 GEMMs take
    for operand B), both from one read of x (bs_quantize_e4m3_2d).  Same
    codes as ``quantize_e4m3``."""
    from . import _lib, _runtime as R

    R.require_cuda(x, "x")
    if x.dim() != 2 or x.dtype != torch.bfloat16:
        raise TypeError("quantize_e4m3_layouts takes a 2-D bfloat16 tensor")
    xc, transposed = _dense_layout(x)  # xc contiguous; x == xc.T when transposed
    rows, cols = xc.shape
    # q of xc is xc's row-major layout; qT of xc is its column-major one
    want_q = col if transposed else row
    want_qT = row if transposed else col
    q = torch.empty((rows, cols), dtype=_FP8_DTYPE, device=x.device) if want_q else None
    qT = torch.empty((cols, rows), dtype=_FP8_DTYPE, device=x.device) if want_qT else None
    ld = xc.stride(0) if rows > 1 else cols  # a single row's stride is arbitrary
    _lib.call("bs_quantize_e4m3_2d", xc.data_ptr(), rows, cols, ld, scale.data_ptr(),
              R.ptr(q), cols, R.ptr(qT), rows, fp8_flags(), R.stream_handle(x.device))
    if transposed:  # x = xc.T: x's row-major form is qT, its column-major form q.T
        return (qT if row else None), (q.T if col else None)
    return (q if row else None), (qT.T if col else None)


def to_fp8_layouts(x: Tensor, row: bool = True, col: bool = False):
    """(x_fp8 row-major or None, x_fp8 column-major or None, scale): to_fp8
    with the layouts the fp8 GEMMs need, without a transpose pass."""
    scale = fp8_scale(x)
    r, c = quantize_e4m3_layouts(x, scale, row, col)
    return r, c, scale


def _transposed_b8(x: Tensor) -> Tensor:
    """A contiguous copy of x.T for a 2-D contiguous 1-byte tensor (CUDA kernel)."""
    from . import _lib, _runtime as R

    rows, cols = x.shape
    out = torch.empty((cols, rows), dtype=x.dtype, device=x.device)
    _lib.call("bs_transpose_b8", x.data_ptr(), rows, cols, cols, out.data_ptr(), rows,
              R.stream_handle(x.device))
    return out


def _row_major_fp8(x: Tensor) -> Tensor:
    """x with unit column stride (row-major), transposing on the GPU if needed."""
    if x.stride(1) == 1 and x.stride(0) >= x.shape[1]:
        return x
    if x.T.is_contiguous():
        return _transposed_b8(x.T)
    return x.contiguous()


# FP8 GEMMs: "tcgen05" -- this library's kernels for every FP8 GEMM
# (bs_gemm_fp8, and the fused ReLU^2 backward bs_gemm_fp8_relu2);
# "cublaslt" -- F.scaled_mm throughout, as the reference; "hybrid" --
# F.scaled_mm for the plain GEMMs and the fused kernel for the ReLU^2
# backward.  BS_FP8_GEMM in the environment overrides the default.
FP8_GEMM = os.environ.get("BS_FP8_GEMM", "cublaslt")


def gemm_fp8(a: Tensor, bt: Tensor, a_scale: Tensor, b_scale: Tensor) -> Tensor | None:
    """bf16(a @ bt.T * a_scale * b_scale) for e4m3 ``a`` [M, K] and ``bt``
    [N, K] (both with unit column stride: the K-major operands of the
    reference's scaled_mm call, lib_sparse/fp8.py:25-49) on the tcgen05
    tensor cores (``kind::f8f6f4``, fp32 accumulation).  ``None`` when the
    operands' alignment rules out the kernel (TMA needs 16-byte aligned bases
    and row strides)."""
    from . import _lib, _runtime as R

    M, K = a.shape
    N = bt.shape[0]
    if (a.dtype != _FP8_DTYPE or bt.dtype != _FP8_DTYPE or a.stride(1) != 1
            or bt.stride(1) != 1 or bt.shape[1] != K):
        return None
    lda = a.stride(0) if M > 1 else K
    ldb = bt.stride(0) if N > 1 else K
    if a.data_ptr() % 16 or bt.data_ptr() % 16 or lda % 16 or ldb % 16:
        return None
    out = torch.empty((M, N), device=a.device, dtype=torch.bfloat16)
    sa = a_scale.reshape(()).to(torch.float32)
    sb = b_scale.reshape(()).to(torch.float32)
    rc = _lib.load().bs_gemm_fp8(a.data_ptr(), lda, bt.data_ptr(), ldb, out.data_ptr(), N,
                                 M, N, K, sa.data_ptr(), sb.data_ptr(),
                                 R.status_word(a.device).data_ptr(), R.stream_handle(a.device))
    if rc == _lib.BS_ERR_ALIGN:
        return None
    _lib.check(rc, "bs_gemm_fp8")
    return out


def _scaled_mm(a: Tensor, b: Tensor, a_scale: Tensor, b_scale: Tensor,
               output_dtype: torch.dtype) -> Tensor:
    """FP8 GEMM with tensor-wise scales (lib_sparse/fp8.py:25-49): A
    row-major, B column-major, on this library's tcgen05 kernel when
    ``FP8_GEMM == "tcgen05"`` and the operands allow it, else cuBLASLt."""
    if a.stride(1) != 1:
        a = _row_major_fp8(a)
    if b.stride(0) != 1:
        b = _row_major_fp8(b.T).T
    if FP8_GEMM == "tcgen05" and output_dtype == torch.bfloat16:
        out = gemm_fp8(a, b.T, a_scale, b_scale)
        if out is not None:
            return out
    return F.scaled_mm(
        mat_a=a, mat_b=b,
        scale_a=a_scale, scale_b=b_scale, output_dtype=output_dtype,
        scale_recipe_a=F.ScalingType.TensorWise, scale_recipe_b=F.ScalingType.TensorWise,
    )


class MatmulFp8(Function):
    """a @ b through FP8 GEMMs in forward and backward (lib_sparse/fp8.py:52-115)."""

    @staticmethod
    def forward(ctx, a: Tensor, b: Tensor, a_scale: Tensor | None = None,
                b_scale: Tensor | None = None) -> Tensor:
        if not CACHE_FP8_MATMUl:
            ctx.save_for_backward(a, b)
            ctx.a_scale, ctx.b_scale = a_scale, b_scale
        if a.dtype == torch.bfloat16:
            assert a_scale is None
            a_fp8, _, a_scale = to_fp8_layouts(a, row=True)
        else:
            assert a_scale is not None
            a_fp8 = a
        if b.dtype == torch.bfloat16:
            assert b_scale is None
            _, b_fp8, b_scale = to_fp8_layouts(b, row=False, col=True)  # B column-major
        else:
            assert b_scale is not None
            b_fp8 = b
        if CACHE_FP8_MATMUl:
            ctx.save_for_backward(a_fp8, b_fp8, a_scale, b_scale)
        return _scaled_mm(_row_major_fp8(a_fp8), b_fp8, a_scale, b_scale,
                          output_dtype=torch.bfloat16)

    @staticmethod
    def backward(ctx, grad_output: Tensor):
        need_a, need_b = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if CACHE_FP8_MATMUl:
            a_fp8, b_fp8, a_scale, b_scale = ctx.saved_tensors
        else:
            a, b = ctx.saved_tensors
            a_scale, b_scale = ctx.a_scale, ctx.b_scale
            # each operand is quantised straight into the layout its GEMM
            # takes: a^T row-major (a column-major) for grad_b, b row-major
            # (so b^T is column-major) for grad_a
            if a.dtype == torch.bfloat16 and a.dim() == 2 and need_b:
                _, a_fp8, a_scale = to_fp8_layouts(a, row=False, col=True)
            elif a.dtype == torch.bfloat16:
                a_fp8, a_scale = to_fp8(a)
            else:
                a_fp8 = a
            if b.dtype == torch.bfloat16 and b.dim() == 2 and need_a:
                b_fp8, _, b_scale = to_fp8_layouts(b, row=True)
            elif b.dtype == torch.bfloat16:
                b_fp8, b_scale = to_fp8(b)
            else:
                b_fp8 = b
        g = grad_output.contiguous()
        if g.dim() == 2 and g.dtype == torch.bfloat16:
            g_fp8, g_col, g_scale = to_fp8_layouts(g, row=need_a or not need_b, col=need_b)
        else:
            g_fp8, g_scale = to_fp8(g)
            g_col = None
        grad_a = grad_b = None
        if need_a:
            grad_a = _scaled_mm(g_fp8, b_fp8.T, g_scale, b_scale, output_dtype=torch.bfloat16)
        if need_b:
            grad_b = _scaled_mm(_row_major_fp8(a_fp8.T), g_col if g_col is not None else g_fp8,
                                a_scale, g_scale, output_dtype=torch.bfloat16)
        return grad_a, grad_b, None, None


def matmul(a: Tensor, b: Tensor, fp8: bool, a_scale: Tensor | None = None,
           b_scale: Tensor | None = None) -> Tensor:
    """a @ b; FP8 GEMM when ``fp8`` (lib_sparse/fp8.py:118-120)."""
    return MatmulFp8.apply(a, b, a_scale, b_scale) if fp8 else a @ b
