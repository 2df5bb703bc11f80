"""Autograd layers that keep the MLP activation compressed between forward
and backward (lib_sparse/layers.py, Maxzhu123/bitsparse).

Weight convention (as in the reference's code): W1 [d_ff, d_in],
W2 [d_out, d_ff], y = relu(x W1^T + b1) W2^T + b2.  Same classes, argument
names and gradient tuples as the reference.
"""
from __future__ import annotations

import torch
from torch import Tensor
from torch.autograd import Function

from .bitsparse import BitsparseTensor, TensorBuffer
from .config import RELU2_SCALE
from .fp8 import is_fp8, matmul, to_fp8, to_fp8_layouts
from .src.functions import dense_to_tilesparse, relu_to_tilesparse_fp8
from .src.operators import (compress_bias_relu, compress_bias_relu_fp8, mask_with_bitmask_,
                            matmul_fp8_relu2_grad, matmul_relu2_grad, matmul_relu_mask,
                            relu2_grad_sparse_)
from .src.sparse_matmul import AspB, AspRelu2B


FUSED_MASK_MIN_K = 0


def _tma_ok(t: Tensor) -> bool:
    """A bf16 matrix the tcgen05 GEMM can read with TMA: unit column stride,
    16-byte aligned base and row stride."""
    return (t.dtype == torch.bfloat16 and t.dim() == 2 and t.stride(1) == 1
            and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0)


def _relu_grad(grad_output: Tensor, W: Tensor, h: BitsparseTensor) -> Tensor:
    """grad_z = (grad_output @ W) masked by h > 0 (lib_sparse/layers.py:47-51).

    The tcgen05 GEMM with the mask in its epilogue (the dense grad_h never
    reaches memory; on B200 at the GPT-2-small backward shape, 8192 x 768 @
    768 x 3072, 39.5 us against 47.6 us for cuBLAS + the mask kernel) when
    both operands can be read by TMA and K >= FUSED_MASK_MIN_K; else the
    cuBLAS GEMM followed by mask_with_bitmask_.
    """
    if not grad_output.is_contiguous():
        grad_output = grad_output.contiguous()
    if grad_output.shape[1] >= FUSED_MASK_MIN_K and _tma_ok(grad_output) and _tma_ok(W):
        return matmul_relu_mask(grad_output, W, h)
    return mask_with_bitmask_(matmul(grad_output, W, False), h)


class ReluLinear(Function):
    """y = relu(z) @ W^T with relu(z) stored compressed (lib_sparse/layers.py:20-66)."""

    @staticmethod
    def forward(ctx, z, W, sparse_data: TensorBuffer | None = None, pack_sbit: bool = False,
                dtype: torch.dtype = torch.bfloat16, bias: Tensor | None = None):
        """``bias`` (optional, not in the reference's signature): y =
        relu(z + bias) @ W^T, with the bias add and the ReLU fused into the
        compression pass for bf16 storage (one read of z)."""
        ctx.dtype = dtype
        ctx.has_bias = bias is not None
        ctx.save_for_backward(W)
        fused = None
        if bias is not None and is_fp8(dtype):
            fused = compress_bias_relu_fp8(z, bias, sparse_data, pack_sbit)
            if fused is not None:
                h, scale, h_sparse = fused
        elif bias is not None:
            fused = compress_bias_relu(z, bias, sparse_data, pack_sbit)
            if fused is not None:
                h, h_sparse = fused
                scale = None
        if fused is None:
            if bias is not None:
                z = z + bias
            h = z.relu_()
            if is_fp8(dtype):
                h, h_sparse = relu_to_tilesparse_fp8(h, sparse_data, pack_sbit)
                scale = h_sparse.scale
            else:
                scale = None
                h_sparse = dense_to_tilesparse(h, scale, sparse_data, pack_sbit)
        ctx.h_sparse = h_sparse
        return matmul(h, W.T, is_fp8(dtype), a_scale=scale)

    @staticmethod
    @torch.compiler.disable
    def backward(ctx, grad_output: Tensor):
        W = ctx.saved_tensors[0]
        needs_z = ctx.needs_input_grad[0]
        needs_bias = ctx.has_bias and ctx.needs_input_grad[5]
        # the bias gradient is the column sum of grad_z, so grad_z is formed
        # whenever either of them is wanted
        want_z = needs_z or needs_bias
        h: BitsparseTensor = ctx.h_sparse
        ctx.h_sparse = None
        fp8 = is_fp8(ctx.dtype)
        if fp8:  # both layouts of to_fp8(grad_output) from one pass
            grad_output, go_col, scale = to_fp8_layouts(grad_output.contiguous(), row=want_z,
                                                        col=True)
        else:
            go_col, scale = grad_output, None
        grad_W2 = AspB(go_col.T, h, A_scale=scale) if ctx.needs_input_grad[1] else None
        grad_z = None
        if want_z and not fp8:
            grad_z = _relu_grad(grad_output, W, h)
        elif want_z:
            grad_h = matmul(grad_output, W, fp8=fp8, a_scale=scale)
            grad_z = mask_with_bitmask_(grad_h, h)
        grad_bias = grad_z.sum(0) if needs_bias else None
        return (grad_z if needs_z else None), grad_W2, None, None, None, grad_bias


class FFNRelu:
    """Two-layer ReLU FFN with the hidden activation stored compressed
    (lib_sparse/layers.py:69-94)."""

    @staticmethod
    def apply(x, W1, W2, b1=None, b2=None, *,
              sparse_data: TensorBuffer | None = None, pack_sbit: bool = False,
              dtype: torch.dtype = torch.bfloat16):
        """x [*bs, d_in], W1 [d_ff, d_in], W2 [d_out, d_ff] -> [*bs, d_out]."""
        bs_dims = x.shape[:-1]
        x = x.reshape(-1, x.shape[-1])
        z = matmul(x, W1.T, is_fp8(dtype))
        if b1 is not None:
            # bias add and ReLU fused into the compression pass
            y = ReluLinear.apply(z, W2, sparse_data, pack_sbit, dtype, b1)
        else:
            y = ReluLinear.apply(z, W2, sparse_data, pack_sbit, dtype)
        y = y.reshape(*bs_dims, y.shape[-1])
        if b2 is not None:
            y = y + b2
        return y


class Relu2Linear(Function):
    """y = k relu(z)^2 @ W^T with relu(z) stored compressed
    (lib_sparse/layers.py:100-151)."""

    @staticmethod
    def forward(ctx, z, W, sparse_data: TensorBuffer | None, pack_sbit: bool = False,
                storage_dtype: torch.dtype = torch.bfloat16, bias: Tensor | None = None):
        """``bias`` (optional, not in the reference's signature): relu(z +
        bias), with the bias add, the ReLU, the fp8 quantisations and the
        square fused into the compression passes."""
        ctx.dtype = storage_dtype
        ctx.has_bias = bias is not None
        ctx.save_for_backward(W)
        fp8 = is_fp8(storage_dtype)
        if bias is not None and fp8:
            fused = compress_bias_relu_fp8(z, bias, sparse_data, pack_sbit, square=True)
            if fused is not None:  # the GEMM operand to_fp8(relu(z + b)^2), stored relu
                h2_fp8, h2_scale, ctx.h_sparse = fused
                return matmul(h2_fp8, W.T, True, a_scale=h2_scale)
        elif bias is not None:
            fused = compress_bias_relu(z, bias, sparse_data, pack_sbit)
            if fused is not None:
                h, ctx.h_sparse = fused
                h.square_()
                h.mul_(RELU2_SCALE)
                return matmul(h, W.T, False)
        if bias is not None:
            z = z + bias
        h = z.relu_()
        if fp8:
            _, h_sparse = relu_to_tilesparse_fp8(h, sparse_data, pack_sbit)
        else:
            h_sparse = dense_to_tilesparse(h, None, sparse_data, pack_sbit)
        ctx.h_sparse = h_sparse
        h.square_()
        h.mul_(RELU2_SCALE)
        return matmul(h, W.T, fp8)

    @staticmethod
    @torch.compiler.disable
    def backward(ctx, grad_output: Tensor):
        W = ctx.saved_tensors[0]
        needs_z = ctx.needs_input_grad[0]
        needs_bias = ctx.has_bias and ctx.needs_input_grad[5]
        want_z = needs_z or needs_bias  # the bias gradient is grad_z's column sum
        h: BitsparseTensor = ctx.h_sparse
        ctx.h_sparse = None
        fp8 = is_fp8(ctx.dtype)
        if fp8:  # both layouts of to_fp8(grad_output) from one pass
            grad_output, go_col, scale = to_fp8_layouts(grad_output.contiguous(), row=want_z,
                                                        col=True)
        else:
            go_col, scale = grad_output, None
        grad_W2 = AspRelu2B(go_col.T, h, A_scale=scale) if ctx.needs_input_grad[1] else None
        grad_z = None
        if want_z and not fp8:
            # one tcgen05 GEMM with the ReLU^2 gradient in its epilogue where
            # it applies (bf16 raw storage), else the two steps
            go = grad_output if grad_output.is_contiguous() else grad_output.contiguous()
            grad_z = matmul_relu2_grad(go, W, h) if _tma_ok(go) and _tma_ok(W) else None
            if grad_z is None:
                grad_z = relu2_grad_sparse_(matmul(grad_output, W, False), h)
        elif want_z:
            # FP8: one tcgen05 FP8 GEMM with the ReLU^2 gradient (and the
            # stored tensor's scale) in its epilogue where it applies
            from . import fp8 as F8
            if F8.FP8_GEMM in ("tcgen05", "hybrid"):
                _, w_col, w_scale = to_fp8_layouts(W, row=False, col=True)
                grad_z = matmul_fp8_relu2_grad(grad_output, w_col.T, scale, w_scale, h)
            if grad_z is None:
                grad_h = matmul(grad_output, W, fp8=fp8, a_scale=scale)
                grad_z = relu2_grad_sparse_(grad_h, h)
        grad_bias = grad_z.sum(0) if needs_bias else None
        return (grad_z if needs_z else None), grad_W2, None, None, None, grad_bias


class FFNRelu2:
    """Two-layer ReLU^2 FFN with the hidden activation stored compressed
    (lib_sparse/layers.py:154-177)."""

    @staticmethod
    def apply(x, W1, W2, b1=None, b2=None, *,
              sparse_data: TensorBuffer | None = None, pack_sbit: bool = False,
              storage_dtype: torch.dtype = torch.bfloat16):
        """x [*bs, d_in], W1 [d_ff, d_in], W2 [d_out, d_ff] -> [*bs, d_out]."""
        bs_dims = x.shape[:-1]
        x = x.reshape(-1, x.shape[-1])
        z = matmul(x, W1.T, is_fp8(storage_dtype))
        if b1 is not None:  # bias add fused into the compression passes
            y = Relu2Linear.apply(z, W2, sparse_data, pack_sbit, storage_dtype, b1)
        else:
            y = Relu2Linear.apply(z, W2, sparse_data, pack_sbit, storage_dtype)
        y = y.reshape(*bs_dims, y.shape[-1])
        if b2 is not None:
            y = y + b2
        return y
