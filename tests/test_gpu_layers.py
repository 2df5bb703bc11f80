"""GPU: the autograd layers against a dense PyTorch reference of the same op.

Tolerances (relative Frobenius error of each output / gradient vs an fp32
reference computed from the same bf16 inputs): bf16 storage 2e-2 (the
bf16 GEMM outputs alone account for about 1e-2), FP8 storage 8e-2 (e4m3
keeps 3 mantissa bits).
"""
import numpy as np
import pytest
import torch

import bitsparse_b200 as B
from bitsparse_b200 import TensorBuffer
import bitsparse_b200.src.sparse_matmul as SM
from bitsparse_b200.layers import FFNRelu, FFNRelu2
from tests.golden.fixtures import has

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def make(T, d, H, do, seed, bias_shift=0.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, d, generator=g).to(torch.bfloat16).cuda()
    W1 = (0.02 * torch.randn(H, d, generator=g)).to(torch.bfloat16).cuda()
    W2 = (0.02 * torch.randn(do, H, generator=g)).to(torch.bfloat16).cuda()
    b1 = torch.full((H,), bias_shift).to(torch.bfloat16).cuda()
    b2 = (0.1 * torch.randn(do, generator=g)).to(torch.bfloat16).cuda()
    gy = torch.randn(T, do, generator=g).to(torch.bfloat16).cuda()
    return x, W1, W2, b1, b2, gy


def dense_ref(x, W1, W2, b1, b2, gy, relu2):
    ps = [t.detach().float().requires_grad_() for t in (x, W1, W2, b1, b2)]
    xf, W1f, W2f, b1f, b2f = ps
    h = torch.relu(xf @ W1f.T + b1f)
    if relu2:
        h = h * h
    y = h @ W2f.T + b2f
    y.backward(gy.float())
    return y.detach(), [p.grad for p in ps]


def run(layer, params, gy, **kw):
    ps = [t.detach().clone().requires_grad_() for t in params]
    y = layer.apply(*ps, **kw)
    y.backward(gy)
    return y.detach(), [p.grad for p in ps]


@pytest.mark.parametrize("relu2", [False, True])
@pytest.mark.parametrize("pack", [False, True])
@pytest.mark.parametrize("arena", [False, True])
def test_ffn_bf16(relu2, pack, arena):
    T, d, H, do = 1024, 256, 1024, 256
    x, W1, W2, b1, b2, gy = make(T, d, H, do, seed=1, bias_shift=-0.02)
    kw = {"pack_sbit": pack}
    if arena:
        kw["sparse_data"] = TensorBuffer(T * H * 2, device="cuda", dtype=torch.bfloat16,
                                         pack_sbit=pack)
    layer = FFNRelu2 if relu2 else FFNRelu
    y, grads = run(layer, (x, W1, W2, b1, b2), gy, **kw)
    yr, gr = dense_ref(x, W1, W2, b1, b2, gy, relu2)
    assert rel(y, yr) < 2e-2
    for n, a, b in zip(("x", "W1", "W2", "b1", "b2"), grads, gr):
        assert rel(a, b) < 2e-2, n
    B.check_status()


def test_ffn_relu_matches_reference_golden(golden):
    """FFNRelu fwd+bwd against the reference's own CPU run (bf16 GEMMs on the
    CPU there, cuBLAS here: equal within bf16 GEMM rounding)."""
    def t(name):
        a = golden["ffn/" + name]
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).cuda()
    if not all(has({k[4:]: 1 for k in golden if k.startswith("ffn/")}, n)
               for n in ("x", "W1", "W2", "b1", "b2", "gy", "y")):
        pytest.skip("ffn fixture stored as digests only")
    params = [t(n) for n in ("x", "W1", "W2", "b1", "b2")]
    y, grads = run(FFNRelu, params, t("gy"))
    assert rel(y, t("y")) < 1e-2
    for n, gt in zip(("x", "W1", "W2", "b1", "b2"), grads):
        if "ffn/d" + n in golden:
            assert rel(gt, t("d" + n)) < 2e-2, n


class _DenseTwin(torch.autograd.Function):
    """The reference's ReluLinear / Relu2Linear (lib_sparse/layers.py:20-151)
    with the activation saved DENSE instead of compressed, built from the
    same matmul calls.  The compressed layers must match it bit for bit:
    compression is lossless, so only the storage differs."""

    @staticmethod
    def forward(ctx, z, W, relu2, fp8, fused_dw=False):
        from bitsparse_b200.fp8 import matmul, to_fp8
        ctx.relu2, ctx.fp8, ctx.fused_dw = relu2, fp8, fused_dw
        ctx.save_for_backward(W)
        h = z.relu_()
        if fp8:
            h_st, scale = to_fp8(h)
        else:
            h_st, scale = h.clone(), None
        ctx.h_st, ctx.scale = h_st, scale
        if relu2:
            h.square_()
            return matmul(h, W.T, fp8)
        return matmul(h_st if fp8 else h, W.T, fp8, a_scale=scale)

    @staticmethod
    def backward(ctx, go):
        from bitsparse_b200.fp8 import matmul, to_fp8
        W = ctx.saved_tensors[0]
        h, scale, fp8 = ctx.h_st, ctx.scale, ctx.fp8
        gscale = None
        if fp8:
            go, gscale = to_fp8(go.contiguous())
        r = h.float()
        mask = r > 0
        if ctx.relu2:
            dense = (r * r).to(torch.bfloat16)
            if scale is not None:
                dense.mul_(scale.square())
            gW = _twin_dw(go, dense, ctx.fused_dw) if not fp8 else \
                matmul(go.T, dense, fp8, a_scale=gscale)
            if fp8:
                gh = matmul(go, W, fp8=fp8, a_scale=gscale)
            else:  # the layer's grad_h comes from the tcgen05 GEMM (ReLU^2 epilogue)
                from bitsparse_b200.src.operators import matmul_relu_mask
                gh = matmul_relu_mask(go.contiguous(), W)
            gz = torch.where(mask, (gh.float() * (2.0 * r)).to(torch.bfloat16),
                             torch.zeros((), dtype=torch.bfloat16, device=gh.device))
            if scale is not None:
                gz.mul_(scale)
        elif not fp8:
            # the layer's own grad_z path (fused masked GEMM), with the mask
            # taken from the dense activation kept here
            from bitsparse_b200.layers import _relu_grad
            from bitsparse_b200.src.functions import dense_to_tilesparse
            gW = _twin_dw(go, h, ctx.fused_dw)
            gz = _relu_grad(go, W, dense_to_tilesparse(h.contiguous(), None))
        else:
            gW = matmul(go.T, h, fp8, a_scale=gscale, b_scale=scale)
            gh = matmul(go, W, fp8=fp8, a_scale=gscale)
            gz = torch.where(mask, gh, torch.zeros((), dtype=gh.dtype, device=gh.device))
        return gz, gW, None, None, None


def _twin_dw(go, dense, fused_dw):
    """The twin's dW2 = go^T @ dense: where the layer's GEMM expands the
    compressed activation inside a tcgen05 GEMM (raw bf16 storage), the same
    tensor-core accumulation on the dense operand (K3 on go^T); else cuBLAS."""
    from bitsparse_b200.src.operators import matmul_relu_mask
    if fused_dw:
        return matmul_relu_mask(go.T.contiguous(), dense.contiguous())
    return go.T @ dense


def _twin_ffn(x, W1, W2, b1, b2, relu2, fp8, fused_dw=False):
    from bitsparse_b200.fp8 import matmul
    z = matmul(x, W1.T, fp8) + b1
    return _DenseTwin.apply(z, W2, relu2, fp8, fused_dw) + b2


@pytest.mark.parametrize("relu2", [False, True])
@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("pack", [False, True])
def test_ffn_bit_exact_vs_dense_activation_twin(relu2, fp8, pack):
    """Compressed FFN == the same FFN with a dense saved activation, exactly."""
    T, d, H, do = 512, 256, 1024, 256
    x, W1, W2, b1, b2, gy = make(T, d, H, do, seed=3, bias_shift=-0.01)
    layer = FFNRelu2 if relu2 else FFNRelu
    dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    kw = {"pack_sbit": pack, ("storage_dtype" if relu2 else "dtype"): dt}
    y, grads = run(layer, (x, W1, W2, b1, b2), gy, **kw)
    ps = [t.detach().clone().requires_grad_() for t in (x, W1, W2, b1, b2)]
    yt = _twin_ffn(*ps, relu2, fp8, fused_dw=SM.FUSED_DW and not fp8 and not pack)
    yt.backward(gy)
    assert torch.equal(y, yt.detach())
    for n, a, p in zip(("x", "W1", "W2", "b1", "b2"), grads, ps):
        assert torch.equal(a, p.grad), n
    B.check_status()


@pytest.mark.parametrize("relu2", [False, True])
def test_ffn_fused_dw_bit_exact(monkeypatch, relu2):
    """With the fused reconstruct + tcgen05 weight-gradient GEMM selected,
    the bf16 FFN equals its dense-activation twin (whose dW2 is the tcgen05
    GEMM of the dense operands) bit for bit."""
    monkeypatch.setattr(SM, "FUSED_DW", True)
    T, d, H, do = 512, 256, 1024, 256
    x, W1, W2, b1, b2, gy = make(T, d, H, do, seed=8, bias_shift=-0.01)
    y, grads = run(FFNRelu2 if relu2 else FFNRelu, (x, W1, W2, b1, b2), gy)
    ps = [t.detach().clone().requires_grad_() for t in (x, W1, W2, b1, b2)]
    yt = _twin_ffn(*ps, relu2, False, fused_dw=True)
    yt.backward(gy)
    assert torch.equal(y, yt.detach())
    for n, a, p in zip(("x", "W1", "W2", "b1", "b2"), grads, ps):
        assert torch.equal(a, p.grad), n
    B.check_status()


@pytest.mark.parametrize("relu2", [False, True])
def test_ffn_fp8(relu2):
    """FP8 storage against the fp32 dense reference: e4m3 operands in four
    GEMMs (3 mantissa bits each) give about 10% relative error on the
    gradients; the tolerance is 0.2."""
    T, d, H, do = 1024, 256, 1024, 256
    x, W1, W2, b1, b2, gy = make(T, d, H, do, seed=2)
    layer = FFNRelu2 if relu2 else FFNRelu
    kw = {"storage_dtype": torch.float8_e4m3fn} if relu2 else {"dtype": torch.float8_e4m3fn}
    y, grads = run(layer, (x, W1, W2, b1, b2), gy, **kw)
    yr, gr = dense_ref(x, W1, W2, b1, b2, gy, relu2)
    assert rel(y, yr) < 0.2
    for n, a, b in zip(("x", "W1", "W2", "b1", "b2"), grads, gr):
        assert rel(a, b) < 0.2, n


def test_ffn_fused_masked_gemm_path_bit_exact(monkeypatch):
    """The bf16 FFN with grad_z from the fused masked tcgen05 GEMM (forced
    for this small K) equals its dense-activation twin bit for bit."""
    import bitsparse_b200.layers as L
    monkeypatch.setattr(L, "FUSED_MASK_MIN_K", 0)
    T, d, H, do = 512, 256, 1024, 256
    x, W1, W2, b1, b2, gy = make(T, d, H, do, seed=5, bias_shift=-0.01)
    y, grads = run(FFNRelu, (x, W1, W2, b1, b2), gy)
    ps = [t.detach().clone().requires_grad_() for t in (x, W1, W2, b1, b2)]
    yt = _twin_ffn(*ps, False, False, fused_dw=SM.FUSED_DW)
    yt.backward(gy)
    assert torch.equal(y, yt.detach())
    for n, a, p in zip(("x", "W1", "W2", "b1", "b2"), grads, ps):
        assert torch.equal(a, p.grad), n
    B.check_status()


@pytest.mark.parametrize("relu2", [False, True])
@pytest.mark.parametrize("fp8", [False, True])
def test_bias_only_gradient(relu2, fp8):
    """x, W1 and W2 frozen, only b1 trains: b1 still gets its gradient (the
    column sum of grad_z), equal to the dense-activation twin's."""
    T, d, H, do = 512, 256, 1024, 256
    x, W1, W2, b1, b2, gy = make(T, d, H, do, seed=6, bias_shift=-0.01)
    layer = FFNRelu2 if relu2 else FFNRelu
    dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    kw = {("storage_dtype" if relu2 else "dtype"): dt}
    bb = b1.detach().clone().requires_grad_()
    y = layer.apply(x, W1, W2, bb, b2, **kw)
    y.backward(gy)
    bt = b1.detach().clone().requires_grad_()
    yt = _twin_ffn(x, W1, W2, bt, b2, relu2, fp8)
    yt.backward(gy)
    assert bb.grad is not None
    assert torch.equal(bb.grad, bt.grad)
    B.check_status()
