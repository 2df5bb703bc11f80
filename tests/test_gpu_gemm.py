"""K3: the tcgen05 GEMM with the ReLU mask fused into its epilogue, against
a torch fp32 reference of the same product (bf16 operands are exact in
fp32; the GEMM rounds its fp32 accumulator to bf16 once, so it is within one
bf16 rounding of the reference plus accumulation-order effects)."""
import pytest
import torch

import bitsparse_b200 as B
from bitsparse_b200.src.functions import dense_to_tilesparse
from bitsparse_b200.src.operators import mask_with_bitmask_, matmul_relu_mask

pytestmark = pytest.mark.gpu

# |ours - fp32 reference| <= RTOL * max|reference| (bf16 has 8 mantissa bits)
RTOL = 1e-2


def _operands(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    b = torch.randn(K, N, generator=g, device="cuda").to(torch.bfloat16)
    h = torch.randn(M, N, generator=g, device="cuda").relu().to(torch.bfloat16)
    return a, b, h


@pytest.mark.parametrize("M, N, K", [(128, 256, 64), (256, 512, 128), (200, 304, 72),
                                     (1000, 776, 768), (64, 1000, 8), (3, 8, 16)])
def test_gemm_matches_fp32_reference(M, N, K):
    a, b, _ = _operands(M, N, K, M + N + K)
    ref = a.float() @ b.float()
    out = matmul_relu_mask(a, b)
    err = (out.float() - ref).abs().max().item()
    assert err <= RTOL * ref.abs().max().item(), (err, ref.abs().max().item())
    B.check_status()


@pytest.mark.parametrize("M, N, K", [(256, 512, 128), (200, 304, 72), (1024, 3072, 768)])
def test_masked_epilogue_matches_mask_with_bitmask(M, N, K):
    a, b, h = _operands(M, N, K, 7 * M + N)
    sp = dense_to_tilesparse(h, None)
    out = matmul_relu_mask(a, b, sp)
    ref = mask_with_bitmask_((a.float() @ b.float()).to(torch.bfloat16), sp).float()
    keep = h > 0
    assert torch.all(out[~keep] == 0)
    assert not torch.any(torch.signbit(out[~keep]))  # +0 like the reference
    err = (out.float() - ref).abs().max().item()
    assert err <= RTOL * ref.abs().max().item()
    B.check_status()


def test_gemm_rejects_misaligned_operands():
    a, b, _ = _operands(64, 64, 64, 1)
    with pytest.raises(RuntimeError):
        matmul_relu_mask(a, b[:, 1:].contiguous()[:, :60].T.contiguous().T)  # ldb not 8-aligned


@pytest.mark.parametrize("M, N, K", [(256, 512, 128), (200, 304, 72), (1024, 3072, 768),
                                     (8192, 3072, 768), (130, 72, 40)])
@pytest.mark.parametrize("arena", [False, True])
def test_relu2_epilogue_equals_two_steps(M, N, K, arena):
    """The ReLU^2 gradient in the GEMM epilogue == the same GEMM's bf16
    output followed by relu2_grad_sparse_, bit for bit (standalone storage
    and a TensorBuffer at an odd offset); and within RTOL of an fp32
    reference of grad_h * 2r."""
    from bitsparse_b200 import TensorBuffer
    from bitsparse_b200.src.operators import matmul_relu2_grad, relu2_grad_sparse_
    a, b, h = _operands(M, N, K, 3 * M + K)
    buf = None
    if arena:
        buf = TensorBuffer(2 * M * N + 64, device="cuda", dtype=torch.bfloat16)
        buf.offset.fill_(37)
    sp = dense_to_tilesparse(h, None, buf)
    out = matmul_relu2_grad(a, b, sp)
    assert out is not None
    two = relu2_grad_sparse_(matmul_relu_mask(a, b), sp)
    assert torch.equal(out, two)
    ref = torch.where(h > 0, (a.float() @ b.float()) * (2 * h.float()), torch.zeros(()).cuda())
    err = (out.float() - ref).abs().max().item()
    assert err <= 2 * RTOL * ref.abs().max().item()
    assert not torch.any(torch.signbit(out[h == 0]))
    B.check_status()


def test_relu2_epilogue_extreme_values():
    """Stored activations over the whole bf16 exponent range (subnormals to
    the largest finite values) and gradients from tiny to large: the fused
    ReLU^2 epilogue still equals the GEMM followed by relu2_grad_sparse_
    (overflow to inf and underflow to zero included)."""
    from bitsparse_b200.src.operators import matmul_relu2_grad, relu2_grad_sparse_
    M, N, K = 512, 512, 64
    g = torch.Generator(device="cuda").manual_seed(11)
    a = (torch.randn(M, K, generator=g, device="cuda")
         * torch.exp2(torch.randint(-60, 60, (M, 1), generator=g, device="cuda").float()))
    a = a.to(torch.bfloat16)
    b = torch.randn(K, N, generator=g, device="cuda").to(torch.bfloat16)
    e = torch.randint(-133, 127, (M, N), generator=g, device="cuda").float()
    h = (torch.rand(M, N, generator=g, device="cuda") * torch.exp2(e))
    h = torch.where(torch.rand(M, N, generator=g, device="cuda") < 0.4, 0.0, h).to(torch.bfloat16)
    sp = dense_to_tilesparse(h, None)
    out = matmul_relu2_grad(a, b, sp)
    two = relu2_grad_sparse_(matmul_relu_mask(a, b), sp)
    finite = torch.isfinite(two.float()) | torch.isinf(two.float())
    assert torch.equal(out[finite], two[finite])
    B.check_status()


@pytest.mark.parametrize("M, N, K", [(128, 256, 128), (256, 512, 256), (200, 304, 96),
                                     (1000, 776, 768), (3, 8, 16), (4096, 4096, 4096)])
def test_fp8_gemm_matches_fp32_reference(M, N, K):
    """The tcgen05 FP8 GEMM (kind::f8f6f4) against an fp32 restatement of
    the reference's tensor-wise scaled product, (a * sa) @ (b * sb)
    (lib_sparse/fp8.py:25-49), within RTOL, and against cuBLASLt's
    F.scaled_mm on the same operands."""
    import torch.nn.functional as F
    from bitsparse_b200.fp8 import gemm_fp8
    g = torch.Generator(device="cuda").manual_seed(M + 3 * N + K)
    a = (torch.randn(M, K, generator=g, device="cuda") * 3).to(torch.float8_e4m3fn)
    bt = (torch.randn(N, K, generator=g, device="cuda") * 3).to(torch.float8_e4m3fn)
    sa = torch.tensor(0.37, device="cuda")
    sb = torch.tensor(1.9e-2, device="cuda")
    out = gemm_fp8(a, bt, sa, sb)
    assert out is not None and out.dtype == torch.bfloat16 and out.shape == (M, N)
    ref = (a.float() * sa) @ (bt.float() * sb).T
    err = (out.float() - ref).abs().max().item()
    assert err <= RTOL * ref.abs().max().item(), (err, ref.abs().max().item())
    if M % 16 == 0 and N % 16 == 0:
        cub = F.scaled_mm(a, bt.T, scale_a=sa, scale_b=sb, output_dtype=torch.bfloat16,
                          scale_recipe_a=F.ScalingType.TensorWise,
                          scale_recipe_b=F.ScalingType.TensorWise)
        assert (out.float() - cub.float()).abs().max().item() <= RTOL * ref.abs().max().item()
    B.check_status()


@pytest.mark.parametrize("M, N, K", [(256, 512, 256), (200, 304, 96), (2048, 3072, 768)])
@pytest.mark.parametrize("scaled", [False, True])
def test_fp8_relu2_epilogue_equals_two_steps(M, N, K, scaled):
    """The FP8 GEMM with the ReLU^2 gradient of an e4m3-stored activation in
    its epilogue == the same FP8 GEMM followed by relu2_grad_sparse_ (which
    also applies the stored tensor's scale), bit for bit."""
    from bitsparse_b200.fp8 import gemm_fp8, to_fp8
    from bitsparse_b200.src.operators import matmul_fp8_relu2_grad, relu2_grad_sparse_
    g = torch.Generator(device="cuda").manual_seed(5 * M + N)
    a = (torch.randn(M, K, generator=g, device="cuda") * 3).to(torch.float8_e4m3fn)
    bt = (torch.randn(N, K, generator=g, device="cuda") * 3).to(torch.float8_e4m3fn)
    sa, sb = torch.tensor(0.21, device="cuda"), torch.tensor(0.033, device="cuda")
    h = (torch.randn(M, N, generator=g, device="cuda") - 0.5).relu().to(torch.bfloat16)
    if scaled:
        hq, hs = to_fp8(h)
    else:
        hq, hs = h.to(torch.float8_e4m3fn), None
    sp = dense_to_tilesparse(hq, hs)
    out = matmul_fp8_relu2_grad(a, bt, sa, sb, sp)
    assert out is not None
    two = relu2_grad_sparse_(gemm_fp8(a, bt, sa, sb), sp)
    assert torch.equal(out, two)
    assert torch.all(out[hq.float() == 0] == 0)
    B.check_status()


def _dw_case(T, D, H, seed, mu=0.0, arena=False):
    from bitsparse_b200.bitsparse import TensorBuffer
    g = torch.Generator(device="cuda").manual_seed(seed)
    go = torch.randn(T, D, generator=g, device="cuda").to(torch.bfloat16)
    h = (torch.randn(T, H, generator=g, device="cuda") + mu).relu().to(torch.bfloat16)
    buf = None
    if arena:  # a shared arena at an odd value offset: runs start unaligned
        buf = TensorBuffer(2 * T * H + 64, device="cuda", dtype=torch.bfloat16)
        buf.offset.fill_(3)
    return go, h, dense_to_tilesparse(h, None, buf)


@pytest.mark.parametrize("T, D, H", [(64, 256, 64), (1000, 384, 200), (130, 512, 72),
                                     (4096, 768, 3072), (8192, 1024, 4096), (2048, 4096, 1024),
                                     (3000, 1280, 520)])
@pytest.mark.parametrize("relu2", [False, True])
@pytest.mark.parametrize("arena", [False, True])
def test_fused_dw_matches_fp32_reference(T, D, H, relu2, arena):
    """K5: go^T @ h (AspB) / go^T @ (h * h) (AspRelu2B, k = 1) with h
    expanded from its compressed tiles inside the tcgen05 GEMM, against the
    fp32 product of the same bf16 operands (h * h rounded to bf16 as the
    reference's ReLU^2 reconstruct does)."""
    from bitsparse_b200.src.operators import matmul_unpack_dw
    go, h, sp = _dw_case(T, D, H, T + D + H, arena=arena)
    dense = (h * h) if relu2 else h
    ref = go.float().T @ dense.float()
    out = matmul_unpack_dw(go.T, sp, relu2)
    assert out is not None and out.shape == (D, H)
    err = (out.float() - ref).abs().max().item()
    assert err <= RTOL * ref.abs().max().item(), (err, ref.abs().max().item())
    B.check_status()


@pytest.mark.parametrize("mu", [-1.5, -3.0, -50.0])
def test_fused_dw_sparse_and_empty(mu):
    """High sparsity (empty 8-value chunks, empty tiles) and an all-zero h."""
    from bitsparse_b200.src.operators import matmul_unpack_dw
    go, h, sp = _dw_case(2048, 512, 1024, 17, mu=mu)
    ref = go.float().T @ h.float()
    out = matmul_unpack_dw(go.T, sp)
    if mu == -50.0:
        assert torch.count_nonzero(out) == 0
    else:
        err = (out.float() - ref).abs().max().item()
        assert err <= RTOL * ref.abs().max().item()
    B.check_status()


def test_fused_dw_equals_dense_tcgen05_gemm():
    """The fused expansion feeds the tensor cores exactly the dense tile: the
    result equals the tcgen05 GEMM of the dense operands (K3, same K-block
    order) bit for bit.  (1024 tokens: too few K blocks to split K, whose
    partial sums would be added in another order.)"""
    from bitsparse_b200.src.operators import matmul_unpack_dw
    go, h, sp = _dw_case(1024, 512, 2048, 5)
    out = matmul_unpack_dw(go.T, sp)
    ref = matmul_relu_mask(go.T.contiguous(), h)
    assert torch.equal(out, ref)
    B.check_status()
