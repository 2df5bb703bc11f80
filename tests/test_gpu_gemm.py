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
