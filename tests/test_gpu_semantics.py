"""GPU: pins the two in-kernel semantics that the CPU fixtures cannot pin.

1. ReLU^2 rounding.  The reference's Triton kernels compute the ReLU^2
   reconstruction (lib_sparse/src/triton_kernels.py:231-238) and gradient
   (:323-329) on the GPU; the golden fixtures come from the Triton CPU
   interpreter, which truncates fp32 -> bf16 casts.  Here a few-line Triton
   kernel restates exactly that arithmetic -- ``RELU2_SCALE * v * v`` on the
   loaded values (bf16 storage: in bf16; fp8 storage: promoted to fp32 and
   stored into the bf16 output), and ``where(bit, grad * (2.0 * RELU2_SCALE *
   r.to(fp32)), 0.0)`` stored into the bf16 gradient -- and runs it on this
   GPU.  Its results must equal the oracle's round-to-nearest-even mode and
   this library's kernels, bit for bit, over every positive bf16 pattern and
   every positive e4m3 code.
2. The reference's ``to_fp8`` is ``@torch.compile``d (lib_sparse/fp8.py:
   123-129).  The same three lines compiled by Inductor on this GPU, and
   run eagerly, are compared bit for bit with this library's scale and
   quantiser in its compiled and eager semantics at several magnitudes.
"""
import numpy as np
import pytest
import torch

import bitsparse_b200 as B
from bitsparse_b200.fp8 import fp8_scale, quantize_e4m3
from bitsparse_b200.src.functions import dense_to_tilesparse
from bitsparse_b200.src.operators import relu2_grad_sparse_, unpack_relu2_batch_
from oracle import bitsparse_oracle as O
from tests.gpu_util import bits, oracle_sparse

pytestmark = pytest.mark.gpu

triton = pytest.importorskip("triton")
import triton.language as tl  # noqa: E402

RELU2_SCALE = 1  # lib_sparse/config.py


@triton.jit
def _relu2_ref_kernel(r_ptr, out_ptr, n, K: tl.constexpr, FP32: tl.constexpr,
                      BLOCK: tl.constexpr):
    offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    m = offs < n
    vals = tl.load(r_ptr + offs, mask=m, other=0.0)
    if FP32:
        v = vals.to(tl.float32)
        vals = K * v * v
    else:
        vals = K * vals * vals
    tl.store(out_ptr + offs, vals, mask=m)


@triton.jit
def _relu2_grad_ref_kernel(grad_ptr, r_ptr, n, K: tl.constexpr, BLOCK: tl.constexpr):
    offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    m = offs < n
    grad = tl.load(grad_ptr + offs, mask=m, other=0.0)
    r = tl.load(r_ptr + offs, mask=m, other=0.0)
    active = r.to(tl.float32) > 0
    s = 2.0 * K * r.to(tl.float32)
    g = tl.where(active, grad * s, 0.0)
    tl.store(grad_ptr + offs, g, mask=m)


def _triton_relu2(r, fp32):
    out = torch.empty(r.shape, dtype=torch.bfloat16, device=r.device)
    n = r.numel()
    _relu2_ref_kernel[(triton.cdiv(n, 1024),)](r, out, n, K=RELU2_SCALE, FP32=fp32, BLOCK=1024)
    return out


def _triton_relu2_grad(grad, r):
    g = grad.clone()
    n = g.numel()
    _relu2_grad_ref_kernel[(triton.cdiv(n, 1024),)](g, r, n, K=RELU2_SCALE, BLOCK=1024)
    return g


def _all_positive_bf16():
    p = np.arange(1, 0x7F81, dtype=np.uint32).astype(np.uint16)  # 0 < x <= +inf
    p = np.concatenate([p, np.zeros(256 * 128 - p.size % (256 * 128), np.uint16)])
    return np.random.default_rng(0).permutation(p).reshape(-1, 256)


def test_triton_relu2_reconstruct_rounds_to_nearest_even():
    xb = _all_positive_bf16()
    x = torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).cuda()
    tri = bits(_triton_relu2(x, fp32=False))
    np.testing.assert_array_equal(tri, O.reconstruct_relu2(O.dense_to_tilesparse(xb, O.DT_BF16)))
    sp = dense_to_tilesparse(x, None)
    out = torch.empty_like(x)
    M, N = x.shape
    unpack_relu2_batch_(sp, out, 0, sp.grid_n, N, M, sp.grid_m * sp.grid_n)
    np.testing.assert_array_equal(bits(out), tri)
    # the truncating interpreter would differ somewhere: the pin is not vacuous
    assert not np.array_equal(
        tri, O.reconstruct_relu2(O.dense_to_tilesparse(xb, O.DT_BF16), rounding="trunc"))
    B.check_status()


def test_triton_relu2_grad_rounds_to_nearest_even():
    xb = _all_positive_bf16()
    g = torch.Generator().manual_seed(3)
    grad = (torch.randn(xb.shape, generator=g) * 3).to(torch.bfloat16)
    x = torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16).cuda()
    gd = grad.cuda()
    tri = bits(_triton_relu2_grad(gd, x))
    osp = O.dense_to_tilesparse(xb, O.DT_BF16)
    gb = grad.view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(tri, O.relu2_grad_sparse(gb.copy(), osp))
    sp = dense_to_tilesparse(x, None)
    ours = relu2_grad_sparse_(gd.clone(), sp)
    np.testing.assert_array_equal(bits(ours), tri)
    B.check_status()


def test_triton_relu2_fp8_storage_matches():
    """fp8 storage: the reconstruction promotes to fp32, squares and is
    stored into bf16 (then the scale^2 multiply, a torch op in the
    reference); over every positive e4m3 code."""
    codes = np.tile(np.arange(1, 0x7F, dtype=np.uint8), 64 * 64 // 126 + 1)[: 64 * 64]
    codes = np.random.default_rng(1).permutation(codes).reshape(64, 64)
    q = torch.from_numpy(codes.copy()).view(torch.float8_e4m3fn).cuda()
    scale = torch.tensor(0.0123, dtype=torch.float32, device="cuda")
    tri = _triton_relu2(q, fp32=True).mul_(scale.square())
    sp = dense_to_tilesparse(q, scale)
    out = torch.empty(64, 64, dtype=torch.bfloat16, device="cuda")
    unpack_relu2_batch_(sp, out, 0, sp.grid_n, 64, 64, sp.grid_m * sp.grid_n)
    np.testing.assert_array_equal(bits(out), bits(tri))
    np.testing.assert_array_equal(bits(out), O.reconstruct_relu2(oracle_sparse(sp)))
    B.check_status()


@torch.no_grad()
def _to_fp8_eager(x):
    scale = (x.detach().abs().max() / torch.finfo(torch.float8_e4m3fn).max).to(torch.float32)
    scale = scale.clamp(min=1e-9)
    return (x / scale).to(torch.float8_e4m3fn), scale


@pytest.mark.parametrize("mag", [1e-6, 1e-3, 0.1, 1.0, 7.0, 300.0, 1e4])
def test_to_fp8_compiled_and_eager(mag):
    """The reference's to_fp8 as it runs there (torch.compile'd on this GPU)
    equals this library's fp8_scale + quantize_e4m3 in compiled semantics,
    bit for bit, scale included; the same function run eagerly equals them
    in eager semantics.  (The two arithmetics differ in about 1-3% of the
    codes of bf16 input, and in the scale.)"""
    from bitsparse_b200.fp8 import fp8_semantics
    compiled = torch.compile(_to_fp8_eager)
    g = torch.Generator().manual_seed(int(mag * 1000) % 9973)
    x = (torch.randn(2048, 4096, generator=g) * mag).to(torch.bfloat16).cuda()
    for mode, fn in (("compiled", compiled), ("eager", _to_fp8_eager)):
        qr, sr = fn(x)
        with fp8_semantics(mode):
            s = fp8_scale(x)
            q = quantize_e4m3(x, s)
        assert s.item() == sr.item(), mode
        assert torch.equal(q.view(torch.uint8), qr.view(torch.uint8)), mode


@pytest.mark.parametrize("mode", ["compiled", "eager"])
@pytest.mark.parametrize("mag", [1.0, 5e37])
def test_estimate_path_and_division_path(mode, mag):
    """The quantisers use the plain estimate x * (1/s) wherever a per-block
    exhaustive check over the bf16 codes proves it gives the definition's
    codes at that scale, and the checked division otherwise.  Magnitude 1
    takes the estimate; 5e37 gives a scale above 2^116, outside the check's
    window, so the division path runs.  Both must equal the reference's
    to_fp8 bit for bit: the flat quantiser (8192 x 10240 gives every thread
    the 16+ groups its check needs), the fused quantise + compress, and the
    fused bias + ReLU (+ square) compress."""
    from bitsparse_b200.fp8 import estimate_exact, fp8_semantics, to_fp8
    from bitsparse_b200.src.functions import relu_to_tilesparse_fp8
    from bitsparse_b200.src.operators import compress_bias_relu_fp8
    from tests.gpu_util import reference_to_fp8
    compiled = mode == "compiled"
    g = torch.Generator(device="cuda").manual_seed(5)
    x = (torch.randn(8192, 10240, generator=g, device="cuda") * mag).to(torch.bfloat16)
    b = (torch.randn(10240, generator=g, device="cuda") * (0.25 * mag)).to(torch.bfloat16)
    qr, sr = reference_to_fp8(x, compiled)
    with fp8_semantics(mode):
        q, s = to_fp8(x)
        assert estimate_exact(s) == (mag == 1.0)
    assert s.item() == sr.item()
    assert torch.equal(q.view(torch.uint8), qr.view(torch.uint8))
    h = torch.relu(x)
    qr, sr = reference_to_fp8(h, compiled)
    with fp8_semantics(mode):
        q, sp = relu_to_tilesparse_fp8(h)
    assert sp.scale.item() == sr.item()
    assert torch.equal(q.view(torch.uint8), qr.view(torch.uint8))
    h = torch.relu(x + b)
    square = mag == 1.0  # h * h of the large case would overflow bf16
    qr, sr = reference_to_fp8(h * h if square else h, compiled)
    with fp8_semantics(mode):
        side, side_scale, sp = compress_bias_relu_fp8(x, b, None, False, square=square)
    assert side_scale.item() == sr.item()
    assert torch.equal(side.view(torch.uint8), qr.view(torch.uint8))
    B.check_status()


@pytest.mark.parametrize("mode", ["compiled", "eager"])
def test_quantise_at_scales_outside_the_check(mode):
    """quantize_e4m3 with a caller's scale that the exactness check refuses
    (2^-133, fp32-subnormal, whose reciprocal overflows): the division path
    gives the definition's codes, e4m3(x / s) by Triton's division
    (compiled) or e4m3(bf16(x / s)) (eager).  The scale is a bf16 value, as
    to_fp8's eager scales are (torch's eager division rounds an fp32 scale
    to the bf16 operand's type first), and |x / s| stays within e4m3's
    range, where torch's eager cast and the saturating hardware conversion
    agree."""
    from bitsparse_b200.fp8 import estimate_exact, fp8_semantics
    g = torch.Generator(device="cuda").manual_seed(6)
    x = (torch.randn(8192, 10240, generator=g, device="cuda") * 1e-39).to(torch.bfloat16)
    s = torch.tensor(2.0 ** -133, device="cuda", dtype=torch.float32)
    with fp8_semantics(mode):
        assert not estimate_exact(s)

    def ref(t, sc):
        return (t / sc).to(torch.float8_e4m3fn)

    qr = (torch.compile(ref) if mode == "compiled" else ref)(x, s)
    with fp8_semantics(mode):
        q = quantize_e4m3(x, s)
    assert torch.equal(q.view(torch.uint8), qr.view(torch.uint8))
