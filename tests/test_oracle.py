"""Pin the CPU oracle to the reference's own outputs (tests/golden/golden.npz).

The fixtures were produced by running the reference lib_sparse on the CPU
(tests/golden/make_golden.py).  Every oracle function the GPU parity tests
rely on is checked here against them, bit for bit.
"""
import hashlib

import numpy as np
import pytest

from oracle import bitsparse_oracle as O
from tests.conftest import golden_cases, parse_case
from tests.golden.fixtures import arena_inputs, case_inputs, check, has
from tests.golden.make_golden import SHAPES_FULL, SPARSITIES


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _payload(vals, start, nnz, bits):
    out = vals.copy()
    sb = np.unpackbits(out, bitorder="little")
    idx = np.arange(sb.size)
    sb &= ((idx >= start * bits) & (idx < (start + nnz) * bits)).astype(np.uint8)
    return np.packbits(sb, bitorder="little")


def test_round_trip_cases(golden):
    cases = golden_cases(golden, "v/")
    assert len(cases) == 3 * 2 * 13
    for case, f in sorted(cases.items()):
        dtype, pack, (M, N), sp_ = parse_case(case)
        dense, grad = case_inputs(f, dtype, (M, N), sp_)
        sp = O.dense_to_tilesparse(dense, dtype, None, pack)
        check(f, "bitmask", sp.bitmask, case)
        check(f, "prefix", sp.prefix, case)
        if pack:
            check(f, "vals", _payload(sp.vals, 0, sp.nnz, O.bits_per_value(dtype)), case)
        else:
            check(f, "vals", sp.vals, case)
        check(f, "recon", O.reconstruct(sp), case)
        if has(f, "recon_relu2"):
            check(f, "recon_relu2", O.reconstruct_relu2(sp, rounding="trunc"), case)
        check(f, "mask_grad", O.mask_with_bitmask(grad.copy(), sp), case)
        check(f, "relu2_grad", O.relu2_grad_sparse(grad.copy(), sp, "trunc"), case)


def test_shared_arena(golden):
    for dtype in (O.DT_BF16, O.DT_E4M3, O.DT_E5M2):
        for pack in (0, 1):
            k = f"a/{dtype}/{pack}/"
            arena = O.Arena(int(golden[k + "size"]), dtype, bool(pack))
            offs = []
            for d in arena_inputs(golden, k, dtype, SHAPES_FULL, SPARSITIES):
                sp = O.dense_to_tilesparse(d, dtype, arena, bool(pack))
                offs.append(sp.vals_offset)
            np.testing.assert_array_equal(offs, golden[k + "vals_offsets"])
            assert arena.offset == int(golden[k + "final_offset"])
            sub = {kk[len(k):]: v for kk, v in golden.items() if kk.startswith(k)}
            check(sub, "arena", arena.vals, k)


def test_config1_fp8(golden):
    torch = pytest.importorskip("torch")
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1024, 3072, generator=g, dtype=torch.float32)
    assert _sha(x.numpy()) == str(golden["c1/x_sha"]), "CPU RNG stream differs"
    h = np.maximum(x.numpy(), 0)
    q, scale = O.to_fp8(h, "float32")
    assert scale == golden["c1/scale"]
    assert _sha(q) == str(golden["c1/q_sha"])
    hb = O.f32_to_bf16(h)
    for name, dense, dt in (("fp8", q, O.DT_E4M3), ("bf16", hb, O.DT_BF16)):
        for pack in (0, 1):
            k = f"c1/{name}/{pack}/"
            if k + "nnz" not in golden:
                continue
            sp = O.dense_to_tilesparse(dense, dt, None, bool(pack))
            assert sp.nnz == int(golden[k + "nnz"])
            assert _sha(sp.bitmask) == str(golden[k + "bitmask_sha"])
            assert _sha(sp.prefix) == str(golden[k + "prefix_sha"])
            v = sp.vals
            if pack:
                v = _payload(v, 0, sp.nnz, O.bits_per_value(dt))
            assert _sha(v) == str(golden[k + "vals_sha"]), k
            assert _sha(O.reconstruct(sp)) == str(golden[k + "recon_sha"])


def test_to_fp8_bf16_matches_torch_eager():
    """The bf16-input branch of to_fp8 against torch eager on the CPU."""
    torch = pytest.importorskip("torch")
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(257, 333, generator=g) * 3).relu().to(torch.bfloat16)
    amax = x.abs().max()
    s = (amax / 448.0).to(torch.float32).clamp(min=1e-9)
    q = (x / s).to(torch.float8_e4m3fn)
    qo, so = O.to_fp8(x.view(torch.uint16).numpy(), "bfloat16")
    assert so == s.item()
    np.testing.assert_array_equal(qo, q.view(torch.uint8).numpy())


def test_fp8_conversions_exhaustive():
    torch = pytest.importorskip("torch")
    # every bf16 bit pattern through both fp8 casts
    allb = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    f = O.bf16_to_f32(allb)
    tf = torch.from_numpy(f.copy())
    for dt, tdt in ((O.DT_E4M3, torch.float8_e4m3fn), (O.DT_E5M2, torch.float8_e5m2)):
        ours = O.f32_to_fp8(f, dt)
        ref = tf.to(tdt).view(torch.uint8).numpy()
        nan = np.isnan(f)
        np.testing.assert_array_equal(ours[~nan], ref[~nan])
        back = O.fp8_to_f32(np.arange(256, dtype=np.uint8), dt)
        tb = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(tdt).float().numpy()
        np.testing.assert_array_equal(np.isnan(back), np.isnan(tb))
        ok = ~np.isnan(back)
        np.testing.assert_array_equal(back[ok], tb[ok])
    # fp32 -> bf16 on random fp32 patterns
    r = np.random.default_rng(0).integers(0, 2 ** 32, 200000, dtype=np.uint64).astype(np.uint32)
    fr = r.view(np.float32)
    ok = ~np.isnan(fr)
    ref = torch.from_numpy(fr.copy()).to(torch.bfloat16).view(torch.uint16).numpy()
    np.testing.assert_array_equal(O.f32_to_bf16(fr)[ok], ref[ok])


def test_prefix_wraps_like_int32_cumsum():
    c = np.full(5, 2 ** 30, dtype=np.int64)
    p = O.tile_prefix(c)
    assert p.dtype == np.uint32 and p[-1] == (5 * 2 ** 30) % 2 ** 32
