"""The per-tile FP8 scale mode (an extension: the reference's to_fp8 is per
tensor).  The CPU restatement in the oracle is its specification: CPU tests
check the restatement's own properties; GPU tests compare the one-pass
kernel and the dequantising reconstruct with it bit for bit."""
import numpy as np
import pytest
import torch

from oracle import bitsparse_oracle as O


def _bits(x: np.ndarray) -> np.ndarray:
    return O.f32_to_bf16(x.astype(np.float32))


def _case(M, N, seed, mu=0.0, specials=False):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((M, N)) * np.exp(rng.standard_normal((M, 1)) * 2) + mu)
    x = x.astype(np.float32)
    if specials:
        x[:64, :64] = 0.0                                  # an all-zero tile
        if N > 64:
            x[0, 64] = np.nan                              # NaN is ignored by the amax
        if M > 64:
            x[64, 0] = np.inf                              # an infinite amax
        x[-1, -1] = -3.0                                   # negatives are never stored
    return _bits(x)


def test_oracle_tile_scaled_properties():
    bits = _case(200, 264, 1, specials=True)
    codes, scales = O.to_fp8_tile_scaled(bits)
    gm, gn, T, _, _ = O.tile_grid(200, 264)
    assert scales.shape == (T,) and scales.dtype == np.float32
    assert scales[0] == 1.0 and not codes[:64, :64].any()  # the zero tile
    x = O.bf16_to_f32(bits)
    for tm in range(gm):
        for tn in range(gn):
            blk = x[tm * 64:(tm + 1) * 64, tn * 64:(tn + 1) * 64]
            a = np.where(np.isnan(blk), 0, np.abs(blk))
            am = np.float32(a.max())
            s = scales[tm * gn + tn]
            if am == 0 or not np.isfinite(am):
                continue
            assert s == np.float32(am / np.float32(448))
            c = codes[tm * 64:(tm + 1) * 64, tn * 64:(tn + 1) * 64]
            # the largest magnitude of the tile maps to +-448 (code 0x7E / 0xFE)
            i = np.unravel_index(np.argmax(a), a.shape)
            assert c[i] & 0x7F == 0x7E
    # dequantised round trip: within half an e4m3 step of each positive value
    sp = O.dense_to_tilesparse(codes, O.DT_E4M3, None, False)
    r = O.bf16_to_f32(O.reconstruct_tile_scaled(sp, scales))
    pos = (x > 0) & np.isfinite(x)
    sfull = np.repeat(np.repeat(scales.reshape(gm, gn), 64, 0), 64, 1)[:200, :264]
    fin = np.isfinite(sfull)
    err = np.abs(r - np.where(pos, x, 0))
    tol = np.maximum(np.abs(x) * 2.0 ** -4, sfull * 2.0 ** -9) * 1.01 + 1e-30
    ok = (err <= tol) | ~fin | (r == 0)
    assert ok[pos].all()




@pytest.mark.gpu
@pytest.mark.parametrize("M, N", [(130, 200), (64, 64), (1, 8), (1000, 3000), (257, 72)])
@pytest.mark.parametrize("pack", [False, True])
@pytest.mark.parametrize("arena", [False, True])
def test_tile_scaled_compress_and_reconstruct_match_oracle(M, N, pack, arena):
    import bitsparse_b200 as B
    from bitsparse_b200 import TensorBuffer
    from bitsparse_b200.src.operators import compress_fp8_tile_scaled, unpack_tile_scaled_
    from tests.gpu_util import bits
    hb = _case(M, N, M * 7 + N, specials=M >= 64 and N >= 64)
    h = torch.from_numpy(hb.view(np.int16)).view(torch.bfloat16).cuda()
    buf = None
    if arena:
        buf = TensorBuffer(M * N + 64, device="cuda", dtype=torch.float8_e4m3fn, pack_sbit=pack)
        buf.offset.fill_(5)
    sp = compress_fp8_tile_scaled(h, buf, pack)
    codes, scales = O.to_fp8_tile_scaled(hb)
    np.testing.assert_array_equal(bits(sp.tile_scales).view(np.uint32), scales.view(np.uint32))
    osp = O.dense_to_tilesparse(codes, O.DT_E4M3, None, pack)
    np.testing.assert_array_equal(bits(sp.bitmask), osp.bitmask)
    np.testing.assert_array_equal(bits(sp.prefix), osp.prefix)
    nnz = int(osp.prefix[-1])
    v = bits(sp.vals)
    if not pack:
        off = int(sp.vals_offset.item())
        np.testing.assert_array_equal(v[off:off + nnz], osp.vals[:nnz])
    else:
        off = int(sp.vals_offset.item())
        dec = O.unpack_values(v, np.arange(off, off + nnz, dtype=np.int64), 7)
        np.testing.assert_array_equal(dec, O.compact_values(codes, M, N, O.DT_E4M3) & 0x7F)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    unpack_tile_scaled_(sp, out)
    np.testing.assert_array_equal(bits(out), O.reconstruct_tile_scaled(osp, scales))
    B.check_status()
