"""GPU parity at the benchmarked sizes: config 3 (8192 x 14336 bf16) at 50%
and 99% sparsity, with per-row Beta(2,2) densities and with zeroed 64-column
strips, and config 4's activation (16384 x 16384 quantised to e4m3: exactly
65536 tiles), raw and pack_sbit.

Inputs are generated on the CPU from fixed seeds.  Bitmask, prefix and raw
values are compared with the oracle byte for byte.  A packed stream is
checked by decoding every value at its logical index (the oracle's decoder,
pinned on the golden fixtures) against the oracle's raw values, and every
bit outside the payload must be zero: together these fix the whole stream
bit for bit.  The FP8 bytes of config 4 are compared with the reference's
to_fp8 (lib_sparse/fp8.py:123-129) run on the same GPU, eagerly and
torch.compile'd."""
import numpy as np
import pytest
import torch

import bitsparse_b200 as B
from bitsparse_b200 import bits_per_value
from bitsparse_b200.src.functions import dense_to_tilesparse, relu_to_tilesparse_fp8
from bitsparse_b200.src.operators import unpack_batch_
from bench import make_relu_bf16
from oracle import bitsparse_oracle as O
from tests.gpu_util import bits, reference_to_fp8

pytestmark = pytest.mark.gpu

M3, N3 = 8192, 14336


def _check_against_oracle(sp, dense_bits, odt, pack):
    M, N = dense_bits.shape
    bm, counts = O.tile_pack(dense_bits, M, N, odt)
    np.testing.assert_array_equal(bits(sp.bitmask), bm)
    prefix = O.tile_prefix(counts)
    np.testing.assert_array_equal(bits(sp.prefix), prefix)
    raw = O.compact_values(dense_bits, M, N, odt)
    nnz = raw.size
    v = bits(sp.vals)
    if not pack:
        np.testing.assert_array_equal(v[:nnz], raw)
        return nnz
    nb = bits_per_value(sp.dtype)
    assert v.size == O.packed_storage_nbytes(nnz, nb)
    dec = O.unpack_values(v, np.arange(nnz, dtype=np.int64), nb)
    keep = (1 << nb) - 1
    np.testing.assert_array_equal(dec, raw.astype(np.uint16) & keep)
    # nothing outside the payload: whole bytes past it, then the last byte's top bits
    end_bits = nnz * nb
    assert not v[(end_bits + 7) // 8:].any()
    if end_bits % 8:
        assert (int(v[end_bits // 8]) >> (end_bits % 8)) == 0
    return nnz


@pytest.mark.parametrize("variant, target, mu", [
    ("A", 0.5, 0.0), ("A", 0.99, -2.3263), ("B", 0.9, 0.0), ("C", 0.9, 0.0)])
@pytest.mark.parametrize("pack", [False, True])
def test_config3_full_size(variant, target, mu, pack):
    x = make_relu_bf16(M3, N3, mu, 17, torch.device("cpu"), variant, target)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    xd = x.cuda()
    sp = dense_to_tilesparse(xd, None, None, pack)
    torch.cuda.synchronize()
    nnz = _check_against_oracle(sp, xb, O.DT_BF16, pack)
    assert abs(1 - nnz / xb.size - target) < 0.03
    out = torch.empty_like(xd)
    unpack_batch_(sp, out, 0, sp.grid_n, N3, M3, sp.grid_m * sp.grid_n)
    assert torch.equal(out, xd)
    B.check_status()


@pytest.mark.parametrize("pack", [False, True])
@pytest.mark.parametrize("semantics", ["compiled", "eager"])
def test_config4_fp8_full_size(pack, semantics):
    """16384 x 16384 relu(N(0,1)) quantised + compressed in one pass:
    T = 65536 tiles (one whole _PACK_CHUNK_TILES chunk of the reference).
    The FP8 bytes are compared with the reference's to_fp8 run on the same
    GPU, eagerly or torch.compile'd."""
    from bitsparse_b200.fp8 import fp8_semantics
    M = N = 16384
    g = torch.Generator().manual_seed(23)
    x = torch.randn(M, N, generator=g).relu_().to(torch.bfloat16)
    xd = x.cuda()
    del x
    q_ref, scale = reference_to_fp8(xd, compiled=semantics == "compiled")
    with fp8_semantics(semantics):
        q, sp = relu_to_tilesparse_fp8(xd, None, pack)
    assert sp.grid_m * sp.grid_n == 65536
    assert sp.scale.item() == scale.item()
    assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8))
    qb = bits(q_ref)
    del q, q_ref
    _check_against_oracle(sp, qb, O.DT_E4M3, pack)
    B.check_status()
