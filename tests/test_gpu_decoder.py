"""GPU: the config-5 decoder whose MLP activations are stored compressed.

Compressed MLP storage (per-layer storage and one shared TensorBuffer arena)
gives bit-identical losses and gradients to each other, and matches the
same decoder with dense MLP activations within bf16 tolerance (the dense
MLP's GEMMs fuse the bias, ours add it in the compression pass)."""
import pytest
import torch

import bitsparse_b200 as B
from bitsparse_b200.decoder import Decoder, DecoderConfig

pytestmark = pytest.mark.gpu


def _run(cfg, tok):
    torch.manual_seed(0)
    m = Decoder(cfg).to(device="cuda", dtype=torch.bfloat16)
    loss = m(tok[:, :-1], tok[:, 1:])
    loss.backward()
    return loss.detach().float(), [p.grad.float() for p in m.parameters()]


def test_decoder_compressed_matches_dense():
    small = dict(vocab=512, layers=2, dim=128, heads=4, mlp=512, seq=64)
    tok = torch.randint(0, 512, (4, 65), generator=torch.Generator().manual_seed(1)).cuda()
    lc, gc = _run(DecoderConfig(compressed=True, **small), tok)
    la, ga = _run(DecoderConfig(compressed=True, arena_fraction=1.0, **small), tok)
    ld, gd = _run(DecoderConfig(compressed=False, **small), tok)
    assert torch.equal(lc, la)
    for a, b in zip(gc, ga):
        assert torch.equal(a, b)
    assert abs(lc.item() - ld.item()) <= 1e-2 * abs(ld.item())
    num = sum(((a - b) ** 2).sum() for a, b in zip(gc, gd)).sqrt()
    den = sum((b ** 2).sum() for b in gd).sqrt()
    assert (num / den).item() < 3e-2
    B.check_status()
