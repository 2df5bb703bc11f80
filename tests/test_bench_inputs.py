"""The bench's synthetic activations have the sparsity their sweep labels
name (a density passed where a sparsity was expected once made the "B90"
case run at 22% sparsity).  CPU only, small shapes."""
import pytest
import torch

from bench import make_relu_bf16

# (target sparsity, mean of the N(mu, 1) draw) as the sweep uses them
CASES = [("A", 0.5, 0.0), ("A", 0.9, -1.2816), ("A", 0.99, -2.3263),
         ("B", 0.5, 0.0), ("B", 0.9, -1.2816), ("C", 0.5, 0.0), ("C", 0.9, -1.2816)]
# per-row Beta densities (B) and randomly chosen zero strips (C: 32 strips at
# this width) scatter more than the plain shift (A)
TOL = {"A": 0.01, "B": 0.02, "C": 0.03}


@pytest.mark.parametrize("variant, target, mu", CASES)
def test_sweep_inputs_have_their_labelled_sparsity(variant, target, mu):
    x = make_relu_bf16(1024, 2048, mu, 7, torch.device("cpu"), variant, target)
    assert x.dtype == torch.bfloat16 and x.shape == (1024, 2048)
    assert bool((x >= 0).all())
    sparsity = float((x == 0).float().mean())
    assert abs(sparsity - target) <= TOL[variant], (variant, target, sparsity)
