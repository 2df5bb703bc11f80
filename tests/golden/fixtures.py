"""Read tests/golden/golden.npz: whole arrays or SHA-256 digests.

Large arrays are stored as digests (``<field>#sha``); their inputs are
regenerated from the stored seed with ``make_golden.gen_input`` and checked
against the stored digest before use.
"""
import hashlib

import numpy as np

from tests.golden.make_golden import gen_input


def digest(arr) -> str:
    return hashlib.sha256(np.ascontiguousarray(arr).tobytes()).hexdigest()


def has(f: dict, field: str) -> bool:
    return field in f or (field + "#sha") in f


def check(f: dict, field: str, got, msg=""):
    """Assert ``got`` equals the stored array (or its digest) bit for bit."""
    got = np.ascontiguousarray(got)
    if field in f:
        want = f[field]
        assert got.size == want.size, f"{msg} {field}: size {got.size} != {want.size}"
        np.testing.assert_array_equal(got.reshape(-1), want.reshape(-1),
                                      err_msg=f"{msg} {field}")
    else:
        assert got.size == int(f[field + "#n"]), f"{msg} {field}: size differs"
        assert digest(got) == str(f[field + "#sha"]), f"{msg} {field}: digest differs"


def _torch_raw(t):
    import torch
    if t.dtype == torch.bfloat16:
        return t.view(torch.uint16).numpy().copy()
    return t.view(torch.uint8).numpy().copy()


def case_inputs(f: dict, dtype: str, shape, sparsity: float):
    """(dense bits, grad bf16 bits) of a 'v/' case."""
    if "dense" in f and "grad" in f:
        return f["dense"].reshape(shape), f["grad"].reshape(shape)
    d, g = gen_input(shape, sparsity, dtype, int(f["seed"]))
    d, g = _torch_raw(d), _torch_raw(g)
    check(f, "dense", d, "regenerated input")
    check(f, "grad", g, "regenerated input")
    return d.reshape(shape), g.reshape(shape)


def arena_inputs(golden: dict, key: str, dtype: str, shapes, sparsities):
    """The eight dense inputs of an 'a/' case, in compression order."""
    out = []
    i = 0
    for shape in shapes:
        for sp in sparsities:
            if key + f"dense{i}" in golden:
                d = golden[key + f"dense{i}"].reshape(shape)
            else:
                t, _ = gen_input(shape, sp, dtype, int(golden[key + "seed0"]) + i)
                d = _torch_raw(t).reshape(shape)
                sub = {k[len(key):]: v for k, v in golden.items() if k.startswith(key)}
                check(sub, f"dense{i}", d, "regenerated arena input")
            out.append(d)
            i += 1
    return out
