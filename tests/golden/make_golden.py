"""Generate the golden fixtures by running the reference's own lib_sparse on CPU.

The reference (Maxzhu123/bitsparse, a Python + Triton package) runs on the CPU
under the Triton interpreter.  This script imports it from a checkout given by
``--reference`` (the path of the reference checkout, required), applies three harness shims that
leave the reference's code untouched, runs every operator of the compression
path on seeded inputs and writes the results as ``golden.npz`` beside this
file.  It only runs where the reference checkout exists; the fixtures it writes
are what the tests read everywhere else.

Shims (none changes the reference's arithmetic):

* ``TRITON_INTERPRET=1`` -- run the Triton kernels on the CPU;
* ``triton.autotune`` limited to its first config -- the autotuner's
  benchmarker needs a GPU driver (configs only change launch shape);
* ``TORCHDYNAMO_DISABLE=1`` -- ``to_fp8`` is ``@torch.compile``'d
  (lib_sparse/fp8.py:123-124) and Inductor cannot build it on this CPU box,
  so it runs eagerly;
* ``builtins.TensorBuffer`` -- lib_sparse/layers.py:24 annotates with a name
  imported only under TYPE_CHECKING (lib_sparse/layers.py:13-14), which
  Python 3.12 evaluates at definition time.

Cases written (key prefixes):

* ``v/<dtype>/<pack>/<shape>/<sparsity>/`` -- the validate.py-style round
  trip (experiments/validate.py:11-32) on standalone storage: input bytes,
  bitmask, prefix, vals (packed payload only), reconstruct, ReLU-mask of a
  gradient, ReLU^2 gradient, and (fp8 only; the bf16 one fails in the
  interpreter) the ReLU^2 reconstruct;
* ``a/<dtype>/<pack>/`` -- eight tensors compressed into one shared
  TensorBuffer (experiments/validate.py:128-139): whole arena bytes, each
  tensor's vals_offset and the final offset;
* ``c1/`` -- config 1: ``x = randn(1024, 3072)`` fp32, CPU
  generator seed 0, ``to_fp8(relu(x))`` then compress; SHA-256 digests of
  every output, the fp8 scale, and the bf16-cast variant;
* ``ffn/`` -- FFNRelu fwd+bwd at a small bf16 shape (outputs and grads).

Arrays above ``SMALL`` bytes are stored as SHA-256 digests (``<key>#sha``);
their inputs are regenerated from the stored seed by ``gen_input`` (torch's
CPU generator is deterministic for a given torch version; the digest of each
regenerated input is checked before use).
"""
from __future__ import annotations

import argparse
import builtins
import hashlib
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

SHAPES_FULL = ((128, 128), (129, 131))
SPARSITIES = (0.0, 0.5, 0.9, 1.0)
SHAPES_RAGGED = ((1, 1), (65, 1), (3, 200), (64, 64), (130, 257))
DTYPES = ("bfloat16", "float8_e4m3fn", "float8_e5m2")


def _setup(reference: str):
    os.environ["TRITON_INTERPRET"] = "1"
    os.environ["TORCHDYNAMO_DISABLE"] = "1"
    import triton

    orig = triton.autotune

    def first_config_only(configs, *args, **kwargs):
        kwargs.pop("restore_value", None)
        return orig(configs[:1], *args, **kwargs)

    triton.autotune = first_config_only
    sys.path.insert(0, reference)
    import lib_sparse.bitsparse as bsm

    builtins.TensorBuffer = bsm.TensorBuffer


def raw(t):
    """Raw bytes of a CPU tensor as a numpy uint8/uint16/uint32 array."""
    import torch

    t = t.contiguous()
    if t.dtype in (torch.bfloat16,):
        return t.view(torch.uint16).numpy().copy()
    if t.element_size() == 1:
        return t.view(torch.uint8).numpy().copy()
    if t.dtype == torch.uint32:
        return t.view(torch.int32).numpy().view(np.uint32).copy()
    return t.numpy().copy()


def sha(t) -> str:
    return hashlib.sha256(raw(t).tobytes()).hexdigest()


def gen_input(shape, sparsity, dtype, seed):
    import torch

    g = torch.Generator().manual_seed(seed)
    d = torch.randn(shape, generator=g, dtype=torch.bfloat16).abs_()
    zero = torch.rand(shape, generator=g) < sparsity
    d.masked_fill_(zero, 0)
    gd = torch.randn(shape, generator=g, dtype=torch.bfloat16)
    return d.to(getattr(torch, dtype)), gd


SMALL = 8192  # arrays above this many bytes are stored as SHA-256 digests


def put(out, key, arr, whole=False):
    """Store small arrays whole and large ones as a ``<key>#sha`` digest."""
    arr = np.ascontiguousarray(arr)
    if whole or arr.nbytes <= SMALL:
        out[key] = arr
    else:
        out[key + "#sha"] = np.array(hashlib.sha256(arr.tobytes()).hexdigest())
        out[key + "#n"] = np.array(arr.size)


def packed_payload(vals_u8, start_value, nnz, bits):
    """Zero every bit of a packed stream outside [start, start+nnz) values.

    The reference packs into ``torch.empty`` storage with read-modify-write
    edges (lib_sparse/src/bitpacking.py:112-117), so bits outside the payload
    are whatever the allocator held.
    """
    out = vals_u8.copy()
    lo, hi = start_value * bits, (start_value + nnz) * bits
    bit_idx = np.arange(out.size * 8)
    keep = (bit_idx >= lo) & (bit_idx < hi)
    bits_arr = np.unpackbits(out, bitorder="little")
    bits_arr &= keep.astype(np.uint8)
    return np.packbits(bits_arr, bitorder="little")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--out", default=str(HERE / "golden.npz"))
    args = ap.parse_args()
    _setup(args.reference)

    import torch
    from lib_sparse.bitsparse import TensorBuffer, bits_per_value
    from lib_sparse.fp8 import to_fp8
    from lib_sparse.layers import FFNRelu
    from lib_sparse.src.functions import dense_to_tilesparse
    from lib_sparse.src.triton_operators import (
        mask_with_bitmask_,
        relu2_grad_sparse_,
        unpack_batch_,
        unpack_relu2_batch_,
    )

    out: dict[str, np.ndarray] = {}

    def P(key, arr, whole=False):
        put(out, key, arr, whole)

    def reconstruct(s, relu2=False):
        M, N = s.shape
        dt = torch.bfloat16 if relu2 else s.dtype
        o = torch.zeros((M, N), dtype=dt)
        fn = unpack_relu2_batch_ if relu2 else unpack_batch_
        fn(s, o, 0, s.grid_n, N, M, s.grid_m * s.grid_n)
        return o

    seed = 1000
    cases = []
    for shape in SHAPES_FULL:
        for sp in SPARSITIES:
            cases.append((shape, sp))
    for shape in SHAPES_RAGGED:
        cases.append((shape, 0.5))

    for dtype in DTYPES:
        fp8 = dtype != "bfloat16"
        for pack in (False, True):
            for shape, sp in cases:
                seed += 1
                d, gd = gen_input(shape, sp, dtype, seed)
                key = f"v/{dtype}/{int(pack)}/{shape[0]}x{shape[1]}/{sp}/"
                s = dense_to_tilesparse(d, None, None, pack)
                nnz = int(s.prefix[-1])
                out[key + "seed"] = np.array(seed)
                P(key + "dense", raw(d))
                P(key + "grad", raw(gd))
                P(key + "bitmask", raw(s.bitmask))
                P(key + "prefix", raw(s.prefix))
                if pack:
                    P(key + "vals", packed_payload(
                        raw(s.vals), 0, nnz, bits_per_value(d.dtype)))
                else:
                    P(key + "vals", raw(s.vals))
                P(key + "recon", raw(reconstruct(s)))
                if fp8:
                    P(key + "recon_relu2", raw(reconstruct(s, relu2=True)))
                P(key + "mask_grad", raw(mask_with_bitmask_(gd.clone(), s)))
                P(key + "relu2_grad", raw(relu2_grad_sparse_(gd.clone(), s)))
                print(key, nnz, flush=True)

            # Shared arena: every full-shape tensor in one TensorBuffer.
            tensors = []
            for shape in SHAPES_FULL:
                for sp in SPARSITIES:
                    seed += 1
                    tensors.append(gen_input(shape, sp, dtype, seed)[0])
            cap = sum(t.numel() for t in tensors)
            if pack:
                cap += 7 * len(tensors)
                size = (cap * bits_per_value(tensors[0].dtype) + 7) // 8
            else:
                size = cap * tensors[0].element_size()
            buf = TensorBuffer(size, device="cpu", dtype=tensors[0].dtype,
                               pack_sbit=pack)
            key = f"a/{dtype}/{int(pack)}/"
            offs = []
            out[key + "seed0"] = np.array(seed - len(tensors) + 1)
            for i, t in enumerate(tensors):
                P(key + f"dense{i}", raw(t))
                s = dense_to_tilesparse(t, None, buf, pack)
                offs.append(int(s.vals_offset))
            out[key + "size"] = np.array(size)
            P(key + "arena", raw(buf.vals))
            out[key + "vals_offsets"] = np.array(offs, dtype=np.int64)
            out[key + "final_offset"] = np.array(int(buf.offset[0]))
            print(key, offs, int(buf.offset[0]), flush=True)

    # Config 1: fp32 N(0,1) 1024x3072, seed 0, to_fp8(relu(x)).
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1024, 3072, generator=g, dtype=torch.float32)
    h = torch.relu(x)
    q, scale = to_fp8(h)
    out["c1/x_sha"] = np.array(sha(x))
    out["c1/scale"] = np.array(float(scale), dtype=np.float32)
    out["c1/q_sha"] = np.array(sha(q))
    for name, dense in (("fp8", q), ("bf16", h.to(torch.bfloat16))):
        for pack in (False, True):
            s = dense_to_tilesparse(dense, scale if name == "fp8" else None,
                                    None, pack)
            nnz = int(s.prefix[-1])
            k = f"c1/{name}/{int(pack)}/"
            out[k + "nnz"] = np.array(nnz)
            out[k + "bitmask_sha"] = np.array(sha(s.bitmask))
            out[k + "prefix_sha"] = np.array(sha(s.prefix))
            v = raw(s.vals)
            if pack:
                v = packed_payload(v, 0, nnz, bits_per_value(dense.dtype))
            out[k + "vals_sha"] = np.array(hashlib.sha256(v.tobytes()).hexdigest())
            out[k + "recon_sha"] = np.array(sha(reconstruct(s)))
            print(k, nnz, flush=True)

    # FFNRelu forward + backward, bf16, small.
    g = torch.Generator().manual_seed(7)
    T, d, H, do = 128, 64, 256, 48
    x = torch.randn(T, d, generator=g).to(torch.bfloat16).requires_grad_()
    W1 = (0.05 * torch.randn(H, d, generator=g)).to(torch.bfloat16).requires_grad_()
    W2 = (0.05 * torch.randn(do, H, generator=g)).to(torch.bfloat16).requires_grad_()
    b1 = (0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).requires_grad_()
    b2 = (0.1 * torch.randn(do, generator=g)).to(torch.bfloat16).requires_grad_()
    gy = torch.randn(T, do, generator=g).to(torch.bfloat16)
    y = FFNRelu.apply(x, W1, W2, b1, b2)
    y.backward(gy)
    for n, t in (("x", x), ("W1", W1), ("W2", W2), ("b1", b1), ("b2", b2),
                 ("gy", gy)):
        P(f"ffn/{n}", raw(t.detach()), whole=True)
    P("ffn/y", raw(y.detach()), whole=True)
    for n, t in (("x", x), ("W1", W1), ("W2", W2), ("b1", b1), ("b2", b2)):
        P(f"ffn/d{n}", raw(t.grad), whole=True)

    np.savez_compressed(args.out, **out)
    print("wrote", args.out, len(out), "arrays")


if __name__ == "__main__":
    main()
