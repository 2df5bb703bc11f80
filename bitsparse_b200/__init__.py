"""bitsparse_b200 -- BitSparse activation compression on B200 (sm_100a).

A drop-in for the reference's ``lib_sparse`` package (Maxzhu123/bitsparse):
the same modules (config, fp8, bitsparse, layers, src.functions,
src.sparse_matmul) and, in ``src.operators``, the operator names of
``lib_sparse.src.triton_operators``, all backed by hand-written CUDA kernels
in ``libbitsparse_b200.so`` (C ABI: include/bitsparse.h).

``install_as_lib_sparse()`` registers this package under the name
``lib_sparse`` so that unmodified callers (``from lib_sparse.layers import
FFNRelu2``) import it.
"""
from __future__ import annotations

import sys

from . import config
from ._runtime import check_status
from .bitsparse import BitsparseTensor, TensorBuffer, bits_per_value, pack_codec, tile_grid

__all__ = ["BitsparseTensor", "TensorBuffer", "bits_per_value", "pack_codec", "tile_grid",
           "check_status", "install_as_lib_sparse", "config"]


def install_as_lib_sparse() -> None:
    """Make ``import lib_sparse...`` resolve to this package (drop-in use)."""
    import importlib

    pkg = sys.modules[__name__]
    sys.modules["lib_sparse"] = pkg
    for sub in ("config", "fp8", "bitsparse", "layers", "src", "src.functions",
                "src.sparse_matmul", "src.bitpacking", "src.operators"):
        mod = importlib.import_module(f"{__name__}.{sub}")
        sys.modules[f"lib_sparse.{sub}"] = mod
    sys.modules["lib_sparse.src.triton_operators"] = sys.modules[f"{__name__}.src.operators"]
