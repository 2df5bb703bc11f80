"""CPU: the C-ABI library loads and exports every entry point that
include/bitsparse.h declares; host-side argument checks return the
documented error codes (these paths touch no GPU)."""
import ctypes
import re
from pathlib import Path

import pytest

from bitsparse_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "bitsparse.h"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(bs_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared()
    assert "bs_compress" in names and "bs_unpack" in names
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) <= set(_lib.exported_symbols())


def test_version_and_workspace_size():
    lib = _lib.load()
    assert b"sm_100a" in lib.bs_version()
    assert lib.bs_compress_workspace_bytes(0) >= 16
    sizes = [lib.bs_compress_workspace_bytes(t) for t in (0, 1, 1000, 65536, 1 << 20)]
    assert sizes == sorted(sizes) and sizes[-1] < 3 * (1 << 20)  # ~2 bytes per tile


@pytest.mark.parametrize("call, code", [
    # unsupported dtype
    (lambda L: L.bs_compress(None, 9, 4, 4, 4, None, None, 1, 1, 1, 0, 0, None, None, None,
                             1, 1 << 20, None, None), _lib.BS_ERR_DTYPE),
    # negative shape
    (lambda L: L.bs_compress(16, 0, -1, 4, 4, None, None, 1, 1, 1, 0, 0, None, None, None,
                             16, 1 << 20, None, None), _lib.BS_ERR_SHAPE),
    # fp32 without a quantisation scale
    (lambda L: L.bs_compress(16, 3, 4, 4, 4, None, None, 1, 1, 1, 0, 0, None, None, None,
                             16, 1 << 20, None, None), _lib.BS_ERR_DTYPE),
    # workspace too small
    (lambda L: L.bs_compress(16, 0, 640, 640, 640, None, None, 16, 16, 16, 10, 0, None, None,
                             None, 16, 64, None, None), _lib.BS_ERR_WORKSPACE),
    # packed storage must be 4-byte aligned
    (lambda L: L.bs_compress(16, 0, 64, 64, 64, None, None, 16, 16, 17, 16, 1, None, None,
                             None, 16, 1 << 20, None, None), _lib.BS_ERR_ALIGN),
    # unpack: scale only with relu2
    (lambda L: L.bs_unpack(16, 16, 16, 16, 0, 0, 16, 64, 0, 1, 64, 64, 1, 0, 16, None),
     _lib.BS_ERR_ARG),
    # unpack: bad store dtype
    (lambda L: L.bs_unpack(16, 16, 16, 16, 3, 0, 16, 64, 0, 1, 64, 64, 1, 0, None, None),
     _lib.BS_ERR_DTYPE),
    # mask: row stride smaller than N
    (lambda L: L.bs_mask_with_bitmask(16, 0, 4, 8, 4, 16, None), _lib.BS_ERR_SHAPE),
    # relu2 grad: fp32 gradient unsupported
    (lambda L: L.bs_relu2_grad(16, 3, 4, 4, 4, 16, 16, 16, 16, 0, 0, None, None),
     _lib.BS_ERR_DTYPE),
    # fp8 scale: misaligned input
    (lambda L: L.bs_fp8_scale(17, 0, 100, 16, 16, None), _lib.BS_ERR_ALIGN),
    # huge M and N: the tile count must not wrap
    (lambda L: L.bs_compress(16, 0, 1 << 40, 1 << 40, 1 << 40, None, None, 16, 16, 16, 16, 0,
                             None, None, None, 16, 1 << 20, None, None), _lib.BS_ERR_SHAPE),
    (lambda L: L.bs_compress(16, 0, 1 << 62, 1 << 62, 1 << 62, None, None, 16, 16, 16, 16, 0,
                             None, None, None, 16, 1 << 20, None, None), _lib.BS_ERR_SHAPE),
    (lambda L: L.bs_compress_noalloc(16, 0, 1 << 40, 1 << 40, 1 << 40, None, None, 16, 16, 16,
                                     16, 0, None, None, None, None, None), _lib.BS_ERR_TOO_LARGE),
])
def test_host_argument_checks(call, code):
    assert call(_lib.load()) == code


def test_empty_batches_are_no_ops():
    L = _lib.load()
    assert L.bs_unpack(16, 16, 16, 16, 0, 0, 16, 64, 0, 1, 64, 0, 0, 0, None, None) == 0
    assert L.bs_mask_with_bitmask(16, 0, 0, 8, 8, 16, None) == 0
    assert L.bs_tile_pack(16, 0, 0, 8, 8, 16, 16, None) == 0
