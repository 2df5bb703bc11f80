"""ctypes binding of libbitsparse_b200.so (the C ABI in include/bitsparse.h).

There is no fallback: if the library is missing or cannot be loaded, every
operator raises.  Device memory comes from PyTorch tensors; the library
allocates nothing.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libbitsparse_b200.so"

BS_OK, BS_ERR_SHAPE, BS_ERR_DTYPE, BS_ERR_ALIGN, BS_ERR_CAPACITY = 0, 1, 2, 3, 4
BS_ERR_LAUNCH, BS_ERR_ARG, BS_ERR_WORKSPACE, BS_ERR_TOO_LARGE = 5, 6, 7, 8
BS_STATUS_CAPACITY, BS_STATUS_TIMEOUT = 1, 2
BS_BF16, BS_E4M3, BS_E5M2, BS_F32 = 0, 1, 2, 3
BS_FP8_COMPILED = 0x100

_ERRORS = {
    BS_ERR_SHAPE: "bad shape",
    BS_ERR_DTYPE: "unsupported dtype",
    BS_ERR_ALIGN: "misaligned pointer",
    BS_ERR_CAPACITY: "capacity",
    BS_ERR_LAUNCH: "CUDA launch failed",
    BS_ERR_ARG: "bad argument",
    BS_ERR_WORKSPACE: "workspace too small",
    BS_ERR_TOO_LARGE: "tensor exceeds the fixed maximum of the no-allocation entry point",
}

_vp, _i64, _i32, _sz = C.c_void_p, C.c_int64, C.c_int, C.c_size_t

# name -> (restype, argtypes)
_SIGS = {
    "bs_version": (C.c_char_p, []),
    "bs_compress_workspace_bytes": (_sz, [_i64]),
    "bs_compress": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _i32,
                           _vp, _vp, _vp, _vp, _sz, _vp, _vp]),
    "bs_compress_noalloc": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _i64,
                                   _i32, _vp, _vp, _vp, _vp, _vp]),
    "bs_compress_noalloc_max_tiles": (_sz, []),
    "bs_compress_bias_relu_fp8": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp,
                                         _vp, _i64, _i32, _vp, _vp, _vp, _vp, _sz, _i32, _vp,
                                         _vp]),
    "bs_fp8_scales_bias_relu": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i32, _vp]),
    "bs_compress_bias_relu": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _i64,
                                     _i32, _vp, _vp, _vp, _vp, _sz, _vp, _vp]),
    "bs_transpose_b8": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _vp]),
    "bs_gemm_bf16_mask": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _vp,
                                 _vp]),
    "bs_gemm_fp8": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp,
                           _vp]),
    "bs_gemm_fp8_relu2": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _vp,
                                 _vp, _vp, _vp, _vp, C.c_float, _vp, _vp, _vp]),
    "bs_compress_fp8_tile_scaled": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _i32,
                                           _vp, _vp, _vp, _vp, _sz, _vp, _vp]),
    "bs_unpack_tile_scaled": (_i32, [_vp, _vp, _vp, _vp, _i32, _vp, _vp, _i64, _i64, _i64, _i64,
                                     _i64, _i64, _vp]),
    "bs_gemm_unpack_dw": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _i32, C.c_float,
                                  _vp, _i64, _vp, _sz, _vp, _vp]),
    "bs_gemm_unpack_dw_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "bs_gemm_bf16_relu2": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _vp,
                                  _vp, _vp, C.c_float, _vp, _vp]),
    "bs_tile_pack": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _vp, _vp]),
    "bs_compact_vals": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _vp, _i64, _i32, _vp, _vp,
                               _vp]),
    "bs_unpack": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _vp, _i64, _i64, _i64, _i64, _i64,
                         _i64, _i32, _vp, _vp]),
    "bs_mask_with_bitmask": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _vp]),
    "bs_unpack_status": (_i32, [_vp, _i32]),
    "bs_quantize_e4m3_2d": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _i32,
                                   _vp]),
    "bs_unpack_relu2_fp8t": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _i64, _vp, C.c_float, _vp,
                                    _vp, _vp, _i64, _i32, _vp]),
    "bs_relu2_grad": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i32, _i32, _vp,
                             _vp]),
    "bs_fp8_scale": (_i32, [_vp, _i32, _i64, _vp, _vp, _vp]),
    "bs_fp8_estimate_exact": (_i32, [_vp, _i32, _vp, _vp]),
    "bs_quantize_e4m3": (_i32, [_vp, _i32, _i64, _vp, _vp, _vp]),
}

_lib = None


def lib_path() -> Path:
    return _LIB_PATH


def load() -> C.CDLL:
    """Load the shared library (once) and declare every entry point."""
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            raise RuntimeError(
                f"{_LIB_PATH.name} is not built; run `python -m bitsparse_b200.build` "
                "(there is no CPU or Triton fallback)")
        lib = C.CDLL(str(_LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(rc: int, what: str) -> None:
    if rc != BS_OK:
        raise RuntimeError(f"{what}: {_ERRORS.get(rc, 'error')} (code {rc})")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
