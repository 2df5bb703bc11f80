"""CPU oracle for the BitSparse compression path -- TEST INFRASTRUCTURE ONLY.

This module is the checker that the CUDA path is compared against.  Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import it; the product (``bitsparse_b200``) never does, and
has no CPU fallback.

It restates, in NumPy integer arithmetic on raw bit patterns, what the
reference's lib_sparse computes (Maxzhu123/bitsparse; citations are
``path:line`` in that project).  Parity is PINNED: ``tests/test_oracle.py``
checks every function here against ``tests/golden/golden.npz``, which
``tests/golden/make_golden.py`` produced by running the reference itself on
the CPU (Triton interpreter).

Values are handled as raw bits: bf16 as ``uint16``, fp8 as ``uint8``.

In-kernel fp32 -> bf16 casts (the ReLU^2 reconstruct and gradient) take a
``rounding`` argument: ``"rne"`` (default) is what the reference's Triton
kernels do on a GPU and what the CUDA path must match; ``"trunc"`` is what
the Triton CPU interpreter that produced the fixtures does, and is used only
to pin these functions against those fixtures.
"""
from __future__ import annotations

import numpy as np

# lib_sparse/config.py:2-9
RELU2_SCALE = 1
BLOCK_M = 64
BLOCK_N = 64
_PACK_CHUNK_TILES = 2 ** 16

DT_BF16, DT_E4M3, DT_E5M2 = "bfloat16", "float8_e4m3fn", "float8_e5m2"
# Largest bit pattern that compares > 0 as a float (sign clear, not NaN):
# bf16 +inf 0x7F80, e4m3fn max-finite 0x7E (0x7F is NaN), e5m2 +inf 0x7C.
_POS_LIMIT = {DT_BF16: 0x7F80, DT_E4M3: 0x7E, DT_E5M2: 0x7C}
_ELT = {DT_BF16: 2, DT_E4M3: 1, DT_E5M2: 1}


def is_fp8(dtype: str) -> bool:
    """lib_sparse/fp8.py:20-22."""
    return dtype in (DT_E4M3, DT_E5M2)


def pack_codec(dtype: str) -> int:
    """lib_sparse/bitsparse.py:8-18: 0 = bf16, 1 = e4m3fn, 2 = e5m2."""
    return {DT_E4M3: 1, DT_E5M2: 2}.get(dtype, 0)


def bits_per_value(dtype: str) -> int:
    """lib_sparse/bitsparse.py:21-23: 15 for bf16, 7 for fp8."""
    return 7 if pack_codec(dtype) else 15


def packed_nbytes(numel: int, bits: int) -> int:
    """lib_sparse/src/bitpacking.py:27-29."""
    return (int(numel) * bits + 7) // 8


def packed_storage_nbytes(numel: int, bits: int) -> int:
    """lib_sparse/src/bitpacking.py:32-34: word-rounded plus one guard word."""
    return (packed_nbytes(numel, bits) + 3) // 4 * 4 + 4


def tile_grid(M: int, N: int, bm: int = BLOCK_M, bn: int = BLOCK_N):
    """lib_sparse/bitsparse.py:120-127."""
    tile_numel = bm * bn
    grid_m = (M + bm - 1) // bm
    grid_n = (N + bn - 1) // bn
    return grid_m, grid_n, grid_m * grid_n, tile_numel, tile_numel // 8


# --------------------------------------------------------------------------
# Scalar formats (bit-exact conversions)
# --------------------------------------------------------------------------
def f32_to_bf16_trunc(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 by truncation: what the Triton CPU interpreter does for
    an in-kernel fp32 -> bf16 cast (triton/runtime/interpreter.py
    ``_convert_float`` with no rounding mode).  On a GPU Triton rounds to
    nearest even; the golden fixtures hold the interpreter's values."""
    x = np.asarray(x, dtype=np.float32)
    return (x.view(np.uint32) >> 16).astype(np.uint16)


def _kernel_cast(rounding: str):
    return f32_to_bf16 if rounding == "rne" else f32_to_bf16_trunc


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (NaN -> quiet NaN)."""
    x = np.asarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r = np.where(nan, (((b >> 16) & 0x8000) | 0x7FC0).astype(np.uint16), r)
    return r


def _fp8_table(dtype: str) -> np.ndarray:
    """Value of every code 0..255 as float64 (NaN for NaN codes)."""
    codes = np.arange(256)
    if dtype == DT_E4M3:
        eb, mb, bias = 4, 3, 7
    else:
        eb, mb, bias = 5, 2, 15
    e = (codes >> mb) & ((1 << eb) - 1)
    m = codes & ((1 << mb) - 1)
    sign = np.where(codes & 0x80, -1.0, 1.0)
    val = np.where(e == 0, m / (1 << mb) * 2.0 ** (1 - bias),
                   (1 + m / (1 << mb)) * 2.0 ** (e.astype(np.float64) - bias))
    val = sign * val
    if dtype == DT_E4M3:
        val[(codes & 0x7F) == 0x7F] = np.nan
    else:
        top = (codes & 0x7F)
        val[top == 0x7C] = sign[top == 0x7C] * np.inf
        val[top > 0x7C] = np.nan
    return val


_FP8_TABLES = {}


def fp8_to_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    if dtype not in _FP8_TABLES:
        _FP8_TABLES[dtype] = _fp8_table(dtype)
    return _FP8_TABLES[dtype][bits.astype(np.int64)].astype(np.float32)


def f32_to_fp8(x: np.ndarray, dtype: str) -> np.ndarray:
    """fp32 -> fp8 bits, round to nearest even, following torch's casts.

    e4m3fn: magnitudes above 464 (the midpoint above 448; 464 itself ties to
    even, 448) become NaN (0x7F);
    e5m2: IEEE overflow to inf (0x7C) at >= 61440; NaN -> 0x7F.
    """
    with np.errstate(invalid="ignore"):
        x = np.asarray(x, dtype=np.float32).astype(np.float64)
    if dtype not in _FP8_TABLES:
        _FP8_TABLES[dtype] = _fp8_table(dtype)
    tab = _FP8_TABLES[dtype]
    top = 0x7E if dtype == DT_E4M3 else 0x7B  # largest finite positive code
    pos = tab[: top + 1]
    a = np.abs(x)
    a_fin = np.where(np.isfinite(a), a, 0.0)
    hi = np.clip(np.searchsorted(pos, a_fin, side="left"), 0, top)
    lo = np.clip(hi - 1, 0, top)
    dlo = a_fin - pos[lo]
    dhi = pos[hi] - a_fin
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo)
    code = np.where(a_fin <= pos[0], 0, code)
    if dtype == DT_E4M3:
        code = np.where(a > 464.0, 0x7F, code)
        code = np.where(np.isnan(a), 0x7F, code)
    else:
        code = np.where(a >= 61440.0, 0x7C, code)
        code = np.where(np.isnan(a), 0x7F, code)
    sign = (np.signbit(x)).astype(np.int64) << 7
    return (code | sign).astype(np.uint8)


def to_float(bits: np.ndarray, dtype: str) -> np.ndarray:
    return bf16_to_f32(bits) if dtype == DT_BF16 else fp8_to_f32(bits, dtype)


# --------------------------------------------------------------------------
# to_fp8 (lib_sparse/fp8.py:123-129), eager semantics
# --------------------------------------------------------------------------
FP8_MAX = 448.0


def to_fp8(x: np.ndarray, in_dtype: str):
    """Per-tensor e4m3fn quantiser of lib_sparse/fp8.py:123-129.

    ``in_dtype`` is ``"float32"`` (x is float32) or ``"bfloat16"`` (x is
    bf16 bits).  Eager PyTorch semantics: for bf16 input ``amax / 448`` is
    rounded to bf16 before ``.to(float32)`` and ``x / scale`` is rounded to
    bf16 before the fp8 cast; for fp32 both stay fp32.  (The reference's
    ``@torch.compile``d to_fp8 on a GPU divides with an approximate
    hardware division, which a CPU cannot restate bit for bit; the tests
    check that semantics against the compiled function itself.)  Returns
    ``(q_bits uint8, scale float32)``.
    """
    if in_dtype == "bfloat16":
        xf = bf16_to_f32(x)
        amax = np.float32(np.max(np.abs(xf))) if xf.size else np.float32(0)
        scale = bf16_to_f32(f32_to_bf16(np.float32(amax) / np.float32(FP8_MAX)))
        scale = np.maximum(np.float32(scale), np.float32(1e-9))
        q = f32_to_fp8(bf16_to_f32(f32_to_bf16(xf / scale)), DT_E4M3)
    else:
        xf = np.asarray(x, dtype=np.float32)
        amax = np.float32(np.max(np.abs(xf))) if xf.size else np.float32(0)
        scale = np.maximum(np.float32(amax) / np.float32(FP8_MAX), np.float32(1e-9))
        q = f32_to_fp8(xf / np.float32(scale), DT_E4M3)
    return q, np.float32(scale)


# --------------------------------------------------------------------------
# Tiles
# --------------------------------------------------------------------------
def _tiles(dense: np.ndarray, M: int, N: int):
    """Dense [M,N] -> [T, 4096] in tile-grid-row-major, row-major-in-tile order.

    Out-of-range elements read as 0 (lib_sparse/src/triton_kernels.py:83).
    """
    gm, gn, T, _, _ = tile_grid(M, N)
    pad = np.zeros((gm * BLOCK_M, gn * BLOCK_N), dtype=dense.dtype)
    pad[:M, :N] = dense.reshape(M, N)
    return pad.reshape(gm, BLOCK_M, gn, BLOCK_N).transpose(0, 2, 1, 3).reshape(T, BLOCK_M * BLOCK_N)


def positive(bits: np.ndarray, dtype: str) -> np.ndarray:
    """``x > 0.0`` on raw bits (lib_sparse/src/triton_kernels.py:86)."""
    return (bits > 0) & (bits <= _POS_LIMIT[dtype])


def tile_pack(dense: np.ndarray, M: int, N: int, dtype: str):
    """lib_sparse/src/triton_kernels.py:63-97: per-tile bitmask + popcount.

    Bit ``j`` of byte ``b`` of tile ``t`` is element ``8b+j`` of the tile in
    row-major order (LSB first).  Returns ``(bitmask uint8[T*512], counts
    int32[T])``.
    """
    tiles = _tiles(dense, M, N)
    mask = positive(tiles, dtype)
    bitmask = np.packbits(mask, axis=1, bitorder="little").reshape(-1)
    counts = mask.sum(axis=1).astype(np.int32)
    return bitmask, counts


def tile_prefix(counts: np.ndarray) -> np.ndarray:
    """lib_sparse/src/functions.py:38-40: prefix[0]=0, inclusive cumsum after.

    The reference scans in int32 and views as uint32, so it wraps mod 2**32.
    """
    p = np.zeros(counts.size + 1, dtype=np.uint64)
    p[1:] = np.cumsum(counts.astype(np.uint64))
    return (p & 0xFFFFFFFF).astype(np.uint32)


def compact_values(dense: np.ndarray, M: int, N: int, dtype: str) -> np.ndarray:
    """lib_sparse/src/triton_kernels.py:105-146: positives in (tile,row,col) order."""
    tiles = _tiles(dense, M, N)
    return tiles[positive(tiles, dtype)]


# --------------------------------------------------------------------------
# 15/7-bit sign-dropped codec (lib_sparse/src/bitpacking.py)
# --------------------------------------------------------------------------
def pack_into(stream: np.ndarray, values: np.ndarray, start_value: int, bits: int):
    """Write ``values`` at logical index ``start_value`` of a packed stream.

    lib_sparse/src/bitpacking.py:58-117: value ``i`` occupies bits
    ``[(start+i)*bits, (start+i+1)*bits)`` of the byte stream, LSB first;
    bits outside that range are left as they were.
    """
    n = values.size
    if n == 0:
        return stream
    v = values.astype(np.uint16)
    vb = np.unpackbits(v.view(np.uint8).reshape(n, 2), axis=1, bitorder="little")
    vb = vb[:, :bits].reshape(-1)
    sbits = np.unpackbits(stream, bitorder="little")
    lo = start_value * bits
    sbits[lo: lo + vb.size] = vb
    stream[:] = np.packbits(sbits, bitorder="little")
    return stream


def unpack_values(stream: np.ndarray, indices: np.ndarray, bits: int) -> np.ndarray:
    """lib_sparse/src/bitpacking.py:37-55: decode logical indices from the
    stream addressed as little-endian uint16 words."""
    idx = indices.astype(np.int64)
    words = np.zeros((stream.size + 5) // 2, dtype=np.uint16)
    words.view(np.uint8)[: stream.size] = stream
    w = (idx * bits) // 16
    sh = (idx * bits) % 16
    w0 = words[w].astype(np.uint32)
    w1 = words[w + 1].astype(np.uint32)
    return (((w0 | (w1 << 16)) >> sh) & ((1 << bits) - 1)).astype(np.uint16)


# --------------------------------------------------------------------------
# Whole-path operations (lib_sparse/src/functions.py, triton_operators.py)
# --------------------------------------------------------------------------
class Sparse:
    """Oracle copy of BitsparseTensor (lib_sparse/bitsparse.py:26-87)."""

    def __init__(self, vals, bitmask, prefix, shape, dtype, vals_offset,
                 pack_sbit, scale=None):
        self.vals, self.bitmask, self.prefix = vals, bitmask, prefix
        self.shape, self.dtype = shape, dtype
        self.vals_offset, self.pack_sbit, self.scale = vals_offset, pack_sbit, scale
        self.grid_m, self.grid_n, self.num_tiles, _, _ = tile_grid(*shape)

    @property
    def nnz(self):
        return int(self.prefix[-1])


class Arena:
    """Oracle copy of TensorBuffer (lib_sparse/bitsparse.py:90-117)."""

    def __init__(self, size: int, dtype: str, pack_sbit: bool):
        self.size, self.dtype, self.pack_sbit = size, dtype, pack_sbit
        if pack_sbit:
            self.vals = np.zeros((size + 3) // 4 * 4 + 4, dtype=np.uint8)
        else:
            elt = _ELT[dtype]
            if size % elt:
                raise ValueError("raw TensorBuffer size must be a multiple of dtype size")
            self.vals = np.zeros(size // elt, dtype=np.uint16 if elt == 2 else np.uint8)
        self.offset = 0


def dense_to_tilesparse(dense: np.ndarray, dtype: str, arena: Arena | None = None,
                        pack_sbit: bool = False, scale=None) -> Sparse:
    """lib_sparse/src/functions.py:55-99 with compact_vals
    (lib_sparse/src/triton_operators.py:36-115)."""
    M, N = dense.shape
    bitmask, counts = tile_pack(dense, M, N, dtype)
    prefix = tile_prefix(counts)
    vals_raw = compact_values(dense, M, N, dtype)
    nnz = vals_raw.size
    bits = bits_per_value(dtype)
    if arena is None:
        off = 0
        if pack_sbit:
            vals = np.zeros(packed_storage_nbytes(nnz, bits), dtype=np.uint8)
            pack_into(vals, vals_raw, 0, bits)
        else:
            vals = vals_raw.copy()
    else:
        vals = arena.vals
        if pack_sbit:
            off = (arena.offset + 7) // 8 * 8  # functions.py:78-81
            pack_into(vals, vals_raw, off, bits)
        else:
            off = arena.offset
            vals[off: off + nnz] = vals_raw
        arena.offset = off + int(prefix[-1])  # functions.py:91-92
    return Sparse(vals, bitmask, prefix, (M, N), dtype, off, pack_sbit, scale)


def _gather_tiles(sp: Sparse, first_m_tile: int, num_tiles_in_batch: int):
    """Per tile of the batch: the bit mask [n,4096] and its values (raw bits)."""
    gn = sp.grid_n
    pid = np.arange(num_tiles_in_batch)
    tile_id = (first_m_tile + pid // gn) * gn + pid % gn
    bm = sp.bitmask.reshape(-1, 512)[tile_id]
    mask = np.unpackbits(bm, axis=1, bitorder="little").astype(bool)
    rank = np.cumsum(mask, axis=1) - 1
    idx = sp.prefix[tile_id].astype(np.int64)[:, None] + sp.vals_offset + rank
    if sp.pack_sbit:
        raw = unpack_values(sp.vals, np.where(mask, idx, 0), bits_per_value(sp.dtype))
        raw = raw if sp.dtype == DT_BF16 else raw.astype(np.uint8)
    else:
        src = sp.vals if sp.vals.size else np.zeros(1, dtype=sp.vals.dtype)
        raw = src[np.where(mask, idx, 0)]
    raw = np.where(mask, raw, 0).astype(raw.dtype)
    return pid, mask, raw


def _store_tiles(out: np.ndarray, pid, tiles, grid_n, batch_rows, K):
    """lib_sparse/src/triton_kernels.py:193-209."""
    n = pid.size
    t = tiles.reshape(n, BLOCK_M, BLOCK_N)
    for i in range(n):
        r0 = (pid[i] // grid_n) * BLOCK_M
        c0 = (pid[i] % grid_n) * BLOCK_N
        rr = min(BLOCK_M, batch_rows - r0)
        cc = min(BLOCK_N, K - c0)
        if rr > 0 and cc > 0:
            out[r0: r0 + rr, c0: c0 + cc] = t[i, :rr, :cc]
    return out


def unpack_batch(sp: Sparse, out: np.ndarray, first_m_tile: int, grid_n: int,
                 K: int, batch_rows: int, num_tiles_in_batch: int) -> np.ndarray:
    """lib_sparse/src/triton_operators.py:118-138 (square_vals=False)."""
    pid, mask, raw = _gather_tiles(sp, first_m_tile, num_tiles_in_batch)
    return _store_tiles(out, pid, raw, grid_n, batch_rows, K)


def _mul_bf16_by_scalar(bits: np.ndarray, s: np.float32) -> np.ndarray:
    """``bf16_tensor.mul_(fp32 0-dim)``: the scalar is cast to bf16 first
    (tensor-iterator common dtype), the product is taken in fp32."""
    sb = bf16_to_f32(f32_to_bf16(np.float32(s)))
    return f32_to_bf16(bf16_to_f32(bits) * sb)


def unpack_relu2_batch(sp: Sparse, out: np.ndarray, first_m_tile: int, grid_n: int,
                       K: int, batch_rows: int, num_tiles_in_batch: int,
                       rounding: str = "rne") -> np.ndarray:
    """lib_sparse/src/triton_operators.py:141-162 and triton_kernels.py:231-238.

    ``out`` is bf16 bits.  fp8 storage squares in fp32; bf16 storage squares
    bf16 x bf16 (exact in fp32, one rounding).  Then ``out *= scale**2``.
    """
    pid, mask, raw = _gather_tiles(sp, first_m_tile, num_tiles_in_batch)
    v = to_float(raw, sp.dtype)
    sq = _kernel_cast(rounding)(np.float32(RELU2_SCALE) * v * v)
    _store_tiles(out, pid, sq, grid_n, batch_rows, K)
    if sp.scale is not None:
        s2 = np.float32(sp.scale) * np.float32(sp.scale)
        out[:] = _mul_bf16_by_scalar(out, s2)
    return out


def _dense_mask(sp: Sparse) -> np.ndarray:
    M, N = sp.shape
    mask = np.unpackbits(sp.bitmask.reshape(-1, 512), axis=1, bitorder="little")
    gm, gn = sp.grid_m, sp.grid_n
    full = mask.reshape(gm, gn, BLOCK_M, BLOCK_N).transpose(0, 2, 1, 3)
    return full.reshape(gm * BLOCK_M, gn * BLOCK_N)[:M, :N].astype(bool)


def mask_with_bitmask(grad: np.ndarray, sp: Sparse) -> np.ndarray:
    """lib_sparse/src/triton_kernels.py:249-276: grad <- bit ? grad : +0."""
    grad[:] = np.where(_dense_mask(sp), grad, 0).astype(grad.dtype)
    return grad


def relu2_grad_sparse(grad: np.ndarray, sp: Sparse, rounding: str = "rne") -> np.ndarray:
    """lib_sparse/src/triton_kernels.py:288-330 plus the ``grad *= scale`` of
    lib_sparse/src/triton_operators.py:200-201.  grad is bf16 bits."""
    M, N = sp.shape
    pid, mask, raw = _gather_tiles(sp, 0, sp.num_tiles)
    r = np.zeros((sp.grid_m * BLOCK_M, sp.grid_n * BLOCK_N), dtype=np.float32)
    rv = to_float(raw, sp.dtype).reshape(sp.grid_m, sp.grid_n, BLOCK_M, BLOCK_N)
    r[:] = rv.transpose(0, 2, 1, 3).reshape(r.shape)
    factor = np.float32(2.0 * RELU2_SCALE) * r[:M, :N]
    g = _kernel_cast(rounding)(bf16_to_f32(grad) * factor)
    grad[:] = np.where(_dense_mask(sp), g, 0).astype(np.uint16)
    if sp.scale is not None:
        grad[:] = _mul_bf16_by_scalar(grad, sp.scale)
    return grad


def reconstruct(sp: Sparse) -> np.ndarray:
    """Whole-tensor reconstruct (experiments/validate.py:35-51)."""
    M, N = sp.shape
    out = np.zeros((M, N), dtype=np.uint16 if sp.dtype == DT_BF16 else np.uint8)
    return unpack_batch(sp, out, 0, sp.grid_n, N, M, sp.num_tiles)


def reconstruct_relu2(sp: Sparse, rounding: str = "rne") -> np.ndarray:
    M, N = sp.shape
    out = np.zeros((M, N), dtype=np.uint16)
    return unpack_relu2_batch(sp, out, 0, sp.grid_n, N, M, sp.num_tiles, rounding)


# ---------------------------------------------------------------------------
# Per-tile FP8 scale mode.  An EXTENSION with no reference counterpart (the
# reference's to_fp8 is per tensor, lib_sparse/fp8.py:123-129), so this
# restatement is the specification the CUDA path is checked against -- its
# parity is unpinned by any reference output.  Every step is IEEE fp32 with
# round-to-nearest-even, which NumPy reproduces exactly.
# ---------------------------------------------------------------------------
def to_fp8_tile_scaled(bits: np.ndarray):
    """bf16 [M, N] bits -> (e4m3 codes [M, N], tile scales float32[T]).

    Tile t (grid-row-major): amax_t = max |x| (NaN ignored); scale_t =
    amax_t / 448, inv_t = 448 / amax_t (fp32 divisions; an all-zero tile has
    scale 1 and inv 0); code = e4m3(fp32(x * inv_t)), round to nearest even."""
    M, N = bits.shape
    gm, gn, T, _, _ = tile_grid(M, N)
    x = np.zeros((gm * BLOCK_M, gn * BLOCK_N), dtype=np.float32)
    x[:M, :N] = bf16_to_f32(bits)
    t = x.reshape(gm, BLOCK_M, gn, BLOCK_N).transpose(0, 2, 1, 3)
    a = np.abs(t)
    a = np.where(np.isnan(a), np.float32(0), a)
    am = a.reshape(gm, gn, -1).max(axis=2).astype(np.float32)
    pos = am > 0
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        scale = np.where(pos, am / np.float32(448), np.float32(1)).astype(np.float32)
        inv = np.where(pos, np.float32(448) / am, np.float32(0)).astype(np.float32)
        q = (t * inv[:, :, None, None]).astype(np.float32)
    codes = f32_to_fp8(q, DT_E4M3).transpose(0, 2, 1, 3).reshape(gm * BLOCK_M, gn * BLOCK_N)
    return np.ascontiguousarray(codes[:M, :N]), scale.reshape(-1)


def reconstruct_tile_scaled(sp: "Sparse", scales: np.ndarray) -> np.ndarray:
    """bf16 bits [M, N] of a per-tile-scaled e4m3 tensor: bf16(value(code) *
    scale_t) where a value is stored, 0 elsewhere."""
    M, N = sp.shape
    codes = reconstruct(sp)
    gm, gn = sp.grid_m, sp.grid_n
    s = np.repeat(np.repeat(scales.reshape(gm, gn), BLOCK_M, 0), BLOCK_N, 1)[:M, :N]
    with np.errstate(invalid="ignore", over="ignore"):
        v = (fp8_to_f32(codes, DT_E4M3) * s).astype(np.float32)
    return np.where(codes != 0, f32_to_bf16(v), np.uint16(0)).astype(np.uint16)
