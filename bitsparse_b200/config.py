"""Tile and codec settings (same names and values as lib_sparse/config.py:1-12)."""

# Constant for RELU^2 scaling: z = RELU2_SCALE * relu(a)^2.
RELU2_SCALE = 1

# Tile shape.  The CUDA kernels are built for 64x64 tiles (one 512-byte
# bitmask per tile); other values are rejected by the operators.
BLOCK_M = 64
BLOCK_N = 64

# Tiles per staging chunk of the reference's packed path.  The fused kernel
# packs in one pass, so this only remains for API compatibility.
_PACK_CHUNK_TILES = 2 ** 16

# Keep FP8 copies of matmul operands for backward (lib_sparse/config.py:12).
CACHE_FP8_MATMUl = False
