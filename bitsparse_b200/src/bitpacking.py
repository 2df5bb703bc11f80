"""Host-side sizes of the packed 15/7-bit value stream.

Same formulas as lib_sparse/src/bitpacking.py:27-34; the packing and
decoding themselves are fused into the CUDA compress / unpack kernels.
"""


def packed_nbytes(numel: int, bits_per_value: int) -> int:
    """Payload bytes of ``numel`` values of ``bits_per_value`` bits."""
    return (int(numel) * bits_per_value + 7) // 8


def packed_storage_nbytes(numel: int, bits_per_value: int) -> int:
    """Word-rounded storage plus one guard word."""
    return ((packed_nbytes(numel, bits_per_value) + 3) // 4) * 4 + 4
