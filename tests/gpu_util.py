"""Helpers shared by the GPU tests: numpy bit arrays <-> CUDA tensors."""
import numpy as np
import torch

from oracle import bitsparse_oracle as O

TORCH_DT = {O.DT_BF16: torch.bfloat16, O.DT_E4M3: torch.float8_e4m3fn,
            O.DT_E5M2: torch.float8_e5m2}


def to_dev(bits: np.ndarray, dtype: str, shape=None) -> torch.Tensor:
    """Raw bits (uint16 bf16 / uint8 fp8) -> CUDA tensor of that dtype."""
    a = np.ascontiguousarray(bits)
    if shape is not None:
        a = a.reshape(shape)
    if dtype == O.DT_BF16:
        t = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    else:
        t = torch.from_numpy(a.view(np.uint8).copy()).view(TORCH_DT[dtype])
    return t.cuda()


def bits(t: torch.Tensor) -> np.ndarray:
    """CUDA tensor -> numpy raw bits (uint16 for 2-byte, uint8 for 1-byte,
    uint32 for prefix)."""
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.uint32:
        return t.view(torch.int32).numpy().view(np.uint32)
    if t.element_size() == 2:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.element_size() == 1:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def oracle_sparse(sp) -> "O.Sparse":
    """BitsparseTensor (CUDA) -> oracle Sparse (to run oracle ops on our output)."""
    dt = {torch.bfloat16: O.DT_BF16, torch.float8_e4m3fn: O.DT_E4M3,
          torch.float8_e5m2: O.DT_E5M2}[sp.dtype]
    scale = None if sp.scale is None else np.float32(sp.scale.item())
    return O.Sparse(bits(sp.vals), bits(sp.bitmask), bits(sp.prefix), tuple(sp.shape), dt,
                    int(sp.vals_offset.reshape(-1)[0].item()), sp.pack_sbit, scale)


def payload(vals: np.ndarray, start: int, nnz: int, nbits: int) -> np.ndarray:
    """Keep only bits [start*nbits, (start+nnz)*nbits) of a packed stream."""
    out = vals.copy()
    sb = np.unpackbits(out, bitorder="little")
    idx = np.arange(sb.size)
    sb &= ((idx >= start * nbits) & (idx < (start + nnz) * nbits)).astype(np.uint8)
    return np.packbits(sb, bitorder="little")


_COMPILED = None


def reference_to_fp8(x: torch.Tensor, compiled: bool = True):
    """The reference's to_fp8 (lib_sparse/fp8.py:123-129), its three lines
    restated here, run on the GPU as the reference runs it: compiled by
    torch.compile (Inductor / Triton), or eagerly."""
    global _COMPILED

    @torch.no_grad()
    def to_fp8(t):
        scale = (t.detach().abs().max() / torch.finfo(torch.float8_e4m3fn).max).to(torch.float32)
        scale = scale.clamp(min=1e-9)
        return (t / scale).to(torch.float8_e4m3fn), scale

    if not compiled:
        return to_fp8(x)
    if _COMPILED is None:
        _COMPILED = torch.compile(to_fp8)
    return _COMPILED(x)
