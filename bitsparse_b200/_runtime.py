"""Host-side plumbing around the C ABI: device scratch, status word, dtypes.

All device memory is owned by PyTorch's caching allocator.  Per device the
library keeps one int32 status word (device errors OR-ed in by kernels) and,
per (device, stream), a scan workspace for bs_compress (zeroed when it is
allocated and after a bounded wait gave up; consistent between launches
otherwise).
"""
from __future__ import annotations

import threading

import ctypes as C

import torch

from . import _lib

_DT = {
    torch.bfloat16: _lib.BS_BF16,
    torch.float8_e4m3fn: _lib.BS_E4M3,
    torch.float8_e5m2: _lib.BS_E5M2,
    torch.float32: _lib.BS_F32,
}

_lock = threading.Lock()
_status: dict[int, torch.Tensor] = {}
_workspaces: dict[tuple[int, int], torch.Tensor] = {}
_amax: dict[tuple[int, int], torch.Tensor] = {}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def require_cuda(t: torch.Tensor, name: str = "tensor") -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (bitsparse_b200 has no CPU path)")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def stream_handle(device: torch.device) -> int:
    """cudaStream_t of the current stream of `device` (as an int)."""
    if _raw_stream is not None:  # the fast accessor (no Stream object built)
        return _raw_stream(_index(device))
    return torch.cuda.current_stream(device).cuda_stream


def status_word(device: torch.device) -> torch.Tensor:
    idx = _index(device)
    s = _status.get(idx)
    if s is not None:
        return s
    with _lock:
        s = _status.get(idx)
        if s is None:
            s = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
            _status[idx] = s
    return s


_ws_bytes: dict[int, int] = {}


def workspace(device: torch.device, num_tiles: int, stream: int | None = None) -> torch.Tensor:
    """Scan workspace for bs_compress on `stream` (default: the current one)."""
    idx = _index(device)
    key = (idx, stream if stream is not None else stream_handle(device))
    need = _ws_bytes.get(num_tiles)
    if need is None:
        need = _ws_bytes[num_tiles] = int(_lib.load().bs_compress_workspace_bytes(int(num_tiles)))
    ws = _workspaces.get(key)
    if ws is not None and ws.numel() >= need:  # the common case: no lock
        return ws
    with _lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < need:
            # Grow geometrically so a sweep of sizes reallocates rarely.
            size = max(need, 2 * (ws.numel() if ws is not None else 0), 1 << 16)
            ws = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
            _workspaces[key] = ws
    return ws


def amax_scratch(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, stream_handle(device))
    with _lock:
        a = _amax.get(key)
        if a is None:
            a = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
            _amax[key] = a
    return a


def check_status(device: torch.device | None = None, reset: bool = True) -> int:
    """Read (synchronously) the device status word and raise on errors.

    A bounded wait that gave up (BS_STATUS_TIMEOUT) leaves the scan workspace
    in an unknown state, so all workspaces of the device are zeroed.
    """
    device = device or torch.device("cuda", torch.cuda.current_device())
    s = status_word(device)
    v = int(s.item())
    u = C.c_int32(0)
    with torch.cuda.device(device):
        _lib.call("bs_unpack_status", C.addressof(u), int(reset))
    v |= u.value
    if v and reset:
        s.zero_()
        if v & _lib.BS_STATUS_TIMEOUT:
            with _lock:
                for (idx, _), ws in _workspaces.items():
                    if idx == (device.index or 0):
                        ws.zero_()
    if v & _lib.BS_STATUS_CAPACITY:
        raise RuntimeError("bitsparse: value storage too small (writes were clipped)")
    if v & _lib.BS_STATUS_TIMEOUT:
        raise RuntimeError("bitsparse: a bounded device wait gave up (scan workspace reset)")
    return v
