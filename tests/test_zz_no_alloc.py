"""GPU: the no-allocation compress entry point against the regular one.

bs_compress_noalloc exists for callers that cannot allocate device memory
(code that runs inside an allocator or under a hook that forbids cudaMalloc,
hosts without a device allocator): its scan scratch is a fixed array inside
the library instead of a caller-provided workspace.  This test calls it
through the C ABI twice in a row, on different inputs, and checks every
output byte against bs_compress with a normal workspace (integer and byte
outputs: the tolerance is exact equality).  It lives in its own file, named
to be collected last, and passes alone or after the other tests.
"""
import ctypes

import pytest
import torch

from bitsparse_b200 import _lib
from bitsparse_b200 import _runtime as R

pytestmark = pytest.mark.gpu


def _compress(lib, fn, dense, dtype_code, with_workspace):
    M, N = dense.shape
    T = ((M + 63) // 64) * ((N + 63) // 64)
    dev = dense.device
    bitmask = torch.full((T * 512,), 0xAB, dtype=torch.uint8, device=dev)
    prefix = torch.full((T + 1,), 7, dtype=torch.int32, device=dev)
    vals = torch.zeros(M * N, dtype=dense.dtype, device=dev)
    nnz = torch.full((1,), -1, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    common = (dense.data_ptr(), dtype_code, M, N, N, None, None, bitmask.data_ptr(),
              prefix.data_ptr(), vals.data_ptr(), M * N, 0, None, None, nnz.data_ptr())
    if with_workspace:
        ws = torch.zeros(lib.bs_compress_workspace_bytes(T), dtype=torch.uint8, device=dev)
        rc = fn(*common, ws.data_ptr(), ws.numel(), status.data_ptr(), stream)
    else:
        rc = fn(*common, status.data_ptr(), stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    assert status.item() == 0
    n = int(nnz.item())
    return bitmask, prefix, vals[:n], n


@pytest.mark.parametrize("dtype, code", [(torch.bfloat16, _lib.BS_BF16),
                                         (torch.float8_e4m3fn, _lib.BS_E4M3)])
def test_noalloc_matches_regular_compress_twice(dtype, code):
    lib = _lib.load()
    g = torch.Generator().manual_seed(21)
    for shape, mu in (((1000, 3000), 0.0), ((4096, 2048), -1.0)):  # two calls in a row
        x = (torch.randn(*shape, generator=g) + mu).relu().to(dtype).cuda()
        ref = _compress(lib, lib.bs_compress, x, code, True)
        got = _compress(lib, lib.bs_compress_noalloc, x, code, False)
        assert got[3] == ref[3] == int((x.float() > 0).sum().item())
        for a, b in zip(got[:3], ref[:3]):
            assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))


def test_noalloc_rejects_tensors_above_its_maximum():
    lib = _lib.load()
    max_tiles = lib.bs_compress_noalloc_max_tiles()
    M = 64 * (max_tiles // 1024 + 1)  # (max/1024 + 1) tile rows x 1024 tile columns
    N = 64 * 1024
    rc = lib.bs_compress_noalloc(16, _lib.BS_BF16, M, N, N, None, None, 16, 16, 16, 0, 0,
                                 None, None, None, None, None)
    assert rc == _lib.BS_ERR_TOO_LARGE
