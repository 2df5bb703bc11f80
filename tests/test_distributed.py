"""Token-row sharding (bitsparse_b200.distributed): shard, compress each
shard, merge (locally or with an all-gather over world_size-2 gloo ranks on
the CPU) == compress the whole tensor.  Shards are compressed by the CPU
oracle here (host logic only); the GPU test compresses them with the
CUDA path."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bitsparse_b200.bitsparse import BitsparseTensor, tile_grid
from bitsparse_b200.distributed import concat_row_shards, gather_bitsparse, row_range
from oracle import bitsparse_oracle as O

_TORCH = {O.DT_BF16: torch.bfloat16, O.DT_E4M3: torch.float8_e4m3fn}


def _input(M, N, dt, seed):
    rng = np.random.default_rng(seed)
    x = np.maximum(rng.standard_normal((M, N)).astype(np.float32) - 0.3, 0)
    return O.f32_to_bf16(x) if dt == O.DT_BF16 else O.f32_to_fp8(x, dt)


def _as_torch(sp: "O.Sparse") -> BitsparseTensor:
    dt = _TORCH[sp.dtype]
    if sp.dtype == O.DT_BF16:
        vals = torch.from_numpy(sp.vals.view(np.int16).copy()).view(dt)
    else:
        vals = torch.from_numpy(sp.vals.copy()).view(dt)
    gm, gn, _, _, _ = tile_grid(*sp.shape, 64, 64)
    return BitsparseTensor(vals, torch.from_numpy(sp.bitmask.copy()),
                           torch.from_numpy(sp.prefix.view(np.int32).copy()).view(torch.uint32),
                           sp.shape, dt, gm, gn, 64, 64)


def _check(merged: BitsparseTensor, full: "O.Sparse"):
    np.testing.assert_array_equal(merged.bitmask.numpy(), full.bitmask)
    np.testing.assert_array_equal(merged.prefix.view(torch.int32).numpy().view(np.uint32),
                                  full.prefix)
    v = merged.vals.view(torch.int16 if merged.vals.element_size() == 2 else torch.uint8)
    np.testing.assert_array_equal(v.numpy().view(full.vals.dtype), full.vals)
    assert tuple(merged.shape) == tuple(full.shape)


@pytest.mark.parametrize("M, world", [(1, 2), (64, 2), (300, 2), (1000, 3), (130, 4),
                                      (4096, 8), (65, 8)])
def test_row_range_partitions_whole_tile_rows(M, world):
    spans = [row_range(M, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == M
    for (a, b), (c, d) in zip(spans, spans[1:]):
        assert b == c and a <= b
    for a, b in spans:
        assert a % 64 == 0 or a == M  # shards start on a tile row (or are empty)


@pytest.mark.parametrize("dt", [O.DT_BF16, O.DT_E4M3])
@pytest.mark.parametrize("M, N, world", [(300, 200, 2), (640, 70, 3), (64, 64, 4)])
def test_concat_row_shards_equals_whole_compress(dt, M, N, world):
    x = _input(M, N, dt, seed=M + N)
    shards = []
    for r in range(world):
        a, b = row_range(M, r, world)
        if b > a:
            shards.append(_as_torch(O.dense_to_tilesparse(x[a:b], dt)))
    _check(concat_row_shards(shards), O.dense_to_tilesparse(x, dt))


def test_concat_rejects_ragged_inner_shard():
    x = _input(100, 64, O.DT_BF16, seed=1)
    a = _as_torch(O.dense_to_tilesparse(x[:50], O.DT_BF16))
    b = _as_torch(O.dense_to_tilesparse(x[50:], O.DT_BF16))
    with pytest.raises(ValueError):
        concat_row_shards([a, b])


def _gather_worker(rank, world, port, M, N):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = _input(M, N, O.DT_BF16, seed=7)
        a, b = row_range(M, rank, world)
        local = _as_torch(O.dense_to_tilesparse(x[a:b], O.DT_BF16))
        merged = gather_bitsparse(local)
        _check(merged, O.dense_to_tilesparse(x, O.DT_BF16))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gather_bitsparse_gloo(world):
    """world_size-2 gloo ranks on the CPU: all-gather of compressed shards."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_gather_worker, args=(world, port, 700, 150), nprocs=world, join=True)


@pytest.mark.gpu
def test_sharded_gpu_compress_concat():
    """Shards compressed by the CUDA path and merged == the whole tensor
    compressed by the CUDA path (one GPU standing in for the ranks)."""
    from bitsparse_b200.src.functions import dense_to_tilesparse
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(1000, 3000, generator=g, device="cuda").relu().to(torch.bfloat16)
    whole = dense_to_tilesparse(x, None)
    shards = [dense_to_tilesparse(x[a:b].contiguous(), None)
              for a, b in (row_range(1000, r, 3) for r in range(3))]
    merged = concat_row_shards(shards)
    assert torch.equal(merged.bitmask, whole.bitmask)
    assert torch.equal(merged.prefix.view(torch.int32), whole.prefix.view(torch.int32))
    assert torch.equal(merged.vals, whole.vals)


def _small_model(seed):
    torch.manual_seed(seed)
    return torch.nn.Sequential(torch.nn.Linear(16, 64), torch.nn.ReLU(), torch.nn.Linear(64, 8),
                               torch.nn.ReLU(), torch.nn.Linear(8, 3))


def _rank_batch(rank):
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randn(32, 16, generator=g), torch.randn(32, 3, generator=g)


def _grad_worker(rank, world, port, op, steps):
    from bitsparse_b200.distributed import GradAllReduce
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = _small_model(0)
        red = GradAllReduce(model.parameters(), bucket_mb=0.001, op=op)  # several buckets
        assert len(red.buckets) > 1
        x, y = _rank_batch(rank)
        # the expected result: every rank's gradients, computed here, summed
        ref = [torch.zeros_like(p) for p in model.parameters()]
        for r in range(world):
            m = _small_model(0)
            xr, yr = _rank_batch(r)
            ((m(xr) - yr) ** 2).sum().backward()
            for acc, p in zip(ref, m.parameters()):
                acc += p.grad
        if op == "avg":
            ref = [g / world for g in ref]
        for _ in range(steps):  # the same instance across steps
            model.zero_grad(set_to_none=True)
            ((model(x) - y) ** 2).sum().backward()
            red.wait()
            for p, g in zip(model.parameters(), ref):
                torch.testing.assert_close(p.grad, g, rtol=1e-5, atol=1e-6)
        red.remove()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("op", ["sum", "avg"])
def test_grad_all_reduce_gloo(op):
    """world_size-2 gloo ranks on the CPU: the bucketed, backward-overlapped
    gradient reduction equals the sum (or mean) of every rank's gradients,
    over repeated steps."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_grad_worker, args=(2, port, op, 3), nprocs=2, join=True)
