"""CPU baseline of the compress + reconstruct round trip -- TEST / BENCH INFRASTRUCTURE.

Runs the oracle restatement of the reference's algorithm
(oracle/bitsparse_oracle.py) on the host cores, sharded by 64-row tile rows
over a process pool (tile rows are independent; the only cross-shard
quantity is the value offset, rebased by an exclusive scan of shard totals,
exactly as one global run would place them).  Only ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs use it.
"""
from __future__ import annotations

import os
import time
from concurrent.futures import ProcessPoolExecutor

import numpy as np

from . import bitsparse_oracle as O


def _round_trip(block: np.ndarray):
    M, N = block.shape
    sp = O.dense_to_tilesparse(block, O.DT_BF16)
    rec = O.reconstruct(sp)
    return sp.nnz, bool(np.array_equal(rec, block))


def synthetic_relu_bf16(M: int, N: int, mu: float = 0.0, seed: int = 0) -> np.ndarray:
    """bf16 bits of relu(N(mu, 1)) (the C3 workload's distribution)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, N), dtype=np.float32) + np.float32(mu)
    return O.f32_to_bf16(np.maximum(x, 0))


def round_trip_bytes(M: int, N: int, nnz: int, elt: int = 2) -> int:
    """Algorithmic bytes of compress + reconstruct of an [M, N] tensor."""
    T = ((M + 63) // 64) * ((N + 63) // 64)
    one = M * N * elt + M * N // 8 + nnz * elt + 4 * (T + 1)
    return 2 * one


class CpuRoundTrip:
    """Times oracle compress + reconstruct of one [M, N] bf16 sample."""

    def __init__(self, M: int, N: int, mu: float = 0.0, workers: int | None = None):
        self.M, self.N = M, N
        self.workers = workers or os.cpu_count() or 1
        self.x = synthetic_relu_bf16(M, N, mu)
        rows = max(64, (M // self.workers + 63) // 64 * 64)
        self.blocks = [self.x[r: r + rows] for r in range(0, M, rows)]
        self.pool = ProcessPoolExecutor(max_workers=min(self.workers, len(self.blocks)))

    def step(self) -> int:
        res = list(self.pool.map(_round_trip, self.blocks))
        assert all(ok for _, ok in res), "oracle round trip failed"
        return sum(n for n, _ in res)

    def measure(self, steps: int = 1, warmup: int = 0):
        for _ in range(warmup):
            self.step()
        t0 = time.perf_counter()
        nnz = 0
        for _ in range(steps):
            nnz = self.step()
        dt = (time.perf_counter() - t0) / steps
        return round_trip_bytes(self.M, self.N, nnz) / dt / 1e9, dt

    def close(self):
        self.pool.shutdown()
