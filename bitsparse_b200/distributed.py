"""Token-row sharding of compressed activations across ranks.

Compression and reconstruction are independent per tile row (64 token rows),
so on N GPUs each rank compresses only its own rows and no communication is
needed on the data path (the reference runs one process per GPU the same
way).  Where a global view is wanted -- one compressed tensor for a
checkpoint, or an activation all-gather -- the shards are merged without
decompressing:

* the bitmasks of whole tile rows are contiguous in the global tile order,
  so they concatenate;
* the global prefix is each shard's prefix offset by the value counts of
  the shards before it (mod 2^32, like the reference's int32 cumsum viewed
  as uint32, lib_sparse/src/functions.py:33-40);
* the raw value streams concatenate.

These are host-side helpers on torch tensors (any device, any
torch.distributed backend); they launch no kernels of their own.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .bitsparse import BitsparseTensor, tile_grid
from .config import BLOCK_M


def row_range(M: int, rank: int, world: int, block: int = BLOCK_M) -> tuple[int, int]:
    """Rows [start, stop) of an [M, N] tensor owned by `rank` of `world`:
    contiguous runs of whole tile rows (the last shard takes the ragged end;
    trailing ranks may get no rows)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} not in a world of {world}")
    tiles_m = (M + block - 1) // block
    per = (tiles_m + world - 1) // world
    start = min(rank * per * block, M)
    stop = min((rank + 1) * per * block, M)
    return start, stop


def _values(sp: BitsparseTensor) -> torch.Tensor:
    """The shard's own nnz raw values (a slice of an arena when shared).

    nnz is the uint32 prefix[-1], which wraps once a shard holds 2^32 values;
    such shards are refused rather than merged with a truncated stream."""
    if sp.shape[0] * sp.shape[1] >= 1 << 32:
        raise ValueError("a shard of 2^32 or more elements cannot be merged: its value "
                         "count does not fit the uint32 prefix")
    nnz = int(sp.prefix[-1].item())
    off = int(sp.vals_offset.reshape(-1)[0].item())
    return sp.vals[off: off + nnz]


def concat_row_shards(shards: list[BitsparseTensor]) -> BitsparseTensor:
    """Merge compressed row shards (in row order) into one compressed tensor
    equal to compressing the concatenated rows.  Raw (not pack_sbit) storage;
    every shard but the last must hold whole tile rows; fp8 shards must share
    one scale."""
    if not shards:
        raise ValueError("no shards")
    s0 = shards[0]
    N = s0.shape[1]
    for i, s in enumerate(shards):
        if s.pack_sbit:
            raise ValueError("concat_row_shards takes raw storage (pack_sbit=False)")
        if s.shape[1] != N or s.dtype != s0.dtype:
            raise ValueError("shards differ in columns or dtype")
        if (s.BLOCK_M, s.BLOCK_N) != (s0.BLOCK_M, s0.BLOCK_N):
            raise ValueError("shards differ in tile size")
        if i < len(shards) - 1 and s.shape[0] % s.BLOCK_M:
            raise ValueError("every shard but the last must hold whole tile rows")
    scales = [s.scale for s in shards]
    if any(sc is not None for sc in scales):
        if any(sc is None for sc in scales) or any(
                not torch.equal(sc.reshape(()), scales[0].reshape(())) for sc in scales):
            raise ValueError("fp8 shards must share one scale")
    M = sum(s.shape[0] for s in shards)
    grid_m, grid_n, _, _, _ = tile_grid(M, N, s0.BLOCK_M, s0.BLOCK_N)
    bitmask = torch.cat([s.bitmask for s in shards])
    pieces, base = [], 0
    for s in shards:
        p = s.prefix.to(torch.int64)
        pieces.append(p[:-1] + base)
        base += int(p[-1].item())
    pieces.append(torch.tensor([base], dtype=torch.int64, device=bitmask.device))
    prefix = (torch.cat(pieces) & 0xFFFFFFFF).to(torch.uint32)
    vals = torch.cat([_values(s) for s in shards])
    return BitsparseTensor(vals, bitmask, prefix, (M, N), s0.dtype, grid_m, grid_n,
                           s0.BLOCK_M, s0.BLOCK_N, scale=s0.scale, pack_sbit=False)


def _all_gather_var(t: torch.Tensor, sizes: list[int], group) -> list[torch.Tensor]:
    """all_gather of 1-D tensors of different lengths (padded to the longest)."""
    n = max(sizes) if sizes else 0
    pad = torch.zeros(n, dtype=t.dtype, device=t.device)
    pad[: t.numel()] = t
    out = [torch.empty_like(pad) for _ in sizes]
    dist.all_gather(out, pad, group=group)
    return [o[:k] for o, k in zip(out, sizes)]


def gather_bitsparse(local: BitsparseTensor, group=None) -> BitsparseTensor:
    """All-gather the row shards of every rank (rank order = row order) into
    the global compressed tensor, on every rank."""
    world = dist.get_world_size(group)
    vals = _values(local)
    dev = local.bitmask.device
    meta = torch.tensor([local.shape[0], local.bitmask.numel(), local.prefix.numel(),
                         vals.numel()], dtype=torch.int64, device=dev)
    metas = [torch.empty_like(meta) for _ in range(world)]
    dist.all_gather(metas, meta, group=group)
    rows, bm_n, pf_n, v_n = ([int(m[i].item()) for m in metas] for i in range(4))
    bms = _all_gather_var(local.bitmask, bm_n, group)
    pfs = _all_gather_var(local.prefix.to(torch.int64), pf_n, group)
    # bf16 / fp8 values travel as raw bytes (not every backend takes fp8)
    vbytes = _all_gather_var(vals.view(torch.uint8), [k * vals.element_size() for k in v_n],
                             group)
    shards = []
    for r in range(world):
        if rows[r] == 0:
            continue
        gm, gn, _, _, _ = tile_grid(rows[r], local.shape[1], local.BLOCK_M, local.BLOCK_N)
        shards.append(BitsparseTensor(vbytes[r].view(local.vals.dtype), bms[r],
                                      pfs[r].to(torch.uint32), (rows[r], local.shape[1]),
                                      local.dtype, gm, gn, local.BLOCK_M, local.BLOCK_N,
                                      scale=local.scale, pack_sbit=False))
    return concat_row_shards(shards)


class GradAllReduce:
    """Data-parallel gradient reduction overlapped with the backward pass.

    The reference's nanoGPT trainer sums every parameter's gradient over the
    ranks after the backward pass, one ``all_reduce`` per parameter
    (``dist.all_reduce(p.grad, op=SUM)``, nanogpt/logs/...txt:385-387).  Here
    the parameters are grouped, in reverse registration order (roughly the
    order the backward pass produces their gradients), into buckets of about
    ``bucket_mb`` MB; a post-accumulate-grad hook counts the gradients of
    each bucket, and when the last one is ready the bucket is flattened and
    its ``all_reduce`` starts asynchronously (NCCL on GPUs, gloo on CPUs)
    while the backward pass continues.  ``wait()`` completes the reductions
    and writes the summed (``op="sum"``) or averaged (``"avg"``) gradients
    back.  One instance serves every step; a parameter without a gradient in
    a step is reduced as zeros.
    """

    def __init__(self, params, group=None, bucket_mb: float = 32.0, op: str = "sum"):
        if op not in ("sum", "avg"):
            raise ValueError("op must be 'sum' or 'avg'")
        self.group, self.op = group, op
        self.params = [p for p in params if p.requires_grad]
        limit = int(bucket_mb * 2**20)
        self.buckets: list[list] = []
        cur, size = [], 0
        for p in reversed(self.params):
            cur.append(p)
            size += p.numel() * p.element_size()
            if size >= limit:
                self.buckets.append(cur)
                cur, size = [], 0
        if cur:
            self.buckets.append(cur)
        self._bucket_of = {}
        for i, b in enumerate(self.buckets):
            for p in b:
                self._bucket_of[p] = i
        self._pending = [len(b) for b in self.buckets]
        self._works: list = [None] * len(self.buckets)
        self._flat: list = [None] * len(self.buckets)
        self._hooks = [p.register_post_accumulate_grad_hook(self._ready) for p in self.params]

    def _launch(self, i: int) -> None:
        grads = [p.grad if p.grad is not None else torch.zeros_like(p) for p in self.buckets[i]]
        flat = torch.cat([g.reshape(-1) for g in grads])
        self._flat[i] = flat
        self._works[i] = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group,
                                         async_op=True)

    def _ready(self, p) -> None:
        i = self._bucket_of[p]
        self._pending[i] -= 1
        if self._pending[i] == 0:
            self._launch(i)

    def wait(self) -> None:
        """Finish every bucket's reduction (launching those whose gradients
        did not all arrive) and write the results into ``p.grad``."""
        world = dist.get_world_size(self.group)
        for i, b in enumerate(self.buckets):
            if self._works[i] is None:
                self._launch(i)
            self._works[i].wait()
            flat = self._flat[i]
            if self.op == "avg":
                flat.div_(world)
            off = 0
            for p in b:
                n = p.numel()
                g = flat[off: off + n].view_as(p)
                if p.grad is None:
                    p.grad = g.clone()
                else:
                    p.grad.copy_(g)
                off += n
            self._works[i] = self._flat[i] = None
            self._pending[i] = len(b)

    def remove(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []
