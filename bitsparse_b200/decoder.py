"""A decoder-only transformer whose MLP activations are stored compressed.

The data-parallel training workload of config 5: a GPT-2-medium-shaped
decoder (24 layers, width 1024, 16 heads, MLP 4096, vocabulary 50304,
sequence 1024) in the layout of the reference's nanoGPT caller
(nanogpt/nanogpt.py:8-146: RMSNorm before attention and MLP, residual
adds, biased linears, an untied output projection and a summed
cross-entropy).  Each MLP is ``FFNRelu`` -- its hidden activation is kept
between forward and backward as a BitsparseTensor -- or, with
``compressed=False``, the same MLP with the activation kept dense, so the
two differ only in how the activation is stored.

Attention is PyTorch's ``scaled_dot_product_attention`` (a library kernel);
only the MLP is this package's.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from .layers import FFNRelu


@dataclass
class DecoderConfig:
    vocab: int = 50304
    layers: int = 24
    dim: int = 1024
    heads: int = 16
    mlp: int = 4096
    seq: int = 1024
    compressed: bool = True
    # compressed MLP activations kept in one TensorBuffer arena shared by all
    # layers (no host sync per layer) holding this fraction of the dense
    # activations' values; 0: each layer allocates its own exact storage
    # (one host sync per layer, the reference's default)
    arena_fraction: float = 0.0


class _Block(nn.Module):
    def __init__(self, cfg: DecoderConfig):
        super().__init__()
        d, h = cfg.dim, cfg.mlp
        self.cfg = cfg
        self.norm1 = nn.RMSNorm(d)
        self.qkv = nn.Linear(d, 3 * d)
        self.proj = nn.Linear(d, d)
        self.norm2 = nn.RMSNorm(d)
        self.fc = nn.Linear(d, h)      # W1 [mlp, dim]
        self.fc_out = nn.Linear(h, d)  # W2 [dim, mlp]

    def _mlp(self, x: Tensor, arena) -> Tensor:
        W1, b1, W2, b2 = self.fc.weight, self.fc.bias, self.fc_out.weight, self.fc_out.bias
        if self.cfg.compressed:
            return FFNRelu.apply(x, W1, W2, b1, b2, sparse_data=arena)
        return F.linear(torch.relu(F.linear(x, W1, b1)), W2, b2)

    def forward(self, x: Tensor, arena=None) -> Tensor:
        B, T, D = x.shape
        H = self.cfg.heads
        q, k, v = self.qkv(self.norm1(x)).view(B, T, 3, H, D // H).unbind(2)
        y = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                           v.transpose(1, 2), is_causal=True)
        x = x + self.proj(y.transpose(1, 2).reshape(B, T, D))
        return x + self._mlp(self.norm2(x), arena)


class Decoder(nn.Module):
    """``Decoder(cfg)(tokens [B, T], targets [B, T]) -> summed loss``."""

    def __init__(self, cfg: DecoderConfig):
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab, cfg.dim)
        self.pos = nn.Embedding(cfg.seq, cfg.dim)
        self.blocks = nn.ModuleList(_Block(cfg) for _ in range(cfg.layers))
        self.norm = nn.RMSNorm(cfg.dim)
        self.head = nn.Linear(cfg.dim, cfg.vocab)
        for p in self.parameters():  # random init ~ N(0, 0.02), as config 5 states
            nn.init.normal_(p, 0.0, 0.02) if p.dim() > 1 else nn.init.zeros_(p)
        for m in self.modules():
            if isinstance(m, nn.RMSNorm):
                nn.init.ones_(m.weight)
        self.arena = None

    def _arena(self, tokens: int, device, dtype):
        """The shared value arena (allocated on first use, reset per step)."""
        from .bitsparse import TensorBuffer
        cfg = self.cfg
        if not cfg.compressed or cfg.arena_fraction <= 0:
            return None
        elt = torch.empty((), dtype=dtype).element_size()
        n = int(cfg.arena_fraction * cfg.layers * tokens * cfg.mlp)
        if self.arena is None or self.arena.vals.numel() < n:
            self.arena = TensorBuffer(n * elt, device=device, dtype=dtype)
        self.arena.offset.zero_()
        return self.arena

    def forward(self, tokens: Tensor, targets: Tensor) -> Tensor:
        T = tokens.shape[1]
        x = self.embed(tokens) + self.pos.weight[:T]
        arena = self._arena(tokens.numel(), x.device, x.dtype)
        for blk in self.blocks:
            x = blk(x, arena)
        logits = self.head(self.norm(x)).float()
        return F.cross_entropy(logits.view(-1, logits.shape[-1]), targets.reshape(-1),
                               reduction="sum")
