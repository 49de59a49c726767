"""Vocabulary-parallel INT8 LM head: each tensor-parallel rank holds V/world head rows.

The reference head (otf_llm/symmetric_2bit_engine.py:50-91) holds all V rows on one
device.  Split by rows, each rank runs the fused INT8 head kernel over its own rows; the
ranks then exchange either the logits (``forward``, which keeps the reference's
``lm_head(h) -> [..., V]`` contract) or one (max logit, global row) pair per batch row
(``argmax``, for greedy decoding: 16 bytes per row instead of 4*V/world).

The combined argmax equals ``torch.argmax`` over the full logit row: the largest value
wins, and among equal values the lowest vocabulary index, because the ranks hold
ascending row ranges and every rank's own pick is already the first of its maxima.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import _native
from .symmetric_2bit_engine import QuantizedLinearHead


def combine_argmax(local_max: torch.Tensor, local_idx: torch.Tensor, row0: int, group=None) -> torch.Tensor:
    """Global greedy ids from every rank's (max logit, local row) per batch row.

    local_max: [M] float, local_idx: [M] int64 (rows of this rank's shard, which starts
    at global row ``row0``).  The pairs travel as float64 (an fp32 logit and an index
    below 2**53 are both exact in it) in one all_gather.
    """
    world = torch.distributed.get_world_size(group)
    pair = torch.stack([local_max.to(torch.float64), (local_idx + row0).to(torch.float64)], dim=-1)
    gathered = [torch.empty_like(pair) for _ in range(world)]
    torch.distributed.all_gather(gathered, pair.contiguous(), group=group)
    allp = torch.stack(gathered, dim=0)                     # [world, M, 2], rank order = vocab order
    vals = allp[..., 0]
    # NaN never wins (the kernel's logits are finite after nan_to_num); the first rank
    # holding the maximum holds the lowest index among the maxima.
    best = torch.argmax(vals, dim=0)                         # first maximum over ranks
    return allp.gather(0, best.view(1, -1, 1).expand(1, -1, 2))[0, :, 1].to(torch.int64)


class VocabParallelHead(nn.Module):
    """Rows [row0, row0 + shard rows) of a V-row INT8 head on this tensor-parallel rank."""

    def __init__(self, shard: QuantizedLinearHead, row0: int, vocab_size: int, group=None):
        super().__init__()
        self.shard = shard
        self.row0 = row0
        self.vocab_size = vocab_size
        self.in_features = shard.in_features
        self.out_features = vocab_size
        self.group = group

    def local_logits(self, x: torch.Tensor) -> torch.Tensor:
        return self.shard(x)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Full fp32 logits [..., V] (all_gather of the shards' logits)."""
        part = self.shard(x)
        lead = part.shape[:-1]
        world = torch.distributed.get_world_size(self.group)
        flat = part.reshape(-1, part.shape[-1]).contiguous()
        gathered = [torch.empty_like(flat) for _ in range(world)]
        torch.distributed.all_gather(gathered, flat, group=self.group)
        return torch.cat(gathered, dim=-1).view(*lead, self.vocab_size)

    def argmax(self, x: torch.Tensor, logits: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Greedy ids [M] for x [M, D] fp16: fused local head + argmax, then one pair exchange."""
        x2d = x.reshape(-1, x.shape[-1]).to(torch.float16).contiguous()
        M = x2d.shape[0]
        if logits is None:
            logits = torch.empty(M, self.shard.out_features, dtype=torch.float32, device=x2d.device)
        idx = _native.i8_head_argmax(x2d, self.shard.weight_int8, self.shard.scales, logits=logits)
        vmax = logits.gather(1, idx.view(-1, 1)).view(-1)
        return combine_argmax(vmax, idx, self.row0, self.group)
