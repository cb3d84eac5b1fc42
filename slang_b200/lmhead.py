"""Vocabulary-sharded tied lm_head with greedy argmax across GPUs.

Rank r of G holds embedding rows [r*V/G, (r+1)*V/G).  Each rank runs the fused
lm_head GEMV + argmax on its shard (``sb_lmhead_argmax`` with the shard's row
offset), which yields one 64-bit key per decode row:
``(orderable(max logit) << 32) | (0xFFFFFFFF - global index)``.  The largest key
over all shards is the global greedy token with the reference's lowest-index
tie rule (gemma4_150/kernels_dsl.py:491-496), so the cross-GPU step is a single
integer MAX all-reduce of 8 bytes per row over NCCL.  The reference is
single-device; this partitioning is new.

Keys are ordered as unsigned integers while NCCL/torch reduce int64 as signed,
so the top bit is flipped around the all-reduce (that maps unsigned order onto
signed order and back).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import kernels as kern

_SIGN = -(1 << 63)  # int64 with only the top bit set


def shard_bounds(vocab: int, rank: int, world: int) -> tuple[int, int]:
    return rank * vocab // world, (rank + 1) * vocab // world


def combine_keys_(keys: torch.Tensor, group=None) -> torch.Tensor:
    """In place: keys <- MAX over ranks (unsigned order), via a signed int64 all-reduce."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return keys
    keys.bitwise_xor_(_SIGN)
    dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=group)
    keys.bitwise_xor_(_SIGN)
    return keys


class ShardedLMHead:
    """This rank's shard of the tied embedding, used as the lm_head."""

    def __init__(self, emb: torch.Tensor, scales: torch.Tensor, rank: int = 0, world: int = 1, group=None,
                 full_table: bool = True):
        vocab = emb.shape[0] * (1 if full_table else world)
        self.lo, self.hi = shard_bounds(vocab, rank, world)
        if full_table:
            emb, scales = emb[self.lo:self.hi], scales[self.lo:self.hi]
        self.emb = emb.contiguous()
        self.scales = scales.contiguous()
        self.group = group
        self.world = world

    def __call__(self, h: torch.Tensor, keys: torch.Tensor | None = None,
                 tokens: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        keys, _ = kern.lmhead_argmax(self.emb, self.scales, h, row_offset=self.lo, keys=keys, want_tokens=False)
        combine_keys_(keys, self.group)
        return keys, kern.keys_to_tokens(keys, tokens)
