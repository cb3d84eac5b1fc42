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


class PeerLMHead(ShardedLMHead):
    """The sharded lm_head with the cross-GPU step done in device memory over
    NVLink instead of an NCCL call.

    Every rank owns a small mailbox (``sb_peer_buffer_create``) that every
    other rank maps (CUDA IPC).  The shard GEMV's CTAs fold their argmax keys
    into this rank's mailbox; the last CTA to finish writes each row's key,
    tagged with the step, into this rank's slot of every rank's mailbox over
    NVLink, waits (bounded) until every rank's slots in its own mailbox carry
    the step's tag, and takes the MAX -- one launch, no fence, no host
    synchronisation, capturable in a CUDA graph.
    The exchange is a function of the call sequence: every rank must call once
    per step.
    """

    def __init__(self, emb: torch.Tensor, scales: torch.Tensor, rank: int = 0, world: int = 1, group=None,
                 full_table: bool = True):
        import ctypes

        super().__init__(emb, scales, rank, world, group, full_table)
        from . import _lib
        self._lib = _lib
        self.rank = rank
        size = int(_lib.load().sb_peer_mailbox_size())
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        _lib.call("sb_peer_buffer_create", size, ctypes.byref(own), handle)
        self.own = own.value
        handles = [bytes(handle)]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened = []
        ptrs = []
        for r, hb in enumerate(handles):
            if r == rank:
                ptrs.append(self.own)
                continue
            p = ctypes.c_void_p()
            buf = (ctypes.c_char * 64).from_buffer_copy(hb)
            _lib.call("sb_peer_buffer_open", buf, ctypes.byref(p))
            self.opened.append(p.value)
            ptrs.append(p.value)
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=emb.device)

    def __call__(self, h: torch.Tensor, keys: torch.Tensor | None = None,
                 tokens: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        k = self.emb.shape[1] * 2
        h2 = h.reshape(-1, k)
        m = h2.shape[0]
        if keys is None:
            keys = torch.empty(m, dtype=torch.int64, device=h.device)
        if tokens is None:
            tokens = torch.empty(m, dtype=torch.int32, device=h.device)
        self._lib.call("sb_lmhead_argmax_peer", kern._ptr(self.emb), kern._ptr(self.scales),
                       kern._DT[self.scales.dtype], kern.group_of(self.scales, k), kern._ptr(h2), kern._DT[h.dtype], m,
                       self.emb.shape[0], k, int(self.lo), kern._ptr(self.peers), self.world, self.own,
                       kern._ptr(keys), kern._ptr(tokens), kern._stream())
        return keys, tokens

    def close(self):
        """Unmap the peers' mailboxes, wait for every rank, free this one."""
        torch.cuda.synchronize()
        for p in self.opened:
            self._lib.call("sb_peer_buffer_close", p)
        self.opened = []
        if self.world > 1:
            dist.barrier(group=self.group)
        if self.own:
            self._lib.call("sb_peer_buffer_free", self.own)
            self.own = None
