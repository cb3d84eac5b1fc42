"""CPU, world_size 2 over gloo: the vocabulary-sharded argmax combine.

Each rank computes the (max, index) keys of its shard with the oracle, then
``slang_b200.lmhead.combine_keys_`` all-reduces them exactly as the GPU path
does over NCCL.  The decoded token must equal the unsharded argmax, including a
tie that straddles the shard boundary (lowest index wins).
"""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import q4
from slang_b200 import lmhead, synth


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        rng = np.random.default_rng(0)
        v, k = 4096, 256
        packed, scales = synth.q4_weight(rng, v, k)
        h = rng.standard_normal((3, k), dtype=np.float32)
        # row 3 of the batch: a tie between row 100 (shard 0) and row 3000 (shard 1)
        logits = q4.gemv(packed, scales, h)
        top = int(np.argmax(logits[2]))
        for r in (100, 3000):
            packed[r] = packed[top]
            scales[r] = (scales[top].astype(np.float32) * 2).astype(np.float16)
        lo, hi = lmhead.shard_bounds(v, rank, world)
        idx, val = q4.lmhead_argmax(packed[lo:hi], scales[lo:hi], h)
        keys = torch.from_numpy(q4.pack_key(val, idx + lo).view(np.int64).copy())
        lmhead.combine_keys_(keys)
        got = q4.unpack_key_index(keys.numpy().view(np.uint64))
        want, _ = q4.lmhead_argmax(packed, scales, h)
        q.put((rank, got.tolist(), want.tolist()))
        dist.destroy_process_group()
    except Exception as e:  # surface the failure to the parent
        q.put((rank, repr(e), None))


def test_sharded_argmax_combine_gloo():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, got, want in results:
        assert want is not None, f"rank {rank} failed: {got}"
        assert got == want, f"rank {rank}: {got} != {want}"
        assert got[2] == 100, "the tie across shards must resolve to the lower index"


def test_combine_is_noop_without_process_group():
    keys = torch.tensor([5, -3], dtype=torch.int64)
    assert lmhead.combine_keys_(keys.clone()).tolist() == [5, -3]
