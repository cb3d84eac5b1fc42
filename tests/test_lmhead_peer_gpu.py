"""GPU: the vocabulary-sharded lm_head with the exchange in peer memory.

One GPU: a single rank's mailbox (world 1) equals sb_lmhead_argmax over
consecutive steps and across CUDA-graph replays (the step parity alternates
the key slots).  Two or more GPUs (skipped otherwise): ranks as spawned
processes on cuda:0..G-1 map each other's mailboxes over CUDA IPC; every
rank's tokens equal the full-vocabulary argmax for several steps.
"""
import os
import socket

import numpy as np
import pytest
import torch

from slang_b200 import kernels as kern
from slang_b200 import lmhead, synth

pytestmark = pytest.mark.gpu


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_peer_lmhead_single_rank_steps_and_graph(cuda):
    rng = np.random.default_rng(31)
    v, k, m = 40000, 1536, 3
    packed, scales = synth.q4_weight(rng, v, k)
    E, S = T(packed, cuda), T(scales, cuda)
    head = lmhead.PeerLMHead(E, S, 0, 1)
    try:
        hs = [T(rng.standard_normal((m, k), dtype=np.float32), cuda) for _ in range(4)]
        for h in hs:  # consecutive steps flip the slot parity
            keys, tok = head(h)
            rk, rt = kern.lmhead_argmax(E, S, h)
            np.testing.assert_array_equal(tok.cpu().numpy(), rt.cpu().numpy())
            np.testing.assert_array_equal(keys.cpu().numpy(), rk.cpu().numpy())
        h = torch.empty_like(hs[0])
        keys = torch.empty(m, dtype=torch.int64, device=cuda)
        tok = torch.empty(m, dtype=torch.int32, device=cuda)
        stream = torch.cuda.Stream()
        with torch.cuda.stream(stream):
            h.copy_(hs[0])
            head(h, keys, tok)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                head(h, keys, tok)
        for src in hs:
            with torch.cuda.stream(stream):
                h.copy_(src)
                g.replay()
            torch.cuda.synchronize()
            _, rt = kern.lmhead_argmax(E, S, src)
            np.testing.assert_array_equal(tok.cpu().numpy(), rt.cpu().numpy())
        kern.device_status()
    finally:
        head.close()


def _worker(rank, world, port, result_dir):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    rng = np.random.default_rng(5)  # every rank builds the same full table
    v, k, m = 65536, 1536, 2
    packed, scales = synth.q4_weight(rng, v, k)
    E, S = T(packed, dev), T(scales, dev)
    head = lmhead.PeerLMHead(E, S, rank, world)
    ok = True
    for step in range(5):
        h = T(np.random.default_rng(100 + step).standard_normal((m, k), dtype=np.float32), dev)
        _, tok = head(h)
        _, ref = kern.lmhead_argmax(E, S, h)
        ok &= bool((tok.cpu() == ref.cpu()).all())
    kern.device_status()
    head.close()
    with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
        f.write("ok" if ok else "mismatch")
    dist.destroy_process_group()


def test_peer_lmhead_across_gpus(tmp_path):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    torch.multiprocessing.spawn(_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert (tmp_path / f"rank{r}").read_text() == "ok", f"rank {r}"
