"""GPU: a cross-GPU wait that runs out reports a timeout and leaves the GPU usable.

The vocabulary-sharded lm_head's exchange in peer memory waits, bounded, until
every rank's step-tagged keys are in its mailbox.  Here a two-rank exchange is opened
on one GPU with only rank 0 calling: the second mailbox stands for a rank that
never arrives (a flag nothing sets).  With the wait limit set to 50 ms the
exchange kernel must return, ``sb_device_status`` must report SB_ERR_TIMEOUT
once, and the context must keep working.  No fault, trap or hang is involved:
the failure is made on the host side by the missing rank.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from oracle import q4
from slang_b200 import _lib, kernels, synth

pytestmark = pytest.mark.gpu


def _mailbox(lib):
    size = int(lib.sb_peer_mailbox_size())
    ptr, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
    _lib.call("sb_peer_buffer_create", size, ctypes.byref(ptr), handle)
    return ptr.value


def test_missing_rank_times_out_and_gpu_stays_usable(cuda):
    lib = _lib.load()
    kernels.device_status()  # start from a clean error word
    rng = np.random.default_rng(17)
    v, k = 4096, 1536
    packed, scales = synth.q4_weight(rng, v, k)
    h = synth.activations(rng, 1, k, dtype=np.float32)
    W, S, Hd = (torch.from_numpy(a).to(cuda) for a in (packed, scales, h))
    own, absent = _mailbox(lib), _mailbox(lib)
    peers = torch.tensor([own, absent], dtype=torch.int64, device=cuda)
    keys = torch.zeros(1, dtype=torch.int64, device=cuda)
    toks = torch.zeros(1, dtype=torch.int32, device=cuda)
    try:
        _lib.call("sb_peer_set_wait_limit_ns", 50_000_000)
        t0 = time.perf_counter()
        # rank 0 of 2 runs its half of the rows; rank 1 never calls
        _lib.call("sb_lmhead_argmax_peer", W.data_ptr(), S.data_ptr(), _lib.SB_F16, 32, Hd.data_ptr(), _lib.SB_F32, 1,
                  v // 2, k, 0, peers.data_ptr(), 2, own, keys.data_ptr(), toks.data_ptr(),
                  torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        rc = lib.sb_device_status(torch.cuda.current_stream().cuda_stream)
        assert rc == _lib.SB_ERR_TIMEOUT, f"expected SB_ERR_TIMEOUT, got {rc}"
        assert 0.04 <= waited < 1.9, f"the exchange returned after {waited:.3f} s (limit 0.05 s)"
        assert int(keys.item()) == 0, "a timed-out exchange must not report a token"
        # the status was consumed, and the context still runs kernels correctly
        assert lib.sb_device_status(torch.cuda.current_stream().cuda_stream) == _lib.SB_OK
        _, tok = kernels.lmhead_argmax(W, S, Hd)
        assert int(tok.item()) == int(q4.lmhead_argmax(packed, scales, h)[0][0])
    finally:
        _lib.call("sb_peer_set_wait_limit_ns", 0)
        torch.cuda.synchronize()
        _lib.call("sb_peer_buffer_free", own)
        _lib.call("sb_peer_buffer_free", absent)
