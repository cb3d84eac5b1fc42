"""GPU: fused causal prefill attention (sb_attn_prefill).

Against a float64 numpy restatement of the reference's prompt attention
(gemma4_150/prefill_gpu.py:259-314: scores = q k^T unscaled, causal mask by
token, softmax, P v) on the same f16 inputs, and against the library's own
three-kernel chain (sb_gemm_f16_f32out -> sb_softmax_causal -> sb_gemm_f16)
at the full 1024-token prompt.  Tolerances are the prefill GEMM bar:
max-rel-err <= 1e-2 of the output's max and cosine >= 0.9999.
"""
import numpy as np
import pytest
import torch

from slang_b200 import _lib
from slang_b200 import kernels as kern

from tests._util import assert_close

pytestmark = pytest.mark.gpu
HD = 256


def _inputs(S, nh, seed, scale=1.0, hd=HD):
    g = torch.Generator().manual_seed(seed)
    # RMS-normalised rows, as qkv_prep produces them (|q . k| up to ~ hd * scale^2)
    q = torch.randn((S, nh, hd), generator=g)
    k = torch.randn((S, hd), generator=g)
    v = torch.randn((S, hd), generator=g)
    q = q / q.pow(2).mean(-1, keepdim=True).sqrt() * scale
    k = k / k.pow(2).mean(-1, keepdim=True).sqrt() * scale
    return q.half(), k.half(), v.half()


def _reference(q, k, v):
    """float64: out[t, h] = softmax_{j <= t}(q[t, h] . k[j]) . v"""
    qn, kn, vn = (x.float().numpy().astype(np.float64) for x in (q, k, v))
    S, nh, _ = qn.shape
    out = np.zeros_like(qn)
    for t in range(S):
        s = qn[t] @ kn[:t + 1].T  # [nh, t + 1]
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[t] = p @ vn[:t + 1]
    return out


@pytest.mark.parametrize("S,nh,scale,hd", [(1, 8, 1.0, 256), (37, 8, 1.0, 256), (200, 8, 0.5, 256),
                                           (130, 3, 1.0, 256), (300, 2, 0.7, 256), (70, 2, 1.0, 64),
                                           (150, 4, 1.0, 128)])
def test_attn_prefill_vs_reference(cuda, S, nh, scale, hd):
    q, k, v = _inputs(S, nh, seed=S * 10 + nh, scale=scale, hd=hd)
    ref = _reference(q, k, v)
    for split in (False, True):
        out = kern.attn_prefill(q.to(cuda), k.to(cuda), v.to(cuda), split=split)
        kern.device_status()
        assert_close(out.float().cpu().numpy(), ref, what=f"attn_prefill S={S} nh={nh} hd={hd} split={split}")


def test_attn_prefill_split_merges_key_chunks(cuda):
    """A long prompt splits each late query tile's keys over several CTAs; the
    merged result equals the unsplit kernel's within f32 rounding."""
    S, nh = 2048, 8
    assert _lib.load().sb_attn_prefill_workspace_size(S, nh, HD) > 0, "expected a split at 2048 tokens"
    q, k, v = (x.to(cuda) for x in _inputs(S, nh, seed=9, scale=0.8))
    whole = kern.attn_prefill(q, k, v, split=False).float()
    split = kern.attn_prefill(q, k, v, split=True).float()
    kern.device_status()
    assert_close(split.cpu().numpy(), whole.cpu().numpy(), what="split vs unsplit")
    # last two tokens against float64 (they see every key)
    qn, kn, vn = (x.float().cpu().numpy().astype(np.float64) for x in (q[-2:], k, v))
    for i, t in enumerate((S - 2, S - 1)):
        s = qn[i] @ kn[:t + 1].T
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        assert_close(split[t].cpu().numpy(), p @ vn[:t + 1], what=f"token {t}")


def test_attn_prefill_matches_three_kernel_chain(cuda):
    """1024-token prompt, 8 heads: fused kernel vs scores GEMM -> softmax -> PV."""
    S, nh = 1024, 8
    q, k, v = (x.to(cuda) for x in _inputs(S, nh, seed=5))
    fused = kern.attn_prefill(q, k, v)
    ldp = S
    scores = torch.empty((S * nh, ldp), dtype=torch.float32, device=cuda)
    p16 = torch.empty((S * nh, ldp), dtype=torch.float16, device=cuda)
    chain = torch.empty((S * nh, HD), dtype=torch.float16, device=cuda)
    s = kern._stream()
    _lib.call("sb_gemm_f16_f32out", q.data_ptr(), k.data_ptr(), scores.data_ptr(), S * nh, S, HD, 1.0, 1, HD, HD,
              ldp, s)
    _lib.call("sb_softmax_causal", scores.data_ptr(), ldp, S * nh, nh, 0, S, 0, p16.data_ptr(), ldp, s)
    _lib.call("sb_gemm_f16", p16.data_ptr(), v.data_ptr(), chain.data_ptr(), S * nh, HD, S, 1.0, 0, ldp, HD, HD, s)
    kern.device_status()
    assert_close(fused.float().reshape(S * nh, HD).cpu().numpy(), chain.float().cpu().numpy(),
                 what="fused vs three-kernel chain")
    # spot rows against float64 (first, middle and last tokens)
    ref_rows = _reference(q[:3].cpu(), k[:3].cpu(), v[:3].cpu())
    assert_close(fused[:3].float().cpu().numpy(), ref_rows, what="first tokens")


def test_attn_prefill_rejects_bad_head_dim(cuda):
    q = torch.zeros((4, 2, 96), dtype=torch.float16, device=cuda)
    k = torch.zeros((4, 96), dtype=torch.float16, device=cuda)
    with pytest.raises(_lib.SlangError):
        kern.attn_prefill(q, k, k)
