"""GPU parity of the 2-bit decode GEMV and lm_head (the checkpoint's 2-bit MLP
weights of layers 15+ and its 2-bit lm_head; gemma4/qat_loader.py:33-38, 52-61)
against the numpy oracle, through the C ABI.

The codes are used exactly and x is rounded to 16-bit integers per group of 32,
as in the 4-bit GEMV, so the same tolerance applies; argmax tokens are
bit-exact.
"""
import numpy as np
import pytest
import torch

from oracle import q4
from slang_b200 import _lib
from slang_b200 import kernels as kern
from slang_b200 import synth
from tests._util import max_rel

pytestmark = pytest.mark.gpu

GEMV_TOL = 2e-4


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


# model shapes (the real checkpoint's wide MLP down has K = 12288) and ragged ones
@pytest.mark.parametrize("n,k", [(6144, 1536), (12288, 1536), (1536, 6144), (1536, 12288), (2560, 1536),
                                 (96, 64), (33, 128), (7, 4096)])
@pytest.mark.parametrize("m", [1, 2, 3, 8])
@pytest.mark.parametrize("xdt", [np.float32, np.float16])
def test_gemv_q2_vs_oracle(cuda, n, k, m, xdt):
    rng = np.random.default_rng(n * 5 + k + m)
    packed, scales = synth.q2_weight(rng, n, k)
    x = rng.standard_normal((m, k), dtype=np.float32).astype(xdt)
    y = kern.gemv_q4(T(packed, cuda), T(scales, cuda), T(x, cuda), bits=2).cpu().numpy()
    kern.device_status()
    ref = q4.gemv(packed, scales, x, bits=2)
    assert max_rel(y, ref) < GEMV_TOL, (n, k, m)


def test_gemv_q2_checkpoint_row_scales(cuda):
    """The checkpoint's format: per-output-row f32 weight_scale [n, 1]."""
    rng = np.random.default_rng(21)
    packed, _ = synth.q2_weight(rng, 12288, 1536)
    rs = (rng.random((12288, 1)) * 0.02 + 0.001).astype(np.float32)
    x = rng.standard_normal((1, 1536), dtype=np.float32)
    y = kern.gemv_q4(T(packed, cuda), T(rs, cuda), T(x, cuda), bits=2).cpu().numpy()
    kern.device_status()
    assert max_rel(y, q4.gemv(packed, rs, x, bits=2)) < GEMV_TOL


def test_gemv_q2_rejects_unaligned_rows(cuda):
    rng = np.random.default_rng(2)
    packed, scales = synth.q2_weight(rng, 16, 96)  # 24-byte rows
    x = rng.standard_normal((1, 96), dtype=np.float32)
    with pytest.raises(_lib.SlangError):
        kern.gemv_q4(T(packed, cuda), T(scales, cuda), T(x, cuda), bits=2)


@pytest.mark.parametrize("m", [1, 3])
def test_lmhead_q2_vs_oracle(cuda, m):
    rng = np.random.default_rng(31 + m)
    packed, scales = synth.q2_weight(rng, 50000, 1536)
    h = rng.standard_normal((m, 1536), dtype=np.float32).astype(np.float16)
    logits = torch.empty((m, 50000), device=cuda)
    keys, tok = kern.lmhead_argmax(T(packed, cuda), T(scales, cuda), T(h, cuda), logits=logits, bits=2)
    kern.device_status()
    ref_tok, _ = q4.lmhead_argmax(packed, scales, h, bits=2)
    np.testing.assert_array_equal(tok.cpu().numpy(), ref_tok)
    assert max_rel(logits.cpu().numpy(), q4.gemv(packed, scales, h, bits=2)) < GEMV_TOL
    np.testing.assert_array_equal(q4.unpack_key_index(keys.cpu().numpy().view(np.uint64)), ref_tok)


def test_lmhead_q2_tie_kat(cuda):
    """Two rows identical to one that beats every other: the lower index wins."""
    rng = np.random.default_rng(43)
    v, k = 262144, 1536
    packed, scales = synth.q2_weight(rng, v, k)
    h = rng.standard_normal((1, k), dtype=np.float32)
    top = int(np.argmax(q4.gemv(packed, scales, h, bits=2)[0]))
    for r in (777, 250000):
        packed[r] = packed[top]
        scales[r] = (scales[top].astype(np.float32) * 2).astype(np.float16)
    _, tok = kern.lmhead_argmax(T(packed, cuda), T(scales, cuda), T(h, cuda), bits=2)
    kern.device_status()
    assert int(tok.item()) == 777
    assert int(q4.argmax_first(q4.gemv(packed, scales, h, bits=2))[0]) == 777


# ------------------------------------------------------------------ fused 2-bit GEMM
# (M, N, K): the pair kernel without and with split-K; the real wide-MLP down
# (K = 12288, splits through the workspace); a ragged one-CTA case
@pytest.mark.parametrize("M,N,K", [(1024, 6144, 1536), (256, 1536, 12288), (1024, 1536, 6144), (37, 512, 1536),
                                   (200, 128, 1536)])
def test_gemm_q2_vs_oracle(cuda, M, N, K):
    from tests._util import assert_close
    rng = np.random.default_rng(M + N + K)
    packed, scales = synth.q2_weight(rng, N, K)
    a = synth.activations(rng, M, K)
    c = kern.gemm_q4(T(a, cuda), T(packed, cuda), T(scales, cuda), bits=2).cpu().numpy()
    kern.device_status()
    assert_close(c, q4.gemm_f64(a, q4.dequant_f16(packed, scales, 2)), what=f"gemm_q2 M={M} N={N} K={K}")
    assert_close(c, a.astype(np.float32) @ q4.dequant_f32(packed, scales, 2).T, what="vs f32 oracle")


def test_gemm_q2_checkpoint_row_scales_and_dequant_chain(cuda):
    """Per-row f32 scales (the checkpoint's weight_scale); the fused kernel equals
    the reference's two-step _dq (bits = 2) -> _gemm within f32 rounding."""
    rng = np.random.default_rng(14)
    N, K, M = 2048, 1536, 256
    packed, _ = synth.q2_weight(rng, N, K)
    rs = (rng.random((N, 1)) * 0.02 + 0.001).astype(np.float32)
    a = synth.activations(rng, M, K)
    A, P, S = T(a, cuda), T(packed, cuda), T(rs, cuda)
    fused = kern.gemm_q4(A, P, S, bits=2)
    W = kern.dequant_f16(P, S, K, N, bits=2)
    C = torch.empty((M, N), dtype=torch.float16, device=cuda)
    kern.gemm(A, W, C, M, N, K)
    kern.device_status()
    np.testing.assert_array_equal(W.cpu().numpy().view(np.uint16), q4.dequant_f16(packed, rs, 2).view(np.uint16))
    f, c = fused.float().cpu().numpy(), C.float().cpu().numpy()
    assert np.abs(f - c).max() <= 2 * np.abs(c).max() * 2 ** -11


@pytest.mark.parametrize("M,N,K", [(1024, 12288, 1536), (256, 256, 12288)])
def test_gemm_q2_geglu_equals_gemm_then_geglu(cuda, M, N, K):
    rng = np.random.default_rng(M * 3 + N + K)
    packed, scales = synth.q2_weight(rng, N, K)
    a = synth.activations(rng, M, K)
    A, P, S = T(a, cuda), T(packed, cuda), T(scales, cuda)
    fused = kern.gemm_q4(A, P, S, geglu=True, bits=2)
    gu = kern.gemm_q4(A, P, S, bits=2)
    chain = torch.empty((M, N // 2), dtype=torch.float16, device=cuda)
    _lib.call("sb_geglu", gu.data_ptr(), _lib.SB_F16, M, N // 2, None, chain.data_ptr(), kern._stream())
    kern.device_status()
    np.testing.assert_array_equal(fused.cpu().numpy(), chain.cpu().numpy())
