"""GPU: the decoder glue kernels against the numpy oracle, through the C ABI.

Residual add + RMSNorm (both kernel forms: warp per row for rows of 256 * c
values, CTA per row otherwise) and q/k/v norm + RoPE + KV-cache store, for the
prefill (f16 qkv, positions start_pos + s) and decode (f32 qkv, per-sequence
positions) layouts.  The kernels multiply by one reciprocal per norm instead
of dividing every element, so they sit within a few f32 ulp of the oracle's
x / sqrt(mean(x^2) + eps): tolerance 1e-5 relative on f32 outputs, one f16
ulp on f16 outputs.
"""
import numpy as np
import pytest
import torch

from oracle import decoder as odec
from slang_b200 import _lib
from slang_b200 import kernels as kern

pytestmark = pytest.mark.gpu
EPS = 1e-6


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def rel(a, b):
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


def assert_f16_within_ulp(got16, ref32):
    """f16 outputs within one f16 ulp of the f32 oracle rounded to f16, or --
    for values that come out of cancellation (x + normed y, a c - b s) far
    below the operands -- within a few f32 ulps of the largest output."""
    g = got16.astype(np.float16).view(np.int16).astype(np.int32)
    r = ref32.astype(np.float16).view(np.int16).astype(np.int32)
    # map sign-magnitude bit patterns to a monotone integer line
    g = np.where(g < 0, -0x8000 - g, g)
    r = np.where(r < 0, -0x8000 - r, r)
    d = np.abs(g - r)
    atol = 4 * 2.0 ** -24 * np.abs(ref32).max()
    bad = (d > 1) & (np.abs(got16.astype(np.float32) - ref32) > atol)
    if bad.any():
        i = np.unravel_index(np.argmax(np.where(bad, d, 0)), d.shape)
        raise AssertionError(f"{d[i]} f16 ulps at {i}: got {got16[i]!r}, oracle {ref32[i]!r}")


@pytest.mark.parametrize("m,n", [(1024, 1536), (5, 256), (3, 2048), (7, 1540), (2, 8192)])
@pytest.mark.parametrize("with_y", [True, False])
@pytest.mark.parametrize("ydt", [np.float16, np.float32])
def test_add_rmsnorm_vs_oracle(cuda, m, n, with_y, ydt):
    rng = np.random.default_rng(m * 31 + n)
    x = rng.standard_normal((m, n), dtype=np.float32)
    y = rng.standard_normal((m, n), dtype=np.float32).astype(ydt)
    w_add = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    w_norm = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    # every device buffer stays referenced until the kernel has run
    X, Y, WA, WN = T(x, cuda), T(y, cuda), T(w_add, cuda), T(w_norm, cuda)
    xo = torch.empty_like(X)
    h = torch.empty_like(X)
    h16 = torch.empty((m, n), dtype=torch.float16, device=cuda)
    _lib.call("sb_add_rmsnorm", X.data_ptr(), Y.data_ptr() if with_y else None,
              _lib.SB_F16 if ydt == np.float16 else _lib.SB_F32, WA.data_ptr() if with_y else None,
              WN.data_ptr(), xo.data_ptr(), h.data_ptr(), h16.data_ptr(), m, n, EPS, kern._stream())
    kern.device_status()
    ref_x = x + odec.rms_norm(y.astype(np.float32), w_add, EPS) if with_y else x
    ref_h = odec.rms_norm(ref_x, w_norm, EPS)
    assert rel(xo.cpu().numpy(), ref_x) < 1e-5
    assert rel(h.cpu().numpy(), ref_h) < 1e-5
    assert_f16_within_ulp(h16.cpu().numpy(), ref_h)


def test_add_rmsnorm_in_place(cuda):
    """x_out may alias x (the decoder updates its residual stream in place)."""
    rng = np.random.default_rng(3)
    m, n = 64, 1536
    x = rng.standard_normal((m, n), dtype=np.float32)
    y = rng.standard_normal((m, n), dtype=np.float32).astype(np.float16)
    w = np.ones(n, np.float32)
    X, Y, W = T(x, cuda), T(y, cuda), T(w, cuda)
    h16 = torch.empty((m, n), dtype=torch.float16, device=cuda)
    _lib.call("sb_add_rmsnorm", X.data_ptr(), Y.data_ptr(), _lib.SB_F16, W.data_ptr(), W.data_ptr(), X.data_ptr(),
              None, h16.data_ptr(), m, n, EPS, kern._stream())
    kern.device_status()
    assert rel(X.cpu().numpy(), x + odec.rms_norm(y.astype(np.float32), w, EPS)) < 1e-5


@pytest.mark.parametrize("hd", [64, 128, 256, 512])
@pytest.mark.parametrize("decode", [False, True])
@pytest.mark.parametrize("q_only", [False, True])
def test_qkv_prep_vs_oracle(cuda, hd, decode, q_only):
    """q/k norm + RoPE + cache store; ``q_only`` is a KV-shared layer (no caches:
    only the q heads, rows of n_heads * head_dim)."""
    rng = np.random.default_rng(hd + decode + 7 * q_only)
    nh, S, max_seq = 8, 37, 64
    ld = (nh + (0 if q_only else 2)) * hd
    cos, sin = odec.rope_tables(max_seq, hd, 10000.0, hd // 4)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    if decode:
        qkv = rng.standard_normal((S, ld), dtype=np.float32)
        pos = rng.integers(0, max_seq, S).astype(np.int32)
        start = 0
    else:
        qkv = rng.standard_normal((S, ld), dtype=np.float32).astype(np.float16)
        start = 5
        pos = np.arange(S, dtype=np.int32) + start
    seqs = S if decode else 1
    kc = torch.zeros((seqs, max_seq, hd), device=cuda)
    vc = torch.zeros_like(kc)
    k16 = torch.zeros((seqs, max_seq, hd), dtype=torch.float16, device=cuda)
    v16 = torch.zeros_like(k16)
    q16 = torch.empty((S, nh, hd), dtype=torch.float16, device=cuda)
    q32 = torch.empty((S, nh, hd), device=cuda)
    P, QKV, QN, KN, C, SN = (T(a, cuda) for a in (pos, qkv, qn, kn, cos, sin))
    caches = (None, None, None, None) if q_only else (kc.data_ptr(), vc.data_ptr(), k16.data_ptr(), v16.data_ptr())
    _lib.call("sb_qkv_prep", QKV.data_ptr(), _lib.SB_F32 if decode else _lib.SB_F16, ld, QN.data_ptr(),
              None if q_only else KN.data_ptr(), C.data_ptr(), SN.data_ptr(), P.data_ptr() if decode else None, start,
              S, nh, hd, EPS, q16.data_ptr(), q32.data_ptr(), *caches, max_seq * hd, kern._stream())
    kern.device_status()
    q32n, q16n = q32.cpu().numpy(), q16.cpu().numpy()
    kcn, vcn = kc.cpu().numpy(), vc.cpu().numpy()
    for s in range(S):
        row = qkv[s].astype(np.float32)
        p = int(pos[s])
        q = odec.apply_rope(odec.rms_norm(row[:nh * hd].reshape(nh, hd), qn, EPS), cos[p], sin[p])
        b = s if decode else 0
        assert rel(q32n[s], q) < 1e-5
        assert_f16_within_ulp(q16n[s], q)
        if q_only:
            continue
        k = odec.apply_rope(odec.rms_norm(row[nh * hd:(nh + 1) * hd].reshape(1, hd), kn, EPS), cos[p], sin[p])[0]
        v = odec.rms_norm(row[(nh + 1) * hd:], None, EPS)
        assert rel(kcn[b, p], k) < 1e-5
        assert rel(vcn[b, p], v) < 1e-5
    if q_only:
        assert not kcn.any() and not vcn.any(), "a q-only prep must not touch the caches"


def _attn_decode_ref(q, kc, vc, pos, window=0):
    """softmax(q K^T) V over keys 0..pos of each sequence (the last ``window``
    of them when set), attention scaling 1.0 (the oracle's decode attention,
    oracle/decoder.py OracleDecoder.layer)."""
    out = np.empty_like(q)
    for b in range(q.shape[0]):
        lo = max(0, int(pos[b]) + 1 - window) if window else 0
        s = q[b].astype(np.float64) @ kc[b, lo:pos[b] + 1].astype(np.float64).T
        s -= s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        out[b] = (p @ vc[b, lo:pos[b] + 1].astype(np.float64)).astype(np.float32)
    return out


# head_dim 512 (the checkpoint's full-attention layers) and sliding windows that
# start inside a split, on a split boundary, or cover everything
@pytest.mark.parametrize("m,nh,hd,max_seq,window", [(3, 8, 512, 300, 0), (4, 8, 256, 700, 512), (5, 2, 64, 200, 40),
                                                    (3, 8, 512, 900, 64), (6, 4, 128, 300, 1000)])
def test_attn_decode_window_and_wide_heads(cuda, m, nh, hd, max_seq, window):
    rng = np.random.default_rng(m + nh + hd + max_seq + window)
    q = rng.standard_normal((m, nh, hd), dtype=np.float32) * np.float32(0.1)
    kc = rng.standard_normal((m, max_seq, hd), dtype=np.float32)
    vc = rng.standard_normal((m, max_seq, hd), dtype=np.float32)
    pos = np.minimum(np.array([0, window, max_seq - 1, 32 * 5 + 7, window + 33, max_seq // 3][:m]), max_seq - 1)
    pos = pos.astype(np.int32)
    Q, KC, VC, P = T(q, cuda), T(kc, cuda), T(vc, cuda), T(pos, cuda)
    got = kern.attn_decode(Q, KC, VC, P, window=window).cpu().numpy()
    kern.device_status()
    ref = _attn_decode_ref(q, kc, vc, pos, window)
    assert np.abs(got - ref).max() <= 2e-5 * np.abs(ref).max()


@pytest.mark.parametrize("S,nh,hd,window", [(200, 8, 512, 0), (300, 2, 64, 64), (130, 4, 256, 17), (96, 8, 512, 40)])
def test_attn_prefill_gemm_chain_window_and_wide_heads(cuda, S, nh, hd, window):
    """The GEMM -> windowed causal softmax -> GEMM prefill attention (used for
    sliding-window and head_dim-512 layers) vs float64 with the same mask."""
    rng = np.random.default_rng(S + nh + hd + window)
    q = (rng.standard_normal((S, nh, hd)) * 0.1).astype(np.float16)
    k = rng.standard_normal((S, hd)).astype(np.float16)
    v = rng.standard_normal((S, hd)).astype(np.float16)
    out = torch.empty((S, nh * hd), dtype=torch.float16, device=cuda)
    kern.attn_prefill_gemm(T(q, cuda), T(k, cuda), T(v, cuda), out, S, window=window)
    kern.device_status()
    got = out.float().cpu().numpy().reshape(S, nh, hd)
    sc = np.einsum("shd,td->hst", q.astype(np.float64), k.astype(np.float64))
    i = np.arange(S)
    mask = i[None, :] > i[:, None]
    if window:
        mask |= i[None, :] < i[:, None] + 1 - window
    sc[:, mask] = -np.inf
    sc -= sc.max(axis=-1, keepdims=True)
    p = np.exp(sc)
    p /= p.sum(axis=-1, keepdims=True)
    ref = np.einsum("hst,td->shd", p, v.astype(np.float64))
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < 1e-2, f"max rel err {err:.3e}"


# (sequences, heads, head_dim, max_seq): the last two make the kernel walk
# several 32-key chunks per split (keys per split 96 and 256)
@pytest.mark.parametrize("m,nh,hd,max_seq", [(3, 2, 64, 100), (5, 8, 256, 1100), (4, 16, 128, 70), (2, 1, 64, 40),
                                             (7, 4, 128, 65), (200, 8, 256, 600), (300, 8, 256, 1100)])
def test_attn_decode_vs_oracle(cuda, m, nh, hd, max_seq):
    rng = np.random.default_rng(m * 7 + nh * 3 + hd + max_seq)
    q = rng.standard_normal((m, nh, hd), dtype=np.float32) * np.float32(0.2)
    kc = rng.standard_normal((m, max_seq, hd), dtype=np.float32)
    vc = rng.standard_normal((m, max_seq, hd), dtype=np.float32)
    edge = [0, 30, 31, 32, 33, max_seq - 1, max_seq // 2]
    pos = np.array([edge[i] if i < len(edge) else rng.integers(0, max_seq) for i in range(m)], np.int32)
    pos = np.minimum(pos, max_seq - 1).astype(np.int32)
    Q, KC, VC, P = T(q, cuda), T(kc, cuda), T(vc, cuda), T(pos, cuda)
    ws = torch.empty(_lib.load().sb_attn_decode_workspace_size(m, nh, hd, max_seq) // 4 + 1, dtype=torch.float32,
                     device=cuda)
    out = torch.empty((m, nh, hd), dtype=torch.float32, device=cuda)
    out16 = torch.empty((m, nh, hd), dtype=torch.float16, device=cuda)
    nbytes = ws.numel() * 4
    _lib.call("sb_attn_decode", Q.data_ptr(), KC.data_ptr(), VC.data_ptr(), max_seq * hd, P.data_ptr(), m, nh, hd,
              max_seq, 0, out.data_ptr(), ws.data_ptr(), nbytes, kern._stream())
    _lib.call("sb_attn_decode_f16", Q.data_ptr(), KC.data_ptr(), VC.data_ptr(), max_seq * hd, P.data_ptr(), m, nh, hd,
              max_seq, 0, out16.data_ptr(), ws.data_ptr(), nbytes, kern._stream())
    kern.device_status()
    ref = _attn_decode_ref(q, kc, vc, pos)
    got = out.cpu().numpy()
    assert np.abs(got - ref).max() <= 2e-5 * np.abs(ref).max()
    g16 = out16.cpu().numpy().astype(np.float32)
    assert np.all(np.abs(g16 - got.astype(np.float16).astype(np.float32)) <= np.abs(got) * 2 ** -10 + 1e-7)


def test_attn_decode_wrapper(cuda):
    """kernels.attn_decode (the torch-facing call) on the Gemma-4-E2B head shape."""
    rng = np.random.default_rng(5)
    m, nh, hd, max_seq = 3, 8, 256, 300
    q = rng.standard_normal((m, nh, hd), dtype=np.float32) * np.float32(0.2)
    kc = rng.standard_normal((m, max_seq, hd), dtype=np.float32)
    vc = rng.standard_normal((m, max_seq, hd), dtype=np.float32)
    pos = np.array([0, 150, 299], np.int32)
    Q, KC, VC, P = T(q, cuda), T(kc, cuda), T(vc, cuda), T(pos, cuda)
    got = kern.attn_decode(Q, KC, VC, P).cpu().numpy()
    got16 = kern.attn_decode(Q, KC, VC, P, f16=True)
    kern.device_status()
    ref = _attn_decode_ref(q, kc, vc, pos)
    assert np.abs(got - ref).max() <= 2e-5 * np.abs(ref).max()
    assert got16.dtype == torch.float16
    assert np.abs(got16.cpu().numpy().astype(np.float32) - ref).max() <= 2e-3 * np.abs(ref).max()
