"""GPU parity: every CUDA entry point against the numpy oracle, through the C ABI.

Bars: bit-exact for dequantised weights and argmax token ids; max-rel-err
<= 1e-2 and cosine >= 0.9999 against the fp32 oracle for matmul outputs
(the GEMVs are checked far tighter, GEMV_TOL: they quantise x to 16 bits per
group of 32 and sum the int4 x int16 products exactly).
"""
import numpy as np
import pytest
import torch

from oracle import q4
from slang_b200 import _lib
from slang_b200 import kernels as kern
from slang_b200 import synth
from tests._util import assert_close, max_rel

pytestmark = pytest.mark.gpu

GEMV_TOL = 2e-4  # max-rel vs the fp32 oracle; x rounding is <= 2^-16 of its group max


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


# ------------------------------------------------------------------ dequant
@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("kind", ["group", "row"])
def test_dequant_bit_exact(cuda, golden, bits, kind):
    packed = golden[f"dq{bits}_packed"]
    scales = golden[f"dq{bits}_gscale"] if kind == "group" else golden[f"dq{bits}_rscale"]
    n_out, n_in = packed.shape[0], packed.shape[1] * 8 // bits
    got = kern.dequant_f16(T(packed, cuda), T(scales, cuda), n_in, n_out).cpu().numpy()
    ref = q4.dequant_f16(packed, scales, bits)
    assert np.count_nonzero(got), "dequant wrote nothing"
    np.testing.assert_array_equal(got.view(np.uint16), ref.view(np.uint16))


def test_dequant_model_shape_bit_exact(cuda):
    packed, scales = synth.q4_weight(np.random.default_rng(3), 6144, 1536)
    got = kern.dequant_f16(T(packed, cuda), T(scales, cuda), 1536, 6144).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint16), q4.dequant_f16(packed, scales, 4).view(np.uint16))


def test_dequant_rejects_odd_width(cuda):
    with pytest.raises(ValueError):
        kern.dequant_f16(torch.zeros(10, dtype=torch.uint8, device=cuda),
                      torch.ones(4, 1, dtype=torch.float16, device=cuda), 8, 4)


# ------------------------------------------------------------------ GEMV
@pytest.mark.parametrize("case", [(0, 512, 1536), (1, 2048, 1536), (2, 256, 256)])
def test_gemv_reference_shapes(cuda, golden, case):
    i, n, k = case
    rng = np.random.default_rng(700 + i)
    packed, scales = synth.q4_weight(rng, n, k)
    x = synth.activations(rng, 1, k)
    y = kern.gemv_q4(T(packed, cuda), T(scales, cuda), T(x, cuda)).cpu().numpy()[0]
    ref = golden[f"gemv_{n}x{k}_y"]
    assert max_rel(y, ref) < GEMV_TOL
    assert_close(y, ref)


@pytest.mark.parametrize("n,k", [(6144, 1536), (2560, 1536), (1536, 2048), (1536, 6144), (12288, 1536),
                                 (96, 64), (33, 96), (7, 4096)])
@pytest.mark.parametrize("m", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("xdt", [np.float32, np.float16])
def test_gemv_shapes_batch_dtypes(cuda, n, k, m, xdt):
    rng = np.random.default_rng(n * 7 + k + m)
    packed, scales = synth.q4_weight(rng, n, k)
    x = rng.standard_normal((m, k), dtype=np.float32).astype(xdt)
    y = kern.gemv_q4(T(packed, cuda), T(scales, cuda), T(x, cuda)).cpu().numpy()
    ref = q4.gemv(packed, scales, x)
    assert max_rel(y, ref) < GEMV_TOL, (n, k, m)


def test_gemv_per_row_f32_scales(cuda):
    rng = np.random.default_rng(9)
    packed, _ = synth.q4_weight(rng, 2048, 1536)
    rs = (rng.random((2048, 1)) * 0.01 + 0.001).astype(np.float32)
    x = rng.standard_normal((1, 1536), dtype=np.float32)
    y = kern.gemv_q4(T(packed, cuda), T(rs, cuda), T(x, cuda)).cpu().numpy()
    assert max_rel(y, q4.gemv(packed, rs, x)) < GEMV_TOL


def test_gemv_config1_vs_reference(cuda):
    import os
    path = os.path.join(os.path.dirname(__file__), "golden", "golden_cfg1.npz")
    packed, scales, x = synth.config1(0)
    y = kern.gemv_q4(T(packed, cuda), T(scales, cuda), T(x, cuda)).cpu().numpy()[0]
    ref = np.load(path)["cfg1_y"] if os.path.exists(path) else q4.gemv(packed, scales, x)[0]
    assert max_rel(y, ref) < GEMV_TOL
    assert_close(y, ref)


def test_gemv_ldy_window_untouched(cuda):
    rng = np.random.default_rng(4)
    packed, scales = synth.q4_weight(rng, 100, 256)
    x = rng.standard_normal((2, 256), dtype=np.float32)
    y = torch.full((2, 128), 7.0, device=cuda)
    kern.gemv_q4(T(packed, cuda), T(scales, cuda), T(x, cuda), y=y)
    yn = y.cpu().numpy()
    assert max_rel(yn[:, :100], q4.gemv(packed, scales, x)) < GEMV_TOL
    assert (yn[:, 100:] == 7.0).all(), "padding beyond n was written"


# ------------------------------------------------------------------ lm_head + argmax
def test_argmax_tie_kat(cuda):
    """Two rows with identical weights: the lower index must win (ties -> lowest)."""
    rng = np.random.default_rng(41)
    v, k = 262144, 256
    packed, scales = synth.q4_weight(rng, v, k)
    h = rng.standard_normal((1, k), dtype=np.float32)
    logits = q4.gemv(packed, scales, h)[0]
    top = int(np.argmax(logits))
    # make rows 12345 and 200000 exact copies of a row that beats everything
    big = packed[top].copy()
    for r in (12345, 200000):
        packed[r] = big
        scales[r] = (scales[top].astype(np.float32) * 2).astype(np.float16)
    keys, tok = kern.lmhead_argmax(T(packed, cuda), T(scales, cuda), T(h, cuda))
    assert int(tok.item()) == 12345
    assert int(q4.argmax_first(q4.gemv(packed, scales, h))[0]) == 12345


@pytest.mark.parametrize("m", [1, 2, 4, 5])
def test_lmhead_small_vs_oracle(cuda, m):
    rng = np.random.default_rng(11 + m)
    packed, scales = synth.q4_weight(rng, 50000, 1536)
    h = rng.standard_normal((m, 1536), dtype=np.float32).astype(np.float16)
    logits = torch.empty((m, 50000), device=cuda)
    keys, tok = kern.lmhead_argmax(T(packed, cuda), T(scales, cuda), T(h, cuda), logits=logits)
    ref_tok, ref_val = q4.lmhead_argmax(packed, scales, h)
    np.testing.assert_array_equal(tok.cpu().numpy(), ref_tok)
    assert max_rel(logits.cpu().numpy(), q4.gemv(packed, scales, h)) < GEMV_TOL
    np.testing.assert_array_equal(q4.unpack_key_index(keys.cpu().numpy().view(np.uint64)), ref_tok)


def test_lmhead_row_offset_and_shard_combine(cuda):
    """Shards with row offsets combine by an integer MAX over keys."""
    rng = np.random.default_rng(5)
    v, k = 65536, 1536
    packed, scales = synth.q4_weight(rng, v, k)
    h = rng.standard_normal((2, k), dtype=np.float32)
    keys = []
    for s in range(4):
        lo, hi = s * v // 4, (s + 1) * v // 4
        kk, _ = kern.lmhead_argmax(T(packed[lo:hi], cuda), T(scales[lo:hi], cuda), T(h, cuda), row_offset=lo,
                                want_tokens=False)
        keys.append(kk.cpu().numpy().view(np.uint64))
    best = np.max(np.stack(keys), axis=0)
    ref_tok, _ = q4.lmhead_argmax(packed, scales, h)
    np.testing.assert_array_equal(q4.unpack_key_index(best), ref_tok)


def test_lmhead_config3_vs_reference(cuda):
    import os
    path = os.path.join(os.path.dirname(__file__), "golden", "golden_cfg3.npz")
    if not os.path.exists(path):
        pytest.skip("config-3 fixture absent")
    g = np.load(path)
    packed, scales, h = synth.config3()
    logits = torch.empty((1, packed.shape[0]), device=cuda)
    _, tok = kern.lmhead_argmax(T(packed, cuda), T(scales, cuda), T(h, cuda), logits=logits)
    assert int(tok.item()) == int(g["cfg3_token"])
    got = logits.cpu().numpy()[0]
    assert max_rel(got[:4096], g["cfg3_logits_head"]) < GEMV_TOL
    np.testing.assert_allclose(got[g["cfg3_top8_idx"]], g["cfg3_top8_val"], rtol=GEMV_TOL, atol=1e-3)


# ------------------------------------------------------------------ tcgen05 GEMMs
SHAPES = [(32, 32, 16), (16, 1536, 1536), (64, 256, 512), (17, 33, 48), (5, 7, 16)]


def _ref_inputs(M, N, K):
    rng = np.random.default_rng(0)  # the reference test's _inputs(M, N, K, seed=0)
    return rng.standard_normal((M, K)).astype(np.float16), rng.standard_normal((N, K)).astype(np.float16)


def _pad8(x):
    return (x + 7) // 8 * 8


def _gemm_f16(cuda, a, b, alpha=1.0, tr=True):
    """Stage operands with row strides padded to multiples of 8 (TMA rule)."""
    M, K = a.shape
    N = b.shape[0] if tr else b.shape[1]
    lda = _pad8(K)
    ldb = _pad8(b.shape[1])
    A = torch.zeros((M, lda), dtype=torch.float16, device=cuda)
    A[:, :K] = T(a, cuda)
    B = torch.zeros((b.shape[0], ldb), dtype=torch.float16, device=cuda)
    B[:, :b.shape[1]] = T(b, cuda)
    C = torch.zeros((M, N), dtype=torch.float16, device=cuda)
    kern.gemm(A, B, C, M, N, K, alpha=alpha, tr=tr, acols=lda, bcols=ldb)
    return C.cpu().numpy()


@pytest.mark.parametrize("shape", SHAPES)
def test_gemm_f16_reference_shapes(cuda, golden, shape):
    M, N, K = shape
    a, b = _ref_inputs(M, N, K)
    c = _gemm_f16(cuda, a, b)
    assert max_rel(c, golden[f"gemm_{M}x{N}x{K}_c64"]) < 3e-3  # tests/test_gemm_dsl.py:124-129


def test_gemm_f16_alpha(cuda, golden):
    a, b = _ref_inputs(32, 32, 16)
    assert max_rel(_gemm_f16(cuda, a, b, alpha=0.375), golden["gemm_alpha_c64"]) < 3e-3


@pytest.mark.parametrize("shape", [(64, 48, 32), (17, 33, 48), (300, 520, 200), (1024, 256, 1024)])
def test_gemm_f16_tr0(cuda, shape):
    M, N, K = shape
    rng = np.random.default_rng(1)
    a = rng.standard_normal((M, K)).astype(np.float16)
    bkn = rng.standard_normal((K, N)).astype(np.float16)
    c = _gemm_f16(cuda, a, bkn, tr=False)
    assert max_rel(c, q4.gemm_f64(a, bkn, tr=False)) < 3e-3


def test_gemm_f16_strided_window(cuda):
    """ldc > N: only the window is written (tests/test_gemm_dsl.py:205-239)."""
    M, N, K, ldc = 40, 24, 64, 40
    rng = np.random.default_rng(2)
    a = rng.standard_normal((M, K)).astype(np.float16)
    b = rng.standard_normal((N, K)).astype(np.float16)
    A, B = T(a, cuda), T(b, cuda)
    C = torch.full((M, ldc), 5.0, dtype=torch.float16, device=cuda)
    kern.gemm(A, B, C, M, N, K, ccols=ldc)
    cn = C.cpu().numpy()
    assert max_rel(cn[:, :N], q4.gemm_f64(a, b)) < 3e-3
    assert (cn[:, N:] == 5.0).all(), "padding beyond N was written"


@pytest.mark.parametrize("M", [128, 1024, 17, 300])
@pytest.mark.parametrize("name", ["gate", "down", "o", "k"])
def test_gemm_q4_vs_oracle(cuda, M, name):
    N, Kd = synth.E2B_SHAPES[name]
    rng = np.random.default_rng(M + Kd)
    packed, scales = synth.q4_weight(rng, N, Kd)
    a = synth.activations(rng, M, Kd)
    c = kern.gemm_q4(T(a, cuda), T(packed, cuda), T(scales, cuda)).cpu().numpy()
    ref = q4.gemm_f64(a, q4.dequant_f16(packed, scales, 4))
    assert_close(c, ref, what=f"gemm_q4 {name} M={M}")
    # and the fp32 oracle of the unrounded weight (the reference's numpy path)
    assert_close(c, a.astype(np.float32) @ q4.dequant_f32(packed, scales, 4).T, what="vs f32 oracle")


def test_gemm_q4_alpha_and_f32_row_scales(cuda):
    rng = np.random.default_rng(8)
    N, Kd, M = 512, 1536, 256
    packed, _ = synth.q4_weight(rng, N, Kd)
    rs = (rng.random((N, 1)) * 0.01 + 0.001).astype(np.float32)
    a = synth.activations(rng, M, Kd)
    c = kern.gemm_q4(T(a, cuda), T(packed, cuda), T(rs, cuda), alpha=0.5).cpu().numpy()
    assert_close(c, 0.5 * q4.gemm_f64(a, q4.dequant_f16(packed, rs, 4)))


def test_gemm_q4_matches_dequant_then_gemm(cuda):
    """The fused kernel equals the reference's two-step _dq -> _gemm within f32 rounding."""
    rng = np.random.default_rng(12)
    N, Kd, M = 6144, 1536, 256
    packed, scales = synth.q4_weight(rng, N, Kd)
    a = synth.activations(rng, M, Kd)
    A, P, S = T(a, cuda), T(packed, cuda), T(scales, cuda)
    fused = kern.gemm_q4(A, P, S)
    W = kern.dequant_f16(P, S, Kd, N)
    C = torch.empty((M, N), dtype=torch.float16, device=cuda)
    kern.gemm(A, W, C, M, N, Kd)
    f, c = fused.float().cpu().numpy(), C.float().cpu().numpy()
    assert np.abs(f - c).max() <= 2 * np.abs(c).max() * 2 ** -11


# (M, N, K): no split; a 6-split cluster reduced in distributed shared memory;
# 16 splits through workspace partials and the finalize kernel
@pytest.mark.parametrize("M,N,K", [(1024, 12288, 1536), (256, 512, 1536), (256, 256, 6144), (37, 512, 1536),
                                   (8, 12288, 1536), (32, 512, 6144), (3, 2048, 2048)])
def test_gemm_q4_geglu_equals_gemm_then_geglu(cuda, M, N, K):
    """GEGLU in the GEMM epilogue is bit-for-bit sb_gemm_q4 followed by sb_geglu."""
    rng = np.random.default_rng(M + N + K)
    packed, scales = synth.q4_weight(rng, N, K)
    a = synth.activations(rng, M, K)
    A, P, S = T(a, cuda), T(packed, cuda), T(scales, cuda)
    fused = kern.gemm_q4(A, P, S, geglu=True)
    gu = kern.gemm_q4(A, P, S)
    chain = torch.empty((M, N // 2), dtype=torch.float16, device=cuda)
    _lib.call("sb_geglu", gu.data_ptr(), _lib.SB_F16, M, N // 2, None, chain.data_ptr(), kern._stream())
    kern.device_status()
    f, c = fused.cpu().numpy(), chain.cpu().numpy()
    assert fused.shape == (M, N // 2)
    np.testing.assert_array_equal(f, c)
    # and against the oracle: GEGLU of the f64 GEMM of the dequantised weight
    ref = q4.gemm_f64(a, q4.dequant_f16(packed, scales, 4)).astype(np.float16).astype(np.float64)
    g, u = ref[:, 0::2], ref[:, 1::2]
    assert_close(f.astype(np.float64), 0.5 * g * (1 + np.tanh(0.7978845608028654 * (g + 0.044715 * g ** 3))) * u,
                 what=f"geglu M={M} N={N} K={K}")


@pytest.mark.parametrize("M,N,geglu", [(1000, 12160, False), (2048, 6144, False), (1000, 12288, True),
                                        (777, 9216, True)])
def test_gemm_q4_persistent_tiles(cuda, M, N, geglu):
    """More CTA-pair tiles than the device holds at once, with a ragged last
    token tile and a last weight pair half past N."""
    K = 1536
    rng = np.random.default_rng(M * 7 + N)
    packed, scales = synth.q4_weight(rng, N, K)
    a = synth.activations(rng, M, K)
    A, P, S = T(a, cuda), T(packed, cuda), T(scales, cuda)
    gu = kern.gemm_q4(A, P, S)
    ref = q4.gemm_f64(a, q4.dequant_f16(packed, scales, 4))
    assert_close(gu.cpu().numpy(), ref, what=f"persistent gemm_q4 M={M} N={N}")
    if geglu:
        fused = kern.gemm_q4(A, P, S, geglu=True)
        chain = torch.empty((M, N // 2), dtype=torch.float16, device=cuda)
        _lib.call("sb_geglu", gu.data_ptr(), _lib.SB_F16, M, N // 2, None, chain.data_ptr(), kern._stream())
        kern.device_status()
        np.testing.assert_array_equal(fused.cpu().numpy(), chain.cpu().numpy())


def test_gemm_q4_workspace_only_beyond_cluster_splits(cuda):
    """Split-K within a cluster needs no workspace; only more than 8 splits do."""
    assert kern.gemm_q4_workspace_size(1024, 1536, 2048) == 0  # o: 3 splits in a cluster
    assert kern.gemm_q4_workspace_size(1024, 1536, 6144) == 0  # down
    assert kern.gemm_q4_workspace_size(256, 256, 6144) > 0  # 16 splits


def test_gemm_q4_kernels_per_call(cuda):
    """sb_gemm_q4_kernels: a split-K finalize launch follows exactly when the
    workspace holds partial planes."""
    for M, N, K in ((1024, 12288, 1536), (1024, 1536, 2048), (256, 256, 6144), (8, 12288, 1536), (32, 512, 6144)):
        assert kern.gemm_q4_kernels(M, N, K) == (2 if kern.gemm_q4_workspace_size(M, N, K) else 1)


def test_gemm_q4_trace_stamps_are_ordered(cuda):
    """The profiling hook: every CTA of a traced launch stamps its phases in order."""
    rng = np.random.default_rng(3)
    M, N, K = 512, 2560, 1536
    packed, scales = synth.q4_weight(rng, N, K)
    a = synth.activations(rng, M, K)
    A, P, S = T(a, cuda), T(packed, cuda), T(scales, cuda)
    buf = torch.zeros(4096 * 16, dtype=torch.int64, device=cuda)
    _lib.call("sb_gemm_q4_trace", buf.data_ptr(), buf.numel() * 8)
    try:
        c = kern.gemm_q4(A, P, S)
    finally:
        _lib.call("sb_gemm_q4_trace", None, 0)
    kern.device_status()
    x = buf.view(4096, 16).cpu().numpy()
    x = x[x[:, 1] > 0]
    tiles = 2 * ((N + 255) // 256) * ((M + 255) // 256)  # CTAs of one K split
    assert len(x) >= tiles and len(x) % tiles == 0
    for row in x:
        assert row[1] <= row[2] <= row[3] and row[2] <= row[4] <= row[8] <= row[9] <= row[11]
        if row[6]:  # the pair's MMA-issuing CTA
            assert row[3] <= row[6] <= row[7] <= row[8]
    assert_close(c.cpu().numpy(), q4.gemm_f64(a, q4.dequant_f16(packed, scales, 4)))


def test_no_device_timeouts(cuda):
    torch.cuda.synchronize()
    kern.device_status()


# ------------------------------------------------------------------ lm_head argmax on the tcgen05 GEMM
@pytest.mark.parametrize("m", [1, 37, 256])
def test_gemm_q4_argmax_vs_oracle(cuda, m):
    """Batched lm_head + greedy argmax in the GEMM epilogue: tokens equal the
    oracle's argmax of the f16-activation GEMM, keys carry the max value."""
    rng = np.random.default_rng(900 + m)
    v, k = 50000, 1536
    packed, scales = synth.q4_weight(rng, v, k)
    h = synth.activations(rng, m, k)
    keys, tok = kern.gemm_q4_argmax(T(h, cuda), T(packed, cuda), T(scales, cuda))
    logits = q4.gemm_f64(h, q4.dequant_f16(packed, scales, 4))
    np.testing.assert_array_equal(tok.cpu().numpy(), np.argmax(logits, axis=1))
    np.testing.assert_array_equal(q4.unpack_key_index(keys.cpu().numpy().view(np.uint64)), np.argmax(logits, axis=1))


def test_gemm_q4_argmax_tie_and_shards(cuda):
    """Ties go to the lowest index; shards with row offsets combine by an integer MAX."""
    rng = np.random.default_rng(77)
    v, k, m = 8192, 1536, 5
    packed, scales = synth.q4_weight(rng, v, k)
    h = synth.activations(rng, m, k)
    top = np.argmax(q4.gemm_f64(h, q4.dequant_f16(packed, scales, 4)), axis=1)
    # copy row top[0] (scaled up so it wins) to a lower and a higher index
    src = int(top[0])
    for r in (100, 7000):
        packed[r] = packed[src]
        scales[r] = (scales[src].astype(np.float32) * 4).astype(np.float16)
    keys, tok = kern.gemm_q4_argmax(T(h, cuda), T(packed, cuda), T(scales, cuda))
    assert int(tok[0].item()) == 100
    ref = np.argmax(q4.gemm_f64(h, q4.dequant_f16(packed, scales, 4)), axis=1)
    np.testing.assert_array_equal(tok.cpu().numpy(), ref)
    parts = []
    for lo, hi in ((0, 4096), (4096, 8192)):
        kk, _ = kern.gemm_q4_argmax(T(h, cuda), T(packed[lo:hi], cuda), T(scales[lo:hi], cuda), row_offset=lo,
                                    want_tokens=False)
        parts.append(kk.cpu().numpy().view(np.uint64))
    np.testing.assert_array_equal(q4.unpack_key_index(np.maximum(parts[0], parts[1])), ref)


# short batches (batched decode): a pair's token tile shrinks to 64 or 128 tokens
@pytest.mark.parametrize("M", [1, 8, 33, 64, 65, 100, 128])
@pytest.mark.parametrize("N,K", [(2560, 1536), (1536, 6144), (12288, 1536)])
def test_gemm_q4_short_batches(cuda, M, N, K):
    rng = np.random.default_rng(M * 13 + N + K)
    packed, scales = synth.q4_weight(rng, N, K)
    a = synth.activations(rng, M, K)
    c = kern.gemm_q4(T(a, cuda), T(packed, cuda), T(scales, cuda)).cpu().numpy()
    kern.device_status()
    assert_close(c, q4.gemm_f64(a, q4.dequant_f16(packed, scales, 4)), what=f"gemm_q4 M={M} N={N} K={K}")
