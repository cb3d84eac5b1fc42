"""CPU: the numpy oracle against vectors produced by the reference's own code.

Fixtures come from tests/golden/make_golden.py, which imports the reference's
gemma4.qat_loader / gemma4.reference / tests/test_gemm_dsl.py and runs them on
seeded inputs.
"""
import os

import numpy as np
import pytest

from oracle import decoder, q4
from slang_b200 import synth
from tests._util import max_rel

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_unpack_kats(golden):
    # tests/test_gemma4_qat_loader.py:18-30 of the reference
    np.testing.assert_array_equal(q4.unpack_signed(golden["kat_int4_in"], 4), golden["kat_int4_out"])
    np.testing.assert_array_equal(q4.unpack_signed(golden["kat_int4_in"], 4), [-8, 0, -8, 7, 0, -8, 7, -1])
    np.testing.assert_array_equal(q4.unpack_signed(golden["kat_int2_in"], 2), [-2, -1, 0, 1])
    np.testing.assert_array_equal(q4.unpack_signed(golden["rand_bytes"], 4), golden["rand_int4"])
    np.testing.assert_array_equal(q4.unpack_signed(golden["rand_bytes"], 2), golden["rand_int2"])


def test_unpack_shapes():
    assert q4.unpack_signed(np.zeros((5, 4), np.uint8), 4).shape == (5, 8)
    assert q4.unpack_signed(np.zeros((5, 4), np.uint8), 2).shape == (5, 16)


def test_pack_roundtrip():
    ints = np.random.default_rng(0).integers(-8, 8, (3, 64))
    np.testing.assert_array_equal(q4.unpack_signed(q4.pack_int4(ints), 4), ints)


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("kind", ["group", "row"])
def test_dequant_f32_matches_reference(golden, bits, kind):
    scales = golden[f"dq{bits}_gscale"] if kind == "group" else golden[f"dq{bits}_rscale"]
    got = q4.dequant_f32(golden[f"dq{bits}_packed"], scales, bits)
    np.testing.assert_array_equal(got, golden[f"dq{bits}_f32_{kind}"])


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_dequant_f16_exact_vs_float64(golden, bits):
    """With f16 scales the f32 product is exact, so dq_f16 equals the float64
    reconstruction rounded to f16 (the reference's check, test_dequant.py:45-51)."""
    packed, scales = golden[f"dq{bits}_packed"], golden[f"dq{bits}_gscale"]
    got = q4.dequant_f16(packed, scales, bits)
    codes = q4.unpack_codes(packed, bits).astype(np.float64) - q4.ZERO_POINT[bits]
    ref = (codes * q4.expand_scales(scales, codes.shape[-1]).astype(np.float64)).astype(np.float16)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("case", [(0, 512, 1536), (1, 2048, 1536), (2, 256, 256)])
def test_gemv_matches_reference(golden, case):
    i, n, k = case
    rng = np.random.default_rng(700 + i)
    packed, scales = synth.q4_weight(rng, n, k)
    x = synth.activations(rng, 1, k)
    y = q4.gemv(packed, scales, x)[0]
    assert max_rel(y, golden[f"gemv_{n}x{k}_y"]) < 1e-5


@pytest.mark.parametrize("shape", [(32, 32, 16), (16, 1536, 1536), (64, 256, 512), (17, 33, 48), (5, 7, 16)])
def test_gemm_oracle_within_reference_tolerance(golden, shape):
    M, N, K = shape
    rng = np.random.default_rng(0)  # the reference test's _inputs(M, N, K, seed=0)
    a = rng.standard_normal((M, K)).astype(np.float16)
    b = rng.standard_normal((N, K)).astype(np.float16)
    c = q4.gemm_f16(a, b)
    ref = golden[f"gemm_{M}x{N}x{K}_c64"]
    assert max_rel(c, ref) < 3e-3  # tests/test_gemm_dsl.py:124-129


def test_argmax_tie_kat():
    # tests/test_kernels_dsl_parity.py:291-316: ties break to the LOWER index
    x = np.random.default_rng(41).standard_normal(262144).astype(np.float32)
    x[12345] = x[200000] = 50.0
    assert int(q4.argmax_first(x)[0]) == 12345


def test_key_packing_orders_like_floats_with_lowest_index_ties():
    vals = np.array([-np.inf, -3.0, -0.0, 0.0, 1e-30, 2.5, 2.5, np.inf], np.float32)
    idx = np.array([7, 6, 5, 4, 3, 2, 1, 0])
    keys = q4.pack_key(vals, idx)
    # +inf wins; among the equal 2.5 keys the lower index (1) ranks higher
    assert int(q4.unpack_key_index(keys.max())) == 0
    k25 = q4.pack_key(np.array([2.5, 2.5], np.float32), np.array([9, 3]))
    assert int(q4.unpack_key_index(k25.max())) == 3
    order = np.argsort(keys[:-1].astype(np.float64))
    assert list(order) == sorted(order, key=lambda i: (vals[i], -idx[i]))


def test_decoder_small_matches_reference(golden):
    cfg = synth.small_config()
    model = synth.random_model(cfg, seed=77)
    o = decoder.OracleDecoder(model, 64)
    toks, margins = o.generate(list(golden["dec_small_prompt"]), 16)
    np.testing.assert_array_equal(toks, golden["dec_small_tokens"])
    np.testing.assert_allclose(margins, golden["dec_small_margins"], rtol=1e-4, atol=1e-4)


@pytest.mark.skipif(not os.path.exists(os.path.join(GOLD, "golden_cfg1.npz")), reason="full fixtures absent")
def test_cfg1_gemv_matches_reference():
    g = np.load(os.path.join(GOLD, "golden_cfg1.npz"))
    packed, scales, x = synth.config1(0)
    assert max_rel(q4.gemv(packed, scales, x)[0], g["cfg1_y"]) < 1e-5


def test_batched_prefill_equals_tokenwise_oracle():
    """The layers-outer oracle prefill (the CPU baseline's workload) computes what
    the token-at-a-time restatement of the reference computes."""
    cfg = synth.small_config()
    model = synth.random_model(cfg, seed=77)
    prompt = synth.prompt_tokens(20, cfg["vocab"], seed=78)
    tw = decoder.OracleDecoder(model, 32)
    for p, t in enumerate(prompt):
        ref = tw.forward(t, p)
    bt = decoder.OracleDecoder(model, 32)
    got = bt.prefill_batched(prompt)
    assert max_rel(got, ref) < 1e-4
    assert int(np.argmax(got)) == int(np.argmax(ref))
    for li in range(cfg["n_layers"]):
        assert max_rel(bt.k_cache[li][:20], tw.k_cache[li][:20]) < 1e-4
        assert max_rel(bt.v_cache[li][:20], tw.v_cache[li][:20]) < 1e-4
