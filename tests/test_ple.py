"""CPU: the per-layer-embedding (PLE) oracle against the reference's own code.

``tests/golden/golden_ple.npz`` comes from tests/golden/make_golden.py, which
runs the reference's ``QATReference`` (``ple=True``) on a 2-layer hidden-1536
model: the scaled PLE table rows, ``_ple_input`` and one ``_layer`` call per
layer with and without the PLE block (``*_mid`` is the layer output before the
block, ``*_out`` after it).  The weights regenerate from the seeds below.
"""
import os

import numpy as np
import pytest

from oracle import ple as ople
from oracle import q4
from slang_b200 import synth
from tests._util import max_rel

GOLD = os.path.join(os.path.dirname(__file__), "golden", "golden_ple.npz")
EPS = 1e-6


@pytest.fixture(scope="module")
def gp():
    return np.load(GOLD)


@pytest.fixture(scope="module")
def weights():
    return synth.ple_weights(hidden=1536, n_layers=2, d=256, vocab=512, seed=4343)


def test_gather_matches_reference(gp, weights):
    rows = ople.ple_gather(gp["ple_ids"], weights["table"], weights["table_scale"], weights["ple_scale"])
    np.testing.assert_array_equal(rows, gp["ple_rows"])


def test_ple_input_matches_reference(gp, weights):
    got = ople.ple_input(gp["ple_x"], gp["ple_rows"], weights["proj"], weights["norm"], 2, 256, EPS)
    assert max_rel(got, gp["ple_in"]) < 1e-5


@pytest.mark.parametrize("layer", [0, 1])
def test_ple_block_matches_reference(gp, weights, layer):
    got = ople.ple_block(gp[f"ple_l{layer}_mid"], gp["ple_in"][:, layer], weights["layers"][layer], EPS)
    assert max_rel(got, gp[f"ple_l{layer}_out"]) < 1e-5


def test_q8_codes_are_biased_int8():
    # code 0 -> -128, 128 -> 0, 255 -> 127 (gemma4_150/export.py:155-157)
    codes = np.array([[0, 128, 255, 1]], np.uint8)
    np.testing.assert_array_equal(q4.unpack_signed(codes, 8), [[-128, 0, 127, -127]])
    w = q4.dequant_f32(codes, np.array([0.5], np.float32), 8)
    np.testing.assert_array_equal(w, [[-64.0, 0.0, 63.5, -63.5]])


def test_bf16_rounding():
    a = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.0e-3], np.float32)
    bits = synth.f32_to_bf16_bits(a)
    back = ople.bf16_to_f32(bits)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: ties to even gives 1.0
    assert back[0] == 1.0 and back[1] == 1.0 and back[3] == -2.5
    assert np.all(np.abs(back - a) <= np.abs(a) * 2.0 ** -8)


def ple_model():
    """The 2-layer model with per-layer embeddings that golden_ple.npz was generated from."""
    cfg = synth.e2b_config(hidden=1536, n_layers=2, n_heads=2, head_dim=256, inter=512, vocab=512, rope_cutoff=32)
    model = synth.random_model(cfg, seed=4242)
    model["ple"] = synth.ple_weights(hidden=1536, n_layers=2, d=256, vocab=512, seed=4343)
    return model


def test_oracle_decoder_with_ple_matches_reference(gp):
    from oracle.decoder import OracleDecoder
    o = OracleDecoder(ple_model(), 32)
    toks, margins = o.generate([int(t) for t in gp["ple_gen_prompt"]], 10)
    np.testing.assert_array_equal(toks, gp["ple_gen_tokens"])
    np.testing.assert_allclose(margins, gp["ple_gen_margins"], rtol=1e-4, atol=1e-4)


def test_ple_changes_the_logits(gp):
    """The same model without its PLE blocks gives other top-2 margins: the
    end-to-end PLE checks are sensitive to the PLE path."""
    from oracle.decoder import OracleDecoder
    model = ple_model()
    del model["ple"]
    _, margins = OracleDecoder(model, 32).generate([int(t) for t in gp["ple_gen_prompt"]], 10)
    assert np.abs(np.array(margins) - gp["ple_gen_margins"]).max() > 0.1


def test_ple_wrappers_reject_host_tensors_and_bad_shapes():
    """The torch wrappers validate on the host before any call into the
    library (no GPU needed): host tensors are refused (the device is checked
    before the dtype), and so are non-tensors."""
    import torch
    from slang_b200 import kernels as kern
    codes = torch.zeros(16, 64, dtype=torch.uint8)
    scale = torch.ones(16)
    x = torch.zeros(1, 64)
    with pytest.raises(ValueError):
        kern.gemv_q8(codes, scale, x)
    with pytest.raises(ValueError):
        kern.gemv_bf16(torch.zeros(4, 32, dtype=torch.bfloat16), x)
    with pytest.raises(ValueError):
        kern.ple_proj_norm_add(codes, scale, torch.zeros(1, 64), torch.zeros(1, 16), torch.ones(16), 1.0, 1e-6)
    with pytest.raises(TypeError):
        kern.gemv_q8(codes.numpy(), scale, x)


def test_synth_ple_weight_shapes():
    w = synth.ple_weights(hidden=256, n_layers=3, d=256, vocab=10, seed=1)
    assert w["table"].shape == (10, 3 * 256 // 2) and w["table_scale"].shape == (10, 3)
    assert w["proj"].shape == (3 * 256, 256) and w["proj"].dtype == np.uint16
    L = w["layers"][2]
    assert L["gate"][0].shape == (256, 256) and L["gate"][1].shape == (256,)
    assert L["proj"][0].shape == (256, 256) and L["post_norm"].shape == (256,)
    assert w["ple_scale"] == 16.0
