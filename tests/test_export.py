"""CPU: the reference's own on-disk format, read by ``manifest.read``.

``tests/golden/export_small`` holds manifest.json + weights.bin written by the
reference's ``gemma4_150.export.export`` from a synthetic QAT checkpoint with
the real tensor names, dtypes and bit widths (``make_golden.py --only export``),
and the greedy run of the reference's weight-only ``QATReference`` (ple=True)
on that checkpoint.  The reader must recover every tensor's layout (flat u32
packed rows, per-row f32 scales, the 2-bit embedding and block-major lm_head,
the packed norm vectors, the per-layer-embedding tensors) so that the oracle,
fed the reader's output, reproduces the reference's tokens.
"""
import os

import numpy as np

from oracle import decoder as odec
from oracle import q4
from slang_b200 import manifest
from tests._util import first_divergence

EXPORT = os.path.join(os.path.dirname(__file__), "golden", "export_small")


def test_reader_recovers_the_export_layout():
    m = manifest.read(EXPORT)
    c = m["config"]
    H, V = c["hidden"], c["vocab"]
    assert (H, c["n_layers"], V, c["n_heads"]) == (256, 3, 768, 2)
    assert c["sliding_window"] == 512 and len(c["layer_specs"]) == 3
    # 2-bit embedding with one f32 scale per row; the separate 2-bit lm_head was
    # written from the same codes and scales (export.py re-lays it out block-major)
    assert m["embed_q"].shape == (V, H // 4) and m["embed_scale"].shape == (V, 1)
    np.testing.assert_array_equal(m["lm_q"], m["embed_q"])
    np.testing.assert_array_equal(m["lm_scale"], m["embed_scale"])
    L = m["layers"][0]
    for name, n_out, n_in in (("q", 128, H), ("k", 64, H), ("v", 64, H), ("o", H, 128), ("gate", 512, H),
                              ("up", 512, H), ("down", H, 512)):
        packed, scale = L[name]
        assert packed.shape == (n_out, n_in // 2) and odec.packed_bits(packed, n_in) == 4, name
        assert scale.shape == (n_out, 1) and scale.dtype == np.float32, name
    assert L["post_attn_norm"].shape == (H,) and L["pre_ffn_norm"].shape == (H,)
    P = m["ple"]
    assert P["table"].shape == (V, 3 * 256 // 2) and P["table_scale"].shape == (V, 3)
    assert P["proj"].dtype == np.float16 and P["proj"].shape == (3 * 256, H)
    assert P["layers"][0]["gate"][0].shape == (256, H) and P["layers"][0]["proj"][0].shape == (H, 256)
    assert 0.7 <= P["layers"][2]["scalar"] <= 1.3


def test_oracle_on_the_export_reproduces_the_reference():
    m = manifest.read(EXPORT)
    g = np.load(os.path.join(EXPORT, "golden_export.npz"))
    assert len(set(g["tokens"].tolist())) >= 8, "the reference's trajectory should move"
    o = odec.OracleDecoder(m, 32)
    toks, margins = o.generate([int(t) for t in g["prompt"]], len(g["tokens"]))
    assert first_divergence(toks, g["tokens"], g["margins"], 1e-4, "oracle on the export") is None
    np.testing.assert_allclose(margins, g["margins"], atol=1e-4)


def test_export_dequant_matches_reference_row_scale_rule():
    """Per-row f32 scales: value = (code - 8) * scale[row] (gemma4/qat_loader.py:98-102)."""
    m = manifest.read(EXPORT)
    packed, scale = m["layers"][1]["o"]
    w = q4.dequant_f32(packed, scale, 4)
    codes = q4.unpack_codes(packed, 4).astype(np.float32) - 8
    np.testing.assert_array_equal(w, codes * scale)


ARCH = os.path.join(os.path.dirname(__file__), "golden", "export_arch")


def test_mixed_architecture_export_layout_and_oracle():
    """The real model's mixed layers (export_arch): sliding head_dim-128 layers
    with a 16-key window, full head_dim-512 layers with partial RoPE, FFN width
    doubling from layer 3, layers 4 and 5 reading the K/V of layers 3 and 2.
    The reader recovers the per-layer structure (no k/v weights for the shared
    layers) and the oracle on it reproduces the reference's tokens."""
    m = manifest.read(ARCH)
    specs = m["config"]["layer_specs"]
    assert [sp["head_dim"] for sp in specs] == [128, 128, 512, 128, 128, 512]
    assert [sp["inter"] for sp in specs] == [256, 256, 256, 512, 512, 512]
    assert [sp["kv_source"] for sp in specs] == [0, 1, 2, 3, 3, 2]
    assert m["config"]["sliding_window"] == 16 and specs[2]["rope_cutoff"] == 64
    assert "k" not in m["layers"][4] and "k_norm" not in m["layers"][5]
    assert m["layers"][2]["q"][0].shape == (2 * 512, 256 // 2)
    g = np.load(os.path.join(ARCH, "golden_export.npz"))
    assert len(set(g["tokens"].tolist())) >= 8, "the reference's trajectory should move"
    toks, margins = odec.OracleDecoder(m, 48).generate([int(t) for t in g["prompt"]], len(g["tokens"]))
    assert first_divergence(toks, g["tokens"], g["margins"], 1e-4, "oracle on the mixed export") is None
    np.testing.assert_allclose(margins, g["margins"], atol=1e-4)
