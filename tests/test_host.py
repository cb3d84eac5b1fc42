"""CPU: host-side logic (manifest format, RoPE tables, synthetic configs)."""
import json
import os

import numpy as np

from oracle import decoder as odec
from slang_b200 import manifest, runner, synth


def test_manifest_roundtrip(tmp_path):
    cfg = synth.small_config()
    model = synth.random_model(cfg, seed=3)
    d = manifest.write(model, str(tmp_path))
    man = json.load(open(os.path.join(d, "manifest.json")))
    # export.py conventions: 4-byte aligned offsets, bytes = file size
    assert all(t["off"] % 4 == 0 for t in man["tensors"].values())
    assert man["bytes"] == os.path.getsize(os.path.join(d, "weights.bin"))
    assert man["tensors"]["L1.q_bits"]["shape"] == [cfg["q_dim"], cfg["hidden"] // 2]
    back = manifest.read(d)
    assert back["config"]["hidden"] == 256 and back["config"]["group"] == 32
    np.testing.assert_array_equal(back["embed_q"], model["embed_q"])
    for i in range(2):
        for n in manifest.PROJ:
            np.testing.assert_array_equal(back["layers"][i][n][0], model["layers"][i][n][0])
            np.testing.assert_array_equal(back["layers"][i][n][1], model["layers"][i][n][1])
        for n in ("in_norm", "q_norm", "k_norm", "post_attn_norm", "pre_ffn_norm", "post_ffn_norm"):
            np.testing.assert_array_equal(back["layers"][i][n], model["layers"][i][n])


def test_rope_tables_match_reference_formula():
    cos, sin = runner.rope_tables(300, 256, 10000.0, 128)
    ocos, osin = odec.rope_tables(300, 256, 10000.0, 128)
    np.testing.assert_array_equal(cos, ocos)
    np.testing.assert_array_equal(sin, osin)


def test_partial_rope_cutoff_is_identity_beyond():
    cos, sin = runner.rope_tables(10, 64, 1e6, 8)
    assert (cos[:, 8:] == 1).all() and (sin[:, 8:] == 0).all()


def test_e2b_config_shapes():
    cfg = synth.e2b_config()
    assert cfg["q_dim"] == 2048 and cfg["inter"] == 6144 and cfg["vocab"] == 262144
    assert synth.E2B_SHAPES["down"] == (1536, 6144)


def test_rint_by_magic_add_matches_round_half_even():
    """The GEMV quantises x_int = rint(x * inv) as the f32 sum x * inv + 1.5 * 2^23,
    reading the integer from the low 16 bits of the sum (q4_dot.cuh rint_bits).
    For every |x * inv| <= 32767 -- ties, negatives and the extremes included --
    that must equal round-half-to-even of the f32 product, and the 32-value
    integer sum must come out of the wrapped 32-bit sum of the words."""
    rng = np.random.default_rng(5)
    f = np.concatenate([
        rng.uniform(-32767.0, 32767.0, 200_000),
        np.arange(-32767, 32768, dtype=np.float64) + 0.5,  # every tie
        np.arange(-32767, 32768, dtype=np.float64),
        [0.0, -0.0, 32767.0, -32767.0, 0.49999997, -0.49999997],
    ]).astype(np.float32)
    f = f[np.abs(f) <= 32767.0]
    s = (f + np.float32(12582912.0)).astype(np.float32)  # one f32 add, rounded to nearest even
    bits = s.view(np.uint32)
    low = (bits & 0xFFFF).astype(np.int32)
    got = np.where(low >= 32768, low - 65536, low)
    np.testing.assert_array_equal(got, np.rint(f).astype(np.int32))
    # bias: the 32-word sum minus 32 copies of 0x4B400000, mod 2^32, is the integer sum
    x = got[:32 * 1000].reshape(1000, 32)
    w = bits[:32 * 1000].reshape(1000, 32).astype(np.uint64)
    wrapped = (w.sum(axis=1) - 32 * 0x4B400000) % (1 << 32)
    signed = np.where(wrapped >= 1 << 31, wrapped.astype(np.int64) - (1 << 32), wrapped.astype(np.int64))
    np.testing.assert_array_equal(signed, x.sum(axis=1))
