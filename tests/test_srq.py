"""CPU: the SRQ oracle pinned to the reference's own code.

``tests/golden/golden_srq.npz`` (``make_golden.py --only srq``) holds the
reference's ``srq`` on known answers and its ``ReferenceSRQ._qlin``
(gemma4_150/reference.py:96-101) on linears of the export_small checkpoint,
whose manifest (written by the reference's export.py) is committed beside it:
the oracle fed the manifest's weights and SRQ scales must reproduce those
outputs exactly.
"""
import os

import numpy as np

from oracle import decoder as odec
from oracle import srq as osrq
from slang_b200 import manifest

GOLD = os.path.join(os.path.dirname(__file__), "golden")
KEY = {"self_attn.q_proj": ("q", "qkv_in", "q_out"), "self_attn.k_proj": ("k", "qkv_in", "k_out"),
       "self_attn.o_proj": ("o", "o_in", "o_out"), "mlp.gate_proj": ("gate", "gate_in", "gate_out"),
       "mlp.up_proj": ("up", "up_in", "up_out"), "mlp.down_proj": ("down", "down_in", "down_out")}


def cases():
    g = np.load(os.path.join(GOLD, "golden_srq.npz"))
    m = manifest.read(os.path.join(GOLD, "export_small"))
    i = 0
    while f"qlin{i}_layer" in g:
        L = int(g[f"qlin{i}_layer"])
        name, kin, kout = KEY[str(g[f"qlin{i}_mod"])]
        layer = m["layers"][L]
        yield g, i, layer[name], layer["srq"][kin], layer["srq"][kout]
        i += 1


def test_srq_known_answers_match_reference():
    g = np.load(os.path.join(GOLD, "golden_srq.npz"))
    np.testing.assert_array_equal(osrq.srq(g["srq_kat_x"], float(g["srq_kat_s"])), g["srq_kat_y"])


def test_manifest_carries_the_srq_scales():
    for g, i, _, s_in, s_out in cases():
        assert np.float32(s_in) == g[f"qlin{i}_in"] and np.float32(s_out) == g[f"qlin{i}_out"]


def test_qlin_oracle_equals_reference_qlin():
    n = 0
    for g, i, (packed, scale), s_in, s_out in cases():
        bits = odec.packed_bits(packed, g[f"qlin{i}_0_x"].shape[0])
        for j in range(2):
            got = osrq.qlin(packed, scale, bits, g[f"qlin{i}_{j}_x"], s_in, s_out)
            np.testing.assert_array_equal(got, g[f"qlin{i}_{j}_y"])
            n += 1
    assert n == 12
