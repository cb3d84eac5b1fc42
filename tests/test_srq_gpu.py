"""GPU: the SRQ linear (``sb_gemv_srq``) and elementwise srq against the oracle.

The oracle is pinned to the reference's ``ReferenceSRQ._qlin`` on the same
weights (tests/test_srq.py).  The GPU forms the dot of the integer input codes
exactly and scales it in a different f32 order than numpy's matvec, so an
output may sit one quantisation step away where ``y / out_scale`` falls within
rounding of a half-way point; everything else is bit-equal.
"""
import os

import numpy as np
import pytest
import torch

from oracle import decoder as odec
from oracle import srq as osrq
from slang_b200 import kernels, manifest
from tests.test_srq import cases

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _check(got, ref, out_scale, what):
    diff = np.abs(got - ref)
    off = diff > 0
    step = np.asarray(out_scale, np.float32)
    assert (diff <= step * 1.0001 + 1e-7).all(), f"{what}: an output is more than one quantisation step off"
    assert off.mean() <= 0.02, f"{what}: {off.sum()} of {off.size} outputs off by one step"


def test_gemv_srq_matches_reference_qlin(cuda):
    for g, i, (packed, scale), s_in, s_out in cases():
        n_in = g[f"qlin{i}_0_x"].shape[0]
        bits = odec.packed_bits(packed, n_in)
        W, S = torch.from_numpy(np.ascontiguousarray(packed)).to(cuda), torch.from_numpy(np.ascontiguousarray(scale)).to(cuda)
        for j in range(2):
            x = g[f"qlin{i}_{j}_x"]
            y = kernels.gemv_srq(W, S, torch.from_numpy(x).to(cuda), s_in, s_out, bits=bits)[0].cpu().numpy()
            _check(y, g[f"qlin{i}_{j}_y"], s_out, f"qlin {i} input {j}")
    kernels.device_status()


def test_gemv_srq_per_row_out_scales_on_fused_qkv(cuda):
    """q|k|v as one weight (as the runner fuses them) with each part's own out scale."""
    m = manifest.read(os.path.join(GOLD, "export_small"))
    L = m["layers"][1]
    packed = np.concatenate([L[n][0] for n in "qkv"])
    scale = np.concatenate([L[n][1] for n in "qkv"])
    s = L["srq"]
    rows = np.concatenate([np.full(len(L[n][0]), s[f"{n}_out"], np.float32) for n in "qkv"])
    x = np.random.default_rng(3).standard_normal((3, packed.shape[1] * 2)).astype(np.float32) * 2
    got = kernels.gemv_srq(torch.from_numpy(packed).to(cuda), torch.from_numpy(scale).to(cuda),
                           torch.from_numpy(x).to(cuda), s["qkv_in"], torch.from_numpy(rows).to(cuda)).cpu().numpy()
    for r in range(3):
        ref = osrq.qlin(packed, scale, 4, x[r], s["qkv_in"], rows)
        _check(got[r], ref, rows, f"fused q|k|v row {r}")
    kernels.device_status()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_elementwise_srq_matches_oracle(cuda, dtype):
    g = np.load(os.path.join(GOLD, "golden_srq.npz"))
    x = np.concatenate([g["srq_kat_x"], np.random.default_rng(4).standard_normal(5000).astype(np.float32) * 3])
    xt = torch.from_numpy(x).to(cuda).to(dtype)
    got = kernels.srq(xt, float(g["srq_kat_s"])).float().cpu().numpy()
    ref = osrq.srq(xt.float().cpu().numpy(), float(g["srq_kat_s"]))
    if dtype == torch.float16:
        ref = ref.astype(np.float16).astype(np.float32)
    np.testing.assert_array_equal(got, ref)
    kernels.device_status()
