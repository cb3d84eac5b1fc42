"""GPU: the decode GEMV with the residual add + RMSNorm as a last-arriver tail
(``sb_gemv_norm_add``, the reference's oproj_73 / down_75 tails), against the
numpy oracle: y = W x, hidden += rmsnorm(y) * w_add, h = rmsnorm(hidden) * w_next.
Both GEMV kernels (K 2048: whole rows per half-warp; K 6144: split K), 2-bit
codes, a batch that takes two launches (each tails its own rows), and two calls
in a row on one counter (the last CTA re-arms it)."""
import numpy as np
import pytest
import torch

from oracle import decoder as odec
from oracle import q4
from slang_b200 import kernels, runner, synth
from tests._util import first_divergence

pytestmark = pytest.mark.gpu
EPS = 1e-6


@pytest.mark.parametrize("n,k,m,bits", [(1536, 2048, 1, 4), (1536, 6144, 3, 4), (1536, 2048, 6, 4),
                                        (1536, 6144, 2, 2), (256, 512, 1, 4)])
def test_gemv_norm_add_vs_oracle(cuda, n, k, m, bits):
    rng = np.random.default_rng(n + k + m + bits)
    packed, scales = (synth.q4_weight if bits == 4 else synth.q2_weight)(rng, n, k)
    w_add = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    w_next = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    W, S, WA, WN = T(packed), T(scales), T(w_add), T(w_next)
    counter = torch.zeros(1, dtype=torch.int32, device=cuda)
    hid = rng.standard_normal((m, n)).astype(np.float32) * 3
    H = T(hid)
    for call in range(2):
        x = rng.standard_normal((m, k)).astype(np.float32)
        h = torch.empty((m, n), device=cuda)
        h16 = torch.empty((m, n), dtype=torch.float16, device=cuda)
        y = kernels.gemv_norm_add(W, S, T(x), H, WA, EPS, w_next=WN, h_out=h, h16_out=h16, counter=counter,
                                  bits=bits)
        torch.cuda.synchronize()
        y_ref = q4.gemv(packed, scales, x, bits)
        hid = hid + odec.rms_norm(y_ref, w_add, EPS)
        h_ref = odec.rms_norm(hid, w_next, EPS)
        yg, hg, xg = y.cpu().numpy(), h.cpu().numpy(), H.cpu().numpy()
        assert np.abs(yg - y_ref).max() <= 2e-4 * np.abs(y_ref).max(), f"call {call}: y"
        assert np.abs(xg - hid).max() <= 2e-4 * np.abs(hid).max(), f"call {call}: hidden"
        assert np.abs(hg - h_ref).max() <= 2e-4 * np.abs(h_ref).max(), f"call {call}: h"
        np.testing.assert_array_equal(h16.cpu().numpy(), hg.astype(np.float16))
        hid = xg  # continue from the GPU's state
    assert int(counter.item()) == 0, "the last CTA re-arms the counter"
    kernels.device_status()


def test_decode_with_norm_tails_follows_oracle(cuda, golden):
    model = synth.random_model(synth.small_config(), seed=77)
    prompt = [int(t) for t in golden["dec_small_prompt"]]
    dm = runner.DeviceModel(model, cuda, 64)
    r = runner.Runner(dm, 1, norm_tails=True)
    first = r.prefill_tokenwise(prompt)
    r.set_state([first], [len(prompt)])
    toks = [first] + r.decode(15)[0].cpu().tolist()
    first_divergence(toks, golden["dec_small_tokens"], golden["dec_small_margins"], 1e-2, "decode with norm tails")
