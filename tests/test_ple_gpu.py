"""GPU: the per-layer-embedding (PLE) kernels against the numpy oracle, through the C ABI.

* ``sb_gemv_q8`` (8-bit codes, per-row scale) with and without the
  gelu_tanh * ple epilogue, ``sb_gemv_bf16``: f32 accumulation in another
  order than numpy's, tolerance 1e-4 of the largest output;
* ``sb_ple_gather``: bit-exact (the same two f32 products per value); ids
  outside the vocabulary give zero rows;
* ``sb_ple_combine`` / ``sb_ple_norm_add`` and the chained per-layer block
  against the oracle and against the reference's own outputs
  (``golden_ple.npz``): 1e-4 relative.
"""
import os

import numpy as np
import pytest
import torch

from oracle import decoder as odec
from oracle import ple as ople
from slang_b200 import _lib
from slang_b200 import kernels as kern
from slang_b200 import synth
from tests._util import max_rel

pytestmark = pytest.mark.gpu
EPS = 1e-6
GOLD = os.path.join(os.path.dirname(__file__), "golden", "golden_ple.npz")


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("n,k", [(256, 1536), (1536, 256), (100, 64), (37, 4096)])
@pytest.mark.parametrize("m", [1, 3, 8, 11])
@pytest.mark.parametrize("with_ple", [False, True])
def test_gemv_q8_vs_oracle(cuda, n, k, m, with_ple):
    rng = np.random.default_rng(n * 7 + k + m)
    codes, scale = synth.q8_weight(rng, n, k, 0.5 / (74 * k ** 0.5), 1.5 / (74 * k ** 0.5))
    x = rng.standard_normal((m, k), dtype=np.float32)
    ple = rng.standard_normal((m, 2 * n), dtype=np.float32)  # rows wider than n: a strided slice
    C, S, X, P = T(codes, cuda), T(scale, cuda), T(x, cuda), T(ple, cuda)
    y = kern.gemv_q8(C, S, X, ple=P[:, n:] if with_ple else None)
    torch.cuda.synchronize()
    ref = ople.q8_gemv(codes, scale, x)
    if with_ple:
        ref = odec.gelu_tanh(ref) * ple[:, n:]
    assert max_rel(y.cpu().numpy(), ref) < 1e-4


@pytest.mark.parametrize("n,k,m", [(8960, 1536, 1), (8960, 1536, 4), (37, 40, 9), (512, 256, 8)])
def test_gemv_bf16_vs_oracle(cuda, n, k, m):
    rng = np.random.default_rng(n + k + m)
    w = synth.f32_to_bf16_bits(rng.normal(0, 0.02, (n, k)).astype(np.float32))
    x = rng.standard_normal((m, k), dtype=np.float32)
    W = T(w.view(np.int16), cuda)
    y = kern.gemv_bf16(W, T(x, cuda), alpha=0.125)
    torch.cuda.synchronize()
    ref = (x @ ople.bf16_to_f32(w).T) * np.float32(0.125)
    assert max_rel(y.cpu().numpy(), ref) < 1e-4


def test_gemv_rejects_bad_shapes(cuda):
    codes = torch.zeros(16, 40, dtype=torch.uint8, device=cuda)  # k % 16 != 0
    with pytest.raises(_lib.SlangError):
        kern.gemv_q8(codes, torch.ones(16, device=cuda), torch.zeros(1, 40, device=cuda))


@pytest.mark.parametrize("vocab,n_layers,d,m", [(512, 2, 256, 3), (4096, 35, 256, 5)])
def test_ple_gather_bit_exact(cuda, vocab, n_layers, d, m):
    w = synth.ple_weights(hidden=256, n_layers=n_layers, d=d, vocab=vocab, seed=11)
    ids = np.random.default_rng(12).integers(0, vocab, m).astype(np.int32)
    ids[-1] = vocab + 5  # out of range -> a zero row
    got = kern.ple_gather(T(ids, cuda), T(w["table"], cuda), T(w["table_scale"], cuda), w["ple_scale"])
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    ref = ople.ple_gather(ids[:-1], w["table"], w["table_scale"], w["ple_scale"])
    np.testing.assert_array_equal(got[:-1], ref)
    assert not got[-1].any()


def test_ple_norm_add_vs_oracle(cuda):
    rng = np.random.default_rng(21)
    m, n = 5, 1536
    proj = rng.standard_normal((m, n), dtype=np.float32)
    hid = (4 * rng.standard_normal((m, n))).astype(np.float32)
    w_post = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    w_next = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    H = T(hid, cuda)
    h = torch.empty_like(H)
    h16 = torch.empty(m, n, dtype=torch.float16, device=cuda)
    kern.ple_norm_add(T(proj, cuda), H, T(w_post, cuda), 0.83, EPS, w_next=T(w_next, cuda), h_out=h, h16_out=h16)
    torch.cuda.synchronize()
    ref = ople.ple_norm_add(proj, hid, w_post, 0.83, EPS)
    assert max_rel(H.cpu().numpy(), ref) < 1e-5
    href = odec.rms_norm(ref, w_next, EPS)
    assert max_rel(h.cpu().numpy(), href) < 1e-5
    assert max_rel(h16.float().cpu().numpy(), href) < 1e-3


@pytest.fixture(scope="module")
def gp():
    return np.load(GOLD)


@pytest.fixture(scope="module")
def small_ple():
    return synth.ple_weights(hidden=1536, n_layers=2, d=256, vocab=512, seed=4343)


def _dev_layer(L, dev):
    return {"gate": (T(L["gate"][0], dev), T(L["gate"][1], dev)),
            "proj": (T(L["proj"][0], dev), T(L["proj"][1], dev)),
            "post_norm": T(L["post_norm"], dev), "scalar": L["scalar"]}


def test_ple_input_vs_reference(cuda, gp, small_ple):
    w = small_ple
    ids = T(gp["ple_ids"].astype(np.int32), cuda)
    got = kern.ple_input(T(gp["ple_x"], cuda), ids, T(w["table"], cuda), T(w["table_scale"], cuda),
                         T(w["proj"].view(np.int16), cuda), T(w["norm"], cuda), 2, 256, EPS, w["ple_scale"])
    torch.cuda.synchronize()
    assert max_rel(got.cpu().numpy(), gp["ple_in"]) < 1e-4


@pytest.mark.parametrize("layer", [0, 1])
def test_ple_block_vs_reference(cuda, gp, small_ple, layer):
    L = _dev_layer(small_ple["layers"][layer], cuda)
    ple_in = T(gp["ple_in"], cuda)  # [m, n_layers, d]
    hid = T(gp[f"ple_l{layer}_mid"], cuda)
    kern.ple_block(hid, ple_in[:, layer], L, EPS)
    torch.cuda.synchronize()
    assert max_rel(hid.cpu().numpy(), gp[f"ple_l{layer}_out"]) < 1e-4


def test_ple_full_shapes_vs_oracle(cuda):
    """E2B shapes (hidden 1536, 35 layers of d = 256; vocabulary cut to 4096
    rows of the 8960-value table) for a decode batch of 4: per-layer input,
    then the PLE block of layers 0 and 34 on it, against the oracle."""
    w = synth.ple_weights(hidden=1536, n_layers=35, d=256, vocab=4096, seed=31)
    rng = np.random.default_rng(32)
    m = 4
    ids = rng.integers(0, 4096, m).astype(np.int32)
    x = (8 * rng.standard_normal((m, 1536))).astype(np.float32)
    rows = ople.ple_gather(ids, w["table"], w["table_scale"], w["ple_scale"])
    ref_in = ople.ple_input(x, rows, w["proj"], w["norm"], 35, 256, EPS)
    got_in = kern.ple_input(T(x, cuda), T(ids, cuda), T(w["table"], cuda), T(w["table_scale"], cuda),
                            T(w["proj"].view(np.int16), cuda), T(w["norm"], cuda), 35, 256, EPS, w["ple_scale"])
    torch.cuda.synchronize()
    assert max_rel(got_in.cpu().numpy(), ref_in) < 1e-4
    for li in (0, 34):
        hid = T(x, cuda)
        kern.ple_block(hid, got_in[:, li], _dev_layer(w["layers"][li], cuda), EPS)
        torch.cuda.synchronize()
        ref = ople.ple_block(x, ref_in[:, li], w["layers"][li], EPS)
        assert max_rel(hid.cpu().numpy(), ref) < 1e-4


@pytest.mark.parametrize("m", [17, 64, 1024])
def test_ple_block_prefill_gemm_route(cuda, m):
    """More than PLE_GEMV_ROWS rows: f16 dequant + tcgen05 GEMMs with f32
    output, the gate tail and the norm-add tail.  f16 operands: the block's
    added term (rmsnorm(proj) * w_post) within the matmul tolerance
    (max-rel 1e-2, cosine 0.9999) of the f32 oracle."""
    from tests._util import assert_close
    assert m > kern.PLE_GEMV_ROWS
    w = synth.ple_weights(hidden=1536, n_layers=2, d=256, vocab=64, seed=41)
    rng = np.random.default_rng(42 + m)
    x = (4 * rng.standard_normal((m, 1536))).astype(np.float32)
    ple_in = rng.standard_normal((m, 2, 256), dtype=np.float32)
    L = w["layers"][1]
    ref = ople.ple_block(x, ple_in[:, 1], L, EPS)
    hid = T(x, cuda)
    dl = _dev_layer(L, cuda)
    kern.ple_block(hid, T(ple_in, cuda)[:, 1], dl, EPS)
    torch.cuda.synchronize()
    got = hid.cpu().numpy()
    s = np.float32(L["scalar"])
    assert_close(got / s - x, ref / s - x, what="PLE block added term")
    assert max_rel(got, ref) < 1e-2
    assert "gate16" in dl and dl["gate16"].dtype == torch.float16


def test_ple_gate_act_and_cast(cuda):
    rng = np.random.default_rng(51)
    m, n = 33, 256
    pre = (3 * rng.standard_normal((m, n))).astype(np.float32)
    ple = rng.standard_normal((m, 2 * n), dtype=np.float32)
    out = torch.empty(m, n, dtype=torch.float16, device=cuda)
    P = T(ple, cuda)
    # two K-split planes: pre = a + b
    a = (0.25 * pre).astype(np.float32)
    PL = T(np.stack([a, pre - a]), cuda)
    _lib.call("sb_ple_gate_act", PL.data_ptr(), n, m * n, 2, P.data_ptr(), 2 * n, out.data_ptr(), n, m, n,
              torch.cuda.current_stream().cuda_stream)
    x16 = torch.empty(m, n, dtype=torch.float16, device=cuda)
    X = T(pre, cuda)
    _lib.call("sb_cast_f16", X.data_ptr(), x16.data_ptr(), m * n, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = odec.gelu_tanh(a + (pre - a)) * ple[:, :n]
    assert max_rel(out.float().cpu().numpy(), ref) < 1e-3
    np.testing.assert_array_equal(x16.cpu().numpy(), pre.astype(np.float16))


@pytest.mark.parametrize("m,n,k,splits", [(1024, 256, 1536, 8), (64, 256, 1536, 3), (200, 300, 512, 4), (130, 1536, 256, 1)])
def test_gemm_f16_f32out_splitk(cuda, m, n, k, splits):
    """Each K split writes its own f32 plane; the planes sum to the full product."""
    g = torch.Generator(device=cuda)
    g.manual_seed(m + n + k)
    a = torch.randn(m, k, device=cuda, generator=g).half()
    b = torch.randn(n, k, device=cuda, generator=g).half()
    c = torch.full((splits, m, n), float("nan"), device=cuda)
    _lib.call("sb_gemm_f16_f32out_splitk", a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, 0.5, 1, k, k, n,
              splits, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = 0.5 * (a.double() @ b.double().T)
    got = c.double().sum(0)
    assert torch.isfinite(got).all()
    assert ((got - ref).abs().max() / ref.abs().max()).item() < 1e-5
    with pytest.raises(_lib.SlangError):  # 5 does not divide ceil(k / 64)
        _lib.call("sb_gemm_f16_f32out_splitk", a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, 0.5, 1, k, k, n,
                  5 if (k // 64) % 5 else 7, torch.cuda.current_stream().cuda_stream)


def _key_logit(key: int) -> float:
    """The max logit held in the top half of a greedy-argmax key."""
    o = (key >> 32) & 0xFFFFFFFF
    bits = o ^ 0x80000000 if o & 0x80000000 else (~o) & 0xFFFFFFFF
    return float(np.array([bits], np.uint32).view(np.float32)[0])


@pytest.mark.parametrize("batched_prefill", [False, True])
def test_runner_with_ple_matches_reference(cuda, gp, batched_prefill):
    """The per-op decode path with a PLE block after every layer (and, batched,
    the prefill's PLE GEMMs): greedy tokens equal the reference's
    QATReference(ple=True) run, and every step's top logit (softcapped) is
    within 1e-3 (token-wise, f32) or 2e-2 (f16 batched prefill) of it."""
    from slang_b200.runner import DeviceModel, Runner
    from tests.test_ple import ple_model
    model = ple_model()
    dm = DeviceModel(model, cuda, 32)
    r = Runner(dm, 1)
    prompt = [int(t) for t in gp["ple_gen_prompt"]]
    first = r.prefill(prompt) if batched_prefill else r.prefill_tokenwise(prompt)
    toks, tops = [first], [_key_logit(int(r.keys[0].item()))]
    for _ in range(9):
        r.decode_step()
        torch.cuda.current_stream().wait_stream(r.stream)
        toks.append(int(r.tok[0].item()))
        tops.append(_key_logit(int(r.keys[0].item())))
    np.testing.assert_array_equal(toks, gp["ple_gen_tokens"])
    cap = model["config"]["softcap"]
    got = cap * np.tanh(np.array(tops) / cap)
    tol = 2e-2 if batched_prefill else 1e-3
    np.testing.assert_allclose(got, gp["ple_gen_top"], rtol=tol)
    assert r.kernel_launches_per_step() == 2 + 2 * 10 + 3 + 2 + (2 if kern.PLE_FUSED_TAIL_ROWS >= 1 else 3) * 2


def test_runner_ple_rejects_other_paths(cuda):
    from slang_b200.runner import DeviceModel, Runner
    from tests.test_ple import ple_model
    dm = DeviceModel(ple_model(), cuda, 16)
    with pytest.raises(ValueError):
        Runner(dm, 1, fused=True)
    with pytest.raises(ValueError):
        Runner(dm, 2, proj="gemm")


def test_ple_input_gemm_route(cuda):
    """A prompt's per-layer inputs through the f16 tcgen05 GEMM (w_proj16):
    within the matmul tolerance of the f32 oracle."""
    from tests._util import assert_close
    w = synth.ple_weights(hidden=1536, n_layers=35, d=256, vocab=256, seed=61)
    rng = np.random.default_rng(62)
    m = 300
    ids = rng.integers(0, 256, m).astype(np.int32)
    x = (8 * rng.standard_normal((m, 1536))).astype(np.float32)
    rows = ople.ple_gather(ids, w["table"], w["table_scale"], w["ple_scale"])
    ref = ople.ple_input(x, rows, w["proj"], w["norm"], 35, 256, EPS)
    W = T(w["proj"].view(np.int16), cuda)
    got = kern.ple_input(T(x, cuda), T(ids, cuda), T(w["table"], cuda), T(w["table_scale"], cuda), W,
                         T(w["norm"], cuda), 35, 256, EPS, w["ple_scale"],
                         w_proj16=W.view(torch.bfloat16).to(torch.float16))
    torch.cuda.synchronize()
    assert_close(got.cpu().numpy(), ref, what="PLE input, GEMM route")


@pytest.mark.parametrize("m", [1, 3, 8])
@pytest.mark.parametrize("with_next", [True, False])
def test_ple_proj_norm_add_fused(cuda, m, with_next):
    """Projection GEMV + last-arriver norm-add tail in one launch, run twice on
    the same counter (it re-arms itself), against the oracle."""
    rng = np.random.default_rng(71 + m)
    codes, scale = synth.q8_weight(rng, 1536, 256, 0.5 / (74 * 16), 1.5 / (74 * 16))
    g = rng.standard_normal((m, 256), dtype=np.float32)
    hid = (4 * rng.standard_normal((m, 1536))).astype(np.float32)
    w_post = (1 + 0.1 * rng.standard_normal(1536)).astype(np.float32)
    w_next = (1 + 0.1 * rng.standard_normal(1536)).astype(np.float32)
    counter = torch.zeros(1, dtype=torch.int32, device=cuda)
    C, S, G = T(codes, cuda), T(scale, cuda), T(g, cuda)
    ref = hid
    H = T(hid, cuda)
    h = torch.empty_like(H)
    for _ in range(2):
        kern.ple_proj_norm_add(C, S, G, H, T(w_post, cuda), 0.9, EPS, w_next=T(w_next, cuda) if with_next else None,
                               h_out=h if with_next else None, counter=counter)
        ref = ople.ple_norm_add(ople.q8_gemv(codes, scale, g), ref, w_post, 0.9, EPS)
    torch.cuda.synchronize()
    assert int(counter.item()) == 0
    assert max_rel(H.cpu().numpy(), ref) < 1e-4
    if with_next:
        assert max_rel(h.cpu().numpy(), odec.rms_norm(ref, w_next, EPS)) < 1e-4
