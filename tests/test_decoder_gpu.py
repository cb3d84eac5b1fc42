"""GPU: the full decoder (every op through the C ABI) against the reference.

* small model (2 layers, hidden 256): greedy tokens equal the reference's own
  ReferenceGemma4 run (golden_small.npz), and the KV caches match the numpy
  oracle within the GEMV tolerance (token-wise path, f32 activations) or the
  f16-activation prefill envelope (batched path);
* config 4 (35 layers, hidden 1536, vocab 262144, 1024-token prompt + 256
  greedy steps): tokens equal the reference's run (golden_cfg4.npz) for both the
  layers-outer batched prefill and the token-wise prefill.  The random-init
  model's greedy trajectory settles on one token, so the per-step max logit is
  compared too (through the keys the lm_head kernel emits).
"""
import os

import numpy as np
import pytest
import torch

from oracle import decoder as odec
from oracle import q4
from slang_b200 import runner, synth

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def small_model():
    cfg = synth.e2b_config(hidden=256, n_layers=2, n_heads=2, head_dim=64, inter=512, vocab=2048, rope_cutoff=32)
    return synth.random_model(cfg, seed=77)


def _key_value(keys):
    """Max logit held in an lm_head key (inverse of the orderable f32 map)."""
    hi = (np.asarray(keys, dtype=np.int64).view(np.uint64) >> np.uint64(32)).astype(np.uint32)
    bits = np.where(hi & 0x80000000, hi & 0x7FFFFFFF, ~hi).astype(np.uint32)
    return bits.view(np.float32)


@pytest.mark.parametrize("batched", [False, True])
def test_small_decoder_tokens_match_reference(cuda, golden, batched):
    model = small_model()
    prompt = [int(t) for t in golden["dec_small_prompt"]]
    toks = runner.greedy_generate(model, prompt, 17, device=cuda, batched_prefill=batched, max_seq=64)
    # golden_small holds 16 tokens generated after the prompt by the reference
    np.testing.assert_array_equal(toks[:16], golden["dec_small_tokens"])


def test_small_decoder_kv_cache_vs_oracle(cuda, golden):
    model = small_model()
    prompt = [int(t) for t in golden["dec_small_prompt"]]
    o = odec.OracleDecoder(model, 64)
    for p, t in enumerate(prompt):
        o.forward(t, p)
    S = len(prompt)
    for batched, tol in ((False, 2e-4), (True, 2e-2)):
        dm = runner.DeviceModel(model, cuda, 64)
        r = runner.Runner(dm, 1)
        r.prefill(prompt) if batched else r.prefill_tokenwise(prompt)
        torch.cuda.synchronize()
        for li in range(model["config"]["n_layers"]):
            for got, ref in ((r.kc[li][0, :S], o.k_cache[li][:S]), (r.vc[li][0, :S], o.v_cache[li][:S])):
                g = got.cpu().numpy()
                rel = np.linalg.norm(g - ref) / np.linalg.norm(ref)
                assert rel < tol, f"layer {li} batched={batched}: KV rel-L2 {rel:.2e}"


def test_batch_of_sequences_is_independent(cuda, golden):
    """Decode 3 sequences at once: each equals its own single-sequence run."""
    model = small_model()
    prompts = [[int(t) for t in golden["dec_small_prompt"]], synth.prompt_tokens(9, 2048, seed=5),
               synth.prompt_tokens(14, 2048, seed=6)]
    singles = [runner.greedy_generate(model, p, 8, device=cuda, max_seq=64) for p in prompts]
    dm = runner.DeviceModel(model, cuda, 64)
    r = runner.Runner(dm, 3)
    firsts = [r.prefill(p, seq=b) for b, p in enumerate(prompts)]
    rest = r.decode(7).cpu().numpy()
    for b in range(3):
        assert [firsts[b]] + rest[b].tolist() == singles[b]


def mid_model():
    """Full-width layers (hidden 1536, 8 heads of 256, FFN 6144) but 3 layers and a 16384-row vocabulary."""
    return synth.random_model(synth.e2b_config(n_layers=3, vocab=16384), seed=21)


def test_fused_decode_matches_per_op_path_and_oracle(cuda):
    model = mid_model()
    prompt = synth.prompt_tokens(40, 16384, seed=22)
    per_op = runner.greedy_generate(model, prompt, 48, device=cuda, max_seq=128)
    fused = runner.greedy_generate(model, prompt, 48, device=cuda, max_seq=128, fused=True)
    assert fused == per_op
    # token-wise prefill through the persistent kernel: KV caches vs the numpy oracle
    dm = runner.DeviceModel(model, cuda, 64)
    r = runner.Runner(dm, 1, fused=True)
    r.prefill_tokenwise(prompt[:20])
    torch.cuda.synchronize()
    o = odec.OracleDecoder(model, 64)
    for p_, t in enumerate(prompt[:20]):
        o.forward(t, p_)
    for li in range(3):
        for got, ref in ((r.kc[li][0, :20], o.k_cache[li][:20]), (r.vc[li][0, :20], o.v_cache[li][:20])):
            rel = np.linalg.norm(got.cpu().numpy() - ref) / np.linalg.norm(ref)
            assert rel < 2e-4, f"layer {li}: KV rel-L2 {rel:.2e}"


@pytest.fixture(scope="module")
def cfg4():
    path = os.path.join(GOLD, "golden_cfg4.npz")
    if not os.path.exists(path):
        pytest.skip("config-4 fixture absent")
    g = np.load(path)
    model = synth.random_model(synth.e2b_config(), seed=1234)
    prompt = synth.prompt_tokens(int(g["cfg4_prompt_len"]), 262144, seed=99)
    return g, model, prompt


@pytest.mark.parametrize("batched,fused", [(True, False), (False, False), (True, True)])
def test_config4_256_greedy_tokens_match_reference(cuda, cfg4, batched, fused):
    g, model, prompt = cfg4
    steps = len(g["cfg4_tokens"])
    S = len(prompt)
    dm = runner.DeviceModel(model, cuda, S + steps + 1)
    r = runner.Runner(dm, 1, fused=fused)
    first = r.prefill(prompt) if batched else r.prefill_tokenwise(prompt)
    tops = [float(_key_value(r.keys.cpu().numpy())[0])]
    if not batched:
        r.set_state([first], [S])
    toks = [first]
    for _ in range(steps - 1):
        r.decode_step()
        torch.cuda.current_stream().wait_stream(r.stream)
        tops.append(float(_key_value(r.keys.cpu().numpy())[0]))
    torch.cuda.current_stream().wait_stream(r.stream)
    toks += r.history[0, S + 1:S + steps].cpu().tolist()
    np.testing.assert_array_equal(toks, g["cfg4_tokens"])
    # max logit per step (pre-softcap) vs the reference's softcapped value
    cap = 30.0
    got = cap * np.tanh(np.array(tops) / cap)
    err = np.abs(got - g["cfg4_top"]).max()
    print(f"config 4 batched={batched} fused={fused}: max |top logit - reference| = {err:.3e}")
    # f16 activations in the batched prefill GEMMs vs the f32 token-wise path
    assert err < (5e-2 if batched else 5e-3)


@pytest.mark.parametrize("batch", [3, 12])
def test_batched_decode_on_tcgen05_gemm(cuda, golden, batch):
    """Config 5's large-batch decode: projections and the lm_head argmax on the
    tcgen05 GEMM (f16 activations).  Every sequence equals its own
    single-sequence run (the GEMV path) for 8 greedy steps."""
    model = small_model()
    prompts = [synth.prompt_tokens(5 + 3 * b, 2048, seed=40 + b) for b in range(batch)]
    singles = [runner.greedy_generate(model, p, 8, device=cuda, max_seq=64) for p in prompts]
    dm = runner.DeviceModel(model, cuda, 64)
    r = runner.Runner(dm, batch, proj="gemm")
    firsts = [r.prefill(p, seq=b) for b, p in enumerate(prompts)]
    rest = r.decode(7).cpu().numpy()
    got = [[firsts[b]] + rest[b].tolist() for b in range(batch)]
    agree = sum(g == s for g, s in zip(got, singles))
    assert agree == batch, f"{batch - agree} of {batch} sequences diverge: {got} vs {singles}"
