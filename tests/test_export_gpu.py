"""GPU: models in the reference's own on-disk format, end to end.

``manifest.read`` loads manifest.json + weights.bin written by the reference's
``gemma4_150.export.export`` (per-row f32 scales, 2-bit embedding and lm_head,
int8 per-layer-embedding linears, f16 per-layer projection); ``DeviceModel``
puts it on the GPU and the runner decodes it through the C ABI.  Two fixtures:

* export_small: three uniform layers;
* export_arch: the real model's mixed layers -- sliding head_dim-128 layers
  with a 16-key window (masking keys in both the prefill and the decode of a
  24-token prompt), full head_dim-512 layers with partial RoPE, FFN width
  doubling from layer 3, layers 4 and 5 reading the K/V of layers 3 and 2.

Greedy tokens follow the reference's weight-only ``QATReference`` run on the
same checkpoint (near ties aside), and a teacher-forced replay matches its 8
largest logits at every step.
"""
import os

import numpy as np
import pytest
import torch

from slang_b200 import manifest, runner
from tests._util import check_top8, first_divergence

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
CAP = 30.0
CASES = ["export_small", "export_arch"]


@pytest.fixture(scope="module", params=CASES)
def export(request):
    d = os.path.join(GOLD, request.param)
    return request.param, manifest.read(d), np.load(os.path.join(d, "golden_export.npz"))


@pytest.mark.parametrize("batched", [False, True])
def test_export_greedy_tokens_follow_reference(cuda, export, batched):
    name, model, g = export
    prompt = [int(t) for t in g["prompt"]]
    toks = runner.greedy_generate(model, prompt, len(g["tokens"]), device=cuda, batched_prefill=batched, max_seq=48)
    first_divergence(toks, g["tokens"], g["margins"], 5e-2 if batched else 1e-2, f"{name} batched={batched}")


@pytest.mark.parametrize("batched", [False, True])
def test_export_teacher_forced_top8(cuda, export, batched):
    name, model, g = export
    prompt = [int(t) for t in g["prompt"]]
    dm = runner.DeviceModel(model, cuda, 48)
    assert dm.embed_bits == 2 and dm.lm_bits == 2 and dm.layers[0]["bits"]["qkv"] == 4
    r = runner.Runner(dm, 1)
    S = len(prompt)
    if batched:
        r.prefill(prompt)
        h0 = r._pf["hlast"][S - 1:S]
    else:
        r.prefill_tokenwise(prompt)
        h0 = r.h
    tol = 5e-2 if batched else 1e-2
    logits = torch.empty((1, model["config"]["vocab"]), dtype=torch.float32, device=cuda)
    worst = 0.0
    for s in range(len(g["tokens"])):
        if s:
            r.set_state([int(g["tokens"][s - 1])], [S + s - 1])
            r.decode_step()
            torch.cuda.current_stream().wait_stream(r.stream)
        dm.lmhead_argmax(h0 if s == 0 else r.h, None, None, logits=logits)
        worst = max(worst, check_top8(logits[0].cpu().numpy(), g["top8_idx"][s], g["top8_val"][s], CAP, tol,
                                      f"{name} batched={batched} step {s}"))
    print(f"{name} teacher-forced batched={batched}: max top-8 logit error {worst:.2e}")


def test_export_refuses_paths_needing_the_group32_format(cuda, export):
    _, model, _ = export
    dm = runner.DeviceModel(model, cuda, 32)
    with pytest.raises(ValueError):
        runner.Runner(dm, 1, fused=True)
    with pytest.raises(ValueError):
        runner.Runner(dm, 16, proj="gemm")


def test_mixed_export_kv_sharing_aliases_the_source_cache(cuda):
    model = manifest.read(os.path.join(GOLD, "export_arch"))
    r = runner.Runner(runner.DeviceModel(model, cuda, 40), 1)
    assert r.kc[4] is r.kc[3] and r.vc[5] is r.vc[2]
    assert r.kc[2].shape[-1] == 512 and r.kc[0].shape[-1] == 128
