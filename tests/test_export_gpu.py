"""GPU: a model in the reference's own on-disk format, end to end.

``manifest.read`` loads ``tests/golden/export_small`` (manifest.json +
weights.bin written by the reference's ``gemma4_150.export.export``: per-row
f32 scales, 2-bit embedding and lm_head, int8 per-layer-embedding linears, f16
per-layer projection); ``DeviceModel`` puts it on the GPU and the runner
decodes it through the C ABI.  Greedy tokens follow the reference's
weight-only ``QATReference`` run on the same checkpoint (near ties aside), and
a teacher-forced replay matches its 8 largest logits at every step.
"""
import os

import numpy as np
import pytest
import torch

from slang_b200 import manifest, runner
from tests._util import check_top8, first_divergence

pytestmark = pytest.mark.gpu
EXPORT = os.path.join(os.path.dirname(__file__), "golden", "export_small")
CAP = 30.0


@pytest.fixture(scope="module")
def export():
    return manifest.read(EXPORT), np.load(os.path.join(EXPORT, "golden_export.npz"))


@pytest.mark.parametrize("batched", [False, True])
def test_export_greedy_tokens_follow_reference(cuda, export, batched):
    model, g = export
    prompt = [int(t) for t in g["prompt"]]
    toks = runner.greedy_generate(model, prompt, len(g["tokens"]), device=cuda, batched_prefill=batched, max_seq=32)
    first_divergence(toks, g["tokens"], g["margins"], 5e-2 if batched else 1e-2, f"export batched={batched}")


def test_export_teacher_forced_top8(cuda, export):
    model, g = export
    prompt = [int(t) for t in g["prompt"]]
    dm = runner.DeviceModel(model, cuda, 32)
    assert dm.embed_bits == 2 and dm.lm_bits == 2 and dm.layers[0]["bits"]["qkv"] == 4
    r = runner.Runner(dm, 1)
    r.prefill_tokenwise(prompt)
    logits = torch.empty((1, model["config"]["vocab"]), dtype=torch.float32, device=cuda)
    S, worst = len(prompt), 0.0
    for s in range(len(g["tokens"])):
        if s:
            r.set_state([int(g["tokens"][s - 1])], [S + s - 1])
            r.decode_step()
            torch.cuda.current_stream().wait_stream(r.stream)
        dm.lmhead_argmax(r.h, None, None, logits=logits)
        worst = max(worst, check_top8(logits[0].cpu().numpy(), g["top8_idx"][s], g["top8_val"][s], CAP, 1e-2,
                                      f"export step {s}"))
    print(f"export teacher-forced: max top-8 logit error {worst:.2e}")


def test_export_refuses_paths_needing_the_group32_format(cuda, export):
    model, _ = export
    dm = runner.DeviceModel(model, cuda, 32)
    with pytest.raises(ValueError):
        runner.Runner(dm, 1, fused=True)
    with pytest.raises(ValueError):
        runner.Runner(dm, 16, proj="gemm")


def test_export_refuses_context_beyond_the_sliding_window(cuda, export):
    model, _ = export
    with pytest.raises(ValueError, match="sliding window"):
        runner.DeviceModel(model, cuda, 1024)
