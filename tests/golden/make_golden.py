"""Generate the golden fixtures in this directory by running the REFERENCE's code.

    python tests/golden/make_golden.py --reference <path to a wakoan/slang checkout> [--full]

What runs from the reference (imported in place, nothing copied):

* ``gemma4.qat_loader.unpack_int4`` / ``unpack_int2`` / ``unpack_bits`` on the
  reference tests' known-answer bytes and on random packed rows;
* ``QATIndex.dequant_embedding_full`` (the per-block ``np.repeat`` dequant,
  gemma4/qat_loader.py:115-121) on synthetic packed tables, through a minimal
  stand-in for its safetensors index;
* ``tests/test_gemm_dsl.py``'s float64 ``reference`` and ``_inputs`` for the GEMM shapes;
* ``gemma4.reference.ReferenceGemma4`` (``ple=False``) for the decoder, with a
  ``_w``/``_embed_row`` override in the style of ``QATReference``
  (gemma4/qat_reference.py:24-37) that serves the synthetic int4 weights; every
  greedy step records its token, top-2 margin and the 8 largest logits with
  their ids (the reference feeds its own token back, so a teacher-forced replay
  on another implementation feeds the same tokens).

``--full`` additionally runs the full-size cases (config-1 GEMV, the 262144-row
lm_head, and the 35-layer decoder: 1024-token prompt + 256 greedy steps; the
decoder alone takes several minutes of CPU).  Outputs are small ``.npz`` files;
inputs are regenerated from the same seeds by ``slang_b200.synth`` where they
are large, and stored verbatim where they are small.
"""
from __future__ import annotations

import argparse
import os
import sys
import time
from types import SimpleNamespace

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from slang_b200 import synth  # noqa: E402


class _StubIndex:
    """Just enough of ``SafetensorsIndex`` for ``QATIndex.dequant_embedding_*``."""

    def __init__(self, tensors: dict):
        self.t = tensors

    def raw(self, name):
        return self.t[name]

    def tensor(self, name, dtype="f32"):
        return np.asarray(self.t[name]).astype(np.float32)


def ref_dequant(packed, scales, bits):
    """Run the reference's per-block dequant on a synthetic table."""
    from gemma4.qat_loader import QATIndex
    q = QATIndex.__new__(QATIndex)
    q.idx = _StubIndex({"model.t.embedding_quantized": packed,
                        "model.t.embedding_scale": scales})
    n_cols = packed.shape[-1] * 8 // bits
    return q.dequant_embedding_full("t", bits, n_cols)


def kats(out):
    from gemma4.qat_loader import unpack_int2, unpack_int4
    # tests/test_gemma4_qat_loader.py:18-30
    b4 = np.array([0x80, 0xF0, 0x08, 0x7F], np.uint8)
    b2 = np.array([0xE4], np.uint8)
    out["kat_int4_in"], out["kat_int4_out"] = b4, unpack_int4(b4)
    out["kat_int2_in"], out["kat_int2_out"] = b2, unpack_int2(b2)
    rng = np.random.default_rng(5)
    rows = rng.integers(0, 256, (7, 48), dtype=np.uint8)
    out["rand_bytes"] = rows
    out["rand_int4"] = unpack_int4(rows)
    out["rand_int2"] = unpack_int2(rows)


def dequant_cases(out):
    rng = np.random.default_rng(131)
    for bits in (2, 4, 8):
        n_out, n_in = 64, 256
        packed = rng.integers(0, 256, (n_out, n_in * bits // 8), dtype=np.uint8)
        gs = np.abs(rng.normal(0, 0.02, (n_out, n_in // 32))).astype(np.float16)
        rs = (rng.random((n_out, 1)).astype(np.float32) * 0.01 + 0.001)
        if bits == 8:
            # the reference's unpack_bits(., 8) reads a byte as signed int8;
            # our biased code is byte+128 (gemma4_150/export.py:155-157)
            signed = packed.view(np.int8)
            biased = (signed.astype(np.int16) + 128).astype(np.uint8)
            out[f"dq{bits}_packed"] = biased
            ref_in = packed
        else:
            out[f"dq{bits}_packed"] = packed
            ref_in = packed
        out[f"dq{bits}_gscale"], out[f"dq{bits}_rscale"] = gs, rs
        out[f"dq{bits}_f32_group"] = ref_dequant(ref_in, gs, bits)
        out[f"dq{bits}_f32_row"] = ref_dequant(ref_in, rs, bits)


def gemv_cases(out, full):
    # reference test shapes (tests/test_gemma4_qat_kernels_gpu.py:42) with group scales
    # inputs: synth.q4_weight + synth.activations from default_rng(700 + case)
    for i, (n, k) in enumerate([(512, 1536), (2048, 1536), (256, 256)]):
        rng = np.random.default_rng(700 + i)
        packed, scales = synth.q4_weight(rng, n, k)
        x = synth.activations(rng, 1, k)
        w = ref_dequant(packed, scales, 4)
        out[f"gemv_{n}x{k}_y"] = w @ x[0].astype(np.float32)
    if full:
        packed, scales, x = synth.config1(0)
        out["cfg1_y"] = ref_dequant(packed, scales, 4) @ x[0].astype(np.float32)


def gemm_cases(out):
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "ref_test_gemm_dsl", os.path.join(REF, "tests", "test_gemm_dsl.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    for (M, N, K) in mod.SHAPES:
        # inputs regenerate as the reference test's _inputs(M, N, K, seed=0)
        a, b = mod._inputs(M, N, K)
        out[f"gemm_{M}x{N}x{K}_c64"] = mod.reference(a, b, 1.0)
    a, b = mod._inputs(32, 32, 16)
    out["gemm_alpha_c64"] = mod.reference(a, b, 0.375)


def lmhead_case(out):
    packed, scales, h = synth.config3()
    w = ref_dequant(packed, scales, 4)
    logits = w @ h[0].astype(np.float32)
    del w
    order = np.argsort(-logits, kind="stable")[:8]
    out["cfg3_token"] = np.int64(np.argmax(logits))
    out["cfg3_top8_idx"] = order
    out["cfg3_top8_val"] = logits[order]
    out["cfg3_logits_head"] = logits[:4096]


class _RefModel:
    """Build a ``ReferenceGemma4(ple=False)`` serving a ``synth.random_model``."""

    def __init__(self, model, max_seq):
        from gemma4.reference import ReferenceGemma4
        from gemma4.loader import PREFIX
        cfg = model["config"]
        spec = lambda i: SimpleNamespace(  # noqa: E731
            index=i, sliding=bool(cfg["sliding_window"]), head_dim=cfg["head_dim"],
            q_dim=cfg["q_dim"], intermediate=cfg["inter"], rope_theta=cfg["rope_theta"],
            rope_cutoff=cfg["rope_cutoff"], kv_source=i, kv_shared=False)
        config = SimpleNamespace(
            hidden_size=cfg["hidden"], num_layers=cfg["n_layers"], num_heads=cfg["n_heads"],
            num_kv_heads=1, vocab_size=cfg["vocab"], rms_norm_eps=cfg["eps"],
            sliding_window=cfg["sliding_window"] or 1 << 30,
            final_logit_softcapping=cfg["softcap"], embed_scale=cfg["embed_scale"],
            layers=[spec(i) for i in range(cfg["n_layers"])])
        names = {"self_attn.q_proj": "q", "self_attn.k_proj": "k", "self_attn.v_proj": "v",
                 "self_attn.o_proj": "o", "mlp.gate_proj": "gate", "mlp.up_proj": "up",
                 "mlp.down_proj": "down", "input_layernorm": "in_norm",
                 "self_attn.q_norm": "q_norm", "self_attn.k_norm": "k_norm",
                 "post_attention_layernorm": "post_attn_norm",
                 "pre_feedforward_layernorm": "pre_ffn_norm",
                 "post_feedforward_layernorm": "post_ffn_norm"}
        cache = {}

        class Ref(ReferenceGemma4):
            def _w(self, name):
                if name in cache:
                    return cache[name]
                if name == PREFIX + "embed_tokens.weight":
                    v = ref_dequant(model["embed_q"], model["embed_scale"], 4)
                elif name == PREFIX + "norm.weight":
                    v = model["final_norm"]
                else:
                    rest = name[len(PREFIX) + len("layers."):-len(".weight")]
                    li, mod = rest.split(".", 1)
                    item = model["layers"][int(li)][names[mod]]
                    v = ref_dequant(item[0], item[1], 4) if isinstance(item, tuple) else item
                cache[name] = v
                return v

            def _embed_row(self, token_id):
                return ref_dequant(model["embed_q"][token_id:token_id + 1],
                                   model["embed_scale"][token_id:token_id + 1], 4)[0]

        self.ref = Ref(config, None, max_seq=max_seq, ple=False)

    def generate(self, prompt, steps, log_every=0):
        logits = None
        t0 = time.time()
        for pos, t in enumerate(prompt):
            logits = self.ref.forward(int(t), pos)
            if log_every and pos % log_every == 0:
                print(f"  prefill pos {pos} {time.time() - t0:.0f}s", flush=True)
        toks, margins, top, top8_idx, top8_val = [], [], [], [], []
        pos = len(prompt)
        for s in range(steps):
            part = np.partition(logits, -2)[-2:]
            margins.append(float(part[1] - part[0]))
            nxt = int(np.argmax(logits))
            toks.append(nxt)
            top.append(float(logits[nxt]))
            # the 8 largest logits of this step (stable: ties keep the lower id first)
            order = np.argsort(-logits, kind="stable")[:8]
            top8_idx.append(order)
            top8_val.append(logits[order])
            if s + 1 < steps:
                # the reference's own greedy token is fed back (a teacher-forced
                # replay of this run feeds exactly these tokens)
                logits = self.ref.forward(nxt, pos)
                pos += 1
            if log_every and s % 32 == 0:
                print(f"  decode step {s} {time.time() - t0:.0f}s", flush=True)
        self.top8 = (np.array(top8_idx, np.int64), np.array(top8_val, np.float32))
        return np.array(toks, np.int64), np.array(margins, np.float32), np.array(top, np.float32)


PLE_TOKENS = (3, 77, 511)


def ple_cases(out):
    """The per-layer-embedding path through the reference's ``QATReference``
    (``ple=True``) on a 2-layer, hidden-1536, d-256 model: its 8-bit linears go
    through ``QATIndex.dequant_weight`` (bit rule, signed int8 times row scale),
    its table through ``dequant_embedding_row``, the model projection through
    the reference's bf16 conversion.  Inputs regenerate from
    ``synth.random_model(seed=4242)`` and ``synth.ple_weights(seed=4343)``."""
    import math
    from gemma4.loader import PREFIX, bf16_to_f32
    from gemma4.qat_loader import QATIndex
    from gemma4.qat_reference import QATReference
    cfg = synth.e2b_config(hidden=1536, n_layers=2, n_heads=2, head_dim=256, inter=512, vocab=512,
                           rope_cutoff=32)
    model = synth.random_model(cfg, seed=4242)
    ple = synth.ple_weights(hidden=1536, n_layers=2, d=256, vocab=512, seed=4343)
    t = {PREFIX + "embed_tokens_per_layer.embedding_quantized": ple["table"],
         PREFIX + "embed_tokens_per_layer.embedding_scale": ple["table_scale"],
         PREFIX + "per_layer_model_projection.weight": bf16_to_f32(ple["proj"]),
         PREFIX + "per_layer_projection_norm.weight": ple["norm"]}
    for li, L in enumerate(ple["layers"]):
        for mod, key in (("per_layer_input_gate", "gate"), ("per_layer_projection", "proj")):
            codes, scale = L[key]
            # the checkpoint stores signed int8; the biased codes are code - 128
            t[f"{PREFIX}layers.{li}.{mod}.weight"] = (codes.astype(np.int16) - 128).astype(np.int8)
            t[f"{PREFIX}layers.{li}.{mod}.weight_scale"] = scale.reshape(-1, 1)
        t[f"{PREFIX}layers.{li}.post_per_layer_input_norm.weight"] = L["post_norm"]
        t[f"{PREFIX}layers.{li}.layer_scalar"] = np.array([L["scalar"]], np.float32)
    q = QATIndex.__new__(QATIndex)
    q.idx = _StubIndex(t)
    q._names = set(t)
    base = _RefModel(model, 8).ref
    config = SimpleNamespace(**vars(base.cfg), hidden_size_per_layer_input=256, ple_scale=math.sqrt(256))

    class Ref(QATReference):
        def _w(self, name):
            if "per_layer" in name or name.endswith("layer_scalar"):
                return super()._w(name)
            return base._w(name)

        def _embed_row(self, token_id):
            return base._embed_row(token_id)

    ref = Ref(config, q, max_seq=8, ple=True)
    xs, ples, rows = [], [], []
    for tok in PLE_TOKENS:
        x = ref._embed_row(tok) * np.float32(config.embed_scale)
        xs.append(x)
        rows.append(ref._ple_table_row(tok).reshape(-1) * np.float32(config.ple_scale))
        ples.append(ref._ple_input(tok, x))
    out["ple_ids"] = np.array(PLE_TOKENS, np.int64)
    out["ple_x"] = np.stack(xs)
    out["ple_rows"] = np.stack(rows)
    out["ple_in"] = np.stack(ples)
    for li in range(2):
        mids, outs = [], []
        for j, x in enumerate(xs):
            mids.append(ref._layer(x, li, j, None))
            outs.append(ref._layer(x, li, j, ples[j][li]))
        out[f"ple_l{li}_mid"] = np.stack(mids)
        out[f"ple_l{li}_out"] = np.stack(outs)
    # greedy generation through the whole model with the PLE blocks
    gen = Ref(config, q, max_seq=32, ple=True)
    holder = SimpleNamespace(ref=gen)
    prompt = synth.prompt_tokens(6, 512, seed=4444)
    toks, margins, top = _RefModel.generate(holder, prompt, 10)
    out["ple_gen_prompt"] = np.array(prompt, np.int64)
    out["ple_gen_tokens"], out["ple_gen_margins"], out["ple_gen_top"] = toks, margins, top


def decoder_small(out):
    cfg = synth.small_config()
    model = synth.random_model(cfg, seed=77)
    prompt = synth.prompt_tokens(12, cfg["vocab"], seed=78)
    ref = _RefModel(model, 64)
    toks, margins, top = ref.generate(prompt, 16)
    out["dec_small_prompt"] = np.array(prompt, np.int64)
    out["dec_small_tokens"], out["dec_small_margins"], out["dec_small_top"] = toks, margins, top
    out["dec_small_top8_idx"], out["dec_small_top8_val"] = ref.top8


def decoder_full(out, prompt_len, steps):
    cfg = synth.e2b_config()
    model = synth.random_model(cfg, seed=1234)
    prompt = synth.prompt_tokens(prompt_len, cfg["vocab"], seed=99)
    ref = _RefModel(model, prompt_len + steps)
    toks, margins, top = ref.generate(prompt, steps, log_every=64)
    out["cfg4_prompt_len"] = np.int64(prompt_len)
    out["cfg4_tokens"], out["cfg4_margins"], out["cfg4_top"] = toks, margins, top
    out["cfg4_top8_idx"], out["cfg4_top8_val"] = ref.top8
    print(f"  config 4: {len(set(toks.tolist()))} distinct tokens in {steps} steps; "
          f"top-2 margin min {margins.min():.4f}, median {np.median(margins):.3f}", flush=True)


# ---------------------------------------------------------------- reference export
EXPORT_DIR = os.path.join(HERE, "export_small")


def _safetensors(path, tensors):
    """Write ``{name: (dtype tag, array)}`` as a safetensors file (8-byte
    little-endian header length, JSON header, raw little-endian data)."""
    import json
    import struct
    header, blobs, off = {}, [], 0
    for name, (tag, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": tag, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * ((-len(h)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def export_checkpoint(model_dir, H=256, nL=3, nH=2, hd=64, inter=512, vocab=768, d=256, seed=5150,
                      ffn_gain=30.0, layer_types=None, hd_full=None, inters=None, kv_shared=0, window=512):
    """A synthetic QAT checkpoint with the reference checkpoint's tensor names,
    dtypes and bit widths (gemma4_150/loader.py:23-32, 62-73;
    gemma4/qat_loader.py:53-62): 4-bit attention and MLP weights with per-row
    f32 ``weight_scale`` [n_out, 1], 2-bit embedding with [vocab, 1] scales, a
    separate 2-bit ``lm_head.weight`` holding the same codes and scales (so the
    tied head of the weight-only reference and the exported head agree), the
    4-bit per-layer table with one scale per d values, int8 PLE linears, bf16
    norms and per-layer projection, scalar SRQ activation scales.  vocab is a
    multiple of 6 so export.py's [24, -1, 4] lm_head re-layout divides evenly.
    ``layer_types`` (sliding/full per layer), ``hd_full`` (head_dim of the full
    layers), ``inters`` (FFN width per layer), ``kv_shared`` (the last layers
    reading an earlier layer's K/V) and ``window`` give the checkpoint the real
    model's mixed architecture (gemma4/loader.py:104-122)."""
    import json
    from slang_b200.synth import f32_to_bf16_bits, q8_weight
    rng = np.random.default_rng(seed)
    srq_rng = np.random.default_rng(seed + 7)  # SRQ scales: a stream of their own, so weights do not move
    LMP = "model.language_model."
    t = {}

    def bf16(a):
        return ("BF16", f32_to_bf16_bits(np.asarray(a, np.float32)))

    def norm(n, gain=1.0):
        return bf16(gain * (1.0 + 0.1 * rng.standard_normal(n)))

    def codes(n_out, n_in, bits):
        per = 8 // bits
        # codes from 1: zero-mean values, 4-bit in [-7, 7], 2-bit in [-1, 1]
        c = rng.integers(1, 1 << bits, (n_out, n_in), dtype=np.uint8)
        packed = np.zeros((n_out, n_in // per), np.uint8)
        for j in range(per):
            packed |= (c[:, j::per] << (bits * j)).astype(np.uint8)
        return packed

    shared_in = {}

    def act_scales(name):
        # linears fed the same activation (q/k/v; gate/up) share its input scale,
        # as export.py's qkv_in / the reference's MLP input quantisation assume
        a, b = srq_rng.uniform(0.02, 0.08, 2).astype(np.float32)
        key = name.rsplit(".", 1)[0] + (".qkv" if "self_attn" in name and "o_proj" not in name else
                                        ".gateup" if ("gate_proj" in name or "up_proj" in name) else name)
        a = shared_in.setdefault(key, a)
        t[name + ".input_activation_scale"] = ("F32", np.array(a, np.float32))
        t[name + ".output_activation_scale"] = ("F32", np.array(b, np.float32))

    def linear(name, n_out, n_in, bits, lo=0.01, hi=0.03):
        t[name + ".weight"] = ("U8", codes(n_out, n_in, bits))
        t[name + ".weight_scale"] = ("F32", rng.uniform(lo, hi, (n_out, 1)).astype(np.float32))
        act_scales(name)

    emb = codes(vocab, H, 2)
    emb_scale = rng.uniform(0.02, 0.06, (vocab, 1)).astype(np.float32)
    t[LMP + "embed_tokens.embedding_quantized"] = ("U8", emb)
    t[LMP + "embed_tokens.embedding_scale"] = ("F32", emb_scale)
    t["lm_head.weight"] = ("U8", emb.copy())
    t["lm_head.weight_scale"] = ("F32", emb_scale.copy())
    t[LMP + "embed_tokens_per_layer.embedding_quantized"] = ("U8", codes(vocab, nL * d, 4))
    t[LMP + "embed_tokens_per_layer.embedding_scale"] = ("F32", np.abs(rng.normal(0, 0.01, (vocab, nL))).astype(np.float32))
    t[LMP + "per_layer_model_projection.weight"] = bf16(rng.normal(0, 0.02, (nL * d, H)))
    t[LMP + "norm.weight"] = norm(H)
    t[LMP + "per_layer_projection_norm.weight"] = norm(d)
    types = layer_types or ["sliding_attention"] * nL
    first_shared = nL - kv_shared
    for L in range(nL):
        p = f"{LMP}layers.{L}."
        lhd = hd_full if (hd_full and types[L] == "full_attention") else hd
        F = inters[L] if inters else inter
        own = L < first_shared
        for n, size, gain in (("input_layernorm", H, 1.0), ("self_attn.q_norm", lhd, 0.1),
                              ("self_attn.k_norm", lhd, 0.1),
                              ("post_attention_layernorm", H, 1.0), ("pre_feedforward_layernorm", H, 1.0),
                              ("post_feedforward_layernorm", H, ffn_gain), ("post_per_layer_input_norm", H, 1.0)):
            if n == "self_attn.k_norm" and not own:
                continue
            t[p + n + ".weight"] = norm(size, gain)
        t[p + "layer_scalar"] = bf16(rng.uniform(0.7, 1.3, 1))
        for m, n_out, n_in in (("self_attn.q_proj", nH * lhd, H), ("self_attn.k_proj", lhd, H),
                               ("self_attn.v_proj", lhd, H), ("self_attn.o_proj", H, nH * lhd),
                               ("mlp.gate_proj", F, H), ("mlp.up_proj", F, H), ("mlp.down_proj", H, F)):
            if m in ("self_attn.k_proj", "self_attn.v_proj") and not own:
                continue
            linear(p + m, n_out, n_in, 4)
        for m, n_out, n_in in (("per_layer_input_gate", d, H), ("per_layer_projection", H, d)):
            c, sc = q8_weight(rng, n_out, n_in, 0.5 / (74.0 * np.sqrt(n_in)), 1.5 / (74.0 * np.sqrt(n_in)))
            t[p + m + ".weight"] = ("I8", (c.astype(np.int16) - 128).astype(np.int8))
            t[p + m + ".weight_scale"] = ("F32", sc.reshape(-1, 1))
            act_scales(p + m)
    os.makedirs(model_dir, exist_ok=True)
    _safetensors(os.path.join(model_dir, "model.safetensors"), t)
    cfg = {"text_config": {
        "hidden_size": H, "num_hidden_layers": nL, "num_attention_heads": nH, "num_key_value_heads": 1,
        "vocab_size": vocab, "rms_norm_eps": 1e-6, "sliding_window": window, "final_logit_softcapping": 30.0,
        "hidden_size_per_layer_input": d, "bos_token_id": 2, "eos_token_id": 1, "num_kv_shared_layers": kv_shared,
        "layer_types": types,
        "rope_parameters": {"sliding_attention": {"rope_theta": 10000.0},
                            "full_attention": {"rope_theta": 1000000.0, "partial_rotary_factor": 0.25}}}}
    with open(os.path.join(model_dir, "config.json"), "w") as f:
        json.dump(cfg, f)


def srq_case():
    """The reference's ``srq`` on known answers (halves, clipping) and its
    ``ReferenceSRQ._qlin`` on linears of the export_small checkpoint (same
    seeds, so the committed manifest holds the same weights and scales),
    inputs drawn to cover the clip range and the round-half boundaries."""
    import shutil
    import tempfile
    from gemma4_150.loader import Ckpt
    from gemma4_150.reference import ReferenceSRQ, srq
    out = {}
    s = np.float32(0.05)
    kat = np.array([0.0, 0.025, 0.075, -0.025, -0.075, 1.0, 6.35, 6.4, -6.4, -6.45, 100.0, -100.0, 0.0249, 0.0251],
                   np.float32)
    out["srq_kat_x"], out["srq_kat_s"], out["srq_kat_y"] = kat, np.float32(s), srq(kat, float(s))
    tmp = tempfile.mkdtemp(prefix="slang_srq_")
    try:
        export_checkpoint(tmp)
        ref = ReferenceSRQ.__new__(ReferenceSRQ)
        ref.c = Ckpt(tmp)
        rng = np.random.default_rng(9090)
        cases = [(0, "self_attn.q_proj"), (0, "self_attn.k_proj"), (1, "self_attn.o_proj"), (1, "mlp.gate_proj"),
                 (2, "mlp.up_proj"), (2, "mlp.down_proj")]
        for i, (L, mod) in enumerate(cases):
            lin = ref.c.linear(L, mod)
            n_in, s_in = lin["n_in"], lin["in_scale"]
            xs = [rng.standard_normal(n_in).astype(np.float32) * np.float32(s_in * 40),
                  # values near round-half points of x / s_in, and beyond the clip range
                  ((rng.integers(-140, 140, n_in) + 0.5) * s_in).astype(np.float32)]
            for j, x in enumerate(xs):
                y, _ = ref._qlin(x, L, mod)
                out[f"qlin{i}_{j}_x"], out[f"qlin{i}_{j}_y"] = x, y.astype(np.float32)
            out[f"qlin{i}_layer"], out[f"qlin{i}_mod"] = np.int64(L), np.array(mod)
            out[f"qlin{i}_in"], out[f"qlin{i}_out"] = np.float32(s_in), np.float32(lin["out_scale"])
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    np.savez_compressed(os.path.join(HERE, "golden_srq.npz"), **out)
    print("wrote golden_srq.npz", len(out))


ARCH = dict(nL=6, hd=128, hd_full=512, inters=[256, 256, 256, 512, 512, 512], kv_shared=2, window=16, vocab=384,
            layer_types=["sliding_attention", "sliding_attention", "full_attention", "sliding_attention",
                         "sliding_attention", "full_attention"])


def export_case(prompt_len=10, steps=16, out_dir=EXPORT_DIR, ckpt=None, seed=5151):
    """Run the reference's ``gemma4_150.export.export`` on the synthetic
    checkpoint (its manifest.json + weights.bin are the fixture) and the
    reference's weight-only ``QATReference`` (ple=True) on the same checkpoint
    for the expected greedy tokens, margins and per-step top-8 logits."""
    import shutil
    import tempfile
    from gemma4.loader import Gemma4Config
    from gemma4.qat_loader import QATIndex
    from gemma4.qat_reference import QATReference
    from gemma4_150.export import export
    tmp = tempfile.mkdtemp(prefix="slang_export_")
    try:
        export_checkpoint(tmp, **(ckpt or {}))
        written = export(tmp)
        os.makedirs(out_dir, exist_ok=True)
        for name in ("manifest.json", "weights.bin"):
            shutil.copy(os.path.join(written, name), os.path.join(out_dir, name))
        qat = QATIndex(tmp)
        config = Gemma4Config(os.path.join(tmp, "config.json"), qat.idx)
        ref = QATReference(config, qat, max_seq=prompt_len + steps + 1, ple=True)
        holder = SimpleNamespace(ref=ref)
        prompt = synth.prompt_tokens(prompt_len, config.vocab_size, seed=seed)
        toks, margins, top = _RefModel.generate(holder, prompt, steps)
        out = {"prompt": np.array(prompt, np.int64), "tokens": toks, "margins": margins, "top": top,
               "top8_idx": holder.top8[0], "top8_val": holder.top8[1]}
        np.savez_compressed(os.path.join(out_dir, "golden_export.npz"), **out)
        print(f"export case {os.path.basename(out_dir)}: {len(set(toks.tolist()))} distinct tokens in {steps}; "
              f"margins min {margins.min():.4f}; weights.bin {os.path.getsize(os.path.join(out_dir, 'weights.bin'))} B")
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def main():
    global REF
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--full", action="store_true")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    REF = os.path.abspath(args.reference)
    sys.path.insert(0, REF)
    only = set(filter(None, args.only.split(",")))

    def want(n):
        return not only or n in only

    if want("small"):
        out = {}
        kats(out)
        dequant_cases(out)
        gemv_cases(out, full=False)
        gemm_cases(out)
        decoder_small(out)
        np.savez_compressed(os.path.join(HERE, "golden_small.npz"), **out)
        print("wrote golden_small.npz", len(out))
    if want("export"):
        export_case()
    if want("srq"):
        srq_case()
    if want("export_arch"):
        # the real model's mixed layers: sliding (head_dim 128, 16-key window) and
        # full (head_dim 512, partial RoPE) attention, FFN width doubling from
        # layer 3, the last two layers reading layers 3 and 2's K/V
        export_case(prompt_len=24, steps=16, out_dir=os.path.join(HERE, "export_arch"), ckpt=ARCH, seed=5152)
    if want("ple"):
        out = {}
        ple_cases(out)
        np.savez_compressed(os.path.join(HERE, "golden_ple.npz"), **out)
        print("wrote golden_ple.npz", len(out))
    if args.full and want("cfg1"):
        out = {}
        gemv_cases({}, full=False)
        packed, scales, x = synth.config1(0)
        out["cfg1_y"] = ref_dequant(packed, scales, 4) @ x[0].astype(np.float32)
        np.savez_compressed(os.path.join(HERE, "golden_cfg1.npz"), **out)
        print("wrote golden_cfg1.npz")
    if args.full and want("cfg3"):
        out = {}
        lmhead_case(out)
        np.savez_compressed(os.path.join(HERE, "golden_cfg3.npz"), **out)
        print("wrote golden_cfg3.npz")
    if args.full and want("cfg4"):
        out = {}
        decoder_full(out, 1024, 256)
        np.savez_compressed(os.path.join(HERE, "golden_cfg4.npz"), **out)
        print("wrote golden_cfg4.npz")


REF = None

if __name__ == "__main__":
    main()
