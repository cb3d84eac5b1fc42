"""Seeded synthetic inputs and random-init models for the benchmark configurations.

There is no checkpoint on this machine, so every workload is generated from a
seed with ``numpy.random.default_rng``:

* packed int4 weights of the single-matrix configurations (GEMV, GEMM,
  lm_head): uniform random bytes, i.e. two independent nibbles uniform in
  ``[0, 15]`` -> values uniform in ``[-8, 7]``, low nibble first;
* packed int4 weights of the random-init decoder: nibbles uniform in
  ``[1, 15]`` -> values uniform in ``[-7, 7]`` (zero mean, see ``random_model``);
* per-group-32 scales: ``|N(0, 0.02)|`` rounded to f16, shape ``[n_out, n_in/32]``;
* activations: ``N(0, 1)`` rounded to f16 (or kept f32 for decode);
* norm weights: ``1 + 0.1 * N(0, 1)`` in f32; the decoder's q/k norms are
  ``QK_NORM_GAIN`` times that and its post-feed-forward norm ``POST_FFN_GAIN``
  times that (see ``random_model``).

The Gemma-4-E2B-shaped decoder is uniform: 35 layers, hidden 1536, FFN 6144,
8 query heads and 1 KV head at head_dim 256, full RoPE (theta 1e4), full causal
attention, tied 262144-row lm_head, final logit softcap 30.
"""
from __future__ import annotations

import math

import numpy as np

GROUP = 32

# Gemma-4-E2B-shaped projection matrices: name -> (n_out, n_in)
E2B_SHAPES = {
    "q": (2048, 1536), "k": (256, 1536), "v": (256, 1536), "o": (1536, 2048),
    "gate": (6144, 1536), "up": (6144, 1536), "down": (1536, 6144),
}


def e2b_config(**over) -> dict:
    cfg = dict(hidden=1536, n_layers=35, n_heads=8, head_dim=256, inter=6144,
               vocab=262144, eps=1e-6, rope_theta=10000.0, rope_cutoff=128,
               softcap=30.0, sliding_window=0, group=GROUP)
    cfg.update(over)
    cfg["q_dim"] = cfg["n_heads"] * cfg["head_dim"]
    cfg["embed_scale"] = math.sqrt(cfg["hidden"])
    return cfg


def small_config() -> dict:
    """The small test decoder: hidden 256, 4 layers, 2 query heads of 64, FFN 512,
    vocab 2048; post-feed-forward norm gain 30 (its greedy run moves at every step)."""
    return e2b_config(hidden=256, n_layers=4, n_heads=2, head_dim=64, inter=512, vocab=2048, rope_cutoff=32,
                      post_ffn_gain=30.0)


def mid_config() -> dict:
    """Full-width layers (hidden 1536, 8 heads of 256, FFN 6144) but 4 layers and a
    16384-row vocabulary; post-feed-forward norm gain 30."""
    return e2b_config(n_layers=4, vocab=16384, post_ffn_gain=30.0)


def q4_weight(rng: np.random.Generator, n_out: int, n_in: int,
              group: int = GROUP) -> tuple[np.ndarray, np.ndarray]:
    """Packed int4 ``[n_out, n_in/2]`` u8 and f16 scales ``[n_out, n_in/group]``."""
    packed = rng.integers(0, 256, (n_out, n_in // 2), dtype=np.uint8)
    scales = np.abs(rng.normal(0.0, 0.02, (n_out, n_in // group))).astype(np.float16)
    return packed, scales


def q4_weight_sym(rng: np.random.Generator, n_out: int, n_in: int,
                  group: int = GROUP) -> tuple[np.ndarray, np.ndarray]:
    """As ``q4_weight`` but every nibble uniform in ``[1, 15]``: values uniform
    in ``[-7, 7]``, so the dequantised weight has zero mean."""
    lo = rng.integers(1, 16, (n_out, n_in // 2), dtype=np.uint8)
    hi = rng.integers(1, 16, (n_out, n_in // 2), dtype=np.uint8)
    scales = np.abs(rng.normal(0.0, 0.02, (n_out, n_in // group))).astype(np.float16)
    return (lo | (hi << 4)).astype(np.uint8), scales


# Gains of the random-init decoder's norm weights (see random_model).
QK_NORM_GAIN = 0.1
POST_FFN_GAIN = 12.0


def q2_weight(rng: np.random.Generator, n_out: int, n_in: int,
              group: int = GROUP) -> tuple[np.ndarray, np.ndarray]:
    """Packed 2-bit ``[n_out, n_in/4]`` u8 (four codes per byte, the checkpoint's
    2-bit layout) and f16 scales ``[n_out, n_in/group]``."""
    packed = rng.integers(0, 256, (n_out, n_in // 4), dtype=np.uint8)
    scales = np.abs(rng.normal(0.0, 0.05, (n_out, n_in // group))).astype(np.float16)
    return packed, scales


def activations(rng: np.random.Generator, m: int, k: int, dtype=np.float16) -> np.ndarray:
    return rng.standard_normal((m, k), dtype=np.float32).astype(dtype)


def config1(seed: int = 0):
    """GEMV config: x f16 [1,1536], W int4 [6144,1536], group-32 f16 scales."""
    rng = np.random.default_rng(seed)
    packed, scales = q4_weight(rng, 6144, 1536)
    x = activations(rng, 1, 1536)
    return packed, scales, x


def config2(m: int = 1024, seed: int = 1):
    """Prefill GEMM config: A f16 [m, K] and the seven E2B projections (seeds 1..7)."""
    mats = {}
    for i, (name, (n, k)) in enumerate(E2B_SHAPES.items()):
        rng = np.random.default_rng(seed + i)
        packed, scales = q4_weight(rng, n, k)
        mats[name] = (packed, scales, activations(rng, m, k))
    return mats


def config3(vocab: int = 262144, hidden: int = 1536, seed: int = 3):
    """Tied lm_head config: int4 embedding [vocab, hidden] + f16 hidden [1, hidden]."""
    rng = np.random.default_rng(seed)
    packed, scales = q4_weight(rng, vocab, hidden)
    h = activations(rng, 1, hidden)
    return packed, scales, h


def random_model(cfg: dict | None = None, seed: int = 1234, symmetric: bool = True,
                 qk_gain: float = QK_NORM_GAIN, post_ffn_gain: float | None = None) -> dict:
    """Random-init Gemma-4-E2B-architecture int4 decoder (layer ``L`` uses seed+1+L).

    The recipe is chosen so that greedy decoding neither collapses onto one
    token nor depends chaotically on rounding -- a parity test needs both a
    trajectory that moves and one that an f32 implementation can reproduce:

    * zero-mean codes (``q4_weight_sym``).  With codes uniform in ``[-8, 7]``
      every row has mean ``-0.5 * scale``, so each projection maps the all-ones
      direction onto itself; over 70 sub-layers that direction takes over the
      residual stream (final hidden states at every position have cosine
      0.998) and the tied lm_head picks one token at every step;
    * q/k norm weights ``qk_gain`` (0.1) times ``1 + 0.1 N(0,1)``.  With unit
      gains the RMS-normed q.k scores at head_dim 256 have a standard deviation
      of 16 (the reference's attention scaling is 1.0): attention is nearly
      hard, and a rounding difference of one ulp in layer 0 grows to a 50 %
      difference of the final hidden state (f32 against f64);
    * post-feed-forward norm weights ``post_ffn_gain`` (``cfg["post_ffn_gain"]``
      when the config sets one, else 12) times ``1 + 0.1 N(0,1)``, so the MLP outputs -- a nonlinear function of the
      current token -- outweigh both the token's own embedding (which makes the
      model repeat its input through the tied lm_head) and the near-constant
      soft attention over the prompt (which pins one token).

    At the benchmark shape (seed 1234, the 1024-token prompt of seed 99) f32
    and f64 forwards agree on the logits to 7e-5 and the greedy tokens move at
    every step.
    """
    cfg = dict(cfg or e2b_config())
    if post_ffn_gain is None:
        post_ffn_gain = cfg.get("post_ffn_gain", POST_FFN_GAIN)
    H, qd, hd, F = cfg["hidden"], cfg["q_dim"], cfg["head_dim"], cfg["inter"]
    shapes = {"q": (qd, H), "k": (hd, H), "v": (hd, H), "o": (H, qd),
              "gate": (F, H), "up": (F, H), "down": (H, F)}
    rng = np.random.default_rng(seed)
    qw = q4_weight_sym if symmetric else q4_weight
    embed_q, embed_scale = qw(rng, cfg["vocab"], H, cfg["group"])

    def norm(r, n):
        return (1.0 + 0.1 * r.standard_normal(n, dtype=np.float32)).astype(np.float32)

    final_norm = norm(rng, H)
    layers = []
    for li in range(cfg["n_layers"]):
        r = np.random.default_rng(seed + 1 + li)
        layer = {name: qw(r, n, k, cfg["group"]) for name, (n, k) in shapes.items()}
        for name, n in (("in_norm", H), ("q_norm", hd), ("k_norm", hd), ("post_attn_norm", H),
                        ("pre_ffn_norm", H), ("post_ffn_norm", H)):
            layer[name] = norm(r, n)
            gain = qk_gain if name in ("q_norm", "k_norm") else post_ffn_gain if name == "post_ffn_norm" else 1.0
            layer[name] = (layer[name] * np.float32(gain)).astype(np.float32)
        layers.append(layer)
    return {"config": cfg, "embed_q": embed_q, "embed_scale": embed_scale,
            "final_norm": final_norm, "layers": layers}


def q8_weight(rng: np.random.Generator, n_out: int, n_in: int, lo: float, hi: float) -> tuple[np.ndarray, np.ndarray]:
    """+128-biased int8 codes ``[n_out, n_in]`` u8 (uniform bytes: values uniform
    in ``[-128, 127]``) and per-row f32 scales ``[n_out]`` uniform in ``[lo, hi)``."""
    codes = rng.integers(0, 256, (n_out, n_in), dtype=np.uint8)
    scale = rng.uniform(lo, hi, n_out).astype(np.float32)
    return codes, scale


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round f32 to bf16 (nearest, ties to even) and return the uint16 bit patterns."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def ple_weights(hidden: int = 1536, n_layers: int = 35, d: int = 256, vocab: int = 262144,
                seed: int = 2024) -> dict:
    """Random-init per-layer-embedding weights of the Gemma-4-E2B layout.

    * ``table`` [vocab, n_layers*d/2] u8 4-bit codes with f32 ``table_scale``
      [vocab, n_layers] (one scale per d values, the checkpoint's blocking),
      scales ``|N(0, 0.01)|``;
    * ``proj`` [n_layers*d, hidden] bf16 bit patterns of ``N(0, 0.02)``, ``norm`` [d];
    * per layer (seed + 1 + L): ``gate`` [d, hidden] and ``proj`` [hidden, d]
      8-bit weights (row scales sized so the outputs are O(1) for O(1)
      inputs), ``post_norm`` [hidden] and ``scalar`` uniform in [0.7, 1.3).
    """
    rng = np.random.default_rng(seed)
    cols = n_layers * d
    table = rng.integers(0, 256, (vocab, cols // 2), dtype=np.uint8)
    table_scale = np.abs(rng.normal(0.0, 0.01, (vocab, n_layers))).astype(np.float32)
    proj = f32_to_bf16_bits(rng.normal(0.0, 0.02, (cols, hidden)).astype(np.float32))
    norm = (1.0 + 0.1 * rng.standard_normal(d, dtype=np.float32)).astype(np.float32)
    layers = []
    for li in range(n_layers):
        r = np.random.default_rng(seed + 1 + li)
        gate = q8_weight(r, d, hidden, 0.5 / (74.0 * math.sqrt(hidden)), 1.5 / (74.0 * math.sqrt(hidden)))
        pj = q8_weight(r, hidden, d, 0.5 / (74.0 * math.sqrt(d)), 1.5 / (74.0 * math.sqrt(d)))
        post = (1.0 + 0.1 * r.standard_normal(hidden, dtype=np.float32)).astype(np.float32)
        layers.append({"gate": gate, "proj": pj, "post_norm": post, "scalar": float(r.uniform(0.7, 1.3))})
    return {"hidden": hidden, "n_layers": n_layers, "d": d, "vocab": vocab, "ple_scale": math.sqrt(d),
            "table": table, "table_scale": table_scale, "proj": proj, "norm": norm, "layers": layers}


def prompt_tokens(n: int, vocab: int, seed: int = 99) -> list[int]:
    """Uniform random token ids (the synthetic stand-in for a text prompt)."""
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]
