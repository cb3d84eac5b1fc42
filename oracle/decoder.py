"""numpy restatement of the reference's weight-only Gemma-4 decoder (oracle).

Test infrastructure only: see ``oracle/__init__.py``.

Restates ``ReferenceGemma4`` with ``ple=False`` (gemma4/reference.py:59-182)
with ``QATReference``-style dequantised weights (gemma4/qat_reference.py:17-37):
one position at a time, f32 throughout, tied lm_head, final softcap.  The
model is the dict built by ``slang_b200.synth.random_model`` (int4 weights
with per-group scales, f32 norm weights); every layer owns its K/V (no KV
sharing) and attends to the full causal context unless ``sliding_window`` is
set.
"""
from __future__ import annotations

import numpy as np

from . import q4


def rms_norm(x: np.ndarray, w: np.ndarray | None, eps: float) -> np.ndarray:
    """``x / sqrt(mean(x^2) + eps) * w`` (gemma4/reference.py:19-33)."""
    var = np.mean(x * x, axis=-1, keepdims=True)
    y = x / np.sqrt(var + np.float32(eps))
    return y if w is None else y * w


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """tanh-approximate GELU (gemma3/reference.py:21-22)."""
    return 0.5 * x * (1.0 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


def gelu_tanh_cube(x: np.ndarray) -> np.ndarray:
    """``gelu_tanh`` with the cube as two multiplies (numpy's float power is
    ~40x slower on large arrays); within an ulp or two of ``x**3``."""
    return 0.5 * x * (1.0 + np.tanh(0.7978845608028654 * (x + 0.044715 * (x * x * x))))


def rope_tables(max_pos: int, head_dim: int, theta: float, cutoff: int) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin ``[max_pos, head_dim/2]`` exactly as gemma4/reference.py:44-50 forms them."""
    half = head_dim // 2
    i = np.arange(half, dtype=np.float32)
    inv_freq = 1.0 / theta ** (2.0 * i / head_dim)
    inv_freq[cutoff:] = 0.0
    cos = np.empty((max_pos, half), np.float32)
    sin = np.empty((max_pos, half), np.float32)
    for p in range(max_pos):
        ang = np.float32(p) * inv_freq
        cos[p] = np.cos(ang, dtype=np.float32)
        sin[p] = np.sin(ang, dtype=np.float32)
    return cos, sin


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """rotate_half RoPE on ``[heads, head_dim]`` (gemma4/reference.py:51-52)."""
    half = x.shape[-1] // 2
    a, b = x[:, :half], x[:, half:]
    return np.concatenate([a * cos - b * sin, b * cos + a * sin], axis=-1)


def layer_specs(cfg: dict) -> list[dict]:
    """Per-layer structure: the model's ``layer_specs`` (a manifest written by
    gemma4_150/export.py:159-165 carries one per layer) or the uniform layer of
    the config, every layer owning its K/V."""
    if cfg.get("layer_specs"):
        return cfg["layer_specs"]
    win = cfg.get("sliding_window", 0)
    return [{"head_dim": cfg["head_dim"], "q_dim": cfg["q_dim"], "inter": cfg["inter"], "kv_source": i,
             "sliding": bool(win), "rope_theta": cfg["rope_theta"], "rope_cutoff": cfg["rope_cutoff"]}
            for i in range(cfg["n_layers"])]


def packed_bits(packed: np.ndarray, n_in: int) -> int:
    """Code width of a packed weight from its row length, as the reference's
    ``_dq`` derives it from the buffer size (gemma4_150/prefill_gpu.py:186-196)."""
    bits = packed.shape[-1] * 8 // n_in
    if bits not in (2, 4, 8) or bits * n_in != packed.shape[-1] * 8:
        raise ValueError(f"packed row of {packed.shape[-1]} bytes does not hold {n_in} 2/4/8-bit codes")
    return bits


class OracleDecoder:
    """Single-position forward with a KV cache (gemma4/reference.py:59-182).

    Without a ``"ple"`` entry in the model this is ``ple=False``; with one (the
    dict of ``slang_b200.synth.ple_weights``) every layer ends with the
    per-layer-embedding block of gemma4/reference.py:154-163, fed by
    ``_ple_input`` (:92-101), as ``oracle.ple`` restates them.  Layers follow
    ``layer_specs``: a layer whose ``kv_source`` is another layer computes no
    K/V and attends over that layer's cache (KV sharing, gemma4/reference.py:
    117-131); a sliding layer masks keys older than ``sliding_window``
    (:126-129).  The lm_head is the model's separate ``lm_q`` table when it has
    one (export.py's ``lmhead_blk``), else the tied embedding (:178)."""

    def __init__(self, model: dict, max_seq: int) -> None:
        cfg = model["config"]
        self.cfg = cfg
        self.model = model
        self.max_seq = max_seq
        self.specs = layer_specs(cfg)
        self.k_cache, self.v_cache = [], []
        for i, sp in enumerate(self.specs):
            own = sp["kv_source"] == i
            self.k_cache.append(np.zeros((max_seq, sp["head_dim"]), np.float32) if own else None)
            self.v_cache.append(np.zeros((max_seq, sp["head_dim"]), np.float32) if own else None)
        self._rope: dict = {}
        self.cos, self.sin = self.rope(0)
        self._w: dict = {}

    def rope(self, li: int) -> tuple[np.ndarray, np.ndarray]:
        sp = self.specs[li]
        key = (sp["head_dim"], sp["rope_theta"], sp["rope_cutoff"])
        if key not in self._rope:
            self._rope[key] = rope_tables(self.max_seq, *key)
        return self._rope[key]

    def _n_in(self, layer: int, name: str) -> int:
        sp = self.specs[layer]
        return {"o": sp["q_dim"], "down": sp["inter"]}.get(name, self.cfg["hidden"])

    def w(self, layer: int, name: str) -> np.ndarray:
        """Dequantised f32 weight, cached (the reference re-dequantises per call)."""
        key = (layer, name)
        if key not in self._w:
            packed, scales = self.model["layers"][layer][name]
            self._w[key] = q4.dequant_f32(packed, scales, packed_bits(packed, self._n_in(layer, name)))
        return self._w[key]

    def embed(self) -> np.ndarray:
        """The lm_head table, dequantised once (tied embedding or ``lm_q``)."""
        if "embed" not in self._w:
            m, H = self.model, self.cfg["hidden"]
            packed, scales = (m["lm_q"], m["lm_scale"]) if "lm_q" in m else (m["embed_q"], m["embed_scale"])
            self._w["embed"] = q4.dequant_f32(packed, scales, packed_bits(packed, H))
        return self._w["embed"]

    def embed_row(self, token: int) -> np.ndarray:
        """Unscaled embedding row (``QATReference._embed_row``, gemma4/qat_reference.py:35-37)."""
        m = self.model
        bits = packed_bits(m["embed_q"], self.cfg["hidden"])
        return q4.dequant_f32(m["embed_q"][token:token + 1], m["embed_scale"][token:token + 1], bits)[0]

    def layer(self, x: np.ndarray, li: int, pos: int) -> np.ndarray:
        """gemma4/reference.py:103-152."""
        cfg, L, sp = self.cfg, self.model["layers"][li], self.specs[li]
        eps, nh, hd = cfg["eps"], cfg["n_heads"], sp["head_dim"]
        cos, sin = self.rope(li)
        residual = x
        h = rms_norm(x, L["in_norm"], eps)
        q = (self.w(li, "q") @ h).reshape(nh, hd)
        q = rms_norm(q, L["q_norm"], eps)
        q = apply_rope(q, cos[pos], sin[pos])
        src = sp["kv_source"]
        if src == li:
            k = (self.w(li, "k") @ h).reshape(1, hd)
            v = (self.w(li, "v") @ h).reshape(1, hd)
            k = rms_norm(k, L["k_norm"], eps)
            k = apply_rope(k, cos[pos], sin[pos])
            v = rms_norm(v, None, eps)
            self.k_cache[li][pos] = k[0]
            self.v_cache[li][pos] = v[0]
        kv_len = pos + 1
        win = cfg.get("sliding_window", 0) if sp["sliding"] else 0
        start = max(0, kv_len - win) if win else 0
        scores = q @ self.k_cache[src][:kv_len].T  # attention scaling 1.0
        if start > 0:
            scores[:, :start] = -1e9
        scores = scores - scores.max(axis=-1, keepdims=True)
        probs = np.exp(scores)
        probs /= probs.sum(axis=-1, keepdims=True)
        attn = probs @ self.v_cache[src][:kv_len]
        o = self.w(li, "o") @ attn.reshape(-1)
        x = residual + rms_norm(o, L["post_attn_norm"], eps)
        residual = x
        h = rms_norm(x, L["pre_ffn_norm"], eps)
        g = self.w(li, "gate") @ h
        u = self.w(li, "up") @ h
        d = self.w(li, "down") @ (gelu_tanh(g) * u)
        return residual + rms_norm(d, L["post_ffn_norm"], eps)

    def forward(self, token: int, pos: int, hiddens: list | None = None) -> np.ndarray:
        """Logits for one token at ``pos`` (gemma4/reference.py:165-182)."""
        from . import ple as ople
        cfg = self.cfg
        x = self.embed_row(token) * np.float32(cfg["embed_scale"])
        P = self.model.get("ple")
        if P is not None:
            rows = ople.ple_gather(np.array([token]), P["table"], P["table_scale"], P["ple_scale"])
            ple_in = ople.ple_input(x, rows, P["proj"], P["norm"], cfg["n_layers"], P["d"], cfg["eps"])[0]
        for li in range(cfg["n_layers"]):
            x = self.layer(x, li, pos)
            if P is not None:
                x = ople.ple_block(x[None], ple_in[li][None], P["layers"][li], cfg["eps"])[0]
            if hiddens is not None:
                hiddens.append(x.copy())
        return self.head(x)

    # ------------------------------------------------------------ batched prefill
    def embed_rows(self, tokens) -> np.ndarray:
        """Scaled embedding rows ``[S, H]`` of a prompt (gemma4/reference.py:168)."""
        ids = np.asarray(tokens, dtype=np.int64)
        m = self.model
        bits = packed_bits(m["embed_q"], self.cfg["hidden"])
        x = q4.dequant_f32(m["embed_q"][ids], m["embed_scale"][ids], bits)
        return x * np.float32(self.cfg["embed_scale"])

    def layer_batched(self, x: np.ndarray, li: int) -> np.ndarray:
        """Layer ``li`` for prompt rows at positions 0..S-1 at once: the
        per-position arithmetic of gemma4/reference.py:103-152 (same norms,
        RoPE, scaling 1.0, causal softmax, GEGLU) in the layers-outer order of
        ``PrefillGPU._layer`` (gemma4_150/prefill_gpu.py:316-395); fills this
        layer's KV cache for those positions."""
        cfg, L, sp = self.cfg, self.model["layers"][li], self.specs[li]
        eps, nh, hd = cfg["eps"], cfg["n_heads"], sp["head_dim"]
        S = x.shape[0]
        half = hd // 2
        cos_t, sin_t = self.rope(li)
        cos, sin = cos_t[:S, None, :], sin_t[:S, None, :]

        def rope(t):  # [S, heads, hd]
            a, b = t[..., :half], t[..., half:]
            return np.concatenate([a * cos - b * sin, b * cos + a * sin], axis=-1)

        h = rms_norm(x, L["in_norm"], eps)
        q = rope(rms_norm((h @ self.w(li, "q").T).reshape(S, nh, hd), L["q_norm"], eps))
        src = sp["kv_source"]
        if src == li:
            k = rope(rms_norm((h @ self.w(li, "k").T).reshape(S, 1, hd), L["k_norm"], eps))[:, 0]
            v = rms_norm(h @ self.w(li, "v").T, None, eps)
            self.k_cache[li][:S] = k
            self.v_cache[li][:S] = v
        k, v = self.k_cache[src][:S], self.v_cache[src][:S]
        scores = np.matmul(q.transpose(1, 0, 2), k.T)  # [nh, S, S]; attention scaling 1.0
        i = np.arange(S)
        masked = i[None, :] > i[:, None]
        win = cfg.get("sliding_window", 0) if sp["sliding"] else 0
        if win:
            masked |= i[None, :] < (i[:, None] + 1 - win)
        scores[:, masked] = -np.inf
        scores -= scores.max(axis=-1, keepdims=True)
        probs = np.exp(scores)
        probs /= probs.sum(axis=-1, keepdims=True)
        attn = np.matmul(probs, v).transpose(1, 0, 2).reshape(S, nh * hd)
        x = x + rms_norm(attn @ self.w(li, "o").T, L["post_attn_norm"], eps)
        h = rms_norm(x, L["pre_ffn_norm"], eps)
        a = gelu_tanh_cube(h @ self.w(li, "gate").T) * (h @ self.w(li, "up").T)
        return x + rms_norm(a @ self.w(li, "down").T, L["post_ffn_norm"], eps)

    def head(self, x_last: np.ndarray) -> np.ndarray:
        """Final norm + lm_head + softcap of one hidden row (gemma4/reference.py:177-180)."""
        cfg = self.cfg
        logits = self.embed() @ rms_norm(x_last, self.model["final_norm"], cfg["eps"])
        cap = cfg["softcap"]
        return cap * np.tanh(logits / cap) if cap else logits

    def prefill_batched(self, tokens) -> np.ndarray:
        """Layers-outer prefill of a prompt at positions 0..S-1; returns the
        logits of the last position (whose argmax is the first generated token).
        Without per-layer embeddings only (the PLE input is per token)."""
        if self.model.get("ple") is not None:
            raise ValueError("prefill_batched covers models without per-layer embeddings")
        x = self.embed_rows(tokens)
        for li in range(self.cfg["n_layers"]):
            x = self.layer_batched(x, li)
        return self.head(x[-1])

    def generate(self, prompt: list[int], steps: int) -> tuple[list[int], list[float]]:
        """Token-at-a-time prefill then greedy decode; returns (tokens, top-2 margins)."""
        logits = None
        for pos, t in enumerate(prompt):
            logits = self.forward(int(t), pos)
        out, margins = [], []
        pos = len(prompt)
        for _ in range(steps):
            top2 = np.partition(logits, -2)[-2:]
            margins.append(float(top2[1] - top2[0]))
            nxt = int(q4.argmax_first(logits)[0])
            out.append(nxt)
            logits = self.forward(nxt, pos)
            pos += 1
        return out, margins
