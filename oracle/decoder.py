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


class OracleDecoder:
    """Single-position forward with a KV cache (gemma4/reference.py:59-182).

    Without a ``"ple"`` entry in the model this is ``ple=False``; with one (the
    dict of ``slang_b200.synth.ple_weights``) every layer ends with the
    per-layer-embedding block of gemma4/reference.py:154-163, fed by
    ``_ple_input`` (:92-101), as ``oracle.ple`` restates them."""

    def __init__(self, model: dict, max_seq: int) -> None:
        cfg = model["config"]
        self.cfg = cfg
        self.model = model
        self.max_seq = max_seq
        hd = cfg["head_dim"]
        self.k_cache = [np.zeros((max_seq, hd), np.float32) for _ in range(cfg["n_layers"])]
        self.v_cache = [np.zeros((max_seq, hd), np.float32) for _ in range(cfg["n_layers"])]
        self.cos, self.sin = rope_tables(max_seq, hd, cfg["rope_theta"], cfg["rope_cutoff"])
        self._w: dict = {}

    def w(self, layer: int, name: str) -> np.ndarray:
        """Dequantised f32 weight, cached (the reference re-dequantises per call)."""
        key = (layer, name)
        if key not in self._w:
            packed, scales = self.model["layers"][layer][name]
            self._w[key] = q4.dequant_f32(packed, scales, 4)
        return self._w[key]

    def embed(self) -> np.ndarray:
        if "embed" not in self._w:
            self._w["embed"] = q4.dequant_f32(self.model["embed_q"], self.model["embed_scale"], 4)
        return self._w["embed"]

    def layer(self, x: np.ndarray, li: int, pos: int) -> np.ndarray:
        """gemma4/reference.py:103-152 for a layer that owns its K/V."""
        cfg, L = self.cfg, self.model["layers"][li]
        eps, nh, hd = cfg["eps"], cfg["n_heads"], cfg["head_dim"]
        residual = x
        h = rms_norm(x, L["in_norm"], eps)
        q = (self.w(li, "q") @ h).reshape(nh, hd)
        q = rms_norm(q, L["q_norm"], eps)
        q = apply_rope(q, self.cos[pos], self.sin[pos])
        k = (self.w(li, "k") @ h).reshape(1, hd)
        v = (self.w(li, "v") @ h).reshape(1, hd)
        k = rms_norm(k, L["k_norm"], eps)
        k = apply_rope(k, self.cos[pos], self.sin[pos])
        v = rms_norm(v, None, eps)
        self.k_cache[li][pos] = k[0]
        self.v_cache[li][pos] = v[0]
        kv_len = pos + 1
        win = cfg.get("sliding_window", 0)
        start = max(0, kv_len - win) if win else 0
        scores = q @ self.k_cache[li][:kv_len].T  # attention scaling 1.0
        if start > 0:
            scores[:, :start] = -1e9
        scores = scores - scores.max(axis=-1, keepdims=True)
        probs = np.exp(scores)
        probs /= probs.sum(axis=-1, keepdims=True)
        attn = probs @ self.v_cache[li][:kv_len]
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
        x = q4.dequant_f32(self.model["embed_q"][token:token + 1],
                           self.model["embed_scale"][token:token + 1], 4)[0]
        x = x * np.float32(cfg["embed_scale"])
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
        x = rms_norm(x, self.model["final_norm"], cfg["eps"])
        logits = self.embed() @ x
        cap = cfg["softcap"]
        return cap * np.tanh(logits / cap) if cap else logits

    # ------------------------------------------------------------ batched prefill
    def embed_rows(self, tokens) -> np.ndarray:
        """Scaled embedding rows ``[S, H]`` of a prompt (gemma4/reference.py:168)."""
        ids = np.asarray(tokens, dtype=np.int64)
        x = q4.dequant_f32(self.model["embed_q"][ids], self.model["embed_scale"][ids], 4)
        return x * np.float32(self.cfg["embed_scale"])

    def layer_batched(self, x: np.ndarray, li: int) -> np.ndarray:
        """Layer ``li`` for prompt rows at positions 0..S-1 at once: the
        per-position arithmetic of gemma4/reference.py:103-152 (same norms,
        RoPE, scaling 1.0, causal softmax, GEGLU) in the layers-outer order of
        ``PrefillGPU._layer`` (gemma4_150/prefill_gpu.py:316-395); fills this
        layer's KV cache for those positions."""
        cfg, L = self.cfg, self.model["layers"][li]
        eps, nh, hd = cfg["eps"], cfg["n_heads"], cfg["head_dim"]
        S = x.shape[0]
        half = hd // 2
        cos, sin = self.cos[:S, None, :], self.sin[:S, None, :]

        def rope(t):  # [S, heads, hd]
            a, b = t[..., :half], t[..., half:]
            return np.concatenate([a * cos - b * sin, b * cos + a * sin], axis=-1)

        h = rms_norm(x, L["in_norm"], eps)
        q = rope(rms_norm((h @ self.w(li, "q").T).reshape(S, nh, hd), L["q_norm"], eps))
        k = rope(rms_norm((h @ self.w(li, "k").T).reshape(S, 1, hd), L["k_norm"], eps))[:, 0]
        v = rms_norm(h @ self.w(li, "v").T, None, eps)
        self.k_cache[li][:S] = k
        self.v_cache[li][:S] = v
        scores = np.matmul(q.transpose(1, 0, 2), k.T)  # [nh, S, S]; attention scaling 1.0
        i = np.arange(S)
        masked = i[None, :] > i[:, None]
        win = cfg.get("sliding_window", 0)
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
        """Final norm + tied lm_head + softcap of one hidden row (gemma4/reference.py:177-180)."""
        cfg = self.cfg
        logits = self.embed() @ rms_norm(x_last, self.model["final_norm"], cfg["eps"])
        cap = cfg["softcap"]
        return cap * np.tanh(logits / cap) if cap else logits

    def prefill_batched(self, tokens) -> np.ndarray:
        """Layers-outer prefill of a prompt at positions 0..S-1; returns the
        logits of the last position (whose argmax is the first generated token)."""
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
