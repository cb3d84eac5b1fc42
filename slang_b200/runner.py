"""Decode runner and layers-outer prefill for the Gemma-4-E2B-shaped int4 decoder.

Host orchestration mirroring the reference's runners:
  * ``Runner.decode_step`` is ``G4._forward`` (gemma4_150/metal_runner.py:372-402):
    embed -> per layer {norm, q|k|v GEMV, q/k norm + RoPE + cache, attention,
    o GEMV, add+norm, gate|up GEMV, GEGLU, down GEMV, add+norm} -> lm_head
    argmax, for ``batch`` independent sequences; the whole step is captured
    once as a CUDA graph and replayed per token, with positions, current
    tokens and the generated history kept on the device
    (gemma4_150/metal_runner.py:439-468 keeps ``gen`` on the GPU the same way).
  * ``Runner.prefill`` is ``PrefillGPU.prefill`` (gemma4_150/prefill_gpu.py:398-436):
    layers outer, tokens inner; every projection is one fused int4 tcgen05
    GEMM at M = prompt length, attention is one fused causal tcgen05 kernel
    (online softmax, scores never leave the SM); it returns the first greedy
    token.
  * ``Runner.prefill_tokenwise`` feeds the prompt through the decode step one
    token at a time (the reference's per-token path, used when batched prefill
    is off, gemma4_150/metal_runner.py:418-425): f32 activations throughout.

q|k|v and gate|up weights are concatenated at load time so each pair/triple is
one launch (the reference's qkv_70 / gateup_74 fuse the same way).  Every
kernel is a ``libslang_b200.so`` entry point; torch only allocates memory and
provides streams and graphs.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import _lib
from . import kernels as kern

_F16, _F32 = _lib.SB_F16, _lib.SB_F32


def rope_tables(max_pos: int, head_dim: int, theta: float, cutoff: int) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin [max_pos, head_dim/2] in f32, formed as gemma4/reference.py:44-50 does."""
    half = head_dim // 2
    i = np.arange(half, dtype=np.float32)
    inv_freq = 1.0 / theta ** (2.0 * i / head_dim)
    inv_freq[cutoff:] = 0.0
    ang = np.arange(max_pos, dtype=np.float32)[:, None] * inv_freq[None, :]
    return np.cos(ang, dtype=np.float32), np.sin(ang, dtype=np.float32)


def _interleave(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    out = np.empty((a.shape[0] * 2,) + a.shape[1:], dtype=a.dtype)
    out[0::2], out[1::2] = a, b
    return out


def _rows(buf: torch.Tensor, m: int, n: int) -> torch.Tensor:
    """A contiguous [m, n] view at the start of a larger buffer (per-layer widths)."""
    return buf.view(-1)[:m * n].view(m, n)


def layer_specs(cfg: dict) -> list[dict]:
    """Per-layer structure: ``cfg["layer_specs"]`` (a reference export carries
    one per layer, gemma4_150/export.py:159-165) or the config's uniform layer."""
    if cfg.get("layer_specs"):
        return cfg["layer_specs"]
    return [{"head_dim": cfg["head_dim"], "q_dim": cfg["q_dim"], "inter": cfg["inter"], "kv_source": i,
             "sliding": bool(cfg.get("sliding_window", 0)), "rope_theta": cfg["rope_theta"],
             "rope_cutoff": cfg["rope_cutoff"]} for i in range(cfg["n_layers"])]


def _bits(packed: np.ndarray, n_in: int) -> int:
    """Code width of a packed weight from its row length (the reference's ``_dq``
    reads it off the buffer size, gemma4_150/prefill_gpu.py:186-196)."""
    bits = packed.shape[-1] * 8 // n_in
    if bits not in (2, 4) or bits * n_in != packed.shape[-1] * 8:
        raise ValueError(f"a packed row of {packed.shape[-1]} bytes holds no 2- or 4-bit codes of {n_in} values")
    return bits


class DeviceModel:
    """The model's weights on one GPU in the layouts the kernels consume.

    Takes either weight format ``manifest.read`` produces: 4-bit codes with
    per-group-32 f16 scales (the benchmark format) or the reference export's
    per-row f32 scales with 2- or 4-bit codes per matrix, a 2-bit embedding
    with per-block scales and a separate 2-bit lm_head.  Layers follow
    ``layer_specs``: each has its own head_dim, q width and FFN width (the
    checkpoint's full-attention layers have head_dim 512, its layers 15+ a
    double-width 2-bit FFN), may read the K/V of an earlier layer instead of
    computing its own (KV sharing) and may attend over a sliding window."""

    def __init__(self, model: dict, device, max_seq: int):
        cfg = model["config"]
        self.cfg = cfg
        self.device = torch.device(device)
        self.max_seq = max_seq
        dev = self.device
        specs = layer_specs(cfg)
        self._check(cfg, specs, max_seq)
        H = cfg["hidden"]

        def T(a, dtype=None):
            t = torch.from_numpy(np.array(a, copy=True))
            return t.to(device=dev, dtype=dtype) if dtype is not None else t.to(dev)

        self.embed_q = T(model["embed_q"])
        self.embed_s = T(model["embed_scale"])
        self.embed_bits = _bits(model["embed_q"], H)
        self.embed_group = kern.group_of(self.embed_s, H)
        if "lm_q" in model:  # a separate lm_head (export.py's lmhead_blk)
            self.lm_q, self.lm_s = T(model["lm_q"]), T(model["lm_scale"])
        else:  # tied (gemma4/reference.py:178)
            self.lm_q, self.lm_s = self.embed_q, self.embed_s
        self.lm_bits = _bits(self.lm_q, H)
        self.final_norm = T(model["final_norm"], torch.float32)
        self.layers = []
        self._rope: dict = {}
        group32 = self.embed_bits == 4 and self.lm_bits == 4 and self.lm_q is self.embed_q
        win = int(cfg.get("sliding_window", 0) or 0)
        for li, (L, sp) in enumerate(zip(model["layers"], specs)):
            own = sp["kv_source"] == li
            bits = {"qkv": _bits(L["q"][0], H), "o": _bits(L["o"][0], sp["q_dim"]), "gu": _bits(L["gate"][0], H),
                    "down": _bits(L["down"][0], sp["inter"])}
            if (own and (_bits(L["k"][0], H) != bits["qkv"] or _bits(L["v"][0], H) != bits["qkv"])) or \
                    _bits(L["up"][0], H) != bits["gu"]:
                raise ValueError(f"layer {li}: q/k/v (or gate/up) weights of different code widths")
            names = ("q", "k", "v") if own else ("q",)  # a KV-shared layer projects q only
            d = {
                "spec": {"hd": sp["head_dim"], "qd": sp["q_dim"], "F": sp["inter"], "own": own,
                         "src": sp["kv_source"], "window": win if sp["sliding"] else 0,
                         "nqkv": sp["q_dim"] + (2 * sp["head_dim"] if own else 0)},
                "qkv": (T(np.concatenate([L[n][0] for n in names])), T(np.concatenate([L[n][1] for n in names]))),
                "o": (T(L["o"][0]), T(L["o"][1])),
                # gate row i and up row i adjacent: GEGLU pairs neighbouring outputs
                "gu": (T(_interleave(L["gate"][0], L["up"][0])), T(_interleave(L["gate"][1], L["up"][1]))),
                "down": (T(L["down"][0]), T(L["down"][1])),
                "bits": bits,
            }
            for n in ("in_norm", "q_norm", "k_norm", "post_attn_norm", "pre_ffn_norm", "post_ffn_norm"):
                d[n] = T(L[n], torch.float32) if n in L else None  # a KV-shared layer has no k_norm
            key = (sp["rope_theta"], sp["rope_cutoff"])
            if key not in self._rope:
                cos, sin = rope_tables(max_seq, sp["head_dim"], *key)
                self._rope[key] = (T(cos), T(sin))
            d["cos"], d["sin"] = self._rope[key]
            group32 = group32 and all(b == 4 for b in bits.values()) and all(
                d[k][1].dtype == torch.float16 and kern.group_of(d[k][1], d[k][0].shape[1] * 2) == 32
                for k in ("qkv", "o", "gu", "down"))
            self.layers.append(d)
        self.cos, self.sin = self.layers[0]["cos"], self.layers[0]["sin"]
        # the persistent one-launch decode step and the GEMM-argmax lm_head take
        # the benchmark format only (4-bit codes, f16 group-32 scales, tied table)
        # and layers of one shape that own their K/V with no window in reach
        sp0 = self.layers[0]["spec"]
        self.uniform = all(d["spec"]["own"] and (d["spec"]["hd"], d["spec"]["qd"], d["spec"]["F"]) ==
                           (sp0["hd"], sp0["qd"], sp0["F"]) and (not d["spec"]["window"] or
                                                                 max_seq <= d["spec"]["window"])
                           for d in self.layers)
        self.group32_f16 = group32 and self.embed_s.dtype == torch.float16 and self.embed_group == 32 and self.uniform
        # per-layer embeddings (the dict of synth.ple_weights or of a reference export), when the model has them
        self.ple = None
        P = model.get("ple")
        if P is not None:
            if P["proj"].dtype == np.float16:  # export.py's f16 cast (gemma4_150/export.py:95)
                proj = proj16 = T(P["proj"])
            else:  # the checkpoint's bf16 bit patterns
                proj = T(P["proj"].view(np.int16))
                proj16 = proj.view(torch.bfloat16).to(torch.float16)  # for the prefill GEMM (made once, at load)
            self.ple = {"table": T(P["table"]), "table_scale": T(P["table_scale"], torch.float32), "proj": proj,
                        "proj16": proj16, "norm": T(P["norm"], torch.float32), "scale": float(P["ple_scale"]),
                        "d": int(P["d"])}
            for d, PL in zip(self.layers, P["layers"]):
                d["ple"] = {"gate": (T(PL["gate"][0]), T(PL["gate"][1], torch.float32)),
                            "proj": (T(PL["proj"][0]), T(PL["proj"][1], torch.float32)),
                            "post_norm": T(PL["post_norm"], torch.float32), "scalar": float(PL["scalar"])}

    @staticmethod
    def _check(cfg: dict, specs: list, max_seq: int) -> None:
        for i, sp in enumerate(specs):
            src = sp["kv_source"]
            if src != i and (src > i or specs[src]["kv_source"] != src or specs[src]["head_dim"] != sp["head_dim"]):
                raise ValueError(f"layer {i} reads the K/V of layer {src}, which must be an earlier layer of the same "
                                 "head_dim that owns its K/V")
            if sp["q_dim"] % sp["head_dim"] or sp["q_dim"] // sp["head_dim"] != cfg["n_heads"]:
                raise ValueError(f"layer {i}: q_dim {sp['q_dim']} is not n_heads x head_dim")

    def embed(self, tokens_ptr: int, m: int, out32, out16, stream: int) -> None:
        """Scaled embedding rows of ``m`` tokens (``embed_00``, gemma4/reference.py:168)."""
        fn = "sb_embed_q4" if self.embed_bits == 4 else "sb_embed_q2"
        _lib.call(fn, self.embed_q.data_ptr(), self.embed_s.data_ptr(), kern._DT[self.embed_s.dtype],
                  self.embed_group, tokens_ptr, m, self.cfg["hidden"], float(self.cfg["embed_scale"]), out32, out16,
                  stream)

    def lmhead_argmax(self, h, keys, tokens, logits=None):
        """lm_head GEMV + greedy argmax of hidden rows ``h``."""
        return kern.lmhead_argmax(self.lm_q, self.lm_s, h, keys=keys, tokens=tokens, logits=logits, bits=self.lm_bits)


class Runner:
    """Decode (and prefill) state for ``batch`` sequences.

    ``proj`` picks the decode projections: "gemv" (the int4 GEMV, 1..8
    sequences, f32 activations), "gemm" (the fused int4 tcgen05 GEMM at
    M = batch with f16 activations and the lm_head argmax in the GEMM
    epilogue, any batch) or "auto" (GEMV up to 8 sequences, GEMM above)."""

    MAX_BATCH = 1024

    # the o and down GEMVs of the GEMV decode path carry the residual add + RMSNorm
    # as a last-arriver tail (sb_gemv_norm_add) instead of a separate kernel
    NORM_TAILS = False

    def __init__(self, dm: DeviceModel, batch: int = 1, fused: bool = False, proj: str = "auto",
                 norm_tails: bool | None = None):
        if proj == "auto":
            proj = "gemv" if batch <= 8 else "gemm"
        if proj not in ("gemv", "gemm"):
            raise ValueError("proj must be 'gemv', 'gemm' or 'auto'")
        if batch < 1 or batch > self.MAX_BATCH or (proj == "gemv" and batch > 8):
            raise ValueError("the GEMV decode path serves 1..8 sequences, the GEMM path 1..%d" % self.MAX_BATCH)
        if fused and batch != 1:
            raise ValueError("the persistent decode kernel serves one sequence")
        if dm.ple is not None and (fused or proj != "gemv"):
            raise ValueError("per-layer embeddings run on the per-op GEMV decode path (fused=False, proj='gemv')")
        if (fused or proj == "gemm") and not dm.group32_f16:
            raise ValueError("the persistent decode step and the GEMM decode path take 4-bit weights with f16 "
                             "group-32 scales, a tied lm_head and uniform layers that own their K/V; use "
                             "fused=False, proj='gemv'")
        self.proj = proj
        self.fused = fused
        self.norm_tails = self.NORM_TAILS if norm_tails is None else bool(norm_tails)
        self.dm = dm
        cfg = dm.cfg
        self.B = batch
        specs = [L["spec"] for L in dm.layers]
        # buffer sizes: the largest layer (layers may differ in head_dim, q and FFN width)
        self.H, self.nh = cfg["hidden"], cfg["n_heads"]
        self.hd = max(sp["hd"] for sp in specs)
        self.F = max(sp["F"] for sp in specs)
        self.qd = max(sp["qd"] for sp in specs)
        self.nqkv = max(sp["nqkv"] for sp in specs)
        self.eps = float(cfg["eps"])
        self.max_seq = dm.max_seq
        dev = dm.device
        B, H, S = batch, self.H, self.max_seq
        self.cache_stride = S * self.hd
        nL = cfg["n_layers"]
        # K/V caches [B, max_seq, head_dim] per layer that owns its K/V; a
        # KV-shared layer holds its source layer's tensors
        self.kc, self.vc = [], []
        for li, sp in enumerate(specs):
            if sp["own"]:
                self.kc.append(torch.zeros((B, S, sp["hd"]), dtype=torch.float32, device=dev))
                self.vc.append(torch.zeros((B, S, sp["hd"]), dtype=torch.float32, device=dev))
            else:
                self.kc.append(self.kc[sp["src"]])
                self.vc.append(self.vc[sp["src"]])
        f32 = lambda *s: torch.zeros(s, dtype=torch.float32, device=dev)  # noqa: E731
        self.x, self.h = f32(B, H), f32(B, H)
        self.qkv, self.q = f32(B, self.nqkv), f32(B, self.qd)
        self.attn, self.o = f32(B, self.qd), f32(B, H)
        self.gu, self.a, self.d = f32(B, 2 * self.F), f32(B, self.F), f32(B, H)
        if dm.ple is not None:
            pd = dm.ple["d"]
            self.ple_in, self.ple_ctx = f32(B, nL, pd), f32(B, nL * pd)
            self.ple_g, self.ple_proj = f32(B, pd), f32(B, H)
            self.ple_counter = torch.zeros(1, dtype=torch.int32, device=dev)  # last-arriver count, self re-arming
        if proj == "gemm":
            f16 = lambda *s: torch.zeros(s, dtype=torch.float16, device=dev)  # noqa: E731
            self.h16, self.qkv16, self.attn16 = f16(B, H), f16(B, self.nqkv), f16(B, self.qd)
            self.o16, self.a16, self.d16 = f16(B, H), f16(B, self.F), f16(B, H)
            ws = max(kern.gemm_q4_workspace_size(B, n, k) for n, k in
                     ((self.nqkv, H), (H, self.qd), (2 * self.F, H), (H, self.F)))
            self.gemm_ws = torch.empty(max(1, ws // 4), dtype=torch.float32, device=dev) if ws else None
        self.tail_counter = torch.zeros(1, dtype=torch.int32, device=dev)  # last-arriver count, self re-arming
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.cur = torch.zeros(B, dtype=torch.int32, device=dev)
        self.tok = torch.zeros(B, dtype=torch.int32, device=dev)
        self.keys = torch.zeros(B, dtype=torch.int64, device=dev)
        self.history = torch.zeros((B, S), dtype=torch.int32, device=dev)
        ws = max(_lib.load().sb_attn_decode_workspace_size(B, self.nh, sp["hd"], S) for sp in specs)
        self.attn_ws = torch.empty(max(1, ws // 4), dtype=torch.float32, device=dev)
        self.stream = torch.cuda.Stream(device=dev)
        if fused:
            self._fused_setup()
        self.graph = None
        self._pf = None  # prefill buffers, sized on first use
        self._pgraphs: dict = {}  # (prompt length, sequence) -> captured prefill

    # ------------------------------------------------------------------ decode
    def _gemv(self, L, key, x, y):
        kern.gemv_q4(L[key][0], L[key][1], x, y=y, bits=L["bits"][key])

    def _decode_ops_gemm(self):
        """One decode step for the batch on the tcgen05 GEMM: f16 activations
        between the projections, the lm_head argmax in the GEMM epilogue."""
        dm, L0 = self.dm, self.dm.layers
        s = kern._stream()
        B, H = self.B, self.H
        ws = self.gemm_ws

        def proj(w, A, C, geglu=False):
            kern.gemm_q4(A, w[0], w[1], C=C, workspace=ws, geglu=geglu)

        dm.embed(self.cur.data_ptr(), B, self.x.data_ptr(), None, s)
        _lib.call("sb_add_rmsnorm", self.x.data_ptr(), None, _F32, None, L0[0]["in_norm"].data_ptr(),
                  self.x.data_ptr(), None, self.h16.data_ptr(), B, H, self.eps, s)
        for li, L in enumerate(L0):
            proj(L["qkv"], self.h16, self.qkv16)
            _lib.call("sb_qkv_prep", self.qkv16.data_ptr(), _F16, self.nqkv, L["q_norm"].data_ptr(),
                      L["k_norm"].data_ptr(), L["cos"].data_ptr(), L["sin"].data_ptr(), self.pos.data_ptr(), 0, B,
                      self.nh, self.hd, self.eps, None, self.q.data_ptr(), self.kc[li].data_ptr(),
                      self.vc[li].data_ptr(), None, None, self.cache_stride, s)
            _lib.call("sb_attn_decode_f16", self.q.data_ptr(), self.kc[li].data_ptr(), self.vc[li].data_ptr(),
                      self.cache_stride, self.pos.data_ptr(), B, self.nh, self.hd, self.max_seq, 0,
                      self.attn16.data_ptr(), self.attn_ws.data_ptr(), self.attn_ws.numel() * 4, s)
            proj(L["o"], self.attn16, self.o16)
            _lib.call("sb_add_rmsnorm", self.x.data_ptr(), self.o16.data_ptr(), _F16, L["post_attn_norm"].data_ptr(),
                      L["pre_ffn_norm"].data_ptr(), self.x.data_ptr(), None, self.h16.data_ptr(), B, H, self.eps, s)
            proj(L["gu"], self.h16, self.a16, geglu=True)
            proj(L["down"], self.a16, self.d16)
            nxt = L0[li + 1]["in_norm"] if li + 1 < len(L0) else dm.final_norm
            _lib.call("sb_add_rmsnorm", self.x.data_ptr(), self.d16.data_ptr(), _F16, L["post_ffn_norm"].data_ptr(),
                      nxt.data_ptr(), self.x.data_ptr(), None, self.h16.data_ptr(), B, H, self.eps, s)
        kern.gemm_q4_argmax(self.h16, dm.embed_q, dm.embed_s, keys=self.keys, tokens=self.tok)
        _lib.call("sb_step_advance", self.pos.data_ptr(), self.tok.data_ptr(), self.cur.data_ptr(),
                  self.history.data_ptr(), self.max_seq, B, s)

    def _decode_ops(self):
        if self.proj == "gemm":
            return self._decode_ops_gemm()
        dm, L0 = self.dm, self.dm.layers
        s = kern._stream()
        lib = _lib.load()
        B, H = self.B, self.H
        dm.embed(self.cur.data_ptr(), B, self.x.data_ptr(), None, s)
        P = dm.ple
        if P is not None:  # per-layer inputs from the scaled embedding (gemma4/reference.py:170)
            kern.ple_input(self.x, self.cur, P["table"], P["table_scale"], P["proj"], P["norm"], len(L0), P["d"],
                           self.eps, P["scale"], out=self.ple_in, ctx=self.ple_ctx)
        _lib.call("sb_add_rmsnorm", self.x.data_ptr(), None, _F32, None, L0[0]["in_norm"].data_ptr(),
                  self.x.data_ptr(), self.h.data_ptr(), None, B, H, self.eps, s)
        for li, L in enumerate(L0):
            sp = L["spec"]
            hd, qd, F, nqkv = sp["hd"], sp["qd"], sp["F"], sp["nqkv"]
            qkv, q, attn = _rows(self.qkv, B, nqkv), _rows(self.q, B, qd), _rows(self.attn, B, qd)
            gu, a = _rows(self.gu, B, 2 * F), _rows(self.a, B, F)
            self._gemv(L, "qkv", self.h, qkv)
            # a KV-shared layer prepares q only and attends over its source layer's cache
            _lib.call("sb_qkv_prep", qkv.data_ptr(), _F32, nqkv, L["q_norm"].data_ptr(),
                      L["k_norm"].data_ptr() if sp["own"] else None, L["cos"].data_ptr(), L["sin"].data_ptr(),
                      self.pos.data_ptr(), 0, B, self.nh, hd, self.eps, None, q.data_ptr(),
                      self.kc[li].data_ptr() if sp["own"] else None, self.vc[li].data_ptr() if sp["own"] else None,
                      None, None, self.max_seq * hd, s)
            _lib.call("sb_attn_decode", q.data_ptr(), self.kc[li].data_ptr(), self.vc[li].data_ptr(),
                      self.max_seq * hd, self.pos.data_ptr(), B, self.nh, hd, self.max_seq, sp["window"],
                      attn.data_ptr(), self.attn_ws.data_ptr(), self.attn_ws.numel() * 4, s)
            nxt = L0[li + 1]["in_norm"] if li + 1 < len(L0) else dm.final_norm
            if self.norm_tails:
                kern.gemv_norm_add(L["o"][0], L["o"][1], attn, self.x, L["post_attn_norm"], self.eps,
                                   w_next=L["pre_ffn_norm"], h_out=self.h, y=self.o, counter=self.tail_counter,
                                   bits=L["bits"]["o"])
            else:
                self._gemv(L, "o", attn, self.o)
                _lib.call("sb_add_rmsnorm", self.x.data_ptr(), self.o.data_ptr(), _F32,
                          L["post_attn_norm"].data_ptr(), L["pre_ffn_norm"].data_ptr(), self.x.data_ptr(),
                          self.h.data_ptr(), None, B, H, self.eps, s)
            self._gemv(L, "gu", self.h, gu)
            _lib.call("sb_geglu", gu.data_ptr(), _F32, B, F, a.data_ptr(), None, s)
            if self.norm_tails:
                kern.gemv_norm_add(L["down"][0], L["down"][1], a, self.x, L["post_ffn_norm"], self.eps, w_next=nxt,
                                   h_out=self.h, y=self.d, counter=self.tail_counter, bits=L["bits"]["down"])
            else:
                self._gemv(L, "down", a, self.d)
                _lib.call("sb_add_rmsnorm", self.x.data_ptr(), self.d.data_ptr(), _F32,
                          L["post_ffn_norm"].data_ptr(), nxt.data_ptr(), self.x.data_ptr(), self.h.data_ptr(), None,
                          B, H, self.eps, s)
            if P is not None:  # PLE block, then the next norm from its output (gemma4/reference.py:154-163)
                Lp = L["ple"]
                kern.gemv_q8(Lp["gate"][0], Lp["gate"][1], self.x, out=self.ple_g, ple=self.ple_in[:, li])
                if B <= kern.PLE_FUSED_TAIL_ROWS:
                    kern.ple_proj_norm_add(Lp["proj"][0], Lp["proj"][1], self.ple_g, self.x, Lp["post_norm"],
                                           Lp["scalar"], self.eps, w_next=nxt, h_out=self.h, proj=self.ple_proj,
                                           counter=self.ple_counter)
                else:
                    kern.gemv_q8(Lp["proj"][0], Lp["proj"][1], self.ple_g, out=self.ple_proj)
                    kern.ple_norm_add(self.ple_proj, self.x, Lp["post_norm"], Lp["scalar"], self.eps, w_next=nxt,
                                      h_out=self.h)
        dm.lmhead_argmax(self.h, self.keys, self.tok)
        _lib.call("sb_step_advance", self.pos.data_ptr(), self.tok.data_ptr(), self.cur.data_ptr(),
                  self.history.data_ptr(), self.max_seq, B, s)
        del lib

    def _fused_setup(self):
        dm, dev = self.dm, self.dm.device
        rows = []
        for li, L in enumerate(dm.layers):
            ptrs = [L[k][0].data_ptr() for k in ("qkv", "o", "gu", "down")]
            ptrs += [L[k][1].data_ptr() for k in ("qkv", "o", "gu", "down")]
            ptrs += [L[n].data_ptr() for n in ("in_norm", "q_norm", "k_norm", "post_attn_norm", "pre_ffn_norm",
                                                "post_ffn_norm")]
            ptrs += [self.kc[li].data_ptr(), self.vc[li].data_ptr()]
            rows.append(ptrs)
        self.layer_table = torch.tensor(rows, dtype=torch.int64, device=dev)
        need = _lib.load().sb_decode_step_fused_scratch_size(self.H, self.nh, self.hd, self.F, self.max_seq)
        if need == 0:
            raise ValueError("this model shape is not supported by the persistent decode kernel")
        self.fused_scratch = torch.zeros(need, dtype=torch.uint8, device=dev)

    def _fused_ops(self):
        dm = self.dm
        _lib.call("sb_decode_step_fused", self.layer_table.data_ptr(), len(dm.layers), dm.embed_q.data_ptr(),
                  dm.embed_s.data_ptr(), dm.final_norm.data_ptr(), dm.cos.data_ptr(), dm.sin.data_ptr(), self.H,
                  self.nh, self.hd, self.F, dm.cfg["vocab"], self.max_seq, self.eps, float(dm.cfg["embed_scale"]),
                  self.pos.data_ptr(), self.cur.data_ptr(), self.tok.data_ptr(), self.history.data_ptr(),
                  self.max_seq, self.keys.data_ptr(), self.fused_scratch.data_ptr(), self.fused_scratch.numel(),
                  kern._stream())

    def kernel_launches_per_step(self) -> int:
        if self.fused:
            return 1
        nL = len(self.dm.layers)
        if self.proj == "gemm":
            B, H, F = self.B, self.H, self.F
            split = lambda n, k: kern.gemm_q4_kernels(B, n, k) - 1  # noqa: E731
            per_layer = (4 + split(self.nqkv, H) + split(H, self.qd) + split(2 * F, H) + split(H, F)
                         + 1 + 2 + 2)  # prep, attention (2), add+norm (2)
            return 2 + nL * per_layer + 2 + 1  # embed + norm, layers, argmax GEMM + tokens, advance
        per_layer = 4 + 1 + 2 + (0 if self.norm_tails else 2) + 1  # 4 GEMVs, prep, attention (2), add+norm (2), geglu
        per_ple = 2 if self.B <= kern.PLE_FUSED_TAIL_ROWS else 3  # per layer: gate GEMV, projection GEMV (+ fused tail)
        ple = 0 if self.dm.ple is None else 2 + per_ple * nL  # + PLE input (GEMV + combine)
        return 2 + nL * per_layer + 2 + 1 + ple  # embed + first norm, layers, lm_head (gemv + tokens), advance

    def capture(self):
        """Warm up, then capture one decode step as a CUDA graph."""
        ops = self._fused_ops if self.fused else self._decode_ops
        with torch.cuda.stream(self.stream):
            saved = (self.pos.clone(), self.cur.clone(), self.history.clone())
            ops()  # first calls set kernel attributes outside capture
            self.pos.copy_(saved[0])
            self.cur.copy_(saved[1])
            self.history.copy_(saved[2])
        torch.cuda.synchronize(self.dm.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            ops()
        return self.graph

    def decode_step(self):
        if self.graph is None:
            self.capture()
        with torch.cuda.stream(self.stream):
            self.graph.replay()

    def decode(self, steps: int) -> torch.Tensor:
        """Greedy-decode `steps` tokens for every sequence; returns [B, steps] (device)."""
        start = self.pos.clone()
        for _ in range(steps):
            self.decode_step()
        torch.cuda.current_stream().wait_stream(self.stream)
        out = torch.stack([self.history[b, int(start[b]) + 1:int(start[b]) + 1 + steps] for b in range(self.B)])
        return out

    def set_state(self, cur, pos):
        with torch.cuda.stream(self.stream):
            self.cur.copy_(torch.as_tensor(cur, dtype=torch.int32))
            self.pos.copy_(torch.as_tensor(pos, dtype=torch.int32))
            for b in range(self.B):
                self.history[b, int(pos[b])] = int(cur[b])

    # ------------------------------------------------------------------ prefill
    def prefill_tokenwise(self, tokens, seq: int = 0) -> int:
        """Run the prompt through the decode step one token at a time (f32 path).

        Only valid for batch == 1 (the step advances every sequence)."""
        if self.B != 1:
            raise ValueError("token-wise prefill drives the whole batch; use batch=1")
        for p, t in enumerate(tokens):
            self.set_state([t], [p])
            self.decode_step()
        torch.cuda.current_stream().wait_stream(self.stream)
        return int(self.tok[0].item())

    def _attn_route(self, sp, S) -> str:
        """Prefill attention of a layer: the fused tcgen05 kernel, or -- for
        head_dim 512 or a sliding window that masks keys at this length -- the
        reference's QK^T -> masked softmax -> PV GEMM chain
        (gemma4_150/prefill_gpu.py:259-313)."""
        return "fused" if sp["hd"] <= 256 and (not sp["window"] or S <= sp["window"]) else "gemm"

    def _prefill_buffers(self, S):
        if self._pf is not None and self._pf["S"] >= S:
            return self._pf
        dev = self.dm.device
        H, F, nh = self.H, self.F, self.nh
        specs = [L["spec"] for L in self.dm.layers]
        f16 = lambda *s: torch.empty(s, dtype=torch.float16, device=dev)  # noqa: E731
        f32 = lambda *s: torch.empty(s, dtype=torch.float32, device=dev)  # noqa: E731
        # per-layer widths vary: activations live in flat buffers of the widest layer
        pf = {"S": S,
              "tok": torch.empty(S, dtype=torch.int32, device=dev),
              "tok_host": torch.empty(S, dtype=torch.int32, pin_memory=True),
              "hid": f32(S, H), "h16": f16(S, H), "hlast": f32(S, H),
              "qkv16": f16(S * self.nqkv), "q16": f16(S * self.qd), "attn16": f16(S * self.qd), "o16": f16(S, H),
              "a16": f16(S * F), "d16": f16(S, H)}
        # f16 K/V for the attention: one scratch pair per head_dim, and a pair of
        # its own for every layer whose K/V a later (KV-shared) layer reads
        sources = {sp["src"] for sp in specs if not sp["own"]}
        pf["kv16"] = {}
        for li, sp in enumerate(specs):
            if sp["own"]:
                key = li if li in sources else ("hd", sp["hd"])
                if key not in pf["kv16"]:
                    pf["kv16"][key] = (f16(self.max_seq, sp["hd"]), f16(self.max_seq, sp["hd"]))
        ws = max(kern.gemm_q4_workspace_size(S, n, k) for sp in specs for n, k in
                 ((sp["nqkv"], H), (H, sp["qd"]), (2 * sp["F"], H), (H, sp["F"])))
        pf["ws"] = torch.empty(max(1, ws // 4), dtype=torch.float32, device=dev)
        if self.dm.ple is not None:
            pd, nL = self.dm.ple["d"], len(self.dm.layers)
            pf["ple_x16"], pf["ple_ctx"], pf["ple_in"] = f16(S, H), f32(S, nL * pd), f32(S, nL, pd)
        aws = max([_lib.load().sb_attn_prefill_workspace_size(S, nh, sp["hd"]) for sp in specs
                   if self._attn_route(sp, S) == "fused"] + [0])
        pf["attn_ws"] = torch.empty(max(4, aws // 4), dtype=torch.float32, device=dev)
        if any(self._attn_route(sp, S) == "gemm" for sp in specs):
            ld = (S + 7) // 8 * 8
            pf["scores"], pf["p16"] = f32(S * nh * ld), f16(S * nh * ld)
        self._pf = pf
        self._pgraphs.clear()  # captured prefills point at the old buffers
        return pf

    def prefill(self, tokens, seq: int = 0, graph: bool = True) -> int:
        """Layers-outer prefill of one prompt into sequence `seq` (positions 0..S-1).

        Returns the first greedy token and leaves the sequence ready to decode
        (cur = that token, pos = S).  The device work of a prompt length is
        captured as a CUDA graph on its first call and replayed afterwards; a
        call copies the prompt from pinned host memory and reads back one token."""
        S = len(tokens)
        if S < 1 or S >= self.max_seq:
            raise ValueError("prompt length out of range")
        pf = self._prefill_buffers(S)
        key = (S, seq)
        with torch.cuda.stream(self.stream):
            pf["tok_host"][:S].copy_(torch.as_tensor(list(tokens), dtype=torch.int32))
            pf["tok"][:S].copy_(pf["tok_host"][:S], non_blocking=True)
            g = self._pgraphs.get(key) if graph else None
            if g is not None:
                g.replay()
            else:
                self._prefill_step(pf, S, seq)
                if graph:
                    torch.cuda.synchronize(self.dm.device)
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=self.stream):
                        self._prefill_step(pf, S, seq)
                    self._pgraphs[key] = g
        torch.cuda.current_stream().wait_stream(self.stream)
        return int(self.tok[seq].item())

    def prefill_graph(self, S: int, seq: int = 0):
        """The captured prefill of length S (after one `prefill` call of that length)."""
        return self._pgraphs[(S, seq)]

    def _prefill_step(self, pf, S, seq, rec=None):
        dm = self.dm
        s = kern._stream()
        self._prefill_ops(pf, S, seq, s, rec)
        # first greedy token from the last prompt position
        dm.lmhead_argmax(pf["hlast"][S - 1:S], self.keys[seq:seq + 1], self.tok[seq:seq + 1])
        self.cur[seq:seq + 1].copy_(self.tok[seq:seq + 1])
        self.pos[seq:seq + 1].fill_(S)
        self.history[seq, S:S + 1].copy_(self.tok[seq:seq + 1])

    def prefill_launches(self, S: int) -> int:
        """Kernels of this library launched by one prefill of length S."""
        H = self.H
        split = lambda n, k: kern.gemm_q4_kernels(S, n, k) - 1  # noqa: E731
        total = 0
        for L in self.dm.layers:
            sp = L["spec"]
            total += (4 + split(sp["nqkv"], H) + split(H, sp["qd"]) + split(2 * sp["F"], H) + split(H, sp["F"])
                      + 1 + 2)  # 4 projections (+ split-K finalizes); prep; two add+norms (GEGLU in the GEMM)
            if self._attn_route(sp, S) == "fused":
                total += 1 + (1 if _lib.load().sb_attn_prefill_workspace_size(S, self.nh, sp["hd"]) else 0)
            else:
                total += 3  # scores GEMM, masked softmax, P.V GEMM
        ple = 0
        if self.dm.ple is not None:  # input: cast, GEMM, combine; per layer 3 launches (GEMVs) or 5 (GEMMs)
            gemv = 2 if S <= kern.PLE_FUSED_TAIL_ROWS else 3
            ple = 3 + len(self.dm.layers) * (gemv if S <= kern.PLE_GEMV_ROWS else 5)
        return 2 + total + 2 + ple

    def prefill_timed_gemms(self, tokens, seq: int = 0):
        """Run one prefill eagerly with CUDA events around every fused projection
        GEMM; returns [(name, M, N, K, ms)]."""
        S = len(tokens)
        pf = self._prefill_buffers(S)
        rec = []
        with torch.cuda.stream(self.stream):
            pf["tok"][:S].copy_(torch.as_tensor(list(tokens), dtype=torch.int32))
            self._prefill_step(pf, S, seq, rec)
        torch.cuda.synchronize(self.dm.device)
        return [(name, m, n, k, e0.elapsed_time(e1)) for name, m, n, k, e0, e1 in rec]

    def _prefill_ops(self, pf, S, seq, s, rec=None):
        dm, Ls = self.dm, self.dm.layers
        H, nh = self.H, self.nh
        ws = pf["ws"]

        def proj(name, A, L, key, C, K, geglu=False):
            W = L[key]
            if rec is not None:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(self.stream)
            kern.gemm_q4(A, W[0], W[1], C=C, workspace=ws, geglu=geglu, bits=L["bits"][key])
            if rec is not None:
                e1.record(self.stream)
                rec.append((name, S, W[0].shape[0], K, e0, e1))

        dm.embed(pf["tok"].data_ptr(), S, pf["hid"].data_ptr(), None, s)
        P = dm.ple
        if P is not None:
            # per-layer inputs of the whole prompt: the model projection as an f16 GEMM (f32 out), then the
            # per-slice norm + table gather (gemma4/reference.py:92-101)
            nL, pd = len(Ls), P["d"]
            _lib.call("sb_cast_f16", pf["hid"].data_ptr(), pf["ple_x16"].data_ptr(), S * H, s)
            _lib.call("sb_gemm_f16_f32out", pf["ple_x16"].data_ptr(), P["proj16"].data_ptr(),
                      pf["ple_ctx"].data_ptr(), S, nL * pd, H, float(H ** -0.5), 1, H, H, nL * pd, s)
            _lib.call("sb_ple_combine", pf["ple_ctx"].data_ptr(), pf["tok"].data_ptr(), P["table"].data_ptr(),
                      P["table_scale"].data_ptr(), P["table"].shape[0], P["norm"].data_ptr(), nL, pd,
                      kern.group_of(P["table_scale"], nL * pd), P["scale"], self.eps, pf["ple_in"].data_ptr(), S, s)
        _lib.call("sb_add_rmsnorm", pf["hid"].data_ptr(), None, _F32, None, Ls[0]["in_norm"].data_ptr(),
                  pf["hid"].data_ptr(), None, pf["h16"].data_ptr(), S, H, self.eps, s)
        for li, L in enumerate(Ls):
            sp = L["spec"]
            lhd, qd, Fl, nqkv = sp["hd"], sp["qd"], sp["F"], sp["nqkv"]
            qkv16, q16, attn16 = _rows(pf["qkv16"], S, nqkv), _rows(pf["q16"], S, qd), _rows(pf["attn16"], S, qd)
            k16, v16 = pf["kv16"].get(sp["src"], pf["kv16"].get(("hd", lhd)))
            proj("qkv", pf["h16"][:S], L, "qkv", qkv16, H)
            kc_off = seq * self.max_seq * lhd * 4
            if sp["own"]:
                _lib.call("sb_qkv_prep", qkv16.data_ptr(), _F16, nqkv, L["q_norm"].data_ptr(), L["k_norm"].data_ptr(),
                          L["cos"].data_ptr(), L["sin"].data_ptr(), None, 0, S, nh, lhd, self.eps, q16.data_ptr(), None,
                          self.kc[li].data_ptr() + kc_off, self.vc[li].data_ptr() + kc_off, k16.data_ptr(),
                          v16.data_ptr(), self.max_seq * lhd, s)
            else:  # KV sharing: q only; K/V are the source layer's (its f16 copies kept for this)
                _lib.call("sb_qkv_prep", qkv16.data_ptr(), _F16, nqkv, L["q_norm"].data_ptr(), None,
                          L["cos"].data_ptr(), L["sin"].data_ptr(), None, 0, S, nh, lhd, self.eps, q16.data_ptr(), None,
                          None, None, None, None, self.max_seq * lhd, s)
            if self._attn_route(sp, S) == "fused":  # causal attention over the prompt: one fused kernel
                _lib.call("sb_attn_prefill_ws", q16.data_ptr(), k16.data_ptr(), v16.data_ptr(), attn16.data_ptr(), S,
                          nh, lhd, pf["attn_ws"].data_ptr(), pf["attn_ws"].numel() * 4, s)
            else:
                ld = (S + 7) // 8 * 8
                kern.attn_prefill_gemm(q16.view(S, nh, lhd), k16, v16, attn16, S, window=sp["window"],
                                       scores=_rows(pf["scores"], S * nh, ld), p16=_rows(pf["p16"], S * nh, ld))
            proj("o", attn16, L, "o", pf["o16"][:S], qd)
            _lib.call("sb_add_rmsnorm", pf["hid"].data_ptr(), pf["o16"].data_ptr(), _F16,
                      L["post_attn_norm"].data_ptr(), L["pre_ffn_norm"].data_ptr(), pf["hid"].data_ptr(), None,
                      pf["h16"].data_ptr(), S, H, self.eps, s)
            # gate|up GEMM with GEGLU in its epilogue: writes a = gelu(gate) * up
            a16 = _rows(pf["a16"], S, Fl)
            proj("gate|up", pf["h16"][:S], L, "gu", a16, H, geglu=True)
            proj("down", a16, L, "down", pf["d16"][:S], Fl)
            last = li + 1 == len(Ls)
            nxt = Ls[li + 1]["in_norm"] if not last else dm.final_norm
            _lib.call("sb_add_rmsnorm", pf["hid"].data_ptr(), pf["d16"].data_ptr(), _F16,
                      L["post_ffn_norm"].data_ptr(), nxt.data_ptr(), pf["hid"].data_ptr(),
                      pf["hlast"].data_ptr() if last else None, None if last else pf["h16"].data_ptr(), S, H,
                      self.eps, s)
            if P is not None:  # PLE block on the prompt rows, then the next norm from its output
                kern.ple_block(pf["hid"][:S], pf["ple_in"][:S, li], L["ple"], self.eps, w_next=nxt,
                               h_out=pf["hlast"][:S] if last else None, h16_out=None if last else pf["h16"][:S])


def greedy_generate(model: dict, prompt, steps: int, device="cuda:0", batched_prefill: bool = True,
                    max_seq: int | None = None, fused: bool = False) -> list[int]:
    """Prefill `prompt`, then greedy-decode until `steps` tokens exist (the first
    comes from the prefill's last position), as the reference's generate loop does."""
    S = len(prompt)
    dm = DeviceModel(model, device, max_seq or (S + steps + 1))
    r = Runner(dm, 1, fused=fused)
    first = r.prefill(prompt) if batched_prefill else r.prefill_tokenwise(prompt)
    if not batched_prefill:
        r.set_state([first], [S])
    if steps <= 1:
        return [first][:steps]
    rest = r.decode(steps - 1)[0].cpu().tolist()
    return [first] + rest
