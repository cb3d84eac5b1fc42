"""manifest.json + weights.bin: the reference's on-disk model format.

The layout follows gemma4_150/export.py:35-56, 163-182: tensors are appended to
weights.bin with 4-byte padding and described by
``{"off", "len", "dtype", "shape"}`` in manifest["tensors"]; per-layer
structure lives in manifest["layers"].  ``read`` loads two dialects of it:

* the reference's own export (gemma4_150/export.py:64-187, the checkpoint's
  real format): quantized weights ``L{i}.{q,k,v,o,gate,up,down}_bits`` as flat
  u32 words of the packed rows, one f32 scale per row (``L{i}.qkv_scales``
  holds q, k and v rows back to back; ``L{i}.{o,gate,up,down}_scale``), the bit
  width of each weight read off its size as the reference's ``_dq`` does
  (gemma4_150/prefill_gpu.py:186-196), the 2-bit embedding ``embed_q`` with its
  flat per-block ``embed_scale``, the separate 2-bit lm_head stored block-major
  ``lmhead_blk`` [24, rows, 4] (export.py:90-93) and ``lmhead_scale``, norms
  packed as ``o_w12`` = post-attention | pre-FFN and ``pleproj_w12s`` =
  post-PLE | next layer's input norm | layer scalar, the per-layer-embedding
  tensors (``ple_q``/``ple_scale``, ``pl_model_proj`` in f16, ``pl_proj_norm``,
  ``L{i}.{plegate,pleproj}_codes``/``_rowscale`` as +128-biased int8), and per
  layer ``head_dim``, ``q_dim``, ``intermediate``, ``sliding``, ``kv_source``,
  ``rope_theta``, ``rope_cutoff``.  The SRQ activation scales
  (``layers[i].scales``) are returned per layer as ``srq`` for the SRQ
  linears (``sb_gemv_srq``); the model runs weight-only, the reference's
  ``s == 0`` branch (gemma4_150/reference.py:30-31), and the GELU tables of
  the SRQ kernels are not read;
* this build's group-scale extension, written by ``write``: the same names for
  the packed weights and norms, plus per-group f16 scale tensors
  ``L{i}.{name}_gscale`` of shape ``[n_out, n_in/group]`` (``config.group``)
  for the benchmark format's per-group-32 scales, and a tied lm_head.
"""
from __future__ import annotations

import json
import math
import os

import numpy as np

PROJ = ("q", "k", "v", "o", "gate", "up", "down")
_DT = {"u8": np.uint8, "u32": np.uint32, "f16": np.float16, "f32": np.float32}


class _Writer:
    """Appends tensors to weights.bin, 4-byte aligned (gemma4_150/export.py:35-56)."""

    def __init__(self, path: str):
        self.f = open(path, "wb")
        self.pos = 0
        self.tensors: dict = {}

    def put(self, name: str, arr: np.ndarray, dtype: str) -> None:
        if name in self.tensors:
            raise KeyError(f"duplicate tensor {name}")
        b = np.ascontiguousarray(arr).tobytes()
        self.f.write(b)
        self.tensors[name] = {"off": self.pos, "len": len(b), "dtype": dtype, "shape": list(arr.shape)}
        self.pos += len(b)
        pad = (-len(b)) % 4
        if pad:
            self.f.write(b"\x00" * pad)
            self.pos += pad

    def close(self):
        self.f.close()


def write(model: dict, out_dir: str) -> str:
    """Write a ``synth.random_model``-style dict as manifest.json + weights.bin."""
    os.makedirs(out_dir, exist_ok=True)
    cfg = model["config"]
    w = _Writer(os.path.join(out_dir, "weights.bin"))
    w.put("embed_q", model["embed_q"], "u8")
    w.put("embed_gscale", model["embed_scale"], "f16")
    w.put("final_norm", model["final_norm"], "f32")
    layers = []
    for i, L in enumerate(model["layers"]):
        w.put(f"L{i}.in_norm", L["in_norm"], "f32")
        w.put(f"L{i}.q_norm", L["q_norm"], "f32")
        w.put(f"L{i}.k_norm", L["k_norm"], "f32")
        w.put(f"L{i}.o_w12", np.concatenate([L["post_attn_norm"], L["pre_ffn_norm"]]), "f32")
        w.put(f"L{i}.down_nw", L["post_ffn_norm"], "f32")
        for name in PROJ:
            packed, scales = L[name]
            w.put(f"L{i}.{name}_bits", packed, "u8")
            w.put(f"L{i}.{name}_gscale", scales, "f16")
        layers.append({"index": i, "sliding": bool(cfg["sliding_window"]), "head_dim": cfg["head_dim"],
                       "q_dim": cfg["q_dim"], "intermediate": cfg["inter"], "shared": False, "kv_source": i,
                       "rope_theta": cfg["rope_theta"], "rope_cutoff": cfg["rope_cutoff"], "scales": {}})
    w.close()
    manifest = {
        "config": {"H": cfg["hidden"], "nL": cfg["n_layers"], "nH": cfg["n_heads"], "vocab": cfg["vocab"],
                   "window": cfg["sliding_window"], "softcap": cfg["softcap"], "embed_scale": cfg["embed_scale"],
                   "eps": cfg["eps"], "group": cfg["group"], "bits": 4},
        "layers": layers, "tensors": w.tensors, "bytes": w.pos,
    }
    with open(os.path.join(out_dir, "manifest.json"), "w") as f:
        json.dump(manifest, f)
    return out_dir


def read(model_dir: str) -> dict:
    """Load manifest.json + weights.bin (memory-mapped) into the model dict the
    runner and the oracle take; either dialect (see the module docstring)."""
    with open(os.path.join(model_dir, "manifest.json")) as f:
        man = json.load(f)
    blob = np.memmap(os.path.join(model_dir, "weights.bin"), np.uint8, "r")

    def get(name):
        t = man["tensors"][name]
        a = blob[t["off"]:t["off"] + t["len"]].view(_DT[t["dtype"]])
        return a.reshape(t["shape"])

    if "embed_gscale" in man["tensors"]:
        return _read_group(man, get)
    return _read_export(man, get)


def _read_group(man: dict, get) -> dict:
    c = man["config"]
    L0 = man["layers"][0]
    cfg = {"hidden": c["H"], "n_layers": c["nL"], "n_heads": c["nH"], "head_dim": L0["head_dim"],
           "q_dim": L0["q_dim"], "inter": L0["intermediate"], "vocab": c["vocab"], "eps": c.get("eps", 1e-6),
           "rope_theta": L0["rope_theta"], "rope_cutoff": L0["rope_cutoff"], "softcap": c["softcap"],
           "sliding_window": c["window"], "group": c["group"], "embed_scale": c.get("embed_scale", math.sqrt(c["H"]))}
    layers = []
    for i in range(c["nL"]):
        o_w12 = get(f"L{i}.o_w12")
        L = {name: (get(f"L{i}.{name}_bits"), get(f"L{i}.{name}_gscale")) for name in PROJ}
        L.update(in_norm=get(f"L{i}.in_norm"), q_norm=get(f"L{i}.q_norm"), k_norm=get(f"L{i}.k_norm"),
                 post_attn_norm=o_w12[:c["H"]], pre_ffn_norm=o_w12[c["H"]:], post_ffn_norm=get(f"L{i}.down_nw"))
        layers.append(L)
    return {"config": cfg, "embed_q": get("embed_q"), "embed_scale": get("embed_gscale"),
            "final_norm": get("final_norm"), "layers": layers}


def _rows(words: np.ndarray, n_out: int) -> np.ndarray:
    """Flat packed words of ``n_out`` rows -> u8 ``[n_out, bytes per row]``
    (export.py's u32 view of the packed rows, gemma4_150/export.py:59-61)."""
    b = np.ascontiguousarray(words).view(np.uint8).reshape(-1)
    if b.size % n_out:
        raise ValueError(f"{b.size} packed bytes do not split into {n_out} rows")
    return b.reshape(n_out, -1)


def _row_scale(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, np.float32).reshape(-1, 1)


def _read_export(man: dict, get) -> dict:
    c = man["config"]
    H, nL, V = c["H"], c["nL"], c["vocab"]
    specs = [{"head_dim": L["head_dim"], "q_dim": L["q_dim"], "inter": L["intermediate"],
              "kv_source": L["kv_source"], "sliding": bool(L["sliding"]), "rope_theta": float(L["rope_theta"]),
              "rope_cutoff": int(L["rope_cutoff"])} for L in man["layers"]]
    L0 = specs[0]
    cfg = {"hidden": H, "n_layers": nL, "n_heads": c["nH"], "head_dim": L0["head_dim"], "q_dim": L0["q_dim"],
           "inter": L0["inter"], "vocab": V, "eps": c.get("eps", 1e-6), "rope_theta": L0["rope_theta"],
           "rope_cutoff": L0["rope_cutoff"], "softcap": c["softcap"],
           "sliding_window": c["window"] if any(sp["sliding"] for sp in specs) else 0,
           "group": None, "embed_scale": float(c["embed_scale"]), "layer_specs": specs, "format": "export"}
    embed_q = get("embed_q")
    embed_scale = np.ascontiguousarray(get("embed_scale"), np.float32).reshape(V, -1)
    # lmhead_blk [24, rows, 4] u32 is the row-major table's words regrouped 96 at a time
    # (export.py:90-93: reshape(-1, 24, 4).transpose(1, 0, 2)); undo the transpose
    blk = get("lmhead_blk")
    lm_q = _rows(np.ascontiguousarray(blk.transpose(1, 0, 2)), V)
    model = {"config": cfg, "embed_q": np.ascontiguousarray(embed_q), "embed_scale": embed_scale,
             "lm_q": lm_q, "lm_scale": _row_scale(get("lmhead_scale")), "final_norm": get("final_norm"),
             "layers": []}
    for i, sp in enumerate(specs):
        qd, hd, F = sp["q_dim"], sp["head_dim"], sp["inter"]
        L = {}
        if sp["kv_source"] == i:
            qkv_s = get(f"L{i}.qkv_scales")
            L["q"] = (_rows(get(f"L{i}.q_bits"), qd), _row_scale(qkv_s[:qd]))
            L["k"] = (_rows(get(f"L{i}.k_bits"), hd), _row_scale(qkv_s[qd:qd + hd]))
            L["v"] = (_rows(get(f"L{i}.v_bits"), hd), _row_scale(qkv_s[qd + hd:qd + 2 * hd]))
            L["k_norm"] = get(f"L{i}.k_norm")
        else:
            L["q"] = (_rows(get(f"L{i}.q_bits"), qd), _row_scale(get(f"L{i}.q_scale")))
        L["o"] = (_rows(get(f"L{i}.o_bits"), H), _row_scale(get(f"L{i}.o_scale")))
        for name, n_out in (("gate", F), ("up", F), ("down", H)):
            L[name] = (_rows(get(f"L{i}.{name}_bits"), n_out), _row_scale(get(f"L{i}.{name}_scale")))
        o_w12 = get(f"L{i}.o_w12")
        L.update(in_norm=get(f"L{i}.in_norm"), q_norm=get(f"L{i}.q_norm"), post_attn_norm=o_w12[:H],
                 pre_ffn_norm=o_w12[H:], post_ffn_norm=get(f"L{i}.down_nw"))
        # the SRQ activation scales of each linear (qkv_in, q_out, k_out, v_out, o_in, o_out, gate_in, ...),
        # for the SRQ arithmetic (gemma4_150/reference.py:96-101); the weight-only path ignores them
        L["srq"] = {k: float(v) for k, v in man["layers"][i].get("scales", {}).items()}
        model["layers"].append(L)
    if "ple_q" in man["tensors"]:
        d = int(c["ple_d"])
        ple = {"hidden": H, "n_layers": nL, "d": d, "vocab": V, "ple_scale": float(c["ple_scale"]),
               "table": get("ple_q"),
               "table_scale": np.ascontiguousarray(get("ple_scale"), np.float32).reshape(V, -1),
               "proj": get("pl_model_proj"), "norm": get("pl_proj_norm"), "layers": []}
        for i in range(nL):
            w12s = get(f"L{i}.pleproj_w12s")
            ple["layers"].append({
                "gate": (_rows(get(f"L{i}.plegate_codes"), d), np.ascontiguousarray(get(f"L{i}.plegate_rowscale"))),
                "proj": (_rows(get(f"L{i}.pleproj_codes"), H), np.ascontiguousarray(get(f"L{i}.pleproj_rowscale"))),
                "post_norm": w12s[:H], "scalar": float(w12s[2 * H])})
        model["ple"] = ple
    return model
