"""manifest.json + weights.bin: the reference's on-disk model format.

The layout follows gemma4_150/export.py:35-56, 163-182: tensors are appended to
weights.bin with 4-byte padding and described by
``{"off", "len", "dtype", "shape"}`` in manifest["tensors"]; per-layer
structure lives in manifest["layers"].  Quantized weights keep export.py's
names (``L{i}.{q,k,v,o,gate,up,down}_bits``, the packed bytes of each row);
this build adds per-group f16 scale tensors ``L{i}.{name}_gscale`` of shape
``[n_out, n_in/group]`` (``config.group``) next to them, since the benchmark
format has per-group-32 scales where the reference checkpoint has one f32
scale per row.  Norm vectors use export.py's names too
(``L{i}.in_norm``, ``L{i}.q_norm``, ``L{i}.k_norm``, ``L{i}.o_w12`` =
post-attention | pre-FFN, ``L{i}.down_nw`` = post-FFN, ``final_norm``).
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
    """Load manifest.json + weights.bin (memory-mapped) back into the model dict."""
    with open(os.path.join(model_dir, "manifest.json")) as f:
        man = json.load(f)
    blob = np.memmap(os.path.join(model_dir, "weights.bin"), np.uint8, "r")

    def get(name):
        t = man["tensors"][name]
        a = blob[t["off"]:t["off"] + t["len"]].view(_DT[t["dtype"]])
        return a.reshape(t["shape"])

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
