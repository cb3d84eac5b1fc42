"""numpy restatement of the reference's static range quantisation (SRQ) (oracle).

Test infrastructure only: see ``oracle/__init__.py``.

The reference's production decode arithmetic quantises the activations at
every quantised linear (gemma4_150/reference.py:7-9):

    y = srq(dequant_weight @ srq(x, in_scale), out_scale)
    srq(x, s) = clip(round(x / s), -128, 127) * s        (s == 0: x unchanged)

``round`` is numpy's round-half-to-even, every operation in f32.
"""
from __future__ import annotations

import numpy as np

from . import q4


def srq(x: np.ndarray, s: float) -> np.ndarray:
    """gemma4_150/reference.py:30-31."""
    x = np.asarray(x, np.float32)
    if s == 0.0:
        return x
    s32 = np.float32(s)
    return (np.clip(np.round(x / s32), -128.0, 127.0) * s32).astype(np.float32)


def qlin(packed: np.ndarray, scales: np.ndarray, bits: int, x: np.ndarray, in_scale: float,
         out_scale) -> np.ndarray:
    """``ReferenceSRQ._qlin`` (gemma4_150/reference.py:96-101) for one row vector
    ``x``: the dequantised weight ((code - zp) * scale) times srq(x, in_scale),
    then srq with ``out_scale`` -- a float, or one scale per output row when the
    rows of several linears are concatenated."""
    w = q4.dequant_f32(packed, scales, bits)
    y = w @ srq(x, in_scale)
    if np.ndim(out_scale) == 0:
        return srq(y, float(out_scale))
    out = np.asarray(out_scale, np.float32)
    return np.array([srq(y[i:i + 1], float(out[i]))[0] for i in range(len(y))], np.float32)
