"""numpy restatement of the reference's per-layer-embedding (PLE) arithmetic (oracle).

Test infrastructure only: see ``oracle/__init__.py``.

Gemma-4-E2B adds, after each layer's MLP, a per-layer-embedding block fed by
one 256-value slice per layer of a per-token input.  The reference computes
(weight-only, f32, gemma4/reference.py:92-101 and :154-163, with the QAT
dequant of gemma4/qat_reference.py:24-45):

* the PLE table row of the token: the 4-bit ``embed_tokens_per_layer`` row
  with one f32 scale per 256 values (gemma4/qat_loader.py:106-113), times
  ``ple_scale = sqrt(256)`` (gemma4/loader.py:125);
* the per-layer input: the bf16 ``per_layer_model_projection`` applied to the
  scaled embedding, times ``hidden**-0.5``, RMS-normed per 256-value slice with
  ``per_layer_projection_norm``, plus the table row, times ``2**-0.5``;
* per layer: ``g = gelu_tanh(W_gate @ x) * ple_in[layer]`` and
  ``x = (x + rms_norm(W_proj @ g, w_post)) * layer_scalar`` with the two 8-bit
  linears ``per_layer_input_gate`` [256, hidden] and ``per_layer_projection``
  [hidden, 256]: signed int8 times a per-row f32 scale
  (gemma4/qat_loader.py:41-48, :58-59, :98-102), stored +128-biased as in
  gemma4_150/export.py:150-157 (``q4.ZERO_POINT[8]``).
"""
from __future__ import annotations

import numpy as np

from . import q4
from .decoder import gelu_tanh, rms_norm


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) to f32: the high half of the f32 word."""
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def ple_gather(ids: np.ndarray, packed: np.ndarray, scales: np.ndarray, ple_scale: float) -> np.ndarray:
    """Scaled PLE table rows ``[m, cols]`` for token ``ids``.

    ``QATIndex.dequant_embedding_row`` (gemma4/qat_loader.py:106-113: signed
    4-bit values times ``np.repeat(scale, block)``) times ``ple_scale``
    (gemma4/reference.py:96); ``plegather_01`` (gemma4_150/kernels_dsl.py:457-478)
    computes the same product per value.
    """
    ids = np.asarray(ids, np.int64)
    rows = q4.dequant_f32(packed[ids], scales[ids], 4)
    return rows * np.float32(ple_scale)


def ple_input(x: np.ndarray, ple_rows: np.ndarray, w_proj_bf16: np.ndarray, w_norm: np.ndarray,
              n_layers: int, d: int, eps: float) -> np.ndarray:
    """Per-layer inputs ``[m, n_layers, d]`` (gemma4/reference.py:92-101).

    ``x`` [m, hidden] is the scaled embedding, ``ple_rows`` [m, n_layers * d]
    the output of :func:`ple_gather`, ``w_proj_bf16`` [n_layers * d, hidden]
    the bf16 bit patterns of ``per_layer_model_projection`` (or its f16 values).
    """
    x = np.atleast_2d(np.asarray(x, np.float32))
    m, hidden = x.shape
    # export.py stores the projection cast to f16 (gemma4_150/export.py:95); the checkpoint holds bf16 bits
    w = (np.asarray(w_proj_bf16, np.float32) if np.asarray(w_proj_bf16).dtype == np.float16
         else bf16_to_f32(w_proj_bf16))
    ctx = (x @ w.T).reshape(m, n_layers, d) * np.float32(hidden ** -0.5)
    ctx = rms_norm(ctx, np.asarray(w_norm, np.float32), eps)
    return (ctx + ple_rows.reshape(m, n_layers, d)) * np.float32(2.0 ** -0.5)


def q8_gemv(codes: np.ndarray, row_scale: np.ndarray, x: np.ndarray) -> np.ndarray:
    """``y[m, n] = sum_k (code[n, k] - 128) * scale[n] * x[m, k]`` in f32.

    The weight-only linear of an 8-bit module (gemma4/qat_loader.py:98-102,
    applied as ``w(name) @ x`` at gemma4/reference.py:159-160).
    """
    w = q4.dequant_f32(codes, row_scale, 8)
    return np.atleast_2d(np.asarray(x, np.float32)) @ w.T


def ple_gate(codes: np.ndarray, row_scale: np.ndarray, x: np.ndarray, ple_in: np.ndarray) -> np.ndarray:
    """``gelu_tanh(W_gate @ x) * ple_in`` (gemma4/reference.py:159)."""
    return gelu_tanh(q8_gemv(codes, row_scale, x)) * np.asarray(ple_in, np.float32)


def ple_norm_add(proj: np.ndarray, x: np.ndarray, w_post: np.ndarray, layer_scalar: float, eps: float) -> np.ndarray:
    """``(x + rms_norm(proj, w_post)) * layer_scalar`` (gemma4/reference.py:160-163)."""
    h = rms_norm(np.asarray(proj, np.float32), np.asarray(w_post, np.float32), eps)
    return (np.asarray(x, np.float32) + h) * np.float32(layer_scalar)


def ple_block(x: np.ndarray, ple_in: np.ndarray, layer: dict, eps: float) -> np.ndarray:
    """One layer's PLE block (gemma4/reference.py:154-163) on ``x`` [m, hidden].

    ``layer`` holds ``gate`` (codes, row scales), ``proj`` (codes, row scales),
    ``post_norm`` and ``scalar`` as built by ``slang_b200.synth.ple_weights``.
    """
    g = ple_gate(layer["gate"][0], layer["gate"][1], x, ple_in)
    proj = q8_gemv(layer["proj"][0], layer["proj"][1], g)
    return ple_norm_add(proj, x, layer["post_norm"], layer["scalar"], eps)
