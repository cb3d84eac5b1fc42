"""numpy restatement of the reference's quantized-matmul arithmetic (oracle).

Test infrastructure only: see ``oracle/__init__.py``.  Every function cites the
reference code it restates (paths relative to the wakoan/slang tree).

Packing convention (shared by every function here):
  * a packed row is a little-endian stream of bytes; value ``i`` of a row sits
    at bit ``bits * i`` of that stream, i.e. low bits first inside each byte
    (gemma4/qat_loader.py:24-38, gemma4_150/loader.py:75-86,
    gemma4_150/kernels_dsl.py:2115-2117);
  * a code ``q`` in ``[0, 2**bits)`` means the integer ``q - 2**(bits-1)``
    (zero point 8 for int4, 2 for int2, 128 for the biased int8 codes that
    gemma4_150/export.py:155-157 writes);
  * a scale tensor is ``[n_out, n_in // group]``: ``group == n_in`` is the
    reference checkpoint's per-row scale (gemma4/qat_loader.py:95-102), ``group
    == 32`` the per-group-32 scales of the benchmark configuration, applied with
    the reference's ``np.repeat(scale, block)`` pattern
    (gemma4/qat_loader.py:106-121).
"""
from __future__ import annotations

import numpy as np

ZERO_POINT = {2: 2, 4: 8, 8: 128}


def unpack_codes(packed: np.ndarray, bits: int) -> np.ndarray:
    """Unsigned codes ``[..., n]`` from packed bytes ``[..., n*bits/8]``.

    Restates gemma4_150/loader.py:75-86 (``Ckpt.codes``): value ``j`` of each
    byte is ``(byte >> bits*j) & mask``, low bits first.
    """
    if bits not in ZERO_POINT:
        raise ValueError(f"unsupported bit width {bits}")
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    per = 8 // bits
    mask = (1 << bits) - 1
    out = np.empty(p.shape[:-1] + (p.shape[-1] * per,), dtype=np.uint8)
    for j in range(per):
        out[..., j::per] = (p >> (bits * j)) & mask
    return out


def unpack_signed(packed: np.ndarray, bits: int) -> np.ndarray:
    """Signed integers (code minus zero point) as int8.

    For 4 bits this is gemma4/qat_loader.py:24-30 (``unpack_int4``: low nibble
    first, minus 8); for 2 bits gemma4/qat_loader.py:33-38 (minus 2).
    """
    return (unpack_codes(packed, bits).astype(np.int16) - ZERO_POINT[bits]).astype(np.int8)


def expand_scales(scales: np.ndarray, n_in: int) -> np.ndarray:
    """Per-element f32 scales ``[n_out, n_in]`` (gemma4/qat_loader.py:115-121)."""
    s = np.asarray(scales).astype(np.float32)
    if s.ndim == 1:
        s = s[:, None]
    block = n_in // s.shape[-1]
    if block * s.shape[-1] != n_in:
        raise ValueError("scale groups must tile n_in")
    return np.repeat(s, block, axis=-1)


def dequant_f32(packed: np.ndarray, scales: np.ndarray, bits: int) -> np.ndarray:
    """Weight-only f32 dequant ``ints * repeat(scale)``.

    Restates gemma4/qat_loader.py:98-102 (per-row) and :115-121 (per-block).
    """
    ints = unpack_signed(packed, bits).astype(np.float32)
    return ints * expand_scales(scales, ints.shape[-1])


def dequant_f16(packed: np.ndarray, scales: np.ndarray, bits: int) -> np.ndarray:
    """GEMM-operand dequant ``f16(scale * (q - ZP))`` computed in f32.

    Restates ``dq_f16`` (gemma4_150/kernels_dsl.py:2101-2138): the product is
    formed in f32 and rounded once to f16 (round to nearest even).
    """
    ints = unpack_signed(packed, bits).astype(np.float32)
    prod = ints * expand_scales(scales, ints.shape[-1])
    return prod.astype(np.float16)


def gemv(packed: np.ndarray, scales: np.ndarray, x: np.ndarray, bits: int = 4) -> np.ndarray:
    """Decode GEMV ``y[m, n] = sum_k W[n, k] * x[m, k]`` with fp32 accumulate.

    Restates ``matvec_dq4`` (gemma4/qat_kernels.py:33-77) and the oracle's
    weight-only linear ``w(name) @ h`` (gemma4/reference.py:114, with
    ``QATReference._w`` dequant, gemma4/qat_reference.py:24-33).
    """
    w = dequant_f32(packed, scales, bits)
    xf = np.atleast_2d(np.asarray(x).astype(np.float32))
    return xf @ w.T


def gemm_f16(a: np.ndarray, b: np.ndarray, alpha: float = 1.0, tr: bool = True) -> np.ndarray:
    """``C = f16(alpha * A @ (B^T if tr else B))`` with f32 accumulation.

    Restates ``gemm_tiled`` (gemma4_150/kernels_dsl.py:34-141).
    """
    af = np.asarray(a, dtype=np.float16).astype(np.float32)
    bf = np.asarray(b, dtype=np.float16).astype(np.float32)
    c = af @ (bf.T if tr else bf)
    return (np.float32(alpha) * c).astype(np.float16)


def gemm_f64(a: np.ndarray, b: np.ndarray, alpha: float = 1.0, tr: bool = True) -> np.ndarray:
    """float64 product from the f16 inputs (tests/test_gemm_dsl.py:21-23)."""
    af = np.asarray(a, dtype=np.float16).astype(np.float64)
    bf = np.asarray(b, dtype=np.float16).astype(np.float64)
    return alpha * (af @ (bf.T if tr else bf))


def gemm_q4(a: np.ndarray, packed: np.ndarray, scales: np.ndarray, alpha: float = 1.0,
            bits: int = 4) -> np.ndarray:
    """Prefill projection ``f16(alpha * A @ dq_f16(W)^T)``.

    Restates the reference's prefill pair ``_dq`` then ``_gemm``
    (gemma4_150/prefill_gpu.py:186-200, 151-170): the weight is first rounded
    to f16 by ``dq_f16`` and the GEMM accumulates in f32.
    """
    return gemm_f16(a, dequant_f16(packed, scales, bits), alpha, tr=True)


def argmax_first(values: np.ndarray) -> np.ndarray:
    """Greedy argmax, ties to the LOWEST index.

    Restates ``argmax1_34``/``argmax2_35`` (gemma4_150/kernels_dsl.py:481-570),
    whose tie rule is the same as ``numpy.argmax``.
    """
    v = np.atleast_2d(np.asarray(values, dtype=np.float32))
    return np.argmax(v, axis=-1).astype(np.int64)


def lmhead_argmax(packed: np.ndarray, scales: np.ndarray, h: np.ndarray, bits: int = 4,
                  chunk: int = 16384) -> tuple[np.ndarray, np.ndarray]:
    """Tied lm_head GEMV then greedy argmax; returns (token ids, max logits).

    Restates gemma4/reference.py:178-179 (``embed @ x`` then the monotonic
    softcap, which cannot change the argmax) with the per-block embedding
    dequant of gemma4/qat_loader.py:115-121.  Rows are processed in chunks so a
    262144-row table never has to be dequantised whole.
    """
    hf = np.atleast_2d(np.asarray(h).astype(np.float32))
    best_v = np.full(hf.shape[0], -np.inf, dtype=np.float32)
    best_i = np.zeros(hf.shape[0], dtype=np.int64)
    for r0 in range(0, packed.shape[0], chunk):
        logits = gemv(packed[r0:r0 + chunk], scales[r0:r0 + chunk], hf, bits)
        i = np.argmax(logits, axis=-1)
        v = logits[np.arange(hf.shape[0]), i]
        better = v > best_v  # strict: an equal later chunk keeps the lower index
        best_v = np.where(better, v, best_v)
        best_i = np.where(better, i + r0, best_i)
    return best_i, best_v


def orderable_u32(v: np.ndarray) -> np.ndarray:
    """Map f32 to u32 so unsigned order equals float order (NaN treated as -inf)."""
    f = np.asarray(v, dtype=np.float32).copy()
    f[np.isnan(f)] = -np.inf
    b = f.view(np.uint32)
    return np.where(b & 0x80000000, ~b, b | 0x80000000).astype(np.uint32)


def pack_key(value: np.ndarray, index: np.ndarray) -> np.ndarray:
    """(max, lowest index) as one u64 so an integer MAX combines shards."""
    hi = orderable_u32(value).astype(np.uint64) << np.uint64(32)
    lo = (np.uint64(0xFFFFFFFF) - np.asarray(index, dtype=np.uint64)) & np.uint64(0xFFFFFFFF)
    return hi | lo


def unpack_key_index(key: np.ndarray) -> np.ndarray:
    return (np.uint64(0xFFFFFFFF) - (np.asarray(key, dtype=np.uint64) & np.uint64(0xFFFFFFFF))).astype(np.int64)


def pack_int4(ints: np.ndarray) -> np.ndarray:
    """Signed int4 ``[n_out, n_in]`` -> packed bytes ``[n_out, n_in/2]``, low nibble first.

    The inverse of ``unpack_signed(., 4)``; the same packing as the reference
    test helper ``_pack4`` (tests/test_gemma4_qat_kernels_gpu.py:24-29) before its
    u32 reinterpretation.
    """
    u = (np.asarray(ints).astype(np.int16) + 8).astype(np.uint8)
    return (u[..., 0::2] | (u[..., 1::2] << 4)).astype(np.uint8)
