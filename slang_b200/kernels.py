"""torch-facing wrappers of the C ABI, named after the reference's operator calls.

Each wrapper validates dtypes/devices, passes raw device pointers and the
current CUDA stream to ``libslang_b200.so`` and raises ``SlangError`` on a
non-zero status.  Buffers are owned by the caller (as the reference runners own
theirs); wrappers only allocate an output when none is given.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import SB_F16, SB_F32

_DT = {torch.float16: SB_F16, torch.float32: SB_F32}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, name: str, dtypes=None, cuda=True):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if cuda and not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if dtypes is not None and t.dtype not in dtypes:
        raise TypeError(f"{name} has dtype {t.dtype}, expected one of {dtypes}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def group_of(scales: torch.Tensor, n_in: int) -> int:
    """Values per scale along K, read off the scale tensor's shape."""
    groups = 1 if scales.dim() == 1 else scales.shape[-1]
    if n_in % groups:
        raise ValueError(f"{groups} scale groups do not tile n_in={n_in}")
    return n_in // groups


def dequant_f16(packed: torch.Tensor, scales: torch.Tensor, n_in: int, n_out: int,
                out: torch.Tensor | None = None, bits: int | None = None) -> torch.Tensor:
    """``PrefillGPU._dq`` (gemma4_150/prefill_gpu.py:186-200): packed -> f16 [n_out, n_in].

    As in the reference, the bit width is read off the packed buffer's size
    unless given.
    """
    _need(packed, "packed", (torch.uint8, torch.int32, torch.uint32))
    _need(scales, "scales", (torch.float16, torch.float32))
    nbytes = packed.numel() * packed.element_size()
    if bits is None:
        bits = nbytes * 8 // (n_in * n_out)
    if bits not in (2, 4, 8) or nbytes * 8 != bits * n_in * n_out:
        raise ValueError(f"odd width for [{n_out}x{n_in}] from {nbytes} packed bytes")
    if out is None:
        out = torch.empty((n_out, n_in), dtype=torch.float16, device=packed.device)
    _need(out, "out", (torch.float16,))
    _lib.call("sb_dequant_f16", _ptr(packed), bits, _ptr(scales), _DT[scales.dtype],
              group_of(scales, n_in), _ptr(out), n_out, n_in, _stream())
    return out


def gemv_q4(w: torch.Tensor, scales: torch.Tensor, x: torch.Tensor,
            y: torch.Tensor | None = None, bits: int = 4) -> torch.Tensor:
    """Decode GEMV ``y[m, n] = x[m] . W[n]`` (matvec_dq4, gemma4/qat_kernels.py:33-77);
    ``bits=2`` for the checkpoint's 2-bit weights (gateup_95 / down_96)."""
    _need(w, "w", (torch.uint8,))
    _need(scales, "scales", (torch.float16, torch.float32))
    _need(x, "x", (torch.float16, torch.float32))
    if bits not in (2, 4):
        raise ValueError(f"bits={bits}: the GEMV takes 2- or 4-bit codes")
    n, k = w.shape[0], w.shape[1] * 8 // bits
    x2 = x.reshape(-1, k)
    m = x2.shape[0]
    if y is None:
        y = torch.empty((m, n), dtype=torch.float32, device=w.device)
    _need(y, "y", (torch.float32,))
    _lib.call("sb_gemv_q4" if bits == 4 else "sb_gemv_q2", _ptr(w), _ptr(scales), _DT[scales.dtype],
              group_of(scales, k), _ptr(x2), _DT[x.dtype], _ptr(y), y.shape[-1], m, n, k, _stream())
    return y


def gemv_srq(w: torch.Tensor, scales: torch.Tensor, x: torch.Tensor, in_scale: float, out_scale=0.0,
             y: torch.Tensor | None = None, bits: int = 4) -> torch.Tensor:
    """SRQ linear ``y = srq(W @ srq(x, in_scale), out)`` (``ReferenceSRQ._qlin``,
    gemma4_150/reference.py:96-101); ``out_scale`` a float or a per-row f32
    tensor [n] (concatenated linears)."""
    _need(w, "w", (torch.uint8,))
    _need(scales, "scales", (torch.float16, torch.float32))
    _need(x, "x", (torch.float16, torch.float32))
    n, k = w.shape[0], w.shape[1] * 8 // bits
    x2 = x.reshape(-1, k)
    m = x2.shape[0]
    if y is None:
        y = torch.empty((m, n), dtype=torch.float32, device=w.device)
    _need(y, "y", (torch.float32,))
    rows = None
    if isinstance(out_scale, torch.Tensor):
        _need(out_scale, "out_scale", (torch.float32,))
        if out_scale.numel() != n:
            raise ValueError("per-row out_scale must hold one scale per output row")
        rows, out_scale = out_scale, 0.0
    _lib.call("sb_gemv_srq", _ptr(w), bits, _ptr(scales), _DT[scales.dtype], group_of(scales, k), _ptr(x2),
              _DT[x.dtype], float(in_scale), float(out_scale), _ptr(rows), _ptr(y), y.shape[-1], m, n, k, _stream())
    return y


def gemv_norm_add(w: torch.Tensor, scales: torch.Tensor, x: torch.Tensor, hidden: torch.Tensor, w_add: torch.Tensor,
                  eps: float, w_next: torch.Tensor | None = None, h_out: torch.Tensor | None = None,
                  h16_out: torch.Tensor | None = None, y: torch.Tensor | None = None,
                  counter: torch.Tensor | None = None, bits: int = 4) -> torch.Tensor:
    """Decode GEMV ``y = W @ x`` whose last-arriving CTA then runs
    ``hidden += rmsnorm(y) * w_add`` and ``h = rmsnorm(hidden) * w_next`` (the
    reference's oproj_73 / down_75 tails); returns y."""
    _need(w, "w", (torch.uint8,))
    _need(scales, "scales", (torch.float16, torch.float32))
    _need(x, "x", (torch.float16, torch.float32))
    for t, name in ((hidden, "hidden"), (w_add, "w_add")):
        _need(t, name, (torch.float32,))
    n, k = w.shape[0], w.shape[1] * 8 // bits
    x2 = x.reshape(-1, k)
    m = x2.shape[0]
    if hidden.numel() != m * n:
        raise ValueError("hidden must hold m x n values")
    if y is None:
        y = torch.empty((m, n), dtype=torch.float32, device=w.device)
    if counter is None:
        counter = _counter(w.device)
    _lib.call("sb_gemv_norm_add", _ptr(w), bits, _ptr(scales), _DT[scales.dtype], group_of(scales, k), _ptr(x2),
              _DT[x.dtype], _ptr(y), m, n, k, _ptr(hidden), _ptr(w_add), _ptr(w_next), _ptr(h_out), _ptr(h16_out),
              float(eps), _ptr(counter), _stream())
    return y


def srq(x: torch.Tensor, scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """Elementwise ``clip(round(x / scale), -128, 127) * scale`` (gemma4_150/reference.py:30-31)."""
    _need(x, "x", (torch.float16, torch.float32))
    if out is None:
        out = torch.empty_like(x)
    _need(out, "out", (torch.float16, torch.float32))
    _lib.call("sb_srq", _ptr(x), _DT[x.dtype], x.numel(), float(scale), _ptr(out), _DT[out.dtype], _stream())
    return out


def lmhead_argmax(emb: torch.Tensor, scales: torch.Tensor, h: torch.Tensor, row_offset: int = 0,
                  keys: torch.Tensor | None = None, tokens: torch.Tensor | None = None,
                  logits: torch.Tensor | None = None, want_tokens: bool = True, bits: int = 4):
    """Fused ``logits_33`` + ``argmax1_34``/``argmax2_35``; returns (keys, tokens).
    ``bits=2`` for the checkpoint's 2-bit lm_head."""
    _need(emb, "emb", (torch.uint8,))
    _need(scales, "scales", (torch.float16, torch.float32))
    _need(h, "h", (torch.float16, torch.float32))
    if bits not in (2, 4):
        raise ValueError(f"bits={bits}: the lm_head takes 2- or 4-bit codes")
    v, k = emb.shape[0], emb.shape[1] * 8 // bits
    h2 = h.reshape(-1, k)
    m = h2.shape[0]
    dev = emb.device
    if keys is None:
        keys = torch.empty(m, dtype=torch.int64, device=dev)
    if want_tokens and tokens is None:
        tokens = torch.empty(m, dtype=torch.int32, device=dev)
    _lib.call("sb_lmhead_argmax" if bits == 4 else "sb_lmhead_argmax_q2", _ptr(emb), _ptr(scales), _DT[scales.dtype],
              group_of(scales, k),
              _ptr(h2), _DT[h.dtype], m, v, k, int(row_offset), _ptr(keys),
              _ptr(tokens) if want_tokens else None, _ptr(logits), _stream())
    return keys, tokens


def keys_to_tokens(keys: torch.Tensor, tokens: torch.Tensor | None = None) -> torch.Tensor:
    if tokens is None:
        tokens = torch.empty(keys.numel(), dtype=torch.int32, device=keys.device)
    _lib.call("sb_keys_to_tokens", _ptr(keys), _ptr(tokens), keys.numel(), _stream())
    return tokens


def gemm(A: torch.Tensor, W: torch.Tensor, C: torch.Tensor, M: int, N: int, K: int, alpha: float = 1.0,
         tr: bool = True, acols: int | None = None, ccols: int | None = None, aoff: int = 0,
         boff: int = 0, coff: int = 0, bcols: int | None = None) -> torch.Tensor:
    """``PrefillGPU._gemm`` (gemma4_150/prefill_gpu.py:151-184) on tcgen05.

    ``C[M,N] = alpha * A[M,K] @ (W[N,K]^T if tr else W[K,N])``, all f16; acols,
    ccols are row strides wider than the operation and aoff/boff/coff are BYTE
    offsets into the buffers, exactly as in the reference.
    """
    for t, nm in ((A, "A"), (W, "W"), (C, "C")):
        _need(t, nm, (torch.float16,))
    lda = acols or K
    ldb = bcols or (K if tr else N)
    ldc = ccols or N
    _lib.call("sb_gemm_f16", A.data_ptr() + aoff, W.data_ptr() + boff, C.data_ptr() + coff, M, N, K,
              float(alpha), 1 if tr else 0, lda, ldb, ldc, _stream())
    return C


def attn_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor | None = None,
                 split: bool = True, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Causal prompt attention (the reference's attn_prefill / _attn_gemm,
    gemma4_150/prefill_gpu.py:259-314): q [S, nh, hd], k, v [S, hd] f16 ->
    out [S, nh, hd] f16 = softmax(q k^T, causal) v, one fused kernel
    (hd in {64, 128, 256})."""
    for t, nm in ((q, "q"), (k, "k"), (v, "v")):
        _need(t, nm, (torch.float16,))
        if not t.is_contiguous():
            raise ValueError(f"{nm} must be contiguous")
    S, nh, hd = q.shape
    if k.shape[0] < S or v.shape[0] < S or k.shape[1] != hd or v.shape[1] != hd:
        raise ValueError("k and v must be [>= S, head_dim]")
    if out is None:
        out = torch.empty_like(q)
    _need(out, "out", (torch.float16,))
    if not split:
        _lib.call("sb_attn_prefill", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), S, nh, hd, _stream())
        return out
    if workspace is None:
        workspace = _workspace(q.device, _lib.load().sb_attn_prefill_workspace_size(S, nh, hd))
    nbytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _lib.call("sb_attn_prefill_ws", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), S, nh, hd,
              _ptr(workspace) if workspace is not None else None, nbytes, _stream())
    return out


def attn_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, pos: torch.Tensor,
                out: torch.Tensor | None = None, f16: bool = False,
                workspace: torch.Tensor | None = None, window: int = 0) -> torch.Tensor:
    """Decode attention (the reference's ``attn_101``, gemma4_150/kernels_dsl.py) for a
    batch of sequences: q [m, nh, hd] f32, caches [m, max_seq, hd] f32 (one KV head),
    pos [m] int32 = each sequence's last cached position; returns softmax(q k^T) v over
    keys 0..pos (the last ``window`` of them for a sliding-window layer) as
    [m, nh, hd] f32 (f16 with ``f16``)."""
    _need(q, "q", (torch.float32,))
    _need(k_cache, "k_cache", (torch.float32,))
    _need(v_cache, "v_cache", (torch.float32,))
    _need(pos, "pos", (torch.int32,))
    m, nh, hd = q.shape
    max_seq = k_cache.shape[1]
    if k_cache.shape != (m, max_seq, hd) or v_cache.shape != k_cache.shape or pos.numel() != m:
        raise ValueError("caches must be [m, max_seq, head_dim] and pos [m]")
    if out is None:
        out = torch.empty((m, nh, hd), dtype=torch.float16 if f16 else torch.float32, device=q.device)
    _need(out, "out", (torch.float16,) if f16 else (torch.float32,))
    need = int(_lib.load().sb_attn_decode_workspace_size(m, nh, hd, max_seq))
    if workspace is None:
        workspace = _workspace(q.device, need)
    nbytes = workspace.numel() * workspace.element_size()
    _lib.call("sb_attn_decode_f16" if f16 else "sb_attn_decode", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
              max_seq * hd, pos.data_ptr(), m, nh, hd, max_seq, int(window), out.data_ptr(), workspace.data_ptr(),
              nbytes, _stream())
    return out


def attn_prefill_gemm(q16: torch.Tensor, k16: torch.Tensor, v16: torch.Tensor, out16: torch.Tensor, S: int,
                      window: int = 0, scores: torch.Tensor | None = None, p16: torch.Tensor | None = None
                      ) -> torch.Tensor:
    """Causal prefill attention as the reference's ``_attn_gemm`` chain
    (gemma4_150/prefill_gpu.py:259-313): scores = q k^T on the tcgen05 f16
    GEMM (f32 out), the causal -- and, with ``window``, sliding-window --
    softmax to f16, out = P v.  Any head_dim the GEMM takes (the
    checkpoint's 512 included).  q16 [S, nh, hd], k16 / v16 [>= S, hd],
    out16 [S, nh * hd]; rows of ``scores`` / ``p16`` are [S * nh, >= S]."""
    nh, hd = q16.shape[1], q16.shape[2]
    ld = ((S + 7) // 8) * 8
    if scores is None:
        scores = torch.empty((S * nh, ld), dtype=torch.float32, device=q16.device)
    if p16 is None:
        p16 = torch.empty((S * nh, ld), dtype=torch.float16, device=q16.device)
    lds, ldp = scores.stride(0), p16.stride(0)
    s = _stream()
    _lib.call("sb_gemm_f16_f32out", q16.data_ptr(), k16.data_ptr(), scores.data_ptr(), S * nh, S, hd, 1.0, 1, hd, hd,
              lds, s)
    _lib.call("sb_softmax_causal", scores.data_ptr(), lds, S * nh, nh, 0, S, int(window), p16.data_ptr(), ldp, s)
    _lib.call("sb_gemm_f16", p16.data_ptr(), v16.data_ptr(), out16.data_ptr(), S * nh, hd, S, 1.0, 0, ldp, hd, hd, s)
    return out16


def gemm_q4(A: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, C: torch.Tensor | None = None,
            alpha: float = 1.0, workspace: torch.Tensor | None = None, geglu: bool = False,
            bits: int = 4) -> torch.Tensor:
    """Fused ``_dq`` + ``_gemm``: ``C = f16(alpha * A @ dq_f16(W)^T)``.

    With ``geglu``, W's rows are interleaved (gate, up) pairs and C [M, N/2]
    receives ``f16(gelu_tanh(gate) * up)`` of the f16-rounded pair (the
    reference's gate/up GEMMs + geglu_b, gemma4_150/prefill_gpu.py:365-372)."""
    _need(A, "A", (torch.float16,))
    _need(w, "w", (torch.uint8,))
    _need(scales, "scales", (torch.float16, torch.float32))
    M, K = A.shape
    N = w.shape[0]
    if bits not in (2, 4):
        raise ValueError(f"bits={bits}: the fused GEMM takes 2- or 4-bit codes")
    if w.shape[1] * 8 // bits != K:
        raise ValueError("packed weight does not match A's K")
    if C is None:
        C = torch.empty((M, N // 2 if geglu else N), dtype=torch.float16, device=A.device)
    _need(C, "C", (torch.float16,))
    if workspace is None:
        need = gemm_q4_workspace_size(M, N, K)
        workspace = _workspace(A.device, need)
    fn = ("sb_gemm_q4" if bits == 4 else "sb_gemm_q2") + ("_geglu" if geglu else "")
    _lib.call(fn, _ptr(A), _ptr(w), _ptr(scales), _DT[scales.dtype], group_of(scales, K),
              _ptr(C), M, N, K, float(alpha), K, C.shape[1], _ptr(workspace) if workspace is not None else None,
              0 if workspace is None else workspace.numel() * workspace.element_size(), _stream())
    return C


def gemm_q4_argmax(A: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, row_offset: int = 0,
                   keys: torch.Tensor | None = None, tokens: torch.Tensor | None = None, alpha: float = 1.0,
                   want_tokens: bool = True):
    """lm_head + greedy argmax for every row of A on the tcgen05 GEMM (the
    batched form of ``lmhead_argmax``); returns (keys, tokens)."""
    _need(A, "A", (torch.float16,))
    _need(w, "w", (torch.uint8,))
    _need(scales, "scales", (torch.float16, torch.float32))
    M, K = A.shape
    N = w.shape[0]
    if w.shape[1] * 2 != K:
        raise ValueError("packed weight does not match A's K")
    if keys is None:
        keys = torch.empty(M, dtype=torch.int64, device=A.device)
    if want_tokens and tokens is None:
        tokens = torch.empty(M, dtype=torch.int32, device=A.device)
    _lib.call("sb_gemm_q4_argmax", _ptr(A), _ptr(w), _ptr(scales), _DT[scales.dtype], group_of(scales, K), M, N, K,
              float(alpha), A.stride(0), int(row_offset), _ptr(keys), _ptr(tokens) if want_tokens else None,
              _stream())
    return keys, tokens


def gemm_q4_workspace_size(M: int, N: int, K: int) -> int:
    return int(_lib.load().sb_gemm_q4_workspace_size(M, N, K))


def gemm_q4_kernels(M: int, N: int, K: int) -> int:
    """Kernels one gemm_q4 call of this shape launches (1, or 2 with a split-K finalize)."""
    return int(_lib.load().sb_gemm_q4_kernels(M, N, K))


_WS: dict = {}


def _workspace(device, nbytes: int):
    """A per-device split-K scratch buffer, grown on demand and reused."""
    if nbytes == 0:
        return None
    key = str(device)
    buf = _WS.get(key)
    if buf is None or buf.numel() * 4 < nbytes:
        buf = torch.empty((nbytes + 3) // 4, dtype=torch.float32, device=device)
        _WS[key] = buf
    return buf


def device_status() -> None:
    """Raise if a bounded device-side wait has timed out since the last check."""
    _lib.call("sb_device_status", _stream())


# ---------------------------------------------------------------- per-layer embeddings (PLE)

def _rows(t: torch.Tensor, name: str, n: int) -> int:
    """Row stride of an f32 [m, n] operand whose rows may be spaced (a slice of a wider tensor)."""
    if t.dtype != torch.float32 or t.dim() != 2 or t.shape[1] != n or t.stride(1) != 1 or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA f32 [m, {n}] tensor with unit column stride")
    return t.stride(0)


def gemv_q8(codes: torch.Tensor, row_scale: torch.Tensor, x: torch.Tensor, out: torch.Tensor | None = None,
            ple: torch.Tensor | None = None) -> torch.Tensor:
    """8-bit linear ``y = x @ ((codes - 128) * row_scale).T`` for decode rows (``sb_gemv_q8``).

    ``codes`` [n, k] u8 are the checkpoint's int8 weights +128-biased
    (gemma4_150/export.py:155-157), ``row_scale`` [n] or [n, 1] f32.  With
    ``ple`` ([m, n] f32, rows may be spaced, e.g. ``ple_in[:, layer]``) the
    result is ``gelu_tanh(y) * ple``: the PLE input gate of
    gemma4/reference.py:159 (``plegate_76``).
    """
    _need(codes, "codes", (torch.uint8,))
    _need(row_scale, "row_scale", (torch.float32,))
    n, k = codes.shape
    if row_scale.numel() != n:
        raise ValueError("row_scale must hold one scale per output row")
    x2 = x.reshape(-1, k) if x.is_contiguous() else x
    ldx = _rows(x2, "x", k)
    m = x2.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=torch.float32, device=x.device)
    ldy = _rows(out, "out", n)
    ld_ple = _rows(ple, "ple", n) if ple is not None else 0
    if ple is not None and ple.shape[0] != m:
        raise ValueError("ple must have one row per activation row")
    _lib.call("sb_gemv_q8", _ptr(codes), _ptr(row_scale), _ptr(x2), ldx, _ptr(out), ldy, m, n, k, _ptr(ple), ld_ple,
              _stream())
    return out


def gemv_bf16(w: torch.Tensor, x: torch.Tensor, alpha: float = 1.0, out: torch.Tensor | None = None) -> torch.Tensor:
    """``y = alpha * x @ w.T`` for a bf16 weight [n, k] (``sb_gemv_bf16``; an f16
    weight, as export.py stores the per-layer projection, takes ``sb_gemv_f16``),
    f32 rows in and out."""
    _need(w, "w", (torch.bfloat16, torch.int16, torch.float16))
    n, k = w.shape
    x2 = x.reshape(-1, k) if x.is_contiguous() else x
    ldx = _rows(x2, "x", k)
    m = x2.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=torch.float32, device=x.device)
    ldy = _rows(out, "out", n)
    fn = "sb_gemv_f16" if w.dtype == torch.float16 else "sb_gemv_bf16"
    _lib.call(fn, _ptr(w), float(alpha), _ptr(x2), ldx, _ptr(out), ldy, m, n, k, _stream())
    return out


def ple_gather(ids: torch.Tensor, table: torch.Tensor, scales: torch.Tensor, ple_scale: float,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """Scaled 4-bit PLE table rows [m, cols] (``sb_ple_gather``; plegather_01,
    gemma4_150/kernels_dsl.py:457-478).  ``table`` [vocab, cols/2] u8,
    ``scales`` [vocab, cols/group] f32, ``ids`` [m] int32."""
    _need(ids, "ids", (torch.int32,))
    _need(table, "table", (torch.uint8,))
    _need(scales, "scales", (torch.float32,))
    vocab, cols = table.shape[0], table.shape[1] * 2
    group = group_of(scales, cols)
    m = ids.numel()
    if out is None:
        out = torch.empty(m, cols, dtype=torch.float32, device=ids.device)
    _need(out, "out", (torch.float32,))
    _lib.call("sb_ple_gather", _ptr(ids), _ptr(table), _ptr(scales), vocab, cols, group, float(ple_scale), _ptr(out),
              m, _stream())
    return out


def ple_input(x: torch.Tensor, ids: torch.Tensor, table: torch.Tensor, scales: torch.Tensor, w_proj: torch.Tensor,
              w_norm: torch.Tensor, n_layers: int, d: int, eps: float, ple_scale: float,
              out: torch.Tensor | None = None, ctx: torch.Tensor | None = None,
              w_proj16: torch.Tensor | None = None) -> torch.Tensor:
    """Per-layer inputs [m, n_layers, d] of ``ReferenceGemma4._ple_input``
    (gemma4/reference.py:92-101): the bf16 model projection of the scaled
    embedding ``x`` times hidden**-0.5, RMS-normed per layer slice, plus the
    gathered table row, times 2**-0.5 (``sb_gemv_bf16`` + ``sb_ple_combine``).
    With more than ``PLE_GEMV_ROWS`` rows and an f16 copy of the projection
    (``w_proj16``) the projection runs as a tcgen05 GEMM on f16 operands."""
    _need(ids, "ids", (torch.int32,))
    _need(table, "table", (torch.uint8,))
    _need(scales, "scales", (torch.float32,))
    _need(w_norm, "w_norm", (torch.float32,))
    hidden = x.shape[-1]
    m = ids.numel()
    cols = n_layers * d
    if table.shape[1] * 2 != cols or w_proj.shape != (cols, hidden) or w_norm.numel() != d:
        raise ValueError("PLE table, projection or norm does not match n_layers * d")
    if m > PLE_GEMV_ROWS and w_proj16 is not None:
        _need(w_proj16, "w_proj16", (torch.float16,))
        x2 = x.reshape(m, hidden)
        _need(x2, "x", (torch.float32,))
        x16 = torch.empty(m, hidden, dtype=torch.float16, device=x.device)
        _lib.call("sb_cast_f16", _ptr(x2), _ptr(x16), m * hidden, _stream())
        if ctx is None:
            ctx = torch.empty(m, cols, dtype=torch.float32, device=x.device)
        _lib.call("sb_gemm_f16_f32out", _ptr(x16), _ptr(w_proj16), _ptr(ctx), m, cols, hidden,
                  float(hidden ** -0.5), 1, hidden, hidden, cols, _stream())
    else:
        ctx = gemv_bf16(w_proj, x.reshape(m, hidden), alpha=float(hidden ** -0.5), out=ctx)
    if out is None:
        out = torch.empty(m, n_layers, d, dtype=torch.float32, device=x.device)
    _need(out, "out", (torch.float32,))
    _lib.call("sb_ple_combine", _ptr(ctx), _ptr(ids), _ptr(table), _ptr(scales), table.shape[0], _ptr(w_norm),
              n_layers, d, group_of(scales, cols), float(ple_scale), float(eps), _ptr(out), m, _stream())
    return out


def ple_norm_add(proj: torch.Tensor, hidden: torch.Tensor, w_post: torch.Tensor, layer_scalar: float, eps: float,
                 w_next: torch.Tensor | None = None, h_out: torch.Tensor | None = None,
                 h16_out: torch.Tensor | None = None) -> torch.Tensor:
    """In place ``hidden = (hidden + rmsnorm(proj) * w_post) * layer_scalar``
    (gemma4/reference.py:160-163), then optionally the next layer's input
    norm into ``h_out`` / ``h16_out`` (``sb_ple_norm_add``)."""
    for t, name in ((proj, "proj"), (hidden, "hidden"), (w_post, "w_post")):
        _need(t, name, (torch.float32,))
    n = hidden.shape[-1]
    m = hidden.numel() // n
    if proj.shape != hidden.shape:
        raise ValueError("proj and hidden must have the same shape")
    _lib.call("sb_ple_norm_add", _ptr(proj), _ptr(hidden), _ptr(w_post), float(layer_scalar), _ptr(w_next),
              _ptr(h_out), _ptr(h16_out), m, n, float(eps), _stream())
    return hidden


def ple_block(hidden: torch.Tensor, ple_in: torch.Tensor, layer: dict, eps: float,
              w_next: torch.Tensor | None = None, h_out: torch.Tensor | None = None,
              h16_out: torch.Tensor | None = None) -> torch.Tensor:
    """One layer's PLE block on ``hidden`` [m, H] in place (gemma4/reference.py:154-163):
    ``g = gelu_tanh(W_gate @ x) * ple_in``, ``x = (x + rmsnorm(W_proj @ g) * w_post) * scalar``.

    ``ple_in`` is that layer's [m, d] slice of :func:`ple_input`; ``layer``
    holds ``gate``/``proj`` (codes, row scales) on the device, ``post_norm``
    and ``scalar``.  Up to ``PLE_GEMV_ROWS`` rows (decode): three launches,
    gate GEMV + GELU * ple, projection GEMV, norm-add tail, all f32.  More rows
    (prefill): the two linears run as tcgen05 GEMMs on f16 operands (the 8-bit
    weights dequantised to f16 once, cached in ``layer`` as ``gate16`` /
    ``proj16``), as the reference's prefill does (gemma4_150/kernels_dsl.py:1775).
    """
    m, H = hidden.shape
    if m <= PLE_FUSED_TAIL_ROWS:
        # gate GEMV (+ gelu * ple), then the projection GEMV whose last CTA runs the norm-add tail
        g = gemv_q8(layer["gate"][0], layer["gate"][1], hidden, ple=ple_in)
        return ple_proj_norm_add(layer["proj"][0], layer["proj"][1], g, hidden, layer["post_norm"],
                                 layer["scalar"], eps, w_next, h_out, h16_out)
    if m <= PLE_GEMV_ROWS:
        g = gemv_q8(layer["gate"][0], layer["gate"][1], hidden, ple=ple_in)
        proj = gemv_q8(layer["proj"][0], layer["proj"][1], g)
    else:
        d = layer["gate"][0].shape[0]
        if "gate16" not in layer:
            layer["gate16"] = dequant_f16(layer["gate"][0], layer["gate"][1].reshape(-1), H, d, bits=8)
            layer["proj16"] = dequant_f16(layer["proj"][0], layer["proj"][1].reshape(-1), d, H, bits=8)
        dev = hidden.device
        x16 = torch.empty(m, H, dtype=torch.float16, device=dev)
        _lib.call("sb_cast_f16", _ptr(hidden), _ptr(x16), m * H, _stream())
        # the gate's output is one or two 128 x 256 tiles wide: split K so the GEMM covers the SMs
        kbs, tiles = -(-H // 64), -(-m // 128) * -(-d // 256)
        splits = max(z for z in range(1, 9) if kbs % z == 0 and (z == 1 or tiles * z <= _num_sms(dev)))
        pre = torch.empty(splits, m, d, dtype=torch.float32, device=dev)
        _lib.call("sb_gemm_f16_f32out_splitk", _ptr(x16), _ptr(layer["gate16"]), _ptr(pre), m, d, H, 1.0, 1, H, H,
                  d, splits, _stream())
        g16 = torch.empty(m, d, dtype=torch.float16, device=dev)
        _lib.call("sb_ple_gate_act", _ptr(pre), d, m * d, splits, _ptr(ple_in), _rows(ple_in, "ple_in", d),
                  _ptr(g16), d, m, d, _stream())
        proj = torch.empty(m, H, dtype=torch.float32, device=dev)
        _lib.call("sb_gemm_f16_f32out", _ptr(g16), _ptr(layer["proj16"]), _ptr(proj), m, H, d, 1.0, 1, d, d, H,
                  _stream())
    return ple_norm_add(proj, hidden, layer["post_norm"], layer["scalar"], eps, w_next, h_out, h16_out)


PLE_GEMV_ROWS = 16
# rows up to which ple_block runs the projection with its norm-add tail in one launch
# (sb_ple_proj_norm_add).  Off: a block alone measured 7.65 against 8.27 us at one row, but
# the 35-layer decode chain 280 against 253 us per token, because the separate tail kernel's
# launch overlaps the GEMV under programmatic dependent launch while the last CTA's tail does
# not; at 8 rows (26.5 against 20.1 us) the last CTA also runs every row's tail in turn.
PLE_FUSED_TAIL_ROWS = 0
_SMS: dict = {}
_COUNTERS: dict = {}


def _counter(dev) -> torch.Tensor:
    """A zeroed device u32 per device for last-arriver tails; each launch re-arms it."""
    key = str(dev)
    if key not in _COUNTERS:
        _COUNTERS[key] = torch.zeros(1, dtype=torch.int32, device=dev)
    return _COUNTERS[key]


def ple_proj_norm_add(codes: torch.Tensor, row_scale: torch.Tensor, g: torch.Tensor, hidden: torch.Tensor,
                      w_post: torch.Tensor, layer_scalar: float, eps: float, w_next: torch.Tensor | None = None,
                      h_out: torch.Tensor | None = None, h16_out: torch.Tensor | None = None,
                      proj: torch.Tensor | None = None, counter: torch.Tensor | None = None) -> torch.Tensor:
    """PLE projection GEMV + norm-add tail in one launch (``sb_ple_proj_norm_add``,
    ``pleproj_77``): hidden [m <= 8, H] updated in place.  Launches on one
    stream may share the counter; concurrent streams need their own."""
    _need(codes, "codes", (torch.uint8,))
    _need(row_scale, "row_scale", (torch.float32,))
    for t, name in ((g, "g"), (hidden, "hidden"), (w_post, "w_post")):
        _need(t, name, (torch.float32,))
    n, k = codes.shape
    m = hidden.shape[0]
    if tuple(hidden.shape) != (m, n) or tuple(g.shape) != (m, k):
        raise ValueError("hidden must be [m, n] and g [m, k] for codes [n, k]")
    if proj is None:
        proj = torch.empty(m, n, dtype=torch.float32, device=hidden.device)
    if counter is None:
        counter = _counter(hidden.device)
    _lib.call("sb_ple_proj_norm_add", _ptr(codes), _ptr(row_scale), _ptr(g), k, _ptr(proj), m, n, k, _ptr(hidden),
              _ptr(w_post), float(layer_scalar), _ptr(w_next), _ptr(h_out), _ptr(h16_out), float(eps),
              _ptr(counter), _stream())
    return hidden


def _num_sms(dev) -> int:
    key = str(dev)
    if key not in _SMS:
        _SMS[key] = torch.cuda.get_device_properties(dev).multi_processor_count
    return _SMS[key]
