"""ctypes binding of ``libslang_b200.so`` (declared in ``include/slang_b200.h``).

The library is built in-tree by ``slang_b200.build``.  Loading fails loudly
when it is missing: there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libslang_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "slang_b200.h")

SB_OK, SB_ERR_ARG, SB_ERR_ALIGN, SB_ERR_CUDA, SB_ERR_TIMEOUT, SB_ERR_WORKSPACE = 0, 1, 2, 3, 4, 5
SB_F16, SB_F32 = 1, 2

_vp, _i, _f, _sz, _i64 = C.c_void_p, C.c_int, C.c_float, C.c_size_t, C.c_int64

SIGNATURES = {
    "sb_version": ([], C.c_char_p),
    "sb_last_error": ([], C.c_char_p),
    "sb_device_status": ([_vp], _i),
    "sb_dequant_f16": ([_vp, _i, _vp, _i, _i, _vp, _i, _i, _vp], _i),
    "sb_gemv_q4": ([_vp, _vp, _i, _i, _vp, _i, _vp, _i, _i, _i, _i, _vp], _i),
    "sb_gemv_q2": ([_vp, _vp, _i, _i, _vp, _i, _vp, _i, _i, _i, _i, _vp], _i),
    "sb_lmhead_argmax": ([_vp, _vp, _i, _i, _vp, _i, _i, _i, _i, _i64, _vp, _vp, _vp, _vp], _i),
    "sb_lmhead_argmax_q2": ([_vp, _vp, _i, _i, _vp, _i, _i, _i, _i, _i64, _vp, _vp, _vp, _vp], _i),
    "sb_keys_to_tokens": ([_vp, _vp, _i, _vp], _i),
    "sb_gemm_f16": ([_vp, _vp, _vp, _i, _i, _i, _f, _i, _i, _i, _i, _vp], _i),
    "sb_gemm_q4": ([_vp, _vp, _vp, _i, _i, _vp, _i, _i, _i, _f, _i, _i, _vp, _sz, _vp], _i),
    "sb_gemm_q4_geglu": ([_vp, _vp, _vp, _i, _i, _vp, _i, _i, _i, _f, _i, _i, _vp, _sz, _vp], _i),
    "sb_gemm_q2": ([_vp, _vp, _vp, _i, _i, _vp, _i, _i, _i, _f, _i, _i, _vp, _sz, _vp], _i),
    "sb_gemm_q2_geglu": ([_vp, _vp, _vp, _i, _i, _vp, _i, _i, _i, _f, _i, _i, _vp, _sz, _vp], _i),
    "sb_gemm_q4_workspace_size": ([_i, _i, _i], _sz),
    "sb_gemm_q4_kernels": ([_i, _i, _i], _i),
    "sb_gemm_q4_trace": ([_vp, _sz], _i),
    "sb_attn_prefill_trace": ([_vp, _sz], _i),
    "sb_gemv_trace": ([_vp, _sz], _i),
    "sb_gemm_q4_noalloc": ([_vp, _vp, _vp, _i, _i, _vp, _i, _i, _i, _f, _i, _i, _vp], _i),
    "sb_gemm_f16_f32out": ([_vp, _vp, _vp, _i, _i, _i, _f, _i, _i, _i, _i, _vp], _i),
    "sb_embed_q4": ([_vp, _vp, _i, _i, _vp, _i, _i, _f, _vp, _vp, _vp], _i),
    "sb_embed_q2": ([_vp, _vp, _i, _i, _vp, _i, _i, _f, _vp, _vp, _vp], _i),
    "sb_add_rmsnorm": ([_vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _i, _i, _f, _vp], _i),
    "sb_qkv_prep": ([_vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp, _vp, _vp, _vp, _vp, _vp,
                     _i64, _vp], _i),
    "sb_softmax_causal": ([_vp, _i, _i, _i, _i, _i, _i, _vp, _i, _vp], _i),
    "sb_geglu": ([_vp, _i, _i, _i, _vp, _vp, _vp], _i),
    "sb_attn_prefill": ([_vp, _vp, _vp, _vp, _i, _i, _i, _vp], _i),
    "sb_attn_prefill_ws": ([_vp, _vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp], _i),
    "sb_peer_mailbox_size": ([], _sz),
    "sb_peer_set_wait_limit_ns": ([C.c_uint64], _i),
    "sb_peer_buffer_create": ([_sz, _vp, _vp], _i),
    "sb_peer_buffer_open": ([_vp, _vp], _i),
    "sb_peer_buffer_close": ([_vp], _i),
    "sb_peer_buffer_free": ([_vp], _i),
    "sb_lmhead_argmax_peer": ([_vp, _vp, _i, _i, _vp, _i, _i, _i, _i, _i64, _vp, _i, _vp, _vp, _vp, _vp], _i),
    "sb_gemm_q4_argmax": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _i, _i64, _vp, _vp, _vp], _i),
    "sb_attn_decode_f16": ([_vp, _vp, _vp, _i64, _vp, _i, _i, _i, _i, _i, _vp, _vp, _sz, _vp], _i),
    "sb_attn_prefill_workspace_size": ([_i, _i, _i], _sz),
    "sb_attn_decode": ([_vp, _vp, _vp, _i64, _vp, _i, _i, _i, _i, _i, _vp, _vp, _sz, _vp], _i),
    "sb_attn_decode_workspace_size": ([_i, _i, _i, _i], _sz),
    "sb_step_advance": ([_vp, _vp, _vp, _vp, _i, _i, _vp], _i),
    "sb_gemv_q8": ([_vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _vp, _i, _vp], _i),
    "sb_ple_proj_norm_add": ([_vp, _vp, _vp, _i, _vp, _i, _i, _i, _vp, _vp, _f, _vp, _vp, _vp, _f, _vp, _vp], _i),
    "sb_gemv_bf16": ([_vp, _f, _vp, _i, _vp, _i, _i, _i, _i, _vp], _i),
    "sb_gemv_f16": ([_vp, _f, _vp, _i, _vp, _i, _i, _i, _i, _vp], _i),
    "sb_gemv_srq": ([_vp, _i, _vp, _i, _i, _vp, _i, _f, _f, _vp, _vp, _i, _i, _i, _i, _vp], _i),
    "sb_srq": ([_vp, _i, _sz, _f, _vp, _i, _vp], _i),
    "sb_gemv_norm_add": ([_vp, _i, _vp, _i, _i, _vp, _i, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _f, _vp, _vp], _i),
    "sb_ple_norm_add": ([_vp, _vp, _vp, _f, _vp, _vp, _vp, _i, _i, _f, _vp], _i),
    "sb_ple_gather": ([_vp, _vp, _vp, _i, _i, _i, _f, _vp, _i, _vp], _i),
    "sb_ple_combine": ([_vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _f, _f, _vp, _i, _vp], _i),
    "sb_ple_gate_act": ([_vp, _i, _i64, _i, _vp, _i, _vp, _i, _i, _i, _vp], _i),
    "sb_gemm_f16_f32out_splitk": ([_vp, _vp, _vp, _i, _i, _i, _f, _i, _i, _i, _i, _i, _vp], _i),
    "sb_cast_f16": ([_vp, _vp, _i64, _vp], _i),
    "sb_decode_step_fused": ([_vp, _i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _f, _vp, _vp, _vp,
                              _vp, _i, _vp, _vp, _sz, _vp], _i),
    "sb_decode_step_fused_scratch_size": ([_i, _i, _i, _i, _i], _sz),
}


class SlangError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed (code {code}): {msg}")
        self.code = code


_lib = None


def header_symbols() -> list[str]:
    """Every function the public header declares."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(sb_[a-z0-9_]+)\s*\(", text)))


def load() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run `python -m slang_b200.build` (the CUDA library is required)")
    lib = C.CDLL(LIB_PATH)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def call(name: str, *args) -> int:
    """Call an entry point; raise SlangError on a non-zero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != SB_OK:
        raise SlangError(name, rc, lib.sb_last_error().decode(errors="replace"))
    return rc
