"""Loader of the in-tree CUDA library librec_b200.so.

The library is the only compute path: if it is missing or fails to load, every
entry point raises.  There is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

from . import abi

LIB_PATH = Path(__file__).resolve().parent / "librec_b200.so"
_lib = None

_SIGNATURES = {
    "rec_last_error": (C.c_int, [C.c_char_p, C.c_size_t]),
    "rec_gemv_int4": (C.c_int, [C.POINTER(abi.RecQMat), C.c_int32, C.c_int64, C.c_int32, C.c_void_p, C.c_void_p,
                                C.c_float, C.c_void_p, C.c_void_p]),
    "rec_gemv_int4_argmax_noalloc": (C.c_int, [C.POINTER(abi.RecQMat), C.c_int32, C.c_int64, C.c_int32,
                                               C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_void_p,
                                               C.c_void_p]),
    "rec_sample_logits": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int64, C.c_void_p, C.c_int32,
                                    C.POINTER(abi.RecSampling), C.c_void_p, C.c_void_p, C.c_void_p]),
    "rec_set_shard": (C.c_int, [C.c_void_p, C.POINTER(abi.RecShard)]),
    "rec_exchange_bytes": (C.c_size_t, [C.c_void_p]),
    "rec_sample_logits_masked": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int64, C.c_void_p, C.c_int32,
                                           C.POINTER(abi.RecSampling), C.c_void_p, C.c_void_p, C.c_int64,
                                           C.c_void_p, C.c_void_p]),
    "rec_prefill_attention": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.POINTER(abi.RecKVLayer), C.c_int32,
                                        C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "rec_prefill_workspace_bytes": (C.c_size_t, [C.c_void_p, C.c_int32]),
    "rec_prefill_chunk": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_size_t,
                                    C.c_void_p]),
    "rec_prefill_chunk_layers": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                           C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "rec_set_kv_rows": (C.c_int, [C.c_void_p, C.c_int32]),
    "rec_decode_layers": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p,
                                    C.c_void_p]),
    "rec_set_fault_injection": (C.c_int, [C.c_void_p, C.c_uint32, C.c_int32]),
    "rec_token_logprob": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int64, C.c_void_p, C.c_int32,
                                    C.POINTER(abi.RecSampling), C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                                    C.c_void_p]),
    "rec_lmhead_sample": (C.c_int, [C.POINTER(abi.RecQMat), C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_int32,
                                    C.c_void_p, C.c_float, C.c_void_p, C.c_int32, C.POINTER(abi.RecSampling),
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "rec_prefill_gemm": (C.c_int, [C.POINTER(abi.RecQMat), C.c_int32, C.c_int64, C.c_int32, C.c_void_p, C.c_int64,
                                   C.c_void_p, C.c_void_p, C.c_void_p]),
    "rec_prefill_moe_workspace_bytes": (C.c_size_t, [C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    "rec_prefill_moe": (C.c_int, [C.POINTER(abi.RecQMat), C.POINTER(abi.RecQMat), C.POINTER(abi.RecQMat), C.c_int32,
                                  C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_int64, C.c_int32, C.c_void_p,
                                  C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p,
                                  C.c_void_p]),
    "rec_decode_sampled": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.POINTER(abi.RecSampling),
                                     C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_int32,
                                     C.c_void_p, C.c_void_p, C.c_void_p]),
    "rec_router_moe": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "rec_kv_append_bulk": (C.c_int, [C.POINTER(abi.RecKVLayer), C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                     C.c_void_p, C.c_int32, C.c_int32, C.c_void_p]),
    "rec_kv_append": (C.c_int, [C.POINTER(abi.RecKVLayer), C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p,
                                C.c_void_p, C.c_void_p, C.c_void_p]),
    "rec_attn_scratch_bytes": (C.c_size_t, [C.c_int32, C.c_int32]),
    "rec_attn_decode": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.POINTER(abi.RecKVLayer), C.c_int32, C.c_int32,
                                  C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p,
                                  C.c_void_p]),
    "rec_quantize_affine": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_void_p]),
    "rec_silu_table": (C.c_int, [C.c_void_p, C.c_void_p]),
    "rec_create": (C.c_int, [C.POINTER(abi.RecModelDesc), C.POINTER(C.c_void_p)]),
    "rec_destroy": (None, [C.c_void_p]),
    "rec_set_weights": (C.c_int, [C.c_void_p, C.POINTER(abi.RecLayerWeights), C.c_int32,
                                  C.POINTER(abi.RecGlobalWeights)]),
    "rec_set_kv": (C.c_int, [C.c_void_p, C.POINTER(abi.RecKVLayer), C.c_int32, C.c_int32]),
    "rec_workspace_bytes": (C.c_size_t, [C.c_void_p]),
    "rec_set_workspace": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "rec_decode_step": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "rec_decode_greedy": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.POINTER(C.c_int32), C.c_int32,
                                    C.c_void_p, C.c_void_p, C.c_void_p]),
    "rec_check_status": (C.c_int, [C.c_void_p, C.c_void_p]),
    "rec_launch_kernel": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p]),
    "rec_schedule_for": (C.c_int32, [C.c_void_p, C.c_int32]),
    "rec_set_profile": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "rec_set_layer_profile": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32]),
}


class RecError(RuntimeError):
    """A device-side status (bounded wait ran out, rejected input)."""


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m rec_b200.build`")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().rec_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(code: int, what: str = "") -> None:
    """Maps a C-ABI return code to the reference's error conventions."""
    if code == abi.REC_OK:
        return
    msg = f"{what}: {last_error()}" if what else last_error()
    if code == abi.REC_ELIMIT:
        raise ValueError("Decode context limit exhausted")
    if code < 0 and code != abi.REC_ECUDA:
        raise ValueError(msg)
    if code > 0:
        raise RecError(f"GPU synchronization failed: device status {code}")
    raise RuntimeError(msg)
