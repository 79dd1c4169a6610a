"""CPU oracle of the rec decode hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline leg and
--impl reference) may import this package.  It is the checker; the product
path (rec_b200) never calls it.

`rec_oracle.c` restates, in the canonical operation order of the CUDA
kernels, the reference's algorithms (recursive-oss/rec,
engine/src/rec_mlx/model.py and kernels/megakernel.py; see the C file header
for line citations).  With identical inputs it matches the GPU bit for bit.
`semantic.py` restates the reference's MLX formulas without any fixed order
and is used for tolerance checks (rel-L2 2e-3 in bf16).

Parity against MLX itself is unpinned: mlx 0.32.0 / mlx-lm 0.31.3 cannot be
installed here and the reference holds no golden vectors; the reference's
own kernel tests (engine/tests/test_kernel_routing.py,
kernels/activation_optimization.py) are restated as known-answer tests.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "librec_oracle.so"
_lib = None

_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        from . import build as _build

        _build.build()
        L = C.CDLL(str(LIB_PATH))
        L.orc_exp.restype = C.c_float
        L.orc_exp.argtypes = [C.c_float]
        L.orc_exp_n.argtypes = [_f32p, _f32p, C.c_int64]
        L.orc_aexp_n.argtypes = [_f32p, _f32p, C.c_int64]
        L.orc_quantize_affine.argtypes = [_f32p, C.c_int64, C.c_int, C.c_int, _u32p, _u16p, _u16p]
        L.orc_gemv_int4.argtypes = [_u32p, _u16p, _u16p, C.c_int, C.c_int64, C.c_int, _u16p, _u16p]
        L.orc_rmsnorm.argtypes = [_u16p, _u16p, C.c_int, C.c_float, _u16p]
        L.orc_rope_table.argtypes = [C.c_float, C.c_int32, C.c_int32, _f32p]
        L.orc_router_logits.argtypes = [_u16p, _u16p, C.c_int, C.c_int, _f32p]
        L.orc_route.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_void_p, _i32p, _f32p]
        L.orc_swiglu.restype = C.c_uint16
        L.orc_swiglu.argtypes = [C.c_uint16, C.c_uint16]
        L.orc_argmax_bf16.restype = C.c_int32
        L.orc_argmax_bf16.argtypes = [_u16p, C.c_int64]
        L.orc_partial_bytes.restype = C.c_int
        L.orc_attention_supers.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                           C.c_void_p, C.c_int]
        L.orc_attention_supers_shard.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                                 C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]
        L.orc_attention_final.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.orc_sample.restype = C.c_int32
        L.orc_sample.argtypes = [_u16p, C.c_int64, C.c_void_p, C.c_int, C.c_void_p, _f32p]
        L.orc_sample_masked.restype = C.c_int32
        L.orc_sample_masked.argtypes = [_u16p, C.c_int64, C.c_void_p, C.c_int, C.c_void_p, _f32p, C.c_void_p]
        L.orc_log.restype = C.c_float
        L.orc_log.argtypes = [C.c_float]
        L.orc_log_n.argtypes = [_f32p, _f32p, C.c_int64]
        L.orc_to_bf.restype = C.c_uint16
        L.orc_to_bf.argtypes = [C.c_float]
        L.orc_to_hf.restype = C.c_uint16
        L.orc_to_hf.argtypes = [C.c_float]
        L.orc_hf.restype = C.c_float
        L.orc_hf.argtypes = [C.c_uint16]
        L.orc_decode_step.restype = C.c_int
        L.orc_mix.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p]
        L.orc_select_topk.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.orc_kv_store.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.orc_token_logprob.restype = C.c_float
        L.orc_token_logprob.argtypes = [_u16p, C.c_int64, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int32]
        L.orc_set_threads.restype = C.c_int
        L.orc_set_threads.argtypes = [C.c_int]
        _lib = L
    return _lib


def set_threads(n: int) -> int:
    """Sets the oracle's OpenMP thread count (overrides OMP_NUM_THREADS);
    returns the count now in use."""
    return int(lib().orc_set_threads(int(n)))


# ---------------------------------------------------------------- bf16 / fp16
def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    """Round to nearest even, NaN -> 0x7fff (same as the C oracle and CUDA)."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def fp16_to_f32(u16: np.ndarray) -> np.ndarray:
    return np.asarray(u16, dtype=np.uint16).view(np.float16).astype(np.float32)


def scale_to_f32(u16: np.ndarray, sd: int) -> np.ndarray:
    return fp16_to_f32(u16) if sd == 0 else bf16_to_f32(u16)


# ---------------------------------------------------------------- primitives
def exp(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().orc_exp_n(x.ravel(), y.ravel(), x.size)
    return y


def aexp(x: np.ndarray) -> np.ndarray:
    """The attention softmax exp (x <= 0; 0 at and below -87)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().orc_aexp_n(x.ravel(), y.ravel(), x.size)
    return y


def quantize(w: np.ndarray, bits: int = 4, sd: int = 0):
    """MLX affine quantization, group 64 along the last axis.  Returns codes
    uint32[..., K*bits/32], scales and biases uint16[..., K/64]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    *lead, k = w.shape
    groups = w.size // 64
    codes = np.zeros((*lead, k * bits // 32), np.uint32)
    scales = np.zeros((*lead, k // 64), np.uint16)
    biases = np.zeros_like(scales)
    lib().orc_quantize_affine(w.reshape(-1), groups, bits, sd, codes.reshape(-1), scales.reshape(-1),
                              biases.reshape(-1))
    return codes, scales, biases


def dequantize(codes, scales, biases, bits: int = 4, sd: int = 0) -> np.ndarray:
    codes = np.asarray(codes, dtype=np.uint32)
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    q = ((codes[..., None] >> shifts) & ((1 << bits) - 1)).reshape(*codes.shape[:-1], -1).astype(np.float32)
    s = np.repeat(scale_to_f32(scales, sd), 64, axis=-1)
    b = np.repeat(scale_to_f32(biases, sd), 64, axis=-1)
    return s * q + b


def gemv(codes, scales, biases, x_bf16, sd: int = 0) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    n, k8 = codes.shape
    y = np.zeros(n, np.uint16)
    lib().orc_gemv_int4(codes.reshape(-1), np.ascontiguousarray(scales, np.uint16).reshape(-1),
                        np.ascontiguousarray(biases, np.uint16).reshape(-1), sd, n, k8 * 8,
                        np.ascontiguousarray(x_bf16, np.uint16), y)
    return y


def rmsnorm(h_bf16, w_bf16, eps: float = 1e-6) -> np.ndarray:
    h = np.ascontiguousarray(h_bf16, np.uint16)
    out = np.zeros_like(h)
    lib().orc_rmsnorm(h, np.ascontiguousarray(w_bf16, np.uint16), h.size, eps, out)
    return out


def rope_table(theta: float, pos0: int, n: int) -> np.ndarray:
    cs = np.zeros((n, 128), np.float32)
    lib().orc_rope_table(theta, pos0, n, cs.reshape(-1))
    return cs


def router_logits(w_bf16, x_bf16) -> np.ndarray:
    w = np.ascontiguousarray(w_bf16, np.uint16)
    e, h = w.shape
    out = np.zeros(e, np.float32)
    lib().orc_router_logits(w.reshape(-1), np.ascontiguousarray(x_bf16, np.uint16), e, h, out)
    return out


def route(logits, k: int, mode: int = 0, bias=None):
    logits = np.ascontiguousarray(logits, np.float32)
    ids = np.zeros(k, np.int32)
    w = np.zeros(k, np.float32)
    bias_arr = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().orc_route(logits, logits.size, k, mode, None if bias_arr is None else bias_arr.ctypes.data, ids, w)
    return ids, w


def select_topk(p, choice, k: int):
    p = np.ascontiguousarray(p, np.float32)
    choice = np.ascontiguousarray(choice, np.float32)
    ids = np.zeros(k, np.int32)
    w = np.zeros(k, np.float32)
    lib().orc_select_topk(p.ctypes.data, choice.ctypes.data, p.size, k, ids.ctypes.data, w.ctypes.data)
    return ids, w


def mix(down_bf16, weights) -> np.ndarray:
    d = np.ascontiguousarray(down_bf16, np.uint16)
    k, h = d.shape
    w = np.ascontiguousarray(weights, np.float32)
    out = np.zeros(h, np.uint16)
    lib().orc_mix(d.ctypes.data, h, w.ctypes.data, k, out.ctypes.data)
    return out


def swiglu(g_bf16: int, u_bf16: int) -> int:
    return int(lib().orc_swiglu(int(g_bf16), int(u_bf16)))


def argmax_bf16(x) -> int:
    x = np.ascontiguousarray(x, np.uint16)
    return int(lib().orc_argmax_bf16(x, x.size))


def log(x: np.ndarray) -> np.ndarray:
    """The kernels' canonical natural logarithm (sampler)."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().orc_log_n(x, y, x.size)
    return y


def sample(logits_bf16, history, params, uniforms, allow=None) -> int:
    """orc_sample on one row: logits uint16[V] (bf16 bits), history int32 ids,
    params a rec_b200.abi.RecSampling, uniforms float32[V] (or None when the
    temperature is 0), allow an optional grammar mask (uint32[ceil(V/32)],
    bit i & 31 of word i >> 5 set = id i allowed; orc_sample_masked)."""
    from rec_b200 import abi

    lg = np.ascontiguousarray(logits_bf16, np.uint16)
    h = np.ascontiguousarray(history if history is not None else np.zeros(0), np.int32)
    u = np.ascontiguousarray(uniforms if uniforms is not None else np.zeros(lg.size), np.float32)
    assert isinstance(params, abi.RecSampling)
    hp = h.ctypes.data if h.size else None
    if allow is None:
        return int(lib().orc_sample(lg, lg.size, hp, h.size, C.byref(params), u))
    m = np.ascontiguousarray(allow, np.uint32)
    assert m.size >= (lg.size + 31) // 32
    return int(lib().orc_sample_masked(lg, lg.size, hp, h.size, C.byref(params), u, m.ctypes.data))


def token_logprob(logits_bf16, history, params, token: int, allow=None) -> float:
    """orc_token_logprob: the reference's reported log-probability of
    `token` (report = penalised, masked logits / T; report[token] -
    logsumexp(report)) in the GPU kernel's summation order."""
    lg = np.ascontiguousarray(logits_bf16, np.uint16)
    h = np.ascontiguousarray(history if history is not None else np.zeros(0), np.int32)
    m = None if allow is None else np.ascontiguousarray(allow, np.uint32)
    return float(lib().orc_token_logprob(lg, lg.size, h.ctypes.data if h.size else None, h.size, C.byref(params),
                                         None if m is None else m.ctypes.data, int(token)))


def pack_allow(allowed_ids, vocab: int) -> np.ndarray:
    """Grammar mask words (uint32[ceil(vocab/32)]) from a list of allowed ids."""
    m = np.zeros((vocab + 31) // 32, np.uint32)
    for i in np.asarray(allowed_ids, np.int64).ravel():
        m[i >> 5] |= np.uint32(1) << np.uint32(i & 31)
    return m


PARTIAL_FLOATS = 130  # (m, l, acc[128]) of one head's attention partial


def attention_supers(q_bf16, kv: dict, n_kv_heads: int, capacity: int, bits: int, T: int, n_super: int):
    """Super-chunk partials float32 [Hq, n_super, 130] of tokens [0, T) of one
    layer's cache (kv: codes / scales / biases arrays [Hkv, capacity, ...])."""
    from rec_b200 import abi

    q = np.ascontiguousarray(q_bf16, np.uint16)
    hq = q.size // 128
    arrs = [np.ascontiguousarray(kv[n]) for n in ("k_codes", "k_scales", "k_biases", "v_codes", "v_scales",
                                                  "v_biases")]
    rec = abi.RecKVLayer(*(a.ctypes.data for a in arrs))
    out = np.zeros((hq, n_super, PARTIAL_FLOATS), np.float32)
    L = lib()
    assert L.orc_partial_bytes() == PARTIAL_FLOATS * 4
    L.orc_attention_supers(q.ctypes.data, C.addressof(rec), hq, n_kv_heads, capacity, bits, T, out.ctypes.data,
                           n_super)
    return out


def attention_supers_shard(q_bf16, kv: dict, n_kv_heads: int, capacity: int, bits: int, T: int, base: int,
                           s_lo: int, s_hi: int):
    """Super-chunk partials [Hq, s_hi - s_lo, 130] of super-chunks [s_lo, s_hi)
    of a T-token context, from a cache slice holding tokens base, base+1, ...
    (kv arrays [Hkv, capacity, ...]): what one rank of a split session owns."""
    from rec_b200 import abi

    q = np.ascontiguousarray(q_bf16, np.uint16)
    hq = q.size // 128
    arrs = [np.ascontiguousarray(kv[n]) for n in ("k_codes", "k_scales", "k_biases", "v_codes", "v_scales",
                                                  "v_biases")]
    rec = abi.RecKVLayer(*(a.ctypes.data for a in arrs))
    out = np.zeros((hq, max(0, s_hi - s_lo), PARTIAL_FLOATS), np.float32)
    if s_hi > s_lo:
        lib().orc_attention_supers_shard(q.ctypes.data, C.addressof(rec), hq, n_kv_heads, capacity, bits, T, base,
                                         s_lo, s_hi, out.ctypes.data)
    return out


def attention_final(supers, sinks_bf16=None):
    """LSE merge of [Hq, n_super, 130] partials (after the optional sink) into
    bf16 [Hq * 128]."""
    sp = np.ascontiguousarray(supers, np.float32)
    hq, n_super, _ = sp.shape
    out = np.zeros(hq * 128, np.uint16)
    sk = None if sinks_bf16 is None else np.ascontiguousarray(sinks_bf16, np.uint16)
    lib().orc_attention_final(sp.ctypes.data, hq, n_super, None if sk is None else sk.ctypes.data,
                              out.ctypes.data)
    return out
