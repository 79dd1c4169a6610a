"""Order-free numpy restatement of the reference's MLX formulas — TEST
INFRASTRUCTURE ONLY (see oracle/__init__.py).

These follow the native MLX model (recursive-oss/rec
engine/src/rec_mlx/model.py) with float64 accumulation and the reference's
bf16 rounding points, and are used to check the canonical restatement and the
CUDA path within the north-star tolerance (rel-L2 2e-3 in bf16).
"""
from __future__ import annotations

import numpy as np

from . import bf16_to_f32, dequantize, f32_to_bf16


def rbf(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(np.asarray(x, np.float32)))


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def gemv(codes, scales, biases, x_bf16, sd: int = 0) -> np.ndarray:
    """fp64 dot of the dequantised matrix with x; float32 result."""
    w = dequantize(codes, scales, biases, 4, sd).astype(np.float64)
    return (w @ bf16_to_f32(x_bf16).astype(np.float64)).astype(np.float32)


def rmsnorm(h_bf16, w_bf16, eps: float = 1e-6) -> np.ndarray:
    """nn.RMSNorm: w * bf16(x * rsqrt(mean(x^2) + eps)) (model.py:266-267)."""
    x = bf16_to_f32(h_bf16).astype(np.float64)
    inv = 1.0 / np.sqrt(np.mean(x * x) + eps)
    return rbf(bf16_to_f32(w_bf16) * rbf((x * inv).astype(np.float32)))


def rope(x: np.ndarray, pos: int, theta: float) -> np.ndarray:
    """nn.RoPE(128, traditional=False, base=theta) on [heads, 128] floats."""
    i = np.arange(64, dtype=np.float64)
    ang = pos * theta ** (-i / 64.0)
    c, s = np.cos(ang), np.sin(ang)
    a, b = x[:, :64].astype(np.float64), x[:, 64:].astype(np.float64)
    return np.concatenate([a * c - b * s, a * s + b * c], axis=1).astype(np.float32)


def attention(q_bf16: np.ndarray, k: np.ndarray, v: np.ndarray, sinks=None, bf16_probs: bool = True) -> np.ndarray:
    """quantized_attention_with_sinks (model.py:108-139) for one query token.
    q: [Hq, 128] bf16 (post-RoPE); k, v: dequantised float [Hkv, T, 128].
    Scores are rounded to bf16 (the quantized matmul returns bf16), softmax in
    fp32 over [scores, sink], probabilities rounded to bf16 before P*V
    (bf16_probs=False keeps them in float64: the exact softmax of the bf16
    scores)."""
    hq = q_bf16.shape[0]
    hkv = k.shape[0]
    rep = hq // hkv
    qs = rbf(bf16_to_f32(q_bf16) * np.float32(1.0 / np.sqrt(128.0)))
    out = np.zeros((hq, 128), np.float32)
    for h in range(hq):
        g = h // rep
        sc = rbf((k[g].astype(np.float64) @ qs[h].astype(np.float64)).astype(np.float32)).astype(np.float64)
        sink = [] if sinks is None else [float(bf16_to_f32(np.array([sinks[h]], np.uint16))[0])]
        allv = np.concatenate([sc, sink])
        p = np.exp(allv - allv.max())
        p = p / p.sum()
        p = rbf(p[: sc.size].astype(np.float32)).astype(np.float64) if bf16_probs else p[: sc.size]
        out[h] = (p @ v[g].astype(np.float64)).astype(np.float32)
    return out


def route(logits: np.ndarray, k: int, mode: int = 0, bias=None):
    """softmax -> top-k -> renormalise (mode 0) or sigmoid + bias selection
    (mode 1, model.py:245-254).  Ties resolve to the lower expert index."""
    l = np.asarray(logits, np.float64)
    if mode == 0:
        p = np.exp(l - l.max())
        p = p / p.sum()
        choice = p
    else:
        p = 1.0 / (1.0 + np.exp(-l))
        choice = p + np.asarray(bias, np.float64)
    ids = np.argsort(-choice, kind="stable")[:k]
    w = p[ids] / (p[ids].sum() + 1e-20)
    return ids.astype(np.int32), w


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """bf16(bf16(g * sig) * u) with sig = bf16(g < 0 ? tail : 1 - tail) and
    tail = 1/(1 + exp(|g|)) in float32 with a correctly rounded exp
    (megakernel.py:770-774)."""
    g = np.asarray(g, np.float32)
    with np.errstate(over="ignore"):
        e = np.exp(np.abs(g).astype(np.float64)).astype(np.float32)
    tail = (np.float32(1) / (np.float32(1) + e)).astype(np.float32)
    sig = rbf(np.where(g < 0, tail, np.float32(1) - tail).astype(np.float32))
    return rbf(rbf(g * sig) * np.asarray(u, np.float32))


def expert_mix(down: np.ndarray, weights: np.ndarray) -> np.ndarray:
    """sum_r bf16(d_r * bf16(w_r)) with a bf16 round after every addition, in
    rank order (mixed_bits.py:42-54, test_kernel_routing.py:154-155)."""
    m = None
    for r in range(down.shape[0]):
        t = rbf(down[r] * rbf(np.float32(weights[r])))
        m = t if m is None else rbf(t + m)
    return m
