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


def attention(q_bf16: np.ndarray, k: np.ndarray, v: np.ndarray, sinks=None, bf16_probs: bool = True,
              bf16_kv: bool = False) -> np.ndarray:
    """quantized_attention_with_sinks (model.py:108-139) for one query token.
    q: [Hq, 128] bf16 (post-RoPE); k, v: dequantised float [Hkv, T, 128].
    Scores are rounded to bf16 (the quantized matmul returns bf16), softmax in
    fp32 over [scores, sink], probabilities rounded to bf16 before P*V
    (bf16_probs=False keeps them in float64: the exact softmax of the bf16
    scores).  bf16_kv: the reference megakernel's bf16 cache
    (megakernel.py:619-693): the scaled query stays fp32 and the scores are
    not rounded."""
    hq = q_bf16.shape[0]
    hkv = k.shape[0]
    rep = hq // hkv
    qs = bf16_to_f32(q_bf16) * np.float32(1.0 / np.sqrt(128.0))
    if not bf16_kv:
        qs = rbf(qs)
    out = np.zeros((hq, 128), np.float32)
    for h in range(hq):
        g = h // rep
        sc = k[g].astype(np.float64) @ qs[h].astype(np.float64)
        if not bf16_kv:
            sc = rbf(sc.astype(np.float32)).astype(np.float64)
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


# ---------------------------------------------------------------- whole model
# The native MLX decoder (recursive-oss/rec engine/src/rec_mlx/model.py) in
# float64 with the reference's bf16 rounding points: every projection output,
# the RoPE'd q / k, the attention output (model.py:108-139), the residual
# adds (model.py:269-271), the router logit (mixed_bits.py:32-38), the SwiGLU
# activation and the rank-order expert mix (mixed_bits.py:42-54), the logits.
# Quantized tensors are dequantized exactly (float32 affine, as MLX does).
# Used to bound the canonical fixed-point order (oracle/rec_oracle.c, and so
# the GPU) against the reference's semantics at layer and model scale.

def _dq(qt, sd: int, rows=None) -> np.ndarray:
    w, s, b = (qt.w, qt.s, qt.b) if rows is None else (qt.w[rows], qt.s[rows], qt.b[rows])
    return dequantize(np.asarray(w, np.uint32), np.asarray(s, np.uint16), np.asarray(b, np.uint16), 4,
                      sd).astype(np.float64)


def _bfv(u16) -> np.ndarray:
    return bf16_to_f32(np.asarray(u16, np.uint16)).astype(np.float64)


def rmsnorm_f(x: np.ndarray, w_bf16, eps: float) -> np.ndarray:
    """rmsnorm on bf16-valued floats; returns bf16-valued float64."""
    x = np.asarray(x, np.float64)
    inv = 1.0 / np.sqrt(np.mean(x * x) + eps)
    return rbf(_bfv(w_bf16) * rbf((x * inv).astype(np.float32))).astype(np.float64)


class SemanticKV:
    """Quantized cache of one layer held by the semantic model: codes /
    scales / biases like the oracle's (model.py:45-82 quantize-on-append)."""

    def __init__(self, layer_arrays: dict, bits: int, vbits: int | None = None):
        self.L = {n: np.array(a, copy=True) for n, a in layer_arrays.items()}
        self.bits = bits
        self.vbits = vbits or bits  # V codes' width (the reference's mixed cache: K 8, V 4)

    def append(self, pos: int, k_bf16v: np.ndarray, v_bf16v: np.ndarray) -> None:
        from . import f32_to_bf16, quantize

        for name, x in (("k", k_bf16v), ("v", v_bf16v)):
            if self.bits == 16:  # a bf16 cache keeps the rows as they are
                self.L[f"{name}_codes"].view(np.uint16)[:, pos] = f32_to_bf16(np.asarray(x, np.float32))
                continue
            c, s, b = quantize(np.asarray(x, np.float32)[:, None, :], self.bits if name == "k" else self.vbits, 1)
            self.L[f"{name}_codes"][:, pos] = c[:, 0]
            self.L[f"{name}_scales"][:, pos] = s[:, 0]
            self.L[f"{name}_biases"][:, pos] = b[:, 0]

    def dequant(self, name: str, upto: int) -> np.ndarray:
        L = self.L
        if self.bits == 16:
            return bf16_to_f32(L[f"{name}_codes"].view(np.uint16)[:, :upto]).astype(np.float64)
        return dequantize(L[f"{name}_codes"][:, :upto], L[f"{name}_scales"][:, :upto], L[f"{name}_biases"][:, :upto],
                          self.bits if name == "k" else self.vbits, 1).astype(np.float64)


def mlp(gate, up, down, sd: int, xn: np.ndarray) -> np.ndarray:
    """SwiGLU MLP (model.py:216-224): bf16 gate / up projections, the
    activation's rounding points, bf16 down projection."""
    g = rbf(_dq(gate, sd) @ xn)
    u = rbf(_dq(up, sd) @ xn)
    return rbf(_dq(down, sd) @ silu_mul(g, u).astype(np.float64))


def layer_step(cfg, L, kv: SemanticKV, h: np.ndarray, pos: int, sd: int) -> np.ndarray:
    """One decoder layer (model.py:258-271) for the token at `pos`; h is the
    bf16-valued residual; returns the new residual (bf16-valued float64).
    Layer options (getattr(L, "kind")): a dense MLP instead of the experts
    (model.py:262-266), no RoPE (model.py:158-163,196-198), attention over the
    last sliding_window positions (model.py:302-313); a shared expert added
    to the routed mix as bf16(mix + shared) (model.py:243,254)."""
    from . import f32_to_bf16

    kind = getattr(L, "kind", 0)
    hq, hkv = cfg.n_q_heads, cfg.n_kv_heads
    xn = rmsnorm_f(h, L.input_norm, cfg.rms_eps)
    q = rbf(_dq(L.q, sd) @ xn).reshape(hq, 128)
    k = rbf(_dq(L.k, sd) @ xn).reshape(hkv, 128)
    v = rbf(_dq(L.v, sd) @ xn).reshape(hkv, 128)
    if L.q_norm is not None:
        q = np.stack([rmsnorm_f(r, L.q_norm, cfg.rms_eps) for r in q])
        k = np.stack([rmsnorm_f(r, L.k_norm, cfg.rms_eps) for r in k])
    if not kind & 2:  # REC_LAYER_NO_ROPE
        q = rbf(rope(q, pos, cfg.rope_theta))
        k = rbf(rope(k, pos, cfg.rope_theta))
    kv.append(pos, k, v)
    K, V = kv.dequant("k", pos + 1), kv.dequant("v", pos + 1)
    if kind & 4:  # REC_LAYER_SLIDING: the last sliding_window positions
        lo = max(0, pos + 1 - cfg.sliding_window)
        K, V = K[:, lo:], V[:, lo:]
    sinks = None if L.sinks is None else np.asarray(L.sinks, np.uint16)
    att = rbf(attention(f32_to_bf16(q.astype(np.float32)), K, V, sinks=sinks, bf16_probs=True,
                        bf16_kv=cfg.kv_bits == 16)).reshape(-1)
    h = rbf(h + rbf(_dq(L.o, sd) @ att.astype(np.float64))).astype(np.float64)
    xn2 = rmsnorm_f(h, L.post_norm, cfg.rms_eps)
    if kind & 1:  # REC_LAYER_DENSE
        return rbf(h + mlp(L.gate, L.up, L.down, sd, xn2).astype(np.float64)).astype(np.float64)
    logits = rbf(_bfv(L.router).reshape(cfg.n_experts, -1) @ xn2).astype(np.float64)
    bias = None if L.expert_bias is None else np.asarray(L.expert_bias, np.float64)
    ids, wts = route(logits, cfg.top_k, cfg.router_mode, bias)
    I, H = cfg.moe_inter, cfg.hidden
    downs = []
    for e in ids:
        g = rbf(_dq(L.gate, sd, slice(int(e) * I, (int(e) + 1) * I)) @ xn2)
        u = rbf(_dq(L.up, sd, slice(int(e) * I, (int(e) + 1) * I)) @ xn2)
        act = silu_mul(g, u).astype(np.float64)
        downs.append(rbf(_dq(L.down, sd, slice(int(e) * H, (int(e) + 1) * H)) @ act))
    mix = expert_mix(np.stack(downs).astype(np.float32), np.asarray(wts, np.float32))
    if getattr(cfg, "shared_inter", 0):
        mix = rbf(mix + mlp(L.shared_gate, L.shared_up, L.shared_down, sd, xn2))
    return rbf(h + mix.astype(np.float64)).astype(np.float64)


def model_step(m, kvs: list, token: int, pos: int):
    """Embedding -> every layer -> final norm -> lm_head (model.py:318-327).
    Returns (logits float64 [V], trace float64 [L + 1, H])."""
    import torch

    cfg = m.cfg
    sd = 0 if cfg.scale_dtype == torch.float16 else 1
    eb = getattr(cfg, "embed_bits", 4)
    E = m.embed
    h = rbf(dequantize(np.asarray(E.w[token:token + 1], np.uint32), np.asarray(E.s[token:token + 1], np.uint16),
                       np.asarray(E.b[token:token + 1], np.uint16), eb, sd)[0].astype(np.float64)).astype(np.float64)
    trace = [h]
    for L, kv in zip(m.layers, kvs):
        h = layer_step(cfg, L, kv, h, pos, sd)
        trace.append(h)
    xf = rmsnorm_f(h, m.final_norm, cfg.rms_eps)
    logits = rbf(_dq(m.lm_head, sd) @ xf).astype(np.float64)
    return logits, np.stack(trace)
