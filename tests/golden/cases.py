"""Seeded golden cases: inputs regenerated from numpy seeds, outputs frozen in
the .npz fixtures beside this file (written by make_golden.py from the C
oracle).

The CPU tests check that the oracle still produces the frozen outputs; the
GPU tests check that the CUDA path produces them through the C ABI.  Inputs
are not stored: numpy's PCG64 streams are stable, and every fixture records
a SHA-256 of its regenerated inputs so that a generator change is reported
as such rather than as a numerical mismatch.
"""
from __future__ import annotations

import hashlib
from dataclasses import replace
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

import oracle
from rec_b200 import abi
from rec_b200.model import ModelConfig

HERE = Path(__file__).resolve().parent

# Small models with the kernels' real shapes (hidden 2048, head_dim 128,
# GQA 8:1) and few layers / experts / vocabulary rows.
GOLDEN_A = ModelConfig(name="golden_a", n_layers=2, n_q_heads=16, n_kv_heads=2, n_experts=8, top_k=2,
                       moe_inter=256, vocab=2048, kv_bits=8)
GOLDEN_B = replace(GOLDEN_A, name="golden_b", n_q_heads=32, n_kv_heads=4, n_experts=16, top_k=6, moe_inter=512,
                   kv_bits=4, scale_dtype=torch.bfloat16, router_mode=abi.REC_ROUTER_SIGMOID,
                   flags=abi.REC_FLAG_SINKS | abi.REC_FLAG_QK_NORM)
# the reference Flint model's layer options (model.py:14-37,155-163,216-271):
# a dense SwiGLU MLP in layer 0 (one 6,144-row matrix triple), a shared expert
# in the MoE layers, a NoPE layer between two sliding-window layers whose
# 40-position window starts inside block 1 (block 0 skipped, a tile cut)
GOLDEN_FLINT = replace(GOLDEN_B, name="golden_flint", n_layers=3, shared_inter=256, dense_layers=(0,),
                       dense_inter=6144, no_rope_layers=(1,), sliding_layers=(0, 2), sliding_window=40,
                       embed_bits=8)
# a bf16 cache (the reference megakernel's kv_format "bf16")
GOLDEN_BF16 = replace(GOLDEN_A, name="golden_bf16", kv_bits=16)
# the reference's mixed cache (K 8-bit, V 4-bit; model.py:35-37,40-82)
GOLDEN_MIXED = replace(GOLDEN_B, name="golden_mixed", kv_bits=8, kv_value_bits=4)
DECODE_CASES = {"decode_a": (GOLDEN_A, 101), "decode_b": (GOLDEN_B, 202), "decode_flint": (GOLDEN_FLINT, 303),
                "decode_bf16": (GOLDEN_BF16, 404), "decode_mixed": (GOLDEN_MIXED, 505)}

CAPACITY = 512
CONTEXT = 300      # cached positions before decoding (a ragged second block)
STEPS = 6
START_TOKEN = 5


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _sd(cfg) -> int:
    return 0 if cfg.scale_dtype == torch.float16 else 1


def _q(rng, n, k, sd, std=0.02):
    w = oracle.bf16_to_f32(oracle.f32_to_bf16((std * rng.standard_normal((n, k), dtype=np.float32))))
    c, s, b = oracle.quantize(w, 4, sd)
    return SimpleNamespace(w=c, s=s, b=b)


def _bf(rng, shape, std, mean=0.0):
    return oracle.f32_to_bf16((mean + std * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32))


def host_model(cfg: ModelConfig, seed: int) -> SimpleNamespace:
    """Weights of `cfg` in host memory: linear weights N(0, 0.02) rounded to
    bf16 then int4 g64; router bf16 N(0, 0.02); embedding rows N(0, 1).  A
    dense-MLP layer draws its matrix triple (dense_inter rows) instead of the
    router and experts; a shared expert is drawn after a MoE layer's experts."""
    rng = np.random.default_rng(seed)
    h, d, sd = cfg.hidden, cfg.head_dim, _sd(cfg)
    layers = []
    for i in range(cfg.n_layers):
        kind = cfg.layer_kind(i)
        common = dict(
            input_norm=_bf(rng, h, 0.1, 1.0), post_norm=_bf(rng, h, 0.1, 1.0),
            q=_q(rng, cfg.n_q_heads * d, h, sd), k=_q(rng, cfg.n_kv_heads * d, h, sd),
            v=_q(rng, cfg.n_kv_heads * d, h, sd), o=_q(rng, h, cfg.n_q_heads * d, sd))
        if kind & abi.REC_LAYER_DENSE:
            I = cfg.dense_inter
            L = SimpleNamespace(**common, router=None, gate=_q(rng, I, h, sd), up=_q(rng, I, h, sd),
                                down=_q(rng, h, I, sd), expert_bias=None, sinks=None, q_norm=None, k_norm=None,
                                kind=kind, shared_gate=None, shared_up=None, shared_down=None)
        else:
            L = SimpleNamespace(
                **common,
                router=_bf(rng, (cfg.n_experts, h), 0.02),
                gate=_q(rng, cfg.n_experts * cfg.moe_inter, h, sd),
                up=_q(rng, cfg.n_experts * cfg.moe_inter, h, sd),
                down=_q(rng, cfg.n_experts * h, cfg.moe_inter, sd),
                expert_bias=None, sinks=None, q_norm=None, k_norm=None, kind=kind, shared_gate=None,
                shared_up=None, shared_down=None)
            if cfg.shared_inter:
                Is = cfg.shared_inter
                L.shared_gate, L.shared_up, L.shared_down = _q(rng, Is, h, sd), _q(rng, Is, h, sd), _q(rng, h, Is, sd)
        if cfg.router_mode == abi.REC_ROUTER_SIGMOID and not kind & abi.REC_LAYER_DENSE:
            L.expert_bias = (0.05 * rng.standard_normal(cfg.n_experts, dtype=np.float32)).astype(np.float32)
        if cfg.flags & abi.REC_FLAG_SINKS:
            L.sinks = _bf(rng, cfg.n_q_heads, 1.0)
        if cfg.flags & abi.REC_FLAG_QK_NORM:
            L.q_norm = _bf(rng, d, 0.1, 1.0)
            L.k_norm = _bf(rng, d, 0.1, 1.0)
        layers.append(L)
    eb = cfg.embed_bits
    w_emb = oracle.bf16_to_f32(oracle.f32_to_bf16(rng.standard_normal((cfg.vocab, h), dtype=np.float32)))
    c, s, b = oracle.quantize(w_emb, eb, sd)
    return SimpleNamespace(cfg=cfg, layers=layers, embed=SimpleNamespace(w=c, s=s, b=b),
                           final_norm=_bf(rng, h, 0.1, 1.0), lm_head=_q(rng, cfg.vocab, h, sd))


def model_sha(m) -> str:
    parts = [m.embed.w, m.lm_head.w, m.final_norm]
    for L in m.layers:
        parts += [L.q.w, L.q.s, L.o.w, L.gate.w, L.down.b] + ([] if L.router is None else [L.router]) + [L.input_norm]
        if getattr(L, "shared_gate", None) is not None:
            parts += [L.shared_gate.w, L.shared_down.b]
    return sha(*parts)


def fill_kv(hkv, cfg: ModelConfig, seed: int) -> None:
    """Positions [0, CONTEXT) of every layer: K, V ~ N(0, 1) rounded to bf16,
    quantized (group 64 along head_dim, bf16 scales)."""
    rng = np.random.default_rng(seed)
    for L in hkv.layers:
        for name in ("k", "v"):
            x = oracle.bf16_to_f32(oracle.f32_to_bf16(
                rng.standard_normal((cfg.n_kv_heads, CONTEXT, 128), dtype=np.float32)))
            if cfg.kv_bits == 16:  # bf16 rows as they are
                L[f"{name}_codes"].view(np.uint16)[:, :CONTEXT] = oracle.f32_to_bf16(x)
                continue
            c, s, b = oracle.quantize(x, cfg.kv_bits if name == "k" else cfg.v_bits, 1)
            L[f"{name}_codes"][:, :CONTEXT] = c
            L[f"{name}_scales"][:, :CONTEXT] = s
            L[f"{name}_biases"][:, :CONTEXT] = b


def kv_sha(layers, lo: int, hi: int) -> str:
    return sha(*(L[n][:, lo:hi] for L in layers for n in sorted(L)))


def run_oracle_decode(cfg: ModelConfig, seed: int) -> dict:
    """Greedy decode of STEPS tokens from START_TOKEN at position CONTEXT."""
    from oracle.host import HostModel

    m = host_model(cfg, seed)
    host = HostModel(m)
    hkv = host.new_kv(CAPACITY)
    fill_kv(hkv, cfg, seed + 1)
    token, ids, shas = START_TOKEN, [], []
    trace0 = logits = None
    for i in range(STEPS):
        logits, trace = host.step(hkv, token, CONTEXT + i, want_trace=True)
        if i == 0:
            trace0 = trace.copy()
        shas.append(sha(logits))
        token = oracle.argmax_bf16(logits)
        ids.append(token)
    return {"input_sha": model_sha(m), "ids": np.array(ids, np.int32), "logits_sha": np.array(shas),
            "last_logits": logits.copy(), "trace0_sha": sha(trace0),
            "kv_new_sha": kv_sha(hkv.layers, CONTEXT, CONTEXT + STEPS)}


# ---- GEMV: one seeded matrix per K, with and without the fused RMSNorm
GEMV_CASES = {"gemv_k2048_fp16": (2048, 0, 31), "gemv_k4096_bf16": (4096, 1, 32), "gemv_k768_fp16": (768, 0, 33)}
GEMV_ROWS = 256 + 2 * 37


def gemv_inputs(k: int, sd: int, seed: int):
    rng = np.random.default_rng(seed)
    w = _q(rng, GEMV_ROWS, k, sd)
    x = _bf(rng, k, 1.0)
    nw = _bf(rng, k, 0.1, 1.0)
    return w, x, nw


def run_oracle_gemv(k: int, sd: int, seed: int) -> dict:
    w, x, nw = gemv_inputs(k, sd, seed)
    out = {"input_sha": sha(w.w, w.s, w.b, x, nw), "y": oracle.gemv(w.w, w.s, w.b, x, sd)}
    if k % 256 == 0:
        out["y_norm"] = oracle.gemv(w.w, w.s, w.b, oracle.rmsnorm(x, nw, 1e-6), sd)
    return out


def load(name: str) -> dict:
    with np.load(HERE / f"{name}.npz", allow_pickle=False) as f:
        return {k: f[k] for k in f.files}
