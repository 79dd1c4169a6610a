"""The canonical fixed-point order (oracle/rec_oracle.c; the GPU equals it
bit for bit) against an fp64 restatement of the reference's formulas with its
bf16 rounding points (oracle/semantic.py), at operation and layer scale.

Per operation, on the same inputs, within the north-star rel-L2 2e-3: the
RMSNorm, the q / k / v, O, gate and down GEMVs, decode attention over a
1,024-token 8-bit cache, the router logits and the expert selection, the
rank-order bf16 mix.  Three input families: Gaussian; heavy-tailed (a
residual with 4 channels at 50-100x the rest: the GEMV puts each input vector
on one 16-bit fixed point, so small elements lose bits); and caches with a
few 12x K rows per head (near-one-hot softmax rows: the P.V fixed point is
set by the largest weight of a tile).

The attention semantics are the reference decode kernel's: an fp32 online
softmax with P.V accumulated in fp32 (megakernel.py:619-693).  The native MLX
forward (model.py:108-139) rounds P to bf16 before P.V; that rounding alone
moves the output ~2.6e-3 (measured here) and is not part of the decode path.

Per layer (teacher-forced: each layer gets the canonical input), the residual
after the layer within 3e-3: the layer's update differs by ~1e-3 of the
update (the per-operation errors above), but both sides round h + update to
bf16, and an update that differs in its last bits flips an ulp of h on some
elements -- an ulp of h is several percent of the update.  Any two
implementations that are not bit-identical differ this way."""
from dataclasses import replace
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle
from oracle import semantic as S
from rec_b200 import abi
from rec_b200.model import CONFIG1_LAYER, TINY
from tests.golden.cases import host_model

TOL = 2e-3
LAYER_TOL = 3e-3
CTX = 1024
CAP = 1280


def _kv(cfg, seed, spikes=0):
    """Host cache layers [Hkv, CAP, ...] with positions [0, CTX) of K, V ~
    N(0, 1) (bf16) quantized; with spikes, that many tokens per head get K
    rows 12x larger (their scores dominate: near-one-hot softmax rows)."""
    from oracle.host import HostKV

    rng = np.random.default_rng(seed)
    hkv = HostKV(cfg, CAP)
    for L in hkv.layers:
        for name in ("k", "v"):
            x = rng.standard_normal((cfg.n_kv_heads, CTX, 128), dtype=np.float32)
            if name == "k" and spikes:
                idx = rng.choice(CTX, spikes, replace=False)
                x[:, idx] *= 12.0
            if cfg.kv_bits == 16:  # a bf16 cache holds the rows as they are
                L[f"{name}_codes"].view(np.uint16)[:, :CTX] = oracle.f32_to_bf16(x)
                continue
            x = oracle.bf16_to_f32(oracle.f32_to_bf16(x))
            c, s, b = oracle.quantize(x, cfg.kv_bits if name == "k" else cfg.v_bits, 1)
            L[f"{name}_codes"][:, :CTX] = c
            L[f"{name}_scales"][:, :CTX] = s
            L[f"{name}_biases"][:, :CTX] = b
    return hkv


def _residual(rng, outliers: bool):
    x = rng.standard_normal(2048).astype(np.float32)
    if outliers:
        ch = rng.choice(2048, 4, replace=False)
        x[ch] *= rng.uniform(50, 100, 4).astype(np.float32)
    return oracle.f32_to_bf16(x)


@pytest.mark.parametrize("case", ["gaussian", "outlier_channels", "near_one_hot"])
def test_operations_against_semantics(case):
    cfg = replace(TINY, n_layers=1)
    m = host_model(cfg, 81)
    L, sd = m.layers[0], 0
    kvl = _kv(cfg, 82, 3 if case == "near_one_hot" else 0).layers[0]
    rng = np.random.default_rng(5)
    h = _residual(rng, case == "outlier_channels")
    bfv = lambda u: oracle.bf16_to_f32(u).astype(np.float64)  # noqa: E731
    errs = {}
    xn = oracle.rmsnorm(h, L.input_norm, cfg.rms_eps)
    errs["rmsnorm"] = S.rel_l2(bfv(xn), S.rmsnorm_f(bfv(h), L.input_norm, cfg.rms_eps))
    for name, qt in (("q", L.q), ("k", L.k), ("v", L.v)):
        y = oracle.gemv(qt.w, qt.s, qt.b, xn, sd)
        errs[f"{name} gemv"] = S.rel_l2(bfv(y), S.rbf(S._dq(qt, sd) @ bfv(xn)))
    q = oracle.gemv(L.q.w, L.q.s, L.q.b, xn, sd)
    sup = oracle.attention_supers(q, kvl, cfg.n_kv_heads, CAP, cfg.kv_bits, CTX, 1)
    att = oracle.attention_final(sup, None)
    K = oracle.dequantize(kvl["k_codes"][:, :CTX], kvl["k_scales"][:, :CTX], kvl["k_biases"][:, :CTX], cfg.kv_bits, 1)
    V = oracle.dequantize(kvl["v_codes"][:, :CTX], kvl["v_scales"][:, :CTX], kvl["v_biases"][:, :CTX], cfg.kv_bits, 1)
    want = S.rbf(S.attention(q.reshape(32, 128), K, V, None, bf16_probs=False)).reshape(-1)
    errs["attention"] = S.rel_l2(bfv(att), want)
    o = oracle.gemv(L.o.w, L.o.s, L.o.b, att, sd)
    errs["o gemv"] = S.rel_l2(bfv(o), S.rbf(S._dq(L.o, sd) @ bfv(att)))
    xn2 = oracle.rmsnorm(h, L.post_norm, cfg.rms_eps)
    logits = oracle.router_logits(L.router, xn2)
    errs["router logits"] = S.rel_l2(logits, S.rbf(S._bfv(L.router).reshape(cfg.n_experts, -1) @ bfv(xn2)))
    ids, wts = oracle.route(logits, cfg.top_k, 0, None)
    ids_s, wts_s = S.route(logits, cfg.top_k, 0, None)
    assert np.array_equal(ids, ids_s)
    errs["route weights"] = S.rel_l2(wts, wts_s)
    I, downs = cfg.moe_inter, []
    for e in ids:
        rows, drows = slice(int(e) * I, (int(e) + 1) * I), slice(int(e) * 2048, (int(e) + 1) * 2048)
        g = oracle.gemv(L.gate.w[rows], L.gate.s[rows], L.gate.b[rows], xn2, sd)
        u = oracle.gemv(L.up.w[rows], L.up.s[rows], L.up.b[rows], xn2, sd)
        errs["gate gemv"] = max(errs.get("gate gemv", 0.0), S.rel_l2(bfv(g), S.rbf(S._dq(L.gate, sd, rows) @ bfv(xn2))))
        act = np.array([oracle.swiglu(int(a), int(b)) for a, b in zip(g, u)], np.uint16)
        assert np.array_equal(bfv(act), S.silu_mul(bfv(g), bfv(u)).astype(np.float64))
        d = oracle.gemv(L.down.w[drows], L.down.s[drows], L.down.b[drows], act, sd)
        errs["down gemv"] = max(errs.get("down gemv", 0.0), S.rel_l2(bfv(d), S.rbf(S._dq(L.down, sd, drows) @ bfv(act))))
        downs.append(d)
    mix = oracle.mix(np.stack(downs), wts)
    errs["mix"] = S.rel_l2(bfv(mix), S.expert_mix(oracle.bf16_to_f32(np.stack(downs)), wts))
    print(case, {k: f"{v:.2e}" for k, v in errs.items()})
    bad = {k: v for k, v in errs.items() if not v < TOL}
    assert not bad, bad


def _teacher_forced(cfg, seed, spikes):
    """Residual rel-L2 of every layer, each started from the canonical input,
    over one decode step at position CTX (both sides quantize their own new
    K / V row into their own copy of the same cache)."""
    from oracle.host import HostModel

    m = host_model(cfg, seed)
    hkv = _kv(cfg, seed + 1, spikes)
    base = [{n: a.copy() for n, a in L.items()} for L in hkv.layers]
    _, tr = HostModel(m).step(hkv, 7, CTX)
    orig = S.attention
    S.attention = lambda q, k, v, sinks=None, bf16_probs=True, **kw: orig(q, k, v, sinks, False, **kw)
    try:
        out = []
        for li in range(cfg.n_layers):
            kv = S.SemanticKV(base[li], cfg.kv_bits, cfg.v_bits)
            sd = 0 if cfg.scale_dtype == torch.float16 else 1
            h_out = S.layer_step(cfg, m.layers[li], kv, oracle.bf16_to_f32(tr[li]).astype(np.float64), CTX, sd)
            out.append(S.rel_l2(oracle.bf16_to_f32(tr[li + 1]), h_out))
        return out
    finally:
        S.attention = orig


# the Flint layer options at the kernels' shapes: a dense 6,144-row MLP, a
# shared expert, a NoPE layer, sliding windows of 300 positions over the
# 1,024-token cache (sigmoid + bias router, sinks, q/k norms, bf16 scales)
FLINT4 = replace(TINY, name="flint4", n_layers=4, top_k=6, moe_inter=512, scale_dtype=torch.bfloat16,
                 router_mode=abi.REC_ROUTER_SIGMOID, flags=abi.REC_FLAG_SINKS | abi.REC_FLAG_QK_NORM,
                 shared_inter=1024, dense_layers=(0,), dense_inter=6144, no_rope_layers=(1, 3),
                 sliding_layers=(0, 2), sliding_window=300)


@pytest.mark.parametrize("name", ["config1_layer", "four_layers", "four_layers_near_one_hot", "flint_options",
                                  "flint_bf16_kv", "mixed_kv"])
def test_layers_against_semantics(name):
    cfg, seed, spikes = {"config1_layer": (CONFIG1_LAYER, 71, 0),
                         "four_layers": (replace(TINY, n_layers=4), 81, 0),
                         "four_layers_near_one_hot": (replace(TINY, n_layers=4), 81, 3),
                         "flint_options": (FLINT4, 91, 0),
                         "flint_bf16_kv": (replace(FLINT4, kv_bits=16), 93, 0),
                         "mixed_kv": (replace(FLINT4, kv_bits=8, kv_value_bits=4), 95, 0)}[name]
    errs = _teacher_forced(cfg, seed, spikes)
    print(name, [f"{e:.2e}" for e in errs])
    assert max(errs) < LAYER_TOL, errs
