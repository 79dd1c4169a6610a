"""CPU checks of the oracle's primitives: the canonical restatement against
the order-free semantic restatement, and the reference's own kernel tests
restated as known-answer cases."""
import numpy as np
import pytest

import oracle
from oracle import semantic


def test_exp_accuracy_and_edges():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.uniform(-103, 88, 200000), rng.uniform(-2, 2, 100000),
                        np.array([0.0, -0.0, 1.0, -1.0, 88.7, -87.3, -100.0])]).astype(np.float32)
    y = oracle.exp(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    normal = ref > np.finfo(np.float32).tiny
    ulp = np.spacing(ref[normal].astype(np.float32)).astype(np.float64)
    err = np.abs(y[normal] - ref[normal]) / ulp
    assert err.max() <= 2.0, err.max()
    assert oracle.exp(np.array([0.0], np.float32))[0] == 1.0
    e = oracle.exp(np.array([-np.inf, np.inf, -200.0, 200.0], np.float32))
    assert e[0] == 0.0 and np.isinf(e[1]) and e[2] == 0.0 and np.isinf(e[3])
    assert np.isnan(oracle.exp(np.array([np.nan], np.float32))[0])


def test_attention_exp_accuracy_and_edges():
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.uniform(-86.9, 0.0, 200000), rng.uniform(-1, 0, 100000),
                        np.array([0.0, -0.0, -1e-30, -0.5, -86.99])]).astype(np.float32)
    y = oracle.aexp(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    ulp = np.spacing(ref.astype(np.float32)).astype(np.float64)
    err = np.abs(y - ref) / ulp
    assert err.max() <= 2.0, err.max()
    assert oracle.aexp(np.array([0.0], np.float32))[0] == 1.0
    z = oracle.aexp(np.array([-87.0, -100.0, -np.inf], np.float32))
    assert (z == 0.0).all()


@pytest.mark.parametrize("T,bits,sinks", [(1, 4, False), (37, 8, True), (300, 4, True), (2049, 8, False),
                                          (20000, 4, True)])
def test_attention_canonical_vs_semantic(T, bits, sinks):
    """The canonical fixed-point attention on a quantized cache against the
    exact softmax of the bf16 scores (float64): per head, its rel-L2 error
    stays within 2x the larger of the reference semantics' own error (bf16
    probabilities) and the bf16 rounding of the exact output.  (Rounding the
    scores to bf16 makes them sensitive to the fp32 summation order: any two
    implementations differ in ~0.5% of the rounded scores at long contexts.)"""
    hq, hkv = 16, 2
    rng = np.random.default_rng(T + bits)
    cap = (T + 255) // 256 * 256
    kv, deq = {}, {}
    for n in ("k", "v"):
        x = oracle.bf16_to_f32(oracle.f32_to_bf16(rng.standard_normal((hkv, T, 128), dtype=np.float32)))
        c, s, b = oracle.quantize(x, bits, 1)
        kv[f"{n}_codes"] = np.zeros((hkv, cap, c.shape[-1]), np.uint32)
        kv[f"{n}_scales"] = np.zeros((hkv, cap, 2), np.uint16)
        kv[f"{n}_biases"] = np.zeros((hkv, cap, 2), np.uint16)
        kv[f"{n}_codes"][:, :T], kv[f"{n}_scales"][:, :T], kv[f"{n}_biases"][:, :T] = c, s, b
        deq[n] = oracle.dequantize(c, s, b, bits, 1).reshape(hkv, T, 128)
    q = oracle.f32_to_bf16(3.0 * rng.standard_normal(hq * 128, dtype=np.float32))
    sk = oracle.f32_to_bf16(rng.standard_normal(hq, dtype=np.float32)) if sinks else None
    n_super = -(-((T + 255) // 256) // 64)
    got = oracle.bf16_to_f32(oracle.attention_final(
        oracle.attention_supers(q, kv, hkv, cap, bits, T, n_super), sk)).reshape(hq, 128)
    sem = semantic.attention(q.reshape(hq, 128), deq["k"], deq["v"], sk)
    exact = semantic.attention(q.reshape(hq, 128), deq["k"], deq["v"], sk, bf16_probs=False)
    for h in range(hq):
        bound = 2.0 * max(semantic.rel_l2(sem[h], exact[h]), semantic.rel_l2(semantic.rbf(exact[h]), exact[h]))
        err = semantic.rel_l2(got[h], exact[h])
        assert err <= bound, (h, err, bound)


def _mlx_affine_numpy(w: np.ndarray, bits: int):
    """Vectorised numpy restatement of mx.quantize(mode='affine') in float32."""
    g = w.reshape(-1, 64).astype(np.float32)
    wmax, wmin = g.max(1), g.min(1)
    n_bins = np.float32((1 << bits) - 1)
    scale = np.maximum((wmax - wmin) / n_bins, np.float32(1e-7)).astype(np.float32)
    side = np.abs(wmin) > np.abs(wmax)
    scale = np.where(side, scale, -scale).astype(np.float32)
    edge = np.where(side, wmin, wmax).astype(np.float32)
    q0 = np.rint(edge / scale).astype(np.float32)
    scale = np.where(q0 != 0, edge / np.where(q0 != 0, q0, 1), scale).astype(np.float32)
    bias = np.where(q0 == 0, np.float32(0), edge).astype(np.float32)
    q = np.clip(np.rint((g - bias[:, None]) / scale[:, None]), 0, n_bins).astype(np.uint32)
    return q, scale, bias


@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_matches_numpy_restatement(bits):
    rng = np.random.default_rng(bits)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    w[0, :64] = 0.0                     # all-zero group
    w[1, :64] = 3.0                     # constant group
    w[2, :64] = np.linspace(-1, 1, 64)  # symmetric
    codes, scales, biases = oracle.quantize(w, bits, sd=1)
    q, s, b = _mlx_affine_numpy(w, bits)
    per = 32 // bits
    unpacked = ((codes.reshape(-1, 64 // per)[..., None] >> (np.arange(per, dtype=np.uint32) * bits))
                & ((1 << bits) - 1)).reshape(-1, 64)
    assert np.array_equal(unpacked, q)
    assert np.array_equal(scales.reshape(-1), oracle.f32_to_bf16(s))
    assert np.array_equal(biases.reshape(-1), oracle.f32_to_bf16(b))


def test_quantize_error_bound():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((256, 2048)) * 0.02).astype(np.float32)
    codes, scales, biases = oracle.quantize(w, 4, sd=0)
    deq = oracle.dequantize(codes, scales, biases, 4, 0)
    s = np.repeat(np.abs(oracle.fp16_to_f32(scales)), 64, axis=-1)
    # The grid is anchored at the group's larger-magnitude edge (so that the
    # edge is exact); the opposite end may clip by up to one step.
    assert np.all(np.abs(deq - w) <= 1.0 * s + 1e-6)
    assert np.mean(np.abs(deq - w) <= 0.5 * s + 1e-6) > 0.99


@pytest.mark.parametrize("k", [768, 2048, 4096])
@pytest.mark.parametrize("sd", [0, 1])
def test_gemv_canonical_vs_semantic(k, sd):
    rng = np.random.default_rng(k + sd)
    n = 512
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    codes, scales, biases = oracle.quantize(w, 4, sd)
    x = oracle.f32_to_bf16(rng.standard_normal(k).astype(np.float32))
    y = oracle.bf16_to_f32(oracle.gemv(codes, scales, biases, x, sd))
    ref = semantic.gemv(codes, scales, biases, x, sd)
    assert semantic.rel_l2(y, ref) < 2e-3
    assert np.max(np.abs(y - ref)) <= 2 ** -7 * np.max(np.abs(ref)) + 1e-6


def test_rmsnorm_canonical_vs_semantic():
    rng = np.random.default_rng(11)
    h = oracle.f32_to_bf16((rng.standard_normal(2048) * 3).astype(np.float32))
    w = oracle.f32_to_bf16((1 + 0.1 * rng.standard_normal(2048)).astype(np.float32))
    a = oracle.bf16_to_f32(oracle.rmsnorm(h, w, 1e-6))
    b = semantic.rmsnorm(h, w, 1e-6)
    assert semantic.rel_l2(a, b) < 2e-3
    assert np.mean(a == b) > 0.99


def _routing_cases():
    """The bias cases of the reference's routing test
    (engine/tests/test_kernel_routing.py:34-46)."""
    p = ((np.arange(256) + 1) / 1024).astype(np.float32)
    partial = (np.arange(256) % 9 / 16).astype(np.float32)
    partial[[7, 31, 64]] = 4
    partial[[2, 17, 93, 201]] = 3
    cases = [("unbiased", np.zeros(256, np.float32)), ("all_ties_with_bias", (1 - p).astype(np.float32)),
             ("partial_ties_with_bias", (partial - p).astype(np.float32))]
    for expert in range(256):
        bias = ((np.arange(256) % 13) / 128).astype(np.float32)
        bias[expert] = 2
        cases.append((f"boost_{expert}", bias))
    return p, cases


def test_routing_known_answers():
    p, cases = _routing_cases()
    for name, bias in cases:
        choice = (p + bias).astype(np.float32)
        ids, w = oracle.select_topk(p, choice, 6)
        # lowest index among equal choices, in descending order of choice
        expect = np.lexsort((np.arange(256), -choice.astype(np.float64)))[:6]
        assert np.array_equal(ids, expect), name
        total = np.float32(0)
        for i in range(6):
            total = np.float32(p[ids[i]] + total)
        ref = p[ids] / np.float32(total + np.float32(1e-20))
        assert np.max(np.abs(w - ref)) < 1e-7, name
        if name.startswith("boost_"):
            assert ids[0] == int(name.split("_")[1])


@pytest.mark.parametrize("seed", [19, 31, 47])
def test_bf16_expert_mix_order(seed):
    """Restates test_kernel_routing.check_reduction: the expert mix rounds to
    bf16 after every addition and differs from an fp32-accumulated mix."""
    rng = np.random.default_rng(seed)
    down = oracle.f32_to_bf16(rng.standard_normal((7, 2048)).astype(np.float32))
    residual = oracle.f32_to_bf16(rng.standard_normal(2048).astype(np.float32))
    probs = rng.uniform(size=256).astype(np.float32)
    bias = rng.uniform(-0.5, 0.5, 256).astype(np.float32)
    ids, w = oracle.select_topk(probs, (probs + bias).astype(np.float32), 6)
    mix = oracle.mix(down[:6], w)
    d = oracle.bf16_to_f32(down)
    expected = semantic.expert_mix(d[:6], w)
    assert np.array_equal(oracle.bf16_to_f32(mix), expected)
    with_shared = semantic.rbf(semantic.rbf(expected + d[6]) + oracle.bf16_to_f32(residual))
    wb = semantic.rbf(w.astype(np.float32))
    fp32_mix = semantic.rbf(semantic.rbf(semantic.rbf(d[:6] * wb[:, None]).sum(0) + d[6])
                            + oracle.bf16_to_f32(residual))
    assert not np.array_equal(with_shared, fp32_mix)


def test_swiglu_exhaustive_against_semantic():
    """All 65,536 bf16 gate patterns x the reference guard's 16 up patterns
    (kernels/activation_optimization.py:62-80): the canonical SiLU product,
    built on the oracle's own exp, equals the reference formula evaluated
    with a correctly rounded exp for every finite gate — the same bar the
    reference's startup guard sets for its fast exp."""
    up_bits = [0, 0x8000, 1, 0x8001, 0x007F, 0x807F, 0x0080, 0x8080, 0x3F80, 0xBF80, 0x7F7F, 0xFF7F,
               0x7F80, 0xFF80, 0x7FC1, 0xFF81]
    gates = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    g = oracle.bf16_to_f32(gates)
    finite_g = np.isfinite(g)
    mismatches = 0
    for ub in up_bits:
        u = oracle.bf16_to_f32(np.array([ub], np.uint16))[0]
        ours = np.array([oracle.swiglu(int(x), ub) for x in gates], np.uint16)
        with np.errstate(all="ignore"):
            ref = oracle.f32_to_bf16(semantic.silu_mul(g, np.full(65536, u, np.float32)))
        ok = (ours == ref) | (np.isnan(oracle.bf16_to_f32(ours)) & np.isnan(oracle.bf16_to_f32(ref)))
        mismatches += int(np.sum(~ok & finite_g))
    assert mismatches == 0, mismatches
