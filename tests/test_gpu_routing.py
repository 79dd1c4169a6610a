"""Expert routing on the GPU at the expert counts the bench uses, against the
oracle, bit for bit.

- The reference's routing known answers (engine/tests/test_kernel_routing.py
  :33-107: 256 experts, top-6, sigmoid + bias; an unbiased case, all choices
  tied, partial ties and one boosted expert per case) run through the
  standalone router (rec_router_moe) and through whole decode steps on every
  schedule, so the persistent kernel's producer-warp routing and k_router
  both see them.  The probabilities are the kernels' own sigmoid of the
  layer's router logits, so the tie patterns are exact in fp32.
- Softmax top-8 over 128 and 64 experts (config 3 and config 1) with ties
  between experts owned by the same lane (e and e + 32, e + 64, e + 96) and
  by neighbouring lanes (2j and 2j + 1)."""
from __future__ import annotations

import ctypes as C
from dataclasses import replace

import numpy as np
import pytest
import torch

import oracle
from oracle.host import HostModel, _np
from rec_b200 import abi
from rec_b200.model import TINY, KVCache, generate_weights
from rec_b200.session import DecodeSession

pytestmark = pytest.mark.gpu

SIG256 = replace(TINY, n_layers=1, n_experts=256, top_k=6, moe_inter=256, router_mode=abi.REC_ROUTER_SIGMOID)
SOFT128 = replace(TINY, n_layers=1, n_experts=128, top_k=8, moe_inter=256)
SOFT64 = replace(TINY, n_layers=1, n_experts=64, top_k=8, moe_inter=256)


def _u16(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _sigmoid(logits: np.ndarray) -> np.ndarray:
    """The kernels' sigmoid: tail = 1 / (1 + exp|g|) with their own exp;
    g < 0 ? tail : 1 - tail, in fp32."""
    g = np.asarray(logits, np.float32)
    tail = (np.float32(1) / (np.float32(1) + oracle.exp(np.abs(g)))).astype(np.float32)
    return np.where(g < 0, tail, (np.float32(1) - tail).astype(np.float32)).astype(np.float32)


def _bias_cases(p: np.ndarray):
    """The reference's bias cases with the layer's own probabilities p
    (test_kernel_routing.py:34-46)."""
    E = p.size
    partial = (np.arange(E) % 9 / 16).astype(np.float32)
    partial[[7, 31, 64]] = 4
    partial[[2, 17, 93, 201]] = 3
    cases = [("unbiased", np.zeros(E, np.float32)), ("all_ties_with_bias", (np.float32(1) - p).astype(np.float32)),
             ("partial_ties_with_bias", (partial - p).astype(np.float32))]
    for expert in range(E):
        bias = ((np.arange(E) % 13) / 128).astype(np.float32)
        bias[expert] = 2
        cases.append((f"boost_{expert}", bias))
    return cases


def _tie(router: torch.Tensor, kind: str) -> None:
    E = router.shape[0]
    if kind == "same_lane":  # experts e, e + 32, e + 64, ... share a lane
        for j in range(32, E, 32):
            router[j:j + 32] = router[0:32]
    elif kind == "adjacent":  # experts 2j and 2j + 1 on neighbouring lanes
        router[1::2] = router[0::2]
    torch.cuda.synchronize()


def _router_moe(sess, layer, h_dev, k):
    from rec_b200._lib import check, lib

    ids = torch.zeros(k, dtype=torch.int32, device="cuda")
    wts = torch.zeros(k, dtype=torch.float32, device="cuda")
    check(lib().rec_router_moe(sess.ctx, layer, C.c_void_p(h_dev.data_ptr()), C.c_void_p(ids.data_ptr()),
                               C.c_void_p(wts.data_ptr()), C.c_void_p(torch.cuda.current_stream().cuda_stream)),
          "rec_router_moe")
    torch.cuda.synchronize()
    return ids.cpu().numpy(), wts.cpu().numpy()


def _oracle_moe(cfg, L, h, bias):
    sd = 1 if cfg.scale_dtype == torch.bfloat16 else 0
    xn = oracle.rmsnorm(h, _np(L.post_norm), cfg.rms_eps)
    logits = oracle.router_logits(_np(L.router), xn)
    ids, wts = oracle.route(logits, cfg.top_k, cfg.router_mode, bias)
    I, H = cfg.moe_inter, cfg.hidden
    gw, gs, gb = _np(L.gate.w), _np(L.gate.s), _np(L.gate.b)
    uw, us, ub = _np(L.up.w), _np(L.up.s), _np(L.up.b)
    dw, ds, db = _np(L.down.w), _np(L.down.s), _np(L.down.b)
    downs = []
    for e in ids:
        rows = slice(int(e) * I, (int(e) + 1) * I)
        g = oracle.gemv(gw[rows], gs[rows], gb[rows], xn, sd)
        u = oracle.gemv(uw[rows], us[rows], ub[rows], xn, sd)
        act = np.array([oracle.swiglu(int(a), int(b)) for a, b in zip(g, u)], np.uint16)
        drows = slice(int(e) * H, (int(e) + 1) * H)
        downs.append(oracle.gemv(dw[drows], ds[drows], db[drows], act, sd))
    mix = oracle.mix(np.stack(downs), wts)
    return ids, wts, oracle.f32_to_bf16(oracle.bf16_to_f32(h) + oracle.bf16_to_f32(mix)), logits


def test_router_moe_reference_bias_cases(cuda):
    """All 259 bias cases through rec_router_moe at 256 experts, top-6."""
    cfg = SIG256
    w = generate_weights(cfg, seed=41, device="cuda")
    kv = KVCache.allocate(cfg, 256)
    sess = DecodeSession(w, kv)
    L = w.layers[0]
    rng = np.random.default_rng(43)
    h = oracle.f32_to_bf16(rng.standard_normal(cfg.hidden, dtype=np.float32))
    xn = oracle.rmsnorm(h, _np(L.post_norm), cfg.rms_eps)
    p = _sigmoid(oracle.router_logits(_np(L.router), xn))
    bad = []
    for name, bias in _bias_cases(p):
        L.expert_bias.copy_(torch.from_numpy(bias))
        h_dev = torch.from_numpy(h.view(np.int16)).cuda()
        ids, wts = _router_moe(sess, 0, h_dev, cfg.top_k)
        want_ids, want_wts, want_h, _ = _oracle_moe(cfg, L, h, bias)
        ok = (np.array_equal(ids, want_ids) and np.array_equal(wts.view(np.uint32), want_wts.view(np.uint32))
              and np.array_equal(_u16(h_dev), want_h))
        if name.startswith("boost_"):
            ok = ok and ids[0] == int(name.split("_")[1])
        if not ok:
            bad.append((name, ids.tolist(), want_ids.tolist()))
    assert not bad, bad[:5]


@pytest.mark.parametrize("schedule", ["mega", "graph", "split"])
def test_decode_reference_bias_cases(cuda, schedule, monkeypatch):
    """The 259 bias cases through full decode steps of a one-layer model with
    256 experts (top-6, sigmoid + bias).  The O projection is zero, so the
    router's input is the RMSNorm of the embedding (the trace's first row)
    and the probabilities are known before the step."""
    monkeypatch.setenv("REC_SCHEDULE", schedule)
    cfg = SIG256
    w = generate_weights(cfg, seed=47, device="cuda")
    L = w.layers[0]
    for t in (L.o.w, L.o.s, L.o.b):
        t.zero_()
    kv = KVCache.allocate(cfg, 256)
    sess = DecodeSession(w, kv)
    host = HostModel(w)
    hkv = host.new_kv(256)
    token = 123
    _, trace = sess.step(token, 0, want_trace=True)
    sess.check_status()
    h0 = _u16(trace)[0]
    xn = oracle.rmsnorm(h0, _np(L.post_norm), cfg.rms_eps)
    p = _sigmoid(oracle.router_logits(_np(L.router), xn))
    bad = []
    hb = host.layers[0].expert_bias  # the host model's pointer to its bias copy
    host_bias = np.ctypeslib.as_array(C.cast(hb, C.POINTER(C.c_float)), shape=(cfg.n_experts,))
    for name, bias in _bias_cases(p):
        L.expert_bias.copy_(torch.from_numpy(bias))
        host_bias[:] = bias
        logits, trace = sess.step(token, 0, want_trace=True)
        sess.check_status()
        ref_logits, ref_trace = host.step(hkv, token, 0)
        if not (np.array_equal(_u16(trace), ref_trace) and np.array_equal(_u16(logits), ref_logits)):
            bad.append(name)
    assert not bad, bad[:8]


@pytest.mark.parametrize("ties", ["none", "same_lane", "adjacent"])
@pytest.mark.parametrize("cfg", [SOFT128, SOFT64], ids=["e128", "e64"])
def test_router_moe_softmax_ties(cuda, cfg, ties):
    w = generate_weights(cfg, seed=53, device="cuda")
    _tie(w.layers[0].router, ties)
    kv = KVCache.allocate(cfg, 256)
    sess = DecodeSession(w, kv)
    rng = np.random.default_rng(59)
    for trial in range(4):
        h = oracle.f32_to_bf16(rng.standard_normal(cfg.hidden, dtype=np.float32))
        h_dev = torch.from_numpy(h.view(np.int16)).cuda()
        ids, wts = _router_moe(sess, 0, h_dev, cfg.top_k)
        want_ids, want_wts, want_h, _ = _oracle_moe(cfg, w.layers[0], h, None)
        assert np.array_equal(ids, want_ids), (trial, ids, want_ids)
        assert np.array_equal(wts.view(np.uint32), want_wts.view(np.uint32)), trial
        assert np.array_equal(_u16(h_dev), want_h), trial


@pytest.mark.parametrize("schedule", ["mega", "graph", "split"])
@pytest.mark.parametrize("ties", ["none", "same_lane", "adjacent"])
@pytest.mark.parametrize("cfg", [SOFT128, SOFT64], ids=["e128", "e64"])
def test_decode_softmax_ties(cuda, cfg, ties, schedule, monkeypatch):
    """Decode steps with 128 / 64 experts, softmax top-8, with tied router
    rows, on every schedule (the persistent kernel's producer routing gives
    each lane 4 / 2 experts)."""
    monkeypatch.setenv("REC_SCHEDULE", schedule)
    w = generate_weights(cfg, seed=61, device="cuda")
    _tie(w.layers[0].router, ties)
    kv = KVCache.allocate(cfg, 256)
    sess = DecodeSession(w, kv)
    host = HostModel(w)
    hkv = host.new_kv(256)
    rng = np.random.default_rng(67)
    for pos in range(6):
        tok = int(rng.integers(0, cfg.vocab))
        logits, trace = sess.step(tok, pos, want_trace=True)
        sess.check_status()
        ref_logits, ref_trace = host.step(hkv, tok, pos)
        assert np.array_equal(_u16(trace), ref_trace), (pos, ties, schedule)
        assert np.array_equal(_u16(logits), ref_logits), (pos, ties, schedule)
