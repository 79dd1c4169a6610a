"""End-to-end decode parity through the C ABI: logits, the per-layer residual
trace, the quantized KV cache and greedy token ids must equal the oracle's bit
for bit."""
from dataclasses import replace

import numpy as np
import pytest
import torch

import oracle
from oracle.host import HostKV, HostModel, _np
from rec_b200 import abi
from rec_b200.model import TINY, KVCache, generate_weights
from rec_b200.session import DecodeSession

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["mega", "graph", "split"])
def schedule(request, monkeypatch):
    """The persistent kernel (default) and the per-kernel CUDA graph."""
    monkeypatch.setenv("REC_SCHEDULE", request.param)
    return request.param

VARIANTS = {
    "tiny_kv8_fp16": TINY,
    "tiny_kv4_bf16_sigmoid": replace(TINY, kv_bits=4, scale_dtype=torch.bfloat16,
                                     router_mode=abi.REC_ROUTER_SIGMOID, top_k=6, moe_inter=512),
    "tiny_sinks_qknorm": replace(TINY, flags=abi.REC_FLAG_SINKS | abi.REC_FLAG_QK_NORM, n_experts=32, top_k=8,
                                 moe_inter=256),
}


def _u16(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _setup(cfg, capacity, seed=0):
    w = generate_weights(cfg, seed=seed, device="cuda")
    kv = KVCache.allocate(cfg, capacity)
    sess = DecodeSession(w, kv)
    host = HostModel(w)
    hkv = host.new_kv(capacity)
    return w, kv, sess, host, hkv


def _compare_kv(kv, hkv, upto):
    for li, (d, h) in enumerate(zip(kv.layers, hkv.layers)):
        for name in d:
            got = _np(d[name])[:, :upto]
            assert np.array_equal(got, h[name][:, :upto]), (li, name)


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_decode_steps_bitexact(cuda, schedule, variant):
    cfg = VARIANTS[variant]
    _, kv, sess, host, hkv = _setup(cfg, 512, seed=3)
    rng = np.random.default_rng(5)
    for pos in range(12):
        tok = int(rng.integers(0, cfg.vocab))
        logits, trace = sess.step(tok, pos, want_trace=True)
        sess.check_status()
        ref_logits, ref_trace = host.step(hkv, tok, pos)
        got_trace = _u16(trace)
        for li in range(cfg.n_layers + 1):
            assert np.array_equal(got_trace[li], ref_trace[li]), (pos, li)
        assert np.array_equal(_u16(logits), ref_logits), pos
    _compare_kv(kv, hkv, 12)


def test_greedy_packet_bitexact(cuda, schedule):
    cfg = TINY
    _, kv, sess, host, hkv = _setup(cfg, 512, seed=9)
    tok, pos = 17, 0
    got = []
    while len(got) < 24:
        ids = sess.greedy(tok, pos, 8)
        got += ids
        pos += len(ids)
        tok = ids[-1]
    ref = []
    tok, pos = 17, 0
    for _ in range(24):
        logits, _ = host.step(hkv, tok, pos, want_trace=False)
        tok = oracle.argmax_bf16(logits)
        ref.append(tok)
        pos += 1
    assert got == ref


def test_greedy_packet_stops_at_eos(cuda, schedule):
    cfg = TINY
    _, kv, sess, host, hkv = _setup(cfg, 512, seed=9)
    first = sess.greedy(17, 0, 8)
    _, kv2, sess2, _, _ = _setup(cfg, 512, seed=9)
    stop = first[3]
    ids = sess2.greedy(17, 0, 8, eos=[stop])
    assert ids == first[: first.index(stop) + 1]


@pytest.mark.parametrize("context", [1000, 16384 + 300])
@pytest.mark.parametrize("bits", [4, 8])
def test_long_context_step_bitexact(cuda, schedule, context, bits):
    """A prefilled synthetic cache (K, V ~ N(0,1) quantized) spanning several
    blocks and, at 16,684 tokens, two super-chunks."""
    cfg = replace(TINY, n_layers=1, kv_bits=bits)
    cap = (context + 256 + 255) // 256 * 256
    w, kv, sess, host, _ = _setup(cfg, cap, seed=21)
    kv.fill_random(context, seed=4)
    hkv = HostKV.from_device(cfg, kv)
    for i in range(3):
        pos = context + i
        logits, trace = sess.step(100 + i, pos, want_trace=True)
        sess.check_status()
        ref_logits, ref_trace = host.step(hkv, 100 + i, pos)
        assert np.array_equal(_u16(trace), ref_trace), pos
        assert np.array_equal(_u16(logits), ref_logits), pos


@pytest.mark.parametrize("ties", [False, True])
@pytest.mark.parametrize("variant", ["tiny_kv8_fp16", "tiny_kv4_bf16_sigmoid"])
def test_router_moe_entry_bitexact(cuda, variant, ties):
    """rec_router_moe (the MoE block of one layer alone) against the oracle's
    RMSNorm -> router -> top-k -> SwiGLU experts -> bf16 mix -> residual.
    With ties, odd router rows repeat the even ones, so every choice value
    occurs twice and the lower expert id must win each tie."""
    import ctypes as C

    from rec_b200._lib import check, lib

    cfg = VARIANTS[variant]
    w, kv, sess, host, hkv = _setup(cfg, 512, seed=11)
    sd = 1 if cfg.scale_dtype == torch.bfloat16 else 0
    rng = np.random.default_rng(13)
    layer = 1 if cfg.n_layers > 1 else 0
    if ties:
        R = w.layers[layer].router
        R[1::2] = R[0::2]
        if w.layers[layer].expert_bias is not None:
            bias = w.layers[layer].expert_bias
            bias[1::2] = bias[0::2]
        torch.cuda.synchronize()
    h = oracle.f32_to_bf16(rng.standard_normal(cfg.hidden, dtype=np.float32))
    h_dev = torch.from_numpy(h.view(np.int16)).cuda()
    ids_dev = torch.zeros(cfg.top_k, dtype=torch.int32, device="cuda")
    wts_dev = torch.zeros(cfg.top_k, dtype=torch.float32, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    check(lib().rec_router_moe(sess.ctx, layer, C.c_void_p(h_dev.data_ptr()), C.c_void_p(ids_dev.data_ptr()),
                               C.c_void_p(wts_dev.data_ptr()), stream), "rec_router_moe")
    torch.cuda.synchronize()
    L = w.layers[layer]
    xn = oracle.rmsnorm(h, _np(L.post_norm), cfg.rms_eps)
    logits = oracle.router_logits(_np(L.router), xn)
    bias = None if L.expert_bias is None else _np(L.expert_bias)
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
    want = oracle.f32_to_bf16(oracle.bf16_to_f32(h) + oracle.bf16_to_f32(mix))
    assert np.array_equal(ids_dev.cpu().numpy(), ids)
    assert np.array_equal(wts_dev.cpu().numpy().view(np.uint32), wts.view(np.uint32))
    assert np.array_equal(_u16(h_dev), want)
