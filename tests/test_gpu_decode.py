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


@pytest.fixture(params=["mega", "graph"])
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
