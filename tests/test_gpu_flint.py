"""The reference Flint model's layer options on the GPU, bit-exact against the
oracle through the C ABI: an always-on shared expert (model.py:243,254), a
dense SwiGLU MLP layer of 6,144 rows (model.py:216-224, `mlp_only_layers`),
a NoPE layer (model.py:158-163) and sliding-window layers (model.py:302-313),
with the sigmoid + bias router, sinks, q/k head norms and bf16 scales; and
the bf16 KV cache of the reference megakernel (kv_format "bf16",
megakernel.py:619-693) and the native path's mixed cache (K 8-bit, V 4-bit,
model.py:35-37,40-82), with and without those options.

Caches are filled with quantized synthetic K, V up to the decode position, so
that the window starts past the first work item (600 tokens: window start in
block 1) and, at 17,000 tokens, inside a 4-block item (block 64 skipped, a
tile of block 65 cut)."""
from dataclasses import replace

import numpy as np
import pytest
import torch

import oracle
from oracle.host import HostKV, HostModel, _np
from rec_b200.model import TINY, TINY_FLINT, KVCache, generate_weights
from rec_b200.session import DecodeSession

pytestmark = pytest.mark.gpu


def _u16(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _setup(cfg, capacity, context, seed):
    w = generate_weights(cfg, seed=seed, device="cuda")
    kv = KVCache.allocate(cfg, capacity)
    kv.fill_random(context, seed=seed + 1)
    torch.cuda.synchronize()
    sess = DecodeSession(w, kv)
    host = HostModel(w)
    hkv = HostKV.from_device(cfg, kv)
    return w, kv, sess, host, hkv


def _compare_rows(kv, hkv, lo, hi):
    for li, (d, h) in enumerate(zip(kv.layers, hkv.layers)):
        for name in d:
            assert np.array_equal(_np(d[name])[:, lo:hi], h[name][:, lo:hi]), (li, name)


VARIANTS = {"flint_kv8": TINY_FLINT, "flint_bf16_kv": replace(TINY_FLINT, kv_bits=16),
            "tiny_bf16_kv": replace(TINY, kv_bits=16),
            # the reference's mixed cache (K 8-bit, V 4-bit), and the other mix
            "flint_k8_v4": replace(TINY_FLINT, kv_value_bits=4),
            "tiny_k4_v8": replace(TINY, kv_bits=4, kv_value_bits=8)}


@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("context", [600, 17000])
def test_flint_decode_steps_bitexact(cuda, variant, context):
    cfg = VARIANTS[variant]
    cap = (context + 8 + 255) // 256 * 256
    _, kv, sess, host, hkv = _setup(cfg, cap, context, seed=41)
    rng = np.random.default_rng(43)
    for i in range(3):
        tok, pos = int(rng.integers(0, cfg.vocab)), context + i
        logits, trace = sess.step(tok, pos, want_trace=True)
        sess.check_status()
        ref_logits, ref_trace = host.step(hkv, tok, pos)
        got = _u16(trace)
        for li in range(cfg.n_layers + 1):
            assert np.array_equal(got[li], ref_trace[li]), (pos, li)
        assert np.array_equal(_u16(logits), ref_logits), pos
    _compare_rows(kv, hkv, context, context + 3)


@pytest.mark.parametrize("variant", ["flint_kv8", "flint_bf16_kv"])
def test_flint_greedy_packet_and_partial_depth(cuda, variant):
    """A 12-token greedy packet on the device equals the oracle's chain; a
    partial-depth step (the dense and the NoPE layer) equals the oracle's."""
    cfg = VARIANTS[variant]
    context = 600
    _, kv, sess, host, hkv = _setup(cfg, 1024, context, seed=51)
    ids = sess.greedy(17, context, 12)
    sess.check_status()
    tok, want = 17, []
    for i in range(12):
        lg, _ = host.step(hkv, tok, context + i, want_trace=False)
        tok = oracle.argmax_bf16(lg)
        want.append(tok)
    assert list(ids) == want
    pos = context + 12
    logits, trace = sess.step_layers(99, pos, 2)
    sess.check_status()
    ref_logits, ref_trace = host.step(hkv, 99, pos, layer_count=2)
    assert np.array_equal(_u16(trace), ref_trace)
    assert np.array_equal(_u16(logits), ref_logits)


@pytest.mark.parametrize("layer", [0, 1])
def test_flint_ffn_entry_bitexact(cuda, layer):
    """rec_router_moe on a dense-MLP layer (norm -> 6,144-row SwiGLU MLP ->
    residual) and on an MoE layer with a shared expert (routed mix, then
    mlp = bf16(mix + shared), then the residual)."""
    import ctypes as C

    from rec_b200._lib import check, lib

    cfg = TINY_FLINT
    w, kv, sess, host, hkv = _setup(cfg, 512, 0, seed=61)
    sd = 1
    h = oracle.f32_to_bf16(np.random.default_rng(63).standard_normal(cfg.hidden, dtype=np.float32))
    h_dev = torch.from_numpy(h.view(np.int16)).cuda()
    ids_dev = torch.zeros(cfg.top_k, dtype=torch.int32, device="cuda")
    wts_dev = torch.zeros(cfg.top_k, dtype=torch.float32, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    check(lib().rec_router_moe(sess.ctx, layer, C.c_void_p(h_dev.data_ptr()), C.c_void_p(ids_dev.data_ptr()),
                               C.c_void_p(wts_dev.data_ptr()), stream), "rec_router_moe")
    torch.cuda.synchronize()
    L = w.layers[layer]
    xn = oracle.rmsnorm(h, _np(L.post_norm), cfg.rms_eps)

    def mlp(g_, u_, d_):
        g = oracle.gemv(_np(g_.w), _np(g_.s), _np(g_.b), xn, sd)
        u = oracle.gemv(_np(u_.w), _np(u_.s), _np(u_.b), xn, sd)
        act = np.array([oracle.swiglu(int(a), int(b)) for a, b in zip(g, u)], np.uint16)
        return oracle.gemv(_np(d_.w), _np(d_.s), _np(d_.b), act, sd)

    if layer == 0:  # dense
        update = mlp(L.gate, L.up, L.down)
    else:
        logits = oracle.router_logits(_np(L.router), xn)
        ids, wts = oracle.route(logits, cfg.top_k, cfg.router_mode, _np(L.expert_bias))
        I, H = cfg.moe_inter, cfg.hidden
        downs = []
        for e in ids:
            r, dr = slice(int(e) * I, (int(e) + 1) * I), slice(int(e) * H, (int(e) + 1) * H)
            g = oracle.gemv(_np(L.gate.w)[r], _np(L.gate.s)[r], _np(L.gate.b)[r], xn, sd)
            u = oracle.gemv(_np(L.up.w)[r], _np(L.up.s)[r], _np(L.up.b)[r], xn, sd)
            act = np.array([oracle.swiglu(int(a), int(b)) for a, b in zip(g, u)], np.uint16)
            downs.append(oracle.gemv(_np(L.down.w)[dr], _np(L.down.s)[dr], _np(L.down.b)[dr], act, sd))
        mix = oracle.mix(np.stack(downs), wts)
        shared = mlp(L.shared_gate, L.shared_up, L.shared_down)
        update = oracle.f32_to_bf16(oracle.bf16_to_f32(mix) + oracle.bf16_to_f32(shared))
        assert np.array_equal(ids_dev.cpu().numpy(), ids)
        assert np.array_equal(wts_dev.cpu().numpy().view(np.uint32), wts.view(np.uint32))
    want = oracle.f32_to_bf16(oracle.bf16_to_f32(h) + oracle.bf16_to_f32(update))
    assert np.array_equal(_u16(h_dev), want)


@pytest.mark.parametrize("kv_bits,kv_value_bits", [(8, 0), (16, 0), (8, 4)])
def test_flint_engine_prefill_and_block(cuda, kv_bits, kv_value_bits):
    """Through the reference-facing API: QATSession.prefill (a model with
    layer options is prefilled by its decode step) and ResidentSampler.block
    at temperature 0 equal the oracle's chain."""
    from rec_b200.engine import build_decoder

    # the window moves within the short prompt
    cfg = replace(TINY_FLINT, sliding_window=24, kv_bits=kv_bits, kv_value_bits=kv_value_bits)
    w = generate_weights(cfg, seed=71, device="cuda")
    engine, sampler = build_decoder(w)
    prompt = [int(t) for t in np.random.default_rng(73).integers(0, cfg.vocab, 40)]
    qs = engine.make_session(max_new_tokens=32)
    logits = qs.prefill(prompt)
    host = HostModel(w)
    hkv = HostKV(cfg, 256)
    for i, t in enumerate(prompt):
        ref, _ = host.step(hkv, t, i, want_trace=False)
    assert np.array_equal(_u16(logits), ref)
    state = qs._state
    first = oracle.argmax_bf16(ref)
    ids = sampler.block(state, first, 8, 0, temperature=0)
    tok, want = first, []
    for i in range(8):
        lg, _ = host.step(hkv, tok, len(prompt) + i, want_trace=False)
        tok = oracle.argmax_bf16(lg)
        want.append(tok)
    assert list(ids) == want
