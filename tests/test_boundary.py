"""The drop-in API's remaining contracts (reference engine/src/rec_mlx):

- logprobs through ResidentSampler.block (masked_sampling.py:126-128,
  145-146, 205-206; engine.py:264,296): the reported value is
  report[id] - logsumexp(report), report = penalised, masked logits / T;
- FullModel.forward(state, token, layer_count) at partial depth
  (megakernel.py:824,861,1224-1233,1272);
- the engine attributes the reference's callers read: `metadata` (the
  layer table, megakernel.py:1008-1088, read by engine.py:326 and
  kernels/activation_optimization.py:20-25), `banks`, `silu`
  (megakernel.py:1110-1112) and `device_profile.chip` (engine.py:244);
- the failure contract (megakernel.py:137-159,1264-1268,1326-1331;
  sampling.py:77-78): a bounded device wait that runs out gives
  RuntimeError("GPU synchronization failed ...") and state["usable"] = False,
  and the next call raises "... invalidated ..."; the context limit and the
  packet size give ValueError.  The wait is made to run out by one CTA that
  skips its grid-barrier arrivals (rec_set_fault_injection), with a short
  poll bound: nothing faults, traps or hangs.
"""
import numpy as np
import pytest
import torch

import oracle
from rec_b200 import abi


def P(temperature=0.0, top_k=0, top_p=1.0, rep=1.0, presence=0.0):
    return abi.RecSampling(temperature, top_k, top_p, rep, presence)


def _reference_logprob(logits_u16, history, p, token, allowed=None):
    """float64 restatement: report = x / T (or x), x the penalised logits
    with disallowed ids at -inf; report[token] - logsumexp(report)."""
    x = oracle.bf16_to_f32(logits_u16).astype(np.float64)
    seen = np.zeros(x.size, bool)
    h = np.asarray(history, np.int64)
    seen[h[(h >= 0) & (h < x.size)]] = True
    if p.repetition_penalty != 1.0:
        x[seen] = np.where(x[seen] < 0, x[seen] * p.repetition_penalty, x[seen] / p.repetition_penalty)
    x[seen] -= p.presence_penalty
    if allowed is not None:
        x = np.where(allowed, x, -np.inf)
    r = x / p.temperature if p.temperature else x
    m = r.max()
    return float(r[token] - (m + np.log(np.sum(np.exp(r - m)))))


LP_CONFIGS = {"greedy": P(), "t07": P(0.7), "t1_presence": P(1.0, 0, 1.0, 1.0, 0.5),
              "config5": P(0.7, 40, 0.95, 1.1), "t13_rep": P(1.3, 0, 1.0, 1.2, 0.0)}


@pytest.mark.parametrize("name", list(LP_CONFIGS))
def test_oracle_token_logprob_matches_reference(name):
    p = LP_CONFIGS[name]
    rng = np.random.default_rng(len(name))
    V = 151936
    logits = oracle.f32_to_bf16((rng.standard_normal(V) * 3).astype(np.float32))
    hist = rng.integers(0, V, 4096).astype(np.int32)
    for tok in [0, int(np.argmax(oracle.bf16_to_f32(logits))), int(rng.integers(V)), V - 1]:
        got = oracle.token_logprob(logits, hist, p, tok)
        want = _reference_logprob(logits, hist, p, tok)
        assert abs(got - want) <= 1e-5 * max(1.0, abs(want)), (tok, got, want)
    assert np.isnan(oracle.token_logprob(logits, hist, p, V))
    allowed = np.zeros(V, bool)
    allowed[rng.integers(0, V, 500)] = True
    allow = oracle.pack_allow(np.flatnonzero(allowed), V)
    tok = int(np.flatnonzero(allowed)[3])
    got = oracle.token_logprob(logits, hist, p, tok, allow=allow)
    want = _reference_logprob(logits, hist, p, tok, allowed)
    assert abs(got - want) <= 1e-5 * max(1.0, abs(want))
    assert oracle.token_logprob(logits, hist, p, int(np.flatnonzero(~allowed)[0]), allow=allow) == -np.inf


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(LP_CONFIGS))
def test_gpu_token_logprob_bitexact(cuda, name):
    """rec_token_logprob against the oracle, bit for bit, for 4 rows of
    151,936 logits (one with a grammar mask)."""
    from rec_b200 import sampling

    p = LP_CONFIGS[name]
    rng = np.random.default_rng(100 + len(name))
    B, V = 4, 151936
    logits = oracle.f32_to_bf16((rng.standard_normal((B, V)) * 3).astype(np.float32))
    hist = rng.integers(0, V, (B, 2048)).astype(np.int32)
    ids = np.array([int(rng.integers(V)) for _ in range(B)], np.int32)
    ids[1] = int(np.argmax(oracle.bf16_to_f32(logits[1])))
    lg = torch.from_numpy(logits.view(np.int16)).cuda().view(torch.bfloat16)
    out = sampling.token_logprob(lg, p, torch.from_numpy(ids).cuda(), torch.from_numpy(hist).cuda())
    got = out.cpu().numpy()
    for b in range(B):
        want = oracle.token_logprob(logits[b], hist[b], p, int(ids[b]))
        assert np.float32(want).view(np.uint32) == got[b].view(np.uint32), (b, got[b], want)


def _tiny_engine(seed=9):
    from rec_b200.engine import build_decoder
    from rec_b200.model import TINY, generate_weights

    w = generate_weights(TINY, seed=seed, device="cuda")
    engine, sampler = build_decoder(w)
    return w, engine, sampler


@pytest.mark.gpu
@pytest.mark.parametrize("temperature", [0.0, 0.8])
def test_gpu_resident_sampler_logprobs(cuda, temperature):
    """ResidentSampler.block(logprobs=list): the ids equal the packet's ids
    without logprobs, and each reported value equals the oracle's on the
    oracle's own decode chain, bit for bit."""
    from oracle.host import HostKV, HostModel
    from rec_b200 import sampling

    w, engine, sampler = _tiny_engine()
    cfg = w.cfg
    prompt, count, seed = [3, 77, 1024, 5], 6, 4321
    kw = dict(temperature=temperature, top_p=0.9 if temperature else 1.0, top_k=30 if temperature else 0,
              presence_penalty=0.4 if temperature else 0.0)

    def run(with_lp):
        state = engine.prefill_state(256)
        for t in prompt[:-1]:
            engine.forward(state, t)
        lps = [] if with_lp else None
        ids = sampler.block(state, prompt[-1], count, seed, logprobs=lps, **kw)
        return ids, lps, state

    fast, _, _ = run(False)
    ids, lps, state = run(True)
    assert ids == fast
    assert len(lps) == len(ids)
    assert state["position"] == len(prompt) - 1 + len(ids)
    host = HostModel(w)
    hkv = HostKV(cfg, 256)
    for i, t in enumerate(prompt[:-1]):
        host.step(hkv, t, i, want_trace=False)
    p = sampling.params(kw["temperature"], kw["top_k"], kw["top_p"], 1.0, kw["presence_penalty"])
    u = sampling.uniforms(count, cfg.vocab, seed, cuda).cpu().numpy() if temperature else None
    tok, seen = prompt[-1], []
    for i in range(len(ids)):
        logits, _ = host.step(hkv, tok, len(prompt) - 1 + i, want_trace=False)
        tok = oracle.sample(logits, np.array(seen, np.int32), p, u[i] if u is not None else None)
        assert tok == ids[i]
        want = oracle.token_logprob(logits, np.array(seen, np.int32), p, tok)
        assert np.float32(want).view(np.uint32) == np.float32(lps[i]).view(np.uint32), (i, lps[i], want)
        seen.append(tok)


@pytest.mark.gpu
def test_gpu_greedy_presence_penalty_takes_filtered_path(cuda):
    """Temperature 0 with a presence penalty: the penalty applies before the
    argmax (the reference routes it through its filtered sampler)."""
    from oracle.host import HostKV, HostModel
    from rec_b200 import sampling

    w, engine, sampler = _tiny_engine(seed=13)
    state = engine.prefill_state(256)
    engine.forward(state, 17)
    ids = sampler.block(state, 40, 8, 0, temperature=0.0, presence_penalty=2.0)
    host = HostModel(w)
    hkv = HostKV(w.cfg, 256)
    host.step(hkv, 17, 0, want_trace=False)
    p = sampling.params(0.0, 0, 1.0, 1.0, 2.0)
    tok, seen, want = 40, [], []
    for i in range(8):
        logits, _ = host.step(hkv, tok, 1 + i, want_trace=False)
        tok = oracle.sample(logits, np.array(seen, np.int32), p, None)
        want.append(tok)
        seen.append(tok)
    assert ids == want


@pytest.mark.gpu
@pytest.mark.parametrize("layer_count", [1, 2, 3])
def test_gpu_forward_partial_depth(cuda, layer_count):
    """forward(state, token, layer_count): logits and the trace of the layers
    run equal the oracle's partial-depth step; the cache rows of the layers
    run are written; a full step afterwards still matches."""
    from dataclasses import replace

    from oracle.host import HostKV, HostModel
    from rec_b200.engine import FullModel
    from rec_b200.model import TINY, generate_weights

    cfg = replace(TINY, n_layers=3)
    w = generate_weights(cfg, seed=31, device="cuda")
    engine = FullModel(w)
    state = engine.prefill_state(256)
    host = HostModel(w)
    hkv = HostKV(cfg, 256)
    for i, t in enumerate([5, 900, 77]):
        logits, trace = engine.forward(state, t)
        host.step(hkv, t, i, want_trace=False)
    logits, trace = engine.forward(state, 1234, layer_count=layer_count)
    assert trace.shape == (layer_count + 1, cfg.hidden)
    ref_logits, ref_trace = host.step(hkv, 1234, 3, layer_count=layer_count)
    u16 = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    assert np.array_equal(u16(trace), ref_trace)
    assert np.array_equal(u16(logits), ref_logits)
    kv = state["kv"].cache
    for li in range(layer_count):
        for name in kv.layers[li]:
            got = kv.layers[li][name][:, 3].contiguous()
            got = got.view(torch.int16).cpu().numpy().view(np.uint16) if got.dtype == torch.bfloat16 else \
                got.cpu().numpy().view(np.uint32)
            assert np.array_equal(got, hkv.layers[li][name][:, 3]), (li, name)
    # the next full step (the deeper layers' row 3 is whatever both wrote)
    for li in range(layer_count, cfg.n_layers):
        for name in kv.layers[li]:
            src = kv.layers[li][name][:, 3].contiguous()
            src = src.view(torch.int16).cpu().numpy().view(np.uint16) if src.dtype == torch.bfloat16 else \
                src.cpu().numpy().view(np.uint32)
            hkv.layers[li][name][:, 3] = src
    logits, trace = engine.forward(state, 66)
    ref_logits, ref_trace = host.step(hkv, 66, 4)
    assert np.array_equal(u16(trace), ref_trace)
    assert np.array_equal(u16(logits), ref_logits)
    with pytest.raises(ValueError):
        engine.forward(state, 1, layer_count=0)
    with pytest.raises(ValueError):
        engine.forward(state, 1, layer_count=cfg.n_layers + 1)


@pytest.mark.gpu
def test_gpu_failure_contract(cuda, monkeypatch):
    """A grid-barrier wait that runs out (one CTA skips its arrivals, poll
    bound 4,096) -> RuntimeError("GPU synchronization failed") and
    usable = False; the next call -> "invalidated"; the device and other
    sessions stay usable."""
    import ctypes as C

    from rec_b200._lib import check, lib

    monkeypatch.setenv("REC_SCHEDULE", "mega")
    w, engine, sampler = _tiny_engine(seed=3)
    state = engine.prefill_state(256)
    engine.forward(state, 5)
    sess = engine._session(state)
    check(lib().rec_set_fault_injection(sess.ctx, 4096, 1), "rec_set_fault_injection")
    with pytest.raises(RuntimeError, match="GPU synchronization failed"):
        engine.forward(state, 6)
    assert state["usable"] is False
    with pytest.raises(RuntimeError, match="invalidated"):
        engine.forward(state, 7)
    with pytest.raises(RuntimeError, match="invalidated"):
        sampler.block(state, 7, 4, 0, temperature=0)
    # the C session refuses further work too
    assert lib().rec_decode_step(sess.ctx, 1, 2, None, None,
                                 C.c_void_p(torch.cuda.current_stream().cuda_stream)) == abi.REC_ESTATE
    # a fresh state on the same device decodes normally
    fresh = engine.prefill_state(256)
    logits, _ = engine.forward(fresh, 5)
    assert torch.isfinite(logits.float()).all()


@pytest.mark.gpu
def test_gpu_limits_and_packet_size(cuda):
    """ValueError("Decode context limit exhausted") past the state's limit,
    and ValueError for packets outside 1..8 (sampling.py:77-78)."""
    w, engine, sampler = _tiny_engine(seed=4)
    state = engine.prefill_state(256, limit=3)
    for t in (1, 2, 3):
        engine.forward(state, t)
    with pytest.raises(ValueError, match="Decode context limit exhausted"):
        engine.forward(state, 4)
    state = engine.prefill_state(256)
    for bad in (0, 9):
        with pytest.raises(ValueError, match="between one and eight"):
            sampler.block(state, 1, bad, 0, temperature=0)
    state = engine.prefill_state(256, limit=4)
    with pytest.raises(ValueError, match="Decode context limit exhausted"):
        sampler.block(state, 1, 5, 0, temperature=0)


def test_layer_metadata_is_the_reference_table():
    """The Flint shape's table: 50 rows; column 1 marks the global layers
    (the rows engine.py:326 leaves out of its sliding bytes), column 2 the
    47 routed layers, whose gate / up / shared gate / shared up shapes are
    the tuple the reference's activation guard asserts
    (kernels/activation_optimization.py:20-25)."""
    from rec_b200.engine import layer_metadata
    from rec_b200.model import FLINT

    rows = layer_metadata(FLINT)
    assert len(rows) == 50 and all(len(r) == 64 for r in rows)
    assert [i for i, r in enumerate(rows[:49]) if r[1]] == sorted(FLINT.no_rope_layers)
    routed = [r for r in rows[:49] if r[2]]
    assert len(routed) == 47 and not rows[0][2] and not rows[1][2]
    assert all(tuple(r[i] for i in (33, 34, 38, 39, 48, 49, 53, 54))
               == (512, 2048, 512, 2048, 1024, 2048, 1024, 2048) for r in routed)
    assert tuple(rows[0][i] for i in (33, 34, 43, 44)) == (6144, 2048, 2048, 6144)
    assert tuple(rows[5][i] for i in (13, 14, 18, 19, 28, 29)) == (4096, 2048, 512, 2048, 2048, 4096)
    assert [r[0] for r in rows[:49]] == [i // 4 for i in range(49)] and rows[49][0] == 12
    assert tuple(rows[49][i] for i in (13, 14, 33, 34)) == (150144, 2048, 150144, 2048)
    # config 3: every layer global and routed, no shared expert
    from rec_b200.model import ModelConfig

    c3 = layer_metadata(ModelConfig(name="config3", n_experts=128, top_k=8, moe_inter=768, vocab=151936))
    assert len(c3) == 49 and all(r[1] == 1 and r[2] == 1 for r in c3[:48])
    assert all(tuple(r[i] for i in (33, 34, 43, 44, 48)) == (768, 2048, 2048, 768, 0) for r in c3[:48])


def test_weight_banks_group_four_layers():
    """engine.banks: each group of four layers' tensors once, in the layer
    fields' order (codes, scales, biases per matrix), the last group
    followed by the embedding, the final norm and lm_head (the reference's
    thirteen banks for 49 layers, megakernel.py:1011-1108)."""
    from rec_b200.engine import weight_banks
    from rec_b200.model import LayerWeights, ModelWeights, QTensor, TINY

    def t():
        return torch.zeros(2)

    def q():
        return QTensor(t(), t(), t())

    layers = [LayerWeights(input_norm=t(), post_norm=t(), q=q(), k=q(), v=q(), o=q(), router=t(), gate=q(), up=q(),
                           down=q(), expert_bias=t(), sinks=None, q_norm=None, k_norm=None) for _ in range(9)]
    w = ModelWeights(TINY, layers, q(), t(), q())
    banks = weight_banks(w)
    per_layer = 2 + 7 * 3 + 2  # norms, seven matrices, router and bias
    assert [len(b) for b in banks] == [4 * per_layer, 4 * per_layer, per_layer + 7]
    ids = [id(x) for b in banks for x in b]
    assert len(ids) == len(set(ids)) == 9 * per_layer + 7
    assert banks[0][0] is layers[0].input_norm and banks[0][2] is layers[0].q.w and banks[1][0] is layers[4].input_norm
    tail = (w.embed.w, w.embed.s, w.embed.b, w.final_norm, w.lm_head.w, w.lm_head.s, w.lm_head.b)
    assert all(a is b for a, b in zip(banks[-1][-7:], tail, strict=True))


def test_state_growth_and_limit_on_the_host():
    """prefill_state / ensure_capacity over a given storage, the contract of
    the reference's shared-KV test (engine/tests/test_shared_kv.py:64-80):
    the state keeps the storage and its table, a packet past the capacity
    grows that storage once and counts it, the limit gives ValueError and an
    unusable state raises "invalidated"."""
    from rec_b200.engine import FullModel

    block = 65536

    class Storage:
        def __init__(self):
            self.capacity, self.metadata, self.grown = 17, [[0] * 64], []

        def grow(self, count):
            self.grown.append(count)
            self.capacity = max(self.capacity, -(-count // block) * block)

    storage = Storage()
    state = FullModel.prefill_state(None, 17, limit=block + 8, storage=storage)
    state["position"] = block - 4
    FullModel.ensure_capacity(None, state, 8)
    assert state["kv"] is storage and state["metadata"] is storage.metadata
    assert state["capacity"] == 2 * block and state["growth_count"] == 1 and state["growth_seconds"] >= 0
    FullModel.ensure_capacity(None, state, 8)  # within the capacity: no growth
    assert state["growth_count"] == 1
    state["position"] = block + 7
    with pytest.raises(ValueError, match="Decode context limit exhausted"):
        FullModel.ensure_capacity(None, state, 2)
    state["usable"] = False
    with pytest.raises(RuntimeError, match="invalidated"):
        FullModel.ensure_capacity(None, state, 1)


@pytest.mark.gpu
def test_gpu_engine_attributes(cuda):
    """engine.silu is the SiLU of every bf16 gate (bit-exact against the
    oracle's SwiGLU with up = 1; NaN gates give NaN); engine.banks holds
    every weight tensor once, in groups of four layers; the state's table
    carries the cache rows in columns 61-62; device_profile.chip names the
    device, so the reference's M4-Max test is false."""
    from rec_b200.engine import layer_metadata

    w, engine, _ = _tiny_engine(seed=3)
    silu = engine.silu.view(torch.int16).cpu().numpy().view(np.uint16)
    want = np.array([oracle.swiglu(g, 0x3F80) for g in range(65536)], np.uint16)
    got_f, want_f = oracle.bf16_to_f32(silu), oracle.bf16_to_f32(want)
    both_nan = np.isnan(got_f) & np.isnan(want_f)
    assert np.array_equal(silu[~both_nan], want[~both_nan])
    assert np.array_equal(np.isnan(got_f), np.isnan(want_f))

    assert len(engine.banks) == -(-len(w.layers) // 4)
    ptrs = [t.data_ptr() for bank in engine.banks for t in bank]
    assert len(ptrs) == len(set(ptrs))
    assert {w.embed.w.data_ptr(), w.lm_head.w.data_ptr(), w.final_norm.data_ptr(),
            w.layers[0].q.w.data_ptr(), w.layers[-1].down.b.data_ptr()} <= set(ptrs)
    assert engine.metadata == layer_metadata(w.cfg)

    state = engine.prefill_state(256)
    cap = state["kv"].cache.capacity
    assert all(r[61:63] == [0, cap] for r in state["metadata"][:-1])
    assert state["metadata"] is state["kv"].metadata
    assert len(state["kv"].banks) == w.cfg.n_layers
    from rec_b200.prefix import PromptCache

    assert sum(L.nbytes for L in PromptCache([], state["kv"]).layers) == state["kv"].nbytes
    assert engine.device_profile.chip == torch.cuda.get_device_name()
    assert engine.device_profile.architecture.startswith("sm_") and engine.device_profile.chip != "M4 Max"
