"""Sampling head: the oracle's canonical sampler against a float64 restatement
of the reference's filter (CPU), and the CUDA sampler against the oracle bit
for bit (GPU, through the C ABI)."""
import zlib

import numpy as np
import pytest
import torch

import oracle
from rec_b200 import abi


def P(temperature=0.0, top_k=0, top_p=1.0, rep=1.0, presence=0.0):
    return abi.RecSampling(temperature, top_k, top_p, rep, presence)


def _penalised(logits_u16, history, rep, presence):
    x = oracle.bf16_to_f32(logits_u16).astype(np.float64)
    seen = np.zeros(x.size, bool)
    h = np.asarray(history, np.int64)
    seen[h[(h >= 0) & (h < x.size)]] = True
    if rep != 1.0:
        x[seen] = np.where(x[seen] < 0, x[seen] * rep, x[seen] / rep)
    x[seen] -= presence
    return x


def reference_sample(logits_u16, history, p, u, allowed=None):
    """filtered_sampling.py:7-22 + categorical (Gumbel-max) in float64 with a
    stable ascending argsort; engine.py:284 for temperature 0; an optional
    boolean grammar mask sets disallowed ids to -inf after the penalties
    (masked_sampling.py:101-110), top-k counting allowed ids only."""
    x = _penalised(logits_u16, history, p.repetition_penalty, p.presence_penalty)
    top_k = p.top_k
    if allowed is not None:
        if not allowed.any():
            return -1
        x = np.where(allowed, x, -np.inf)
        top_k = min(top_k, int(allowed.sum()))
    if p.temperature == 0:
        return int(np.argmax(x))
    m = x.max()
    lp = x - (m + np.log(np.sum(np.exp(x - m))))
    g = -np.log(-np.log(u.astype(np.float64)))
    if top_k == 0:
        z = x + g if (p.temperature == 1 and p.top_p >= 1) else lp / p.temperature + g
        return int(np.argmax(z))
    size = lp.size
    idx = np.argsort(lp, kind="stable")
    values = lp[idx]
    keep_p = np.cumsum(np.exp(values)) > 1 - p.top_p if p.top_p < 1 else np.ones(size, bool)
    threshold = values[-top_k]
    pos = np.arange(size)
    tie_start = np.min(np.where((values == threshold) & keep_p, pos, size))
    greater = np.sum(values > threshold)
    keep = keep_p & ((values > threshold) | ((values == threshold) & (pos < tie_start + top_k - greater)))
    mask = np.zeros(size, bool)
    mask[idx] = keep
    z = np.where(mask, lp / p.temperature + g, -np.inf)
    return int(np.argmax(z))


def _case(rng, V, ties=False):
    x = rng.standard_normal(V).astype(np.float32) * 3
    if ties:
        x = np.round(x * 2) / 2  # few distinct values
    return oracle.f32_to_bf16(x)


def test_log_accuracy():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.uniform(1e-38, 1e3, 100000), rng.uniform(0, 1, 100000),
                        [1e-45, 1e-40, 1.0, 2.0, 0.5]]).astype(np.float32)
    y = oracle.log(x).astype(np.float64)
    r = np.log(x.astype(np.float64))
    ulp = np.spacing(np.abs(r).astype(np.float32)).astype(np.float64)
    assert (np.abs(y - r) / np.maximum(ulp, 1e-45)).max() <= 2.0
    e = oracle.log(np.array([0.0, -0.0, np.inf, -1.0], np.float32))
    assert e[0] == -np.inf and e[1] == -np.inf and e[2] == np.inf and np.isnan(e[3])


CONFIGS = {
    "greedy": P(),
    "greedy_penalties": P(0.0, 0, 1.0, 1.1, 0.5),
    "t1_unfiltered": P(1.0),
    "t07_unfiltered": P(0.7),
    "config5": P(0.7, 40, 0.95, 1.1),
    "topk1": P(0.9, 1, 1.0),
    "topk_only": P(1.3, 50, 1.0, 1.0, 0.2),
    "tight_p": P(0.5, 200, 0.3),
}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_oracle_sampler_matches_reference_rule(name):
    p = CONFIGS[name]
    agree = total = 0
    for seed in range(40):
        rng = np.random.default_rng(seed)
        V = 3000
        lg = _case(rng, V, ties=seed % 3 == 0)
        hist = rng.integers(0, V, 200)
        u = rng.random(V, dtype=np.float32)
        got = oracle.sample(lg, hist, p, u)
        want = reference_sample(lg, hist, p, u)
        total += 1
        agree += got == want
    # float64 vs the canonical fp32 order may only differ on the rare draw
    # whose top-p boundary or Gumbel maximum is within rounding
    assert agree >= total - 1, (agree, total)


def test_oracle_sampler_tie_rule_exact():
    # 60 logits tie at the top-k threshold; top_p = 1: the kept tied ids are
    # the lowest-index ones
    V = 500
    x = np.full(V, -5.0, np.float32)
    x[:10] = 3.0
    x[100:160] = 1.0
    lg = oracle.f32_to_bf16(x)
    p = P(1.0, 20, 1.0)
    rng = np.random.default_rng(3)
    hits = set()
    for s in range(300):
        u = rng.random(V, dtype=np.float32)
        i = oracle.sample(lg, [], p, u)
        assert i == reference_sample(lg, [], p, u)
        hits.add(i)
    assert hits <= set(range(10)) | set(range(100, 110))
    assert hits & set(range(100, 110))


def _allow_rows(rng, B, V):
    """Grammar masks of varied density: half, 1 %, three ids, one id, none
    (row 5), everything, and two rows at random densities."""
    rows = []
    for b in range(B):
        kind = b % 8
        if kind == 0:
            m = rng.random(V) < 0.5
        elif kind == 1:
            m = rng.random(V) < 0.01
        elif kind == 2:
            m = np.zeros(V, bool)
            m[rng.choice(V, 3, replace=False)] = True
        elif kind == 3:
            m = np.zeros(V, bool)
            m[V - 1] = True  # the last id, in the partial tail word
        elif kind == 4:
            m = np.zeros(V, bool)
        elif kind == 5:
            m = np.ones(V, bool)
        else:
            m = rng.random(V) < rng.uniform(0.001, 0.2)
        rows.append(m)
    return rows


@pytest.mark.parametrize("name", list(CONFIGS))
def test_oracle_sampler_grammar_mask(name):
    p = CONFIGS[name]
    agree = total = 0
    for seed in range(16):
        rng = np.random.default_rng(100 + seed)
        V = 3001  # a partial tail word
        lg = _case(rng, V, ties=seed % 3 == 0)
        hist = rng.integers(0, V, 200)
        u = rng.random(V, dtype=np.float32)
        for m in _allow_rows(rng, 8, V):
            got = oracle.sample(lg, hist, p, u, allow=oracle.pack_allow(np.flatnonzero(m), V))
            want = reference_sample(lg, hist, p, u, m)
            if not m.any():
                assert got == -1
            elif m.sum() == 1:
                assert got == int(np.flatnonzero(m)[0])
            else:
                assert m[got]
            total += 1
            agree += got == want
    assert agree >= total - 1, (agree, total)


def test_oracle_sampler_mask_all_allowed_is_unmasked():
    rng = np.random.default_rng(5)
    V = 2048
    lg = _case(rng, V)
    u = rng.random(V, dtype=np.float32)
    full = oracle.pack_allow(np.arange(V), V)
    for p in CONFIGS.values():
        assert oracle.sample(lg, [], p, u, allow=full) == oracle.sample(lg, [], p, u)


# ---------------------------------------------------------------------------- GPU
@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CONFIGS))
def test_gpu_sampler_bitexact(cuda, name):
    from rec_b200 import sampling

    p = CONFIGS[name]
    B, V = 8, 151936
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    rows = [_case(rng, V, ties=(b % 2 == 1)) for b in range(B)]
    lg = np.stack(rows)
    hist = rng.integers(0, V, (B, 4096)).astype(np.int32)
    u = torch.rand(B, V, generator=torch.Generator(device=cuda).manual_seed(7), device=cuda)
    ids = sampling.sample_logits(torch.from_numpy(lg.view(np.int16)).to(cuda).view(torch.bfloat16), p,
                                 u if p.temperature > 0 else None, torch.from_numpy(hist).to(cuda))
    ids = ids.cpu().numpy()
    uh = u.cpu().numpy()
    for b in range(B):
        assert ids[b] == oracle.sample(lg[b], hist[b], p, uh[b]), b


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CONFIGS))
def test_gpu_sampler_grammar_mask_bitexact(cuda, name):
    from rec_b200 import sampling

    p = CONFIGS[name]
    B, V = 8, 151937  # a partial tail word
    rng = np.random.default_rng(zlib.crc32(b"mask" + name.encode()))
    lg = np.stack([_case(rng, V, ties=(b % 2 == 1)) for b in range(B)])
    hist = rng.integers(0, V, (B, 1024)).astype(np.int32)
    masks = _allow_rows(rng, B, V)
    W = (V + 31) // 32 + 3  # padded row stride
    allow = np.zeros((B, W), np.uint32)
    for b, m in enumerate(masks):
        allow[b, : (V + 31) // 32] = oracle.pack_allow(np.flatnonzero(m), V)
    u = torch.rand(B, V, generator=torch.Generator(device=cuda).manual_seed(11), device=cuda)
    ids = sampling.sample_logits(torch.from_numpy(lg.view(np.int16)).to(cuda).view(torch.bfloat16), p,
                                 u if p.temperature > 0 else None, torch.from_numpy(hist).to(cuda),
                                 allow=torch.from_numpy(allow.view(np.int32)).to(cuda))
    ids = ids.cpu().numpy()
    uh = u.cpu().numpy()
    for b in range(B):
        want = oracle.sample(lg[b], hist[b], p, uh[b], allow=allow[b])
        assert ids[b] == want, (b, ids[b], want)
        assert (want == -1) == (not masks[b].any())


@pytest.mark.gpu
def test_gpu_sampler_threshold_ties(cuda):
    from rec_b200 import sampling

    V = 151936
    x = np.full(V, -5.0, np.float32)
    x[:10] = 3.0
    x[70000:70300] = 1.0  # 300 ties at the threshold, spread over many threads
    lg = oracle.f32_to_bf16(x)
    p = P(0.8, 40, 0.99)
    g = torch.Generator(device=cuda).manual_seed(3)
    for _ in range(4):
        u = torch.rand(V, generator=g, device=cuda)
        i = int(sampling.sample_logits(torch.from_numpy(lg.view(np.int16)).to(cuda).view(torch.bfloat16), p, u)[0])
        assert i == oracle.sample(lg, [], p, u.cpu().numpy())


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 3, 8])
def test_gpu_sample_head_config5(cuda, batch):
    """Config 5: final RMSNorm + int4 lm_head 2048 -> 151,936 + penalty 1.1
    over 4,096 history ids, T 0.7, top-k 40, top-p 0.95, Philox uniforms."""
    from rec_b200 import ops, sampling
    from rec_b200.model import QTensor

    V, H = 151936, 2048
    g = torch.Generator(device=cuda).manual_seed(5)
    w = torch.randn(V, H, generator=g, device=cuda) * 0.02
    lm = QTensor(*ops.quantize_affine(w, 4, torch.float16))
    del w
    fn = (1 + 0.1 * torch.randn(H, generator=g, device=cuda)).to(torch.bfloat16)
    h = torch.randn(batch, H, generator=g, device=cuda).to(torch.bfloat16)
    hist = torch.randint(0, V, (batch, 4096), generator=g, device=cuda, dtype=torch.int32)
    u = sampling.uniforms(batch, V, 11, cuda)
    p = sampling.params(0.7, 40, 0.95, 1.1)
    ids, logits = sampling.sample_head(h, fn, lm, torch.float16, p, u, hist)
    ids = ids.cpu().numpy()
    codes = lm.w.cpu().numpy().view(np.uint32)
    sc = lm.s.view(torch.int16).cpu().numpy().view(np.uint16)
    bi = lm.b.view(torch.int16).cpu().numpy().view(np.uint16)
    fnh = fn.view(torch.int16).cpu().numpy().view(np.uint16)
    for b in range(batch):
        hb = h[b].view(torch.int16).cpu().numpy().view(np.uint16)
        ref_logits = oracle.gemv(codes, sc, bi, oracle.rmsnorm(hb, fnh, 1e-6), 0)
        assert np.array_equal(logits[b].view(torch.int16).cpu().numpy().view(np.uint16), ref_logits)
        assert ids[b] == oracle.sample(ref_logits, hist[b].cpu().numpy(), p, u[b].cpu().numpy())


@pytest.mark.gpu
def test_gpu_resident_sampler_block(cuda):
    """ResidentSampler.block with temperature > 0 through the engine API: ids
    equal the oracle's decode + sampler with the same Philox uniforms."""
    from oracle.host import HostKV, HostModel
    from rec_b200 import sampling
    from rec_b200.engine import build_decoder
    from rec_b200.model import TINY, generate_weights

    cfg = TINY
    w = generate_weights(cfg, seed=9, device="cuda")
    engine, sampler = build_decoder(w)
    state = engine.prefill_state(512)
    prompt = [3, 77, 1024, 5]
    for t in prompt[:-1]:
        engine.forward(state, t)
    ids = sampler.block(state, prompt[-1], 6, 1234, temperature=0.8, top_p=0.9, top_k=30,
                        presence_penalty=0.4)
    assert state["position"] == len(prompt) - 1 + len(ids)
    host = HostModel(w)
    hkv = HostKV(cfg, 512)
    for i, t in enumerate(prompt[:-1]):
        host.step(hkv, t, i, want_trace=False)
    u = sampling.uniforms(6, cfg.vocab, 1234, cuda).cpu().numpy()
    p = sampling.params(0.8, 30, 0.9, 1.0, 0.4)
    tok, want, seen = prompt[-1], [], []
    for i in range(6):
        logits, _ = host.step(hkv, tok, len(prompt) - 1 + i, want_trace=False)
        tok = oracle.sample(logits, np.array(seen, np.int32), p, u[i])
        want.append(tok)
        seen.append(tok)
    assert ids == want


@pytest.mark.parametrize("schedule", ["mega", "graph", "split"])
def test_gpu_resident_sampler_eos(cuda, schedule, monkeypatch):
    """A sampled packet stops recording at an EOS id (included), on both
    schedules, and the ids before it equal the packet without EOS."""
    monkeypatch.setenv("REC_SCHEDULE", schedule)
    from rec_b200.engine import build_decoder
    from rec_b200.model import TINY, generate_weights

    w = generate_weights(TINY, seed=5, device="cuda")

    def packet(eos):
        engine, sampler = build_decoder(w, eos_tokens=eos)
        state = engine.prefill_state(256)
        for t in (9, 40):
            engine.forward(state, t)
        return sampler.block(state, 7, 8, 99, temperature=1.0, top_k=20, top_p=0.95, presence_penalty=0.2), state

    full, _ = packet(())
    assert len(full) == 8
    stop = full[4]
    cut, state = packet((stop,))
    k = full.index(stop)
    assert cut == full[: k + 1]
    assert state["position"] == 2 + len(cut)


class _ToyGrammar:
    """Stands in for the reference's ConstraintSession (grammar.py:46-104):
    stop ids and the matcher callback _advance(token, active) that returns
    the next step's allow words.  Its rule: after token t the allowed ids are
    (31 t + 7 j) mod V for j < 40."""

    def __init__(self, V, stops):
        self.V, self.stops, self.accepted = V, tuple(stops), []

    def allowed(self, t):
        return sorted({(31 * t + 7 * j) % self.V for j in range(40)})

    def _advance(self, token, active):
        self.accepted.append(token)
        return oracle.pack_allow(self.allowed(token), self.V)


@pytest.mark.gpu
@pytest.mark.parametrize("temperature", [0.0, 0.8])
def test_gpu_resident_sampler_grammar(cuda, temperature):
    """ResidentSampler.block with a grammar: every id is allowed by the mask
    in force, the packet stops at a grammar stop id, and the ids equal the
    oracle's decode + masked sampler chain with the same uniforms."""
    from oracle.host import HostKV, HostModel
    from rec_b200 import sampling
    from rec_b200.engine import build_decoder
    from rec_b200.model import TINY, generate_weights

    cfg = TINY
    V = cfg.vocab
    w = generate_weights(cfg, seed=21, device="cuda")
    engine, sampler = build_decoder(w)
    prompt = [11, 300, 5]
    count, seed = 8, 77
    p = sampling.params(temperature, 30 if temperature else 0, 0.95 if temperature else 1.0, 1.0,
                        0.3 if temperature else 0.0)
    host = HostModel(w)
    u = sampling.uniforms(count, V, seed, cuda).cpu().numpy()

    def expected(stops, first_allowed):
        g = _ToyGrammar(V, stops)
        hkv = HostKV(cfg, 256)
        for i, t in enumerate(prompt[:-1]):
            host.step(hkv, t, i, want_trace=False)
        tok, out, seen = prompt[-1], [], []
        allow = oracle.pack_allow(first_allowed, V)
        for i in range(count):
            logits, _ = host.step(hkv, tok, len(prompt) - 1 + i, want_trace=False)
            tok = oracle.sample(logits, np.array(seen, np.int32), p, u[i] if temperature else None, allow=allow)
            assert tok >= 0 and (allow[tok >> 5] >> (tok & 31)) & 1
            out.append(tok)
            seen.append(tok)
            allow = g._advance(tok, True)
            if tok in stops:
                break
        return out

    first = list(range(100, 160))
    free = expected((), first)
    for stops in [(), (free[3],)]:
        g = _ToyGrammar(V, stops)
        state = engine.prefill_state(256)
        for t in prompt[:-1]:
            engine.forward(state, t)
        state["grammar_mask"] = np.concatenate([oracle.pack_allow(first, V), np.ones(1, np.uint32)])
        ids = sampler.block(state, prompt[-1], count, seed, temperature=temperature, top_p=p.top_p, top_k=p.top_k,
                            presence_penalty=p.presence_penalty, grammar=g)
        assert ids == expected(stops, first)
        assert g.accepted == ids
        assert state["position"] == len(prompt) - 1 + len(ids)
        if stops:
            assert ids == free[: free.index(stops[0]) + 1]
