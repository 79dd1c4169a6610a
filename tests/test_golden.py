"""Golden fixtures (tests/golden): the oracle (CPU) and the CUDA path (GPU,
through the C ABI) must both reproduce the frozen outputs bit for bit."""
import numpy as np
import pytest
import torch

import oracle
from golden import cases


@pytest.mark.parametrize("name", list(cases.GEMV_CASES))
def test_oracle_gemv_golden(name):
    k, sd, seed = cases.GEMV_CASES[name]
    want = cases.load(name)
    got = cases.run_oracle_gemv(k, sd, seed)
    assert str(got["input_sha"]) == str(want["input_sha"]), "regenerated inputs changed"
    assert np.array_equal(got["y"], want["y"])
    if "y_norm" in want:
        assert np.array_equal(got["y_norm"], want["y_norm"])


@pytest.mark.parametrize("name", list(cases.DECODE_CASES))
def test_oracle_decode_golden(name):
    cfg, seed = cases.DECODE_CASES[name]
    want = cases.load(name)
    got = cases.run_oracle_decode(cfg, seed)
    assert str(got["input_sha"]) == str(want["input_sha"]), "regenerated inputs changed"
    assert np.array_equal(got["ids"], want["ids"])
    assert list(got["logits_sha"]) == list(want["logits_sha"])
    assert np.array_equal(got["last_logits"], want["last_logits"])
    assert str(got["trace0_sha"]) == str(want["trace0_sha"])
    assert str(got["kv_new_sha"]) == str(want["kv_new_sha"])


# ---------------------------------------------------------------------------- GPU
def _dev(a, dev):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    elif a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).to(dev)


def _u16(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(cases.GEMV_CASES))
def test_gpu_gemv_golden(cuda, name):
    from rec_b200 import ops

    k, sd, seed = cases.GEMV_CASES[name]
    want = cases.load(name)
    w, x, nw = cases.gemv_inputs(k, sd, seed)
    st = torch.float16 if sd == 0 else torch.bfloat16
    W, S, B = _dev(w.w, cuda), _dev(w.s, cuda).view(st), _dev(w.b, cuda).view(st)
    X = _dev(x, cuda).view(torch.bfloat16)
    assert np.array_equal(_u16(ops.gemv_int4(W, S, B, X)), want["y"])
    if "y_norm" in want:
        NW = _dev(nw, cuda).view(torch.bfloat16)
        assert np.array_equal(_u16(ops.gemv_int4(W, S, B, X, norm_weight=NW, eps=1e-6)), want["y_norm"])


def _device_weights(m, dev):
    from rec_b200.model import LayerWeights, ModelWeights, QTensor

    st = m.cfg.scale_dtype

    def q(t):
        return QTensor(_dev(t.w, dev), _dev(t.s, dev).view(st), _dev(t.b, dev).view(st))

    def bf(a):
        return None if a is None else _dev(a, dev).view(torch.bfloat16)

    def qo(t):
        return None if t is None else q(t)

    layers = [LayerWeights(input_norm=bf(L.input_norm), post_norm=bf(L.post_norm), q=q(L.q), k=q(L.k), v=q(L.v),
                           o=q(L.o), router=bf(L.router), gate=q(L.gate), up=q(L.up), down=q(L.down),
                           expert_bias=None if L.expert_bias is None else _dev(L.expert_bias, dev),
                           sinks=bf(L.sinks), q_norm=bf(L.q_norm), k_norm=bf(L.k_norm), kind=L.kind,
                           shared_gate=qo(L.shared_gate), shared_up=qo(L.shared_up), shared_down=qo(L.shared_down))
              for L in m.layers]
    return ModelWeights(m.cfg, layers, q(m.embed), bf(m.final_norm), q(m.lm_head))


@pytest.fixture(params=["mega", "graph", "split"])
def schedule(request, monkeypatch):
    monkeypatch.setenv("REC_SCHEDULE", request.param)
    return request.param


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(cases.DECODE_CASES))
def test_gpu_decode_golden(cuda, schedule, name):
    from oracle.host import HostKV
    from rec_b200.model import KVCache
    from rec_b200.session import DecodeSession

    cfg, seed = cases.DECODE_CASES[name]
    want = cases.load(name)
    m = cases.host_model(cfg, seed)
    assert cases.model_sha(m) == str(want["input_sha"])
    hkv = HostKV(cfg, cases.CAPACITY)
    cases.fill_kv(hkv, cfg, seed + 1)
    weights = _device_weights(m, cuda)
    kv = KVCache.allocate(cfg, cases.CAPACITY)
    for d, h in zip(kv.layers, hkv.layers):
        for n in d:
            d[n].copy_(_dev(h[n], cuda).view(d[n].dtype))
    sess = DecodeSession(weights, kv)
    token, ids = cases.START_TOKEN, []
    for i in range(cases.STEPS):
        logits, trace = sess.step(token, cases.CONTEXT + i, want_trace=True)
        lg = _u16(logits)
        assert cases.sha(lg) == str(want["logits_sha"][i]), f"step {i}"
        if i == 0:
            assert cases.sha(_u16(trace)) == str(want["trace0_sha"])
        token = oracle.argmax_bf16(lg)
        ids.append(token)
    sess.check_status()
    assert ids == want["ids"].tolist()
    assert np.array_equal(lg, want["last_logits"])
    layers = [{n: _u16(t) if t.dtype != torch.int32 else t.cpu().numpy().view(np.uint32) for n, t in L.items()}
              for L in kv.layers]
    assert cases.kv_sha(layers, cases.CONTEXT, cases.CONTEXT + cases.STEPS) == str(want["kv_new_sha"])
