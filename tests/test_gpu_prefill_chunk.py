"""Chunked prompt prefill (rec_prefill_chunk through QATSession.prefill;
reference quantized.py:102-148).

Per operation, with the same inputs, against fp64 restatements of the
reference's formulas at the north-star tolerance (rel-L2 2e-3): the
projection and MoE GEMMs (test_gpu_prefill.py) and here the causal attention
over the quantized cache (rec_prefill_attention).

End to end, against the token-by-token decode path: the two paths differ at
the 1e-3 level in the hidden states (fp32 tensor-core accumulation vs the
canonical exact-integer GEMV, bf16 vs fixed-point attention arithmetic), and
quantize-on-append amplifies that.  A projected K or V value one bf16 ulp
apart lands on another 8-bit (4-bit) code in about 1 % of the entries, which
moves an attention output by a whole quantization step; with one layer and
one token this alone gives ~2.3e-3 in the hidden state, while with the
attention removed the chunk is within 2.6e-4 of the decode path (measured).
Any two implementations that are not bit-identical diverge this way, the
reference's own prefill (bf16-dequantizing quantized matmuls) and decode
included.  The end-to-end checks are therefore: the same greedy id, and the
logits within rel-L2 1e-2 (2 layers) / 4e-2 (48 layers, 1,024 tokens).
Every token's result is independent of the other rows of a tile, so the
logits do not depend on where the prompt is cut into chunks: bit for bit."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle
from oracle import semantic
from rec_b200 import abi

pytestmark = pytest.mark.gpu

TOL = 2e-3  # north-star rel-L2, per operation


def _f(t):
    return t.float().cpu().numpy().astype(np.float64)


def _prefill(engine, tokens, mode, chunk):
    engine.prefill_chunk_size = chunk
    s = engine.make_session(max_new_tokens=16, prefill_mode=mode)
    logits = s.prefill(tokens)
    return s, logits


@pytest.mark.parametrize("bits,sinks", [(8, False), (4, True)])
def test_prefill_attention_matches_fp64(cuda, bits, sinks):
    """37 query tokens at positions 300..336 over a 4-/8-bit cache of 337
    rows: each (token, head) output against the exact softmax of the bf16
    scores (fp64) over dequantized K, V (semantic.attention)."""
    from rec_b200._lib import check, lib

    hq, hkv, T, p0 = 32, 4, 37, 300
    n = p0 + T
    cap = 512
    rng = np.random.default_rng(bits)
    words = 128 * bits // 32
    host = {}
    for name in ("k", "v"):
        x = oracle.bf16_to_f32(oracle.f32_to_bf16(rng.standard_normal((hkv, n, 128), dtype=np.float32)))
        c, s, b = oracle.quantize(x, bits, 1)
        host[name] = (c, s, b)
    dev = {}
    for name, (c, s, b) in host.items():
        cc = np.zeros((hkv, cap, words), np.uint32)
        ss = np.zeros((hkv, cap, 2), np.uint16)
        bb = np.zeros((hkv, cap, 2), np.uint16)
        cc[:, :n], ss[:, :n], bb[:, :n] = c, s, b
        dev[name] = [torch.from_numpy(cc.view(np.int32)).cuda(), torch.from_numpy(ss.view(np.int16)).cuda(),
                     torch.from_numpy(bb.view(np.int16)).cuda()]
    rec = abi.RecKVLayer(dev["k"][0].data_ptr(), dev["k"][1].data_ptr(), dev["k"][2].data_ptr(),
                         dev["v"][0].data_ptr(), dev["v"][1].data_ptr(), dev["v"][2].data_ptr())
    q = oracle.f32_to_bf16(rng.standard_normal((T, hq, 128), dtype=np.float32))
    sk = oracle.f32_to_bf16(rng.standard_normal(hq, dtype=np.float32)) if sinks else None
    qd = torch.from_numpy(q.view(np.int16)).cuda()
    sd = torch.from_numpy(sk.view(np.int16)).cuda() if sinks else None
    out = torch.zeros(T, hq * 128, dtype=torch.int16, device="cuda")
    check(lib().rec_prefill_attention(C.c_void_p(qd.data_ptr()), hq, hkv, C.byref(rec), cap, bits, p0, T,
                                      C.c_void_p(sd.data_ptr()) if sinks else None, C.c_void_p(out.data_ptr()),
                                      C.c_void_p(torch.cuda.current_stream().cuda_stream)), "rec_prefill_attention")
    torch.cuda.synchronize()
    got = oracle.bf16_to_f32(out.cpu().numpy().view(np.uint16)).reshape(T, hq, 128).astype(np.float64)
    kd = oracle.dequantize(*host["k"], bits, 1)
    vd = oracle.dequantize(*host["v"], bits, 1)
    worst = 0.0
    for t in range(T):
        upto = p0 + t + 1
        want = semantic.attention(q[t], kd[:, :upto], vd[:, :upto], sinks=sk, bf16_probs=False)
        worst = max(worst, semantic.rel_l2(got[t], want))
    assert worst < TOL, worst


@pytest.fixture(scope="module")
def tiny(cuda):
    from rec_b200.engine import FullModel
    from rec_b200.model import TINY, generate_weights

    w = generate_weights(TINY, seed=23, device="cuda")
    return w, FullModel(w)


@pytest.mark.parametrize("n_tokens", [1, 37, 700])
def test_chunked_prefill_against_decode_path(tiny, n_tokens):
    w, engine = tiny
    rng = np.random.default_rng(n_tokens)
    tokens = rng.integers(0, w.cfg.vocab, n_tokens).tolist()
    _, ref = _prefill(engine, tokens, "decode", 1024)
    s, got = _prefill(engine, tokens, "chunked", 256)
    err = semantic.rel_l2(_f(got), _f(ref))
    print(f"tiny, {n_tokens} tokens: logits rel-L2 {err:.3e}")
    assert err < 1e-2, err
    assert int(torch.argmax(got.float())) == int(torch.argmax(ref.float()))
    # the chunk cut does not change a bit
    _, one = _prefill(engine, tokens, "chunked", 1024)
    assert torch.equal(one.view(torch.int16), got.view(torch.int16))
    # decoding continues from the prefilled cache
    nxt = s.forward_token(int(torch.argmax(got.float())))
    assert torch.isfinite(nxt.float()).all()


def test_prefill_interrupt_between_layers(tiny):
    """interrupt_between_layers (quantized.py:129-133, model.py:309-314): the
    chunks run layer by layer through rec_prefill_chunk_layers give the same
    bits as whole chunks; a stop requested between two layers of a chunk
    raises PrefillCancelled, and a later prefill is unaffected."""
    from rec_b200.errors import PrefillCancelled

    w, engine = tiny
    tokens = np.random.default_rng(5).integers(0, w.cfg.vocab, 300).tolist()
    _, whole = _prefill(engine, tokens, "chunked", 256)
    s = engine.make_session(max_new_tokens=16)
    by_layer = s.prefill(tokens, interrupt_between_layers=True)
    assert torch.equal(by_layer.view(torch.int16), whole.view(torch.int16))
    polls = []

    def stop():  # poll 1: before chunk 0; poll 2: between its layers 0 and 1
        polls.append(1)
        return len(polls) == 2

    with pytest.raises(PrefillCancelled):
        engine.make_session(max_new_tokens=16).prefill(tokens, should_stop=stop, interrupt_between_layers=True)
    assert len(polls) == 2
    _, again = _prefill(engine, tokens, "chunked", 256)
    assert torch.equal(again.view(torch.int16), whole.view(torch.int16))


def test_chunked_prefill_without_attention_is_close(cuda):
    """One layer with the O projection zeroed (attention cannot reach the
    residual): the chunk's hidden state is within the per-operation bound of
    the decode path's, which locates the end-to-end difference in the
    quantized K / V rows."""
    from dataclasses import replace

    from rec_b200.engine import FullModel
    from rec_b200.model import TINY, generate_weights

    cfg = replace(TINY, n_layers=1)
    w = generate_weights(cfg, seed=29, device="cuda")
    for t in (w.layers[0].o.w, w.layers[0].o.s, w.layers[0].o.b):
        t.zero_()
    engine = FullModel(w)
    tokens = list(range(200, 205))
    _, ref = _prefill(engine, tokens, "decode", 1024)
    _, got = _prefill(engine, tokens, "chunked", 1024)
    err = semantic.rel_l2(_f(got), _f(ref))
    assert err < TOL, err


def test_config3_prompt_1k(cuda):
    """The config-3 model (48 layers, 128 experts top-8, vocab 151,936, 8-bit
    cache) on a 1,024-token prompt: chunked prefill against the decode path,
    same greedy id."""
    from rec_b200.engine import FullModel
    from rec_b200.model import CONFIG3, generate_weights

    w = generate_weights(CONFIG3, seed=0, device="cuda")
    engine = FullModel(w)
    tokens = torch.randint(0, CONFIG3.vocab, (1024,), generator=torch.Generator().manual_seed(1)).tolist()
    _, ref = _prefill(engine, tokens, "decode", 1024)
    _, got = _prefill(engine, tokens, "chunked", 1024)
    err = semantic.rel_l2(_f(got), _f(ref))
    r = np.sort(_f(ref))
    print(f"config-3 1K prompt: logits rel-L2 {err:.3e}, decode-path top-1/top-2 margin {r[-1] - r[-2]:.4f}")
    assert err < 4e-2, err
    assert int(torch.argmax(got.float())) == int(torch.argmax(ref.float()))
