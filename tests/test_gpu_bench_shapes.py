"""Parity at the shapes the bench times: the CUDA path against the oracle,
bit for bit, on the configurations of BASELINE.json rather than on small
models.

- config 3 (48 layers, 128 experts top-8, vocab 151,936, 8-bit cache): the
  prompt is prefilled by decode steps, then 65 greedy tokens from position
  1,023 on each of the three schedules (persistent kernel, CUDA graph,
  split), in two device-side packets.  On a mismatch the first diverging
  step is reported with the oracle's top-1 / top-2 logit margin there.
- config 1 (one decoder layer, 64 experts, 1,024-token 8-bit cache): decode
  steps with logits and the residual trace on every schedule.
- config 4 (the 48-layer model at 258,048 tokens, 4-bit cache): four decode
  steps on the schedule the session picks there (the CUDA graph) and on the
  persistent kernel, logits and trace per step.

The reference's bar for this is validate_resident.py:233-289 (bit-exact
trace and logits against the native forward; packet equals scalar)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from oracle.host import HostKV, HostModel
from rec_b200.model import CONFIG1_LAYER, CONFIG3, CONFIG4, KVCache, generate_weights
from rec_b200.session import DecodeSession

pytestmark = pytest.mark.gpu

PROMPT = 1024
GREEDY = 65
SCHEDULES = ["mega", "graph", "split"]


def _u16(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _margin(logits_u16) -> float:
    x = np.sort(oracle.bf16_to_f32(logits_u16).astype(np.float64))
    return float(x[-1] - x[-2])


def _snapshot(kv: KVCache):
    return [{n: t.clone() for n, t in L.items()} for L in kv.layers]


def _restore(kv: KVCache, snap):
    for L, S in zip(kv.layers, snap):
        for n in L:
            L[n].copy_(S[n])
    torch.cuda.synchronize()


@pytest.fixture(scope="module")
def config3(cuda):
    """Config-3 weights (seed 0, as bench.py), the prompt (seed 1) prefilled
    by decode steps, and the oracle's greedy chain from there."""
    cfg = CONFIG3
    cap = (PROMPT + GREEDY + 255) // 256 * 256
    w = generate_weights(cfg, seed=0, device="cuda")
    kv = KVCache.allocate(cfg, cap)
    prompt = torch.randint(0, cfg.vocab, (PROMPT,), generator=torch.Generator().manual_seed(1)).tolist()
    sess = DecodeSession(w, kv)
    sess.prefill(prompt[:-1])
    snap = _snapshot(kv)
    host = HostModel(w)
    hkv = HostKV.from_device(cfg, kv)
    ids, margins = [], []
    tok = prompt[-1]
    for i in range(GREEDY):
        logits, _ = host.step(hkv, tok, PROMPT - 1 + i, want_trace=False)
        tok = oracle.argmax_bf16(logits)
        ids.append(tok)
        margins.append(_margin(logits))
    yield dict(cfg=cfg, w=w, kv=kv, sess=sess, snap=snap, hkv=hkv, prompt=prompt, ids=ids, margins=margins)
    del host, hkv


@pytest.mark.parametrize("schedule", SCHEDULES)
def test_config3_greedy_bitexact(config3, schedule, monkeypatch):
    monkeypatch.setenv("REC_SCHEDULE", schedule)
    d = config3
    _restore(d["kv"], d["snap"])
    sess = d["sess"]
    got = sess.greedy(d["prompt"][-1], PROMPT - 1, 33)
    got += sess.greedy(-1, PROMPT - 1 + 33, GREEDY - 33)  # continues from the device's token and position
    want = d["ids"]
    if got != want:
        i = next(j for j in range(min(len(got), len(want))) if got[j] != want[j]) if len(got) == len(want) else 0
        pytest.fail(f"{schedule}: first diverging greedy step {i} (position {PROMPT - 1 + i}): got {got[i]}, "
                    f"oracle {want[i]}, oracle top-1/top-2 logit margin {d['margins'][i]:.6g}")
    # the K/V rows the packets appended
    for li, (L, H) in enumerate(zip(d["kv"].layers, d["hkv"].layers)):
        for n in L:
            g = L[n][:, PROMPT - 1:PROMPT - 1 + GREEDY].contiguous()
            g = g.view(torch.int16).cpu().numpy().view(np.uint16) if g.dtype == torch.bfloat16 else \
                g.cpu().numpy().view(np.uint32)
            assert np.array_equal(g, H[n][:, PROMPT - 1:PROMPT - 1 + GREEDY]), (schedule, li, n)


@pytest.mark.parametrize("schedule", SCHEDULES)
def test_config1_layer_steps_bitexact(cuda, schedule, monkeypatch):
    """Config 1: one decoder layer (64 experts top-8, I 768) over a
    1,024-token 8-bit cache of quantized K, V ~ N(0, 1), three steps."""
    monkeypatch.setenv("REC_SCHEDULE", schedule)
    cfg = CONFIG1_LAYER
    ctx = 1024
    w = generate_weights(cfg, seed=0, device="cuda")
    kv = KVCache.allocate(cfg, 1280)
    kv.fill_random(ctx, seed=7)
    sess = DecodeSession(w, kv)
    host = HostModel(w)
    hkv = HostKV.from_device(cfg, kv)
    for i in range(3):
        logits, trace = sess.step(11 + 7 * i, ctx + i, want_trace=True)
        sess.check_status()
        ref_logits, ref_trace = host.step(hkv, 11 + 7 * i, ctx + i)
        assert np.array_equal(_u16(trace), ref_trace), (schedule, i)
        assert np.array_equal(_u16(logits), ref_logits), (schedule, i)


CONFIG4_CONTEXT = 258048


@pytest.fixture(scope="module")
def config4(cuda):
    cfg = CONFIG4
    cap = (CONFIG4_CONTEXT + 8 + 255) // 256 * 256
    w = generate_weights(cfg, seed=0, device="cuda")
    kv = KVCache.allocate(cfg, cap)
    kv.fill_random(CONFIG4_CONTEXT, seed=2)
    snap_rows = slice(CONFIG4_CONTEXT, CONFIG4_CONTEXT + 8)
    sess = DecodeSession(w, kv)
    host = HostModel(w)
    hkv = HostKV.from_device(cfg, kv)
    ref = []
    for i in range(4):
        logits, trace = host.step(hkv, 1000 + i, CONFIG4_CONTEXT + i)
        ref.append((logits, trace))
    yield dict(cfg=cfg, kv=kv, sess=sess, ref=ref, rows=snap_rows)
    del host, hkv


@pytest.mark.parametrize("schedule", ["auto", "mega"])
def test_config4_258k_steps_bitexact(config4, schedule, monkeypatch):
    """Four decode steps of the 48-layer model at 258,048 tokens (4-bit
    cache), against the oracle, logits and trace."""
    from rec_b200._lib import lib

    if schedule == "auto":
        monkeypatch.delenv("REC_SCHEDULE", raising=False)
        assert lib().rec_schedule_for(config4["sess"].ctx, CONFIG4_CONTEXT) == 1  # the graph schedule
    else:
        monkeypatch.setenv("REC_SCHEDULE", schedule)
    sess = config4["sess"]
    for i in range(4):
        logits, trace = sess.step(1000 + i, CONFIG4_CONTEXT + i, want_trace=True)
        sess.check_status()
        ref_logits, ref_trace = config4["ref"][i]
        assert np.array_equal(_u16(trace), ref_trace), (schedule, i)
        assert np.array_equal(_u16(logits), ref_logits), (schedule, i)
