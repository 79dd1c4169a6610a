"""Sampling head on the GPU: penalties, temperature, top-k / top-p with
injected uniforms (reference engine.py:279-301, masked_sampling.py:98-125,
filtered_sampling.py:7-22, sampling.py:48-52).

The uniforms are drawn on the device from torch's Philox generator, one per
vocabulary entry per token (the Gumbel noise of the reference's categorical
draw is -log(-log u)); passing the same uniforms to the oracle reproduces the
ids bit for bit.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import abi
from ._lib import check, lib


def params(temperature=0.0, top_k=0, top_p=1.0, repetition_penalty=1.0, presence_penalty=0.0) -> abi.RecSampling:
    return abi.RecSampling(float(temperature), int(top_k), float(top_p), float(repetition_penalty),
                           float(presence_penalty))


def uniforms(batch: int, vocab: int, seed: int, device) -> torch.Tensor:
    """fp32 [batch, vocab] in [0, 1) from a seeded Philox stream on `device`."""
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return torch.rand(batch, vocab, generator=g, device=device, dtype=torch.float32)


def sample_logits(logits: torch.Tensor, p: abi.RecSampling, u: torch.Tensor | None = None,
                  history: torch.Tensor | None = None, out: torch.Tensor | None = None,
                  allow: torch.Tensor | None = None) -> torch.Tensor:
    """ids int32 [B] for bf16 logits [B, V] (or [V]); history int32 [B, n]
    (or [n]); u fp32 [B, V] (required when temperature > 0); allow an
    optional grammar mask, int32/uint32 words [B, W] (or [W]) with
    W >= ceil(V / 32), bit i & 31 of word i >> 5 set for each allowed id
    (rec_sample_logits_masked; a row with no allowed id gives -1)."""
    if logits.dtype != torch.bfloat16 or not logits.is_cuda:
        raise ValueError("logits must be a bf16 CUDA tensor")
    lg = logits.reshape(1, -1) if logits.dim() == 1 else logits
    B, V = lg.shape
    if lg.stride(1) != 1:
        raise ValueError("logits rows must be contiguous")
    if history is not None:
        history = history.reshape(B, -1) if history.dim() == 1 else history
        history = history.to(torch.int32).contiguous()
    if u is not None:
        u = u.reshape(B, V).contiguous()
        if u.dtype != torch.float32:
            raise ValueError("uniforms must be float32")
    if allow is not None:
        allow = allow.reshape(B, -1) if allow.dim() == 1 else allow
        if allow.element_size() != 4 or allow.device != lg.device or allow.stride(1) != 1:
            raise ValueError("allow must be 32-bit words on the logits' device, rows contiguous")
        if allow.shape[1] < (V + 31) // 32:
            raise ValueError("allow rows must hold ceil(V / 32) words")
    ids = out if out is not None else torch.empty(B, dtype=torch.int32, device=lg.device)
    stream = torch.cuda.current_stream().cuda_stream
    check(lib().rec_sample_logits_masked(C.c_void_p(lg.data_ptr()), B, V, lg.stride(0),
                                         C.c_void_p(history.data_ptr()) if history is not None else None,
                                         history.shape[1] if history is not None else 0, C.byref(p),
                                         C.c_void_p(u.data_ptr()) if u is not None else None,
                                         C.c_void_p(allow.data_ptr()) if allow is not None else None,
                                         allow.stride(0) if allow is not None else 0, C.c_void_p(ids.data_ptr()),
                                         C.c_void_p(stream)), "rec_sample_logits_masked")
    return ids


def sample_head(h: torch.Tensor, final_norm: torch.Tensor, lm_head, scale_dtype: torch.dtype, p: abi.RecSampling,
                u: torch.Tensor | None = None, history: torch.Tensor | None = None, eps: float = 1e-6):
    """Final RMSNorm + int4 lm_head GEMV + sampler for B hidden rows
    (config 5) through rec_lmhead_sample.  Returns (ids int32 [B], logits
    bf16 [B, V])."""
    from .ops import scale_dtype_code

    hb = h.reshape(-1, h.shape[-1]).contiguous()
    B, H = hb.shape
    V = lm_head.w.shape[0]
    logits = torch.empty(B, V, dtype=torch.bfloat16, device=h.device)
    ids = torch.empty(B, dtype=torch.int32, device=h.device)
    m = abi.RecQMat(lm_head.w.data_ptr(), lm_head.s.data_ptr(), lm_head.b.data_ptr())
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    hist = None
    hist_len = 0
    if history is not None and history.numel():
        hist = history.to(torch.int32).reshape(B, -1).contiguous()
        hist_len = hist.shape[1]
    if p.temperature > 0 and u is None:
        raise ValueError("temperature > 0 needs uniforms")
    uu = None if u is None else u.to(torch.float32).reshape(B, -1).contiguous()
    check(lib().rec_lmhead_sample(C.byref(m), scale_dtype_code(scale_dtype), V, H, C.c_void_p(hb.data_ptr()), B,
                                  C.c_void_p(final_norm.data_ptr()), float(eps),
                                  C.c_void_p(hist.data_ptr()) if hist is not None else None, hist_len, C.byref(p),
                                  C.c_void_p(uu.data_ptr()) if uu is not None else None,
                                  C.c_void_p(logits.data_ptr()), C.c_void_p(ids.data_ptr()), stream),
          "rec_lmhead_sample")
    return ids, logits


def sampled_block(engine, state, token, count, seed, *, temperature, top_p, top_k, presence_penalty, eos=()):
    """ResidentSampler.block for temperature > 0 through rec_decode_sampled:
    the packet decodes and samples on the device with the step's uniforms,
    feeding each id back without a host round trip.  state["presence_mask"]
    (float [V], the reference's key) marks the ids the presence penalty
    applies to; the packet's ids are added to it afterwards."""
    sess = engine._session(state)
    V = engine.weights.cfg.vocab
    dev = sess.logits.device
    p = params(temperature, top_k, top_p, 1.0, presence_penalty)
    u = uniforms(count, V, seed, dev).contiguous()
    mask = state.get("presence_mask")
    if presence_penalty and mask is None:
        mask = torch.zeros(V, dtype=torch.float32, device=dev)
        state["presence_mask"] = mask
    hist = hist_len = None
    cap = 0
    if presence_penalty:
        seen = torch.nonzero(mask).to(torch.int32).reshape(-1)
        cap = int(seen.numel()) + count
        hist = torch.zeros(cap, dtype=torch.int32, device=dev)
        hist[: seen.numel()] = seen
        hist_len = torch.tensor([seen.numel()], dtype=torch.int32, device=dev)
    eos_ids = list(eos)[:8]
    eos_arr = (C.c_int32 * max(1, len(eos_ids)))(*eos_ids) if eos_ids else None
    ids_dev = torch.zeros(count, dtype=torch.int32, device=dev)
    produced = torch.zeros(1, dtype=torch.int32, device=dev)
    pos = state["position"]

    def run():
        stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        check(lib().rec_decode_sampled(sess.ctx, int(token), pos, count, C.byref(p), C.c_void_p(u.data_ptr()),
                                       C.c_void_p(hist.data_ptr()) if hist is not None else None,
                                       C.c_void_p(hist_len.data_ptr()) if hist_len is not None else None, cap,
                                       eos_arr, len(eos_ids), C.c_void_p(ids_dev.data_ptr()),
                                       C.c_void_p(produced.data_ptr()), stream), "rec_decode_sampled")
        sess.check_status()
        n = int(produced.item())
        ids = ids_dev[:n].tolist()
        if any(t < 0 for t in ids):
            raise RuntimeError("Invalid sampled chain")
        if presence_penalty and ids:
            mask[torch.tensor(ids, dtype=torch.long, device=dev)] = 1.0
        return ids

    return engine._guard(state, run)


def _grammar_words(mask, words: int, device) -> torch.Tensor | None:
    """The allow words of a grammar mask (uint32 words + a trailing active
    flag word, the reference's state["grammar_mask"], grammar.py:86-88), as
    int32 [words] on `device`; None when the flag word is 0 (inactive).  Ids
    past the grammar's words are not allowed."""
    m = torch.as_tensor(np.asarray(mask, dtype=np.uint32).view(np.int32))
    if m.numel() < 2:
        raise ValueError("grammar_mask must hold the allow words and the active flag word")
    if int(m[-1]) == 0:
        return None
    out = torch.zeros(words, dtype=torch.int32)
    n = min(words, m.numel() - 1)
    out[:n] = m[:n]
    return out.to(device)


def token_logprob(logits: torch.Tensor, p: abi.RecSampling, ids: torch.Tensor, history: torch.Tensor | None = None,
                  allow: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """The reference's reported log-probability of each row's id
    (rec_token_logprob): report = penalised, grammar-masked logits / T (or
    the logits at T = 0); report[id] - logsumexp(report), fp32 [B]."""
    lg = logits.reshape(1, -1) if logits.dim() == 1 else logits
    B, V = lg.shape
    if history is not None:
        history = history.reshape(B, -1) if history.dim() == 1 else history
        history = history.to(torch.int32).contiguous()
    if allow is not None:
        allow = allow.reshape(B, -1) if allow.dim() == 1 else allow
    res = out if out is not None else torch.empty(B, dtype=torch.float32, device=lg.device)
    stream = torch.cuda.current_stream().cuda_stream
    check(lib().rec_token_logprob(C.c_void_p(lg.data_ptr()), B, V, lg.stride(0),
                                  C.c_void_p(history.data_ptr()) if history is not None else None,
                                  history.shape[1] if history is not None else 0, C.byref(p),
                                  C.c_void_p(allow.data_ptr()) if allow is not None else None,
                                  allow.stride(0) if allow is not None else 0, C.c_void_p(ids.data_ptr()),
                                  C.c_void_p(res.data_ptr()), C.c_void_p(stream)), "rec_token_logprob")
    return res


def filtered_block(engine, state, token, count, seed, *, temperature, top_p, top_k, presence_penalty, grammar=None,
                   logprobs=None, eos=()):
    """ResidentSampler.block on the reference's filtered path
    (kernels/sampling.py:80-96 -> masked_sampling.py:33-212): taken with a
    grammar, with logprobs, or with a presence penalty at temperature 0.
    Every step decodes one token, applies the presence penalty (ids sampled
    so far, state["presence_mask"]) and the grammar's allow words, samples on
    the device (greedy at temperature 0; otherwise the step's row of the
    seeded uniforms, the same draws as the device-side sampled packet), and,
    when `logprobs` is a list, appends report[id] - logsumexp(report) with
    report = the masked, penalised logits / T.  With a grammar the id goes to
    its host matcher (grammar._advance), whose result is the next step's mask
    (state["grammar_mask"]), and the packet stops after one of grammar.stops;
    without one it stops after an EOS id.  One host round trip per token."""
    sess = engine._session(state)
    V = engine.weights.cfg.vocab
    dev = sess.logits.device
    words = (V + 31) // 32
    p = params(temperature, top_k, top_p, 1.0, presence_penalty)
    u = uniforms(count, V, seed, dev) if temperature > 0 else None
    mask = state.get("presence_mask")
    if presence_penalty and mask is None:
        mask = torch.zeros(V, dtype=torch.float32, device=dev)
        state["presence_mask"] = mask
    stops = set(int(t) for t in (getattr(grammar, "stops", ()) if grammar is not None else eos))
    ids_dev = torch.zeros(1, dtype=torch.int32, device=dev)
    lp_dev = torch.zeros(1, dtype=torch.float32, device=dev)
    pos = state["position"]

    def run():
        out, lps = [], []
        tok = int(token)
        for i in range(count):
            allow = None
            if grammar is not None:
                allow = _grammar_words(state["grammar_mask"], words, dev)
                if allow is None:
                    break
            logits, _ = sess.step(tok, pos + i)
            hist = torch.nonzero(mask).to(torch.int32).reshape(1, -1) if presence_penalty else None
            sample_logits(logits.reshape(1, V), p, u[i] if u is not None else None, hist, out=ids_dev, allow=allow)
            if logprobs is not None:
                token_logprob(logits.reshape(1, V), p, ids_dev, hist, allow, out=lp_dev)
            sess.check_status()
            tok = int(ids_dev.item())
            if tok < 0:
                raise RuntimeError("Grammar allows no token" if grammar is not None else "Invalid sampled chain")
            out.append(tok)
            if logprobs is not None:
                lps.append(float(lp_dev.item()))
            if presence_penalty:
                mask[tok] = 1.0
            if grammar is not None:
                nxt = np.asarray(grammar._advance(tok, True), dtype=np.uint32)
                state["grammar_mask"] = np.concatenate([nxt, np.ones(1, np.uint32)])
            if tok in stops:
                break
        return out, lps

    ids, lps = engine._guard(state, run)
    if not ids:
        raise RuntimeError("Grammar session is inactive")
    if logprobs is not None:
        logprobs.extend(lps)
    return ids


def grammar_block(engine, state, token, count, seed, grammar, *, temperature, top_p, top_k, presence_penalty,
                  logprobs=None):
    """ResidentSampler.block with a grammar constraint (reference
    masked_sampling.py:33-212 with grammar.py:46-104): filtered_block with
    the grammar's allow words after the presence penalty.  The matcher runs
    on the CPU, so each token makes one host round trip (the reference orders
    its GPU work behind the same callback)."""
    return filtered_block(engine, state, token, count, seed, temperature=temperature, top_p=top_p, top_k=top_k,
                          presence_penalty=presence_penalty, grammar=grammar, logprobs=logprobs)
