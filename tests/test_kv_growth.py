"""KV growth without copying (reference cache.py:47-84 appends 65,536-token
bank blocks): the codes are reserved in virtual memory for the state's limit
and backed in 32,768-token blocks (rec_b200.vmm).  A growth keeps every row already
written in place, the session and its device pointers stay the same, and
decoding across the block boundary stays bit-exact against the oracle."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _u32(t):
    return t.contiguous().cpu().numpy().view(np.uint32)


def test_reserved_codes_grow_in_place(cuda):
    from rec_b200.vmm import BLOCK_TOKENS, ReservedCodes

    rc = ReservedCodes(4, 3 * BLOCK_TOKENS, 32, cuda)
    rc.grow(1000)
    assert rc.rows == BLOCK_TOKENS
    v = rc.view()
    assert v.shape == (4, BLOCK_TOKENS, 32) and v.stride(0) == 3 * BLOCK_TOKENS * 32
    g = torch.Generator(device=cuda).manual_seed(3)
    pattern = torch.randint(-2**31, 2**31 - 1, (4, BLOCK_TOKENS, 32), generator=g, device=cuda, dtype=torch.int32)
    v.copy_(pattern)
    base = v.data_ptr()
    rc.grow(2 * BLOCK_TOKENS + 5)
    w = rc.view()
    assert w.shape[1] == 3 * BLOCK_TOKENS and w.data_ptr() == base
    assert torch.equal(w[:, :BLOCK_TOKENS], pattern)
    w[:, BLOCK_TOKENS:].fill_(7)  # every backed row of every head is writable
    assert int((w[:, BLOCK_TOKENS:] == 7).sum().item()) == 4 * 2 * BLOCK_TOKENS * 32
    torch.cuda.synchronize()
    with pytest.raises(ValueError):
        rc.grow(3 * BLOCK_TOKENS + 1)
    rc.release()


def test_engine_growth_across_a_block_is_bitexact(cuda):
    from oracle.host import HostKV, HostModel
    from rec_b200.engine import FullModel
    from rec_b200.model import TINY, generate_weights
    from rec_b200.vmm import BLOCK_TOKENS

    cfg = TINY
    w = generate_weights(cfg, seed=17, device="cuda")
    engine = FullModel(w)
    state = engine.prefill_state(256, limit=2 * BLOCK_TOKENS + 100)
    storage = state["kv"]
    assert state["capacity"] == BLOCK_TOKENS
    start = BLOCK_TOKENS - 3
    storage.cache.fill_random(start, seed=5)
    sess = storage.session
    ptrs = [L["k_codes"].data_ptr() for L in storage.cache.layers]
    host = HostModel(w)
    hkv = HostKV.from_device(cfg, storage.cache)
    state["position"] = start
    u16 = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    for i in range(6):
        logits, trace = engine.forward(state, 100 + i)
        ref_logits, ref_trace = host.step(hkv, 100 + i, start + i)
        assert np.array_equal(u16(trace), ref_trace), i
        assert np.array_equal(u16(logits), ref_logits), i
    assert state["growth_count"] == 1 and state["capacity"] == 2 * BLOCK_TOKENS
    assert storage.session is sess
    assert [L["k_codes"].data_ptr() for L in storage.cache.layers] == ptrs
    # the rows decoded after the growth are the oracle's
    for li, (L, H) in enumerate(zip(storage.cache.layers, hkv.layers)):
        assert np.array_equal(_u32(L["k_codes"][:, start:start + 6]), H["k_codes"][:, start:start + 6]), li
        assert np.array_equal(_u32(L["v_codes"][:, start:start + 6]), H["v_codes"][:, start:start + 6]), li
    # past the reservation: one move into a larger reservation, still exact
    state["limit"] = 3 * BLOCK_TOKENS
    engine.ensure_capacity(state, 2 * BLOCK_TOKENS - state["position"] + 10)
    assert state["growth_count"] == 2 and state["capacity"] == 3 * BLOCK_TOKENS
    logits, trace = engine.forward(state, 7)
    ref_logits, ref_trace = host.step(hkv, 7, start + 6)
    assert np.array_equal(u16(logits), ref_logits)
