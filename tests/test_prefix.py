"""Prompt-prefix reuse (reference prefix.py:10-118, quantized.py:102-148):
the selection rules on the host (CPU), and a reused prefill whose logits and
next greedy tokens equal a fresh prefill's bit for bit (GPU)."""
import pytest
import torch

from rec_b200.prefix import Checkpoint, PromptCache, select_prefix


def _cache(n, checkpoints):
    return PromptCache(list(range(n)), storage="kv", logits=f"logits@{n}",
                       checkpoints=[Checkpoint(p, f"logits@{p}") for p in checkpoints])


def test_select_prefix_extends_whole_cache():
    c = _cache(40, [16, 32])
    got, common = select_prefix(c, list(range(40)) + [7, 8])
    assert got is c and common == 40 and len(got.tokens) == 40 and got.logits == "logits@40"


def test_select_prefix_rolls_back_to_checkpoint():
    c = _cache(40, [16, 32])
    got, common = select_prefix(c, list(range(37)) + [999, 1000])
    assert common == 37 and got is c
    assert got.tokens == list(range(32)) and got.logits == "logits@32"
    assert [k.position for k in got.checkpoints] == [16]


def test_select_prefix_exact_checkpoint_and_shorter_prompt():
    c = _cache(40, [16, 32])
    got, common = select_prefix(c, list(range(32)))
    assert common == 32 and got.tokens == list(range(32)) and got.logits == "logits@32"


def test_select_prefix_drops_cache_without_checkpoint():
    c = _cache(40, [16, 32])
    got, common = select_prefix(c, [5, 6, 7])
    assert got is None and common == 0
    got, common = select_prefix(_cache(40, [16, 32]), list(range(10)) + [77])
    assert got is None and common == 10
    assert select_prefix(None, [1, 2]) == (None, 0)


def test_checkpoint_keeps_two():
    c = PromptCache([], storage=None)
    c.checkpoint()
    assert c.checkpoints == []
    for n in (4, 8, 12):
        c.advance(range(n - len(c.tokens)), f"l{n}")
        c.checkpoint()
    assert [k.position for k in c.checkpoints] == [8, 12]
    f = c.fork()
    f.tokens.append(1)
    assert len(c.tokens) == 12 and f.storage is c.storage



def test_layers_sum_sliding_bytes_as_the_reference_engine():
    """engine.py:323-329 sums `cache.nbytes` over the prompt cache's layers
    whose metadata row has column 1 clear (the sliding-window layers)."""
    from types import SimpleNamespace

    from rec_b200.engine import layer_metadata
    from rec_b200.model import TINY_FLINT

    layers = [{"k_codes": torch.zeros(4, 16 * (i + 1), dtype=torch.int32),
               "k_scales": torch.zeros(4, 2, dtype=torch.bfloat16)} for i in range(TINY_FLINT.n_layers)]
    c = PromptCache([1, 2], storage=SimpleNamespace(cache=SimpleNamespace(layers=layers)))
    sliding = sum(cache.nbytes for row, cache in zip(layer_metadata(TINY_FLINT)[:3], c.layers, strict=True)
                  if not row[1])
    assert [L.nbytes for L in c.layers] == [4 * 16 * 4 + 16, 4 * 32 * 4 + 16, 4 * 48 * 4 + 16]
    assert sliding == c.layers[0].nbytes + c.layers[2].nbytes  # TINY_FLINT's sliding layers are 0 and 2


@pytest.mark.gpu
def test_gpu_prefill_with_prefix_bitexact(cuda):
    from rec_b200.engine import build_decoder
    from rec_b200.model import TINY, generate_weights

    w = generate_weights(TINY, seed=13, device="cuda")
    g = torch.Generator().manual_seed(2)
    a = torch.randint(0, TINY.vocab, (40,), generator=g).tolist()
    b = a[:37] + torch.randint(0, TINY.vocab, (9,), generator=g).tolist()
    ext = b + torch.randint(0, TINY.vocab, (5,), generator=g).tolist()

    def fresh(tokens):
        engine, sampler = build_decoder(w)
        engine.prefill_chunk_size = 16
        s = engine.make_session(max_new_tokens=16)
        logits = s.prefill(tokens)
        nxt = sampler.block(s._state, int(torch.argmax(logits.float())), 4, 0, temperature=0.0)
        return logits, nxt

    engine, sampler = build_decoder(w)
    engine.prefill_chunk_size = 16
    first = engine.make_session(max_new_tokens=16)
    first.prefill(a)
    assert [c.position for c in first.prompt_cache.checkpoints] == [16, 32]
    sampler.block(first._state, 3, 4, 0, temperature=0.0)  # decode writes past the prompt
    cache = first.prompt_cache
    for prompt, cached in ((b, 32), (ext, 46)):  # roll back to a checkpoint, then extend a whole cache
        s = engine.make_session(max_new_tokens=16)
        logits = s.prefill(prompt, prefix=cache)
        assert s.cached_tokens == cached
        cache = s.prompt_cache
        nxt = sampler.block(s._state, int(torch.argmax(logits.float())), 4, 0, temperature=0.0)
        want_logits, want_next = fresh(prompt)
        assert torch.equal(logits.view(torch.int16), want_logits.view(torch.int16))
        assert nxt == want_next


class _FakeSession:
    """Stands in for the device session: a chunk's 'logits' are its last
    token, and every call is recorded."""

    def __init__(self):
        self.calls = []

    def prefill_chunk(self, part, begin, want_logits=True, layers=None):
        self.calls.append((tuple(part), begin, layers, want_logits))
        return torch.tensor([float(part[-1])])

    def check_status(self):
        pass


def _fake_engine(n_layers=3, chunk=2):
    from types import SimpleNamespace

    sess = _FakeSession()
    storage = SimpleNamespace(capacity=64)
    engine = SimpleNamespace(
        prefill_chunk_size=chunk, cfg=SimpleNamespace(has_layer_options=False, n_layers=n_layers),
        model=SimpleNamespace(context_limit=32), _session=lambda state: sess, _guard=lambda state, fn: fn(),
        prefill_state=lambda capacity, limit=None, storage=None, _kv=storage: {"kv": _kv})
    return engine, sess


def test_cancelled_prefill_keeps_the_last_completed_chunk():
    """The reference's test_prefix_rollback.py:65-85 on this QATSession: a
    stop before the second chunk leaves the first chunk's tokens and logits
    in the prompt cache, which a later prompt reuses."""
    from rec_b200.engine import QATSession
    from rec_b200.errors import PrefillCancelled

    engine, sess = _fake_engine()
    session = QATSession(engine, 1)
    checks = iter([False, True])
    with pytest.raises(PrefillCancelled):
        session.prefill([1, 2, 3, 4], should_stop=lambda: next(checks))
    assert session.prompt_cache.tokens == [1, 2] and session.prompt_cache.logits.item() == 2
    restored, common = select_prefix(session.prompt_cache, [1, 2, 5])
    assert common == 2 and restored is session.prompt_cache
    assert sess.calls == [((1, 2), 0, None, True)]


def test_interrupt_between_layers_polls_before_each_layer():
    """interrupt_between_layers (quantized.py:129-133, model.py:309-314):
    each chunk runs as one call per layer, the logits with the last layer; a
    stop before a later layer of the first chunk cancels with no chunk
    completed."""
    from rec_b200.engine import QATSession
    from rec_b200.errors import PrefillCancelled

    engine, sess = _fake_engine(n_layers=3)
    logits = QATSession(engine, 1).prefill([1, 2, 3], interrupt_between_layers=True)
    assert logits.item() == 3
    assert sess.calls == [((1, 2), 0, (0, 1), False), ((1, 2), 0, (1, 2), False), ((1, 2), 0, (2, 3), True),
                          ((3,), 2, (0, 1), False), ((3,), 2, (1, 2), False), ((3,), 2, (2, 3), True)]
    engine, sess = _fake_engine(n_layers=3)
    polls = []
    session = QATSession(engine, 1)
    with pytest.raises(PrefillCancelled):
        session.prefill([1, 2, 3], should_stop=lambda: polls.append(1) or len(polls) == 3,
                        interrupt_between_layers=True)
    assert [c[2] for c in sess.calls] == [(0, 1), (1, 2)] and session.prompt_cache.tokens == []
