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
