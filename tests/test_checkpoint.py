"""rec_b200.checkpoint.load_reference_checkpoint on CPU: a checkpoint written
under the reference's tensor names (its module paths, model.py:140-327;
experts stacked [E, N, K/8]; codes as 32-bit words or their bytes; router
and sinks in float32, as MLX keeps them) loads back into exactly the codes,
scales, biases and vectors it was written from."""
import json

import numpy as np
import pytest
import torch

from golden import cases
from rec_b200 import abi
from rec_b200.checkpoint import load_reference_checkpoint


def _i32(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32))


def _bf(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.int16)).view(torch.bfloat16)


def _write(m, cfg, directory, byte_codes: bool):
    t = {}

    def q(prefix, qt, stacked=0):
        w, s, b = qt.w, qt.s, qt.b
        if stacked:
            w, s, b = (x.reshape(stacked, x.shape[0] // stacked, x.shape[1]) for x in (w, s, b))
        t[prefix + ".weight"] = (torch.from_numpy(np.ascontiguousarray(w).view(np.uint8)) if byte_codes
                                 else _i32(w))
        t[prefix + ".scales"] = _bf(s) if cfg.scale_dtype == torch.bfloat16 else torch.from_numpy(s.view(np.float16))
        t[prefix + ".biases"] = _bf(b) if cfg.scale_dtype == torch.bfloat16 else torch.from_numpy(b.view(np.float16))

    for i, L in enumerate(m.layers):
        p, a, mm = f"model.layers.{i}.", f"model.layers.{i}.self_attn.", f"model.layers.{i}.mlp."
        t[p + "input_layernorm.weight"] = _bf(L.input_norm)
        t[p + "post_attention_layernorm.weight"] = _bf(L.post_norm)
        for n in "qkvo":
            q(a + f"{n}_proj", getattr(L, n))
        t[a + "q_norm.weight"] = _bf(L.q_norm)
        t[a + "k_norm.weight"] = _bf(L.k_norm)
        t[a + "softmax_offset"] = _bf(L.sinks).float()
        if L.kind & abi.REC_LAYER_DENSE:
            q(mm + "gate_proj", L.gate)
            q(mm + "up_proj", L.up)
            q(mm + "down_proj", L.down)
        else:
            t[mm + "gate.weight"] = _bf(L.router).float()
            t[mm + "gate.expert_bias"] = torch.from_numpy(L.expert_bias)
            q(mm + "switch_mlp.gate_proj", L.gate, cfg.n_experts)
            q(mm + "switch_mlp.up_proj", L.up, cfg.n_experts)
            q(mm + "switch_mlp.down_proj", L.down, cfg.n_experts)
            q(mm + "shared_expert.gate_proj", L.shared_gate)
            q(mm + "shared_expert.up_proj", L.shared_up)
            q(mm + "shared_expert.down_proj", L.shared_down)
    q("model.embed_tokens", m.embed)
    t["model.norm.weight"] = _bf(m.final_norm)
    q("lm_head", m.lm_head)
    from safetensors.torch import save_file

    names = sorted(t)
    half = len(names) // 2  # two shards
    save_file({n: t[n].contiguous() for n in names[:half]}, str(directory / "model-00001-of-00002.safetensors"))
    save_file({n: t[n].contiguous() for n in names[half:]}, str(directory / "model-00002-of-00002.safetensors"))
    (directory / "config.json").write_text(json.dumps({"model_type": "flint", "eos_token_id": 3}))


def _u16(x):
    return x.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("byte_codes", [False, True])
def test_checkpoint_round_trip(tmp_path, byte_codes):
    cfg, seed = cases.DECODE_CASES["decode_flint"]
    m = cases.host_model(cfg, seed)
    _write(m, cfg, tmp_path, byte_codes)
    w = load_reference_checkpoint(tmp_path, cfg, device="cpu")

    def same_q(got, want):
        assert np.array_equal(got.w.numpy().view(np.uint32), want.w)
        assert np.array_equal(_u16(got.s), want.s) and np.array_equal(_u16(got.b), want.b)

    for L, H in zip(w.layers, m.layers):
        assert L.kind == H.kind
        for n in ("q", "k", "v", "o", "gate", "up", "down"):
            same_q(getattr(L, n), getattr(H, n))
        for n in ("input_norm", "post_norm", "q_norm", "k_norm", "sinks"):
            assert np.array_equal(_u16(getattr(L, n)), getattr(H, n)), n
        if not H.kind & abi.REC_LAYER_DENSE:
            assert np.array_equal(_u16(L.router), H.router)
            assert np.array_equal(L.expert_bias.numpy(), H.expert_bias)
            for n in ("shared_gate", "shared_up", "shared_down"):
                same_q(getattr(L, n), getattr(H, n))
        else:
            assert L.router is None
    same_q(w.embed, m.embed)
    same_q(w.lm_head, m.lm_head)
    assert np.array_equal(_u16(w.final_norm), m.final_norm)
    assert w.eos_tokens == (3,)  # config.json's eos_token_id, an id or a list (quantized.py:77)


def test_checkpoint_missing_tensor_is_named(tmp_path):
    cfg, seed = cases.DECODE_CASES["decode_flint"]
    m = cases.host_model(cfg, seed)
    _write(m, cfg, tmp_path, False)
    from safetensors.torch import load_file, save_file

    shard = tmp_path / "model-00002-of-00002.safetensors"
    t = load_file(str(shard))
    gone = sorted(t)[0]
    del t[gone]
    save_file(t, str(shard))
    with pytest.raises(KeyError, match=gone.replace(".", r"\.")):
        load_reference_checkpoint(tmp_path, cfg, device="cpu")


def test_checkpoint_extra_tensor_is_refused(tmp_path):
    cfg, seed = cases.DECODE_CASES["decode_flint"]
    m = cases.host_model(cfg, seed)
    _write(m, cfg, tmp_path, False)
    from safetensors.torch import load_file, save_file

    shard = tmp_path / "model-00001-of-00002.safetensors"
    t = load_file(str(shard))
    t["model.layers.0.mlp.unexpected.weight"] = torch.zeros(4)
    save_file(t, str(shard))
    with pytest.raises(ValueError, match="not part of the model"):
        load_reference_checkpoint(tmp_path, cfg, device="cpu")


@pytest.mark.gpu
def test_gpu_checkpoint_decodes_the_golden_case(cuda, tmp_path):
    """The golden Flint case written as a reference checkpoint, loaded onto
    the device and decoded through the C ABI, reproduces the frozen fixture."""
    import oracle
    from oracle.host import HostKV
    from rec_b200.model import KVCache
    from rec_b200.session import DecodeSession

    cfg, seed = cases.DECODE_CASES["decode_flint"]
    want = cases.load("decode_flint")
    m = cases.host_model(cfg, seed)
    _write(m, cfg, tmp_path, True)
    weights = load_reference_checkpoint(tmp_path, cfg, device="cuda")
    hkv = HostKV(cfg, cases.CAPACITY)
    cases.fill_kv(hkv, cfg, seed + 1)
    kv = KVCache.allocate(cfg, cases.CAPACITY)
    for d, h in zip(kv.layers, hkv.layers):
        for n in d:
            d[n].copy_(torch.from_numpy(h[n].view(np.int32) if h[n].dtype == np.uint32 else h[n].view(np.int16))
                       .to("cuda").view(d[n].dtype))
    sess = DecodeSession(weights, kv)
    token, ids = cases.START_TOKEN, []
    for i in range(cases.STEPS):
        logits, _ = sess.step(token, cases.CONTEXT + i)
        lg = _u16(logits.cpu())
        assert cases.sha(lg) == str(want["logits_sha"][i]), f"step {i}"
        token = oracle.argmax_bf16(lg)
        ids.append(token)
    sess.check_status()
    assert ids == want["ids"].tolist()


def test_checkpoint_config_json_gives_the_model(tmp_path):
    """Without an explicit ModelConfig the loader reads config.json (the
    reference's ModelArgs keys, kv_format "native": MLX's quantized cache)
    and arrives at the golden Flint case's configuration."""
    from dataclasses import replace

    cfg, seed = cases.DECODE_CASES["decode_flint"]
    m = cases.host_model(cfg, seed)
    _write(m, cfg, tmp_path, False)
    (tmp_path / "config.json").write_text(json.dumps({
        "model_type": "flint", "hidden_size": cfg.hidden, "num_hidden_layers": cfg.n_layers,
        "num_attention_heads": cfg.n_q_heads, "num_key_value_heads": cfg.n_kv_heads, "head_dim": cfg.head_dim,
        "num_experts": cfg.n_experts, "num_experts_per_tok": cfg.top_k, "moe_intermediate_size": cfg.moe_inter,
        "shared_expert_intermediate_size": cfg.shared_inter, "intermediate_size": cfg.dense_inter,
        "mlp_only_layers": list(cfg.dense_layers), "no_rope_layer_indices": list(cfg.no_rope_layers),
        "layer_types": ["sliding_attention" if i in cfg.sliding_layers else "full_attention"
                        for i in range(cfg.n_layers)],
        "sliding_window": cfg.sliding_window, "vocab_size": cfg.vocab, "rms_norm_eps": cfg.rms_eps,
        "rope_theta": cfg.rope_theta, "kv_key_bits": cfg.kv_bits, "kv_value_bits": cfg.kv_bits,
        "kv_group_size": 64, "tie_word_embeddings": False, "quantization": {"group_size": 64, "bits": 4},
        "mlx_export": {"bits": 4, "routed_expert_bits": 4, "embedding_bits": cfg.embed_bits},
        "eos_token_id": [5, 7]}))
    w = load_reference_checkpoint(tmp_path, kv_format="native", device="cpu")
    assert replace(w.cfg, name=cfg.name) == cfg
    assert w.eos_tokens == (5, 7) and w.context_limit == 262144
