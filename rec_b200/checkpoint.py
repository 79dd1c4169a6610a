"""Weights of a reference checkpoint (a directory of `config.json` and
`model-*.safetensors` shards, engine/src/rec_mlx/checkpoint.py:5-31) as a
ModelWeights for this library.

The tensor names are the reference model's module paths (model.py:140-327,
quantized.py:36-60): `model.embed_tokens`, `model.layers.{i}.self_attn.
{q,k,v,o}_proj`, `.q_norm`, `.k_norm`, `.softmax_offset` (the attention
sinks), `.input_layernorm`, `.post_attention_layernorm`, and either
`.mlp.{gate,up,down}_proj` (a dense MLP layer) or `.mlp.gate` (the router
and its `expert_bias`), `.mlp.switch_mlp.{gate,up,down}_proj` (the routed
experts, [E, N, K/8]) and `.mlp.shared_expert.{gate,up,down}_proj`;
`model.norm`, `lm_head`.  Each quantized matrix is `.weight` (uint32 codes,
or uint8 bytes of them, as the reference's `sanitize` accepts),
`.scales`, `.biases`.  Nothing is dequantized: the codes, scales and biases
are used as stored (the routed experts' [E, N, K/8] stacks become [E·N,
K/8]); the router is taken in bf16 and the sinks in bf16, as the
reference's decode kernel reads them (megakernel.py:406-419, quantized.py:57).
"""
from __future__ import annotations

import json
from pathlib import Path

import torch

from . import abi
from .model import LayerWeights, ModelConfig, ModelWeights, QTensor, config_from_reference


def _load_tensors(directory: Path) -> dict:
    from safetensors.torch import load_file

    shards = sorted(directory.glob("model-*.safetensors"))
    if not shards:
        raise FileNotFoundError(f"no model-*.safetensors in {directory}")
    tensors = {}
    for path in shards:
        part = load_file(str(path), device="cpu")
        dup = tensors.keys() & part.keys()
        if dup:
            raise ValueError(f"tensor {sorted(dup)[0]} appears in more than one shard")
        tensors.update(part)
    return tensors


def load_reference_checkpoint(directory, cfg: ModelConfig | None = None, *, kv_format: str = "bf16",
                              device="cuda") -> ModelWeights:
    """ModelWeights of the checkpoint in `directory` on `device`.  cfg
    defaults to config_from_reference(config.json, kv_format=...); the
    model's end ids are config.json's `eos_token_id` (an id or a list, as
    quantized.py:77 keeps them)."""
    directory = Path(directory)
    config_path = directory / "config.json"
    config = json.loads(config_path.read_text()) if cfg is None or config_path.exists() else {}
    if cfg is None:
        cfg = config_from_reference(config, kv_format=kv_format)
    t = _load_tensors(directory)
    dev = torch.device(device)
    used = set()

    def get(name):
        if name not in t:
            raise KeyError(f"checkpoint has no tensor {name}")
        used.add(name)
        return t[name]

    def codes(x):
        if x.dtype == torch.uint8:  # bytes of the uint32 words
            x = x.contiguous().view(torch.int32)
        elif x.dtype == torch.uint32:
            x = x.view(torch.int32)
        if x.dtype != torch.int32:
            raise ValueError(f"quantized codes must be 32-bit words, got {x.dtype}")
        return x

    def qmat(prefix, rows, cols, bits=4, stacked=0):
        w, s, b = codes(get(prefix + ".weight")), get(prefix + ".scales"), get(prefix + ".biases")
        if stacked:  # [E, N, K*bits/32] -> [E*N, K*bits/32]
            w, s, b = (x.reshape(stacked * x.shape[1], x.shape[2]) for x in (w, s, b))
        want = (rows, cols * bits // 32)
        if tuple(w.shape) != want or tuple(s.shape) != (rows, cols // 64) or tuple(b.shape) != (rows, cols // 64):
            raise ValueError(f"{prefix}: shapes {tuple(w.shape)}, {tuple(s.shape)}; expected {want}, "
                             f"({rows}, {cols // 64})")
        return QTensor(w.contiguous().to(dev), s.to(cfg.scale_dtype).contiguous().to(dev),
                       b.to(cfg.scale_dtype).contiguous().to(dev))

    def vec(name, dtype=torch.bfloat16):
        return get(name).to(dtype).contiguous().to(dev)

    H, d = cfg.hidden, cfg.head_dim
    layers = []
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}."
        a = p + "self_attn."
        kind = cfg.layer_kind(i)
        common = dict(input_norm=vec(p + "input_layernorm.weight"), post_norm=vec(p + "post_attention_layernorm.weight"),
                      q=qmat(a + "q_proj", cfg.n_q_heads * d, H), k=qmat(a + "k_proj", cfg.n_kv_heads * d, H),
                      v=qmat(a + "v_proj", cfg.n_kv_heads * d, H), o=qmat(a + "o_proj", H, cfg.n_q_heads * d),
                      sinks=vec(a + "softmax_offset"), q_norm=vec(a + "q_norm.weight"),
                      k_norm=vec(a + "k_norm.weight"), kind=kind)
        m = p + "mlp."
        if kind & abi.REC_LAYER_DENSE:
            I = cfg.dense_inter
            L = LayerWeights(**common, router=None, gate=qmat(m + "gate_proj", I, H), up=qmat(m + "up_proj", I, H),
                             down=qmat(m + "down_proj", H, I))
        else:
            E, I = cfg.n_experts, cfg.moe_inter
            L = LayerWeights(**common, router=vec(m + "gate.weight"),
                             expert_bias=vec(m + "gate.expert_bias", torch.float32),
                             gate=qmat(m + "switch_mlp.gate_proj", E * I, H, stacked=E),
                             up=qmat(m + "switch_mlp.up_proj", E * I, H, stacked=E),
                             down=qmat(m + "switch_mlp.down_proj", E * H, I, stacked=E))
            if cfg.shared_inter:
                Is = cfg.shared_inter
                L.shared_gate = qmat(m + "shared_expert.gate_proj", Is, H)
                L.shared_up = qmat(m + "shared_expert.up_proj", Is, H)
                L.shared_down = qmat(m + "shared_expert.down_proj", H, Is)
        layers.append(L)
    embed = qmat("model.embed_tokens", cfg.vocab, H, bits=cfg.embed_bits)
    final_norm = vec("model.norm.weight")
    lm_head = qmat("lm_head", cfg.vocab, H)
    extra = sorted(set(t) - used)
    if extra:  # strict, as the reference loads (quantized.py:42)
        raise ValueError(f"{len(extra)} checkpoint tensors are not part of the model, e.g. {extra[0]}")
    eos = config.get("eos_token_id", ())
    eos = (eos,) if isinstance(eos, int) else tuple(int(e) for e in eos or ())
    return ModelWeights(cfg, layers, embed, final_norm, lm_head, expert_range=(0, cfg.n_experts), eos_tokens=eos)
