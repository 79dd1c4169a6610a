"""Shape-faithful random model in host memory for CPU timing runs — TEST
INFRASTRUCTURE ONLY (see oracle/__init__.py).

The CPU baseline's cost does not depend on weight values, only on shapes, so
this builds int4 g64 tensors directly (uniform codes, fp16 scales/biases with
the magnitude N(0, 0.02) weights quantize to) instead of sampling and
quantizing ~30 G normals on the host.
"""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np

from . import f32_to_bf16


def _q(rng, n, k, std=0.02):
    codes = rng.integers(0, 2**32, size=(n, k // 8), dtype=np.uint32)
    step = np.float32(6 * std / 15)
    scales = (step * (0.8 + 0.4 * rng.random((n, k // 64), dtype=np.float32))).astype(np.float16)
    biases = (-7.5 * scales.astype(np.float32)).astype(np.float16)
    return SimpleNamespace(w=codes, s=scales.view(np.uint16), b=biases.view(np.uint16))


def _bf(rng, shape, std, mean=0.0):
    return f32_to_bf16((mean + std * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32))


def random_model(cfg, seed: int = 0):
    rng = np.random.default_rng(seed)
    h, d = cfg.hidden, cfg.head_dim
    layers = []
    for _ in range(cfg.n_layers):
        layers.append(SimpleNamespace(
            input_norm=_bf(rng, h, 0.1, 1.0), post_norm=_bf(rng, h, 0.1, 1.0),
            q=_q(rng, cfg.n_q_heads * d, h), k=_q(rng, cfg.n_kv_heads * d, h), v=_q(rng, cfg.n_kv_heads * d, h),
            o=_q(rng, h, cfg.n_q_heads * d), router=_bf(rng, (cfg.n_experts, h), 0.02),
            gate=_q(rng, cfg.n_experts * cfg.moe_inter, h), up=_q(rng, cfg.n_experts * cfg.moe_inter, h),
            down=_q(rng, cfg.n_experts * h, cfg.moe_inter), expert_bias=None, sinks=None, q_norm=None,
            k_norm=None))
    return SimpleNamespace(cfg=cfg, layers=layers, embed=_q(rng, cfg.vocab, h, std=1.0),
                           final_norm=_bf(rng, h, 0.1, 1.0), lm_head=_q(rng, cfg.vocab, h))
