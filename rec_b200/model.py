"""Model configurations, synthetic weights and KV storage for the decode path.

The layout of every tensor is the reference's MLX layout
(engine/src/rec_mlx/quantized.py:26-36, megakernel.py:161-170):
int4 g64 affine weights as uint32 codes [N, K/8] (stored as int32 tensors)
with scales/biases [N, K/64]; expert weights stacked [E*N, K]; the quantized
KV cache as codes [Hkv, C, 128*bits/32] with bf16 scales/biases [Hkv, C, 2]
(model.py:40-82).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field, replace
from typing import ClassVar

import torch

from . import abi


@dataclass(frozen=True)
class ModelConfig:
    """Shape of the decoder (reference ModelArgs, model.py:14-37)."""
    name: str = "custom"
    hidden: int = 2048
    n_layers: int = 48
    n_q_heads: int = 32
    n_kv_heads: int = 4
    head_dim: int = 128
    n_experts: int = 128
    top_k: int = 8
    moe_inter: int = 768
    vocab: int = 151936
    scale_dtype: torch.dtype = torch.float16
    kv_bits: int = 8
    router_mode: int = abi.REC_ROUTER_SOFTMAX
    flags: int = 0
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    # Flint layer options (reference ModelArgs, model.py:14-37): an always-on
    # shared expert of shared_inter rows in every MoE layer; dense SwiGLU MLP
    # layers (`mlp_only_layers`) of dense_inter rows; layers without RoPE
    # (`no_rope_layer_indices`); sliding-window layers (`layer_types`) that
    # attend the last sliding_window positions.  Any of them puts the model
    # on the graph schedule.
    shared_inter: int = 0
    dense_layers: tuple = ()
    dense_inter: int = 0
    no_rope_layers: tuple = ()
    sliding_layers: tuple = ()
    sliding_window: int = 0
    embed_bits: int = 4  # 8: the production checkpoint's int8 embedding
    kv_value_bits: int = 0  # V codes' width when it differs from kv_bits (the reference's K8 / V4 cache)

    def layer_kind(self, i: int) -> int:
        """REC_LAYER_* bits of layer i."""
        return ((abi.REC_LAYER_DENSE if i in self.dense_layers else 0)
                | (abi.REC_LAYER_NO_ROPE if i in self.no_rope_layers else 0)
                | (abi.REC_LAYER_SLIDING if i in self.sliding_layers else 0))

    @property
    def has_layer_options(self) -> bool:
        """Options that put the model on the graph schedule (and its prefill
        on the decode step): the Flint layer options and a bf16 cache."""
        return bool(self.shared_inter or self.dense_layers or self.no_rope_layers or self.sliding_layers
                    or self.kv_bits == 16 or self.embed_bits == 8 or self.v_bits != self.kv_bits)

    @property
    def v_bits(self) -> int:
        """Bits of the V codes (kv_bits unless the cache is mixed)."""
        return self.kv_value_bits or self.kv_bits

    def desc(self) -> abi.RecModelDesc:
        return abi.RecModelDesc(
            hidden=self.hidden, n_layers=self.n_layers, n_q_heads=self.n_q_heads, n_kv_heads=self.n_kv_heads,
            head_dim=self.head_dim, n_experts=self.n_experts, top_k=self.top_k, moe_inter=self.moe_inter,
            vocab=self.vocab, group_size=64,
            scale_dtype=abi.REC_SCALE_FP16 if self.scale_dtype == torch.float16 else abi.REC_SCALE_BF16,
            kv_bits=self.kv_bits, router_mode=self.router_mode, flags=self.flags, rms_eps=self.rms_eps,
            rope_theta=self.rope_theta, shared_inter=self.shared_inter,
            dense_inter=self.dense_inter if self.dense_layers else 0,
            sliding_window=self.sliding_window if self.sliding_layers else 0, embed_bits=self.embed_bits,
            kv_value_bits=self.kv_value_bits)

    def weight_bytes_per_token(self) -> int:
        """Algorithmic bytes streamed per decode step (weights only)."""
        g = 0.5 + 4 / 64  # int4 codes + fp16/bf16 scale and bias per 64
        h, d = self.hidden, self.head_dim
        attn = (self.n_q_heads + 2 * self.n_kv_heads) * d * h + h * self.n_q_heads * d
        experts = (self.top_k * self.moe_inter + self.shared_inter) * 3 * h
        moe_layer = (attn + experts) * g + self.n_experts * h * 2 + 2 * h * 2
        dense_layer = (attn + 3 * self.dense_inter * h) * g + 2 * h * 2
        n_dense = len(self.dense_layers)
        total = (self.n_layers - n_dense) * moe_layer + n_dense * dense_layer
        return int(total + self.vocab * h * g + h * 2 + h * g)

    def kv_bytes_per_token(self, context: int) -> int:
        scales = 2 * 2 * self.head_dim // 64 if self.kv_bits < 16 else 0  # a bf16 cache has none
        per = self.n_kv_heads * (self.head_dim * (self.kv_bits + self.v_bits) // 8 + 2 * scales)
        return self.n_layers * per * context


# BASELINE.json configurations
CONFIG1_LAYER = ModelConfig(name="config1_layer", n_layers=1, n_experts=64, vocab=4096, kv_bits=8)
CONFIG3 = ModelConfig(name="config3_flint_shaped_48L_128E", n_layers=48, n_experts=128, kv_bits=8)
CONFIG4 = replace(CONFIG3, name="config4_252k_4bit_kv", kv_bits=4)
# small shapes for parity tests (same kernels, fewer layers/experts/vocab)
TINY = ModelConfig(name="tiny", n_layers=2, n_experts=16, top_k=4, vocab=4096, kv_bits=8)
# the reference Flint model's layer structure at test size (model.py:14-37,
# 155-163,216-271): sigmoid + bias router with top-6, a shared expert, dense
# MLP in layer 0, a NoPE ("global") layer between RoPE'd sliding-window layers,
# attention sinks and q/k head norms, bf16 scales
TINY_FLINT = ModelConfig(name="tiny_flint", n_layers=3, n_experts=16, top_k=6, moe_inter=512, vocab=4096,
                         kv_bits=8, scale_dtype=torch.bfloat16, router_mode=abi.REC_ROUTER_SIGMOID,
                         flags=abi.REC_FLAG_SINKS | abi.REC_FLAG_QK_NORM, shared_inter=1024, dense_layers=(0,),
                         dense_inter=6144, no_rope_layers=(1,), sliding_layers=(0, 2), sliding_window=300,
                         embed_bits=8)
# The reference's Flint checkpoint at full size (model.py:14-37; megakernel.py:
# 992-1004 asserts 49 layers, hidden 2048, 32/4 heads x 128, 256 experts
# top-6, window 513, vocab 150,144): dense MLP layers 0-1 (I 6,144), shared
# expert 1,024, routed I 512, sigmoid + bias router, sinks, q/k norms, int8
# embedding, bf16 scales, the production megakernel's bf16 cache, RoPE theta
# 10,000.  Which layers are global (NoPE, full attention) comes from the
# checkpoint's config, which the reference does not ship: one in four is
# assumed here (layers 3, 7, ..., 47), the rest slide over 513 positions.
_FLINT_GLOBAL = tuple(range(3, 49, 4))
FLINT = ModelConfig(name="flint_full_shape", n_layers=49, n_experts=256, top_k=6, moe_inter=512, vocab=150144,
                    kv_bits=16, scale_dtype=torch.bfloat16, router_mode=abi.REC_ROUTER_SIGMOID,
                    flags=abi.REC_FLAG_SINKS | abi.REC_FLAG_QK_NORM, shared_inter=1024, dense_layers=(0, 1),
                    dense_inter=6144, no_rope_layers=_FLINT_GLOBAL,
                    sliding_layers=tuple(i for i in range(49) if i not in _FLINT_GLOBAL), sliding_window=513,
                    embed_bits=8, rope_theta=10000.0)


# The reference's ModelArgs defaults (engine/src/rec_mlx/model.py:14-37).
_REFERENCE_ARGS = dict(hidden_size=2048, intermediate_size=6144, moe_intermediate_size=512,
                       shared_expert_intermediate_size=1024, num_hidden_layers=49, num_attention_heads=32,
                       num_key_value_heads=4, head_dim=128, num_experts=256, num_experts_per_tok=6,
                       vocab_size=150144, rms_norm_eps=1e-6, rope_theta=10000.0, sliding_window=513,
                       layer_types=[], no_rope_layer_indices=[], mlp_only_layers=[0, 1],
                       tie_word_embeddings=False, kv_key_bits=8, kv_value_bits=4, kv_group_size=64)


def config_from_reference(config: dict, *, kv_format: str = "bf16", name: str = "from_reference") -> ModelConfig:
    """The ModelConfig of a reference checkpoint's config.json (the
    reference's ModelArgs fields, engine/src/rec_mlx/model.py:14-37; absent
    keys take its defaults).  The Flint decoder always has the sigmoid + bias
    router (model.py:245-254), a shared expert (model.py:243), attention sinks
    and q/k head norms (model.py:155-163), bf16 scales and biases.

    kv_format: "bf16" (the production engine's cache, checkpoint.py:7) or
    "native" (MLX's MixedQuantizedKVCache with kv_key_bits / kv_value_bits,
    model.py:35-37).  `mlx_export.embedding_bits` gives the embedding's code
    width (8 in the production export, checkpoint.py:26-28).  Raises
    ValueError for what these kernels do not take: tied embeddings, routed
    experts other than int4, quantization other than int4 group 64, KV
    groups other than 64, unknown layer types."""
    a = dict(_REFERENCE_ARGS)
    a.update({k: v for k, v in config.items() if k in _REFERENCE_ARGS})
    n = int(a["num_hidden_layers"])
    if a["tie_word_embeddings"]:
        raise ValueError("tied embeddings are not supported: the lm_head is its own int4 matrix")
    q = config.get("quantization", {"group_size": 64, "bits": 4})
    if q.get("group_size") != 64 or q.get("bits") != 4:
        raise ValueError("expected int4 group-64 quantization")
    export = config.get("mlx_export", {})
    if export.get("routed_expert_bits", 4) != 4 or export.get("bits", 4) != 4:
        raise ValueError("routed experts and projections must be int4")
    embed_bits = int(export.get("embedding_bits", 4))
    if a["kv_group_size"] != 64:
        raise ValueError("the KV cache is quantized in groups of 64")
    types = list(a["layer_types"]) or ["full_attention"] * n
    if len(types) != n or not set(types) <= {"full_attention", "sliding_attention"}:
        raise ValueError("layer_types must name 'full_attention' or 'sliding_attention' for every layer")
    if kv_format == "bf16":
        kv_bits, kv_value_bits = 16, 0
    elif kv_format == "native":
        kv_bits = int(a["kv_key_bits"])
        kv_value_bits = int(a["kv_value_bits"]) if int(a["kv_value_bits"]) != kv_bits else 0
    else:
        raise ValueError("kv_format must be 'bf16' or 'native'")
    dense = tuple(int(i) for i in a["mlp_only_layers"])
    return ModelConfig(
        name=name, hidden=int(a["hidden_size"]), n_layers=n, n_q_heads=int(a["num_attention_heads"]),
        n_kv_heads=int(a["num_key_value_heads"]), head_dim=int(a["head_dim"]), n_experts=int(a["num_experts"]),
        top_k=int(a["num_experts_per_tok"]), moe_inter=int(a["moe_intermediate_size"]),
        vocab=int(a["vocab_size"]), scale_dtype=torch.bfloat16, kv_bits=kv_bits, kv_value_bits=kv_value_bits,
        router_mode=abi.REC_ROUTER_SIGMOID, flags=abi.REC_FLAG_SINKS | abi.REC_FLAG_QK_NORM,
        rms_eps=float(a["rms_norm_eps"]), rope_theta=float(a["rope_theta"]),
        shared_inter=int(a["shared_expert_intermediate_size"]), dense_layers=dense,
        dense_inter=int(a["intermediate_size"]) if dense else 0,
        no_rope_layers=tuple(int(i) for i in a["no_rope_layer_indices"]),
        sliding_layers=tuple(i for i, t in enumerate(types) if t == "sliding_attention"),
        sliding_window=int(a["sliding_window"]), embed_bits=embed_bits)


def _quantize(w: torch.Tensor, bits: int, scale_dtype: torch.dtype):
    if w.is_cuda:
        from .ops import quantize_affine

        return quantize_affine(w.float().contiguous(), bits, scale_dtype)
    raise ValueError("synthetic weights are quantized on the GPU; pass a CUDA device")


def _normal(gen: torch.Generator, shape, std: float, device) -> torch.Tensor:
    x = torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * std
    return x.to(torch.bfloat16).float()  # weights exist as bf16 before quantization


def _norm_weight(gen, h, device) -> torch.Tensor:
    return (1.0 + 0.1 * torch.randn(h, generator=gen, device=device)).to(torch.bfloat16)


@dataclass
class QTensor:
    w: torch.Tensor  # int32 [N, K/8]
    s: torch.Tensor  # fp16/bf16 [N, K/64]
    b: torch.Tensor

    def rec(self) -> abi.RecQMat:
        return abi.RecQMat(self.w.data_ptr(), self.s.data_ptr(), self.b.data_ptr())

    def nbytes(self) -> int:
        return self.w.numel() * 4 + self.s.numel() * 2 + self.b.numel() * 2


@dataclass
class LayerWeights:
    input_norm: torch.Tensor
    post_norm: torch.Tensor
    q: QTensor
    k: QTensor
    v: QTensor
    o: QTensor
    router: torch.Tensor
    gate: QTensor
    up: QTensor
    down: QTensor
    expert_bias: torch.Tensor | None = None
    sinks: torch.Tensor | None = None
    q_norm: torch.Tensor | None = None
    k_norm: torch.Tensor | None = None
    kind: int = 0                       # REC_LAYER_* bits
    shared_gate: QTensor | None = None  # the shared expert (MoE layers of a model with shared_inter)
    shared_up: QTensor | None = None
    shared_down: QTensor | None = None

    def rec(self) -> abi.RecLayerWeights:
        def p(t):
            return None if t is None else t.data_ptr()

        def qm(t):
            return t.rec() if t is not None else abi.RecQMat()

        return abi.RecLayerWeights(
            input_norm=p(self.input_norm), post_norm=p(self.post_norm), q=self.q.rec(), k=self.k.rec(),
            v=self.v.rec(), o=self.o.rec(), router=p(self.router), expert_bias=p(self.expert_bias),
            gate=self.gate.rec(), up=self.up.rec(), down=self.down.rec(), sinks=p(self.sinks),
            q_norm=p(self.q_norm), k_norm=p(self.k_norm), kind=self.kind, shared_gate=qm(self.shared_gate),
            shared_up=qm(self.shared_up), shared_down=qm(self.shared_down))


@dataclass
class ModelWeights:
    cfg: ModelConfig
    layers: list[LayerWeights]
    embed: QTensor
    final_norm: torch.Tensor
    lm_head: QTensor
    expert_range: tuple[int, int] = (0, 0)  # experts held (expert parallelism)
    _keep: list = field(default_factory=list)
    eos_tokens: tuple = ()  # the model's end ids (config.json eos_token_id; quantized.py:77)
    context_limit: ClassVar[int] = 262144  # positions a session may reach (quantized.py:17)

    def rec_layers(self):
        arr = (abi.RecLayerWeights * len(self.layers))(*[L.rec() for L in self.layers])
        self._keep.append(arr)
        return arr

    def rec_global(self) -> abi.RecGlobalWeights:
        g = abi.RecGlobalWeights(embed=self.embed.rec(), final_norm=self.final_norm.data_ptr(),
                                 lm_head=self.lm_head.rec())
        self._keep.append(g)
        return g


def generate_weights(cfg: ModelConfig, seed: int = 0, device: str | torch.device = "cuda",
                     expert_range: tuple[int, int] | None = None) -> ModelWeights:
    """Random-init weights of the configuration: linear weights ~N(0, 0.02)
    rounded to bf16, then int4 g64 affine-quantized; router bf16 ~N(0, 0.02);
    embedding rows ~N(0, 1).  With expert_range=(lo, hi) only experts
    [lo, hi) are materialised (expert parallelism); the rest are still drawn so
    that every rank sees the same values."""
    device = torch.device(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    h, d, sd = cfg.hidden, cfg.head_dim, cfg.scale_dtype
    lo, hi = expert_range if expert_range is not None else (0, cfg.n_experts)

    def qmat(n, k, std=0.02):
        return QTensor(*_quantize(_normal(gen, (n, k), std, device), 4, sd))

    def experts(n, k):
        parts = []
        for e in range(cfg.n_experts):
            w = _normal(gen, (n, k), 0.02, device)
            if lo <= e < hi:
                parts.append(_quantize(w, 4, sd))
        return QTensor(*(torch.cat([p[i] for p in parts]) for i in range(3)))

    if cfg.has_layer_options and expert_range is not None and expert_range != (0, cfg.n_experts):
        raise ValueError("layer options run on one GPU (no expert parallelism)")
    layers = []
    for i in range(cfg.n_layers):
        kind = cfg.layer_kind(i)
        common = dict(input_norm=_norm_weight(gen, h, device), post_norm=_norm_weight(gen, h, device),
                      q=qmat(cfg.n_q_heads * d, h), k=qmat(cfg.n_kv_heads * d, h), v=qmat(cfg.n_kv_heads * d, h),
                      o=qmat(h, cfg.n_q_heads * d))
        if kind & abi.REC_LAYER_DENSE:  # a dense SwiGLU MLP (model.py:216-224), no router
            I = cfg.dense_inter
            L = LayerWeights(**common, router=None, gate=qmat(I, h), up=qmat(I, h), down=qmat(h, I), kind=kind)
            if cfg.flags & abi.REC_FLAG_SINKS:
                L.sinks = torch.randn(cfg.n_q_heads, generator=gen, device=device).to(torch.bfloat16)
            if cfg.flags & abi.REC_FLAG_QK_NORM:
                L.q_norm = _norm_weight(gen, d, device)
                L.k_norm = _norm_weight(gen, d, device)
            layers.append(L)
            continue
        L = LayerWeights(
            **common,
            router=_normal(gen, (cfg.n_experts, h), 0.02, device).to(torch.bfloat16),
            gate=experts(cfg.moe_inter, h), up=experts(cfg.moe_inter, h), down=experts(h, cfg.moe_inter),
            kind=kind)
        if cfg.shared_inter:  # the always-on shared expert (model.py:243,254)
            Is = cfg.shared_inter
            L.shared_gate, L.shared_up, L.shared_down = qmat(Is, h), qmat(Is, h), qmat(h, Is)
        if cfg.router_mode == abi.REC_ROUTER_SIGMOID:
            L.expert_bias = (0.05 * torch.randn(cfg.n_experts, generator=gen, device=device)).float()
        if cfg.flags & abi.REC_FLAG_SINKS:
            L.sinks = torch.randn(cfg.n_q_heads, generator=gen, device=device).to(torch.bfloat16)
        if cfg.flags & abi.REC_FLAG_QK_NORM:
            L.q_norm = _norm_weight(gen, d, device)
            L.k_norm = _norm_weight(gen, d, device)
        layers.append(L)
    embed = QTensor(*_quantize(_normal(gen, (cfg.vocab, h), 1.0, device), cfg.embed_bits, sd))
    final_norm = _norm_weight(gen, h, device)
    lm_head = qmat(cfg.vocab, h)
    return ModelWeights(cfg, layers, embed, final_norm, lm_head, expert_range=(lo, hi))


@dataclass
class KVCache:
    """Quantized KV storage for every layer, capacity C (multiple of 256).
    A cache made by `reserve` has its codes in reserved virtual memory
    (rec_b200.vmm): C is the head stride, only rows [0, rows) are backed, and
    `grow` backs more rows in place; the tensors in `layers` then cover the
    backed rows."""
    cfg: ModelConfig
    capacity: int
    layers: list[dict]
    reserved: list | None = None  # per layer {"k_codes": ReservedCodes, "v_codes": ...}
    rows: int = 0                 # backed rows (== capacity for an ordinary cache)

    def __post_init__(self):
        if not self.rows:
            self.rows = self.capacity

    @classmethod
    def reserve(cls, cfg: ModelConfig, capacity: int, rows: int, device="cuda") -> "KVCache":
        """Codes reserved for `capacity` rows (a multiple of 65,536) and backed
        for `rows`; scales and biases allocated for the full capacity."""
        from .vmm import ReservedCodes

        words = {"k_codes": 128 * cfg.kv_bits // 32, "v_codes": 128 * cfg.v_bits // 32}
        dev = torch.device(device)
        layers, reserved = [], []
        for _ in range(cfg.n_layers):
            R = {n: ReservedCodes(cfg.n_kv_heads, capacity, words[n], dev) for n in ("k_codes", "v_codes")}
            L = {}
            for kv in ("k", "v"):
                L[f"{kv}_codes"] = None
                L[f"{kv}_scales"] = torch.zeros(cfg.n_kv_heads, capacity, 2, dtype=torch.bfloat16, device=dev)
                L[f"{kv}_biases"] = torch.zeros(cfg.n_kv_heads, capacity, 2, dtype=torch.bfloat16, device=dev)
            layers.append(L)
            reserved.append(R)
        obj = cls(cfg, capacity, layers, reserved, rows=1)
        obj.rows = 0
        obj.grow(rows)
        return obj

    def grow(self, rows: int) -> None:
        """Backs rows [0, rows) of a reserved cache (rows already written stay
        in place)."""
        if self.reserved is None:
            raise ValueError("only a reserved cache grows in place")
        if rows <= self.rows:
            return
        for L, R in zip(self.layers, self.reserved):
            for n, rc in R.items():
                rc.grow(rows)
                L[n] = rc.view()
        self.rows = self.reserved[0]["k_codes"].rows

    @classmethod
    def allocate(cls, cfg: ModelConfig, capacity: int, device="cuda") -> "KVCache":
        if capacity % 256:
            raise ValueError("KV capacity must be a multiple of 256")
        words = {"k": 128 * cfg.kv_bits // 32, "v": 128 * cfg.v_bits // 32}
        layers = []
        for _ in range(cfg.n_layers):
            L = {}
            for kv in ("k", "v"):
                L[f"{kv}_codes"] = torch.zeros(cfg.n_kv_heads, capacity, words[kv], dtype=torch.int32, device=device)
                L[f"{kv}_scales"] = torch.zeros(cfg.n_kv_heads, capacity, 2, dtype=torch.bfloat16, device=device)
                L[f"{kv}_biases"] = torch.zeros(cfg.n_kv_heads, capacity, 2, dtype=torch.bfloat16, device=device)
            layers.append(L)
        return cls(cfg, capacity, layers)

    def rec(self):
        arr = (abi.RecKVLayer * len(self.layers))(*[
            abi.RecKVLayer(*(L[n].data_ptr() for n in ("k_codes", "k_scales", "k_biases", "v_codes", "v_scales",
                                                       "v_biases"))) for L in self.layers])
        return arr

    def view(self, layer: int, name: str, upto: int | None = None) -> torch.Tensor:
        """Tensor `name` of a layer restricted to rows [0, upto) (default: the
        backed rows)."""
        n = self.rows if upto is None else min(upto, self.rows)
        return self.layers[layer][name][:, :n]

    def nbytes(self) -> int:
        """Bytes of device memory the cache holds (backed rows only for
        reserved codes)."""
        return sum(t.numel() * t.element_size() for L in self.layers for t in L.values())

    def fill_random(self, upto: int, seed: int = 0, start: int = 0) -> None:
        """Fills positions [start, upto) by quantizing synthetic K, V ~ N(0, 1)
        (group 64 along head_dim) — the long-context caches of BASELINE.json
        configs 2 and 4 are built this way instead of by prefill."""
        from .ops import quantize_affine

        gen = torch.Generator(device=self.layers[0]["k_codes"].device)
        gen.manual_seed(seed)
        dev = self.layers[0]["k_codes"].device
        chunk = 16384
        for L in self.layers:
            for kv in ("k", "v"):
                for p0 in range(start, upto, chunk):
                    p1 = min(upto, p0 + chunk)
                    x = torch.randn(self.cfg.n_kv_heads, p1 - p0, 128, generator=gen, device=dev)
                    x = x.to(torch.bfloat16).float()
                    if self.cfg.kv_bits == 16:  # bf16 rows (a pair per 32-bit word)
                        L[f"{kv}_codes"][:, p0:p1] = x.to(torch.bfloat16).view(torch.int16).view(torch.int32)
                        continue
                    c, s, b = quantize_affine(x, self.cfg.kv_bits if kv == "k" else self.cfg.v_bits, torch.bfloat16)
                    L[f"{kv}_codes"][:, p0:p1] = c
                    L[f"{kv}_scales"][:, p0:p1] = s
                    L[f"{kv}_biases"][:, p0:p1] = b
