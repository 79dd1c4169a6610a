"""Drop-in replacement of the reference decoder API on B200.

Mirrors recursive-oss/rec engine/src/rec_mlx:
  kernels/__init__.py:1-65      build_decoder(model, *, optimized) -> (engine, resident_sampler)
  kernels/megakernel.py:983-1337 FullModel: forward, make_session, prefill_state, ensure_capacity
  kernels/sampling.py:17-169     ResidentSampler.block
  quantized.py:98-151            QATSession.prefill / forward_token

State dict keys and error conventions follow the reference
(megakernel.py:1264-1268, 1308-1337; sampling.py:77-78): a device-wait
timeout raises RuntimeError("GPU synchronization failed: ...") and marks the
state unusable; reusing it raises "Session was invalidated ..."; running past
the limit raises ValueError("Decode context limit exhausted"); packets must
hold 1..8 tokens.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, fields

import torch

from . import abi
from ._lib import RecError
from .model import KVCache, ModelConfig, ModelWeights, QTensor
from .session import DecodeSession

WIDTH = 8  # resident packet size (sampling.py:8)
GROUP_LAYERS = 4  # layers per weight group (the reference packs one bank per four layers)


@dataclass(frozen=True)
class DeviceProfile:
    """The engine's device (reference kernels/device.py:4-13): `chip` is the
    CUDA device name, `architecture` its compute capability; `workers` the
    SM count the persistent schedule spreads over."""

    chip: str
    architecture: str
    workers: int
    prefill_chunk_size: int


def layer_metadata(cfg: ModelConfig) -> list[list[int]]:
    """The engine's layer table, one row of 64 per layer and a last row for
    the globals, with the reference's column meaning
    (kernels/megakernel.py:1008-1088).  Column 0 is the layer's group of four
    (the reference's weight bank), 1 is 1 when the layer attends over the
    whole context (not a sliding-window layer), 2 is 1 when it routes
    experts.  Each quantized matrix takes five columns — the byte offsets of
    its codes, scales and biases within the bank, then its rows (per expert)
    and columns — at 10 (q), 15 (k), 20 (v), 25 (o), 30 (gate), 35 (up), 40
    (down) and, for the shared expert, 45 / 50 / 55; the last row holds the
    embedding at 10 and lm_head at 30.  Here every weight is its own device
    tensor rather than a slice of a packed bank, so the offset columns (3-9,
    the first three of each matrix, 60) hold 0."""
    H, d = cfg.hidden, cfg.head_dim
    rows = []

    def linear(row, base, n, k):
        row[base + 3:base + 5] = [n, k]

    for i in range(cfg.n_layers):
        kind = cfg.layer_kind(i)
        row = [0] * 64
        moe = not kind & abi.REC_LAYER_DENSE
        row[0:3] = [i // GROUP_LAYERS, int(not kind & abi.REC_LAYER_SLIDING), int(moe)]
        linear(row, 10, cfg.n_q_heads * d, H)
        linear(row, 15, cfg.n_kv_heads * d, H)
        linear(row, 20, cfg.n_kv_heads * d, H)
        linear(row, 25, H, cfg.n_q_heads * d)
        inter = cfg.moe_inter if moe else cfg.dense_inter
        linear(row, 30, inter, H)
        linear(row, 35, inter, H)
        linear(row, 40, H, inter)
        if moe and cfg.shared_inter:
            linear(row, 45, cfg.shared_inter, H)
            linear(row, 50, cfg.shared_inter, H)
            linear(row, 55, H, cfg.shared_inter)
        rows.append(row)
    last = [0] * 64
    last[0] = (cfg.n_layers - 1) // GROUP_LAYERS
    linear(last, 10, cfg.vocab, H)
    linear(last, 30, cfg.vocab, H)
    rows.append(last)
    return rows


def weight_banks(weights: ModelWeights) -> list[tuple]:
    """The device tensors of each group of four layers, in the layer
    fields' order (a quantized matrix as codes, scales, biases), the last
    group followed by the embedding, the final norm and lm_head — the
    reference's thirteen weight banks (kernels/megakernel.py:1011-1108),
    held as separate tensors instead of one packed buffer per group."""
    def flat(obj):
        out = []
        for f in fields(obj):
            v = getattr(obj, f.name)
            if isinstance(v, QTensor):
                out += [v.w, v.s, v.b]
            elif isinstance(v, torch.Tensor):
                out.append(v)
        return out

    banks = []
    for first in range(0, len(weights.layers), GROUP_LAYERS):
        banks.append([t for L in weights.layers[first:first + GROUP_LAYERS] for t in flat(L)])
    banks[-1] += [weights.embed.w, weights.embed.s, weights.embed.b, weights.final_norm,
                  weights.lm_head.w, weights.lm_head.s, weights.lm_head.b]
    return [tuple(b) for b in banks]


class KVStorage:
    """Growable quantized KV storage of a state (reference cache.py:47-119).

    The cache's codes are reserved in virtual memory for the state's limit
    (rounded up to 32,768-token blocks; the reference's bank blocks hold
    65,536) and backed block by block as the context grows (rec_b200.vmm): a growth maps new
    memory behind the rows already written, without copying them and without
    a new session.  A state that outgrows its reservation (a prompt cache
    reused under a larger limit) is moved once into a larger reservation."""

    def __init__(self, weights: ModelWeights, capacity: int, device, limit: int | None = None):
        self.weights = weights
        self.device = device
        self.capacity = 0
        self.cache: KVCache | None = None
        self.session: DecodeSession | None = None
        self.reserve_rows = self._reserve(max(capacity, limit or 0))
        self.grow(capacity)

    @staticmethod
    def _reserve(n: int) -> int:
        from .vmm import BLOCK_TOKENS

        return max(BLOCK_TOKENS, -(-n // BLOCK_TOKENS) * BLOCK_TOKENS)

    @classmethod
    def wrap(cls, weights: ModelWeights, cache: KVCache, session: DecodeSession) -> "KVStorage":
        """Storage around an existing cache and session (no copy)."""
        obj = cls.__new__(cls)
        obj.weights, obj.cache, obj.session = weights, cache, session
        obj.device = cache.layers[0]["k_codes"].device
        obj.capacity = cache.capacity
        return obj

    def grow(self, count: int) -> None:
        """Backs at least `count` positions."""
        if self.cache is not None and count <= self.capacity:
            return
        if self.cache is not None and self.cache.reserved is not None and count <= self.cache.capacity:
            self.cache.grow(count)  # in place: new blocks behind the written rows
            self.session.set_rows(self.cache.rows)
            self.capacity = self.cache.rows
            return
        old = self.cache
        self.reserve_rows = max(self.reserve_rows, self._reserve(count))
        from .vmm import BLOCK_TOKENS

        if self.reserve_rows <= BLOCK_TOKENS:
            # a limit within one block: the whole cache at once (one ordinary
            # allocation, no mapping calls on the prefill's critical path)
            new = KVCache.allocate(self.weights.cfg, self.reserve_rows, self.device)
        else:
            new = KVCache.reserve(self.weights.cfg, self.reserve_rows, count, self.device)
        if old is not None:  # outgrew the reservation: one move into the larger one
            for dst, src in zip(new.layers, old.layers):
                for name in dst:
                    n = min(src[name].shape[1], dst[name].shape[1])
                    dst[name][:, :n].copy_(src[name][:, :n])
        self.cache = new
        self.capacity = new.rows
        self.session = DecodeSession(self.weights, new)

    @property
    def nbytes(self) -> int:
        return self.cache.nbytes() if self.cache is not None else 0

    @property
    def banks(self) -> list[tuple]:
        """Each layer's cache tensors (codes, scales, biases of K and V), the
        counterpart of the reference's KV banks (cache.py:68)."""
        return [tuple(layer.values()) for layer in self.cache.layers]

    @property
    def metadata(self) -> list[list[int]]:
        """The engine's layer table with columns 61-62 set as the
        reference's storage sets them (cache.py:53-66): the layer's element
        offset in its bank (0: each layer is its own tensor) and its rows (the
        cache's head stride; a sliding layer reads only its window of them).
        The same object until the cache moves into a larger reservation."""
        cached = getattr(self, "_metadata", None)
        if cached is None or cached[0] is not self.cache:
            rows = layer_metadata(self.weights.cfg)
            for row in rows[:-1]:
                row[61:63] = [0, self.cache.capacity]
            cached = self._metadata = (self.cache, rows)
        return cached[1]


class FullModel:
    """B200 decode engine for one model (one GPU)."""

    def __init__(self, weights: ModelWeights, *, prefill_chunk_size: int = 1024, device="cuda"):
        self.model = weights
        self.weights = weights
        self.cfg = weights.cfg
        self.device = torch.device(device)
        self.prefill_chunk_size = prefill_chunk_size
        props = torch.cuda.get_device_properties(self.device)
        self.workers = props.multi_processor_count
        self.device_profile = DeviceProfile(props.name, f"sm_{props.major}{props.minor}", self.workers,
                                            prefill_chunk_size)
        self.schedule = {"workers": self.workers, "graph": "per-token CUDA graph, programmatic dependent launch"}
        self.metadata = layer_metadata(self.cfg)
        self.banks = weight_banks(weights)
        # bf16[65536]: the SiLU of every bf16 gate (megakernel.py:1110-1112)
        self.silu = torch.empty(65536, dtype=torch.bfloat16, device=self.device)
        from . import _lib

        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().rec_silu_table(self.silu.data_ptr(),
                                                 torch.cuda.current_stream(self.device).cuda_stream))

    # -- state ---------------------------------------------------------------
    def prefill_state(self, capacity, *, limit=None, storage=None):
        if storage is None:
            storage = KVStorage(self.weights, capacity, self.device, limit=limit)
        else:
            storage.grow(capacity)
        return {"usable": True, "kv": storage, "metadata": storage.metadata, "position": 0, "initial": 0,
                "capacity": storage.capacity, "limit": capacity if limit is None else limit,
                "growth_count": 0, "growth_seconds": 0.0}

    def ensure_capacity(self, state, count):
        if not state["usable"]:
            raise RuntimeError("Session was invalidated by a GPU synchronization failure")
        required = state["position"] + count
        if required > state["limit"]:
            raise ValueError("Decode context limit exhausted")
        if required > state["capacity"]:
            started = time.perf_counter()
            state["kv"].grow(required)
            state["capacity"] = state["kv"].capacity
            state["metadata"] = state["kv"].metadata
            state["growth_count"] += 1
            state["growth_seconds"] += time.perf_counter() - started

    def _session(self, state) -> DecodeSession:
        return state["kv"].session

    def _guard(self, state, fn):
        try:
            return fn()
        except RecError as exc:
            state["usable"] = False
            raise RuntimeError(f"GPU synchronization failed: {exc}") from None

    # -- one step -------------------------------------------------------------
    def forward(self, state, token, layer_count=None):
        """One token through the first `layer_count` layers (all of them by
        default); returns (logits bf16[V], trace bf16[layer_count + 1, H]),
        as megakernel.py:1224-1301: the final norm and lm_head follow the
        last layer run."""
        L = self.cfg.n_layers if layer_count is None else int(layer_count)
        if not 1 <= L <= self.cfg.n_layers:
            raise ValueError(f"layer_count must be between 1 and {self.cfg.n_layers}")
        self.ensure_capacity(state, 1)
        sess = self._session(state)

        def run():
            if L == self.cfg.n_layers:
                logits, trace = sess.step(int(token), state["position"], want_trace=True)
            else:
                logits, trace = sess.step_layers(int(token), state["position"], L, want_trace=True)
            sess.check_status()
            return logits.clone(), trace.clone()

        out = self._guard(state, run)
        state["position"] += 1
        return out

    def make_session(self, *, max_new_tokens=512, prefill_mode: str = "chunked") -> "QATSession":
        return QATSession(self, max_new_tokens, prefill_mode)


class QATSession:
    """Prefill + scalar decode (reference quantized.py:98-151).  The prompt is
    prefilled in chunks of engine.prefill_chunk_size tokens through
    rec_prefill_chunk: projections and experts on the tensor cores, causal
    attention over the quantized cache.  Its results match the token-by-token
    decode path within a tolerance (fp32 tensor-core accumulation) and do not
    depend on where the chunks are cut.  prefill_mode="decode" runs the prompt
    through the decode step token by token instead (the cache then holds
    exactly what decoding would have written)."""

    context_limit = ModelWeights.context_limit

    def __init__(self, engine: FullModel, max_new_tokens: int, prefill_mode: str = "chunked"):
        if prefill_mode not in ("chunked", "decode"):
            raise ValueError("prefill_mode must be 'chunked' or 'decode'")
        self.prefill_mode = prefill_mode
        self.engine, self.maximum = engine, max_new_tokens
        self._state = None
        self.cached_tokens = 0
        self.common_prefix_tokens = 0
        self.prompt_cache = None

    def prefill(self, tokens, *, prefix=None, should_stop=lambda: False, interrupt_between_layers=False):
        """Chunked prefill (quantized.py:102-148).  `prefix` is the
        `prompt_cache` of an earlier session: its K/V rows for the common
        prompt prefix are reused in place (prefix.py:83-118), and only the
        rest of the prompt runs.  `should_stop` is polled before each chunk
        (PrefillCancelled); with interrupt_between_layers also before each
        layer of a chunk, each layer finished on the device before the next
        poll (model.py:309-314) — through rec_prefill_chunk_layers, with the
        same bits as the whole chunk — and on the decode-step path before
        each token."""
        from .errors import PrefillCancelled
        from .prefix import PromptCache, select_prefix

        tokens = [int(t) for t in tokens]
        limit = len(tokens) + self.maximum
        if limit > self.engine.model.context_limit:
            raise ValueError("prompt plus output allowance exceeds the context limit")
        prefix, self.common_prefix_tokens = select_prefix(prefix, tokens)
        self.cached_tokens = 0 if prefix is None else len(prefix.tokens)
        storage = None if prefix is None else prefix.storage
        state = self.engine.prefill_state(len(tokens) + 1, limit=limit, storage=storage)
        self.prompt_cache = prefix or PromptCache([], state["kv"])
        sess = self.engine._session(state)
        logits = self.prompt_cache.logits
        chunk = self.engine.prefill_chunk_size
        for begin in range(self.cached_tokens, len(tokens), chunk):
            if should_stop():
                raise PrefillCancelled()
            self.prompt_cache.checkpoint()
            part = tokens[begin:begin + chunk]
            # the tensor-core chunk path covers the routed-expert layers; a model
            # with Flint layer options (shared expert, dense / NoPE / sliding
            # layers) is prefilled by its decode step
            if self.prefill_mode == "chunked" and not self.engine.cfg.has_layer_options:
                if interrupt_between_layers:
                    n = self.engine.cfg.n_layers
                    for layer in range(n):
                        if layer and should_stop():
                            raise PrefillCancelled()
                        out = self.engine._guard(state, lambda: sess.prefill_chunk(
                            part, begin, want_logits=layer == n - 1, layers=(layer, layer + 1)))
                        self.engine._guard(state, sess.check_status)
                else:
                    out = self.engine._guard(state, lambda: sess.prefill_chunk(part, begin))
            else:
                for i, t in enumerate(part):
                    if i and interrupt_between_layers and should_stop():
                        raise PrefillCancelled()
                    out, _ = sess.step(t, begin + i, want_logits=i == len(part) - 1)
            self.engine._guard(state, sess.check_status)
            logits = out.clone()
            self.prompt_cache.advance(part, logits)
        if should_stop():
            raise PrefillCancelled()
        if logits is None:
            raise ValueError("prefill needs at least one prompt token")
        state["capacity"] = state["kv"].capacity
        state["position"] = state["initial"] = len(tokens)
        self._state = state
        return logits.clone()

    def forward_token(self, token):
        return self.engine.forward(self._state, token)[0]


class ResidentSampler:
    """Packets of up to 8 tokens decoded with the next token fed back on the
    device (reference sampling.py:62-169, resident_block.py:12-88).  The
    packet stops after one of `eos_tokens`, by default the model's own end
    ids (engine.model.eos_tokens, as sampling.py:22,99-105 reads them)."""

    def __init__(self, engine: FullModel, eos_tokens=()):
        self.engine = engine
        self.eos_tokens = list(eos_tokens) if eos_tokens else list(getattr(engine.model, "eos_tokens", ()))

    def block(self, state, token, count, seed, *, temperature=1.0, top_p=1.0, top_k=0, presence_penalty=0.0,
              grammar=None, logprobs=None):
        if not 1 <= count <= WIDTH:
            raise ValueError("Resident packet must contain between one and eight tokens")
        self.engine.ensure_capacity(state, count)
        if grammar is not None or logprobs is not None or (presence_penalty and temperature == 0):
            # the reference's filtered path (kernels/sampling.py:80-96)
            from .sampling import filtered_block

            ids = filtered_block(self.engine, state, token, count, seed, temperature=temperature, top_p=top_p,
                                 top_k=top_k, presence_penalty=presence_penalty, grammar=grammar, logprobs=logprobs,
                                 eos=self.eos_tokens)
        elif temperature != 0:
            from .sampling import sampled_block

            ids = sampled_block(self.engine, state, token, count, seed, temperature=temperature, top_p=top_p,
                                top_k=top_k, presence_penalty=presence_penalty, eos=self.eos_tokens)
        else:
            sess = self.engine._session(state)
            ids = self.engine._guard(state, lambda: sess.greedy(int(token), state["position"], count,
                                                                self.eos_tokens))
        if not 1 <= len(ids) <= count:
            raise RuntimeError("Invalid sampled chain")
        state["position"] += len(ids)
        return ids


def build_decoder(model: ModelWeights, *, optimized: bool = True, eos_tokens=()):
    """(engine, resident_sampler) for a model, as kernels.build_decoder."""
    engine = FullModel(model)
    return engine, (ResidentSampler(engine, eos_tokens) if optimized else None)


def build_decoder_from_checkpoint(directory, *, kv_format: str = "bf16", optimized: bool = True, eos_tokens=(),
                                  device="cuda"):
    """build_decoder for a reference checkpoint directory (config.json +
    model-*.safetensors, engine/src/rec_mlx/checkpoint.py:5-31): the weights
    through rec_b200.checkpoint.load_reference_checkpoint (kv_format "bf16"
    as the production engine, or "native" for MLX's K8/V4 cache)."""
    from .checkpoint import load_reference_checkpoint

    weights = load_reference_checkpoint(directory, kv_format=kv_format, device=device)
    return build_decoder(weights, optimized=optimized, eos_tokens=eos_tokens)
