"""A decode session on one GPU: the C-ABI context with its weights, KV cache
and workspace (all device memory owned by torch)."""
from __future__ import annotations

import ctypes as C

import torch

from . import abi
from ._lib import RecError, check, lib
from .model import KVCache, ModelWeights


class DecodeSession:
    """One decode session; with `plan` (rec_b200.shard.ShardPlan) and a
    process group it is this rank's part of a session split over the group's
    GPUs: `weights` hold the plan's experts, `kv` its local capacity, and every
    rank must make the same calls in the same order."""

    def __init__(self, weights: ModelWeights, kv: KVCache, plan=None, group=None, shard_schedule: str = "mega"):
        """shard_schedule (split sessions): "mega" runs the persistent kernel
        with the exchanges inside it; "graph" runs the CUDA graph of
        standalone kernels (attention on this rank's KV with the standalone
        kernel, the exchanges as separate kernels).  Fixed for the session."""
        if shard_schedule not in ("mega", "graph"):
            raise ValueError("shard_schedule must be 'mega' or 'graph'")
        self.weights = weights
        self.kv = kv
        self.cfg = weights.cfg
        self.plan = plan
        self._desc = self.cfg.desc()
        handle = C.c_void_p()
        check(lib().rec_create(C.byref(self._desc), C.byref(handle)), "rec_create")
        self.ctx = handle
        if plan is not None:
            self._shard = abi.RecShard(plan.world, plan.rank, plan.expert_lo, plan.expert_hi, plan.super_lo,
                                       plan.super_hi, plan.capacity)
            self._shard.schedule = 1 if shard_schedule == "graph" else 0
            check(lib().rec_set_shard(self.ctx, C.byref(self._shard)), "rec_set_shard")
        self._layers = weights.rec_layers()
        self._global = weights.rec_global()
        check(lib().rec_set_weights(self.ctx, self._layers, len(weights.layers), C.byref(self._global)),
              "rec_set_weights")
        self._kv = kv.rec()
        check(lib().rec_set_kv(self.ctx, self._kv, len(kv.layers), kv.capacity), "rec_set_kv")
        if kv.rows < kv.capacity:
            check(lib().rec_set_kv_rows(self.ctx, kv.rows), "rec_set_kv_rows")
        if plan is not None:
            self._setup_exchange(group)
        nbytes = lib().rec_workspace_bytes(self.ctx)
        self.workspace = torch.empty(nbytes + 256, dtype=torch.uint8, device=kv.layers[0]["k_codes"].device)
        base = self.workspace.data_ptr()
        aligned = (base + 255) // 256 * 256
        check(lib().rec_set_workspace(self.ctx, C.c_void_p(aligned), nbytes), "rec_set_workspace")
        dev = self.workspace.device
        self.logits = torch.empty(self.cfg.vocab, dtype=torch.bfloat16, device=dev)
        self.trace = torch.empty(self.cfg.n_layers + 1, self.cfg.hidden, dtype=torch.bfloat16, device=dev)
        self.ids = torch.zeros(64, dtype=torch.int32, device=dev)
        self.produced = torch.zeros(1, dtype=torch.int32, device=dev)
        self.usable = True

    def _setup_exchange(self, group):
        """Peer-mapped exchange buffers (torch symmetric memory over the
        group), zeroed on every rank before any launch."""
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        nbytes = int(lib().rec_exchange_bytes(self.ctx))
        dev = self.kv.layers[0]["k_codes"].device
        try:
            symm.set_backend("CUDA")
        except Exception:  # already chosen by an earlier allocation
            pass
        group = group if group is not None else dist.group.WORLD
        self.exchange = symm.empty(nbytes, dtype=torch.uint8, device=dev)
        self.exchange.zero_()
        torch.cuda.synchronize(dev)
        self._symm = symm.rendezvous(self.exchange, group)
        ptrs = list(self._symm.buffer_ptrs)
        if len(ptrs) != self.plan.world:
            raise RuntimeError("symmetric memory group size does not match the shard plan")
        for q, p in enumerate(ptrs):
            self._shard.exchange[q] = p
        check(lib().rec_set_shard(self.ctx, C.byref(self._shard)), "rec_set_shard")
        dist.barrier(group=group)

    def set_rows(self, rows: int) -> None:
        """The cache now backs rows [0, rows) (a reserved cache that grew in
        place; rec_set_kv_rows)."""
        check(lib().rec_set_kv_rows(self.ctx, int(rows)), "rec_set_kv_rows")

    def __del__(self):
        ctx = getattr(self, "ctx", None)
        if ctx:
            try:
                lib().rec_destroy(ctx)
            except Exception:
                pass
            self.ctx = None

    @staticmethod
    def _stream():
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def step(self, token: int, position: int, want_trace: bool = False, want_logits: bool = True):
        """One decode step; returns (logits bf16[V] or None, trace bf16[L+1, H] or None)."""
        check(lib().rec_decode_step(self.ctx, int(token), int(position),
                                    C.c_void_p(self.logits.data_ptr()) if want_logits else None,
                                    C.c_void_p(self.trace.data_ptr()) if want_trace else None, self._stream()),
              "rec_decode_step")
        return (self.logits if want_logits else None), (self.trace if want_trace else None)

    def step_layers(self, token: int, position: int, layer_count: int, want_trace: bool = True):
        """One decode step through the first `layer_count` layers only
        (rec_decode_layers); returns (logits bf16[V], trace bf16[layer_count
        + 1, H] or None)."""
        check(lib().rec_decode_layers(self.ctx, int(token), int(position), int(layer_count),
                                      C.c_void_p(self.logits.data_ptr()),
                                      C.c_void_p(self.trace.data_ptr()) if want_trace else None, self._stream()),
              "rec_decode_layers")
        return self.logits, (self.trace[: layer_count + 1] if want_trace else None)

    def prefill(self, tokens, start: int = 0) -> None:
        """Runs tokens through the decode step at positions start.. (fills the
        cache exactly as decoding would)."""
        for i, t in enumerate(tokens):
            self.step(int(t), start + i, want_logits=False)
        self.check_status()

    def prefill_chunk(self, tokens, start: int, want_logits: bool = True, layers: tuple[int, int] | None = None):
        """One prompt chunk at positions start.. through rec_prefill_chunk
        (tensor-core projections and experts, causal attention over the
        quantized cache); returns the last token's logits (bf16 [V]) or None.
        Results are independent of how a prompt is cut into chunks.
        `layers` = (begin, end) runs only those layers
        (rec_prefill_chunk_layers): the ranges of one chunk are called in
        order with the same tokens and start, and the logits come with the
        range that ends at the last layer."""
        t = len(tokens)
        dev = self.workspace.device
        nbytes = int(lib().rec_prefill_workspace_bytes(self.ctx, t))
        ws = getattr(self, "_pf_ws", None)
        if ws is None or ws.numel() < nbytes + 256:
            if layers is not None and layers[0] > 0:
                raise ValueError("a layer range after the first needs the workspace of its chunk")
            ws = self._pf_ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
        base = (ws.data_ptr() + 255) // 256 * 256
        tok = torch.tensor([int(x) for x in tokens], dtype=torch.int32, device=dev)
        out = C.c_void_p(self.logits.data_ptr()) if want_logits else None
        if layers is None:
            check(lib().rec_prefill_chunk(self.ctx, C.c_void_p(tok.data_ptr()), int(start), t, out, C.c_void_p(base),
                                          nbytes, self._stream()), "rec_prefill_chunk")
        else:
            check(lib().rec_prefill_chunk_layers(self.ctx, C.c_void_p(tok.data_ptr()), int(start), t, int(layers[0]),
                                                 int(layers[1]), out, C.c_void_p(base), nbytes, self._stream()),
                  "rec_prefill_chunk_layers")
        self._pf_tokens = tok  # alive until the stream has read it
        return self.logits if want_logits else None

    def greedy(self, token: int, position: int, count: int, eos=()):
        """Up to `count` greedy tokens with device-side feedback; stops after
        an EOS id.  Returns the produced ids (host list)."""
        eos = list(eos)
        arr = (C.c_int32 * max(1, len(eos)))(*eos) if eos else None
        check(lib().rec_decode_greedy(self.ctx, int(token), int(position), int(count), arr, len(eos),
                                      C.c_void_p(self.ids.data_ptr()), C.c_void_p(self.produced.data_ptr()),
                                      self._stream()), "rec_decode_greedy")
        self.check_status()
        n = int(self.produced.item())
        return self.ids[:n].tolist()

    def greedy_async(self, token: int, position: int, count: int, eos=()) -> None:
        """Enqueues a greedy packet without synchronising (ids stay on device)."""
        eos = list(eos)
        arr = (C.c_int32 * max(1, len(eos)))(*eos) if eos else None
        check(lib().rec_decode_greedy(self.ctx, int(token), int(position), int(count), arr, len(eos),
                                      C.c_void_p(self.ids.data_ptr()), C.c_void_p(self.produced.data_ptr()),
                                      self._stream()), "rec_decode_greedy")

    def check_status(self) -> None:
        s = lib().rec_check_status(self.ctx, self._stream())
        if s > 0:
            self.usable = False
            raise RecError(f"GPU synchronization failed: device status {s}")
        if s < 0:
            check(s, "rec_check_status")
