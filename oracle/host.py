"""Host-memory copy of a model for the C oracle's full decode step — TEST
INFRASTRUCTURE ONLY (see oracle/__init__.py)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from rec_b200 import abi

from . import lib


def _np(t) -> np.ndarray:
    """torch tensor (or numpy array) -> contiguous host numpy (uint16 for
    16-bit, uint32 for int32).  The array shares memory with a fresh host copy
    of the tensor; no second copy is made."""
    if isinstance(t, np.ndarray):
        return np.ascontiguousarray(t)
    import torch

    t = t.detach().contiguous()
    t = t.cpu() if t.is_cuda else t.clone()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.int32:
        return t.numpy().view(np.uint32)
    return t.numpy()


class HostModel:
    """Holds numpy copies of a rec_b200.model.ModelWeights and runs the
    oracle's decode step on them."""

    def __init__(self, weights):
        self.cfg = weights.cfg
        self.desc = self.cfg.desc()
        self._arrays = []

        def keep(a):
            self._arrays.append(a)
            return a.ctypes.data

        def q(qt):
            return abi.RecQMat(keep(_np(qt.w)), keep(_np(qt.s)), keep(_np(qt.b)))

        def opt(t):
            return None if t is None else keep(_np(t))

        def qopt(qt):
            return abi.RecQMat() if qt is None else q(qt)

        layers = []
        for L in weights.layers:
            layers.append(abi.RecLayerWeights(
                input_norm=keep(_np(L.input_norm)), post_norm=keep(_np(L.post_norm)), q=q(L.q), k=q(L.k),
                v=q(L.v), o=q(L.o), router=opt(L.router), expert_bias=opt(L.expert_bias), gate=q(L.gate),
                up=q(L.up), down=q(L.down), sinks=opt(L.sinks), q_norm=opt(L.q_norm), k_norm=opt(L.k_norm),
                kind=getattr(L, "kind", 0), shared_gate=qopt(getattr(L, "shared_gate", None)),
                shared_up=qopt(getattr(L, "shared_up", None)), shared_down=qopt(getattr(L, "shared_down", None))))
        self.layers = (abi.RecLayerWeights * len(layers))(*layers)
        self.glob = abi.RecGlobalWeights(embed=q(weights.embed), final_norm=keep(_np(weights.final_norm)),
                                         lm_head=q(weights.lm_head))
        L = lib()
        L.orc_decode_step.argtypes = [C.POINTER(abi.RecModelDesc), C.POINTER(abi.RecLayerWeights),
                                      C.POINTER(abi.RecGlobalWeights), C.POINTER(abi.RecKVLayer), C.c_int,
                                      C.c_int, C.c_int, C.c_void_p, C.c_void_p]

    def new_kv(self, capacity: int) -> "HostKV":
        return HostKV(self.cfg, capacity)

    def step(self, kv: "HostKV", token: int, pos: int, want_trace: bool = True, layer_count: int | None = None):
        """One decode step; with layer_count, only the first layer_count
        layers run before the final norm and lm_head (FullModel.forward's
        partial depth)."""
        cfg = self.cfg
        desc = self.desc
        n = cfg.n_layers
        if layer_count is not None and layer_count != cfg.n_layers:
            n = int(layer_count)
            desc = abi.RecModelDesc.from_buffer_copy(self.desc)
            desc.n_layers = n
        logits = np.zeros(cfg.vocab, np.uint16)
        trace = np.zeros((n + 1, cfg.hidden), np.uint16) if want_trace else None
        rc = lib().orc_decode_step(C.byref(desc), self.layers, C.byref(self.glob), kv.rec, kv.capacity,
                                   int(token), int(pos), logits.ctypes.data,
                                   trace.ctypes.data if trace is not None else None)
        if rc != 0:
            raise ValueError("oracle decode step rejected its inputs")
        return logits, trace


class HostKV:
    def __init__(self, cfg, capacity: int):
        vbits = getattr(cfg, "kv_value_bits", 0) or cfg.kv_bits
        words = {"k": 128 * cfg.kv_bits // 32, "v": 128 * vbits // 32}
        self.capacity = capacity
        self.layers = []
        recs = []
        for _ in range(cfg.n_layers):
            L = {}
            for kv in ("k", "v"):
                L[f"{kv}_codes"] = np.zeros((cfg.n_kv_heads, capacity, words[kv]), np.uint32)
                L[f"{kv}_scales"] = np.zeros((cfg.n_kv_heads, capacity, 2), np.uint16)
                L[f"{kv}_biases"] = np.zeros((cfg.n_kv_heads, capacity, 2), np.uint16)
            self.layers.append(L)
            recs.append(abi.RecKVLayer(*(L[n].ctypes.data for n in ("k_codes", "k_scales", "k_biases", "v_codes",
                                                                     "v_scales", "v_biases"))))
        self.rec = (abi.RecKVLayer * len(recs))(*recs)

    @classmethod
    def from_device(cls, cfg, kvcache) -> "HostKV":
        h = cls(cfg, kvcache.capacity)
        for dst, src in zip(h.layers, kvcache.layers):
            for name in dst:
                a = _np(src[name])  # a reserved cache's codes cover its backed rows only
                dst[name][:, : a.shape[1]] = a
        return h
