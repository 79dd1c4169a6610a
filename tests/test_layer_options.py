"""Host-side checks of the Flint layer options (no device needed): the full
Flint configuration pins the shape the reference's megakernel asserts, and
rec_set_weights accepts or refuses layer kinds and their matrices by the
rules of include/rec_b200.h.  The pointers here are 16-byte-aligned host
buffers that no kernel ever reads (rec_set_weights only records them)."""
import ctypes as C

import numpy as np
import pytest

from rec_b200 import _lib, abi
from rec_b200.model import FLINT, TINY_FLINT, config_from_reference


def test_flint_config_is_the_reference_shape():
    """megakernel.py:992-1004: 49 layers, hidden 2048, (heads, kv heads,
    head dim, experts, top-k, window, vocab) = (32, 4, 128, 256, 6, 513,
    150144); model.py:14-37: dense layers 0-1 of 6,144, routed 512, shared
    1,024; mixed_bits.py:25: an int8 embedding."""
    c = FLINT
    assert (c.n_layers, c.hidden) == (49, 2048)
    assert (c.n_q_heads, c.n_kv_heads, c.head_dim, c.n_experts, c.top_k, c.sliding_window, c.vocab) == \
        (32, 4, 128, 256, 6, 513, 150144)
    assert (c.dense_layers, c.dense_inter, c.moe_inter, c.shared_inter, c.embed_bits) == ((0, 1), 6144, 512, 1024, 8)
    assert c.router_mode == abi.REC_ROUTER_SIGMOID and c.kv_bits == 16
    assert set(c.no_rope_layers).isdisjoint(c.sliding_layers)
    assert set(c.no_rope_layers) | set(c.sliding_layers) == set(range(49))
    d = c.desc()
    assert (d.shared_inter, d.dense_inter, d.sliding_window, d.embed_bits, d.kv_bits) == (1024, 6144, 513, 8, 16)
    kinds = [c.layer_kind(i) for i in range(49)]
    assert kinds[0] & abi.REC_LAYER_DENSE and kinds[1] & abi.REC_LAYER_DENSE
    assert not any(k & abi.REC_LAYER_DENSE for k in kinds[2:])


class _Host:
    """Aligned host buffers standing in for device weights (never read)."""

    def __init__(self):
        self.keep = []

    def ptr(self):
        a = np.zeros(64, np.uint8)
        self.keep.append(a)
        return (a.ctypes.data + 15) // 16 * 16

    def qmat(self):
        return abi.RecQMat(self.ptr(), self.ptr(), self.ptr())


def _layers(cfg, h: _Host, drop_shared=None, kind_override=None):
    out = []
    for i in range(cfg.n_layers):
        kind = cfg.layer_kind(i) if kind_override is None or i != kind_override[0] else kind_override[1]
        dense = kind & abi.REC_LAYER_DENSE
        shared = cfg.shared_inter and not dense and i != drop_shared
        L = abi.RecLayerWeights(
            input_norm=h.ptr(), post_norm=h.ptr(), q=h.qmat(), k=h.qmat(), v=h.qmat(), o=h.qmat(),
            router=None if dense else h.ptr(), expert_bias=h.ptr(), gate=h.qmat(), up=h.qmat(), down=h.qmat(),
            sinks=h.ptr(), q_norm=h.ptr(), k_norm=h.ptr(), kind=kind,
            shared_gate=h.qmat() if shared else abi.RecQMat(), shared_up=h.qmat() if shared else abi.RecQMat(),
            shared_down=h.qmat() if shared else abi.RecQMat())
        out.append(L)
    return (abi.RecLayerWeights * len(out))(*out)


def _set(cfg, layers, h):
    lib = _lib.lib()
    ctx = C.c_void_p()
    desc = cfg.desc()
    assert lib.rec_create(C.byref(desc), C.byref(ctx)) == abi.REC_OK, _lib.last_error()
    g = abi.RecGlobalWeights(embed=h.qmat(), final_norm=h.ptr(), lm_head=h.qmat())
    try:
        return lib.rec_set_weights(ctx, layers, cfg.n_layers, C.byref(g)), _lib.last_error()
    finally:
        lib.rec_destroy(ctx)


@pytest.fixture
def built():
    if not _lib.LIB_PATH.exists():
        pytest.skip("librec_b200.so not built")


def test_layer_options_accepted(built):
    h = _Host()
    rc, msg = _set(TINY_FLINT, _layers(TINY_FLINT, h), h)
    assert rc == abi.REC_OK, msg


def test_shared_expert_matrices_required(built):
    h = _Host()
    rc, msg = _set(TINY_FLINT, _layers(TINY_FLINT, h, drop_shared=1), h)
    assert rc == abi.REC_EINVAL and "shared-expert" in msg


def test_unknown_kind_bits_refused(built):
    h = _Host()
    rc, msg = _set(TINY_FLINT, _layers(TINY_FLINT, h, kind_override=(1, 64)), h)
    assert rc == abi.REC_EINVAL and "kind" in msg


def test_sliding_layer_needs_a_window(built):
    from dataclasses import replace

    cfg = replace(TINY_FLINT, sliding_layers=())  # desc.sliding_window = 0
    h = _Host()
    rc, msg = _set(cfg, _layers(cfg, h, kind_override=(2, abi.REC_LAYER_SLIDING)), h)
    assert rc == abi.REC_EINVAL and "sliding" in msg


def test_dense_layer_needs_dense_inter(built):
    from dataclasses import replace

    cfg = replace(TINY_FLINT, dense_layers=())  # desc.dense_inter = 0
    h = _Host()
    rc, msg = _set(cfg, _layers(cfg, h, kind_override=(0, abi.REC_LAYER_DENSE)), h)
    assert rc == abi.REC_EINVAL and "dense" in msg


def _flint_config_json():
    """A config.json of the reference's shape (ModelArgs fields and the export
    keys checkpoint.py checks), with FLINT's assumed global layers."""
    glob = list(FLINT.no_rope_layers)
    return {"model_type": "flint", "num_hidden_layers": 49, "vocab_size": 150144, "mlp_only_layers": [0, 1],
            "layer_types": ["full_attention" if i in glob else "sliding_attention" for i in range(49)],
            "no_rope_layer_indices": glob, "sliding_window": 513, "rope_theta": 10000.0,
            "quantization": {"group_size": 64, "bits": 4},
            "mlx_export": {"bits": 4, "routed_expert_bits": 4, "embedding_bits": 8}}


def test_config_from_reference_is_the_flint_shape():
    got = config_from_reference(_flint_config_json(), name=FLINT.name)
    assert got == FLINT
    native = config_from_reference(_flint_config_json(), kv_format="native")
    assert (native.kv_bits, native.kv_value_bits, native.v_bits) == (8, 4, 4)


def test_config_from_reference_refuses_what_the_kernels_do_not_take():
    base = _flint_config_json()
    for change in ({"tie_word_embeddings": True}, {"kv_group_size": 32},
                   {"mlx_export": {"bits": 4, "routed_expert_bits": 3, "embedding_bits": 8}},
                   {"quantization": {"group_size": 32, "bits": 4}},
                   {"layer_types": ["chunked_attention"] * 49}):
        with pytest.raises(ValueError):
            config_from_reference({**base, **change})
    with pytest.raises(ValueError):
        config_from_reference(base, kv_format="fp8")


def test_config_from_reference_creates_a_session(built):
    lib = _lib.lib()
    for fmt in ("bf16", "native"):
        desc = config_from_reference(_flint_config_json(), kv_format=fmt).desc()
        ctx = C.c_void_p()
        assert lib.rec_create(C.byref(desc), C.byref(ctx)) == abi.REC_OK, _lib.last_error()
        lib.rec_destroy(ctx)
