"""The C-ABI library loads without a GPU and exports every function that
include/rec_b200.h declares; the ctypes mirror matches the header's
constants and structure sizes.  No compute calls."""
import ctypes as C
import re
from pathlib import Path

import pytest

from rec_b200 import _lib, abi

HEADER = Path(__file__).resolve().parents[1] / "include" / "rec_b200.h"


def _declared():
    text = HEADER.read_text()
    return re.findall(r"REC_API\s+[\w\s\*]+?\b(rec_\w+)\s*\(", text)


def _lib_or_skip():
    if not _lib.LIB_PATH.exists():
        pytest.skip("librec_b200.so not built")
    return _lib.lib()


def test_header_declares_entry_points():
    names = _declared()
    assert len(names) == len(set(names))
    for n in ("rec_create", "rec_decode_step", "rec_decode_greedy", "rec_gemv_int4", "rec_quantize_affine",
              "rec_gemv_int4_argmax_noalloc"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _lib_or_skip()
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_signatures_cover_the_header():
    assert set(_declared()) <= set(_lib._SIGNATURES)


def test_constants_match_header():
    text = HEADER.read_text()
    for name in ("REC_OK", "REC_EINVAL", "REC_ECUDA", "REC_ESTATE", "REC_ELIMIT", "REC_DEV_BULK_TIMEOUT",
                 "REC_DEV_COUNTER_TIMEOUT", "REC_DEV_BAD_TOKEN", "REC_DEV_BAD_POSITION", "REC_SCALE_FP16",
                 "REC_SCALE_BF16", "REC_ROUTER_SOFTMAX", "REC_ROUTER_SIGMOID", "REC_FLAG_SINKS", "REC_FLAG_QK_NORM",
                 "REC_LAYER_DENSE", "REC_LAYER_NO_ROPE", "REC_LAYER_SLIDING"):
        m = re.search(rf"\b{name}\s*=\s*(-?\d+)", text)
        assert m, name
        assert int(m.group(1)) == getattr(abi, name), name


def test_struct_sizes():
    p = C.sizeof(C.c_void_p)
    assert C.sizeof(abi.RecModelDesc) == 21 * 4
    assert C.sizeof(abi.RecQMat) == 3 * p
    # pointers, then the int32 kind (padded to a pointer) and the shared expert
    assert C.sizeof(abi.RecLayerWeights) == (2 + 4 * 3 + 2 + 3 * 3 + 3 + 1 + 3 * 3) * p
    assert C.sizeof(abi.RecGlobalWeights) == (3 + 1 + 3) * p
    assert C.sizeof(abi.RecKVLayer) == 6 * p


def test_argument_errors_need_no_device():
    lib = _lib_or_skip()
    out = C.c_void_p()
    desc = abi.RecModelDesc(hidden=1000, n_layers=1, n_q_heads=32, n_kv_heads=4, head_dim=128, n_experts=8,
                            top_k=2, moe_inter=256, vocab=64, group_size=64)
    assert lib.rec_create(C.byref(desc), C.byref(out)) == abi.REC_EINVAL
    assert "hidden" in _lib.last_error().lower()


def test_schedule_rule_needs_no_device(monkeypatch):
    """rec_schedule_for: the persistent kernel below 24 MiB of attended KV per
    layer, the graph above; REC_SCHEDULE forces any of the three (split only
    when forced); more than 256 experts always take the graph."""
    lib = _lib_or_skip()

    def ctx(kv_bits, n_experts=128):
        desc = abi.RecModelDesc(hidden=2048, n_layers=2, n_q_heads=32, n_kv_heads=4, head_dim=128,
                                n_experts=n_experts, top_k=8, moe_inter=768, vocab=4096, group_size=64,
                                kv_bits=kv_bits)
        out = C.c_void_p()
        assert lib.rec_create(C.byref(desc), C.byref(out)) == abi.REC_OK, _lib.last_error()
        return out

    monkeypatch.delenv("REC_SCHEDULE", raising=False)
    c4, c8 = ctx(4), ctx(8)
    for c, per_token in ((c4, 4 * 144), (c8, 4 * 272)):
        edge = 24 * 1024 * 1024 // per_token  # tokens at which the persistent kernel stops
        assert lib.rec_schedule_for(c, 1023) == 0
        assert lib.rec_schedule_for(c, edge - 2) == 0
        assert lib.rec_schedule_for(c, edge + 1) == 1
        assert lib.rec_schedule_for(c, 258047) == 1
    monkeypatch.setenv("REC_SCHEDULE", "mega")
    assert lib.rec_schedule_for(c4, 258047) == 0
    monkeypatch.setenv("REC_SCHEDULE", "graph")
    assert lib.rec_schedule_for(c4, 10) == 1
    monkeypatch.setenv("REC_SCHEDULE", "split")
    assert lib.rec_schedule_for(c4, 10) == 2
    monkeypatch.delenv("REC_SCHEDULE")
    c512 = ctx(8, n_experts=512)
    assert lib.rec_schedule_for(c512, 10) == 1
    assert lib.rec_schedule_for(None, 10) == -1
    # a model with a shared expert (a Flint layer option) runs on the graph
    desc = abi.RecModelDesc(hidden=2048, n_layers=2, n_q_heads=32, n_kv_heads=4, head_dim=128, n_experts=16,
                            top_k=4, moe_inter=768, vocab=4096, group_size=64, kv_bits=8, shared_inter=1024)
    cs = C.c_void_p()
    assert lib.rec_create(C.byref(desc), C.byref(cs)) == abi.REC_OK, _lib.last_error()
    monkeypatch.setenv("REC_SCHEDULE", "mega")
    assert lib.rec_schedule_for(cs, 10) == 1
    monkeypatch.delenv("REC_SCHEDULE")
    for c in (c4, c8, c512, cs):
        lib.rec_destroy(c)


def test_flint_options_are_checked_without_a_device():
    """Shared expert, dense-MLP and sliding-window sizes outside the kernels'
    shapes are refused at rec_create."""
    lib = _lib_or_skip()

    def create(**kw):
        base = dict(hidden=2048, n_layers=2, n_q_heads=32, n_kv_heads=4, head_dim=128, n_experts=16, top_k=4,
                    moe_inter=768, vocab=4096, group_size=64, kv_bits=8)
        base.update(kw)
        desc = abi.RecModelDesc(**base)
        out = C.c_void_p()
        rc = lib.rec_create(C.byref(desc), C.byref(out))
        if rc == abi.REC_OK:
            lib.rec_destroy(out)
        return rc

    assert create(shared_inter=1024, dense_inter=6144, sliding_window=513) == abi.REC_OK
    assert create(shared_inter=300) == abi.REC_EINVAL
    assert create(dense_inter=3000) == abi.REC_EINVAL
    assert create(sliding_window=-1) == abi.REC_EINVAL
    assert create(embed_bits=8) == abi.REC_OK
    assert create(embed_bits=3) == abi.REC_EINVAL
    assert create(kv_value_bits=4) == abi.REC_OK  # K 8-bit, V 4-bit: the reference's mixed cache
    assert create(kv_bits=16, kv_value_bits=4) == abi.REC_EINVAL
