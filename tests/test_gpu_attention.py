"""Decode attention of one layer through rec_attn_decode against the oracle,
bit for bit: the appended K/V row and the output, over ragged contexts
(1 token, partial tiles, block / item / super-chunk edges) and both cache
widths.  The RoPE table is the identity so the oracle sees q as given."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle
from rec_b200 import abi

pytestmark = pytest.mark.gpu

# the last three are config 2's long contexts (131,072 and 258,048 tokens)
CASES = [(1, 8), (37, 4), (256, 8), (257, 4), (1028, 8), (1028, 4), (4097, 8), (16384, 8), (16385, 4), (20000, 8),
         (70000, 4), (131072, 8), (258048, 4), (258048, 8)]


def _dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    elif a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).cuda()


def _host(t, dt):
    return t.cpu().numpy().view(dt)


@pytest.mark.parametrize("T,bits", CASES)
@pytest.mark.parametrize("heads", [(32, 4), (16, 2)])
def test_attention_matches_oracle(cuda, T, bits, heads):
    from rec_b200._lib import check, lib

    hq, hkv = heads
    if hq == 16 and T > 5000:
        pytest.skip("one long case per head count is enough")
    rng = np.random.default_rng(T * 10 + bits + hq)
    cap = (T + 255) // 256 * 256
    words = 128 * bits // 32
    kv = {}
    for n in ("k", "v"):
        x = oracle.bf16_to_f32(oracle.f32_to_bf16(rng.standard_normal((hkv, T - 1, 128), dtype=np.float32)))
        c, s, b = oracle.quantize(x, bits, 1) if T > 1 else (np.zeros((hkv, 0, words), np.uint32),
                                                             np.zeros((hkv, 0, 2), np.uint16),
                                                             np.zeros((hkv, 0, 2), np.uint16))
        kv[f"{n}_codes"] = np.zeros((hkv, cap, words), np.uint32)
        kv[f"{n}_scales"] = np.zeros((hkv, cap, 2), np.uint16)
        kv[f"{n}_biases"] = np.zeros((hkv, cap, 2), np.uint16)
        kv[f"{n}_codes"][:, : T - 1] = c
        kv[f"{n}_scales"][:, : T - 1] = s
        kv[f"{n}_biases"][:, : T - 1] = b
    qkv = oracle.f32_to_bf16(rng.standard_normal((hq + 2 * hkv) * 128, dtype=np.float32))
    sinks = oracle.f32_to_bf16(rng.standard_normal(hq, dtype=np.float32)) if T % 2 else None
    dev = {n: _dev(a) for n, a in kv.items()}
    rec = abi.RecKVLayer(*(dev[n].data_ptr() for n in ("k_codes", "k_scales", "k_biases", "v_codes", "v_scales",
                                                      "v_biases")))
    rope = torch.zeros(cap, 128, dtype=torch.float32, device="cuda")
    rope[:, :64] = 1.0
    pos = torch.tensor([T - 1], dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    nbytes = lib().rec_attn_scratch_bytes(hq, cap)
    scratch = torch.empty(nbytes + 256, dtype=torch.uint8, device="cuda")
    base = (scratch.data_ptr() + 255) // 256 * 256
    out = torch.empty(hq * 128, dtype=torch.int16, device="cuda")
    qkv_d = _dev(qkv)
    sk = _dev(sinks) if sinks is not None else None
    check(lib().rec_attn_decode(C.c_void_p(qkv_d.data_ptr()), hq, hkv, C.byref(rec), cap, bits,
                                C.c_void_p(rope.data_ptr()), C.c_void_p(sk.data_ptr()) if sk is not None else None,
                                C.c_void_p(pos.data_ptr()), C.c_void_p(base), nbytes, C.c_void_p(out.data_ptr()),
                                C.c_void_p(status.data_ptr()), C.c_void_p(torch.cuda.current_stream().cuda_stream)),
          "rec_attn_decode")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    # oracle: append the new row, then attend
    lay = {n: a.copy() for n, a in kv.items()}
    arrs = [lay[n] for n in ("k_codes", "k_scales", "k_biases", "v_codes", "v_scales", "v_biases")]
    orec = abi.RecKVLayer(*(a.ctypes.data for a in arrs))
    L = oracle.lib()
    L.orc_kv_store.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    k_new = np.ascontiguousarray(qkv[hq * 128:(hq + hkv) * 128])
    v_new = np.ascontiguousarray(qkv[(hq + hkv) * 128:])
    L.orc_kv_store(C.addressof(orec), hkv, cap, bits, T - 1, k_new.ctypes.data, v_new.ctypes.data)
    for n in lay:
        got = _host(dev[n], lay[n].dtype)
        assert np.array_equal(got[:, T - 1], lay[n][:, T - 1]), n
    n_super = -(-((T + 255) // 256) // 64)
    sup = oracle.attention_supers(qkv[: hq * 128], lay, hkv, cap, bits, T, n_super)
    want = oracle.attention_final(sup, sinks)
    got = _host(out, np.uint16)
    bad = np.flatnonzero(got != want)
    assert bad.size == 0, (bad[:8], got[bad[:8]], want[bad[:8]])


@pytest.mark.parametrize("bits", [4, 8])
def test_kv_append_matches_oracle(cuda, bits):
    """rec_kv_append (quantize-on-append alone) against the oracle's append,
    bit for bit, and an out-of-range position reported without a write."""
    from rec_b200._lib import check, lib

    hkv, cap, pos = 4, 512, 301
    rng = np.random.default_rng(bits)
    words = 128 * bits // 32
    kv = {}
    for n in ("k", "v"):
        kv[f"{n}_codes"] = np.zeros((hkv, cap, words), np.uint32)
        kv[f"{n}_scales"] = np.zeros((hkv, cap, 2), np.uint16)
        kv[f"{n}_biases"] = np.zeros((hkv, cap, 2), np.uint16)
    k_new = oracle.f32_to_bf16(3.0 * rng.standard_normal(hkv * 128, dtype=np.float32))
    v_new = oracle.f32_to_bf16(rng.standard_normal(hkv * 128, dtype=np.float32))
    dev = {n: _dev(a) for n, a in kv.items()}
    rec = abi.RecKVLayer(*(dev[n].data_ptr() for n in ("k_codes", "k_scales", "k_biases", "v_codes", "v_scales",
                                                      "v_biases")))
    kd, vd = _dev(k_new), _dev(v_new)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for p, want_status in ((pos, 0), (cap, 4)):
        pd = torch.tensor([p], dtype=torch.int32, device="cuda")
        check(lib().rec_kv_append(C.byref(rec), hkv, cap, bits, C.c_void_p(kd.data_ptr()), C.c_void_p(vd.data_ptr()),
                                  C.c_void_p(pd.data_ptr()), C.c_void_p(status.data_ptr()), stream), "rec_kv_append")
        torch.cuda.synchronize()
        assert int(status.item()) == want_status
    lay = {n: a.copy() for n, a in kv.items()}
    arrs = [lay[n] for n in ("k_codes", "k_scales", "k_biases", "v_codes", "v_scales", "v_biases")]
    orec = abi.RecKVLayer(*(a.ctypes.data for a in arrs))
    L = oracle.lib()
    L.orc_kv_store.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    L.orc_kv_store(C.addressof(orec), hkv, cap, bits, pos, k_new.ctypes.data, v_new.ctypes.data)
    for n in lay:
        assert np.array_equal(_host(dev[n], lay[n].dtype), lay[n]), n


@pytest.mark.parametrize("bits", [4, 8])
def test_kv_append_bulk_matches_oracle(cuda, bits):
    """rec_kv_append_bulk (a prefill chunk's quantize-on-append) against the
    oracle's per-row append, bit for bit, for 77 rows at an odd start; rows
    past the capacity are refused before any write."""
    from rec_b200._lib import check, lib

    hkv, cap, p0, t = 4, 512, 123, 77
    rng = np.random.default_rng(10 + bits)
    words = 128 * bits // 32
    kv = {}
    for n in ("k", "v"):
        kv[f"{n}_codes"] = np.zeros((hkv, cap, words), np.uint32)
        kv[f"{n}_scales"] = np.zeros((hkv, cap, 2), np.uint16)
        kv[f"{n}_biases"] = np.zeros((hkv, cap, 2), np.uint16)
    k_new = oracle.f32_to_bf16(3.0 * rng.standard_normal((t, hkv * 128), dtype=np.float32))
    v_new = oracle.f32_to_bf16(rng.standard_normal((t, hkv * 128), dtype=np.float32))
    dev = {n: _dev(a) for n, a in kv.items()}
    rec = abi.RecKVLayer(*(dev[n].data_ptr() for n in ("k_codes", "k_scales", "k_biases", "v_codes", "v_scales",
                                                      "v_biases")))
    kd, vd = _dev(k_new), _dev(v_new)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    check(lib().rec_kv_append_bulk(C.byref(rec), hkv, cap, bits, C.c_void_p(kd.data_ptr()), C.c_void_p(vd.data_ptr()),
                                   p0, t, stream), "rec_kv_append_bulk")
    with pytest.raises(ValueError):
        check(lib().rec_kv_append_bulk(C.byref(rec), hkv, cap, bits, C.c_void_p(kd.data_ptr()),
                                       C.c_void_p(vd.data_ptr()), cap - 10, t, stream), "rec_kv_append_bulk")
    torch.cuda.synchronize()
    lay = {n: a.copy() for n, a in kv.items()}
    arrs = [lay[n] for n in ("k_codes", "k_scales", "k_biases", "v_codes", "v_scales", "v_biases")]
    orec = abi.RecKVLayer(*(a.ctypes.data for a in arrs))
    L = oracle.lib()
    L.orc_kv_store.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    for j in range(t):
        kj, vj = np.ascontiguousarray(k_new[j]), np.ascontiguousarray(v_new[j])
        L.orc_kv_store(C.addressof(orec), hkv, cap, bits, p0 + j, kj.ctypes.data, vj.ctypes.data)
    for n in lay:
        assert np.array_equal(_host(dev[n], lay[n].dtype), lay[n]), n
