"""The tensor-core prefill projection (rec_prefill_gemm, tcgen05) against an
fp64 GEMM of the dequantized int4 weights.  Each dequantized weight enters
the MMAs as two bf16 parts (~16 significant bits) and Y is rounded to bf16,
so the bound is a relative L2 error of 4e-3 per row and no element off by
more than 2% of its row's RMS."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle
from rec_b200 import abi

pytestmark = pytest.mark.gpu

CASES = [(128, 64, 256), (128, 2048, 256), (200, 2048, 512), (1000, 768, 2048), (1024, 2048, 4096)]


@pytest.mark.parametrize("T,K,N", CASES)
@pytest.mark.parametrize("sd", [0, 1])
def test_prefill_gemm_matches_fp64(cuda, T, K, N, sd):
    from rec_b200._lib import check, lib

    rng = np.random.default_rng(T + K + N + sd)
    w = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    codes, scales, biases = oracle.quantize(w, 4, sd)
    wd = oracle.dequantize(codes, scales, biases, 4, sd).reshape(N, K).astype(np.float64)
    x = oracle.f32_to_bf16(rng.standard_normal((T, K), dtype=np.float32))
    want = oracle.bf16_to_f32(x).astype(np.float64) @ wd.T

    def dev(a):
        a = np.ascontiguousarray(a)
        return torch.from_numpy(a.view(np.int32) if a.dtype == np.uint32 else a.view(np.int16)).cuda()

    cd, sdv, bd, xd = dev(codes.reshape(N, -1)), dev(scales.reshape(N, -1)), dev(biases.reshape(N, -1)), dev(x)
    y = torch.zeros(T, N, dtype=torch.int16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    m = abi.RecQMat(cd.data_ptr(), sdv.data_ptr(), bd.data_ptr())
    check(lib().rec_prefill_gemm(C.byref(m), sd, N, K, C.c_void_p(xd.data_ptr()), T, C.c_void_p(y.data_ptr()),
                                 C.c_void_p(status.data_ptr()), C.c_void_p(torch.cuda.current_stream().cuda_stream)),
          "rec_prefill_gemm")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    got = oracle.bf16_to_f32(y.cpu().numpy().view(np.uint16)).astype(np.float64)
    rms = np.sqrt((want ** 2).mean(axis=1)) + 1e-30
    rel = np.linalg.norm(got - want, axis=1) / (np.linalg.norm(want, axis=1) + 1e-30)
    assert rel.max() < 4e-3, rel.max()
    assert (np.abs(got - want) / rms[:, None]).max() < 0.02


def _bf(a):
    return oracle.bf16_to_f32(oracle.f32_to_bf16(np.asarray(a, np.float32))).astype(np.float64)


MOE_CASES = [(300, 2, 8, 512, 256), (700, 4, 16, 2048, 768)]


@pytest.mark.parametrize("T,k,E,H,I", MOE_CASES)
def test_prefill_moe_matches_fp64(cuda, T, k, E, H, I):
    """rec_prefill_moe (grouped tcgen05 GEMMs over the experts' token groups)
    against an fp64 restatement with the same bf16 rounding points: g, u and
    d rounded to bf16, act = bf16(bf16(g * bf16(sigmoid g)) * u), the mix in
    rank order with a bf16 rounding after each add, then the residual.  The
    kernel multiplies each dequantized weight as w_hi + w_lo (two bf16
    parts, ~16 significant bits), so the reference uses the dequantized
    weights unrounded; the remaining difference is fp32 vs fp64 accumulation,
    which flips a bf16 rounding now and then: per token a relative L2 error
    below 2e-3, no output off by more than 2^-5 (the outputs are O(1)), fewer
    than 1% of them off at all.  The last expert gets no token."""
    from rec_b200._lib import check, lib

    sd = 0
    rng = np.random.default_rng(T + E)

    def qmat(rows, cols):
        w = (0.02 * rng.standard_normal((rows, cols))).astype(np.float32)
        c, s, b = oracle.quantize(w, 4, sd)
        wd = oracle.dequantize(c, s, b, 4, sd).reshape(rows, cols).astype(np.float64)
        return (c.reshape(rows, -1), s.reshape(rows, -1), b.reshape(rows, -1)), wd

    (gq, gw), (uq, uw), (dq, dw) = qmat(E * I, H), qmat(E * I, H), qmat(E * H, I)
    x = oracle.f32_to_bf16(rng.standard_normal((T, H), dtype=np.float32))
    resid = oracle.f32_to_bf16(rng.standard_normal((T, H), dtype=np.float32))
    ids = np.stack([rng.choice(E - 1, k, replace=False) for _ in range(T)]).astype(np.int32)
    wts = rng.random((T, k), dtype=np.float32)
    wts /= wts.sum(axis=1, keepdims=True)

    xf = oracle.bf16_to_f32(x).astype(np.float64)
    want = np.zeros((T, H))
    for t in range(T):
        mix = None
        for r in range(k):
            e = int(ids[t, r])
            g = _bf(gw[e * I:(e + 1) * I] @ xf[t])
            u = _bf(uw[e * I:(e + 1) * I] @ xf[t])
            act = _bf(_bf(g * _bf(1.0 / (1.0 + np.exp(-g)))) * u)
            d = _bf(dw[e * H:(e + 1) * H] @ act)
            term = _bf(d * _bf(wts[t, r]))
            mix = term if mix is None else _bf(term + mix)
        want[t] = _bf(oracle.bf16_to_f32(resid[t]).astype(np.float64) + mix)

    def dev(a):
        a = np.ascontiguousarray(a)
        if a.dtype == np.uint32:
            return torch.from_numpy(a.view(np.int32)).cuda()
        if a.dtype == np.uint16:
            return torch.from_numpy(a.view(np.int16)).cuda()
        return torch.from_numpy(a).cuda()

    mats = [[dev(p) for p in q] for q in (gq, uq, dq)]
    recs = [abi.RecQMat(m[0].data_ptr(), m[1].data_ptr(), m[2].data_ptr()) for m in mats]
    xd, rd, idd, wd_ = dev(x), dev(resid), dev(ids), dev(wts)
    y = torch.zeros(T, H, dtype=torch.int16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    nb = lib().rec_prefill_moe_workspace_bytes(T, k, H, I, E)
    assert nb > 0
    ws = torch.empty(nb + 256, dtype=torch.uint8, device="cuda")
    base = (ws.data_ptr() + 255) // 256 * 256
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):  # the workspace is reused: counts and cursors start over
        check(lib().rec_prefill_moe(C.byref(recs[0]), C.byref(recs[1]), C.byref(recs[2]), sd, E, I, H,
                                    C.c_void_p(xd.data_ptr()), T, k, C.c_void_p(idd.data_ptr()),
                                    C.c_void_p(wd_.data_ptr()), C.c_void_p(rd.data_ptr()), C.c_void_p(y.data_ptr()),
                                    C.c_void_p(base), nb, C.c_void_p(status.data_ptr()), stream), "rec_prefill_moe")
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        got = oracle.bf16_to_f32(y.cpu().numpy().view(np.uint16)).astype(np.float64)
        # an fp32-vs-fp64 accumulation difference flips a bf16 rounding of g,
        # u or d now and then; the output moves by an ulp of the values
        # involved (all O(1) here), on few elements
        err = np.abs(got - want)
        rel = np.linalg.norm(got - want, axis=1) / (np.linalg.norm(want, axis=1) + 1e-30)
        assert rel.max() < 2e-3, rel.max()
        assert err.max() <= 2.0 ** -5, err.max()
        assert (err > 0).mean() < 0.01, (err > 0).mean()
