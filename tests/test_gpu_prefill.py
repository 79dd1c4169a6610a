"""The tensor-core prefill projection (rec_prefill_gemm, tcgen05) against an
fp64 GEMM of the dequantized int4 weights.  The weights are dequantized to
bf16 before the MMA (~2^-9 relative per weight) and Y is rounded to bf16, so
the bound is a relative L2 error of 4e-3 per row (measured ~1.6e-3 for
random inputs) and no element off by more than 2% of its row's RMS."""
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
