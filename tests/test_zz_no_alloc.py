"""rec_gemv_int4_argmax_noalloc: the int4 GEMV + greedy argmax whose scratch is
a static device array instead of caller memory.

Its logits must equal rec_gemv_int4's bit for bit and its token must be the
lowest-index maximum of those logits, on consecutive calls (the scratch keeps
the previous call's contents).  This file is collected last and also runs
alone in a fresh process, where its first call performs the per-device
set-up.
"""
import ctypes as C

import numpy as np
import pytest
import torch

MAX_ROWS_WITHOUT_Y = 262144


def _noalloc(m, sd, n, k, x, norm_w, eps, y, token):
    from rec_b200 import _lib

    fn = _lib.lib().rec_gemv_int4_argmax_noalloc
    ptr = lambda t: C.c_void_p(0 if t is None else t.data_ptr())  # noqa: E731
    return fn(C.byref(m), sd, n, k, ptr(x), ptr(norm_w), float(eps), ptr(y), ptr(token),
              C.c_void_p(torch.cuda.current_stream().cuda_stream))


def _first_argmax(y: torch.Tensor) -> int:
    v = y.float().cpu().numpy()
    return int(np.argmax(v))  # first index among equal maxima


def _matrix(n, k, seed, dev):
    from rec_b200 import ops

    g = torch.Generator(device=dev).manual_seed(seed)
    w = torch.randn(n, k, generator=g, device=dev) * 0.02
    return ops.quantize_affine(w, 4, torch.float16)


@pytest.mark.gpu
def test_noalloc_matches_gemv_on_consecutive_calls(cuda):
    from rec_b200 import _lib, ops

    n, k = 151936, 2048  # lm_head of the config-3 model
    w, s, b = _matrix(n, k, 11, cuda)
    g = torch.Generator(device=cuda).manual_seed(12)
    xs = [(torch.randn(k, generator=g, device=cuda)).to(torch.bfloat16) for _ in range(3)]
    norm_w = (1 + 0.1 * torch.randn(k, generator=g, device=cuda)).to(torch.bfloat16)
    m = ops.qmat(w, s, b)
    token = torch.empty(1, dtype=torch.int32, device=cuda)
    for call, (x, nw) in enumerate([(xs[0], None), (xs[1], norm_w), (xs[2], None)]):
        y_ref = ops.gemv_int4(w, s, b, x, norm_weight=nw, eps=1e-6)
        torch.cuda.synchronize()
        want = _first_argmax(y_ref)
        if call == 2 and want > 0:
            # copy the winning row to row 0 (another CTA): the tie goes to row 0
            lo = 0
            w[lo].copy_(w[want])
            s[lo].copy_(s[want])
            b[lo].copy_(b[want])
            y_ref = ops.gemv_int4(w, s, b, x)
            torch.cuda.synchronize()
            assert y_ref[lo].item() == y_ref[want].item()
            want = lo
        y = torch.full((n,), 7.0, dtype=torch.bfloat16, device=cuda)
        _lib.check(_noalloc(m, 0, n, k, x, nw, 1e-6, y, token), "rec_gemv_int4_argmax_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16)), f"call {call}: logits differ"
        assert int(token.item()) == want, f"call {call}: token {int(token.item())} != {want}"
        # logits kept in the scratch (no y buffer)
        token.fill_(-5)
        _lib.check(_noalloc(m, 0, n, k, x, nw, 1e-6, None, token), "rec_gemv_int4_argmax_noalloc")
        torch.cuda.synchronize()
        assert int(token.item()) == want, f"call {call} (no y): token {int(token.item())} != {want}"


@pytest.mark.gpu
@pytest.mark.parametrize("k,sd", [(4096, 1), (768, 0)])
def test_noalloc_other_shapes(cuda, k, sd):
    from rec_b200 import _lib, ops

    n = 4096 + 2 * 37
    g = torch.Generator(device=cuda).manual_seed(k + sd)
    w = torch.randn(n, k, generator=g, device=cuda) * 0.02
    w, s, b = ops.quantize_affine(w, 4, torch.float16 if sd == 0 else torch.bfloat16)
    m = ops.qmat(w, s, b)
    token = torch.empty(1, dtype=torch.int32, device=cuda)
    for rep in range(2):
        x = torch.randn(k, generator=g, device=cuda).to(torch.bfloat16)
        y_ref = ops.gemv_int4(w, s, b, x)
        y = torch.empty(n, dtype=torch.bfloat16, device=cuda)
        _lib.check(_noalloc(m, sd, n, k, x, None, 1e-6, y, token), "rec_gemv_int4_argmax_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16)), f"rep {rep}"
        assert int(token.item()) == _first_argmax(y_ref), f"rep {rep}"
        # and directly against the CPU oracle's GEMV of the same inputs
        import oracle
        from oracle.host import _np

        assert np.array_equal(_np(y), oracle.gemv(_np(w), _np(s), _np(b), _np(x), sd)), f"rep {rep} (oracle)"


def test_noalloc_rejects_rows_beyond_scratch():
    """Argument checks run before any CUDA call (no device needed)."""
    from rec_b200 import _lib, abi

    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built")
    m = abi.RecQMat(16, 16, 16)  # never dereferenced: the size check fails first
    fn = _lib.lib().rec_gemv_int4_argmax_noalloc
    rc = fn(C.byref(m), 0, MAX_ROWS_WITHOUT_Y + 2, 2048, C.c_void_p(16), C.c_void_p(0), 1e-6, C.c_void_p(0),
            C.c_void_p(16), C.c_void_p(0))
    assert rc == abi.REC_EINVAL
    assert "262144-row logits scratch" in _lib.last_error()

