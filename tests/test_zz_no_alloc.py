"""The allocation-free RMSNorm backward entry point, called through its exported C
symbol the way a caller that cannot allocate device memory would (all buffers are
made by the test; the entry point itself allocates nothing), checked against the
library's regular RMSNorm backward on two consecutive calls.

This file is named to be collected last so a failure here never hides other tests."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _symbol():
    from tinytron_b200.ops import _ext

    _ext.load()  # loads the library (and its libtorch dependencies) into the process
    lib = ctypes.CDLL(str(_ext.so_path()))
    fn = lib.tt_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return fn


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _case(M, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, D, device="cuda", generator=g)
    rstd = torch.rsqrt(x.pow(2).mean(-1) + 1e-6)
    w = torch.rand(D, device="cuda", generator=g) + 0.5
    gh = torch.randn(M, D, device="cuda", generator=g).bfloat16()
    gres = torch.randn(M, D, device="cuda", generator=g)
    return x, rstd, w, gh, gres


def _reference(x, rstd, w, gh, gres, dw0):
    from tinytron_b200.ops import _ext

    C = _ext.load()
    M, D = x.shape
    gx = torch.empty_like(x)
    gd = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    dw = dw0.clone()
    scratch = torch.empty(C.rmsnorm_bwd_scratch_numel(M, D), device="cuda")
    C.rmsnorm_bwd(gh, x, rstd, w, gres, gx, gd, dw, True, scratch)
    return gx, gd, dw


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


def test_noalloc_matches_regular_entry_point_twice():
    fn = _symbol()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    dw = torch.zeros(2048, device="cuda")
    for call, (M, D, seed) in enumerate([(3000, 2048, 1), (517, 2048, 2)]):
        x, rstd, w, gh, gres = _case(M, D, seed)
        ref_gx, ref_gd, ref_dw = _reference(x, rstd, w, gh, gres, dw)
        gx = torch.full_like(x, float("nan"))
        gd = torch.full((M, D), float("nan"), device="cuda", dtype=torch.bfloat16)
        rc = fn(_ptr(gh), _ptr(x), _ptr(rstd), _ptr(w), _ptr(gres), _ptr(gx), _ptr(gd), _ptr(dw), M, D, 1, stream)
        torch.cuda.synchronize()
        assert rc == 0, f"call {call}: return code {rc}"
        assert _rel(gx, ref_gx) < 1e-5
        assert _rel(gd, ref_gd) < 1e-2
        assert _rel(dw, ref_dw) < 1e-5  # accumulated across both calls, like the reference path


def test_noalloc_rejects_oversized_problem():
    fn = _symbol()
    M, D = 16 * 1024 + 16, 1024  # ceil(M/16) * D > 2^20 scratch floats
    t = torch.empty(1, device="cuda")
    rc = fn(_ptr(t), _ptr(t), _ptr(t), _ptr(t), None, None, None, _ptr(t), M, D, 0,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 2


def test_noalloc_overwrite_mode_and_optional_outputs():
    """accumulate_dw=0 overwrites dw; g_res and gx may be NULL (only g_delta and dw written)."""
    from tinytron_b200.ops import _ext

    C = _ext.load()
    fn = _symbol()
    M, D = 777, 1024
    x, rstd, w, gh, _ = _case(M, D, 7)
    ref_gd = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    ref_dw = torch.zeros(D, device="cuda")
    C.rmsnorm_bwd(gh, x, rstd, w, None, None, ref_gd, ref_dw, False, torch.empty(C.rmsnorm_bwd_scratch_numel(M, D),
                                                                                   device="cuda"))
    gd = torch.full((M, D), float("nan"), device="cuda", dtype=torch.bfloat16)
    dw = torch.full((D,), 123.0, device="cuda")  # overwritten, not added to
    rc = fn(_ptr(gh), _ptr(x), _ptr(rstd), _ptr(w), None, None, _ptr(gd), _ptr(dw), M, D, 0,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rc == 0
    assert _rel(gd, ref_gd) < 1e-2
    assert _rel(dw, ref_dw) < 1e-5


def test_noalloc_rejects_bad_hidden_size():
    fn = _symbol()
    t = torch.empty(64, device="cuda")
    rc = fn(_ptr(t), _ptr(t), _ptr(t), _ptr(t), None, None, None, _ptr(t), 4, 12, 0,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 1  # D must be a multiple of 8
