"""The allocation-free RMSNorm backward, called through its exported C symbol.

``rlb_rmsnorm_bwd_noalloc`` keeps its dw partial sums in a fixed device array
instead of a caller buffer.  It must agree with the regular ``rmsnorm_bwd``
entry point on two calls in a row (the second call sees the first call's stale
scratch), and must refuse dims beyond its limit without launching.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from rl_project_b200.ops import _ext

    mod = _ext.native()
    lib = ctypes.CDLL(mod.__file__)
    fn = lib.rlb_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int, ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p]
    lib.rlb_rmsnorm_bwd_noalloc_scratch_bytes.restype = ctypes.c_longlong
    lib.rlb_rmsnorm_bwd_noalloc_init.restype = ctypes.c_int
    return mod, lib


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _call(lib, h, w, rstd, dy, dres, dx, dw):
    stream = torch.cuda.current_stream().cuda_stream
    rows, dim = h.numel() // h.shape[-1], h.shape[-1]
    return lib.rlb_rmsnorm_bwd_noalloc(_ptr(h), _ptr(w), _ptr(rstd), _ptr(dy), _ptr(dres), _ptr(dx), _ptr(dw),
                                       int(dw.dtype == torch.float32), rows, dim, ctypes.c_void_p(stream))


def _inputs(rows, dim, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    h = torch.randn(rows, dim, device="cuda", generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(dim, device="cuda", generator=g)).bfloat16()
    dy = torch.randn(rows, dim, device="cuda", generator=g).bfloat16()
    dres = torch.randn(rows, dim, device="cuda", generator=g).bfloat16()
    rstd = torch.rsqrt(h.float().pow(2).mean(-1) + 1e-5).contiguous()
    return h, w, rstd, dy, dres


# w is always bf16 (as for the regular entry point); dw may be written as bf16 or fp32
@pytest.mark.parametrize("rows,dim,dw_dtype,with_res", [
    (4096, 2048, torch.bfloat16, True),
    (3001, 4096, torch.float32, False),
    (1, 256, torch.bfloat16, False),
    (20000, 8192, torch.float32, True),  # the scratch cap binds: 128 partial rows, each block strides over many rows
])
def test_noalloc_matches_regular_entry_point(rows, dim, dw_dtype, with_res):
    mod, lib = _lib()
    assert lib.rlb_rmsnorm_bwd_noalloc_init() == 0  # setup ahead of the first call (idempotent)
    assert lib.rlb_rmsnorm_bwd_noalloc_scratch_bytes() == 4 << 20
    for seed in (0, 1):  # two calls in a row; the second reuses the first call's scratch
        h, w, rstd, dy, dres = _inputs(rows, dim, seed)
        dres = dres if with_res else None
        dx_ref, dw_ref = mod.rmsnorm_bwd(h, w, rstd, dy, dres)
        dx = torch.empty_like(h)
        dw = torch.empty(dim, device="cuda", dtype=dw_dtype)
        assert _call(lib, h, w, rstd, dy, dres, dx, dw) == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(dx, dx_ref, rtol=0, atol=0)  # same kernel, same rows per block
        scale = dw_ref.float().abs().max().item()
        torch.testing.assert_close(dw.float(), dw_ref.float(), rtol=1e-2, atol=1e-4 * scale)


def test_noalloc_rejects_dims_beyond_limit():
    _, lib = _lib()
    for dim in (16384, 1000, 128):  # above 8192, not a multiple of 256
        h = torch.empty(2, dim, device="cuda", dtype=torch.bfloat16)
        w = torch.empty(dim, device="cuda", dtype=torch.bfloat16)
        rstd = torch.empty(2, device="cuda")
        rc = _call(lib, h, w, rstd, h, None, torch.empty_like(h), torch.empty_like(w))
        assert rc == 1  # cudaErrorInvalidValue, nothing launched


@pytest.mark.parametrize("dw_dtype", [torch.bfloat16, torch.float32])
def test_noalloc_zero_rows_gives_zero_dw(dw_dtype):
    _, lib = _lib()
    dim = 1024
    h = torch.empty(0, dim, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(dim, device="cuda", dtype=torch.bfloat16)
    rstd = torch.empty(0, device="cuda")
    dw = torch.full((dim,), 7.0, device="cuda", dtype=dw_dtype)  # stale values must be overwritten
    # a pointer of a zero-size tensor may be null, which the alignment check accepts (nothing is read)
    assert _call(lib, h, w, rstd, h, None, torch.empty_like(h), dw) == 0
    torch.cuda.synchronize()
    assert torch.count_nonzero(dw).item() == 0
