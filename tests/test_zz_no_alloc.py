"""The allocation-free INT8 linear entry point, through the C ABI.

h3b_int8_linear_noalloc serves callers that cannot allocate device memory
(for example a C or FFI host that binds libh3b without a device allocator, or
a serving loop that must not call cudaMalloc mid-step): it keeps the int8
activation codes and row scales in fixed arrays inside the library instead of
caller-provided scratch.  Its output must equal h3b_int8_linear's (the
allocating entry point) bit for bit, on consecutive calls that reuse the same
built-in arrays with different shapes and data, and it must refuse calls that
do not fit those arrays.  This file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

h3b = pytest.importorskip("h3b")
from h3b._lib import H3B_OK, lib  # noqa: E402

DEV = torch.device("cuda", 0)
ERR_ARG = -1


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _inputs(M, K, N, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).to(DEV)
    ws = (torch.rand(N, generator=g) * 9e-3 + 1e-3).to(DEV)
    b = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    return x, w, ws, b


def _allocating(x, w, ws, b, stream):
    M, K = x.shape
    N = w.shape[0]
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    xq = torch.empty(M, K, dtype=torch.int8, device=DEV)
    xs = torch.empty(M, dtype=torch.float32, device=DEV)
    rc = lib.h3b_int8_linear(_p(x), M, K, _p(w), _p(ws), _p(b), N, _p(out), _p(xq), _p(xs), stream)
    assert rc == H3B_OK, lib.h3b_last_error()
    return out


def _noalloc(x, w, ws, b, stream):
    M, K = x.shape
    N = w.shape[0]
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    rc = lib.h3b_int8_linear_noalloc(_p(x), M, K, _p(w), _p(ws), _p(b), N, _p(out), stream)
    assert rc == H3B_OK, lib.h3b_last_error()
    return out


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls():
    torch.cuda.set_device(DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    # two calls in a row: the second reuses the built-in arrays the first filled
    # (different shape, bias present, then absent)
    for (M, K, N, seed, with_bias) in [(2048, 4096, 1024, 1, True), (777, 5120, 5120, 2, False)]:
        x, w, ws, b = _inputs(M, K, N, seed)
        if not with_bias:
            b = None
        ref = _allocating(x, w, ws, b, stream)
        got = _noalloc(x, w, ws, b, stream)
        torch.cuda.synchronize(DEV)
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), f"mismatch at M={M} K={K} N={N}"
    assert h3b.status() == 0


def test_noalloc_rejects_calls_beyond_its_arrays():
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    M, K, N = 4096, 4096, 128  # 16 MiB of codes: twice the built-in array
    x = torch.zeros(M, K, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(N, K, dtype=torch.int8, device=DEV)
    ws = torch.ones(N, device=DEV)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    rc = lib.h3b_int8_linear_noalloc(_p(x), M, K, _p(w), _p(ws), None, N, _p(out), stream)
    assert rc == ERR_ARG
    assert b"exceeds the built-in" in lib.h3b_last_error()
