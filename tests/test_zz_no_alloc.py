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


def _inputs(M, K, N, seed, dev=DEV):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).to(dev)
    ws = (torch.rand(N, generator=g) * 9e-3 + 1e-3).to(dev)
    b = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    return x, w, ws, b


def _allocating(x, w, ws, b, stream):
    M, K = x.shape
    N = w.shape[0]
    dev = x.device
    out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    xq = torch.empty(M, K, dtype=torch.int8, device=dev)
    xs = torch.empty(M, dtype=torch.float32, device=dev)
    rc = lib.h3b_int8_linear(_p(x), M, K, _p(w), _p(ws), _p(b), N, _p(out), _p(xq), _p(xs), stream)
    assert rc == H3B_OK, lib.h3b_last_error()
    return out


def _noalloc(x, w, ws, b, stream):
    M, K = x.shape
    N = w.shape[0]
    out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
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


def test_noalloc_on_a_second_device():
    """Each GPU has its own copy of the built-in arrays, looked up with that GPU
    current: after calls on device 0, calls on device 1 (two in a row) still
    equal the allocating entry point there."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    x0, w0, ws0, b0 = _inputs(512, 1024, 256, 5)
    s0 = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    with torch.cuda.device(DEV):
        first = _noalloc(x0, w0, ws0, b0, s0)
    dev1 = torch.device("cuda", 1)
    with torch.cuda.device(dev1):
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev1).cuda_stream)
        for (M, K, N, seed) in [(1000, 2048, 512, 3), (64, 5120, 1024, 4)]:
            x, w, ws, b = _inputs(M, K, N, seed, dev1)
            ref = _allocating(x, w, ws, b, stream)
            got = _noalloc(x, w, ws, b, stream)
            torch.cuda.synchronize(dev1)
            assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), f"device 1 mismatch at M={M}"
    with torch.cuda.device(DEV):
        again = _noalloc(x0, w0, ws0, b0, s0)
        torch.cuda.synchronize(DEV)
    assert torch.equal(first.view(torch.int16), again.view(torch.int16))
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
