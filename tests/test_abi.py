"""The C ABI library loads and exports every entry point include/h3b.h declares (CPU only, no compute calls)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "h3b.h")
LIB = os.path.join(ROOT, "minimax-h3-multi-dgx-spark_b200", "h3b", "libh3b.so")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^H3B_API\s+[\w\s\*]*?\b(h3b_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_entry_points():
    names = declared()
    assert "h3b_int8_mm_scaled" in names and "h3b_norm_mod" in names and "h3b_a2a_pack" in names
    assert len(names) >= 19


def test_library_exports_every_declared_symbol():
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} is not built (run __graft_entry__.build())")
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (h3b_\w+)", out))
    missing = [n for n in declared() if n not in exported]
    assert not missing, f"not exported: {missing}"
    L = ctypes.CDLL(LIB)
    for n in declared():
        assert hasattr(L, n)
    L.h3b_abi_version.restype = ctypes.c_int
    assert L.h3b_abi_version() == 2


def test_every_declaration_cites_a_reference_interface():
    """Each declaration block in the header names the reference file it replaces
    (or states that it is plumbing with no reference counterpart)."""
    src = open(HEADER).read()
    blocks = re.split(r"\n(?=/\*)", src)
    for b in blocks:
        fns = re.findall(r"^H3B_API\s+[\w\s\*]*?\b(h3b_\w+)\s*\(", b, flags=re.M)
        # plumbing, and the allocation-free linear (no counterpart in the reference)
        core = [f for f in fns if not f.startswith(("h3b_abi", "h3b_last", "h3b_status", "h3b_ipc"))
                and f != "h3b_int8_linear_noalloc"]
        if "h3b_int8_linear_noalloc" in fns:
            assert "No counterpart in the reference" in b
        if core:
            assert re.search(r"\.py:\d+", b), f"no reference citation for {core}"


def test_python_binding_signatures_cover_header():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "minimax-h3-multi-dgx-spark_b200"))
    from h3b import _lib
    bound = {name for name, _, _ in _lib.SIGNATURES}
    assert set(declared()) <= bound


def test_entry_points_reject_bad_arguments_before_any_device_work():
    """Argument checks run on the host before any CUDA call: a NULL pointer or an
    unsupported shape returns H3B_ERR_ARG (-1) with a message naming the entry
    point (the GEMM's checks name "h3b GEMM"), on a machine without a GPU too
    (the error behaviour a caller binds to)."""
    import sys
    sys.path.insert(0, os.path.join(ROOT, "minimax-h3-multi-dgx-spark_b200"))
    from h3b._lib import lib
    p0 = ctypes.c_void_p(0)
    cases = [
        ("h3b_quant_rowwise", lambda: lib.h3b_quant_rowwise(p0, 64, 4, 64, p0, p0, p0)),
        ("h3b_quant_rowwise_convrot", lambda: lib.h3b_quant_rowwise_convrot(p0, 256, 4, 256, 128, p0, p0, p0)),
        ("h3b_int8_mm_scaled", lambda: lib.h3b_int8_mm_scaled(p0, p0, p0, p0, p0, p0, 4, 8, 100, p0)),
        ("h3b_norm_mod", lambda: lib.h3b_norm_mod(p0, p0, 1e-6, p0, p0, p0, p0, 4, 64, 1, p0)),
        ("h3b_rms_norm", lambda: lib.h3b_rms_norm(p0, p0, 1e-6, p0, 4, 64, p0)),
        ("h3b_a2a_pack", lambda: lib.h3b_a2a_pack(p0, 64, p0, 4, 32, 32, 2, p0)),
        ("h3b_a2a_inv_quant", lambda: lib.h3b_a2a_inv_quant(None, 64, 0, 4, 32, 2, p0, p0, p0)),
        ("h3b_peer_barrier", lambda: lib.h3b_peer_barrier(None, 9, 0, 1, 1000, p0)),
        ("h3b_int8_linear_noalloc", lambda: lib.h3b_int8_linear_noalloc(p0, 70000, 128, p0, p0, p0, 8, p0, p0)),
        # a size that fits the built-in arrays, NULL operands: rejected before the
        # scratch lookup (which would create a CUDA context)
        ("h3b_int8_linear_noalloc", lambda: lib.h3b_int8_linear_noalloc(p0, 64, 128, p0, p0, p0, 8, p0, p0)),
    ]
    for name, call in cases:
        rc = call()
        assert rc == -1, f"{name} returned {rc}"
        msg = lib.h3b_last_error().decode()
        assert name in msg or ("mm_scaled" in name and "GEMM" in msg), f"{name}: unexpected message {msg!r}"
