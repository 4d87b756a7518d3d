"""The C ABI boundary without a GPU: the library loads, exports every symbol
include/g4b.h declares, and rejects bad calls before launching anything."""
import ctypes as C
import os
import re
import subprocess
import sys

import pytest

from g4b import _lib as L

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "g4b.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^G4B_API [^(]*?\b(g4b_\w+)\(", src, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("g4b_gemv_i4", "g4b_reduce_partials", "g4b_dequant_i4", "g4b_cast", "g4b_cast_i8",
                 "g4b_last_error", "g4b_query", "g4b_version", "g4b_stream_wait"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = L.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/g4b.h but not exported"
    # and the Python binding covers every declared symbol
    assert set(declared_symbols()) <= set(L.SIGNATURES), set(declared_symbols()) - set(L.SIGNATURES)


def test_library_has_no_hard_driver_dependency():
    out = subprocess.run(["ldd", L.lib_path()], capture_output=True, text=True).stdout
    assert "libcuda.so" not in out and "not found" not in out


def test_version_and_query():
    lib = L.load()
    assert lib.g4b_version() == 100
    assert L.query(L.Q_VERSION) == 100
    assert L.query(12345) == -1


def test_null_arguments_rejected():
    lib = L.load()
    st = lib.g4b_gemv_i4(None, 0, 1, None, None, 0, 1.0, None, 0, 256, 256, 0, None, 0, None)
    assert st == L.G4B_E_ARG
    assert "NULL" in L.last_error()


def test_shape_errors_rejected_before_launch():
    lib = L.load()
    buf = C.create_string_buffer(4096 + 16)
    p = (C.addressof(buf) + 15) & ~15
    # N not a multiple of 16
    assert lib.g4b_gemv_i4(p, 0, 1, p, p, 0, 1.0, p, 0, 24, 64, 0, None, 0, None) == L.G4B_E_SHAPE
    # K not a multiple of 32
    assert lib.g4b_gemv_i4(p, 0, 1, p, p, 0, 1.0, p, 0, 64, 48, 0, None, 0, None) == L.G4B_E_SHAPE
    # split that does not divide K/32
    assert lib.g4b_gemv_i4(p, 0, 1, p, p, 0, 1.0, p, 0, 64, 96, 2, None, 0, None) == L.G4B_E_SHAPE
    # bad enums
    assert lib.g4b_gemv_i4(p, 7, 1, p, p, 0, 1.0, p, 0, 64, 64, 0, None, 0, None) == L.G4B_E_ARG
    assert lib.g4b_gemv_i4(p, 0, 1, p, p, 9, 1.0, p, 0, 64, 64, 0, None, 0, None) == L.G4B_E_ARG
    # misaligned pointer
    assert lib.g4b_gemv_i4(p + 4, 0, 1, p, p, 0, 1.0, p, 0, 64, 64, 0, None, 0, None) == L.G4B_E_ALIGN
    assert lib.g4b_cast_i8(p, 1, p, p, 4, 24, None) == L.G4B_E_SHAPE
    assert lib.g4b_cast(p, 0, p, 0, 16, None) == L.G4B_E_ARG


def test_no_device_is_reported_not_crashed():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    lib = L.load()
    buf = C.create_string_buffer(4096 + 16)
    p = (C.addressof(buf) + 15) & ~15
    st = lib.g4b_gemv_i4(p, 0, 1, p, p, 0, 1.0, p, 0, 64, 64, 0, None, 0, None)
    assert st in (L.G4B_E_CUDA, L.G4B_E_ARCH)
    assert L.query(L.Q_DEVICE_OK) == 0


def test_fault_injection_fails_the_nth_call():
    code = (
        "import sys; sys.path.insert(0, %r);\n"
        "from g4b import _lib as L\n"
        "lib = L.load()\n"
        "a = lib.g4b_gemv_i4(None,0,1,None,None,0,1.0,None,0,64,64,0,None,0,None)\n"
        "b = lib.g4b_gemv_i4(None,0,1,None,None,0,1.0,None,0,64,64,0,None,0,None)\n"
        "c = lib.g4b_gemv_i4(None,0,1,None,None,0,1.0,None,0,64,64,0,None,0,None)\n"
        "print(a, b, c, L.last_error() if False else '')\n"
    ) % os.path.join(REPO, "gemma4-12b-snapdragonx2elite_b200")
    env = dict(os.environ, G4B_FAULT="gemv_i4:2")
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, check=True).stdout
    a, b, c = map(int, out.split()[:3])
    assert (a, b, c) == (L.G4B_E_ARG, L.G4B_E_FAULT_INJECTED, L.G4B_E_ARG)


def test_g4b_error_carries_code_and_message():
    with pytest.raises(L.G4BError) as ei:
        L.check("g4b_gemv_i4", L.load().g4b_gemv_i4(None, 0, 1, None, None, 0, 1.0, None, 0, 64, 64, 0, None, 0, None))
    assert ei.value.code == L.G4B_E_ARG
