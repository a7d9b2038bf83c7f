"""CPU-side checks of the C ABI: the library builds for sm_100a, loads, exports
every entry point include/r4q.h declares, and rejects bad arguments with a
status code before touching the GPU."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def lib():
    from r4q import build
    build.build()
    from r4q import lib as L
    return L


def declared():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"\b(r4q_\w+)\s*\(", h.read_text()))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared()
    assert "r4q_gemv_int4" in names and "r4q_last_error" in names
    assert len(names) >= 8


def test_every_declared_symbol_is_exported(lib):
    for n in declared():
        assert hasattr(lib.LIB, n), f"{n} declared in include/ but not exported"
        assert n in lib.EXPORTS, f"{n} has no ctypes signature in r4q/lib.py"


def test_version_and_workspace_query(lib):
    assert lib.LIB.r4q_version() >= 100
    w = lib.LIB.r4q_gemv_workspace_bytes(16, 5120, 5120)
    assert w >= 16 * 5120 * 4


@pytest.mark.parametrize("B,N,K,code", [
    (0, 64, 64, -1), (17, 64, 64, -1), (1, 60, 64, -1), (1, 64, 48, -1),
])
def test_bad_shapes_rejected_without_gpu(lib, B, N, K, code):
    fake = ctypes.c_void_p(16)   # never dereferenced: validation fails first
    st = lib.LIB.r4q_gemv_int4(fake, K, fake, fake, fake, N, B, N, K, 0, None, 0, None)
    assert st == code
    assert "gemv" in lib.last_error()


def test_null_pointers_rejected(lib):
    assert lib.LIB.r4q_gemv_int4(None, 64, None, None, None, 64, 1, 64, 64, 0, None, 0, None) == -1
    assert lib.LIB.r4q_dequant_int4(None, None, None, 16, 32, None) == -1
    assert lib.LIB.r4q_fp16_to_fp8(None, None, 5, None) == -1


def test_misaligned_rejected(lib):
    p = ctypes.c_void_p(18)
    q = ctypes.c_void_p(32)
    assert lib.LIB.r4q_gemv_int4(p, 64, q, q, q, 64, 1, 64, 64, 0, None, 0, None) == -2


def prototypes():
    """name -> parameter count of every r4q_* prototype in include/*.h."""
    out = {}
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", " ", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b(r4q_\w+)\s*\(([^;{]*?)\)\s*;", text):
            params = m.group(2).strip()
            out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_ctypes_signatures_match_the_header(lib):
    """Every ctypes binding in r4q/lib.py has as many arguments as the C
    prototype: a parameter added on one side only is caught here."""
    protos = prototypes()
    assert len(protos) >= 20
    for name, (_res, args) in lib._SIGS.items():
        assert name in protos, f"{name} bound in r4q/lib.py but not declared in include/"
        assert len(args) == protos[name], f"{name}: {len(args)} ctypes args, {protos[name]} in the header"
