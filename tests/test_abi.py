"""The C-ABI library loads and exports every symbol include/*.h declares.
No GPU is touched: only symbol lookup and argument-free calls."""
import re
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def declared_symbols():
    syms = set()
    for h in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        syms |= set(re.findall(r"\b(mb_[a-z0-9_]+)\s*\(", text))
    return sorted(syms)


@pytest.fixture(scope="module")
def lib():
    from metalbench_b200 import _lib
    if not _lib.LIB_PATH.exists():
        from metalbench_b200 import build
        build.build()
    return _lib.lib()


def test_header_declares_symbols():
    assert "mb_run" in declared_symbols() and "mb_init" in declared_symbols()


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(REPO / "metalbench_b200" / "libmb200.so")],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (mb_[a-z0-9_]+)$", out, flags=re.M))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, f"declared but not exported: {missing}"


def test_ctypes_signatures_cover_header(lib):
    from metalbench_b200 import _lib
    assert set(declared_symbols()) == set(_lib.SIGNATURES), \
        set(declared_symbols()) ^ set(_lib.SIGNATURES)


def test_kernel_table_names(lib):
    names = lib.mb_kernel_names().decode().split(",")
    for n in ("transpose_2d", "transpose_batched"):
        assert n in names


def test_run_without_init_reports_not_init(lib):
    from metalbench_b200 import _lib
    rc = lib.mb_run(b"transpose_2d", None, 0, None, 0, None, 0, 1, None)
    assert rc == -6 and "mb_init" in _lib.last_error()


def test_device_status_reader_and_clearer_without_a_device(lib):
    """mb_device_status / mb_clear_device_status allocate nothing: with no
    status word on the current device (or no device at all) they report a
    clean 0 and succeed."""
    import ctypes
    v = ctypes.c_uint32(123)
    assert lib.mb_device_status(ctypes.byref(v)) == 0
    assert v.value == 0
    assert lib.mb_clear_device_status() == 0
