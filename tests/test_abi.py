"""The C-ABI library loads on CPU and exports exactly what include/b2e.h declares.
No compute call is made here (there is no GPU)."""

import ctypes as C
import re
import subprocess

import pytest

from hackathon_b200 import _lib
from tests.conftest import REPO

HEADER = REPO / "include" / "b2e.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^B2E_API\s+[\w\s\*]+?\b(b2e_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_binding():
    assert declared_symbols() == _lib.exported_symbols()


def test_library_exports_every_declared_symbol():
    if not _lib.LIB_PATH.exists():
        pytest.fail(f"{_lib.LIB_PATH} is not built: run python -m hackathon_b200.build")
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, f"not exported: {missing}"
    # and nothing else leaks out of the library under the b2e_ prefix
    extra = sorted(s for s in exported if s.startswith("b2e_") and s not in declared_symbols())
    assert not extra, f"undeclared exports: {extra}"


def test_library_loads_and_reports_errors_without_a_gpu():
    L = _lib.lib()
    assert L.b2e_version().startswith(b"b2e")
    # argument checks run before any CUDA call: a null handle is refused with a message
    rc = L.b2e_engine_step(None, None, None, 1, None)
    assert rc == -1
    assert b"null" in L.b2e_last_error()
    with pytest.raises(_lib.B2EError):
        _lib.check(L.b2e_engine_slot_bytes(None, None))


def test_state_kernel_grid_setting_is_checked_and_returns_the_previous_value():
    """b2e_set_state_kernel_waves only records a process-wide launch choice (no
    device work): out-of-range values are refused with B2E_ERR_INVALID and leave
    it unchanged; a valid one returns the previous value."""
    L = _lib.lib()
    prev = C.c_int32(-1)
    assert L.b2e_set_state_kernel_waves(8, C.byref(prev)) == 0
    start = prev.value
    for bad in (-1, 65, 1000):
        assert L.b2e_set_state_kernel_waves(bad, C.byref(prev)) == -1  # B2E_ERR_INVALID
        assert b"waves" in L.b2e_last_error()
    assert L.b2e_set_state_kernel_waves(0, C.byref(prev)) == 0 and prev.value == 8
    assert L.b2e_set_state_kernel_waves(start, None) == 0


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setenv("B2E_LIB", str(tmp_path / "absent.so"))
    with pytest.raises(_lib.B2ELibraryError):
        _lib.lib()
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.delenv("B2E_LIB")
    _lib.lib()
