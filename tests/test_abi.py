"""CPU: the C-ABI library builds, loads without a GPU, and exports every declared entry point."""
import re
import subprocess
from pathlib import Path

from nvfp4_qsa import _build, _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "nvfp4_qsa.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(nvqsa_\w+)\s*\(", text)))


def test_library_builds_and_exports_every_declared_symbol():
    lib = _build.build()
    declared = declared_symbols()
    assert len(declared) >= 9
    nm = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (nvqsa_\w+)", nm))
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    assert set(declared) == set(_native.EXPORTED_SYMBOLS)


def test_library_loads_without_gpu_and_reports_status_text():
    lib = _native.load()
    assert lib.nvqsa_abi_version() == 1
    assert _native.status_text(0) == "ok"
    assert "workspace" in _native.status_text(5)


def test_status_codes_map_to_python_exceptions():
    import pytest
    with pytest.raises(NotImplementedError):
        _native.check(3, "x")
    with pytest.raises(ValueError):
        _native.check(2, "x")
    with pytest.raises(RuntimeError):
        _native.check(7, "x")
