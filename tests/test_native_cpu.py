"""CPU checks of the C-ABI library: it loads, exports every declared entry point, and
fails cleanly (NULL + message, never a crash) where no GPU is present."""
import ctypes as ct
import re
import subprocess

import pytest

from conftest import ROOT

HEADERS = sorted((ROOT / "include").glob("*/*.h"))


def declared_symbols():
    names = []
    for h in HEADERS:
        names += re.findall(r"^MACE_EXPORT[^;(]*?\b(\w+)\s*\(", h.read_text(), re.M)
    return names


def test_header_declares_reference_abi():
    names = declared_symbols()
    for ref in ("mace_create_mh1", "mace_create_mh1_head", "mace_destroy", "mace_last_error", "mace_calculate",
                "mace_diagnostics"):
        assert ref in names


def test_library_exports_every_declared_symbol(library):
    lib = ct.CDLL(str(library))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_create_fails_cleanly_without_a_gpu(library, archive_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from mace_inference import native
    lib = native.load(library)
    assert lib.mace_create_mh1(str(archive_path).encode(), 0) is None
    assert lib.mace_last_error().decode()
    assert lib.mace_create_mh1(None, 0) is None
    assert "Null archive path" in lib.mace_last_error().decode()
    energy = (ct.c_double * 1)()
    virial = (ct.c_float * 9)()
    cell = (ct.c_float * 9)()
    assert lib.mace_calculate(None, 0, None, None, cell, energy, None, None, virial) == -1
    assert "Null calculator" in lib.mace_last_error().decode()


def test_cli_usage(library):
    exe = ROOT / "lasp-pis_b200" / "bin" / "mace-main"
    assert subprocess.run([str(exe)], capture_output=True).returncode == 2
    r = subprocess.run([str(exe), "--help"], capture_output=True, text=True)
    assert r.returncode == 0 and "Usage: mace-main" in r.stdout
    r = subprocess.run([str(exe), "m.pwm", "s.arc", "--bogus"], capture_output=True, text=True)
    assert r.returncode == 1 and "unknown option" in r.stderr
