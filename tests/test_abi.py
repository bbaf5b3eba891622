"""CPU checks of the C ABI: the libraries load, export every symbol the headers
declare, and reject bad arguments on the host (no GPU call is made)."""
import ctypes
import os
import re
import subprocess

import pytest

import edifice_b200
from edifice_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header):
    txt = open(os.path.join(ROOT, "include", header)).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(\w+)\s*\(", txt, flags=re.M)))


def _exported(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True,
                         check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T " in ln}


@pytest.fixture(scope="module", autouse=True)
def built():
    build.build()


def test_library_loads_and_reports_version():
    lib = edifice_b200.load()
    assert lib.edb_version().decode().startswith("edifice_b200")


def test_every_declared_symbol_is_exported():
    names = _declared("edifice_b200.h")
    assert "edb_linear_scan_fwd" in names and len(names) >= 7
    exp = _exported(_lib.LIB_PATH)
    missing = [n for n in names if n not in exp]
    assert not missing, missing
    # every declared entry point also has a ctypes prototype
    assert set(names) <= set(_lib.SIGNATURES)


@pytest.mark.parametrize("prec", ["f32", "bf16"])
def test_shims_export_reference_names(prec):
    names = _declared("edifice_cuda_kernels.h")
    assert "fused_linear_scan_launch" in names
    exp = _exported(build.SHIMS[prec])
    missing = [n for n in names if n not in exp]
    assert not missing, missing
    ctypes.CDLL(build.SHIMS[prec])  # resolves against libedifice_b200.so


def test_status_strings():
    assert _lib.status_string(0) == "ok"
    assert "shape" in _lib.status_string(1001)
    assert "dtype" in _lib.status_string(1002)


def test_host_validation_rejects_bad_arguments():
    lib = edifice_b200.load()
    dummy = ctypes.c_void_p(16)
    # bad dtype, bad shape, null pointers: all rejected before any CUDA call
    assert lib.edb_linear_scan_fwd(7, dummy, dummy, None, dummy, 1, 1, 1, None) == 1002
    assert lib.edb_linear_scan_fwd(1, dummy, dummy, None, dummy, 0, 4, 4, None) == 1001
    assert lib.edb_linear_scan_fwd(1, None, dummy, None, dummy, 1, 4, 4, None) == 1000
    assert lib.edb_mingru_bwd(0, dummy, dummy, None, dummy, None, dummy, dummy, None, 1, 4, 4,
                              None) == 1000
    assert lib.edb_mingru_fwd(0, dummy, dummy, None, dummy, 2, -1, 4, None) == 1001
    # GatedDeltaNet: alpha is required; a too-small workspace is refused
    assert lib.edb_gated_delta_net_fwd(0, dummy, dummy, dummy, dummy, 1, None, dummy, None, 1,
                                       4, 2, 8, None) == 1000
    assert lib.edb_gated_delta_net_fwd(0, dummy, dummy, dummy, dummy, 1, dummy, dummy, None, 1,
                                       4, 2, 256, None) != 0
    need = lib.edb_gated_delta_net_bwd_workspace(0, 1, 1, 4, 2, 8, 0)
    assert need > 0
    assert lib.edb_gated_delta_net_bwd(0, dummy, dummy, dummy, dummy, 1, dummy, dummy, None,
                                       dummy, dummy, dummy, dummy, dummy, 1, 4, 2, 8, dummy,
                                       need - 1, None) == 1004
