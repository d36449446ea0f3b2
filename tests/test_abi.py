"""CPU tests of the drop-in boundary: the plugin and the loader load, export every
symbol the public header declares, and report "no device" cleanly without a GPU
(the reference engine's contract, README.md:11)."""
import ctypes as C
import os
import subprocess
import sys

import pytest

from katali_lab_b200 import build as B
from katali_lab_b200.plugin import (KataliHybridDesc, KataliHybridLayerW, KataliMoeDesc, Plugin,
                                    header_symbols)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def built():
    B.build()
    return B.PLUGIN, B.LOADER


def exported(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_header_declares_reference_call_sites():
    # every katali_cuda_* name the reference calls (katali_dense_cuda.c) is declared
    needed = {"katali_cuda_probe", "katali_cuda_status", "katali_cuda_malloc", "katali_cuda_free",
              "katali_cuda_upload", "katali_cuda_download", "katali_cuda_supports_type",
              "katali_cuda_matvec"}
    assert needed <= set(header_symbols())


def test_plugin_exports_exactly_the_header(built):
    syms = {s for s in exported(built[0]) if s.startswith("katali_cuda_")}
    assert syms == set(header_symbols())


def test_loader_exports_the_header(built):
    syms = {s for s in exported(built[1]) if s.startswith("katali_cuda_")}
    assert set(header_symbols()) <= syms


def test_plugin_links_no_cuda_shared_library(built):
    out = subprocess.run(["ldd", built[0]], capture_output=True, text=True).stdout
    assert "libcudart" not in out and "libtorch" not in out and "libpython" not in out


def _loader_probe(env):
    code = ("import ctypes as C,sys;L=C.CDLL(sys.argv[1]);"
            "L.katali_cuda_status.restype=C.c_char_p;"
            "print(L.katali_cuda_probe());print(L.katali_cuda_status().decode())")
    r = subprocess.run([sys.executable, "-c", code, B.LOADER], capture_output=True, text=True,
                       env={**os.environ, **env}, timeout=120)
    assert r.returncode == 0, r.stderr
    probe, status = r.stdout.strip().split("\n", 1)
    return int(probe), status


def test_loader_disabled_by_env(built):
    probe, status = _loader_probe({"KATALI_CUDA": "0"})
    assert probe == 0 and "KATALI_CUDA=0" in status


def test_loader_bad_path_reports_reason(built):
    probe, status = _loader_probe({"KATALI_CUDA_DLL": "/nonexistent/libkatali_cuda.so"})
    assert probe == 0 and "cannot load" in status


def test_loader_finds_sibling_plugin(built):
    import torch
    probe, status = _loader_probe({"KATALI_CUDA_DLL": ""})
    if torch.cuda.is_available():
        assert probe == 1, status
    else:
        assert probe == 0 and status and "cannot load" not in status


def test_no_device_is_an_error_code_not_a_crash(built):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    p = Plugin()
    assert not p.probe()
    assert p.status()
    ptr = C.c_void_p()
    assert p.L.katali_cuda_malloc(C.byref(ptr), 16) == 1  # KATALI_ERR_NO_DEVICE
    desc = KataliMoeDesc(8, 512, 256, 2, 12, 12, 14, 1, None)
    h = C.c_void_p()
    assert p.L.katali_cuda_moe_create(C.byref(desc), C.byref(h)) == 1
    # the decoders check their arguments first, then the device
    layer = (KataliHybridLayerW * 1)()
    hd = KataliHybridDesc(n_layers=1, hidden=2048, vocab=256, kv_cap=16, layers=layer)
    assert p.L.katali_cuda_hybrid_create(None, C.byref(h)) == 3
    assert p.L.katali_cuda_hybrid_create(C.byref(hd), None) == 3
    assert p.L.katali_cuda_hybrid_create(C.byref(hd), C.byref(h)) == 1
    assert not h.value


def test_argument_checks_before_device(built):
    p = Plugin()
    assert p.L.katali_cuda_supports_type(12) == 1
    assert p.L.katali_cuda_supports_type(14) == 1
    assert p.L.katali_cuda_supports_type(0) == 0
    assert p.L.katali_cuda_matvec(2, None, 1, 256, None, None) == 4  # unsupported type
    bad = KataliMoeDesc(8, 512, 256, 0, 12, 12, 14, 1, None)  # top_k 0
    h = C.c_void_p()
    assert p.L.katali_cuda_moe_create(C.byref(bad), C.byref(h)) == 3
    assert p.L.katali_cuda_strerror(6) == b"device-side wait timed out"


def test_check_cli_reports_no_device():
    """The command-line check (cuda-info equivalent) exits 2 with the probe's reason when no
    usable GPU is present (this CPU-only test runs where CUDA is unavailable)."""
    import subprocess

    import torch
    from katali_lab_b200.build import CHECK
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    r = subprocess.run([CHECK, "info"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2
    assert "katali_cuda:" in r.stdout
    r = subprocess.run([CHECK, "check"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2
