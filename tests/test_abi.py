"""CPU tests of the C ABI boundary: the library loads and exports exactly the
functions include/stealcode_b200.h declares (no compute call needs a GPU)."""
import os
import re
import subprocess

from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "stealcode_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sc_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("sc_q8_repack", "sc_q8_gemm", "sc_q8_gemm_host", "sc_q8mat_gemm_t", "sc_attn_stream",
                 "sc_attn_stream_host", "sc_attn_stream_ring", "sc_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from stealcode_b200 import _lib

    names = declared_functions()
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (sc_[a-z0-9_]+)$", out, flags=re.M))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    for n in names:
        assert getattr(_lib.lib, n) is not None


def test_binding_matches_header():
    from stealcode_b200 import _lib

    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_abi_version_and_error_string():
    from stealcode_b200 import _lib

    assert _lib.lib.sc_abi_version() == 1
    assert isinstance(_lib.last_error(), str)


def test_invalid_arguments_rejected_without_gpu():
    """Argument validation happens before any CUDA call."""
    import ctypes

    from stealcode_b200 import _lib

    h = ctypes.c_void_p()
    assert _lib.lib.sc_q8_repack(None, 4, 64, 34, 2, ctypes.byref(h)) == _lib.SC_ERR_INVALID
    assert _lib.lib.sc_q8_gemm(None, None, 1, 0, 0, None, None, 0, 0, None, 0, None) == _lib.SC_ERR_INVALID
    assert "null" in _lib.last_error()
    assert _lib.lib.sc_q8_gemm_host(0, 64, 1, None, 68, 34, 2, None, None) == _lib.SC_OK  # zero dims no-op
    assert _lib.lib.sc_attn_stream_ring(None, 0, None, None, 0, None, None, 0, 1, None, 0, None, None, 8,
                                        1024, 8, 0.1, 0, 0, 7, 10, 8, 6, None, 0, None) == _lib.SC_ERR_INVALID


def test_ops_fail_loudly_without_library(tmp_path):
    """A package copy without the built library must raise ImportError, not fall back."""
    import shutil
    import sys

    pkg = tmp_path / "stealcode_b200"
    shutil.copytree(os.path.join(ROOT, "stealcode_b200"), pkg,
                    ignore=shutil.ignore_patterns("*.so", "_build", "csrc", "__pycache__"))
    code = ("import sys; sys.path.insert(0, %r)\n"
            "try:\n import stealcode_b200.ops\nexcept ImportError as e:\n print('IMPORTERROR', e)\n") % str(tmp_path)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True)
    assert "IMPORTERROR" in r.stdout
