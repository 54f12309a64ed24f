"""The C-ABI library loads and exports every entry point include/tts_cuda.h declares, and the
ctypes binding knows each of them. No GPU call is made."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tts_cuda.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"TTS_API\s+[\w\s\*]+?\b(tts_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib_path():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "dream-tts_b200"))
    import build
    return build.build()


def test_header_declares_entry_points():
    names = declared()
    assert "tts_proj_forward" in names and "tts_conv1d_nlc" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (tts_\w+)", out))
    missing = [n for n in declared() if n not in exported]
    assert not missing, missing


def test_ctypes_binding_covers_header(lib_path):
    from ttsnn import _lib
    lib = _lib.load()
    assert lib.tts_abi_version() == 1
    assert sorted(_lib.SIGNATURES) == declared()


def test_errors_without_gpu_are_reported_not_raised(lib_path):
    import ctypes as C
    from ttsnn import _lib
    lib = _lib.load()
    p = C.c_void_p()
    rc = lib.tts_ctx_create(0, 0, C.byref(p))
    assert rc == 1 and "max_lanes" in _lib.last_error()
    rc = lib.tts_proj_forward(None, None, 1, 64, None, 128, 0, None, 0, None)
    assert rc == 1 and "proj" in _lib.last_error()
