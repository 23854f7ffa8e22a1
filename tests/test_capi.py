"""The C-ABI library loads and exports exactly what include/llambda_cuda.h
declares; host-side behaviour that needs no GPU."""
import ctypes
import hashlib
import os
import re
import subprocess

import numpy as np
import pytest

import llambda_b200 as LB
from llambda_b200 import _native as N

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "llambda_cuda.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"LLAMBDA_CUDA_API\s+[^;(]*?\b(llambda_cuda_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    syms = declared_symbols()
    assert len(syms) >= 20
    lib = LB.lib()
    for s in syms:
        assert hasattr(lib, s), s
    out = subprocess.run(["nm", "-D", "--defined-only", N.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = sorted(set(re.findall(r"\bT (llambda_cuda_\w+)", out)))
    assert exported == syms  # nothing else leaks (static cudart stays private)
    assert set(N.SIGNATURES) == set(syms)


def test_sha256_matches_fips_vectors():
    assert LB.sha256(b"abc") == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"
    assert LB.sha256(b"") == hashlib.sha256(b"").hexdigest()
    rng = np.random.default_rng(0)
    for n in (55, 56, 63, 64, 65, 119, 120, 1000, 4096 + 7):
        data = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert LB.sha256(data) == hashlib.sha256(data).hexdigest()
    out = ctypes.create_string_buffer(10)
    assert LB.lib().llambda_cuda_sha256(b"abc", 3, out, 10) == -1
    assert "65-byte" in N.last_error()


def test_versions_and_probe_without_gpu():
    assert LB.bridge_version().startswith("cuda-")
    assert "CUDA runtime" in LB.runtime_version()
    rc = LB.probe()
    assert rc in (0, 1)
    if rc == 0:
        assert N.last_error()


def test_null_arguments_are_errors_not_crashes():
    L = LB.lib()
    h = ctypes.c_void_p(123)
    assert L.llambda_cuda_session_create(None, ctypes.byref(h)) == -1
    assert "required" in N.last_error()
    assert L.llambda_cuda_session_create_from_tensor(12, 256, 1, 1, None, 144, ctypes.byref(h)) == -1
    assert h.value is None  # *result cleared on entry
    assert L.llambda_cuda_moe_session_create(None, ctypes.byref(h)) == -1
    assert L.llambda_cuda_session_input_element_count(None) == 0
    assert L.llambda_cuda_session_output_element_count(None) == 0
    assert L.llambda_cuda_moe_session_hidden(None) == 0
    L.llambda_cuda_session_destroy(None)
    L.llambda_cuda_moe_session_destroy(None)
    assert L.llambda_cuda_session_run(None, None, 0, None, 0) == -1


def test_projection_file_header_roundtrip(tmp_path):
    from llambda_b200.accelerator import PROJECTION_HEADER, write_projection_file
    data = np.arange(144 * 3, dtype=np.uint8)
    p = write_projection_file(str(tmp_path / "t.bin"), LB.TYPE_Q4_K, 256, 3, 1, data)
    raw = open(p, "rb").read()
    magic, ver, t, ne0, ne1, ne2, nbytes, off = PROJECTION_HEADER.unpack(raw[:56])
    assert (magic, ver, t, ne0, ne1, ne2, nbytes) == (b"LLBCUDA1", 1, 12, 256, 3, 1, 432)
    assert raw[off:] == data.tobytes()
    with pytest.raises(ValueError):
        write_projection_file(str(tmp_path / "u.bin"), LB.TYPE_Q4_K, 256, 4, 1, data)


def test_session_create_without_device_fails_cleanly():
    if LB.probe() == 1:
        pytest.skip("a device is present")
    blk = np.zeros(144, np.uint8)
    blk[1] = 0x3C
    with pytest.raises(LB.LlambdaCudaError):
        LB.ProjectionSession.from_tensor(LB.TYPE_Q4_K, 256, 1, blk)
