"""C ABI checks that need no GPU: the library loads, exports exactly what
include/oxide_ops.h declares, and rejects bad arguments / injected faults
before it touches the device."""
import ctypes as C
import os
import re
import subprocess

import pytest

from conftest import PKG, ROOT

HEADER = os.path.join(ROOT, "include", "oxide_ops.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(oxide_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_header_symbols_are_exported(olib):
    lib = olib.lib()
    for name in header_functions():
        assert hasattr(lib, name), f"{name} declared in include/oxide_ops.h but not exported"


def test_binding_covers_header(olib):
    assert sorted(olib.SIGNATURES) == header_functions()


def test_only_oxide_symbols_exported(olib):
    out = subprocess.run(["nm", "-D", "--defined-only", olib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = [l.split()[-1] for l in out.splitlines() if " T " in l]
    assert exported and all(s.startswith("oxide_") for s in exported), \
        [s for s in exported if not s.startswith("oxide_")][:10]


def test_status_strings(olib):
    names = {olib.status_name(c) for c in range(0, -8, -1)}
    assert "OXIDE_OK" in names and "OXIDE_ERR_INVALID_ARG" in names and len(names) == 8
    assert olib.status_name(-99) == "OXIDE_ERR_UNKNOWN"
    assert olib.lib().oxide_version().decode().startswith("oxide-b200")


def test_zero_size_is_noop(olib):
    lib = olib.lib()
    assert lib.oxide_add_f32(None, None, None, 0, None) == 0
    assert lib.oxide_rms_norm_bf16(None, None, None, 0, 4096, 1e-5, None) == 0
    assert lib.oxide_softmax_f32(None, None, 0, 10, 1, None) == 0
    assert lib.oxide_argmax_rows_f32(None, 0, 10, None, None) == 0


FAKE = 0x1000  # never dereferenced: every case below fails validation first


@pytest.mark.parametrize("call", [
    lambda l: l.oxide_add_f32(None, FAKE, FAKE, 8, None),
    lambda l: l.oxide_binary_f32(7, FAKE, 8, FAKE, 8, FAKE, 8, None),
    lambda l: l.oxide_binary_f32(0, FAKE, 3, FAKE, 8, FAKE, 8, None),   # 8 % 3 != 0
    lambda l: l.oxide_binary_f32(0, FAKE, 16, FAKE, 8, FAKE, 8, None),  # na > n
    lambda l: l.oxide_rms_norm_f32(FAKE, FAKE, FAKE, 4, 0, 1e-5, None),
    lambda l: l.oxide_rms_norm_f32(FAKE, FAKE, FAKE, 1 << 40, 1 << 30, 1e-5, None),
    lambda l: l.oxide_add_rms_norm_f32(FAKE, FAKE, FAKE, FAKE, FAKE, 4, 8, 1e-5, None),  # h == y
    lambda l: l.oxide_scale_mask_softmax_f32(FAKE, FAKE, 4, 8, 1.0, None, 0, FAKE, 0, 0, None),
    lambda l: l.oxide_scale_mask_softmax_f32(FAKE, FAKE, 4, 8, 1.0, None, 0, None, 1, 9, None),
    lambda l: l.oxide_softmax_f32(FAKE, FAKE, 2, 4, 3, None),  # inner > 1 in place
    lambda l: l.oxide_rope_bf16(FAKE, FAKE, 4, None, None, 0, FAKE, FAKE, 8, None, 16, 128, 0, None),
    lambda l: l.oxide_rope_bf16(FAKE, FAKE, 4, None, None, 0, FAKE, FAKE, 16, None, 16, 7, 0, None),
    lambda l: l.oxide_rope_bf16(FAKE, FAKE, 4, None, None, 0, FAKE, FAKE, 16, None, 16, 128, 2, None),
    lambda l: l.oxide_argmax_rows_f32(FAKE, 4, 0, FAKE, None),
    lambda l: l.oxide_reduce_rows_f32(5, FAKE, 4, 4, FAKE, None),
    lambda l: l.oxide_rope_table_host_f32(1e4, 3, 4, FAKE, FAKE),
    lambda l: l.oxide_device_status(0, None),
])
def test_invalid_arguments(olib, call):
    assert call(olib.lib()) == olib.ERR_INVALID_ARG
    assert olib.last_error() != ""


def test_reduce_workspace_checked(olib):
    lib = olib.lib()
    need = lib.oxide_reduce_workspace_bytes(1 << 20)
    assert need >= 8
    out = C.c_double()
    assert lib.oxide_reduce_f32(0, FAKE, 1 << 20, C.addressof(out), None, need, None) == olib.ERR_WORKSPACE
    assert lib.oxide_reduce_f32(0, FAKE, 1 << 20, C.addressof(out), FAKE, need - 8, None) == olib.ERR_WORKSPACE


def test_fault_injection_fires_once(olib):
    lib = olib.lib()
    lib.oxide_debug_fail_next(b"oxide_rms_norm_f32")
    # another op is not affected, and a zero-size call of the armed op still fails
    assert lib.oxide_add_f32(None, None, None, 0, None) == 0
    assert lib.oxide_rms_norm_f32(None, None, None, 0, 1, 1e-5, None) == olib.ERR_INJECTED
    assert "injected" in olib.last_error()
    assert lib.oxide_rms_norm_f32(None, None, None, 0, 1, 1e-5, None) == 0
    lib.oxide_debug_fail_next(b"*")
    assert lib.oxide_softmax_f32(None, None, 0, 1, 1, None) == olib.ERR_INJECTED
    lib.oxide_debug_fail_next(b"oxide_add_f32")
    lib.oxide_debug_fail_next(None)  # clears
    assert lib.oxide_add_f32(None, None, None, 0, None) == 0


def test_last_error_is_per_thread(olib):
    import threading

    lib = olib.lib()
    assert lib.oxide_argmax_rows_f32(FAKE, 4, 0, FAKE, None) == olib.ERR_INVALID_ARG
    seen = {}

    def worker():
        seen["msg"] = olib.last_error()

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert seen["msg"] == "" and "cols" in olib.last_error()


def test_rope_table_host_matches_oracle(olib, orc):
    # Host-side model set-up: same glibc calls as the oracle -> identical tables.
    import numpy as np

    cos = np.empty((64, 64), np.float32)
    sin = np.empty((64, 64), np.float32)
    assert olib.lib().oxide_rope_table_host_f32(1e6, 128, 64, cos.ctypes.data, sin.ctypes.data) == 0
    oc, osn = orc.rope_table(1e6, 128, 64)
    assert np.array_equal(cos, oc) and np.array_equal(sin, osn)


def test_pipe_create_without_device_fails_cleanly(olib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a device is present")
    h = C.c_void_p()
    rc = olib.lib().oxide_pipe_create(0, 1 << 20, 3, C.byref(h))
    assert rc == olib.ERR_INVALID_ARG and not h.value


def test_package_fails_loudly_without_library(tmp_path, monkeypatch):
    import importlib

    from oxide_b200 import _lib

    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(ImportError):
        _lib.lib()
    importlib.reload(_lib)


def test_fastdiv_formula():
    # Host restatement of oxide_common.cuh's FastDiv: q = (umulhi(n, m) + n) >> s.
    import random

    def make(d):
        s = 0
        while (1 << s) < d:
            s += 1
        m = ((((1 << s) - d) << 32) // d + 1) & 0xFFFFFFFF
        return m, s

    rng = random.Random(1)
    divisors = [1, 2, 3, 7, 512, 1000, 1024, 4095, 32000, (1 << 31) - 1, 1 << 31, (1 << 31) + 1,
                (1 << 32) - 1] + [rng.randrange(1, 1 << 32) for _ in range(200)]
    for d in divisors:
        m, s = make(d)
        for n in [0, 1, d - 1, d, d + 1, (1 << 32) - 1] + [rng.randrange(0, 1 << 32) for _ in range(200)]:
            n &= 0xFFFFFFFF
            q = (((n * m) >> 32) + n) >> s
            assert q == n // d, (d, n)
