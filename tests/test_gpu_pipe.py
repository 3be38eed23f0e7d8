"""Host-buffer pipeline (oxide_pipe_*): results equal the oracle (and the
device-buffer entry points) for pageable and page-locked host memory, across
many chunks and a ragged last chunk."""
import ctypes as C

import numpy as np
import pytest
import torch

from _util import assert_bits_equal, assert_parity_rel, assert_ulp, rms_norm_exact

pytestmark = pytest.mark.gpu
F = np.float32


@pytest.fixture()
def pipe(cuda):
    from oxide_b200._lib import call, lib

    h = C.c_void_p()
    call("oxide_pipe_create", 0, 1 << 20, 3, C.byref(h))  # 1 MiB chunks: many chunks
    yield h
    lib().oxide_pipe_destroy(h)


def host(a, pinned):
    if not pinned:
        return np.ascontiguousarray(a)
    t = torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
    return t.numpy()  # a numpy view of page-locked memory (t kept alive by the view)


@pytest.mark.parametrize("pinned", [False, True])
def test_pipe_binary_and_broadcast(pipe, orc, pinned):
    from oxide_b200._lib import call

    rng = np.random.default_rng(1)
    n = 3 * (1 << 20) + 4096 * 3  # ragged last chunk
    a = host(rng.standard_normal(n, dtype=F), pinned)
    b = host(rng.standard_normal(n, dtype=F), pinned)
    out = host(np.zeros(n, F), pinned)
    call("oxide_pipe_binary_f32", pipe, 0, a.ctypes.data, n, b.ctypes.data, n, out.ctypes.data, n)
    assert_bits_equal(out, orc.binary(0, a, b))
    s = host(rng.uniform(0.5, 1.5, 4096).astype(F), pinned)
    call("oxide_pipe_binary_f32", pipe, 2, a.ctypes.data, n, s.ctypes.data, 4096, out.ctypes.data, n)
    assert_bits_equal(out, orc.binary(2, a, s, n))


@pytest.mark.parametrize("pinned", [False, True])
def test_pipe_silu_mul(pipe, orc, pinned):
    from oxide_b200._lib import call

    rng = np.random.default_rng(2)
    n = 5 * (1 << 18) + 3
    g = host(rng.standard_normal(n, dtype=F) * F(4), pinned)
    u = host(rng.standard_normal(n, dtype=F), pinned)
    out = host(np.zeros(n, F), pinned)
    call("oxide_pipe_silu_mul_f32", pipe, g.ctypes.data, u.ctypes.data, out.ctypes.data, n)
    # identical to the device-buffer entry point
    from oxide_b200 import ops

    dev = ops.silu_mul(torch.from_numpy(np.array(g)).cuda(), torch.from_numpy(np.array(u)).cuda())
    assert_bits_equal(out, dev.cpu().numpy())
    assert_ulp(out, orc.silu_mul(g, u), 8)


def test_pipe_rms_norm(pipe, orc):
    from oxide_b200._lib import call

    rng = np.random.default_rng(3)
    rows, cols = 300, 4096
    x = rng.standard_normal((rows, cols), dtype=F)
    w = rng.uniform(0.5, 1.5, cols).astype(F)
    out = np.zeros_like(x)
    call("oxide_pipe_rms_norm_f32", pipe, x.ctypes.data, w.ctypes.data, out.ctypes.data, rows,
         cols, 1e-5)
    assert_parity_rel(out, orc.rms_norm(x, w, 1e-5), rms_norm_exact(x, w, 1e-5), 1e-5)


def test_pipe_rejects_bad_arguments(pipe, olib):
    lib = olib.lib()
    buf = np.zeros(16, F)
    p = buf.ctypes.data
    assert lib.oxide_pipe_binary_f32(pipe, 0, p, 3, p, 16, p, 16) == olib.ERR_INVALID_ARG
    assert lib.oxide_pipe_binary_f32(None, 0, p, 16, p, 16, p, 16) == olib.ERR_INVALID_ARG
    # a row larger than the 1 MiB chunk
    assert lib.oxide_pipe_rms_norm_f32(pipe, p, p, p, 1, 1 << 20, 1e-5) == olib.ERR_UNSUPPORTED
