"""Argument checks of oxide_b200.pipe, on CPU.

The oxide_pipe_* entry points size every host read and write from the counts
they are given, so the wrapper must reject arrays of the wrong dtype, shape or
layout before it calls them.  A Pipe with no device handle is enough here:
valid arguments reach the handle check ("pipe is closed"), invalid ones fail
earlier with their own message."""
import ctypes as C

import numpy as np
import pytest

from oxide_b200.pipe import Pipe

F, BF = np.float32, np.uint16


@pytest.fixture()
def pipe():
    p = Pipe.__new__(Pipe)
    p._h = C.c_void_p()
    p._keep = []
    p._deferred = False
    return p


def z(*shape, dtype=F):
    return np.zeros(shape, dtype)


def closed(fn, *a, **k):
    with pytest.raises(ValueError, match="pipe is closed"):
        fn(*a, **k)


def test_valid_arguments_reach_the_handle(pipe):
    closed(pipe.add, z(8, 16), z(8, 16))
    closed(pipe.mul_rowbcast, z(8, 16), z(16))
    closed(pipe.add_mul_rowbcast, z(8, 16), z(8, 16), z(16))
    closed(pipe.silu_mul, z(64), z(64))
    closed(pipe.rms_norm, z(4, 32), z(32), 1e-5)
    closed(pipe.add_rms_norm, z(4, 32), z(4, 32), z(32), 1e-5)
    closed(pipe.add_rms_norm, z(4, 32, dtype=BF), z(4, 32, dtype=BF), z(32, dtype=BF), 1e-5)
    closed(pipe.scale_mask_softmax, z(8, 64), 0.5, lens=np.zeros(2, np.int32), rows_per_len=4)
    closed(pipe.argmax_rows, z(3, 100))
    closed(pipe.rope_bf16, z(2, 4, 8, dtype=BF), z(16, 4), z(16, 4), k=z(2, 1, 8, dtype=BF))
    closed(pipe.sync)


def test_dtype_shape_and_layout_are_checked(pipe):
    with pytest.raises(TypeError, match="dtype"):
        pipe.add(z(8, 16), z(8, 16, dtype=np.float64))
    with pytest.raises(TypeError, match="numpy array"):
        pipe.silu_mul([1.0], z(1))
    with pytest.raises(ValueError, match="C-contiguous"):
        pipe.silu_mul(z(8, 16).T, z(16, 8))
    with pytest.raises(ValueError, match="same shape"):
        pipe.silu_mul(z(64), z(63))
    with pytest.raises(ValueError, match="s must have shape"):
        pipe.mul_rowbcast(z(8, 16), z(8))
    with pytest.raises(ValueError, match="one value per column"):
        pipe.add_mul_rowbcast(z(8, 16), z(8, 16), z(8))
    with pytest.raises(ValueError, match="w must have shape"):
        pipe.rms_norm(z(4, 32), z(31), 1e-5)
    with pytest.raises(TypeError, match="dtype"):
        pipe.add_rms_norm(z(4, 32, dtype=BF), z(4, 32), z(32), 1e-5)
    with pytest.raises(ValueError, match="expected shape"):
        pipe.rms_norm(z(4, 32), z(32), 1e-5, out=z(4, 16))
    with pytest.raises(ValueError, match="lens needs"):
        pipe.scale_mask_softmax(z(8, 64), 0.5, lens=np.zeros(3, np.int32), rows_per_len=4)
    with pytest.raises(ValueError, match="cos and sin"):
        pipe.rope_bf16(z(2, 4, 8, dtype=BF), z(16, 8), z(16, 8))
    with pytest.raises(ValueError, match="positions"):
        pipe.rope_bf16(z(2, 4, 8, dtype=BF), z(16, 4), z(16, 4), positions=np.zeros(3, np.int32))
    with pytest.raises(ValueError, match="op must be"):
        pipe.binary("pow", z(4), z(4))
