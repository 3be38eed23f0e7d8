"""Argument checks of the tensor-level ops, on CPU.

Every kernel sizes its reads and writes by the input's element count and
dtype, so an operand or output of another dtype or size would be read or
written past its end on the device.  oxide_b200.ops rejects those before it
touches a device; these tests call it with CPU tensors, which would fail the
device check, to show the shape/dtype error comes first."""
import pytest
import torch

from oxide_b200 import OxideError, ops

f32, bf16 = torch.float32, torch.bfloat16


def t(*shape, dtype=f32):
    return torch.zeros(shape, dtype=dtype)


def raises(match, fn, *a, **k):
    with pytest.raises(OxideError, match=match):
        fn(*a, **k)


def test_add_layer_norm_weight_bias_and_out():
    x = t(4, 64)
    raises("weight dtype", ops.add_layer_norm, x, x, t(64, dtype=bf16), t(64), 1e-5)
    raises("bias dtype", ops.add_layer_norm, x, x, t(64), t(64, dtype=bf16), 1e-5)
    raises("out must be", ops.add_layer_norm, x, x, t(64), t(64), 1e-5, out=t(4, 32))
    raises("out must be", ops.add_layer_norm, x, x, t(64), t(64), 1e-5, out=t(4, 64, dtype=bf16))
    raises("residual", ops.add_layer_norm, x, t(4, 64, dtype=bf16), t(64), t(64), 1e-5)


def test_layer_norm_weight_bias_and_out():
    x = t(4, 64, dtype=bf16)
    raises("weight dtype", ops.layer_norm, x, t(64), t(64, dtype=bf16), 1e-5)
    raises("out must be", ops.layer_norm, x, t(64, dtype=bf16), t(64, dtype=bf16), 1e-5, out=t(4, 64))


def test_add_mul_rowbcast_out():
    a, s = t(8, 32), t(32)
    raises("out must be", ops.add_mul_rowbcast, a, a, s, out=t(8, 16))
    raises("out must be", ops.add_mul_rowbcast, a, a, s, out=t(8, 32, dtype=bf16))
    buf = t(8, 32)
    raises("must not alias s", ops.add_mul_rowbcast, a, a, buf[0], out=buf)
    raises("share shape and dtype", ops.add_mul_rowbcast, a, a, t(32, dtype=bf16))


def test_mul_rowbcast_operand():
    raises("s dtype", ops.mul_rowbcast, t(8, 32), t(32, dtype=bf16))
    raises("last dim", ops.mul_rowbcast, t(8, 32), t(16))


def test_norms():
    x = t(4, 64)
    raises("weight dtype", ops.rms_norm, x, t(64, dtype=bf16), 1e-5)
    raises("out must be", ops.rms_norm, x, t(64), 1e-5, out=t(4, 63))
    raises("residual", ops.add_rms_norm, x, t(4, 32), t(64), 1e-5)
    raises("h must be", ops.add_rms_norm, x, x, t(64), 1e-5, h=t(4, 64, dtype=bf16))
    raises("y must be", ops.add_rms_norm, x, x, t(64), 1e-5, y=t(3, 64))
    h = t(4, 64)
    raises("must not alias", ops.add_rms_norm, x, x, t(64), 1e-5, h=h, y=h)


def test_silu_mul_and_unary():
    g = t(16)
    raises("up dtype", ops.silu_mul, g, t(16, dtype=bf16))
    raises("out must be", ops.silu_mul, g, g, out=t(15))
    raises("out must be", ops.unary, 0, g, out=t(16, dtype=bf16))


def test_softmax_lens_and_out():
    x = t(64, 128)
    lens = torch.zeros(3, dtype=torch.int32)
    raises("lens needs", ops.scale_mask_softmax, x, 0.1, lens=lens, rows_per_len=16)
    raises("out must be", ops.scale_mask_softmax, x, 0.1, out=t(64, 64))
    raises("out must be float32", ops.softmax_with_temperature, t(2, 8, dtype=bf16), 1.0, out=t(2, 8, dtype=bf16))


def test_rope():
    q, k = t(8, 4, 16, dtype=bf16), t(8, 2, 16, dtype=bf16)
    cos = sin = t(8, 8)
    raises("k dtype", ops.rope, q, t(8, 2, 16), cos, sin)
    raises("q_out must be", ops.rope, q, k, cos, sin, q_out=t(8, 4, 16))
    raises("k_out must be", ops.rope, q, k, cos, sin, k_out=t(8, 1, 16, dtype=bf16))
    raises("float32", ops.rope, q, k, t(8, 8, dtype=bf16), sin)


def test_reduce_repeat_kv_decode_attention():
    x = t(1000)
    raises("workspace must hold", ops.reduce, x, 0, workspace=torch.zeros(8, dtype=torch.uint8))
    raises("one float64", ops.reduce, x, 0, out=t(1))
    kv = t(1, 2, 8, 16)
    raises("out must be", ops.repeat_kv, kv, 2, out=t(1, 2, 8, 16))
    raises("n_rep", ops.repeat_kv, kv, 0)
    q = t(1, 4, 16)
    raises("k_cache dtype", ops.decode_attention, q, t(1, 2, 8, 16, dtype=bf16), t(1, 2, 8, 16, dtype=bf16))
    raises("out must be", ops.decode_attention, q, kv, kv, out=t(1, 4, 8))
    raises("lens needs", ops.decode_attention, t(2, 4, 16), t(2, 2, 8, 16), t(2, 2, 8, 16),
           lens=torch.zeros(1, dtype=torch.int32))
    raises("workspace must hold", ops.decode_attention, q, kv, kv, workspace=torch.zeros(4, dtype=torch.uint8))
