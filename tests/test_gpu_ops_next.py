"""Parity of the remaining elementwise ops of the reference (relu, gelu,
gelu_quick, sigmoid, tanh, exp, log, sqrt, pow, clamp, neg, abs) and of
layer_norm against the CPU oracle, through the C ABI.

Bars (stated per op): bit-exact where the op is one IEEE operation or a
selection (relu, neg, abs, clamp, sqrt); within a few ulp where CUDA's
expf / logf / tanhf / powf replace glibc's (each within 2 ulp of the exact
value; the reference's chain then rounds the same steps); gelu additionally
allows 2^-22 |x| absolute where 1 + tanh(..) cancels for x << 0.  bf16 results
are within one bf16 ulp (gelu: or the same absolute slack).  layer_norm: within
1e-5 of the exact (f64) value relative to |normalized * w| + |b| and to the
reference within that plus the reference's own sequential-sum drift.
"""
import numpy as np
import pytest

from _util import bf16_to_f32, misaligned_copy, to_dev, to_np, ulp_bf16, ulp_f32

F = np.float32

ULP_BAR = {  # op -> max ulp of the f32 result vs the oracle
    "relu": 0, "neg": 0, "abs": 0, "clamp": 0, "sqrt": 0,
    "exp": 4, "log": 4, "tanh": 4, "pow": 8, "sigmoid": 8, "gelu_quick": 8, "gelu": 8,
}


def _inputs(op, n, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(n) * 4).astype(F)
    if op in ("log", "sqrt", "pow"):
        x = np.abs(x) + F(1e-3)
    specials = np.array([0.0, 1.0, -1.0, 0.5, 30.0, -30.0, 100.0, -100.0, np.inf, -np.inf, np.nan],
                        F)
    if op in ("log", "sqrt", "pow"):
        specials = np.array([0.0, 1.0, 0.5, 2.0, 1e-30, 1e30, np.inf, -1.0, np.nan], F)
    x[: specials.size] = specials
    return x


def _params(op):
    return {"pow": (1.7, 0.0), "clamp": (-1.5, 2.5)}.get(op, (0.0, 0.0))


def _same_nan_and_zero(got, ref):
    gn, rn = np.isnan(got), np.isnan(ref)
    assert np.array_equal(gn, rn), "NaN positions differ"
    m = ~gn & ~((got == 0) & (ref == 0))  # +0 and -0 both accepted where the reference gives a zero
    return m


@pytest.mark.gpu
@pytest.mark.parametrize("op", list(ULP_BAR))
def test_unary_f32_matches_oracle(cuda, orc, op):
    from oxide_b200 import _lib, ops

    code = getattr(_lib, op.upper())
    x = _inputs(op, 100003, 500 + code)  # odd length: vector body + scalar tail
    a, b = _params(op)
    got = to_np(ops.unary(code, to_dev(x), a, b))
    ref = orc.unary(code, x, a, b)
    m = _same_nan_and_zero(got, ref)
    d = ulp_f32(got[m], ref[m])
    if op == "gelu":  # 1 + tanh(v) cancels for x << 0
        slack = np.abs(got[m].astype(np.float64) - ref[m]) <= 2.0 ** -22 * np.abs(x[m].astype(np.float64))
        d = np.where(slack, 0, d)
    assert d.max(initial=0) <= ULP_BAR[op], f"{op}: max {d.max()} ulp"
    # unaligned pointers take the scalar kernel: same results
    got2 = to_np(ops.unary(code, misaligned_copy(x), a, b))
    m2 = _same_nan_and_zero(got2, got)
    assert np.array_equal(got2[m2].view(np.uint32), got[m2].view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("op", list(ULP_BAR))
def test_unary_bf16_matches_oracle(cuda, orc, op):
    from oxide_b200 import _lib, ops

    code = getattr(_lib, op.upper())
    x = orc.f32_to_bf16(_inputs(op, 4099, 600 + code))
    a, b = _params(op)
    got = to_np(ops.unary(code, to_dev(x), a, b))
    ref = orc.unary(code, x, a, b)
    gf, rf = bf16_to_f32(got), bf16_to_f32(ref)
    m = _same_nan_and_zero(gf, rf)
    d = ulp_bf16(got[m], ref[m])
    if op == "gelu":
        xf = bf16_to_f32(x)[m].astype(np.float64)
        d = np.where(np.abs(gf[m].astype(np.float64) - rf[m]) <= 2.0 ** -22 * np.abs(xf), 0, d)
    assert d.max(initial=0) <= (0 if ULP_BAR[op] == 0 else 1), f"{op}: max {d.max()} bf16 ulp"


@pytest.mark.gpu
def test_named_activation_entry_points_match_unary(cuda):
    import torch

    from oxide_b200 import _lib

    x = torch.randn(5000, device=cuda)
    st = torch.cuda.current_stream().cuda_stream
    for name, code in (("relu", _lib.RELU), ("gelu", _lib.GELU), ("sigmoid", _lib.SIGMOID),
                       ("tanh", _lib.TANH)):
        a = torch.empty_like(x)
        b = torch.empty_like(x)
        _lib.call(f"oxide_{name}_f32", x.data_ptr(), a.data_ptr(), x.numel(), st)
        _lib.call("oxide_unary_f32", code, x.data_ptr(), b.data_ptr(), x.numel(), 0.0, 0.0, st)
        assert torch.equal(a, b), name


@pytest.mark.gpu
def test_unary_argument_errors(cuda):
    import torch

    from oxide_b200 import _lib

    x = torch.zeros(16, device=cuda)
    st = torch.cuda.current_stream().cuda_stream
    assert _lib.raw("oxide_unary_f32", _lib.CLAMP, x.data_ptr(), x.data_ptr(), 16, 2.0, 1.0,
                    st) == _lib.ERR_INVALID_ARG
    assert "min <= max" in _lib.last_error()
    assert _lib.raw("oxide_unary_f32", 99, x.data_ptr(), x.data_ptr(), 16, 0.0, 0.0,
                    st) == _lib.ERR_INVALID_ARG
    assert _lib.raw("oxide_unary_f32", _lib.EXP, None, None, 0, 0.0, 0.0, st) == _lib.OK


def _ln_scale(x, w, b):
    x = x.astype(np.float64)
    mean = x.mean(axis=1, keepdims=True)
    sd = np.sqrt(((x - mean) ** 2).mean(axis=1, keepdims=True) + np.float64(F(1e-5)))
    nrm = (x - mean) / sd
    exact = nrm * w.astype(np.float64) + b.astype(np.float64)
    return exact, np.abs(nrm * w.astype(np.float64)) + np.abs(b.astype(np.float64))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows,cols", [(3, 1), (8, 33), (16, 768), (4, 4096), (3, 5000), (2, 20000)])
def test_layer_norm_matches_oracle(cuda, orc, dtype, rows, cols):
    from oxide_b200 import ops

    rng = np.random.default_rng(rows * 7919 + cols)
    x = (rng.standard_normal((rows, cols)) * 3 + 1).astype(F)
    w = rng.uniform(0.5, 1.5, cols).astype(F)
    b = rng.uniform(-0.5, 0.5, cols).astype(F)
    if dtype == "bf16":
        x, w, b = orc.f32_to_bf16(x), orc.f32_to_bf16(w), orc.f32_to_bf16(b)
    got = to_np(ops.layer_norm(to_dev(x), to_dev(w), to_dev(b), 1e-5))
    ref = orc.layer_norm(x, w, b, 1e-5)
    xf = bf16_to_f32(x) if dtype == "bf16" else x
    wf = bf16_to_f32(w) if dtype == "bf16" else w
    bf = bf16_to_f32(b) if dtype == "bf16" else b
    exact, scale = _ln_scale(xf, wf, bf)
    if dtype == "f32":
        g = got.astype(np.float64)
        lim = 1e-5 * scale + 1e-30
        assert np.all(np.abs(g - exact) <= lim), "kernel vs exact"
        assert np.all(np.abs(g - ref) <= lim + np.abs(ref - exact)), "kernel vs reference + its drift"
    else:
        d = ulp_bf16(got, ref)
        gd = np.abs(bf16_to_f32(got).astype(np.float64) - bf16_to_f32(ref))
        ok = (d <= 1) | (gd <= 2.0 ** -8 * scale)  # cancellation in w * n + b
        assert ok.all(), f"max {d.max()} bf16 ulp"


@pytest.mark.gpu
def test_layer_norm_constant_rows_and_shape_errors(cuda, orc):
    import torch

    from oxide_b200 import OxideError, ops

    x = torch.full((5, 768), 2.5, device=cuda)
    w = torch.rand(768, device=cuda) + 0.5
    b = torch.rand(768, device=cuda) - 0.5
    y = ops.layer_norm(x, w, b, 1e-5)
    assert torch.equal(y, b.expand_as(y))  # mean exact, deviations 0, 0 * w + b = b
    with pytest.raises(OxideError, match="bias shape"):
        ops.layer_norm(x, w, b[:10], 1e-5)
    with pytest.raises(OxideError, match="weight shape"):
        ops.layer_norm(x, w[:10], b, 1e-5)
