"""The C oracle against an independent numpy restatement of the same loop bodies.

Order-dependent sums are restated as explicit sequential float32 loops, so the
ops without transcendental calls (binary ops, RMSNorm, RoPE, argmax, row
reductions) must agree bit-for-bit.  numpy's float32 exp/pow/cos/sin are not
glibc's, so ops that call them are compared within a small ulp bound.
"""
import numpy as np
import pytest

F = np.float32


def ulp_diff(a, b):
    a = np.ascontiguousarray(a, F).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, F).view(np.int32).astype(np.int64)
    a = np.where(a < 0, -(a & 0x7FFFFFFF), a)
    b = np.where(b < 0, -(b & 0x7FFFFFFF), b)
    return np.abs(a - b)


def np_binary(op, a, b, n):
    i = np.arange(n)
    x, y = a[i % a.size], b[i % b.size]
    return [x + y, x - y, x * y, x / y][op].astype(F)


def np_rms_norm(x, w, eps):
    rows, cols = x.shape
    out = np.empty_like(x)
    for r in range(rows):
        ss = F(0)
        for v in x[r]:
            ss = F(ss + F(v * v))
        rms = np.sqrt(F(F(ss / F(cols)) + F(eps)))
        out[r] = (x[r] / rms) * w
    return out


def np_softmax_rows(s):
    out = np.empty_like(s)
    for r in range(s.shape[0]):
        m = F(-np.inf)
        for v in s[r]:
            m = max(m, v)
        e = np.exp(s[r] - m).astype(F)
        tot = F(0)
        for v in e:
            tot = F(tot + v)
        out[r] = e / tot
    return out


def np_rope(x, cos, sin, pos):
    # x [tokens, heads, d] token-major
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    c = cos[pos][:, None, :]
    s = sin[pos][:, None, :]
    return np.concatenate([(x1 * c) - (x2 * s), (x1 * s) + (x2 * c)], axis=-1).astype(F)


@pytest.mark.parametrize("op", [0, 1, 2, 3])
@pytest.mark.parametrize("na,nb,n", [(37, 37, 37), (60, 12, 60), (12, 60, 60), (4, 6, 24)])
def test_binary_bit_exact(orc, op, na, nb, n):
    rng = np.random.default_rng(op * 100 + n)
    a = rng.standard_normal(na, dtype=F)
    b = rng.standard_normal(nb, dtype=F) + F(3.0)
    assert np.array_equal(orc.binary(op, a, b, n), np_binary(op, a, b, n))


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 17), (5, 128), (2, 4096)])
def test_rms_norm_bit_exact(orc, rows, cols):
    rng = np.random.default_rng(rows * cols)
    x = rng.standard_normal((rows, cols), dtype=F)
    w = rng.uniform(0.5, 1.5, cols).astype(F)
    assert np.array_equal(orc.rms_norm(x, w, 1e-5), np_rms_norm(x, w, 1e-5))


def test_add_rms_norm_bit_exact(orc):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, 96), dtype=F)
    r = rng.standard_normal((4, 96), dtype=F)
    w = rng.uniform(0.5, 1.5, 96).astype(F)
    h, y = orc.add_rms_norm(x, r, w, 1e-6)
    assert np.array_equal(h, x + r)
    assert np.array_equal(y, np_rms_norm(x + r, w, 1e-6))


def test_bf16_rms_norm_matches_widened_f32(orc):
    rng = np.random.default_rng(4)
    xb = orc.f32_to_bf16(rng.standard_normal((3, 64), dtype=F))
    wb = orc.f32_to_bf16(rng.uniform(0.5, 1.5, 64).astype(F))
    ref = orc.f32_to_bf16(np_rms_norm(orc.bf16_to_f32(xb).reshape(3, 64), orc.bf16_to_f32(wb), 1e-5))
    assert np.array_equal(orc.rms_norm(xb, wb, 1e-5), ref.reshape(3, 64))


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 31), (4, 500)])
def test_softmax_within_ulps(orc, rows, cols):
    rng = np.random.default_rng(rows + cols)
    x = rng.standard_normal((rows, cols), dtype=F) * F(4)
    got = orc.softmax(x, rows, cols, 1)
    assert ulp_diff(got, np_softmax_rows(x)).max() <= 4


def test_softmax_inner_dim(orc):
    rng = np.random.default_rng(9)
    x = rng.standard_normal((2, 5, 3), dtype=F)  # softmax over dim 1
    got = orc.softmax(x, 2, 5, 3).reshape(2, 5, 3)
    ref = np.transpose(np_softmax_rows(np.transpose(x, (0, 2, 1)).reshape(6, 5)).reshape(2, 3, 5),
                       (0, 2, 1))
    assert ulp_diff(got, ref).max() <= 4


def test_scale_mask_softmax_within_ulps(orc):
    rng = np.random.default_rng(12)
    rows, cols = 6, 200
    x = rng.standard_normal((rows, cols), dtype=F) * F(11.3)
    mask = np.where(rng.random(cols) < 0.2, -np.inf, 0.0).astype(F)
    scale = F(1.0) / np.sqrt(F(128))
    got = orc.scale_mask_softmax(x, cols, scale, mask=mask)
    s = (x * scale).astype(F) + mask[np.arange(cols) % cols]
    assert ulp_diff(got, np_softmax_rows(s.astype(F))).max() <= 4


def test_silu_mul_within_ulps(orc):
    rng = np.random.default_rng(13)
    g = rng.standard_normal(5000, dtype=F) * F(3)
    u = rng.standard_normal(5000, dtype=F)
    ref = ((g * (F(1) / (F(1) + np.exp(-g).astype(F)))) * u).astype(F)
    assert ulp_diff(orc.silu_mul(g, u), ref).max() <= 4


def test_rope_bit_exact(orc):
    rng = np.random.default_rng(14)
    cos, sin = orc.rope_table(1e6, 64, 20)
    x = rng.standard_normal((20, 3, 64), dtype=F)
    pos = rng.integers(0, 20, 20).astype(np.int32)
    assert np.array_equal(orc.rope(x, 20, 3, 64, 0, cos, sin, positions=pos), np_rope(x, cos, sin, pos))
    # head-major layout is the same rotation on a transposed tensor
    xh = np.ascontiguousarray(np.transpose(x, (1, 0, 2)))
    got = orc.rope(xh, 20, 3, 64, 1, cos, sin, positions=pos)
    assert np.array_equal(np.transpose(got, (1, 0, 2)), np_rope(x, cos, sin, pos))


def test_rope_table_within_ulps(orc):
    head_dim, max_pos = 128, 300
    cos, sin = orc.rope_table(1e6, head_dim, max_pos)
    i = np.arange(head_dim // 2, dtype=F)
    freq = np.power(F(1e6), (F(-2.0) * i) / F(head_dim)).astype(F)
    ang = (np.arange(max_pos, dtype=F)[:, None] * freq[None, :]).astype(F)
    # cos/sin of the same f32 angle, correctly rounded via f64
    assert np.max(np.abs(cos - np.cos(ang.astype(np.float64)).astype(F))) < 1e-5
    assert np.max(np.abs(sin - np.sin(ang.astype(np.float64)).astype(F))) < 1e-5


def test_argmax_matches_numpy(orc):
    rng = np.random.default_rng(15)
    x = rng.standard_normal((50, 777), dtype=F)
    x[3, 100] = x[3, 200] = 99.0  # tie -> lowest index
    assert np.array_equal(orc.argmax_rows(x, 777), np.argmax(x, axis=1).astype(np.uint32))


def test_row_reductions_bit_exact(orc):
    rng = np.random.default_rng(16)
    x = rng.standard_normal((7, 333), dtype=F)
    for op in (orc.RED_SUM, orc.RED_MAX, orc.RED_SUMSQ):
        ref = []
        for row in x:
            acc = F(-np.inf) if op == orc.RED_MAX else F(0)
            for v in row:
                acc = max(acc, v) if op == orc.RED_MAX else F(acc + (v if op == orc.RED_SUM else F(v * v)))
            ref.append(acc)
        assert np.array_equal(orc.reduce_rows(op, x, 333), np.array(ref, F))


def test_unary_ops_match_numpy(orc):
    rng = np.random.default_rng(77)
    x = (rng.standard_normal(20000) * 3).astype(F)
    pos = np.abs(x) + F(1e-3)
    o = orc
    exact_ops = [(o.RELU, x, np.maximum(x, F(0))), (o.NEG, x, -x), (o.ABS, x, np.abs(x)),
                 (o.SQRT, pos, np.sqrt(pos)), (o.CLAMP, x, np.clip(x, F(-1.5), F(2.5)))]
    for op, inp, want in exact_ops:
        got = o.unary(op, inp, -1.5, 2.5)
        assert np.array_equal(got, want.astype(F)), op
    # transcendental ops: numpy's f32 exp/log/tanh/pow (its own SIMD routines)
    # differ from glibc's by up to a few ulp
    def close(got, want, n):
        d = np.abs(got.view(np.int32).astype(np.int64) - want.astype(F).view(np.int32).astype(np.int64))
        assert d.max() <= n, d.max()
    close(o.unary(o.EXP, x), np.exp(x), 4)
    close(o.unary(o.LOG, pos), np.log(pos), 4)
    close(o.unary(o.TANH, x), np.tanh(x), 4)
    close(o.unary(o.POW, pos, 1.7), np.power(pos, F(1.7)), 4)
    # sigmoid / gelu_quick: the reference expression evaluated step by step in f32
    e = np.exp(-x).astype(F)
    close(o.unary(o.SIGMOID, x), (F(1) / (F(1) + e)).astype(F), 4)
    n = (F(-1.702) * x).astype(F)
    close(o.unary(o.GELU_QUICK, x), (x * (F(1) / (F(1) + np.exp(n).astype(F))).astype(F)).astype(F), 4)
    # gelu against float64 (1 + tanh cancels for x << 0: compare absolutely there)
    x64 = x.astype(np.float64)
    g64 = 0.5 * x64 * (1 + np.tanh(np.sqrt(2 / np.pi) * (x64 + 0.044715 * x64 ** 3)))
    got = o.unary(o.GELU, x).astype(np.float64)
    assert np.all(np.abs(got - g64) <= 1e-6 * np.abs(g64) + 2e-7 * np.abs(x64))


def test_layer_norm_matches_numpy(orc):
    rng = np.random.default_rng(78)
    rows, cols = 37, 1000
    x = (rng.standard_normal((rows, cols)) * 2 + 0.5).astype(F)
    w = rng.uniform(0.5, 1.5, cols).astype(F)
    b = rng.uniform(-0.5, 0.5, cols).astype(F)
    # the reference's loops, vectorised per row with the same sequential f32 sums
    want = np.empty_like(x)
    for r in range(rows):
        s = F(0)
        for v in x[r]:
            s = F(s + v)
        mean = F(s / F(cols))
        ss = F(0)
        for v in x[r]:
            d = F(v - mean)
            ss = F(ss + F(d * d))
        sd = np.sqrt(F(F(ss / F(cols)) + F(1e-5)))
        want[r] = (((x[r] - mean).astype(F) / sd).astype(F) * w).astype(F) + b
    assert np.array_equal(orc.layer_norm(x, w, b, 1e-5), want)
