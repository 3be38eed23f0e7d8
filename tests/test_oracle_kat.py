"""Known-answer tests that pin the CPU oracle (hand-derived expected values).

The reference ships no golden vectors, so these KATs -- each derived by hand
from the reference formula -- and the independent numpy restatement in
test_oracle_numpy.py are what pin the oracle.
"""
import math

import numpy as np

F = np.float32


def test_rms_norm_constant_row(orc):
    # src/ops/norm.rs:33-47 on a constant row c = 0.5: every partial sum of
    # c*c = 0.25 is exact, so ss = 0.25 * cols exactly.
    cols, eps = 4096, F(1e-5)
    x = np.full((3, cols), 0.5, dtype=F)
    w = np.linspace(0.5, 1.5, cols, dtype=F)
    rms = np.sqrt(F(F(F(0.25 * cols) / F(cols)) + eps))
    expect = (F(0.5) / rms) * w
    y = orc.rms_norm(x, w, eps)
    assert np.array_equal(y, np.broadcast_to(expect, x.shape))


def test_softmax_constant_row_is_uniform(orc):
    # exp(0) = 1 for every key, sum = n exactly, p = 1/n.
    for n in (1, 7, 1000, 4096):
        x = np.full((2, n), 3.25, dtype=F)
        p = orc.softmax(x, 2, n, 1)
        assert np.array_equal(p, np.full_like(x, F(1.0) / F(n)))


def test_silu_known_values(orc):
    x = np.array([0.0, -0.0, -100.0, 100.0], dtype=F)
    y = orc.silu(x)
    assert y[0] == 0.0 and y[1] == 0.0
    assert y[2] == 0.0 and math.copysign(1.0, y[2]) < 0  # -100 * (1/(1+inf)) = -0
    assert y[3] == F(100.0)  # exp(-100) underflows the f32 sum to exactly 1


def test_rope_position_zero_is_identity(orc):
    cos, sin = orc.rope_table(1e6, 128, 4)
    assert np.all(cos[0] == 1.0) and np.all(sin[0] == 0.0)
    x = np.random.default_rng(5).standard_normal((1, 4, 128), dtype=F)  # [tokens=1, heads, d]
    y = orc.rope(x, 1, 4, 128, 0, cos, sin)
    assert np.array_equal(y, x)


def test_rope_table_first_frequency_is_position(orc):
    # freq_0 = theta^0 = 1, so angle = pos and cos/sin are glibc cosf/sinf(pos):
    # within 1 ulp of the correctly rounded value.
    cos, sin = orc.rope_table(1e4, 64, 50)
    for pos in range(50):
        for got, ref in ((cos[pos, 0], math.cos(pos)), (sin[pos, 0], math.sin(pos))):
            assert abs(float(got) - ref) <= float(np.spacing(F(abs(ref)))) + 1e-45


def test_rope_rotation_by_hand(orc):
    # head_dim 2: one pair (x1, x2) rotated by the angle of the table row.
    cos = np.array([[0.5]], dtype=F)
    sin = np.array([[0.25]], dtype=F)
    x = np.array([[[2.0, 4.0]]], dtype=F)
    y = orc.rope(x, 1, 1, 2, 0, cos, sin)
    assert y.ravel().tolist() == [2.0 * 0.5 - 4.0 * 0.25, 2.0 * 0.25 + 4.0 * 0.5]


def test_argmax_ties_signed_zero_and_nan(orc):
    x = np.array([
        [1.0, 3.0, 3.0, 2.0],        # tie -> lowest index
        [-0.0, 0.0, -1.0, -0.0],     # -0 == +0 -> index 0
        [np.nan, -np.inf, np.nan, -5.0],  # NaN below everything
        [np.nan, np.nan, np.nan, np.nan],  # all NaN -> index 0
        [-np.inf, -np.inf, -np.inf, -np.inf],
    ], dtype=F)
    assert orc.argmax_rows(x, 4).tolist() == [1, 0, 3, 0, 0]


def test_masked_softmax_full_length_equals_plain(orc):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((4, 300), dtype=F)
    plain = orc.softmax(x, 4, 300, 1)
    lens = np.array([300, 300], dtype=np.int32)
    masked = orc.scale_mask_softmax(x, 300, 1.0, lens=lens, rows_per_len=2)
    assert np.array_equal(plain, masked)


def test_masked_softmax_lens_and_causal(orc):
    x = np.zeros((4, 5), dtype=F)
    # lens: rows 0-1 keep 2 keys, rows 2-3 keep 0 keys (written as zeros)
    p = orc.scale_mask_softmax(x, 5, 1.0, lens=np.array([2, 0], np.int32), rows_per_len=2)
    assert np.array_equal(p[:2], np.tile(np.array([0.5, 0.5, 0, 0, 0], F), (2, 1)))
    assert np.array_equal(p[2:], np.zeros((2, 5), F))
    # causal with q_len = cols: row i keeps keys 0..i
    q = orc.scale_mask_softmax(np.zeros((5, 5), F), 5, 1.0, causal_q_len=5)
    for i in range(5):
        assert np.array_equal(q[i, : i + 1], np.full(i + 1, F(1.0) / F(i + 1)))
        assert np.all(q[i, i + 1:] == 0)


def test_additive_mask_all_neg_inf_gives_nan_like_reference(orc):
    # src/ops/attention.rs:71-79 with every key at -inf: max = -inf, exp(nan).
    x = np.zeros((1, 4), F)
    p = orc.scale_mask_softmax(x, 4, 1.0, mask=np.full(4, -np.inf, F))
    assert np.all(np.isnan(p))


def test_binary_broadcast_modulo(orc):
    a = np.arange(12, dtype=F)
    b = np.array([10.0, 20.0, 30.0], dtype=F)
    assert orc.binary(orc.ADD, a, b).tolist() == [a[i] + b[i % 3] for i in range(12)]
    assert orc.binary(orc.MUL, a, b).tolist() == [a[i] * b[i % 3] for i in range(12)]
    assert orc.binary(orc.SUB, b, a).tolist() == [b[i % 3] - a[i] for i in range(12)]


def test_global_reductions_exact(orc):
    n = 3_000_001
    x = np.arange(n, dtype=F) % 1024  # small integers: every f64 sum is exact
    total = float(np.sum(x.astype(np.float64)))
    assert orc.reduce(orc.RED_SUM, x) == total
    assert orc.reduce(orc.RED_SUMSQ, x) == float(np.sum(x.astype(np.float64) ** 2))
    assert orc.reduce(orc.RED_MAX, x) == 1023.0
    # thread count does not change the f64 result (fixed chunking)
    assert orc.reduce(orc.RED_SUM, x, threads=4) == total


def test_naive_f32_sum_stalls(orc):
    # Why whole-tensor results are f64: the sequential f32 sum of 2^25 ones
    # stops at 2^24.
    x = np.ones(1 << 25, dtype=F)
    assert orc.reduce_seq_f32(orc.RED_SUM, x) == float(1 << 24)
    assert orc.reduce(orc.RED_SUM, x) == float(1 << 25)


def test_threads_do_not_change_results(orc):
    rng = np.random.default_rng(11)
    x = rng.standard_normal((64, 1000), dtype=F)
    w = rng.uniform(0.5, 1.5, 1000).astype(F)
    assert np.array_equal(orc.rms_norm(x, w, 1e-5, threads=1), orc.rms_norm(x, w, 1e-5, threads=4))
    assert np.array_equal(orc.softmax(x, 64, 1000, 1, threads=1), orc.softmax(x, 64, 1000, 1, threads=3))


def test_bf16_rounding_round_to_nearest_even(orc):
    # bf16 keeps 7 fraction bits: the ulp at 1.0 is 2^-7.
    vals = np.array([1.0, 1.0 + 2**-8, 1.0 + 3 * 2**-8, 1.0 + 2**-9, -2.5, 65504.0], dtype=F)
    bits = orc.f32_to_bf16(vals)
    back = orc.bf16_to_f32(bits)
    # 1 + 2^-8 is the midpoint of 1 and 1 + 2^-7 -> ties to even (1.0);
    # 1 + 3*2^-8 is the midpoint of 1 + 2^-7 and 1 + 2^-6 -> even (1 + 2^-6).
    assert back.tolist() == [1.0, 1.0, 1.0 + 2**-6, 1.0, -2.5, 65536.0]
    # the C library's scalar rounding agrees with the numpy one
    assert [orc.lib().orc_f32_to_bf16(float(v)) for v in vals] == bits.tolist()


def test_unary_known_values(orc):
    o = orc
    x = np.array([-2.0, -0.5, 0.0, 0.5, 2.0, np.nan], dtype=F)
    relu = o.unary(o.RELU, x)
    assert np.array_equal(relu[:5], np.array([0, 0, 0, 0.5, 2.0], F)) and relu[5] == 0.0  # f32::max(NaN, 0) = 0
    assert o.unary(o.SIGMOID, np.array([0.0], F))[0] == F(0.5)  # 1 / (1 + exp(0)) = 1/2 exactly
    assert o.unary(o.GELU, np.array([0.0], F))[0] == 0.0
    assert o.unary(o.GELU_QUICK, np.array([0.0], F))[0] == 0.0
    assert o.unary(o.TANH, np.array([0.0], F))[0] == 0.0
    assert o.unary(o.EXP, np.array([0.0], F))[0] == 1.0
    assert o.unary(o.LOG, np.array([1.0], F))[0] == 0.0
    assert np.isneginf(o.unary(o.LOG, np.array([0.0], F))[0])
    assert np.array_equal(o.unary(o.SQRT, np.array([4.0, 2.25], F)), np.array([2.0, 1.5], F))
    assert np.array_equal(o.unary(o.POW, np.array([2.0, 3.0], F), 3.0), np.array([8.0, 27.0], F))
    c = o.unary(o.CLAMP, x, -1.0, 1.0)
    assert np.array_equal(c[:5], np.array([-1, -0.5, 0, 0.5, 1], F)) and np.isnan(c[5])  # NaN stays
    assert np.array_equal(o.unary(o.NEG, x[:5]), -x[:5])
    assert np.array_equal(o.unary(o.ABS, x[:5]), np.abs(x[:5]))
    # large |x|: sigmoid saturates, gelu(x) -> x for x >> 0 and -> -0 / 0 for x << 0
    big = np.array([30.0, -30.0], F)
    assert np.array_equal(o.unary(o.SIGMOID, big), np.array([1.0, F(np.exp(np.float64(-30.0)))], F)) or \
        o.unary(o.SIGMOID, big)[0] == 1.0
    assert o.unary(o.GELU, np.array([10.0], F))[0] == F(10.0)


def test_layer_norm_constant_row_gives_bias(orc):
    # src/ops/norm.rs:92-113: a constant row has mean = c exactly (c * n / n), every
    # deviation 0, so normalized = 0 and out = 0 * w + b = b.
    cols = 768
    x = np.full((4, cols), 1.75, F)
    w = np.linspace(0.5, 1.5, cols, dtype=F)
    b = np.linspace(-1.0, 1.0, cols, dtype=F)
    assert np.array_equal(orc.layer_norm(x, w, b, 1e-5), np.broadcast_to(b, x.shape))


def test_layer_norm_two_values_by_hand(orc):
    # row [a, -a, a, -a]: mean 0, var a^2, std sqrt(a^2 + eps); out = +-a / std * w + b
    a, eps = F(2.0), F(1e-5)
    x = np.array([[a, -a, a, -a]], F)
    w = np.array([1.0, 2.0, 0.5, 1.0], F)
    b = np.array([0.0, 0.25, -0.5, 1.0], F)
    sd = np.sqrt(F(F(a * a) + eps))
    expect = (np.array([a, -a, a, -a], F) / sd) * w + b
    assert np.array_equal(orc.layer_norm(x, w, b, eps)[0], expect.astype(F))
