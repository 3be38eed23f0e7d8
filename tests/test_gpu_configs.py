"""Parity at the benchmark configurations themselves: the exact shapes, value
distributions and seeds the benchmark times (oxide_b200.workloads C1-C5),
each run through the C ABI and compared with the oracle's restatement of the
reference's loops (src/ops/norm.rs:33-47, src/ops/matmul.rs:136-158,
src/ops/activation.rs:30-33,97-120, src/ops/attention.rs:41,63-79,139-155),
with the tolerances of tests/test_gpu_parity.py.  The C5 chain is checked on
its first 2048-token sequence, every op in order, each op fed by the previous
op's device output exactly as the benchmark chains them."""
import math

import numpy as np
import pytest
import torch

from _util import (BF16_ULP, F32_REL, assert_bits_equal, assert_parity_rel, assert_silu_f32_parity, assert_ulp,
                   rms_norm_exact, smax_close, to_dev, to_np)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def threads(orc):
    return orc.max_threads()


def test_c1_rms_norm_f32(cuda, orc, threads):
    """C1: x [2048, 4096] ~ N(0,1), w ~ U(0.5, 1.5), eps 1e-5, seed 0."""
    from oxide_b200 import ops
    from oxide_b200.workloads import C1

    c = C1()
    x, w = c.inputs()
    got = to_np(ops.rms_norm(to_dev(x), to_dev(w), c.eps))
    ref = orc.rms_norm(x, w, c.eps, threads=threads)
    assert_parity_rel(got, ref, rms_norm_exact(x, w, c.eps), F32_REL)


def test_c2_add_mul_silu_mul_f32(cuda, orc, threads):
    """C2: h = a + b, y = h * s (row broadcast), o = silu(gate) * up, seed 1;
    the three kernels and shapes of the benchmark's step."""
    from oxide_b200._lib import call
    from oxide_b200.workloads import C2

    c = C2()
    a, b, s, gate, up = c.inputs()
    ta, tb, ts = to_dev(a), to_dev(b), to_dev(s)
    th, ty = torch.empty_like(ta), torch.empty_like(ta)
    call("oxide_add_f32", ta.data_ptr(), tb.data_ptr(), th.data_ptr(), a.size, None)
    call("oxide_mul_rowbcast_f32", th.data_ptr(), ts.data_ptr(), ty.data_ptr(), c.rows, c.cols, None)
    torch.cuda.synchronize()
    rh = orc.binary(orc.ADD, a, b, threads=threads)
    assert_bits_equal(to_np(th), rh)
    assert_bits_equal(to_np(ty), orc.binary(orc.MUL, rh, s, rh.size, threads=threads))
    del ta, tb, th, ty
    tg, tu = to_dev(gate), to_dev(up)
    to = torch.empty_like(tg)
    call("oxide_silu_mul_f32", tg.data_ptr(), tu.data_ptr(), to.data_ptr(), gate.size, None)
    torch.cuda.synchronize()
    got, ref = to_np(to), orc.silu_mul(gate, up, threads=threads)
    assert_silu_f32_parity(got, ref, gate, orc, threads)


def test_c3_masked_decode_softmax_and_argmax_f32(cuda, orc, threads):
    """C3: scores [8, 32, 1, 32768] = z * sqrt(128) with the seed-2 lengths
    len_b ~ U[1024, 32768] masking the last keys, scale 1/sqrt(128); logits
    [64, 32000] ~ N(0,1), indices bit-exact."""
    from oxide_b200 import ops
    from oxide_b200.workloads import C3

    c = C3()
    scores, lens, logits = c.inputs()
    got = ops.scale_mask_softmax(to_dev(scores), c.scale, lens=to_dev(lens), rows_per_len=c.heads)
    ref = orc.scale_mask_softmax(scores, c.keys, c.scale, lens=lens, rows_per_len=c.heads, threads=threads)
    smax_close(to_np(got), ref, scores, c.keys, "f32", c.scale, lens=lens, rows_per_len=c.heads)
    g = to_np(got).reshape(c.batch, c.heads, c.keys)
    for bi, n in enumerate(lens):
        assert np.all(g[bi, :, n:] == 0), "masked keys must be exactly 0"
    idx = ops.argmax(to_dev(logits))
    assert np.array_equal(to_np(idx).astype(np.uint32), orc.argmax_rows(logits, c.vocab, threads=threads))


def test_c4_rope_bf16(cuda, orc, threads):
    """C4: q [4096, 32, 128], k [4096, 8, 128] bf16 ~ N(0,1), positions
    0..4095, theta 1e6, f32 tables, seed 3: bit-exact."""
    from oxide_b200 import ops
    from oxide_b200.workloads import C4

    c = C4()
    q, k = c.inputs()
    cos, sin = ops.rope_table(c.theta, c.head_dim, c.tokens)
    rcos, rsin = orc.rope_table(c.theta, c.head_dim, c.tokens)
    assert_bits_equal(cos.numpy(), rcos)
    assert_bits_equal(sin.numpy(), rsin)
    tq, tk = ops.rope(to_dev(q), to_dev(k), cos.cuda(), sin.cuda())
    assert_bits_equal(to_np(tq), orc.rope(q, c.tokens, c.q_heads, c.head_dim, 0, rcos, rsin, threads=threads))
    assert_bits_equal(to_np(tk), orc.rope(k, c.tokens, c.k_heads, c.head_dim, 0, rcos, rsin, threads=threads))


def test_c5_chain_first_sequence_bf16(cuda, orc, threads):
    """C5 (seed 4), sequence 0 of the 64 x 2048-token batch -- the same rows
    the benchmark's chain reads for it: add+RMSNorm -> RoPE (positions
    0..2047) -> scale + causal mask + softmax over [32 x 2048, 2048] ->
    SiLU*up -> residual add -> final RMSNorm -> logits argmax -> global sum of
    squares, each op on the device output of the one before (the oracle
    chains its own outputs, which the earlier ops match bit for bit)."""
    from oxide_b200 import ops
    from oxide_b200.workloads import C5

    c = C5()
    T = c.seq_len
    d = c.device_inputs(0, 1, cuda)
    h_np = {k: to_np(v) for k, v in d.items()}
    cos, sin = ops.rope_table(c.theta, c.head_dim, T)
    pos = torch.arange(T, dtype=torch.int32, device=cuda)
    scale = 1.0 / math.sqrt(c.head_dim)

    h, y = ops.add_rms_norm(d["x"], d["r"], d["w"], c.eps)
    rh, ry = orc.add_rms_norm(h_np["x"], h_np["r"], h_np["w"], c.eps, threads=threads)
    assert_bits_equal(to_np(h), rh)
    assert_ulp(to_np(y), ry, BF16_ULP)

    tq, tk = ops.rope(d["q"], d["k"], cos.cuda(), sin.cuda(), pos)
    rcos, rsin = cos.numpy(), sin.numpy()
    assert_bits_equal(to_np(tq), orc.rope(h_np["q"], T, c.q_heads, c.head_dim, 0, rcos, rsin,
                                          np.arange(T), threads=threads))
    assert_bits_equal(to_np(tk), orc.rope(h_np["k"], T, c.k_heads, c.head_dim, 0, rcos, rsin,
                                          np.arange(T), threads=threads))

    p = ops.scale_mask_softmax(d["scores"], scale, causal_q_len=T)
    rp = orc.scale_mask_softmax(h_np["scores"], T, scale, causal_q_len=T, threads=threads)
    smax_close(to_np(p), rp, h_np["scores"], T, "bf16", scale, causal_q=T)
    del p, rp

    act = ops.silu_mul(d["gate"], d["up"])
    assert_ulp(to_np(act), orc.silu_mul(h_np["gate"], h_np["up"], threads=threads), BF16_ULP)

    h2 = ops.add(h, d["mlp"])
    rh2 = orc.binary(orc.ADD, rh, h_np["mlp"], threads=threads).reshape(rh.shape)
    assert_bits_equal(to_np(h2), rh2)

    yf = ops.rms_norm(h2, d["w"], c.eps)
    ryf = orc.rms_norm(rh2, h_np["w"], c.eps, threads=threads)
    assert_ulp(to_np(yf), ryf, BF16_ULP)

    idx = ops.argmax(d["logits"])
    assert np.array_equal(to_np(idx).astype(np.uint32), orc.argmax_rows(h_np["logits"], c.vocab, threads=threads))

    ss = float(ops.reduce(yf, 2).item())
    own = orc.reduce(2, to_np(yf), threads=threads)  # f64 sum of squares of the same bf16 values
    chained = orc.reduce(2, ryf, threads=threads)
    assert abs(ss - own) <= F32_REL * abs(own)
    assert abs(ss - chained) <= F32_REL * abs(chained)
