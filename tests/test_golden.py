"""Committed golden vectors (tests/golden/oracle_vectors.npz).

CPU: the oracle still reproduces every stored output bit for bit.
GPU: the kernels, fed the stored inputs, match the stored outputs within the
parity tolerances (bit-exact where the contract says so).
"""
import os

import numpy as np
import pytest

from _util import assert_bits_equal, assert_close_rel, assert_ulp, to_dev, to_np, ulp_f32

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "oracle_vectors.npz")


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


def test_oracle_reproduces_golden_vectors(orc, golden):
    import importlib.util

    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(os.path.dirname(GOLDEN), "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    fresh = mg.build()
    assert sorted(fresh) == sorted(golden)
    for k, v in golden.items():
        assert fresh[k].dtype == v.dtype and fresh[k].shape == v.shape, k
        assert fresh[k].tobytes() == v.tobytes(), k


@pytest.mark.gpu
def test_kernels_match_golden_vectors(cuda, golden):
    import torch

    from oxide_b200 import ops

    g = golden
    d = lambda k: to_dev(g[k])  # noqa: E731
    assert_bits_equal(to_np(ops.add(d("add_f32.a"), d("add_f32.b"))), g["add_f32.out"])
    assert_bits_equal(to_np(ops.div(d("add_f32.a"), torch.abs(d("add_f32.b")) + 0.5)),
                      g["div_f32.out"])
    assert_bits_equal(to_np(ops.mul(d("mulb_f32.x"), d("mulb_f32.s"))).reshape(-1), g["mulb_f32.out"])
    assert_bits_equal(to_np(ops.add(d("add_bf16.a"), d("add_bf16.b"))), g["add_bf16.out"])
    assert_ulp(to_np(ops.silu_mul(d("silu_mul_f32.g"), d("silu_mul_f32.u"))), g["silu_mul_f32.out"], 8)
    assert_ulp(to_np(ops.silu_mul(d("silu_mul_bf16.g"), d("silu_mul_bf16.u"))),
               g["silu_mul_bf16.out"], 1)
    assert_close_rel(to_np(ops.rms_norm(d("rms_f32.x"), d("rms_f32.w"), 1e-5)), g["rms_f32.out"], 1e-5)
    assert_ulp(to_np(ops.rms_norm(d("rms_bf16.x"), d("rms_bf16.w"), 1e-5)), g["rms_bf16.out"], 1)
    h, y = ops.add_rms_norm(d("rms_bf16.x"), d("addrms_bf16.r"), d("rms_bf16.w"), 1e-5)
    assert_bits_equal(to_np(h), g["addrms_bf16.h"])
    assert_ulp(to_np(y), g["addrms_bf16.y"], 1)
    assert_close_rel(to_np(ops.softmax(d("smax_f32.x"), 1)), g["smax_f32.out"], 1e-5)
    got = ops.scale_mask_softmax(d("smax_f32.x"), 0.125, lens=d("smax_lens.lens"), rows_per_len=2)
    assert_close_rel(to_np(got), g["smax_lens_f32.out"], 1e-5)
    got = ops.scale_mask_softmax(d("smax_f32.x"), 0.125, mask=d("smax_mask.mask"))
    assert_close_rel(to_np(got), g["smax_mask_f32.out"], 1e-5)
    got = ops.scale_mask_softmax(d("smax_causal_bf16.x"), 0.25, causal_q_len=4)
    assert_ulp(to_np(got), g["smax_causal_bf16.out"], 1)
    cos, sin, pos = d("rope.cos"), d("rope.sin"), d("rope.pos")
    assert_bits_equal(to_np(ops.rope(d("rope_f32.x"), None, cos, sin, pos)), g["rope_f32.out"])
    assert_bits_equal(to_np(ops.rope(d("rope_bf16.x"), None, cos, sin, pos)), g["rope_bf16.out"])
    assert_bits_equal(to_np(ops.rope(d("rope_head_f32.x"), None, cos, sin, pos, layout="head")),
                      g["rope_head_f32.out"])
    assert np.array_equal(to_np(ops.argmax(d("argmax_f32.x"))).astype(np.uint32), g["argmax_f32.out"])
    assert np.array_equal(to_np(ops.argmax(d("argmax_bf16.x"))).astype(np.uint32), g["argmax_bf16.out"])
    ulp_bar = {"relu": 0, "neg": 0, "abs": 0, "clamp": 0, "sqrt": 0, "exp": 4, "log": 4, "tanh": 4,
               "pow": 8, "sigmoid": 8, "gelu_quick": 8, "gelu": 8}
    codes = {"relu": 0, "gelu": 1, "gelu_quick": 2, "sigmoid": 3, "tanh": 4, "exp": 5, "log": 6,
             "sqrt": 7, "pow": 8, "clamp": 9, "neg": 10, "abs": 11}
    for name, bar in ulp_bar.items():
        inp = d("unary.xpos") if name in ("log", "sqrt", "pow") else d("unary.x")
        a, b = {"pow": (1.7, 0.0), "clamp": (-1.5, 2.5)}.get(name, (0.0, 0.0))
        got = to_np(ops.unary(codes[name], inp, a, b))
        ref = g[f"unary_{name}.out"]
        if bar == 0:
            assert_bits_equal(got, ref)
        elif name == "gelu":  # 1 + tanh(v) cancels for x << 0: absolute slack 2^-22 |x|
            xs = g["unary.x"].astype(np.float64)
            ok = (ulp_f32(got, ref) <= bar) | (np.abs(got.astype(np.float64) - ref) <= 2.0 ** -22 * np.abs(xs))
            assert ok.all()
        else:
            assert_ulp(got, ref, bar)
    y = to_np(ops.layer_norm(d("ln.x"), d("ln.w"), d("ln.b"), 1e-5))
    sc = np.abs(g["ln_f32.out"] - g["ln.b"]) + np.abs(g["ln.b"])
    assert np.all(np.abs(y - g["ln_f32.out"]) <= 1e-5 * sc + 1e-6)
    x = d("red.x")
    for op, name in ((0, "sum"), (1, "max"), (2, "sumsq")):
        rows = to_np(ops.reduce_rows(x, op))
        ref = g[f"red_rows_{name}.out"]
        if op == 1:
            assert_bits_equal(rows, ref)
        else:
            tol = 1e-5 * np.sum(np.abs(g["red.x"].astype(np.float64)) ** (1 + (op == 2)), axis=1)
            assert np.all(np.abs(rows.astype(np.float64) - ref) <= tol)
        total = float(ops.reduce(x, op).item())
        want = float(g[f"red_all_{name}.out"])
        assert abs(total - want) <= (0 if op == 1 else 1e-5 * np.sum(np.abs(g["red.x"].astype(np.float64)) ** (1 + (op == 2))))
    # repeat_kv and the KV-cache append: bit-exact copies
    assert_bits_equal(to_np(ops.repeat_kv(d("repeat_kv.x"), 3)), g["repeat_kv.out"])
    cache = ops.KvCache(1, 2, 2, 16, 8, dtype=torch.float32)
    cache.update(0, torch.zeros(2, 2, 2, 16, device=cuda), torch.zeros(2, 2, 2, 16, device=cuda))
    cache.update(0, d("kv_append.k"), d("kv_append.v"))
    assert_bits_equal(to_np(cache.k_cache[0]), g["kv_append.kc"])
    assert_bits_equal(to_np(cache.v_cache[0]), g["kv_append.vc"])
    # one-token attention: f32 within 2e-5 of the row's scale, bf16 within one bf16 ulp
    q, kc, vc, lens = d("dec.q"), d("dec.kc"), d("dec.vc"), d("dec.lens")
    out = to_np(ops.decode_attention(q, kc, vc, lens))
    ref = g["dec_f32.out"]
    assert np.all(np.abs(out - ref) <= 2e-5 * np.abs(ref).max(axis=-1, keepdims=True) + 1e-7)
    out = ops.decode_attention(d("dec_bf16.q"), d("dec_bf16.kc"), d("dec_bf16.vc"), lens)
    assert_ulp(to_np(out), g["dec_bf16.out"], 1)
    # sampling: probabilities within 1e-5 of the row max; tokens equal (short prefixes
    # walk the reference's loops; these rows sit far from any running-sum boundary)
    x, u = d("smp.x"), d("smp.u")
    probs = torch.empty(6, 500, device=cuda)
    for name, tk, tp in (("topk", 50, 1.0), ("topp", 50, 0.9), ("greedy", 1, 1.0)):
        tok = to_np(ops.sample_next_token(x, u, 0.8, tk, tp, probs_out=probs)).astype(np.uint32)
        assert np.array_equal(tok, g[f"smp_{name}.tok"]), name
    pref = g["smp.probs"]
    assert np.all(np.abs(to_np(probs) - pref) <= 1e-5 * pref.max(axis=-1, keepdims=True))
    assert np.array_equal(to_np(ops.sample_next_token(d("smp_bf16.x"), u, 0.8, 50, 1.0)).astype(np.uint32),
                          g["smp_bf16_topk.tok"])
    # weight decode: bit-exact
    from oxide_b200 import _lib

    bits = d("wdec.bits")
    for code, key in ((1, "wdec_f16.out"), (2, "wdec_bf16.out")):
        out = torch.empty(bits.numel(), dtype=torch.float32, device=cuda)
        _lib.call("oxide_decode_weights_f32", bits.data_ptr(), bits.numel(), code, out.data_ptr(), 0)
        assert np.array_equal(to_np(out).view(np.uint32), g[key].view(np.uint32)), key
