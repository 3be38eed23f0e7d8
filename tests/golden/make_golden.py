"""Generate tests/golden/oracle_vectors.npz: small seeded inputs for every op
of the hot path and the CPU oracle's outputs for them.

    python tests/golden/make_golden.py

The reference crate cannot be built or run here (Rust, no toolchain, and it
does not compile), so these vectors come from the oracle restatement of its
src/ops loop bodies; the oracle itself is pinned by hand-derived known answers
(test_oracle_kat.py) and an independent numpy restatement
(test_oracle_numpy.py).  The fixtures freeze those outputs so that a change
to the oracle or to a kernel is caught against committed numbers, and so the
GPU tests have vectors that need no oracle run.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as orc  # noqa: E402

F = np.float32


def build() -> dict:
    rng = np.random.default_rng(20251201)
    g = {}

    def bf(a):
        return orc.f32_to_bf16(np.asarray(a, F))

    # binary ops with broadcast (src/ops/matmul.rs:136-158)
    a = rng.standard_normal(1000, dtype=F)
    b = rng.standard_normal(1000, dtype=F)
    s = rng.uniform(0.5, 1.5, 128).astype(F)
    x = rng.standard_normal((7, 128), dtype=F)
    g["add_f32.a"], g["add_f32.b"], g["add_f32.out"] = a, b, orc.binary(0, a, b)
    g["div_f32.out"] = orc.binary(3, a, np.abs(b) + F(0.5))
    g["mulb_f32.x"], g["mulb_f32.s"], g["mulb_f32.out"] = x, s, orc.binary(2, x, s, x.size)
    ab, bb = bf(a), bf(b)
    g["add_bf16.a"], g["add_bf16.b"], g["add_bf16.out"] = ab, bb, orc.binary(0, ab, bb)
    # silu * up (src/ops/activation.rs:21-37, src/layers/attention.rs:144-145)
    gt, up = rng.standard_normal(999, dtype=F) * F(4), rng.standard_normal(999, dtype=F)
    g["silu_mul_f32.g"], g["silu_mul_f32.u"], g["silu_mul_f32.out"] = gt, up, orc.silu_mul(gt, up)
    g["silu_mul_bf16.g"], g["silu_mul_bf16.u"] = bf(gt), bf(up)
    g["silu_mul_bf16.out"] = orc.silu_mul(bf(gt), bf(up))
    # RMSNorm and add + RMSNorm (src/ops/norm.rs:33-47)
    x = rng.standard_normal((5, 256), dtype=F)
    r = rng.standard_normal((5, 256), dtype=F)
    w = rng.uniform(0.5, 1.5, 256).astype(F)
    g["rms_f32.x"], g["rms_f32.w"], g["rms_f32.out"] = x, w, orc.rms_norm(x, w, 1e-5)
    g["rms_bf16.x"], g["rms_bf16.w"] = bf(x), bf(w)
    g["rms_bf16.out"] = orc.rms_norm(bf(x), bf(w), 1e-5)
    h, y = orc.add_rms_norm(bf(x), bf(r), bf(w), 1e-5)
    g["addrms_bf16.r"], g["addrms_bf16.h"], g["addrms_bf16.y"] = bf(r), h, y
    # softmax and scale + mask + softmax (src/ops/activation.rs:95-120,
    # src/ops/attention.rs:41,60,63-79)
    x = rng.standard_normal((6, 300), dtype=F) * F(3)
    g["smax_f32.x"], g["smax_f32.out"] = x, orc.softmax(x, 6, 300, 1)
    lens = np.array([300, 17, 0], np.int32)
    g["smax_lens.lens"] = lens
    g["smax_lens_f32.out"] = orc.scale_mask_softmax(x, 300, 0.125, lens=lens, rows_per_len=2)
    mask = np.where(rng.random(300) < 0.25, -np.inf, 0.5).astype(F)
    g["smax_mask.mask"] = mask
    g["smax_mask_f32.out"] = orc.scale_mask_softmax(x, 300, 0.125, mask=mask)
    xc = rng.standard_normal((8, 64), dtype=F) * F(2)
    g["smax_causal_bf16.x"] = bf(xc)
    g["smax_causal_bf16.out"] = orc.scale_mask_softmax(bf(xc), 64, 0.25, causal_q_len=4)
    # RoPE (src/ops/attention.rs:139-155; table src/models/mistral.rs:91-115)
    cos, sin = orc.rope_table(1e6, 64, 16)
    q = rng.standard_normal((10, 3, 64), dtype=F)
    pos = rng.integers(0, 16, 10).astype(np.int32)
    g["rope.cos"], g["rope.sin"], g["rope.pos"] = cos, sin, pos
    g["rope_f32.x"], g["rope_f32.out"] = q, orc.rope(q, 10, 3, 64, 0, cos, sin, pos)
    g["rope_bf16.x"] = bf(q)
    g["rope_bf16.out"] = orc.rope(bf(q), 10, 3, 64, 0, cos, sin, pos)
    qh = np.ascontiguousarray(np.transpose(q, (1, 0, 2)))
    g["rope_head_f32.x"], g["rope_head_f32.out"] = qh, orc.rope(qh, 10, 3, 64, 1, cos, sin, pos)
    # argmax (src/tokenizer.rs:213-232 with k = 1)
    x = rng.standard_normal((20, 500), dtype=F)
    x[1, [3, 77]] = 9.0
    x[2] = np.nan
    x[2, 400] = -np.inf
    x[3] = -0.0
    x[3, 10] = 0.0
    g["argmax_f32.x"], g["argmax_f32.out"] = x, orc.argmax_rows(x, 500)
    g["argmax_bf16.x"] = bf(x)
    g["argmax_bf16.out"] = orc.argmax_rows(bf(x), 500)
    # unary ops (src/ops/activation.rs, src/ops/math.rs) and layer_norm (src/ops/norm.rs:53-117)
    x = rng.standard_normal(777, dtype=F) * F(3)
    g["unary.x"] = x
    g["unary.xpos"] = xpos = np.abs(x) + F(0.01)
    for name, op, inp, a, b in (("relu", orc.RELU, x, 0, 0), ("gelu", orc.GELU, x, 0, 0),
                                ("gelu_quick", orc.GELU_QUICK, x, 0, 0), ("sigmoid", orc.SIGMOID, x, 0, 0),
                                ("tanh", orc.TANH, x, 0, 0), ("exp", orc.EXP, x, 0, 0),
                                ("log", orc.LOG, xpos, 0, 0), ("sqrt", orc.SQRT, xpos, 0, 0),
                                ("pow", orc.POW, xpos, 1.7, 0), ("clamp", orc.CLAMP, x, -1.5, 2.5),
                                ("neg", orc.NEG, x, 0, 0), ("abs", orc.ABS, x, 0, 0)):
        g[f"unary_{name}.out"] = orc.unary(op, inp, a, b)
    x = rng.standard_normal((6, 320), dtype=F) * F(2) + F(0.5)
    w = rng.uniform(0.5, 1.5, 320).astype(F)
    b = rng.uniform(-0.5, 0.5, 320).astype(F)
    g["ln.x"], g["ln.w"], g["ln.b"] = x, w, b
    g["ln_f32.out"] = orc.layer_norm(x, w, b, 1e-5)
    g["ln_bf16.out"] = orc.layer_norm(bf(x), bf(w), bf(b), 1e-5)
    # repeat_kv (src/ops/attention.rs:161-201) and the KV-cache append (src/cache/kv_cache.rs:55-85)
    x = rng.standard_normal((2, 2, 5, 16), dtype=F)
    g["repeat_kv.x"], g["repeat_kv.out"] = x, orc.repeat_kv(x, 3)
    kc = np.zeros((2, 2, 8, 16), F)
    vc = np.zeros((2, 2, 8, 16), F)
    k = rng.standard_normal((2, 2, 3, 16), dtype=F)
    v = rng.standard_normal((2, 2, 3, 16), dtype=F)
    assert orc.kv_append(kc, vc, k, v, 2)
    g["kv_append.k"], g["kv_append.v"], g["kv_append.kc"], g["kv_append.vc"] = k, v, kc, vc
    # one-token attention over a cache (src/ops/attention.rs:41-87, GQA head map of repeat_kv)
    q = rng.standard_normal((2, 8, 128), dtype=F)
    kc = rng.standard_normal((2, 2, 40, 128), dtype=F)
    vc = rng.standard_normal((2, 2, 40, 128), dtype=F)
    lens = np.array([40, 13], np.int32)
    g["dec.q"], g["dec.kc"], g["dec.vc"], g["dec.lens"] = q, kc, vc, lens
    g["dec_f32.out"] = orc.decode_attention(q, kc, vc, lens)
    g["dec_bf16.q"], g["dec_bf16.kc"], g["dec_bf16.vc"] = bf(q), bf(kc), bf(vc)
    g["dec_bf16.out"] = orc.decode_attention(bf(q), bf(kc), bf(vc), lens)
    # token sampling (src/tokenizer.rs:166-232, src/pipeline.rs:181-205)
    x = rng.standard_normal((6, 500), dtype=F) * F(3)
    u = rng.random(6).astype(F)
    g["smp.x"], g["smp.u"] = x, u
    for name, tk, tp in (("topk", 50, 1.0), ("topp", 50, 0.9), ("greedy", 1, 1.0)):
        tok, probs = orc.sample(x, 0.8, tk, tp, u)
        g[f"smp_{name}.tok"] = tok
    g["smp.probs"] = orc.softmax_with_temperature(x, 0.8)
    g["smp_bf16.x"] = bf(x)
    g["smp_bf16_topk.tok"] = orc.sample(bf(x), 0.8, 50, 1.0, u)[0]
    # weight decode (src/loading/safetensors.rs:48-82; BF16 read as bf16)
    h = rng.integers(0, 65536, 300).astype(np.uint16)
    h[:8] = [0x0000, 0x8000, 0x0001, 0x03FF, 0x7C00, 0xFC00, 0x7E01, 0x7C01]
    g["wdec.bits"] = h
    g["wdec_f16.out"] = orc.decode_weights(h.view(np.uint8), orc.WDT_F16)
    g["wdec_bf16.out"] = orc.decode_weights(h.view(np.uint8), orc.WDT_BF16)
    # reductions
    x = rng.standard_normal((9, 333), dtype=F)
    g["red.x"] = x
    for op, name in ((0, "sum"), (1, "max"), (2, "sumsq")):
        g[f"red_rows_{name}.out"] = orc.reduce_rows(op, x, 333)
        g[f"red_all_{name}.out"] = np.array(orc.reduce(op, x), np.float64)
    return g


def main():
    g = build()
    path = os.path.join(HERE, "oracle_vectors.npz")
    np.savez_compressed(path, **g)
    print(f"wrote {path}: {len(g)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
