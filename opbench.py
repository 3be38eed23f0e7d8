"""Op-level benchmark: one hot-path op at a benchmark-config shape.

    python opbench.py --op rms_norm_f32_c1 [--rows R] [--iters N] [--sets S]

Runs the op `iters` times back to back over `sets` rotating input/output
buffer sets (default: enough sets to exceed 2.5x the L2 size, so every launch
reads from HBM), timed with CUDA events on the launching stream, and prints
one JSON line: microseconds per launch and achieved GB/s of algorithmic bytes.
--rows shrinks the row count (for profiler captures of a smaller case).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "mistralrs-oxide_b200"))

from oxide_b200 import ops  # noqa: E402
from oxide_b200 import _lib  # noqa: E402
from oxide_b200._lib import call  # noqa: E402
from oxide_b200.workloads import C1, C2, C3, C4, C5, NKV  # noqa: E402

BF16 = torch.bfloat16


def _stream():
    return torch.cuda.current_stream().cuda_stream


def build(op: str, rows: int | None, dev):
    """Returns (make_set, run, bytes_per_launch, shape) for the op."""
    g = torch.Generator(device=dev)
    g.manual_seed(0)

    def rn(*shape, dtype=torch.float32):
        return torch.randn(shape, generator=g, device=dev, dtype=dtype)

    if op == "rms_norm_f32_c1":
        c = C1()
        R = rows or c.rows
        w = torch.rand(c.cols, generator=g, device=dev) + 0.5
        mk = lambda: (rn(R, c.cols), torch.empty(R, c.cols, device=dev))  # noqa: E731
        run = lambda s: ops.rms_norm(s[0], w, c.eps, out=s[1])  # noqa: E731
        return mk, run, 2 * R * c.cols * 4 + c.cols * 4, [R, c.cols]
    if op in ("add_f32_c2", "mul_f32_c2", "silu_mul_f32_c2"):
        c = C2()
        R = rows or c.rows
        if op == "silu_mul_f32_c2":
            mk = lambda: (rn(R, c.inter), rn(R, c.inter), torch.empty(R, c.inter, device=dev))  # noqa: E731
            run = lambda s: ops.silu_mul(s[0], s[1], out=s[2])  # noqa: E731
            return mk, run, 3 * R * c.inter * 4, [R, c.inter]
        if op == "add_f32_c2":
            mk = lambda: (rn(R, c.cols), rn(R, c.cols), torch.empty(R, c.cols, device=dev))  # noqa: E731
            run = lambda s: call("oxide_add_f32", s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(),  # noqa: E731
                                 R * c.cols, _stream())
            return mk, run, 3 * R * c.cols * 4, [R, c.cols]
        sv = torch.rand(c.cols, generator=g, device=dev) + 0.5
        mk = lambda: (rn(R, c.cols), torch.empty(R, c.cols, device=dev))  # noqa: E731
        run = lambda s: call("oxide_mul_rowbcast_f32", s[0].data_ptr(), sv.data_ptr(),  # noqa: E731
                             s[1].data_ptr(), R, c.cols, _stream())
        return mk, run, 2 * R * c.cols * 4 + c.cols * 4, [R, c.cols]
    if op == "add_mul_f32_c2":
        # (a + b) * s: the C2 residual add and row-broadcast multiply in one pass
        c = C2()
        R = rows or c.rows
        sv = torch.rand(c.cols, generator=g, device=dev) + 0.5
        mk = lambda: (rn(R, c.cols), rn(R, c.cols), torch.empty(R, c.cols, device=dev))  # noqa: E731
        run = lambda s: ops.add_mul_rowbcast(s[0], s[1], sv, out=s[2])  # noqa: E731
        return mk, run, 3 * R * c.cols * 4 + c.cols * 4, [R, c.cols]
    if op == "softmax_f32_c3":
        c = C3()
        _, lens, _ = c.inputs()
        R = rows or c.batch * c.heads
        tl = torch.from_numpy(lens).to(dev)
        mk = lambda: (rn(R, c.keys) * math.sqrt(c.head_dim), torch.empty(R, c.keys, device=dev))  # noqa: E731
        run = lambda s: ops.scale_mask_softmax(s[0], c.scale, lens=tl, rows_per_len=c.heads,  # noqa: E731
                                               out=s[1])
        nb = int(sum(min(int(lens[r // c.heads]), c.keys) for r in range(R))) * 4 + R * c.keys * 4
        return mk, run, nb, [R, c.keys]
    if op in ("decode_attn_bf16_c3", "decode_attn_f32_c3"):
        # one decode step of attention at the C3 batch: q [8, 32, 128], KV caches
        # [8, 8, 32768, 128] with the C3 per-sequence lengths
        c = C3()
        _, lens, _ = c.inputs()
        kvh = NKV
        dt = BF16 if op == "decode_attn_bf16_c3" else torch.float32
        es = 2 if dt == BF16 else 4
        tl = torch.from_numpy(lens).to(dev)
        ws = torch.empty(int(_lib.lib().oxide_decode_attention_workspace_bytes(c.batch, c.heads, c.keys, c.head_dim)),
                         dtype=torch.uint8, device=dev)
        mk = lambda: (rn(c.batch, c.heads, c.head_dim, dtype=dt), rn(c.batch, kvh, c.keys, c.head_dim, dtype=dt),  # noqa: E731
                      rn(c.batch, kvh, c.keys, c.head_dim, dtype=dt),
                      torch.empty(c.batch, c.heads, c.head_dim, dtype=dt, device=dev))
        run = lambda s: ops.decode_attention(s[0], s[1], s[2], tl, workspace=ws, out=s[3])  # noqa: E731
        nb = int(np.sum(np.minimum(lens, c.keys))) * kvh * c.head_dim * es * 2 + 2 * c.batch * c.heads * c.head_dim * es
        return mk, run, nb, [c.batch, c.heads, kvh, c.keys, c.head_dim]
    if op in ("decode_weights_bf16_f32", "decode_weights_f16_f32"):
        # safetensors element decode of one Mistral MLP matrix [14336, 4096] to f32
        n = (rows or 14336) * 4096
        code = _lib.WDT_BF16 if op == "decode_weights_bf16_f32" else _lib.WDT_F16
        out = torch.empty(n, dtype=torch.float32, device=dev)
        mk = lambda: (torch.randint(0, 2**15, (n,), dtype=torch.int16, device=dev, generator=g),)  # noqa: E731
        run = lambda s: call("oxide_decode_weights_f32", s[0].data_ptr(), n, code, out.data_ptr(),  # noqa: E731
                             _stream())
        return mk, run, n * 6, [n]
    if op == "softmax_temperature_f32_c3":
        # softmax_with_temperature alone over the C3 logits [64, 32000]
        c = C3()
        R = rows or c.logit_rows
        out = torch.empty(R, c.vocab, dtype=torch.float32, device=dev)
        mk = lambda: (rn(R, c.vocab) * 3,)  # noqa: E731
        run = lambda s: ops.softmax_with_temperature(s[0], 0.7, out=out)  # noqa: E731
        return mk, run, 2 * R * c.vocab * 4, [R, c.vocab]
    if op in ("sample_topk_f32_c3", "sample_topp_f32_c3"):
        # token sampling over the C3 logits [64, 32000]: the reference's defaults
        # (T = 1, top-k 50), and top-p 0.9 at T = 0.7
        c = C3()
        R = rows or c.logit_rows
        topk = op == "sample_topk_f32_c3"
        u = torch.rand(R, generator=g, device=dev)
        mk = lambda: (rn(R, c.vocab) * 3,)  # noqa: E731
        run = lambda s: ops.sample_next_token(s[0], u, 1.0 if topk else 0.7, 50,  # noqa: E731
                                              1.0 if topk else 0.9)
        return mk, run, R * c.vocab * 4 + R * 8, [R, c.vocab]
    if op == "argmax_f32_c3":
        c = C3()
        R = rows or c.logit_rows
        idx = torch.empty(R, dtype=torch.int32, device=dev)
        mk = lambda: (rn(R, c.vocab),)  # noqa: E731
        run = lambda s: call("oxide_argmax_rows_f32", s[0].data_ptr(), R, c.vocab, idx.data_ptr(),  # noqa: E731
                             _stream())
        return mk, run, R * c.vocab * 4 + R * 4, [R, c.vocab]
    if op == "rope_bf16_c4":
        c = C4()
        T = rows or c.tokens
        cos, sin = ops.rope_table(c.theta, c.head_dim, T)
        cos, sin = cos.to(dev), sin.to(dev)
        mk = lambda: (rn(T, c.q_heads, c.head_dim, dtype=BF16), rn(T, c.k_heads, c.head_dim, dtype=BF16),  # noqa: E731
                      torch.empty(T, c.q_heads, c.head_dim, dtype=BF16, device=dev),
                      torch.empty(T, c.k_heads, c.head_dim, dtype=BF16, device=dev))
        run = lambda s: ops.rope(s[0], s[1], cos, sin, q_out=s[2], k_out=s[3])  # noqa: E731
        nb = 2 * T * (c.q_heads + c.k_heads) * c.head_dim * 2 + 2 * T * (c.head_dim // 2) * 4
        return mk, run, nb, [T, c.q_heads + c.k_heads, c.head_dim]
    if op in ("copy_like_c1", "copy_like_c3", "copy_like_argmax_c3"):
        # the size-matched ceiling of the small configs: this library's own
        # one-read-one-write elementwise kernel (f32 relu) over as many bytes
        # as the op's algorithmic count, and torch's device copy of the same
        moved = {"copy_like_c1": C1().bytes(), "copy_like_c3": C3().bytes_softmax(C3().inputs()[1]),
                 "copy_like_argmax_c3": C3().bytes_argmax()}[op]
        n = moved // 8 // 4 * 4  # f32 elements read and written (whole vectors)
        mk = lambda: (torch.empty(n, device=dev), torch.empty(n, device=dev))  # noqa: E731
        run = lambda s: ops.unary(_lib.RELU, s[0], out=s[1])  # noqa: E731
        return mk, run, 8 * n, [n]
    if op in ("torch_copy_like_c1", "torch_copy_like_c3"):
        moved = {"torch_copy_like_c1": C1().bytes(), "torch_copy_like_c3": C3().bytes_softmax(C3().inputs()[1])}[op]
        n = moved // 8 // 4 * 4
        mk = lambda: (torch.empty(n, device=dev), torch.empty(n, device=dev))  # noqa: E731
        run = lambda s: s[1].copy_(s[0])  # noqa: E731
        return mk, run, 8 * n, [n]
    if op == "reduce_rows_sumsq_bf16_c5":
        # per-row sum of squares (RMSNorm's inner loop as its own op), [131072 x 4096] bf16
        c = C5()
        R = rows or c.rows
        res = torch.empty(R, dtype=torch.float32, device=dev)
        mk = lambda: (rn(R, c.hidden, dtype=BF16),)  # noqa: E731
        run = lambda s: call("oxide_reduce_rows_bf16", _lib.RED_SUMSQ, s[0].data_ptr(), R, c.hidden,  # noqa: E731
                             res.data_ptr(), _stream())
        return mk, run, R * c.hidden * 2 + R * 4, [R, c.hidden]
    if op == "add_bf16_c5":
        # the decoder-layer chain's residual add, [131072 x 4096] bf16
        c = C5()
        R = rows or c.rows
        mk = lambda: (rn(R, c.hidden, dtype=BF16), rn(R, c.hidden, dtype=BF16),  # noqa: E731
                      torch.empty(R, c.hidden, dtype=BF16, device=dev))
        run = lambda s: call("oxide_add_bf16", s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(),  # noqa: E731
                             R * c.hidden, _stream())
        return mk, run, 3 * R * c.hidden * 2, [R, c.hidden]
    if op == "rope_bf16_c5":
        # the decoder-layer chain's RoPE: 64 x 2048 tokens in place, positions t mod 2048
        c = C5()
        T = rows or c.rows
        cos, sin = ops.rope_table(c.theta, c.head_dim, c.seq_len)
        cos, sin = cos.to(dev), sin.to(dev)
        pos = (torch.arange(T, device=dev, dtype=torch.int32) % c.seq_len).contiguous()
        mk = lambda: (rn(T, c.q_heads, c.head_dim, dtype=BF16), rn(T, c.k_heads, c.head_dim, dtype=BF16))  # noqa: E731
        run = lambda s: ops.rope(s[0], s[1], cos, sin, pos, q_out=s[0], k_out=s[1])  # noqa: E731
        nb = 2 * T * (c.q_heads + c.k_heads) * c.head_dim * 2 + T * 4
        return mk, run, nb, [T, c.q_heads + c.k_heads, c.head_dim]
    if op in ("gelu_f32_c2", "tanh_f32_c2", "relu_f32_c2"):
        # remaining activations (src/ops/activation.rs) at the C2 MLP shape
        c = C2()
        R = rows or c.rows
        code = {"gelu_f32_c2": _lib.GELU, "tanh_f32_c2": _lib.TANH, "relu_f32_c2": _lib.RELU}[op]
        mk = lambda: (rn(R, c.inter), torch.empty(R, c.inter, device=dev))  # noqa: E731
        run = lambda s: ops.unary(code, s[0], out=s[1])  # noqa: E731
        return mk, run, 2 * R * c.inter * 4, [R, c.inter]
    if op == "layer_norm_f32_c1":
        # layer_norm (src/ops/norm.rs:53-117) at the C1 shape
        c = C1()
        R = rows or c.rows
        w = torch.rand(c.cols, generator=g, device=dev) + 0.5
        bias = torch.rand(c.cols, generator=g, device=dev) - 0.5
        mk = lambda: (rn(R, c.cols), torch.empty(R, c.cols, device=dev))  # noqa: E731
        run = lambda s: ops.layer_norm(s[0], w, bias, c.eps, out=s[1])  # noqa: E731
        return mk, run, 2 * R * c.cols * 4 + 2 * c.cols * 4, [R, c.cols]
    c = C5()
    if op == "layer_norm_bf16_c5":
        R = rows or c.rows
        w = torch.ones(c.hidden, dtype=BF16, device=dev)
        bias = torch.zeros(c.hidden, dtype=BF16, device=dev)
        mk = lambda: (rn(R, c.hidden, dtype=BF16), torch.empty(R, c.hidden, dtype=BF16, device=dev))  # noqa: E731
        run = lambda s: ops.layer_norm(s[0], w, bias, c.eps, out=s[1])  # noqa: E731
        return mk, run, 2 * R * c.hidden * 2 + 2 * c.hidden * 2, [R, c.hidden]
    if op == "add_layer_norm_bf16_c5":
        # layer_norm(x + r) at the C5 hidden shape
        R = rows or c.rows
        w = torch.ones(c.hidden, dtype=BF16, device=dev)
        bias = torch.zeros(c.hidden, dtype=BF16, device=dev)
        mk = lambda: (rn(R, c.hidden, dtype=BF16), rn(R, c.hidden, dtype=BF16),  # noqa: E731
                      torch.empty(R, c.hidden, dtype=BF16, device=dev))
        run = lambda s: ops.add_layer_norm(s[0], s[1], w, bias, c.eps, out=s[2])  # noqa: E731
        return mk, run, 3 * R * c.hidden * 2 + 2 * c.hidden * 2, [R, c.hidden]
    if op == "repeat_kv_bf16_c5":
        # GQA head repetition of the C5 key cache: [64, 8, 2048, 128] -> [64, 32, 2048, 128]
        R = rows or c.seqs
        rep = c.q_heads // c.k_heads
        mk = lambda: (rn(R, c.k_heads, c.seq_len, c.head_dim, dtype=BF16),  # noqa: E731
                      torch.empty(R, c.q_heads, c.seq_len, c.head_dim, dtype=BF16, device=dev))
        run = lambda s: ops.repeat_kv(s[0], rep, out=s[1])  # noqa: E731
        nb = R * c.k_heads * c.seq_len * c.head_dim * 2 * (1 + rep)
        return mk, run, nb, [R, c.k_heads, c.seq_len, c.head_dim]
    if op == "kv_append_bf16_c5":
        # prefill append of the C5 keys and values into caches of 4096 positions
        R = rows or c.seqs
        M = 2 * c.seq_len
        kc = torch.zeros(R, c.k_heads, M, c.head_dim, dtype=BF16, device=dev)
        vc = torch.zeros_like(kc)
        mk = lambda: (rn(R, c.k_heads, c.seq_len, c.head_dim, dtype=BF16),  # noqa: E731
                      rn(R, c.k_heads, c.seq_len, c.head_dim, dtype=BF16))
        run = lambda s: call("oxide_kv_cache_append_bf16", kc.data_ptr(), vc.data_ptr(), s[0].data_ptr(),  # noqa: E731
                             s[1].data_ptr(), R, c.k_heads, M, c.head_dim, 0, c.seq_len, _stream())
        nb = 4 * R * c.k_heads * c.seq_len * c.head_dim * 2
        return mk, run, nb, [R, c.k_heads, c.seq_len, c.head_dim]
    if op in ("rms_norm_bf16_c5", "add_rms_norm_bf16_c5", "sumsq_bf16_c5"):
        R = rows or c.rows
        w = torch.ones(c.hidden, dtype=BF16, device=dev)
        if op == "rms_norm_bf16_c5":
            mk = lambda: (rn(R, c.hidden, dtype=BF16), torch.empty(R, c.hidden, dtype=BF16, device=dev))  # noqa: E731
            run = lambda s: ops.rms_norm(s[0], w, c.eps, out=s[1])  # noqa: E731
            return mk, run, 2 * R * c.hidden * 2 + c.hidden * 2, [R, c.hidden]
        if op == "sumsq_bf16_c5":
            ws = torch.empty(ops.workspace_bytes(R * c.hidden), dtype=torch.uint8, device=dev)
            res = torch.empty((), dtype=torch.float64, device=dev)
            mk = lambda: (rn(R, c.hidden, dtype=BF16),)  # noqa: E731
            run = lambda s: ops.reduce(s[0], 2, workspace=ws, out=res)  # noqa: E731
            return mk, run, R * c.hidden * 2 + 8, [R, c.hidden]
        mk = lambda: (rn(R, c.hidden, dtype=BF16), rn(R, c.hidden, dtype=BF16),  # noqa: E731
                      torch.empty(R, c.hidden, dtype=BF16, device=dev),
                      torch.empty(R, c.hidden, dtype=BF16, device=dev))
        run = lambda s: ops.add_rms_norm(s[0], s[1], w, c.eps, h=s[2], y=s[3])  # noqa: E731
        return mk, run, 4 * R * c.hidden * 2 + c.hidden * 2, [R, c.hidden]
    if op == "softmax_bf16_c5":
        T = c.seq_len
        R = rows or c.seqs * c.q_heads * T
        R = max(T, R // T * T)
        mk = lambda: (rn(R, T, dtype=BF16), torch.empty(R, T, dtype=BF16, device=dev))  # noqa: E731
        run = lambda s: ops.scale_mask_softmax(s[0], 1.0 / math.sqrt(c.head_dim), causal_q_len=T,  # noqa: E731
                                               out=s[1])
        blocks = R // T
        nb = blocks * (T * (T + 1) // 2) * 2 + R * T * 2
        return mk, run, nb, [R, T]
    if op == "silu_mul_bf16_c5":
        R = rows or c.rows
        mk = lambda: (rn(R, c.inter, dtype=BF16), rn(R, c.inter, dtype=BF16),  # noqa: E731
                      torch.empty(R, c.inter, dtype=BF16, device=dev))
        run = lambda s: ops.silu_mul(s[0], s[1], out=s[2])  # noqa: E731
        return mk, run, 3 * R * c.inter * 2, [R, c.inter]
    if op == "argmax_bf16_c5":
        R = rows or c.rows
        idx = torch.empty(R, dtype=torch.int32, device=dev)
        mk = lambda: (rn(R, c.vocab, dtype=BF16),)  # noqa: E731
        run = lambda s: call("oxide_argmax_rows_bf16", s[0].data_ptr(), R, c.vocab, idx.data_ptr(),  # noqa: E731
                             _stream())
        return mk, run, R * c.vocab * 2 + R * 4, [R, c.vocab]
    raise SystemExit(f"unknown op {op}")


OPS = ["rms_norm_f32_c1", "add_f32_c2", "mul_f32_c2", "add_mul_f32_c2", "silu_mul_f32_c2", "softmax_f32_c3",
       "argmax_f32_c3", "rope_bf16_c4", "rope_bf16_c5", "add_bf16_c5", "reduce_rows_sumsq_bf16_c5", "rms_norm_bf16_c5", "add_rms_norm_bf16_c5",
       "softmax_bf16_c5", "silu_mul_bf16_c5", "argmax_bf16_c5", "sumsq_bf16_c5",
       "gelu_f32_c2", "tanh_f32_c2", "relu_f32_c2", "layer_norm_f32_c1", "layer_norm_bf16_c5", "add_layer_norm_bf16_c5",
       "repeat_kv_bf16_c5", "kv_append_bf16_c5", "decode_attn_bf16_c3", "decode_attn_f32_c3",
       "softmax_temperature_f32_c3", "sample_topk_f32_c3", "sample_topp_f32_c3",
       "decode_weights_bf16_f32", "decode_weights_f16_f32", "copy_like_c1", "copy_like_c3",
       "copy_like_argmax_c3", "torch_copy_like_c1", "torch_copy_like_c3"]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", required=True, choices=OPS + ["all"])
    ap.add_argument("--rows", type=int, default=None)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--sets", type=int, default=None)
    a = ap.parse_args(argv)
    dev = torch.device("cuda")
    l2 = getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 126 << 20)
    for op in (OPS if a.op == "all" else [a.op]):
        mk, run, nbytes, shape = build(op, a.rows, dev)
        nsets = a.sets or max(1, min(16, math.ceil(2.5 * l2 / nbytes)))
        sets = [mk() for _ in range(nsets)]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for s in sets:  # warm-up: first-launch set-up of each kernel, outside capture
                run(s)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        # The launches are captured in one CUDA graph so host launch overhead
        # does not pace short kernels.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(a.iters):
                run(sets[i % nsets])
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 3
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (a.iters * reps)
        del graph
        print(json.dumps({"op": op, "shape": shape, "us_per_launch": round(us, 2),
                          "gbs": round(nbytes / us / 1e3, 1), "bytes": nbytes, "sets": nsets,
                          "iters": a.iters}), flush=True)
        del sets
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
