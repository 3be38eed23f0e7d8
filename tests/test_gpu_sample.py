"""Token sampling on the GPU (softmax_with_temperature + sample_top_p /
sample_top_k, src/tokenizer.rs:166-232, src/pipeline.rs:181-205) against the
CPU oracle, through the C ABI.

Bars.  Probabilities: within 1e-5 of the exact (f64) softmax relative to the
row max, and to the oracle within that plus the oracle's own sequential-sum
drift.  Tokens: when the kept prefix needs at most 2048 candidates (top-k up
to 2048, top-p with a short nucleus) the kernel runs the reference's
sequential f32 loops over the sorted candidates, so its token equals the
reference's walk on the kernel's probabilities bit for bit; against the
oracle's own probabilities, whose exp_sum carries the drift of a sequential
32k-term f32 sum, top-k tokens agree (at most one row per case may differ)
and top-p tokens lie within that drift.  Longer prefixes use f64 running sums
of the bisection: the token equals the exact-arithmetic selection away from a
boundary (1e-6) and lies within the reference's own sequential f32 drift
(n 2^-24 of the total) of the oracle's.  Ties, empty prefixes, NaN rows and
the other edge cases of the reference's code are bit-exact.
"""
import numpy as np
import pytest

from _util import SAMPLE_INVALID, bf16_to_f32, in_drift_band, sample_exact, to_dev, to_np

F = np.float32
INV32 = -1  # OXIDE_SAMPLE_INVALID through an int32 tensor


def _logits(rows, vocab, seed, scale=3.0):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((rows, vocab)) * scale).astype(F)


def _run(x, u, temperature, top_k, top_p):
    import torch

    from oxide_b200 import ops

    xd = to_dev(x)  # uint16 arrays arrive as bf16
    rows, vocab = x.shape
    probs = torch.empty(rows, vocab, dtype=torch.float32, device=xd.device)
    tok = ops.sample_next_token(xd, to_dev(np.asarray(u, F)), temperature, top_k, top_p, probs_out=probs)
    return to_np(tok).astype(np.int64), to_np(probs)


GATHER = 2048  # the kernel walks the reference's loops exactly over at most this many candidates


def _walk_is_exact(p, top_k, top_p):
    """Whether the kernel takes its exact path for this row: the candidates
    (every probability >= the prefix's last value; for top-p the prefix
    reaching top_p (1 + 2 gam)) number at most GATHER."""
    p = np.asarray(p, np.float64)
    n = p.size
    ps = np.sort(p)[::-1]
    if np.float32(top_p) < np.float32(1.0):
        nu = n * 2.0 ** -24
        tq = max(float(np.float32(top_p)), 5e-324) * (1 + 2 * nu / (1 - nu))
        c = np.cumsum(ps)
        if tq >= c[-1]:
            return n <= GATHER
        v = ps[int(np.searchsorted(c, tq, side="left"))]
    else:
        k = min(int(top_k), n)
        v = ps[k - 1]
    return int(np.count_nonzero(p >= v)) <= GATHER


def _check_tokens(orc, tok, probs, ref_tok, ref_probs, u, top_k, top_p):
    """Per row: on the exact path the kernel's token equals the reference's
    loops (the oracle's walk) run on the kernel's own probabilities; otherwise
    it equals the exact-arithmetic selection on them away from a boundary.
    Against the oracle (its own probabilities) the token is within the drift
    band of the reference's sequential sums: its exp_sum (a 32k-term f32 sum,
    ~1e-5 from the exact one) scales every probability, which moves top-p's
    absolute threshold; for top-k the scale cancels in r = u * total and at
    most one row may differ.  Returns the number of rows that took the exact
    path."""
    exact_rows = moved = 0
    for r in range(tok.size):
        ref = INV32 if ref_tok[r] == SAMPLE_INVALID else int(ref_tok[r])
        if _walk_is_exact(probs[r], top_k, top_p):
            exact_rows += 1
            walk = orc.sample_probs(probs[r], top_k, top_p, u[r])
            assert tok[r] == walk, f"row {r}: {tok[r]} vs the reference's walk on these probabilities {walk}"
            moved += int(tok[r] != ref)
            assert in_drift_band(tok[r], ref, ref_probs[r]), f"row {r}: {tok[r]} vs oracle {ref}"
        else:
            want, margin = sample_exact(probs[r], top_k, top_p, u[r])
            if margin > 1e-6:
                assert tok[r] == want, f"row {r}: {tok[r]} vs exact selection {want} (margin {margin:.2e})"
            assert in_drift_band(tok[r], ref, ref_probs[r]), f"row {r}: {tok[r]} vs oracle {ref}"
    if top_p >= 1.0:  # top-k: the exp_sum drift scales every running sum alike and cancels
        assert moved <= 1, f"{moved} rows differ from the oracle on the exact path"
    return exact_rows


def _softmax_exact(x, t):
    s = x.astype(np.float64) / np.float64(F(t))
    e = np.exp(s - s.max(axis=-1, keepdims=True))
    return e / e.sum(axis=-1, keepdims=True)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,vocab", [(4, 1000), (3, 1001), (3, 32000), (2, 32768), (2, 40000),
                                        (3, 40003), (1, 70000), (1, 150000), (1, 262144)])
def test_softmax_with_temperature_matches_oracle(cuda, orc, rows, vocab):
    from oxide_b200 import ops

    x = _logits(rows, vocab, vocab)
    for t in (1.0, 0.7, 2.5):
        got = to_np(ops.softmax_with_temperature(to_dev(x), t))
        ref = orc.softmax_with_temperature(x, t)
        exact = _softmax_exact(x, t)
        pm = exact.max(axis=-1, keepdims=True)
        assert np.all(np.abs(got - exact) <= 1e-5 * pm), "kernel vs exact"
        assert np.all(np.abs(got - ref) <= 1e-5 * pm + np.abs(ref - exact)), "kernel vs oracle + its drift"


@pytest.mark.gpu
def test_softmax_with_temperature_bf16(cuda, orc):
    from oxide_b200 import ops

    x = orc.f32_to_bf16(_logits(3, 32000, 9))
    got = to_np(ops.softmax_with_temperature(to_dev(x), 0.8))
    ref = orc.softmax_with_temperature(x, 0.8)
    exact = _softmax_exact(bf16_to_f32(x), 0.8)
    pm = exact.max(axis=-1, keepdims=True)
    assert np.all(np.abs(got - exact) <= 1e-5 * pm)
    assert np.all(np.abs(got - ref) <= 1e-5 * pm + np.abs(ref - exact))


CASES = [  # (rows, vocab, temperature, top_k, top_p, logit scale)
    (64, 32000, 1.0, 50, 1.0, 3.0),        # the reference's defaults (InferenceParams)
    (64, 32000, 0.7, 1, 1.0, 3.0),         # greedy through top-k
    (64, 32000, 1.0, 32000, 1.0, 1.0),     # top-k over the whole, flat row
    (64, 32000, 0.8, 1000, 1.0, 2.0),
    (64, 32000, 1.0, 50, 0.9, 3.0),        # top-p with a peaked row
    (64, 32000, 1.0, 50, 0.9, 0.5),        # top-p with a flat row: a long nucleus
    (64, 32000, 1.3, 50, 0.5, 2.0),
    (64, 32000, 0.7, 50, 0.9, 3.0),        # the benchmark's top-p case: 500-1900 candidates narrowed in-CTA
    (64, 32000, 1.0, 300, 1.0, 3.0),       # top-k above the narrowing's 256 cap: narrowed to >= 300 keys
    (64, 32000, 1.5, 50, 0.99, 2.0),       # a long nucleus: the narrowing stops short of 256
    (16, 1000, 1.0, 7, 1.0, 1.0),
    (8, 32001, 1.0, 50, 0.9, 2.0),         # rows not 16-byte aligned: element loads and stores
    (8, 70000, 1.0, 50, 0.95, 2.0),        # cluster of 4 CTAs
    (4, 150000, 0.9, 100, 1.0, 3.0),       # cluster of 8
    (4, 262144, 1.0, 50, 0.8, 1.0),
]


@pytest.mark.gpu
@pytest.mark.parametrize("rows,vocab,t,top_k,top_p,scale", CASES)
def test_sample_matches_oracle(cuda, orc, rows, vocab, t, top_k, top_p, scale):
    x = _logits(rows, vocab, 1000 + vocab + top_k, scale)
    u = np.random.default_rng(7 + rows).random(rows).astype(F)
    tok, probs = _run(x, u, t, top_k, top_p)
    ref_tok, ref_probs = orc.sample(x, t, top_k, top_p, u, threads=8)
    exact_rows = _check_tokens(orc, tok, probs, ref_tok, ref_probs, u, top_k, top_p)
    if top_k <= 1000 and top_p >= 1.0:
        assert exact_rows == rows  # short prefixes take the exact walk


@pytest.mark.gpu
def test_sample_bf16_matches_oracle(cuda, orc):
    x = orc.f32_to_bf16(_logits(32, 32000, 77))
    u = np.random.default_rng(3).random(32).astype(F)
    tok, probs = _run(x, u, 0.9, 40, 0.92)
    ref_tok, ref_probs = orc.sample(x, 0.9, 40, 0.92, u)
    _check_tokens(orc, tok, probs, ref_tok, ref_probs, u, 40, 0.92)


@pytest.mark.gpu
def test_sample_ties_follow_index_order(cuda, orc):
    """Equal probabilities keep ascending index order (the stable sort): a
    uniform row picks index ceil(u * k) - 1 of its first k; a prefix cut inside
    a run of ties keeps the lowest indices of the run."""
    rows, vocab = 8, 5000
    x = np.zeros((rows, vocab), F)
    u = np.array([0.0, 0.013, 0.25, 0.5, 0.74, 0.9, 0.999, 0.99999994], F)
    tok, probs = _run(x, u, 1.0, 50, 1.0)
    ref_tok, _ = orc.sample(x, 1.0, 50, 1.0, u)
    assert np.array_equal(tok, ref_tok.astype(np.int64))
    assert np.all(tok < 50)
    # a run of 100 equal maxima cut at k = 30, plus a greedy pick among ties
    x = _logits(rows, vocab, 5, 1.0)
    x[:, 700:800] = 9.0
    for k in (30, 1, 100, 150):
        tok, probs = _run(x, u, 1.0, k, 1.0)
        ref_tok, ref_probs = orc.sample(x, 1.0, k, 1.0, u)
        assert _check_tokens(orc, tok, probs, ref_tok, ref_probs, u, k, 1.0) == rows
        if k <= 100:
            assert np.all((tok >= 700) & (tok < 700 + k))
    assert np.all(_run(x, u, 1.0, 1, 1.0)[0] == 700)


@pytest.mark.gpu
def test_sample_edge_cases(cuda, orc):
    """The reference's corner behaviour: top_k 0 and vocab 1 give 0, top_p <= 0
    or a tiny top_p keeps only the max, u = 0 takes the first element, a NaN
    top_p takes the top-k path, rows whose probabilities hold NaN are marked."""
    x = _logits(6, 3000, 11)
    u = np.array([0.3, 0.0, 0.999, 0.5, 0.7, 0.1], F)
    first = np.argmax(x, axis=1)
    assert np.all(_run(x, u, 1.0, 0, 1.0)[0] == 0)                    # empty prefix
    assert np.array_equal(_run(x, u, 1.0, 50, 0.0)[0], first)          # top_p = 0: the max
    assert np.array_equal(_run(x, u, 1.0, 50, -1.0)[0], first)
    assert np.array_equal(_run(x, u, 1.0, 50, 1e-9)[0], first)
    assert _run(x, u, 1.0, 50, 1.0)[0][1] == first[1]                  # u = 0
    a, _ = _run(x, u, 1.0, 50, float("nan"))                           # NaN top_p: top-k path
    b, _ = _run(x, u, 1.0, 50, 1.0)
    assert np.array_equal(a, b)
    one = np.array([[np.nan], [2.0], [-np.inf], [np.inf], [0.0], [1.0]], F)
    assert np.all(_run(one, u, 1.0, 50, 1.0)[0] == 0)                  # vocab 1
    bad = x.copy()
    bad[0, 17] = np.nan
    bad[1, 5] = np.inf
    bad[2, :] = -np.inf
    tok, probs = _run(bad, u, 1.0, 50, 0.9)
    ref_tok, _ = orc.sample(bad, 1.0, 50, 0.9, u)
    assert list(tok[:3]) == [INV32] * 3 and all(ref_tok[:3] == SAMPLE_INVALID)
    assert np.array_equal(tok[3:], ref_tok[3:].astype(np.int64))
    assert np.all(np.isnan(probs[0])) and np.all(np.isnan(probs[2]))
    tok, _ = _run(x, u, 0.0, 50, 1.0)                                  # x / 0 -> +-inf
    assert np.all(tok == INV32)
    tok, probs = _run(x, u, -1.0, 5, 1.0)                              # negative T reverses the order
    ref_tok, ref_probs = orc.sample(x, -1.0, 5, 1.0, u)
    _check_tokens(orc, tok, probs, ref_tok, ref_probs, u, 5, 1.0)
    assert np.all(np.isin(tok, np.argsort(x, axis=1, kind="stable")[:, :5]))


@pytest.mark.gpu
def test_sample_empty_vocab_and_errors(cuda):
    import torch

    from oxide_b200 import _lib, ops

    x = torch.zeros(3, 0, device=cuda)
    u = torch.full((3,), 0.5, device=cuda)
    assert torch.all(ops.sample_next_token(x, u) == 0)
    big = torch.zeros(1, 262145, device=cuda)
    with pytest.raises(_lib.OxideError, match="262144"):
        ops.sample_next_token(big, u[:1])
    y = torch.zeros(3, 10, device=cuda)
    with pytest.raises(_lib.OxideError, match="uniforms"):
        _lib.call("oxide_sample_f32", y.data_ptr(), 3, 10, 1.0, 50, 1.0, None,
                  torch.empty(3, dtype=torch.int32, device=cuda).data_ptr(), None, 0)
