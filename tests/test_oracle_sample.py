"""Pins of the oracle's token sampling (softmax_with_temperature,
sample_top_p, sample_top_k: src/tokenizer.rs:166-232): hand-derived known
answers, an independent numpy restatement of the same sequential f32 steps,
and the exact-arithmetic selection on the oracle's own probabilities."""
import numpy as np
import pytest

from _util import SAMPLE_INVALID, in_drift_band, sample_exact

F = np.float32


def _np_reference(x, t, top_k, top_p, u):
    """The reference's steps in numpy f32: x / T, max, a sequential sum of
    exp(s - m) (cumsum is sequential), p = e / sum, a stable descending sort,
    sequential running sums."""
    s = (x / F(t)).astype(F)
    m = np.max(s)
    e = np.exp((s - m).astype(F)).astype(F)
    p = (e / np.cumsum(e, dtype=F)[-1]).astype(F)
    if p.size >= 2 and np.isnan(p).any():
        return SAMPLE_INVALID, p
    order = np.argsort(-p, kind="stable")
    ps = p[order]
    c = np.cumsum(ps, dtype=F)
    if F(top_p) < F(1.0):
        hit = np.nonzero(c >= F(top_p))[0]
        keep = int(hit[0]) + 1 if hit.size else p.size
    else:
        keep = min(int(top_k), p.size)
    if keep == 0:
        return 0, p
    total = np.cumsum(ps[:keep], dtype=F)[-1]
    r = F(F(u) * total)
    hit = np.nonzero(c[:keep] >= r)[0]
    return int(order[hit[0]] if hit.size else order[keep - 1]), p


def test_sample_known_answers(orc):
    x = np.array([[1.0, 2.0, 3.0, 3.0]], F)
    p = orc.softmax_with_temperature(x, 1.0)[0]
    assert p[2] == p[3] and p[0] < p[1] < p[2]
    e = np.exp(np.array([-2.0, -1.0, 0.0, 0.0]))
    assert np.allclose(p, e / e.sum(), rtol=1e-6)
    assert orc.sample(x, 1.0, 1, 1.0, [0.5])[0][0] == 2          # ties: lower index first
    assert orc.sample(x, 1.0, 50, 1.0, [0.0])[0][0] == 2          # u = 0: the first element
    assert orc.sample(x, 1.0, 50, 1.0, [0.9999])[0][0] == 0       # the last of the prefix
    assert orc.sample(x, 1.0, 0, 1.0, [0.3])[0][0] == 0           # empty prefix -> 0
    assert orc.sample(x, 1.0, 50, 0.5, [0.99])[0][0] == 3         # nucleus {2, 3}
    assert orc.sample(x, 1.0, 50, 0.5, [0.2])[0][0] == 2
    assert orc.sample(x, 1.0, 2, 1.0, [0.6])[0][0] == 3
    assert orc.sample(np.array([[np.nan, 1.0]], F), 1.0, 5, 1.0, [0.3])[0][0] == SAMPLE_INVALID
    assert orc.sample(np.array([[np.nan]], F), 1.0, 5, 1.0, [0.3])[0][0] == 0  # one element: no compare
    assert orc.sample(np.array([[1.0, -np.inf]], F), 1.0, 5, 1.0, [0.99])[0][0] == 0
    assert orc.sample(np.array([[-np.inf, -np.inf]], F), 1.0, 5, 1.0, [0.5])[0][0] == SAMPLE_INVALID
    # temperature divides: T = 0.5 doubles the logits
    assert np.array_equal(orc.softmax_with_temperature(x, 0.5), orc.softmax_with_temperature(x * 2, 1.0))


@pytest.mark.parametrize("t,top_k,top_p,scale", [(1.0, 50, 1.0, 3.0), (0.7, 1000, 1.0, 1.0),
                                                 (1.0, 50, 0.9, 0.5), (1.2, 5, 0.3, 2.0)])
def test_sample_matches_numpy_restatement(orc, t, top_k, top_p, scale):
    rng = np.random.default_rng(int(t * 10) + top_k)
    x = (rng.standard_normal((24, 4000)) * scale).astype(F)
    u = rng.random(24).astype(F)
    tok, probs = orc.sample(x, t, top_k, top_p, u)
    for r in range(x.shape[0]):
        want, p = _np_reference(x[r], t, top_k, top_p, u[r])
        # numpy's exp and glibc's expf may differ in the last bit
        assert np.allclose(probs[r], p, rtol=4 * 2.0 ** -23, atol=0)
        _, margin = sample_exact(probs[r], top_k, top_p, u[r])
        if margin > 1e-5:
            assert tok[r] == want


def test_oracle_agrees_with_exact_selection(orc):
    """The oracle's sequential f32 walk picks the exact-arithmetic selection
    away from a boundary, and otherwise a token within its own rounding drift."""
    rng = np.random.default_rng(4)
    x = (rng.standard_normal((40, 32000)) * 2).astype(F)
    u = rng.random(40).astype(F)
    for top_k, top_p in ((50, 1.0), (32000, 1.0), (50, 0.9)):
        tok, probs = orc.sample(x, 1.0, top_k, top_p, u, threads=4)
        for r in range(x.shape[0]):
            want, margin = sample_exact(probs[r], top_k, top_p, u[r])
            if margin > 1e-4:
                assert tok[r] == want
            assert in_drift_band(int(tok[r]), want, probs[r])
