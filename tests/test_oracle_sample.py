"""The oracle's sample step against a line-by-line Python restatement of the
examples' sample (_example/gpt2/main.go:78-105, _example/qwen/main.go:115-150):
greedy scan at temperature <= 0, otherwise tempered float64 weights, a sort by
weight (ties to the lower id here; Go's sort.Slice leaves them unspecified) and
the draw r = u * sum walked down the sorted list. CPU only."""
import math

import numpy as np
import pytest

from oracle import oracle as O


def go_sample(logits, temp, u):
    v = np.asarray(logits, np.float32)
    if temp <= 0:
        best = 0
        for i in range(len(v)):
            if v[i] > v[best]:
                best = i
        return best
    maxl = v[0]
    for x in v:
        if x > maxl:
            maxl = x
    cands, total = [], 0.0
    for i, x in enumerate(v):
        p = math.exp(float(np.float32(x - maxl)) / temp)  # float32 difference, as Go's v-maxl
        cands.append((p, i))
        total += p
    cands.sort(key=lambda c: (-c[0], c[1]))
    r = u * total
    for p, i in cands:
        r -= p
        if r <= 0:
            return i
    return cands[0][1]


def _logits(n, seed, kind):
    rng = np.random.default_rng(seed)
    v = (rng.standard_normal(n) * 3).astype(np.float32)
    if kind == "ties" and n > 4:
        v[1::3] = v[0]  # many equal logits, equal weights
    if kind == "neginf" and n > 4:
        v[::5] = -np.inf
    return v


@pytest.mark.parametrize("n", [1, 5, 1000, 50257])
@pytest.mark.parametrize("kind", ["plain", "ties", "neginf"])
def test_oracle_sample_matches_go_restatement(n, kind):
    v = _logits(n, n + len(kind), kind)
    for temp in (0.0, -1.0, 0.3, 1.0, 2.5):
        for u in (0.0, 0.25, 0.5, 0.9999999):
            assert O.sample(v, temp, u) == go_sample(v, temp, u), (n, kind, temp, u)


def test_oracle_sample_greedy_is_first_max():
    v = np.array([1, 3, 3, 2], np.float32)
    assert O.sample(v, 0.0, 0.7) == 1


def test_oracle_sample_u_zero_takes_the_top_weight():
    v = np.array([0.5, 4.0, 4.0, -1.0], np.float32)
    assert O.sample(v, 1.0, 0.0) == 1  # the first of the two top weights (lower id)
