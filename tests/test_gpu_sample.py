"""GPU sample step (tq_sample, through the C ABI) against the oracle's
restatement of the examples' sample (_example/gpt2/main.go:78-105): the same
token for greedy and tempered draws over vocabulary sizes from 1 to the Qwen2
vocabulary, with tied and -inf logits, and the argument errors."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tensai_b200 import _lib
from tensai_b200.decode import sample

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def device():
    import torch
    torch.cuda.init()
    _lib.check(_lib.load().tq_set_device(0))


def _logits(n, seed, kind):
    rng = np.random.default_rng(seed)
    v = (rng.standard_normal(n) * 3).astype(np.float32)
    if kind == "ties" and n > 4:
        v[1::3] = v[0]
    if kind == "neginf" and n > 4:
        v[::5] = -np.inf
    return v


@pytest.mark.parametrize("n", [1, 7, 1000, 50257, 152064])
@pytest.mark.parametrize("kind", ["plain", "ties", "neginf"])
def test_sample_matches_oracle(n, kind):
    v = _logits(n, 7 * n + len(kind), kind)
    rng = np.random.default_rng(n)
    draws = [0.0, 0.5, 0.999999] + list(rng.random(5))
    for temp in (0.0, -0.5, 0.2, 0.8, 1.0, 3.0):
        for u in draws:
            assert sample(v, temp, u) == O.sample(v, temp, u), (n, kind, temp, u)


def test_sample_greedy_keeps_a_leading_nan():
    v = np.array([np.nan, 1.0, 5.0], np.float32)
    assert sample(v, 0.0, 0.0) == O.sample(v, 0.0, 0.0) == 0
    w = np.array([1.0, np.nan, 5.0, 5.0], np.float32)
    assert sample(w, 0.0, 0.0) == O.sample(w, 0.0, 0.0) == 2


def test_sample_rejects_bad_arguments():
    L = _lib.load()
    v = np.zeros(4, np.float32)
    tok = ctypes.c_int()
    p = v.ctypes.data_as(ctypes.c_void_p)
    assert L.tq_sample(p, 0, 1.0, 0.5, ctypes.byref(tok)) == _lib.TQ_ERR_ARG
    assert L.tq_sample(p, 4, float("nan"), 0.5, ctypes.byref(tok)) == _lib.TQ_ERR_ARG
    assert L.tq_sample(p, 4, 1.0, 1.5, ctypes.byref(tok)) == _lib.TQ_ERR_ARG
    assert L.tq_sample(None, 4, 1.0, 0.5, ctypes.byref(tok)) == _lib.TQ_ERR_ARG
    assert L.tq_sample(p, 4, 0.0, 7.0, ctypes.byref(tok)) == _lib.TQ_OK  # u unused at temperature 0
