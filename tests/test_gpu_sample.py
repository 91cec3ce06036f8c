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


# ---- sampling inside the decode engines ----------------------------------------

GPT2_TINY = dict(n_layer=2, n_head=2, d=128, ffn=512, vocab=1000, ctx=64)
QWEN_TINY = dict(n_layer=2, n_head=4, n_kv=2, d=256, ffn=512, vocab=1000, ctx=64, eps=1e-6, theta=1e6)


def test_gpt2_sampling_with_zero_draws_is_greedy():
    from tensai_b200.decode import Gpt2, synth_tokens
    prompt = synth_tokens(12, GPT2_TINY["vocab"], 5)
    with Gpt2(GPT2_TINY, 5, 0.02) as m:
        greedy = m.generate(prompt, 20)
        m.set_sampling(0.7, np.zeros(20))
        assert np.array_equal(m.generate(prompt, 20), greedy)  # u = 0 takes the heaviest candidate
        m.set_sampling(0.0)
        assert np.array_equal(m.generate(prompt, 20), greedy)


def test_gpt2_first_sampled_token_matches_oracle():
    """The first generated token comes from the fp32 prefill's logits, which
    the oracle also returns: the engine's draw must pick the oracle's token."""
    from tensai_b200.decode import Gpt2, synth_tokens
    prompt = synth_tokens(12, GPT2_TINY["vocab"], 6)
    _, _, first = O.gpt2_generate(GPT2_TINY, 6, 0.02, prompt, 1)
    rng = np.random.default_rng(6)
    with Gpt2(GPT2_TINY, 6, 0.02) as m:
        for temp in (0.05, 0.5, 1.0, 2.0):
            for u in list(rng.random(4)) + [0.0, 0.999]:
                m.set_sampling(temp, [u])
                assert int(m.generate(prompt, 1)[0]) == O.sample(first, temp, u), (temp, u)


def test_engine_sampling_is_reproducible_and_checks_draws():
    from tensai_b200.decode import Gpt2, Qwen, synth_tokens
    prompt = synth_tokens(10, 1000, 7)
    draws = np.random.default_rng(7).random(16)
    with Gpt2(GPT2_TINY, 7, 0.02) as m:
        m.set_sampling(1.0, draws)
        a = m.generate(prompt, 16)
        assert np.array_equal(a, m.generate(prompt, 16))
        with pytest.raises(_lib.TensaiError):
            m.generate(prompt, 17)  # more tokens than draws
        with pytest.raises(_lib.TensaiError):
            m.set_sampling(1.0, [0.5, 1.5])
        with pytest.raises(_lib.TensaiError):
            m.set_sampling(float("nan"), draws)
    with Qwen(QWEN_TINY, 7, 0.02) as q:
        greedy = q.generate(prompt, 16)
        q.set_sampling(0.9, np.zeros(16))
        assert np.array_equal(q.generate(prompt, 16), greedy)
        q.set_sampling(1.0, draws)
        b = q.generate(prompt, 16)
        assert np.array_equal(b, q.generate(prompt, 16))
        assert ((b >= 0) & (b < 1000)).all()
