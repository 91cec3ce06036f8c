"""CPU checks of the GPT-2 decode oracle (oracle/tq_model.c).

* Its prefill logits match an independent float64 numpy restatement of
  _example/gpt2/model.go:361-401 on a small random-init model.
* Its greedy decode reproduces the committed golden token ids of the
  GPT-2-small int8 config (tests/golden/make_golden_decode.py).
"""
import os

import numpy as np
import pytest

from oracle import oracle as O

TINY = dict(n_layer=2, n_head=2, d=128, ffn=512, vocab=1000, ctx=64)


def _np_prefill_logits(cfg, seed, sigma, prompt):
    """float64 restatement of prefill (model.go:361-401) with fp32 weights."""
    d, ffn, V, nh = cfg["d"], cfg["ffn"], cfg["vocab"], cfg["n_head"]
    hd = d // nh
    wte = O.synth((V, d), seed, 1, sigma).astype(np.float64)
    wpe = O.synth((cfg["ctx"], d), seed, 2, sigma).astype(np.float64)
    T = len(prompt)
    x = wte[prompt] + wpe[:T]

    def ln(v):
        m = v.mean(-1, keepdims=True)
        return (v - m) / np.sqrt(((v - m) ** 2).mean(-1, keepdims=True) + 1e-5)

    for l in range(cfg["n_layer"]):
        s0 = 16 + 8 * l
        wa = O.synth((d, 3 * d), seed, s0, sigma).astype(np.float64)
        wp = O.synth((d, d), seed, s0 + 1, sigma).astype(np.float64)
        wf = O.synth((d, ffn), seed, s0 + 2, sigma).astype(np.float64)
        wf2 = O.synth((ffn, d), seed, s0 + 3, sigma).astype(np.float64)
        qkv = ln(x) @ wa
        q, k, v = qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:]
        att = np.zeros_like(q)
        for h in range(nh):
            sl = slice(h * hd, (h + 1) * hd)
            s = q[:, sl] @ k[:, sl].T / 8
            s = s + np.triu(np.full((T, T), -np.inf), 1)
            p = np.exp(s - s.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            att[:, sl] = p @ v[:, sl]
        x = x + att @ wp
        hmid = ln(x) @ wf
        hmid = 0.5 * hmid * (1 + np.tanh(0.7978845608028654 * (hmid + 0.044715 * hmid ** 3)))
        x = x + hmid @ wf2
    return ln(x[-1:]) @ wte.T


@pytest.mark.parametrize("seed", [3, 11])
def test_oracle_prefill_matches_float64_restatement(seed):
    prompt = O.synth_tokens(20, TINY["vocab"], seed)
    _, _, first = O.gpt2_generate(TINY, seed, 0.02, prompt, 1)
    ref = _np_prefill_logits(TINY, seed, 0.02, prompt)[0]
    err = np.linalg.norm(first - ref) / np.linalg.norm(ref)
    assert err < 1e-5, err


def test_oracle_decode_is_deterministic_and_uses_the_int8_weights():
    prompt = O.synth_tokens(16, TINY["vocab"], 5)
    a = O.gpt2_generate(TINY, 5, 0.02, prompt, 12)
    b = O.gpt2_generate(TINY, 5, 0.02, prompt, 12)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    assert (a[0] >= 0).all() and (a[0] < TINY["vocab"]).all()


def test_oracle_rejects_bad_configs():
    with pytest.raises(ValueError):
        O.gpt2_generate(dict(TINY, n_head=3), 1, 0.02, [1, 2], 2)  # head size not 64
    with pytest.raises(ValueError):
        O.gpt2_generate(TINY, 1, 0.02, list(range(60)), 10)  # beyond the context


def test_golden_gpt2_tokens_reproduce():
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "gpt2_decode_golden.npz"))
    prompt = O.synth_tokens(128, O.GPT2_SMALL["vocab"], int(z["seed"]))
    assert np.array_equal(prompt, z["prompt"])
    toks, margins, _ = O.gpt2_generate(O.GPT2_SMALL, int(z["seed"]), float(z["sigma"]), prompt, 32)
    assert np.array_equal(toks, z["tokens"][:32])
