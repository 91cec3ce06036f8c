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


QTINY = dict(n_layer=2, n_head=4, n_kv=2, d=256, ffn=512, vocab=1000, ctx=64, eps=1e-6, theta=1e6)


def _deq4(w):
    """Dequantized QuantizeMatrix4 weights, float64 [rows, cols]."""
    rows, cols = w.shape
    q, s = O.quantize4(w)
    half = cols // 2
    B = q[: rows * half].reshape(rows, half)
    n = np.concatenate([(B & 15).astype(np.int64) - 8, (B >> 4).astype(np.int64) - 8], axis=1).astype(np.float64)
    g = s.reshape(-1, cols).astype(np.float64)
    return n * np.repeat(g, 64, axis=0)[:rows]


def _np_qwen_logits(cfg, seed, sigma, prompt):
    """float64 restatement of the Qwen2 step (model.go:232-307) over the
    prompt with the dequantized int4 weights; the logits after the last token."""
    d, ffn, V, nh, nkv = cfg["d"], cfg["ffn"], cfg["vocab"], cfg["n_head"], cfg["n_kv"]
    hd, grp = d // nh, nh // nkv
    emb = O.synth((V, d), seed, 1, sigma).astype(np.float64)
    lm = _deq4(O.synth((d, V), seed, 2, sigma))
    L = []
    for l in range(cfg["n_layer"]):
        s0 = 32 + 16 * l
        L.append([_deq4(O.synth(sh, seed, s0 + i, sigma)) for i, sh in enumerate(
            [(d, d), (d, nkv * hd), (d, nkv * hd), (d, d), (d, ffn), (d, ffn), (ffn, d)])])

    def rms(v):
        return v / np.sqrt((v * v).mean() + cfg["eps"])

    def rope(hv, pos):
        half = hd // 2
        i = np.arange(half)
        f = cfg["theta"] ** (-2.0 * i / hd)
        c, s = np.cos(pos * f), np.sin(pos * f)
        a, b = hv[:half].copy(), hv[half:].copy()
        return np.concatenate([a * c - b * s, b * c + a * s])

    kc = [[] for _ in L]
    vc = [[] for _ in L]
    for pos, tok in enumerate(prompt):
        x = emb[tok].copy()
        for l, (wq, wk, wv, wo, wg, wu, wd) in enumerate(L):
            a = rms(x)
            q, k, v = a @ wq, a @ wk, a @ wv
            q = np.concatenate([rope(q[h * hd:(h + 1) * hd], pos) for h in range(nh)])
            k = np.concatenate([rope(k[h * hd:(h + 1) * hd], pos) for h in range(nkv)])
            kc[l].append(k)
            vc[l].append(v)
            K, Vv = np.array(kc[l]), np.array(vc[l])
            att = np.zeros(d)
            for h in range(nh):
                g = h // grp
                sc = K[:, g * hd:(g + 1) * hd] @ q[h * hd:(h + 1) * hd] / np.sqrt(hd)
                p = np.exp(sc - sc.max())
                p /= p.sum()
                att[h * hd:(h + 1) * hd] = p @ Vv[:, g * hd:(g + 1) * hd]
            x = x + att @ wo
            a = rms(x)
            gt, up = a @ wg, a @ wu
            x = x + (gt / (1 + np.exp(-gt)) * up) @ wd
    return rms(x) @ lm


@pytest.mark.parametrize("seed", [1, 2])
def test_qwen_oracle_matches_float64_restatement(seed):
    prompt = O.synth_tokens(12, QTINY["vocab"], seed)
    _, _, logits = O.qwen_generate(QTINY, seed, 0.02, prompt, 1, prompt_logits=True)
    ref = _np_qwen_logits(QTINY, seed, 0.02, prompt)
    err = np.linalg.norm(logits - ref) / np.linalg.norm(ref)
    assert err < 1e-5, err
