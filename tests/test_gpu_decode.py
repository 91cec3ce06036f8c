"""GPU greedy decode engines against the CPU oracle, through the C ABI.

Bar: the generated token ids are identical to the oracle's (the GPT-2 -q8
loop of _example/gpt2, restated in oracle/tq_model.c), for small models
and for the GPT-2-small int8 config (128-token prompt, 256 tokens) against
the committed golden ids.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from tensai_b200 import _lib
from tensai_b200.decode import GPT2_SMALL, Gpt2, synth_tokens

pytestmark = pytest.mark.gpu

TINY = dict(n_layer=2, n_head=2, d=128, ffn=512, vocab=1000, ctx=64)


@pytest.fixture(scope="module", autouse=True)
def device():
    import torch
    torch.cuda.init()
    _lib.check(_lib.load().tq_set_device(0))


def _first_divergence(a, b, margins):
    bad = np.nonzero(np.asarray(a) != np.asarray(b))[0]
    if len(bad) == 0:
        return None
    i = int(bad[0])
    return f"token {i}: gpu {a[i]} oracle {b[i]}, oracle top-1 margin {float(margins[i]):.3g}"


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_tiny_gpt2_matches_oracle(seed):
    prompt = synth_tokens(16, TINY["vocab"], seed)
    assert np.array_equal(prompt, O.synth_tokens(16, TINY["vocab"], seed))
    want, margins, _ = O.gpt2_generate(TINY, seed, 0.02, prompt, 40)
    with Gpt2(TINY, seed) as m:
        got = m.generate(prompt, 40)
    assert np.array_equal(got, want), _first_divergence(got, want, margins)


def test_tiny_gpt2_wider_model_and_long_context():
    cfg = dict(n_layer=3, n_head=4, d=256, ffn=1024, vocab=3000, ctx=300)
    prompt = synth_tokens(100, cfg["vocab"], 9)
    want, margins, _ = O.gpt2_generate(cfg, 9, 0.02, prompt, 150)
    with Gpt2(cfg, 9) as m:
        got = m.generate(prompt, 150)
    assert np.array_equal(got, want), _first_divergence(got, want, margins)


def test_gpt2_small_int8_config_matches_golden_tokens():
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "gpt2_decode_golden.npz"))
    prompt = synth_tokens(128, GPT2_SMALL["vocab"], int(z["seed"]))
    assert np.array_equal(prompt, z["prompt"])
    with Gpt2(GPT2_SMALL, int(z["seed"]), float(z["sigma"])) as m:
        got = m.generate(prompt, 256)
        again = m.generate(prompt, 256)  # a fresh sequence on the same resident model
    assert np.array_equal(got, z["tokens"]), _first_divergence(got, z["tokens"], z["margins"])
    assert np.array_equal(again, got)


def test_generate_argument_errors():
    with Gpt2(TINY, 1) as m:
        with pytest.raises(_lib.TensaiError) as e:
            m.generate([5, TINY["vocab"]], 2)
        assert e.value.code == _lib.TQ_ERR_ARG
        with pytest.raises(_lib.TensaiError) as e:
            m.generate(list(range(10)), TINY["ctx"])  # beyond the context
        assert e.value.code == _lib.TQ_ERR_ARG
    with pytest.raises(_lib.TensaiError) as e:
        Gpt2(dict(TINY, n_head=4), 1)  # head size 32: not the example's 64
    assert e.value.code == _lib.TQ_ERR_ARG


def test_freed_model_handle_is_rejected():
    import ctypes
    m = Gpt2(TINY, 1)
    h = m.handle
    m.free()
    L = _lib.load()
    out = np.empty(2, np.int32)
    p = np.array([1, 2], np.int32)
    rc = L.tq_gpt2_generate(h, p.ctypes.data_as(ctypes.c_void_p), 2, 2, out.ctypes.data_as(ctypes.c_void_p), None)
    assert rc == _lib.TQ_ERR_HANDLE
    assert L.tq_gpt2_free(h) == _lib.TQ_OK
