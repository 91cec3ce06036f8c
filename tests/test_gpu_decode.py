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


# ---- checkpoint loading (tq_gpt2_create_empty / tq_gpt2_load_tensor) -----------

def _gpt2_checkpoint(cfg, seed, sigma, ln=1.0, scale_in=1.0):
    """The random-init model's weights under the example's tensor names
    (Conv1D [in, out] layout, F32, a "transformer." prefix and an attention-mask
    buffer as Hugging Face files carry them); layer-norm weights `ln`, biases
    0; scale_in multiplies the matrices right after ln_1 and ln_2 (c_attn,
    c_fc)."""
    d, ffn, vocab, ctx = cfg["d"], cfg["ffn"], cfg["vocab"], cfg["ctx"]
    f32 = np.float32
    t = {"wte.weight": O.synth((vocab, d), seed, 1, sigma), "wpe.weight": O.synth((ctx, d), seed, 2, sigma),
         "ln_f.weight": np.ones(d, f32), "ln_f.bias": np.zeros(d, f32)}
    for l in range(cfg["n_layer"]):
        s0, p = 16 + 8 * l, f"h.{l}."
        t[p + "attn.c_attn.weight"] = O.synth((d, 3 * d), seed, s0, sigma) * f32(scale_in)
        t[p + "attn.c_proj.weight"] = O.synth((d, d), seed, s0 + 1, sigma)
        t[p + "mlp.c_fc.weight"] = O.synth((d, ffn), seed, s0 + 2, sigma) * f32(scale_in)
        t[p + "mlp.c_proj.weight"] = O.synth((ffn, d), seed, s0 + 3, sigma)
        for b, n in (("attn.c_attn.bias", 3 * d), ("attn.c_proj.bias", d), ("mlp.c_fc.bias", ffn),
                     ("mlp.c_proj.bias", d), ("ln_1.bias", d), ("ln_2.bias", d)):
            t[p + b] = np.zeros(n, f32)
        t[p + "ln_1.weight"] = np.full(d, ln, f32)
        t[p + "ln_2.weight"] = np.full(d, ln, f32)
        t[p + "attn.bias"] = np.ones((1, 1, 4, 4), f32)  # a mask buffer: not a weight
    return {"transformer." + k: v for k, v in t.items()}


def test_gpt2_checkpoint_of_the_random_weights_gives_the_same_ids(tmp_path):
    from tensai_b200 import safetensors as ST
    from tensai_b200.decode import Gpt2
    p = str(tmp_path / "gpt2.safetensors")
    ST.SaveFile(p, _gpt2_checkpoint(TINY, 8, 0.02))
    prompt = synth_tokens(16, TINY["vocab"], 8)
    with Gpt2(TINY, 8, 0.02) as ref, Gpt2.from_checkpoint(TINY, p) as got:
        assert np.array_equal(got.generate(prompt, 24), ref.generate(prompt, 24))


def test_gpt2_checkpoint_layer_norm_weights_feed_their_matrices(tmp_path):
    """ln_1 / ln_2 weights of 2 against c_attn / c_fc doubled: the same model
    bit for bit (a power of two passes exactly through the fp32 prefill, the
    int8 scales and the activations)."""
    from tensai_b200 import safetensors as ST
    from tensai_b200.decode import Gpt2
    pa, pb = str(tmp_path / "a.safetensors"), str(tmp_path / "b.safetensors")
    ST.SaveFile(pa, _gpt2_checkpoint(TINY, 9, 0.02, ln=2.0))
    ST.SaveFile(pb, _gpt2_checkpoint(TINY, 9, 0.02, scale_in=2.0))
    prompt = synth_tokens(16, TINY["vocab"], 9)
    with Gpt2.from_checkpoint(TINY, pa) as a, Gpt2.from_checkpoint(TINY, pb) as b:
        assert np.array_equal(a.generate(prompt, 24), b.generate(prompt, 24))


def test_gpt2_checkpoint_loading_errors(tmp_path):
    import torch

    from tensai_b200 import safetensors as ST
    from tensai_b200.decode import Gpt2
    d = TINY["d"]
    with Gpt2(TINY, 1, 0.02) as m:
        with pytest.raises(_lib.TensaiError, match="random-init"):
            m.load_tensor("ln_f.weight", torch.ones(d, device="cuda"))
    unknown, short = str(tmp_path / "unknown.safetensors"), str(tmp_path / "short.safetensors")
    ST.SaveFile(unknown, {"h.0.attn.rotary": np.ones(d, np.float32)})
    ST.SaveFile(short, {"ln_f.weight": np.ones(d + 1, np.float32)})
    with pytest.raises(_lib.TensaiError, match="unknown GPT-2 tensor"):
        Gpt2.from_checkpoint(TINY, unknown)
    with pytest.raises(_lib.TensaiError, match="expected"):
        Gpt2.from_checkpoint(TINY, short)
