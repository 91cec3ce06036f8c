"""Host mirror of the whole-model greedy decode engines (C ABI tq_gpt2_*).

Gpt2 stands for the GPT-2 example's model (_example/gpt2/model.go) with
random-init weights: Gpt2(cfg, seed, sigma).generate(prompt, n) runs the
fp32 prefill and the int8 decode steps on the GPU and returns the greedy
token ids (main.go:163-170 at temperature 0).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

GPT2_SMALL = dict(n_layer=12, n_head=12, d=768, ffn=3072, vocab=50257, ctx=1024)


class Gpt2Config(ctypes.Structure):
    _fields_ = [("n_layer", ctypes.c_int), ("n_head", ctypes.c_int), ("d", ctypes.c_int), ("ffn", ctypes.c_int),
                ("vocab", ctypes.c_int), ("ctx", ctypes.c_int)]


def synth_tokens(n: int, vocab: int, seed: int) -> np.ndarray:
    """Seeded uniform token ids in [0, vocab): a stand-in for a tokenized prompt."""
    out = np.empty(n, np.int32)
    _lib.check(_lib.load().tq_synth_tokens(out.ctypes.data_as(ctypes.c_void_p), n, vocab, seed))
    return out


class Gpt2:
    """A resident random-init GPT-2 on the current device."""

    def __init__(self, cfg: dict, seed: int, sigma: float = 0.02):
        self.cfg = dict(cfg)
        h = ctypes.c_uint64()
        c = Gpt2Config(**self.cfg)
        _lib.check(_lib.load().tq_gpt2_create(ctypes.byref(c), seed, ctypes.c_float(sigma), ctypes.byref(h)))
        self.handle = h.value
        self.last_times_ms = (0.0, 0.0)

    def generate(self, prompt, n: int) -> np.ndarray:
        """Greedy ids of the n tokens after the prompt; last_times_ms holds the
        device time of the prefill and of the decode steps."""
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.empty(n, np.int32)
        t = (ctypes.c_float * 2)()
        _lib.check(_lib.load().tq_gpt2_generate(self.handle, p.ctypes.data_as(ctypes.c_void_p), len(p), n,
                                                out.ctypes.data_as(ctypes.c_void_p), t))
        self.last_times_ms = (t[0], t[1])
        return out

    def free(self) -> None:
        if self.handle:
            _lib.load().tq_gpt2_free(self.handle)
            self.handle = 0

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.free()
