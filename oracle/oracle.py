"""ctypes front end for the CPU oracle (libtq_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
and by bench.py's CPU-baseline leg, always as the checker or the timed CPU
baseline, never as the product path.

The functions restate mattn/tensai's Go code (file:line in tq_oracle.c):
  quantize8   -> QuantizeMatrix            quant.go:37-72
  quantize4   -> QuantizeMatrix4           quant4.go:28-89
  q8_matmul   -> (*QMatrix).MatVec         quant.go:77-103 (+ :108-122 / quant_simd.go:12-48)
  q4_matmul   -> (*Q4Matrix).MatVec        quant4.go:93-119 (+ :126-154 / quant4_simd.go:17-57)
  gpt2_generate -> GPT-2 -q8 greedy loop   _example/gpt2/model.go:179-401, main.go:69-77,163-170
  qwen_generate -> Qwen2 -q4 greedy loop   _example/qwen/model.go:182-307, main.go:225-240
  sample        -> sample (temperature)    _example/gpt2/main.go:78-105 (= _example/qwen/main.go:115-150)
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libtq_oracle.so")
_lib = None

GENERIC = 0
AVX2 = 1
Q4_GROUP = 64


def build() -> str:
    """Compiles the oracle with its Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P, I, U64, F, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_float, ctypes.c_size_t
        L.tqo_synth_fill.argtypes = [P, SZ, U64, U64, F]
        L.tqo_synth_fill.restype = None
        L.tqo_set_threads.argtypes = [I]
        L.tqo_set_threads.restype = I
        L.tqo_get_threads.argtypes = []
        L.tqo_get_threads.restype = I
        L.tqo_quantize8.argtypes = [P, I, I, P, P]
        L.tqo_quantize8.restype = None
        L.tqo_quantize4.argtypes = [P, I, I, P, P]
        L.tqo_quantize4.restype = I
        L.tqo_q8_matmul.argtypes = [P, P, I, I, P, P, I, I]
        L.tqo_q8_matmul.restype = None
        L.tqo_q4_matmul.argtypes = [P, P, I, I, P, P, I, I]
        L.tqo_q4_matmul.restype = None
        L.tqo_gpt2_generate.argtypes = [P, U64, F, P, I, I, P, P, P, P]
        L.tqo_gpt2_generate.restype = I
        L.tqo_qwen_generate.argtypes = [P, U64, F, P, I, I, P, P, P, P]
        L.tqo_qwen_generate.restype = I
        L.tqo_qwen_time_steps.argtypes = [P, I, I, P]
        L.tqo_qwen_time_steps.restype = I
        L.tqo_synth_tokens.argtypes = [P, I, I, U64]
        L.tqo_synth_tokens.restype = None
        L.tqo_sample.argtypes = [P, I, ctypes.c_double, ctypes.c_double]
        L.tqo_sample.restype = I
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def set_threads(n: int) -> int:
    return lib().tqo_set_threads(int(n))


def synth(shape, seed: int, stream: int, sigma: float) -> np.ndarray:
    """Seeded synthetic float32 tensor: Irwin-Hall(12) normal, std sigma.

    Element i of (seed, stream) is identical on the GPU generator."""
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, dtype=np.float32)
    if n:
        lib().tqo_synth_fill(_p(out), n, seed & (2**64 - 1), stream & (2**64 - 1), np.float32(sigma))
    return out.reshape(shape)


def glorot_sigma(rows: int, cols: int) -> float:
    """sqrtF(2/(rows+cols)) as float32, the gain RandomMatrix uses (tensor.go:269-277)."""
    return float(np.sqrt(np.float32(2.0) / np.float32(rows + cols), dtype=np.float32))


def quantize8(w: np.ndarray):
    """QuantizeMatrix: returns (q int8 [rows*cols+16], scale f32 [cols])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    q = np.empty(rows * cols + 16, dtype=np.int8)
    s = np.empty(cols, dtype=np.float32)
    lib().tqo_quantize8(_p(w), rows, cols, _p(q), _p(s))
    return q, s


def quantize4(w: np.ndarray):
    """QuantizeMatrix4: returns (q uint8 [rows*cols/2+16], scale f32 [groups*cols]).

    Raises ValueError with the reference's message on an odd column count."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    if cols % 2:
        raise ValueError(f"tensai: quantize4 needs an even column count, got {cols}")
    groups = (rows + Q4_GROUP - 1) // Q4_GROUP
    q = np.empty(rows * (cols // 2) + 16, dtype=np.uint8)
    s = np.empty(groups * cols, dtype=np.float32)
    rc = lib().tqo_quantize4(_p(w), rows, cols, _p(q), _p(s))
    assert rc == 0
    return q, s


def q8_matmul(q, scale, rows, cols, x, variant=AVX2):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, rows)
    out = np.empty((x.shape[0], cols), dtype=np.float32)
    lib().tqo_q8_matmul(_p(q), _p(scale), rows, cols, _p(x), _p(out), x.shape[0], variant)
    return out


def q4_matmul(q, scale, rows, cols, x, variant=AVX2):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, rows)
    out = np.empty((x.shape[0], cols), dtype=np.float32)
    lib().tqo_q4_matmul(_p(q), _p(scale), rows, cols, _p(x), _p(out), x.shape[0], variant)
    return out


def q8_exact(q, scale, rows, cols, x) -> np.ndarray:
    """float64 recomputation over the same codes (quant_test.go:30-39)."""
    Q = q[: rows * cols].astype(np.float64).reshape(rows, cols)
    x = np.asarray(x, dtype=np.float64).reshape(-1, rows)
    return (x @ Q) * scale.astype(np.float64)[None, :]


def q4_exact(q, scale, rows, cols, x) -> np.ndarray:
    """float64 recomputation per group over the same nibbles (quant4_test.go:31-49)."""
    half = cols // 2
    B = q[: rows * half].reshape(rows, half)
    N = np.concatenate([(B & 0x0F).astype(np.int64) - 8, (B >> 4).astype(np.int64) - 8], axis=1).astype(np.float64)
    x = np.asarray(x, dtype=np.float64).reshape(-1, rows)
    groups = (rows + Q4_GROUP - 1) // Q4_GROUP
    S = scale.astype(np.float64).reshape(groups, cols)
    want = np.zeros((x.shape[0], cols))
    for g in range(groups):
        lo, hi = g * Q4_GROUP, min((g + 1) * Q4_GROUP, rows)
        want += (x[:, lo:hi] @ N[lo:hi]) * S[g][None, :]
    return want


def unpack4(q, rows, cols) -> np.ndarray:
    """Nibble codes (-8..7) as int8 [rows, cols] in column order."""
    half = cols // 2
    B = q[: rows * half].reshape(rows, half)
    return np.concatenate([(B & 0x0F).astype(np.int8) - 8, (B >> 4).astype(np.int8) - 8], axis=1)


class Gpt2Cfg(ctypes.Structure):
    _fields_ = [("n_layer", ctypes.c_int), ("n_head", ctypes.c_int), ("d", ctypes.c_int), ("ffn", ctypes.c_int),
                ("vocab", ctypes.c_int), ("ctx", ctypes.c_int)]


GPT2_SMALL = dict(n_layer=12, n_head=12, d=768, ffn=3072, vocab=50257, ctx=1024)


def sample(logits, temp: float, u: float) -> int:
    """The examples' sample step (_example/gpt2/main.go:78-105) with the
    caller's uniform draw u (rng.Float64()); ties in p go to the lower id."""
    v = np.ascontiguousarray(logits, np.float32)
    return int(lib().tqo_sample(_p(v), len(v), float(temp), float(u)))


def synth_tokens(n: int, vocab: int, seed: int) -> np.ndarray:
    """Seeded uniform token ids in [0, vocab) (a stand-in for a tokenized prompt)."""
    out = np.empty(n, np.int32)
    lib().tqo_synth_tokens(_p(out), n, vocab, seed)
    return out


def gpt2_generate(cfg: dict, seed: int, sigma: float, prompt, n_gen: int, seconds=None):
    """Greedy GPT-2 generation with int8 decode weights on the CPU: returns
    (token ids [n_gen], top-1 margins [n_gen], prefill logits [vocab]); if
    `seconds` is a list it receives the prefill and decode wall times."""
    c = Gpt2Cfg(**cfg)
    prompt = np.ascontiguousarray(prompt, np.int32)
    toks = np.empty(n_gen, np.int32)
    margins = np.empty(n_gen, np.float32)
    first = np.empty(cfg["vocab"], np.float32)
    secs = np.zeros(2, np.float64)
    rc = lib().tqo_gpt2_generate(ctypes.byref(c), seed, sigma, _p(prompt), len(prompt), n_gen, _p(toks),
                                 _p(margins), _p(first), _p(secs))
    if rc != 0:
        raise ValueError("tqo_gpt2_generate: bad configuration")
    if seconds is not None:
        seconds[:] = [float(secs[0]), float(secs[1])]
    return toks, margins, first


class QwenCfg(ctypes.Structure):
    _fields_ = [("n_layer", ctypes.c_int), ("n_head", ctypes.c_int), ("n_kv", ctypes.c_int), ("d", ctypes.c_int),
                ("ffn", ctypes.c_int), ("vocab", ctypes.c_int), ("ctx", ctypes.c_int), ("eps", ctypes.c_double),
                ("theta", ctypes.c_double)]


QWEN_7B = dict(n_layer=28, n_head=28, n_kv=4, d=3584, ffn=18944, vocab=152064, ctx=2560, eps=1e-6, theta=1e6)


def qwen_time_steps(cfg: dict, pos0: int, n_steps: int):
    """Wall seconds of n_steps decode steps at cached positions pos0.. of a
    Qwen2 of shape cfg (seeded filler weights and caches: the timing of a
    long-context step without minutes of weight building), and of the build."""
    c = QwenCfg(**cfg)
    secs = (ctypes.c_double * 2)()
    rc = lib().tqo_qwen_time_steps(ctypes.byref(c), int(pos0), int(n_steps), secs)
    if rc:
        raise ValueError("tqo_qwen_time_steps: bad configuration")
    return float(secs[0]), float(secs[1])


def qwen_generate(cfg: dict, seed: int, sigma: float, prompt, n_gen: int, seconds=None, prompt_logits=False):
    """Greedy Qwen2 generation with int4 weights on the CPU, the prompt fed
    token by token: returns (token ids [n_gen], top-1 margins [n_gen]) and,
    with prompt_logits=True, also the logits after the last prompt token."""
    c = QwenCfg(**cfg)
    prompt = np.ascontiguousarray(prompt, np.int32)
    toks = np.empty(n_gen, np.int32)
    margins = np.empty(n_gen, np.float32)
    secs = np.zeros(2, np.float64)
    logits = np.empty(cfg["vocab"], np.float32)
    rc = lib().tqo_qwen_generate(ctypes.byref(c), seed, sigma, _p(prompt), len(prompt), n_gen, _p(toks),
                                 _p(margins), _p(secs), _p(logits))
    if rc != 0:
        raise ValueError("tqo_qwen_generate: bad configuration")
    if seconds is not None:
        seconds[:] = [float(secs[0]), float(secs[1])]
    return (toks, margins, logits) if prompt_logits else (toks, margins)
