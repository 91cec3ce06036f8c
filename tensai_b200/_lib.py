"""ctypes binding of libtensai_cuda.so (the C ABI in include/tensai_cuda.h).

The library is built in-tree (tensai_b200/libtensai_cuda.so). There is no CPU
fallback: if the shared library is missing or fails to load, importing the
binding raises, so a GPU run can never silently take another path.
"""
from __future__ import annotations

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("TENSAI_CUDA_LIB", os.path.join(_HERE, "libtensai_cuda.so"))
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "tensai_cuda.h")

TQ_OK = 0
TQ_ERR_ARG = -1
TQ_ERR_SHAPE = -2
TQ_ERR_HANDLE = -3
TQ_ERR_CUDA = -4
TQ_ERR_NOMEM = -5
TQ_ERR_UNSUPPORTED = -6
TQ_ERR_TIMEOUT = -7

P = ctypes.c_void_p
I = ctypes.c_int
U64 = ctypes.c_uint64
SZ = ctypes.c_size_t
F = ctypes.c_float
PU64 = ctypes.POINTER(ctypes.c_uint64)
PI = ctypes.POINTER(ctypes.c_int)

# name -> (restype, argtypes); every symbol declared in include/tensai_cuda.h.
SIGNATURES = {
    "tq_version": (I, []),
    "tq_last_error": (ctypes.c_char_p, []),
    "tq_device_count": (I, [PI]),
    "tq_set_device": (I, [I]),
    "tq_q8_upload": (I, [P, P, I, I, PU64]),
    "tq_q4_upload": (I, [P, P, I, I, PU64]),
    "tq_quantize8": (I, [P, I, I, P, P]),
    "tq_quantize4": (I, [P, I, I, P, P]),
    "tq_quantize8_dev": (I, [P, I, I, P, PU64]),
    "tq_quantize4_dev": (I, [P, I, I, P, PU64]),
    "tq_quantize8_linear_dev": (I, [P, I, I, I, P, PU64]),
    "tq_quantize4_linear_dev": (I, [P, I, I, I, P, PU64]),
    "tq_matrix_info": (I, [U64, PI, PI, PI]),
    "tq_download": (I, [U64, P, P]),
    "tq_free": (I, [U64]),
    "tq_matvec": (I, [U64, P, SZ, P, SZ]),
    "tq_matmul": (I, [U64, P, P, I]),
    "tq_matmul_dev": (I, [U64, P, P, I, P]),
    "tq_matmul_dev_fixed": (I, [U64, P, P, I, P]),
    "tq_synth_dev": (I, [P, SZ, U64, U64, F, P]),
    "tq_device_status": (I, [ctypes.POINTER(ctypes.c_uint)]),
    "tq_gpt2_create": (I, [P, U64, F, PU64]),
    "tq_gpt2_generate": (I, [U64, P, I, I, P, P]),
    "tq_gpt2_free": (I, [U64]),
    "tq_synth_tokens": (I, [P, I, I, U64]),
    "tq_nccl_unique_id": (I, [P]),
    "tq_qwen_create": (I, [P, U64, F, I, I, P, PU64]),
    "tq_qwen_generate": (I, [U64, P, I, I, P, P]),
    "tq_qwen_set_prefill": (I, [U64, I]),
    "tq_qwen_exchange": (I, [U64, ctypes.POINTER(ctypes.c_int)]),
    "tq_qwen_create_empty": (I, [P, PU64]),
    "tq_qwen_load_tensor": (I, [U64, ctypes.c_char_p, P, I, I, I]),
    "tq_sample": (I, [P, I, ctypes.c_double, ctypes.c_double, ctypes.POINTER(ctypes.c_int)]),
    "tq_gpt2_set_sampling": (I, [U64, ctypes.c_double, P, I]),
    "tq_gpt2_create_empty": (I, [P, PU64]),
    "tq_gpt2_load_tensor": (I, [U64, ctypes.c_char_p, P, I, I, I]),
    "tq_qwen_set_sampling": (I, [U64, ctypes.c_double, P, I]),
    "tq_qwen_free": (I, [U64]),
    "tq_qwen_shard_plan": (I, [P, I, I, P]),
    "tq_chain_create": (I, [P, I, PU64]),
    "tq_chain_run": (I, [U64, P]),
    "tq_chain_free": (I, [U64]),
    "tq_set_matvec_kernel": (I, [I]),
    "tq_debug_fail_allocs": (I, [I]),
}

ABI_VERSION = 1

TQ_LINEAR_F32 = 0
TQ_LINEAR_F16 = 1
TQ_LINEAR_BF16 = 2
TQ_EXCHANGE_NONE = 0
TQ_EXCHANGE_NCCL = 1
TQ_EXCHANGE_PEER = 2
TQ_CHAIN_EPI_NONE = 0
TQ_CHAIN_EPI_SWIGLU = 1
TQ_CHAIN_EPI_RESID = 2


class ChainOp(ctypes.Structure):
    """tq_chain_op of include/tensai_cuda.h."""

    _fields_ = [("matrix", ctypes.c_uint64), ("x", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("epilogue", ctypes.c_int), ("resid", ctypes.c_void_p), ("norm_w", ctypes.c_void_p),
                ("norm_from", ctypes.c_int), ("eps", ctypes.c_double)]


class TensaiError(RuntimeError):
    """A failing library call; .code is the TQ_ERR_* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


_lib = None


def header_symbols() -> list[str]:
    """Function names declared in include/tensai_cuda.h."""
    with open(HEADER_PATH) as f:
        text = f.read()
    return sorted(set(re.findall(r"^TQ_EXPORT\s+[^(]*?\b(tq_\w+)\s*\(", text, flags=re.M)))


def load():
    """Loads and type-annotates the library (once). Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libtensai_cuda.so not found at {LIB_PATH}; build it with "
            "`python -c 'import __graft_entry__ as g; g.build()'` or `make -C tensai_b200/csrc`")
    L = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    if L.tq_version() != ABI_VERSION:
        raise ImportError(f"libtensai_cuda.so ABI {L.tq_version()} != expected {ABI_VERSION}")
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != TQ_OK:
        msg = load().tq_last_error().decode()
        raise TensaiError(rc, msg)
