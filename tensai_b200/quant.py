"""Host-side mirror of tensai's quantized-matrix API (quant.go, quant4.go).

Names, fields, argument meaning and error behaviour follow the Go package, so
code written against it reads the same here:

    q := tensai.QuantizeMatrix(m)            q = QuantizeMatrix(m)
    err := q.MatVec(x, out)                  err = q.MatVec(x, out)
    q4, err := tensai.QuantizeMatrix4(m)     q4, err = QuantizeMatrix4(m)

Errors are returned as values (None on success), as the Go functions return
``error``; their messages are the reference's ("tensai: ..."). All compute
runs in libtensai_cuda.so on the GPU: quantization on the device (bit-exact
with quant.go:37-72 / quant4.go:28-89), MatVec against codes kept resident in
HBM after the first call. There is no CPU fallback.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import TensaiError

Q4_GROUP = 64  # q4Group, quant4.go:12


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


class Matrix:
    """Row-major float32 matrix (tensor.go:24-28)."""

    def __init__(self, rows: int, cols: int, data=None):
        self.Rows, self.Cols = int(rows), int(cols)
        if data is None:
            self.Data = np.zeros(self.Rows * self.Cols, dtype=np.float32)
        else:
            self.Data = np.ascontiguousarray(data, dtype=np.float32).reshape(-1)
            if self.Data.size != self.Rows * self.Cols:
                raise ValueError(f"tensai: matrix {rows}x{cols} has {self.Data.size} elements")


def NewMatrix(rows: int, cols: int) -> Matrix:
    return Matrix(rows, cols)


class _Resident:
    """Device twin of a quantized matrix: uploaded once, resident until Free."""

    bits = 0

    def __init__(self):
        self._h = 0

    def handle(self) -> int:
        if not self._h:
            L = _lib.load()
            h = ctypes.c_uint64()
            up = L.tq_q8_upload if self.bits == 8 else L.tq_q4_upload
            _lib.check(up(_p(self.Q), _p(self.Scale), self.Rows, self.Cols, ctypes.byref(h)))
            self._h = h.value
        return self._h

    def Free(self) -> None:
        """Releases the device copy (idempotent, like GPUTensor.Free)."""
        if self._h:
            _lib.load().tq_free(self._h)
            self._h = 0

    def __del__(self):
        try:
            self.Free()
        except Exception:
            pass

    def _shape_error(self, x, out):
        name = "qmatvec" if self.bits == 8 else "q4matvec"
        return TensaiError(_lib.TQ_ERR_SHAPE, f"tensai: {name} shape mismatch: x={len(x)} out={len(out)}, "
                                              f"want {self.Rows}x{self.Cols}")

    def MatVec(self, x, out):
        """out = x @ Q for one activation row (quant.go:77 / quant4.go:93).

        x: float32 array of Rows, out: float32 array of Cols (overwritten).
        Returns None, or the reference's shape-mismatch error."""
        if len(x) != self.Rows or len(out) != self.Cols:
            return self._shape_error(x, out)
        xa = np.ascontiguousarray(x, dtype=np.float32)
        assert isinstance(out, np.ndarray) and out.dtype == np.float32 and out.flags.c_contiguous
        rc = _lib.load().tq_matvec(self.handle(), _p(xa), xa.size, _p(out), out.size)
        if rc != _lib.TQ_OK:
            return TensaiError(rc, _lib.load().tq_last_error().decode())
        return None

    def MatMul(self, x, out, m: int):
        """out[m][Cols] = x[m][Rows] @ Q: the batched form (m MatVec calls in one)."""
        xa = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        if xa.size != m * self.Rows or out.size != m * self.Cols:
            return self._shape_error(x, out)
        rc = _lib.load().tq_matmul(self.handle(), _p(xa), _p(out), m)
        if rc != _lib.TQ_OK:
            return TensaiError(rc, _lib.load().tq_last_error().decode())
        return None


class QMatrix(_Resident):
    """int8 codes with one scale per output column (quant.go:29-33):
    W[i][j] ~= Q[i*Cols+j] * Scale[j]; Q carries the reference's 16 pad bytes."""

    bits = 8

    def __init__(self, rows: int, cols: int, Q=None, Scale=None):
        super().__init__()
        self.Rows, self.Cols = int(rows), int(cols)
        self.Q = np.zeros(self.Rows * self.Cols + 16, dtype=np.int8) if Q is None else np.ascontiguousarray(Q, np.int8)
        self.Scale = np.zeros(self.Cols, dtype=np.float32) if Scale is None else np.ascontiguousarray(Scale, np.float32)


class Q4Matrix(_Resident):
    """int4 codes, offset-binary, column-split nibbles: byte (i, j) holds column
    j (low) and column j+Cols/2 (high); one scale per (64-row group, column)
    (quant4.go:20-24)."""

    bits = 4

    def __init__(self, rows: int, cols: int, Q=None, Scale=None):
        super().__init__()
        self.Rows, self.Cols = int(rows), int(cols)
        groups = (self.Rows + Q4_GROUP - 1) // Q4_GROUP
        self.Q = (np.zeros(self.Rows * (self.Cols // 2) + 16, dtype=np.uint8) if Q is None
                  else np.ascontiguousarray(Q, np.uint8))
        self.Scale = (np.zeros(groups * self.Cols, dtype=np.float32) if Scale is None
                      else np.ascontiguousarray(Scale, np.float32))


def QuantizeMatrix(m: Matrix) -> QMatrix:
    """Column-wise absmax int8 quantization on the GPU (quant.go:37-72).

    The codes/scales come back in the reference layout and the device copy
    stays resident for MatVec."""
    L = _lib.load()
    q = QMatrix(m.Rows, m.Cols)
    _lib.check(L.tq_quantize8(_p(m.Data), m.Rows, m.Cols, _p(q.Q), _p(q.Scale)))
    return q


def QuantizeMatrix4(m: Matrix):
    """Group-wise int4 quantization on the GPU (quant4.go:28-89).

    Returns (Q4Matrix, None), or (None, error) for an odd column count with the
    reference's message (quant4.go:29-31)."""
    if m.Cols % 2 != 0:
        return None, TensaiError(_lib.TQ_ERR_ARG, f"tensai: quantize4 needs an even column count, got {m.Cols}")
    L = _lib.load()
    q = Q4Matrix(m.Rows, m.Cols)
    _lib.check(L.tq_quantize4(_p(m.Data), m.Rows, m.Cols, _p(q.Q), _p(q.Scale)))
    return q, None


# ---- device-resident helpers (torch tensors as plain device buffers) --------

def quantize_dev(w, bits: int, stream=None) -> int:
    """Quantizes a float32 CUDA tensor [rows, cols] into a resident handle."""
    L = _lib.load()
    h = ctypes.c_uint64()
    fn = L.tq_quantize8_dev if bits == 8 else L.tq_quantize4_dev
    st = ctypes.c_void_p(stream.cuda_stream if stream is not None else None)
    _lib.check(fn(ctypes.c_void_p(w.data_ptr()), w.shape[0], w.shape[1], st, ctypes.byref(h)))
    return h.value


def quantize_linear_dev(w, bits: int, stream=None) -> int:
    """Quantizes a checkpoint Linear weight, a CUDA tensor [out, in] of
    float32, float16 or bfloat16, into a resident handle of the matrix the
    loader makes with Matrix().T() (_example/qwen/model.go:126-140):
    rows = in, cols = out."""
    import torch
    kinds = {torch.float32: _lib.TQ_LINEAR_F32, torch.float16: _lib.TQ_LINEAR_F16, torch.bfloat16: _lib.TQ_LINEAR_BF16}
    if w.dtype not in kinds or w.dim() != 2 or not w.is_contiguous():
        raise ValueError("tensai: a contiguous 2-D float32, float16 or bfloat16 Linear weight is required")
    L = _lib.load()
    h = ctypes.c_uint64()
    fn = L.tq_quantize8_linear_dev if bits == 8 else L.tq_quantize4_linear_dev
    st = ctypes.c_void_p(stream.cuda_stream if stream is not None else None)
    _lib.check(fn(ctypes.c_void_p(w.data_ptr()), kinds[w.dtype], w.shape[0], w.shape[1], st, ctypes.byref(h)))
    return h.value


def matmul_dev(handle: int, x, out, stream=None) -> None:
    """out[m, cols] = x[m, rows] @ W on the device (CUDA tensors, float32)."""
    st = ctypes.c_void_p(stream.cuda_stream if stream is not None else None)
    _lib.check(_lib.load().tq_matmul_dev(handle, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                         x.shape[0] if x.dim() == 2 else 1, st))


class Chain:
    """A chain of dependent single-row matvecs run as one launch (tq_chain_create).

    ops: sequence of dicts with keys handle, x, out (CUDA float32 tensors or
    device addresses) and optionally epilogue ("none" | "swiglu" | "resid"),
    resid, norm_w, norm_from, eps."""

    _EPI = {"none": _lib.TQ_CHAIN_EPI_NONE, "swiglu": _lib.TQ_CHAIN_EPI_SWIGLU, "resid": _lib.TQ_CHAIN_EPI_RESID}

    def __init__(self, ops):
        def addr(t):
            if t is None:
                return None
            return t if isinstance(t, int) else t.data_ptr()

        arr = (_lib.ChainOp * len(ops))()
        for i, o in enumerate(ops):
            arr[i].matrix = o["handle"]
            arr[i].x = addr(o["x"])
            arr[i].out = addr(o["out"])
            arr[i].epilogue = self._EPI[o.get("epilogue", "none")]
            arr[i].resid = addr(o.get("resid"))
            arr[i].norm_w = addr(o.get("norm_w"))
            arr[i].norm_from = o.get("norm_from", -1)
            arr[i].eps = o.get("eps", 0.0)
        h = ctypes.c_uint64()
        self.handle = 0
        _lib.check(_lib.load().tq_chain_create(arr, len(ops), ctypes.byref(h)))
        self.handle = h.value

    def run(self, stream=None) -> None:
        st = ctypes.c_void_p(stream.cuda_stream if stream is not None else None)
        _lib.check(_lib.load().tq_chain_run(self.handle, st))

    def free(self) -> None:
        if self.handle:
            _lib.load().tq_chain_free(self.handle)
            self.handle = 0

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.free()


def synth_dev(out, seed: int, stream_id: int, sigma: float, stream=None) -> None:
    """Fills a float32 CUDA tensor with the seeded generator shared with the oracle."""
    st = ctypes.c_void_p(stream.cuda_stream if stream is not None else None)
    _lib.check(_lib.load().tq_synth_dev(ctypes.c_void_p(out.data_ptr()), out.numel(), seed, stream_id,
                                        ctypes.c_float(sigma), st))


def download(handle: int, bits: int, rows: int, cols: int):
    """Codes and scales of a handle in the reference layout (with 16 pad bytes)."""
    groups = (rows + Q4_GROUP - 1) // Q4_GROUP
    if bits == 8:
        q = np.empty(rows * cols + 16, dtype=np.int8)
        s = np.empty(cols, dtype=np.float32)
    else:
        q = np.empty(rows * (cols // 2) + 16, dtype=np.uint8)
        s = np.empty(groups * cols, dtype=np.float32)
    _lib.check(_lib.load().tq_download(handle, _p(q), _p(s)))
    return q, s


def free(handle: int) -> None:
    _lib.load().tq_free(handle)
