"""CPU tests of the drop-in boundary: libtensai_cuda.so loads, exports every
entry point include/tensai_cuda.h declares, and its host-side argument
checks return the reference's errors without touching a GPU."""
import ctypes
import subprocess

import numpy as np
import pytest

from tensai_b200 import _lib


@pytest.fixture(scope="module")
def L():
    return _lib.load()


def test_exports_every_header_symbol(L):
    declared = _lib.header_symbols()
    assert len(declared) >= 15
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    assert set(declared) == set(_lib.SIGNATURES), "ctypes table out of sync with the header"
    # No symbol of the implementation leaks: everything exported is declared.
    extra = sorted(s for s in exported if s.startswith("tq_") and s not in declared)
    assert not extra, extra


def test_version(L):
    assert L.tq_version() == _lib.ABI_VERSION


def test_unknown_handle_is_an_error_not_a_crash(L):
    x = np.zeros(4, np.float32)
    out = np.zeros(4, np.float32)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    rc = L.tq_matvec(12345, p(x), 4, p(out), 4)
    assert rc == _lib.TQ_ERR_HANDLE
    assert b"invalid or freed matrix handle" in L.tq_last_error()
    assert L.tq_matmul(999, p(x), p(out), 1) == _lib.TQ_ERR_HANDLE
    assert L.tq_matrix_info(999, None, None, None) == _lib.TQ_ERR_HANDLE


def test_free_is_idempotent(L):
    assert L.tq_free(0) == _lib.TQ_OK
    assert L.tq_free(777) == _lib.TQ_OK


def test_odd_columns_rejected_before_any_device_work(L):
    w = np.zeros((4, 3), np.float32)
    q = np.zeros(64, np.uint8)
    s = np.zeros(16, np.float32)
    rc = L.tq_quantize4(w.ctypes.data_as(ctypes.c_void_p), 4, 3, q.ctypes.data_as(ctypes.c_void_p),
                        s.ctypes.data_as(ctypes.c_void_p))
    assert rc == _lib.TQ_ERR_ARG
    assert L.tq_last_error() == b"tensai: quantize4 needs an even column count, got 3"
    h = ctypes.c_uint64()
    assert L.tq_q4_upload(q.ctypes.data_as(ctypes.c_void_p), s.ctypes.data_as(ctypes.c_void_p), 4, 3,
                          ctypes.byref(h)) == _lib.TQ_ERR_ARG


def test_null_and_negative_arguments(L):
    h = ctypes.c_uint64()
    assert L.tq_q8_upload(None, None, 4, 4, ctypes.byref(h)) == _lib.TQ_ERR_ARG
    assert L.tq_q8_upload(None, None, 4, 4, None) == _lib.TQ_ERR_ARG
    q = np.zeros(32, np.int8)
    s = np.zeros(4, np.float32)
    assert L.tq_q8_upload(q.ctypes.data_as(ctypes.c_void_p), s.ctypes.data_as(ctypes.c_void_p), -1, 4,
                          ctypes.byref(h)) == _lib.TQ_ERR_ARG
    assert L.tq_device_count(None) == _lib.TQ_ERR_ARG


def test_mirror_shape_error_matches_reference_wording():
    from tensai_b200 import QMatrix, Q4Matrix, QuantizeMatrix4, NewMatrix
    q = QMatrix(4, 4)
    err = q.MatVec(np.zeros(3, np.float32), np.zeros(4, np.float32))
    assert str(err) == "tensai: qmatvec shape mismatch: x=3 out=4, want 4x4"
    q4 = Q4Matrix(4, 4)
    err = q4.MatVec(np.zeros(3, np.float32), np.zeros(4, np.float32))
    assert str(err) == "tensai: q4matvec shape mismatch: x=3 out=4, want 4x4"
    m, err = QuantizeMatrix4(NewMatrix(4, 3))
    assert m is None and str(err) == "tensai: quantize4 needs an even column count, got 3"


def test_missing_library_fails_loudly(tmp_path):
    code = ("import os, sys; os.environ['TENSAI_CUDA_LIB'] = sys.argv[1]\n"
            "from tensai_b200 import _lib\n"
            "try:\n    _lib.load()\nexcept ImportError as e:\n    print('IMPORTERROR', e)\n")
    r = subprocess.run(["python", "-c", code, str(tmp_path / "nope.so")], capture_output=True, text=True,
                       cwd=_lib._HERE + "/..")
    assert "IMPORTERROR" in r.stdout


def test_sample_argument_checks_need_no_gpu(L):
    """tq_sample rejects its bad arguments before any CUDA call (the sample
    step of _example/gpt2/main.go:78-105 takes a non-empty logit slice)."""
    v = np.zeros(4, np.float32)
    tok = ctypes.c_int(-7)
    p = v.ctypes.data_as(ctypes.c_void_p)
    assert L.tq_sample(p, 0, 1.0, 0.5, ctypes.byref(tok)) == _lib.TQ_ERR_ARG
    assert "at least one logit" in L.tq_last_error().decode()
    assert L.tq_sample(p, 4, float("nan"), 0.5, ctypes.byref(tok)) == _lib.TQ_ERR_ARG
    assert L.tq_sample(p, 4, 1.0, -0.1, ctypes.byref(tok)) == _lib.TQ_ERR_ARG
    assert L.tq_sample(None, 4, 1.0, 0.5, ctypes.byref(tok)) == _lib.TQ_ERR_ARG
    assert tok.value == -7  # nothing written on an error


def test_sampling_settings_of_an_unknown_model_are_an_error(L):
    d = (ctypes.c_double * 1)(0.5)
    assert L.tq_gpt2_set_sampling(98765, 1.0, d, 1) == _lib.TQ_ERR_HANDLE
    assert L.tq_qwen_set_sampling(98765, 1.0, d, 1) == _lib.TQ_ERR_HANDLE
