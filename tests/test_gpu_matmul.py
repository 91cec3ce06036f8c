"""GPU parity tests of the M >= 16 matmul (tcgen05 kind::tf32 with fp32
accumulators), through the C ABI, against the CPU oracle.

Bar: relative L2 error <= 2e-3 against the oracle's AVX2 MatVec applied to
every activation row (the reference has no batched call: M rows are M
MatVec calls), overall and per row, and against the float64 recomputation
over the same codes.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tensai_b200 import Q4Matrix, QMatrix, _lib

pytestmark = pytest.mark.gpu

TF32_REL_L2 = 2e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module", autouse=True)
def device():
    import torch
    torch.cuda.init()
    _lib.check(_lib.load().tq_set_device(0))


def _run(bits, rows, cols, m, seed=5, reps=1):
    w = O.synth((rows, cols), seed, 21, 0.02)
    q, s = (O.quantize8 if bits == 8 else O.quantize4)(w)
    qm = (QMatrix if bits == 8 else Q4Matrix)(rows, cols, q, s)
    x = O.synth((m, rows), seed, 22, 1.0)
    outs = []
    for _ in range(reps):
        out = np.full((m, cols), np.nan, np.float32)
        assert qm.MatMul(x, out, m) is None
        outs.append(out)
    qm.Free()
    return q, s, x, outs


def _check(bits, rows, cols, m, seed=5):
    q, s, x, (out,) = _run(bits, rows, cols, m, seed)
    assert np.isfinite(out).all()
    ref = (O.q8_matmul if bits == 8 else O.q4_matmul)(q, s, rows, cols, x, O.AVX2)
    err = rel_l2(out, ref)
    assert err <= TF32_REL_L2, (bits, rows, cols, m, err)
    for r in range(m):
        assert rel_l2(out[r], ref[r]) <= TF32_REL_L2, (r, rel_l2(out[r], ref[r]))
    exact = (O.q8_exact if bits == 8 else O.q4_exact)(q, s, rows, cols, x)
    assert rel_l2(out, exact) <= TF32_REL_L2
    return err


def test_int4_4096_m64_config():
    """int4 group-64 batched matmul M=64 on W [4096 x 4096]."""
    err = _check(4, 4096, 4096, 64)
    assert err > 0  # tf32 operands: not silently the fp32 path


@pytest.mark.parametrize("m", [16, 17, 31, 33, 64, 65, 100, 128, 129, 300])
def test_int4_every_row_count(m):
    _check(4, 1000, 1030, m)


@pytest.mark.parametrize("m", [16, 24, 64, 128, 200])
def test_int8_row_counts(m):
    _check(8, 777, 1100, m)


@pytest.mark.parametrize("bits,rows,cols", [(8, 768, 2304), (8, 3072, 768), (8, 100, 3), (4, 130, 6),
                                            (4, 65, 2002), (8, 1, 1), (4, 64, 2), (8, 4095, 4097),
                                            (4, 4097, 4098), (4, 3584, 4736), (8, 64, 128), (4, 63, 256)])
def test_ragged_shapes(bits, rows, cols):
    _check(bits, rows, cols, 16)
    _check(bits, rows, cols, 40)


def test_int4_mlp_shapes_prefill_chunk():
    _check(4, 4096, 11008, 32)
    _check(4, 11008, 4096, 32)


def test_matmul_is_bit_reproducible():
    _, _, _, outs = _run(4, 4096, 4096, 64, seed=9, reps=3)
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    assert np.array_equal(outs[0].view(np.uint32), outs[2].view(np.uint32))


def test_zero_matrix_gives_zero():
    rows, cols, m = 200, 260, 20
    q, s = O.quantize4(np.zeros((rows, cols), np.float32))
    qm = Q4Matrix(rows, cols, q, s)
    out = np.full((m, cols), np.nan, np.float32)
    assert qm.MatMul(O.synth((m, rows), 1, 2, 1.0), out, m) is None
    qm.Free()
    assert not out.any()


def test_no_timeouts_recorded():
    import ctypes
    bits = ctypes.c_uint(0)
    _lib.check(_lib.load().tq_device_status(ctypes.byref(bits)))
    assert bits.value == 0
