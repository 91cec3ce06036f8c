"""tq_matmul_dev_fixed: the allocation-free matvec entry point, through the C ABI.

Its results must match tq_matmul_dev (the CUDA-core kernel it shares, and the
default tensor-core kernel) and the CPU oracle (the AVX2 restatement of
quant_simd.go / quant4_simd.go) within the matvec tolerance (1e-5 relative
L2), on consecutive calls that reuse the fixed scratch, and the two
consecutive calls must agree bit for bit. The file sorts last so that it also runs after every other GPU test
in one process; it passes alone in a fresh process too.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tensai_b200 import _lib
from tensai_b200 import quant as Q

pytestmark = pytest.mark.gpu

REL_L2 = 1e-5


def _rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.linalg.norm(b)
    return np.linalg.norm(a - b) / (d if d > 0 else 1.0)


@pytest.fixture(scope="module")
def lib():
    import torch
    L = _lib.load()
    _lib.check(L.tq_set_device(0))
    torch.cuda.set_device(0)
    return L


def _case(bits, rows, cols, m, seed):
    import torch
    w = torch.empty(rows, cols, device="cuda")
    Q.synth_dev(w, seed, 1, 0.02)
    h = Q.quantize_dev(w, bits)
    del w
    x = torch.empty(m, rows, device="cuda")
    Q.synth_dev(x, seed, 2, 1.0)
    torch.cuda.synchronize()  # inputs were made on the default stream; the calls use their own
    return h, x


def _call(fn, h, x, m, cols, stream):
    import torch
    out = torch.full((m, cols), float("nan"), device="cuda")
    torch.cuda.synchronize()
    rc = fn(h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()), m, ctypes.c_void_p(stream.cuda_stream))
    _lib.check(rc)
    stream.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("bits,rows,cols,m", [
    (4, 4096, 11008, 1), (4, 11008, 4096, 3), (8, 4096, 4096, 1), (8, 1024, 4096, 8),
    (4, 1000, 1030, 5), (8, 77, 130, 2), (4, 64, 256, 4),
])
def test_fixed_matches_existing_entry(lib, bits, rows, cols, m):
    import torch
    st = torch.cuda.Stream()
    h, x = _case(bits, rows, cols, m, seed=11 + rows + m)
    try:
        first = _call(lib.tq_matmul_dev_fixed, h, x, m, cols, st)
        second = _call(lib.tq_matmul_dev_fixed, h, x, m, cols, st)
        _lib.check(lib.tq_set_matvec_kernel(1))
        try:
            cuda_core = _call(lib.tq_matmul_dev, h, x, m, cols, st)
        finally:
            _lib.check(lib.tq_set_matvec_kernel(0))
        default = _call(lib.tq_matmul_dev, h, x, m, cols, st)
        q, sc = Q.download(h, bits, rows, cols)
        want = (O.q8_matmul if bits == 8 else O.q4_matmul)(q, sc, rows, cols, x.cpu().numpy())
    finally:
        Q.free(h)
    assert np.isfinite(first).all() and np.isfinite(second).all()
    np.testing.assert_array_equal(first, second)
    assert _rel_l2(first, cuda_core) <= REL_L2
    assert _rel_l2(second, cuda_core) <= REL_L2
    assert _rel_l2(first, default) <= REL_L2
    assert _rel_l2(second, default) <= REL_L2
    assert _rel_l2(first, want) <= REL_L2
    assert _rel_l2(second, want) <= REL_L2


def test_fixed_allocates_no_device_memory(lib):
    import torch
    st = torch.cuda.Stream()
    h, x = _case(4, 4096, 11008, 2, seed=5)
    out = torch.empty(2, 11008, device="cuda")
    torch.cuda.synchronize()
    args = (h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()), 2, ctypes.c_void_p(st.cuda_stream))
    try:
        _lib.check(lib.tq_matmul_dev_fixed(*args))  # set-up of this device (already done if other tests ran)
        st.synchronize()
        free0, _ = torch.cuda.mem_get_info()
        for _ in range(3):
            _lib.check(lib.tq_matmul_dev_fixed(*args))
        st.synchronize()
        free1, _ = torch.cuda.mem_get_info()
    finally:
        Q.free(h)
    assert free1 == free0


def test_fixed_first_call_of_each_kernel_allocates_nothing(lib):
    """The set-up (first call on the device) loads every kernel the entry point
    can launch, so the first call of each (bits, rows per launch) afterwards
    takes no device memory either."""
    import torch
    st = torch.cuda.Stream()
    cases = [(bits, m) + _case(bits, 256, 512, m, seed=40 + bits + m) for bits in (8, 4) for m in (1, 2, 3, 4)]
    outs = [torch.empty(m, 512, device="cuda") for _, m, _, _ in cases]
    torch.cuda.synchronize()
    try:
        bits, m, h, x = cases[0]
        _lib.check(lib.tq_matmul_dev_fixed(h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(outs[0].data_ptr()), m,
                                           ctypes.c_void_p(st.cuda_stream)))  # set-up (a no-op if done before)
        st.synchronize()
        free0, _ = torch.cuda.mem_get_info()
        for (bits, m, h, x), out in zip(cases, outs):
            _lib.check(lib.tq_matmul_dev_fixed(h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()), m,
                                               ctypes.c_void_p(st.cuda_stream)))
        st.synchronize()
        free1, _ = torch.cuda.mem_get_info()
        bits_out = ctypes.c_uint(7)
        _lib.check(lib.tq_device_status(ctypes.byref(bits_out)))  # no timeout, and the fixed word is read
    finally:
        for _, _, h, _ in cases:
            Q.free(h)
    assert free1 == free0
    assert bits_out.value == 0


def test_fixed_rejects_matrices_beyond_its_scratch(lib):
    import torch
    cols = 4097 * 128  # int8: 4097 column tiles, one more than the fixed counters hold
    w = torch.empty(2, cols, device="cuda")
    Q.synth_dev(w, 3, 1, 0.02)
    h = Q.quantize_dev(w, 8)
    x = torch.ones(1, 2, device="cuda")
    out = torch.empty(1, cols, device="cuda")
    try:
        rc = lib.tq_matmul_dev_fixed(h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()), 1, None)
        msg = lib.tq_last_error().decode()
    finally:
        Q.free(h)
    assert rc == _lib.TQ_ERR_UNSUPPORTED
    assert "4096 column tiles" in msg and "tq_matmul_dev" in msg


def test_fixed_argument_errors(lib):
    import torch
    h, x = _case(8, 128, 256, 1, seed=9)
    out = torch.empty(1, 256, device="cuda")
    try:
        assert lib.tq_matmul_dev_fixed(h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()), -1,
                                       None) == _lib.TQ_ERR_ARG
        assert lib.tq_matmul_dev_fixed(h, None, ctypes.c_void_p(out.data_ptr()), 1, None) == _lib.TQ_ERR_ARG
        assert lib.tq_matmul_dev_fixed(h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()), 0,
                                       None) == _lib.TQ_OK
    finally:
        Q.free(h)
    assert lib.tq_matmul_dev_fixed(h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()), 1,
                                   None) == _lib.TQ_ERR_HANDLE
