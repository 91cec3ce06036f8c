"""GPU parity tests of the quantizers and the M<=15 dequant-matvec, through the
C ABI (libtensai_cuda.so), against the CPU oracle.

Bars (from the task's contract):
  * codes and scales: bit-exact with the oracle's QuantizeMatrix/QuantizeMatrix4;
  * matvec: relative L2 error <= 1e-5 against the oracle's AVX2 and generic
    variants, and every element within the reference test's
    1e-3*(1+|want|) of the float64 recomputation (quant_test.go:40).
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tensai_b200 import NewMatrix, Matrix, QMatrix, Q4Matrix, QuantizeMatrix, QuantizeMatrix4, _lib
from tensai_b200 import quant as Q

pytestmark = pytest.mark.gpu

REL_L2 = 1e-5


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def same_bits(a, b):
    return np.array_equal(np.asarray(a).view(np.uint8), np.asarray(b).view(np.uint8))


@pytest.fixture(scope="module", autouse=True)
def device():
    import torch
    torch.cuda.init()
    _lib.check(_lib.load().tq_set_device(0))


# 0: the default choice per row count, 1: CUDA-core matvec with per-warp
# copies, 3: single-launch CUDA-core matvec (2 rows per launch), 4: tensor-core
# matvec with a digit-plane launch, 5: int4 rows on the tensor cores by
# mma.sync over the K-packed copy (int8 as 3). 2 is retired.
@pytest.fixture(params=[0, 1, 3, 4, 5], ids=["default", "cudacore", "cudacore-1launch", "tcgen05", "mma-int4"])
def kernel(request):
    L = _lib.load()
    _lib.check(L.tq_set_matvec_kernel(request.param))
    yield request.param
    _lib.check(L.tq_set_matvec_kernel(0))


# ---- quantizers ---------------------------------------------------------------

EDGE_SHAPES = [(1, 2), (1, 9), (7, 13), (16, 16), (33, 10), (64, 32), (65, 34), (130, 6), (768, 2304),
               (200, 50), (3, 130)]


@pytest.mark.parametrize("rows,cols", EDGE_SHAPES)
def test_quantize8_bit_exact(rows, cols):
    w = O.synth((rows, cols), 31, rows * 100000 + cols, O.glorot_sigma(rows, cols))
    w[:, cols // 2] = 0  # an all-zero column
    q = QuantizeMatrix(Matrix(rows, cols, w))
    qo, so = O.quantize8(w)
    assert same_bits(q.Q, qo) and same_bits(q.Scale, so)


@pytest.mark.parametrize("rows,cols", [s for s in EDGE_SHAPES if s[1] % 2 == 0])
def test_quantize4_bit_exact(rows, cols):
    w = O.synth((rows, cols), 41, rows * 100000 + cols, O.glorot_sigma(rows, cols))
    w[:, 0] = 0
    q, err = QuantizeMatrix4(Matrix(rows, cols, w))
    assert err is None
    qo, so = O.quantize4(w)
    assert same_bits(q.Q, qo) and same_bits(q.Scale, so)


def test_quantize_golden_fixtures():
    import os
    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "quant_golden.npz"))
    for name in d["names"]:
        name = str(name)
        w, bits = d[f"{name}.w"], int(d[f"{name}.bits"])
        rows, cols = w.shape
        if bits == 8:
            q = QuantizeMatrix(Matrix(rows, cols, w))
        else:
            q, err = QuantizeMatrix4(Matrix(rows, cols, w))
            assert err is None
        assert same_bits(q.Q, d[f"{name}.q"]), name
        assert same_bits(q.Scale, d[f"{name}.scale"]), name
        out = np.zeros(cols, np.float32)
        assert q.MatVec(d[f"{name}.x"], out) is None
        want = d[f"{name}.want"]
        assert np.all(np.abs(out - want) <= 1e-3 * (1 + np.abs(want))), name


@pytest.mark.parametrize("seed", range(4))
def test_quantize_halfway_values(seed):
    """Values exactly on k*s + s/2 (round half away from zero) and +-maxAbs."""
    rng = np.random.default_rng(seed)
    rows, cols = 130, 40
    for bits, levels in ((8, 127), (4, 7)):
        w = np.zeros((rows, cols), np.float32)
        for j in range(cols):
            s = np.float32(2.0 ** rng.integers(-10, 3))
            w[:, j] = (rng.integers(-levels, levels, size=rows).astype(np.float32) + np.float32(0.5)) * s
            w[rng.integers(0, rows), j] = np.float32(levels) * s * (1 if j % 2 else -1)
        if bits == 8:
            q = QuantizeMatrix(Matrix(rows, cols, w))
            qo, so = O.quantize8(w)
        else:
            q, _ = QuantizeMatrix4(Matrix(rows, cols, w))
            qo, so = O.quantize4(w)
        assert same_bits(q.Q, qo) and same_bits(q.Scale, so)


@pytest.mark.parametrize("bits", [8, 4])
def test_device_generator_and_quantizer_at_config_size(bits):
    """The on-device synthetic weights equal the host generator bit for bit, and
    quantizing them on the device equals the oracle (4096 x 11008, C2 up)."""
    import torch
    rows, cols = 4096, 11008
    w = torch.empty(rows, cols, device="cuda", dtype=torch.float32)
    Q.synth_dev(w, 1234, 5, 0.02)
    torch.cuda.synchronize()
    wh = O.synth((rows, cols), 1234, 5, 0.02)
    assert same_bits(w.cpu().numpy(), wh)
    h = Q.quantize_dev(w, bits)
    try:
        qd, sd = Q.download(h, bits, rows, cols)
        qo, so = (O.quantize8 if bits == 8 else O.quantize4)(wh)
        assert same_bits(qd, qo) and same_bits(sd, so)
    finally:
        Q.free(h)


# ---- matvec ports of the reference tests ---------------------------------------

@pytest.mark.parametrize("rows,cols", [(768, 2304), (16, 16), (7, 13), (1, 9)])
def test_quantize_matvec(rows, cols, kernel):
    """TestQuantizeMatVec (quant_test.go:9-70) on the GPU path."""
    w = O.synth((rows, cols), 31, rows * 100000 + cols, O.glorot_sigma(rows, cols))
    q = QuantizeMatrix(Matrix(rows, cols, w))
    x = O.synth((rows,), 31, 1, 1.0)
    out = np.zeros(cols, np.float32)
    assert q.MatVec(x, out) is None
    want = O.q8_exact(q.Q, q.Scale, rows, cols, x)[0]
    assert np.all(np.abs(out - want) <= 1e-3 * (1 + np.abs(want)))
    full = x.astype(np.float64) @ w.astype(np.float64)
    assert np.abs(want - full).max() <= 0.5
    for v in (O.AVX2, O.GENERIC):
        assert rel_l2(out, O.q8_matmul(q.Q, q.Scale, rows, cols, x, v)[0]) <= REL_L2

    q0 = QuantizeMatrix(NewMatrix(4, 4))
    out0 = np.full(4, 7, np.float32)
    assert q0.MatVec(np.zeros(4, np.float32), out0) is None
    assert not out0.any()
    err = q0.MatVec(np.zeros(3, np.float32), out0)
    assert err is not None and "shape mismatch" in str(err)


@pytest.mark.parametrize("rows,cols", [(768, 2304), (64, 32), (33, 10), (1, 2)])
def test_quantize4_matvec(rows, cols, kernel):
    """TestQuantize4MatVec (quant4_test.go:9-78) on the GPU path."""
    w = O.synth((rows, cols), 41, rows * 100000 + cols, O.glorot_sigma(rows, cols))
    q, err = QuantizeMatrix4(Matrix(rows, cols, w))
    assert err is None
    x = O.synth((rows,), 41, 1, 1.0)
    out = np.zeros(cols, np.float32)
    assert q.MatVec(x, out) is None
    want = O.q4_exact(q.Q, q.Scale, rows, cols, x)[0]
    assert np.all(np.abs(out - want) <= 1e-3 * (1 + np.abs(want)))
    full = x.astype(np.float64) @ w.astype(np.float64)
    assert np.abs(want - full).max() <= 1.0
    for v in (O.AVX2, O.GENERIC):
        assert rel_l2(out, O.q4_matmul(q.Q, q.Scale, rows, cols, x, v)[0]) <= REL_L2

    _, err = QuantizeMatrix4(NewMatrix(4, 3))
    assert err is not None
    q4, _ = QuantizeMatrix4(NewMatrix(4, 4))
    assert q4.MatVec(np.zeros(3, np.float32), np.zeros(4, np.float32)) is not None


# ---- config sizes, every M, ragged shapes --------------------------------------

def _check_matmul(bits, rows, cols, m, seed=7):
    w = O.synth((rows, cols), seed, 11, 0.02)
    q, s = (O.quantize8 if bits == 8 else O.quantize4)(w)
    qm = (QMatrix if bits == 8 else Q4Matrix)(rows, cols, q, s)
    x = O.synth((m, rows), seed, 12, 1.0)
    out = np.zeros((m, cols), np.float32)
    assert qm.MatMul(x, out, m) is None
    ref = (O.q8_matmul if bits == 8 else O.q4_matmul)(q, s, rows, cols, x, O.AVX2)
    err = rel_l2(out, ref)
    assert err <= REL_L2, (bits, rows, cols, m, err)
    # per row too: every activation row is its own MatVec in the reference
    for r in range(m):
        assert rel_l2(out[r], ref[r]) <= REL_L2
    qm.Free()
    return out


@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 6, 7, 8])
def test_int8_c1_all_m(m, kernel):
    _check_matmul(8, 4096, 4096, m)


@pytest.mark.parametrize("m", [1, 4, 8])
@pytest.mark.parametrize("rows,cols", [(4096, 11008), (11008, 4096)])
def test_int4_c2_mlp_pair(rows, cols, m, kernel):
    _check_matmul(4, rows, cols, m)


@pytest.mark.parametrize("m", [1, 2, 3, 5, 6, 7])
def test_int4_other_m(m, kernel):
    _check_matmul(4, 1000, 1030, m)


@pytest.mark.parametrize("bits,rows,cols", [(8, 768, 50257), (8, 3072, 768), (8, 100, 3), (4, 130, 6),
                                            (4, 65, 2002), (4, 3584, 18944), (8, 1, 1), (4, 64, 2),
                                            (8, 4095, 4097), (4, 4097, 4098)])
def test_ragged_shapes(bits, rows, cols, kernel):
    _check_matmul(bits, rows, cols, 1)
    _check_matmul(bits, rows, cols, 3)


def test_more_than_8_rows_runs_in_chunks(kernel):
    # 9..15 rows stay on the matvec kernels, 8 rows per launch
    _check_matmul(8, 512, 640, 11)
    _check_matmul(4, 512, 640, 15)


# int4 4096 x 11008 runs the stream-K split (cross-CTA partials in CTA order);
# int8 4096 x 4096 and int4 1000 x 1030 the cluster split (distributed shared
# memory, rank order) of the default kernel.
@pytest.mark.parametrize("bits,rows,cols", [(4, 4096, 11008), (8, 4096, 4096), (4, 1000, 1030)])
def test_results_are_bit_reproducible(kernel, bits, rows, cols):
    w = O.synth((rows, cols), 3, 1, 0.02)
    q, s = (O.quantize8 if bits == 8 else O.quantize4)(w)
    qm = (QMatrix if bits == 8 else Q4Matrix)(rows, cols, q, s)
    x = O.synth((rows,), 3, 2, 1.0)
    outs = []
    for _ in range(3):
        out = np.zeros(cols, np.float32)
        assert qm.MatVec(x, out) is None
        outs.append(out)
    assert same_bits(outs[0], outs[1]) and same_bits(outs[0], outs[2])


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("out_f,in_f", [(130, 200), (10, 33), (4608, 3584), (2, 1)])
def test_quantize_linear_weight_bit_exact(dtype, bits, out_f, in_f):
    """Quantize-on-load: a checkpoint Linear weight [out, in] in its own dtype
    quantizes, transposed and widened inside the kernel, to exactly the codes
    and scales QuantizeMatrix / QuantizeMatrix4 give for Matrix().T()
    (_example/qwen/model.go:126-140; BF16 widening safetensors.go:187-190)."""
    import torch
    dt = getattr(torch, dtype)
    w32 = O.synth((out_f, in_f), 61, out_f * 7 + in_f, 0.05)
    w = torch.from_numpy(w32).cuda().to(dt)
    h = Q.quantize_linear_dev(w, bits)
    torch.cuda.synchronize()
    wt = np.ascontiguousarray(w.float().cpu().numpy().T)  # the loader's f32 transpose, widened exactly
    q, s = Q.download(h, bits, in_f, out_f)
    qo, so = (O.quantize8 if bits == 8 else O.quantize4)(wt)
    assert np.array_equal(q, qo) and same_bits(s, so)
    Q.free(h)


def test_quantize_linear_weight_rejects_odd_int4_width_and_unknown_type():
    import torch
    L = _lib.load()
    w = torch.zeros((3, 64), device="cuda")
    h = ctypes.c_uint64()
    assert L.tq_quantize4_linear_dev(ctypes.c_void_p(w.data_ptr()), _lib.TQ_LINEAR_F32, 3, 64, None, ctypes.byref(h)) == _lib.TQ_ERR_ARG
    assert "even column count" in L.tq_last_error().decode()
    assert L.tq_quantize8_linear_dev(ctypes.c_void_p(w.data_ptr()), 7, 3, 64, None, ctypes.byref(h)) == _lib.TQ_ERR_ARG


def test_host_matvec_replays_follow_new_inputs_and_regrown_staging(kernel):
    """Host-pointer MatVec calls replay a captured graph from a matrix's second
    call on: alternating a small and a larger matrix (the larger one regrows
    the staging buffers and drops the graphs) with fresh inputs every call,
    every result must be the oracle's for that call's input, and a repeated
    input must give the first call's bits."""
    mats = []
    for bits, rows, cols, seed in ((4, 256, 512, 41), (8, 1024, 3000, 42), (4, 4096, 11008, 43)):
        w = O.synth((rows, cols), seed, 1, 0.02)
        q, sc = (O.quantize8 if bits == 8 else O.quantize4)(w)
        mats.append((bits, rows, cols, q, sc, (QMatrix if bits == 8 else Q4Matrix)(rows, cols, q, sc)))
    first = {}
    for it in range(4):
        for i, (bits, rows, cols, q, sc, qm) in enumerate(mats):
            x = O.synth((rows,), 50 + it % 2, i, 1.0)
            out = np.zeros(cols, np.float32)
            assert qm.MatVec(x, out) is None
            want = (O.q8_matmul if bits == 8 else O.q4_matmul)(q, sc, rows, cols, x)[0]
            assert rel_l2(out, want) <= REL_L2, (it, i)
            key = (i, it % 2)
            if key in first:
                assert same_bits(out, first[key]), (it, i)
            else:
                first[key] = out


@pytest.mark.parametrize("m", [1, 4])
@pytest.mark.parametrize("bits", [8, 4])
def test_nan_activation_makes_every_output_nan(bits, m, kernel):
    """A NaN activation reaches every output of its row, as in the
    reference's float products (NaN times any code, zero included, is NaN);
    the kernels that turn activations into integer digits must not hide it.
    The other rows stay finite."""
    rows, cols = 1000, 1030
    w = O.synth((rows, cols), 5, 1, 0.02)
    q, s = (O.quantize8 if bits == 8 else O.quantize4)(w)
    qm = (QMatrix if bits == 8 else Q4Matrix)(rows, cols, q, s)
    x = O.synth((m, rows), 5, 2, 1.0)
    x[0, 123] = np.nan
    out = np.zeros((m, cols), np.float32)
    assert qm.MatMul(x, out, m) is None
    assert np.isnan(out[0]).all()
    assert np.isfinite(out[1:]).all()
    qm.Free()


def _digit_kernel(kernel, bits, m):
    """Whether (kernel, bits, rows) runs on the tensor cores with integer
    activation digits (tq_set_matvec_kernel's table): those give NaN for a
    64-row group holding an infinity, which has no digits."""
    if kernel == 4:
        return True
    if kernel == 5:
        return bits == 4
    if kernel == 0:
        return (bits == 4 and m == 1) or m >= 3
    return False


@pytest.mark.parametrize("m", [1, 4])
@pytest.mark.parametrize("bits", [8, 4])
def test_infinite_activation_makes_every_output_non_finite(bits, m, kernel):
    """An infinite activation leaves no output of its row finite, as in the
    reference (Inf times a nonzero code is +-Inf, times a zero code NaN). The
    CUDA-core kernels give the reference's values: the oracle's +-Inf / NaN
    pattern column for column. The digit kernels give NaN for every column of
    the row. The other rows stay finite."""
    rows, cols = 1000, 1030
    w = O.synth((rows, cols), 6, 1, 0.02)
    q, s = (O.quantize8 if bits == 8 else O.quantize4)(w)
    qm = (QMatrix if bits == 8 else Q4Matrix)(rows, cols, q, s)
    x = O.synth((m, rows), 6, 2, 1.0)
    x[0, 321] = np.inf
    out = np.zeros((m, cols), np.float32)
    assert qm.MatMul(x, out, m) is None
    assert not np.isfinite(out[0]).any()
    assert np.isfinite(out[1:]).all()
    if _digit_kernel(kernel, bits, m):
        assert np.isnan(out[0]).all()
    else:
        want = (O.q8_matmul if bits == 8 else O.q4_matmul)(q, s, rows, cols, x[:1])[0]
        assert np.array_equal(np.isnan(out[0]), np.isnan(want))
        assert np.array_equal(out[0][~np.isnan(want)], want[~np.isnan(want)])
    qm.Free()


def test_device_pointer_path_on_a_torch_stream():
    import torch
    rows, cols, m = 2048, 3000, 4
    w = torch.empty(rows, cols, device="cuda")
    Q.synth_dev(w, 5, 1, 0.02)
    x = torch.empty(m, rows, device="cuda")
    Q.synth_dev(x, 5, 2, 1.0)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        h = Q.quantize_dev(w, 8, st)
        out = torch.empty(m, cols, device="cuda")
        Q.matmul_dev(h, x, out, st)
    st.synchronize()
    qd, sd = Q.download(h, 8, rows, cols)
    ref = O.q8_matmul(qd, sd, rows, cols, x.cpu().numpy())
    assert rel_l2(out.cpu().numpy(), ref) <= REL_L2
    Q.free(h)


def test_handle_lifecycle_and_download_roundtrip():
    rows, cols = 70, 12
    w = O.synth((rows, cols), 1, 1, 0.5)
    q, s = O.quantize4(w)
    L = _lib.load()
    h = ctypes.c_uint64()
    _lib.check(L.tq_q4_upload(q.ctypes.data_as(ctypes.c_void_p), s.ctypes.data_as(ctypes.c_void_p), rows, cols,
                              ctypes.byref(h)))
    bits, r, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _lib.check(L.tq_matrix_info(h.value, ctypes.byref(bits), ctypes.byref(r), ctypes.byref(c)))
    assert (bits.value, r.value, c.value) == (4, rows, cols)
    qd, sd = Q.download(h.value, 4, rows, cols)
    assert same_bits(qd, q) and same_bits(sd, s)
    assert L.tq_free(h.value) == 0
    assert L.tq_free(h.value) == 0  # double free: no-op
    x = np.zeros(rows, np.float32)
    out = np.zeros(cols, np.float32)
    assert L.tq_matvec(h.value, x.ctypes.data_as(ctypes.c_void_p), rows, out.ctypes.data_as(ctypes.c_void_p),
                       cols) == _lib.TQ_ERR_HANDLE


def test_injected_allocation_failure_is_reported():
    L = _lib.load()
    q = np.zeros(64 + 16, np.int8)
    s = np.zeros(8, np.float32)
    h = ctypes.c_uint64()
    L.tq_debug_fail_allocs(1)
    rc = L.tq_q8_upload(q.ctypes.data_as(ctypes.c_void_p), s.ctypes.data_as(ctypes.c_void_p), 8, 8, ctypes.byref(h))
    assert rc == _lib.TQ_ERR_NOMEM and b"allocation" in L.tq_last_error()
    # the library keeps working afterwards
    _lib.check(L.tq_q8_upload(q.ctypes.data_as(ctypes.c_void_p), s.ctypes.data_as(ctypes.c_void_p), 8, 8,
                              ctypes.byref(h)))
    L.tq_free(h.value)


def test_no_timeouts_recorded():
    """No kernel of this module gave up a bounded wait."""
    bits = ctypes.c_uint(0)
    _lib.check(_lib.load().tq_device_status(ctypes.byref(bits)))
    assert bits.value == 0
