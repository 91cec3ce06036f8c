"""CPU tests of the oracle (oracle/tq_oracle.c) — the checker the CUDA path is
held to. They port the reference's own tests (quant_test.go:9-70,
quant4_test.go:9-78) shape for shape, pin the C restatement against an
independent numpy restatement and hand-computed answers, and check the
committed golden fixtures."""
import os

import numpy as np
import pytest

import refquant  # noqa: E402
from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quant_golden.npz")


def same_bits(a, b):
    return np.array_equal(np.asarray(a).view(np.uint8), np.asarray(b).view(np.uint8))


# ---- hand-computed known answers ---------------------------------------------

def test_hand_int8():
    # col0: maxAbs 127 -> s=1, inv=1: 127->127.5->127, 2.5->3.0->3
    # col1: maxAbs 63.5 -> s=0.5, inv=2: -63.5*2=-127->-127.5->-127, 1*2=2->2.5->2
    w = np.array([[127, -63.5], [2.5, 1.0]], dtype=np.float32)
    q, s = O.quantize8(w)
    assert list(q[:4]) == [127, -127, 3, 2] and list(q[4:]) == [0] * 16
    assert list(s) == [1.0, 0.5]


def test_hand_int4():
    # col0: s=1: 7->15 (nibble 7+8), -2.5->-3->5; col1: s=0.5, inv=2: -3.5->-7->1, 1.75->3.5->4->12
    # byte(i,0) = nib(col0) | nib(col1)<<4
    w = np.array([[7, -3.5], [-2.5, 1.75]], dtype=np.float32)
    q, s = O.quantize4(w)
    assert list(q[:2]) == [0x1F, 0xC5] and list(q[2:]) == [0] * 16
    assert list(s) == [1.0, 0.5]


def test_zero_scales():
    q, s = O.quantize8(np.zeros((4, 4), np.float32))
    assert not q.any() and not s.any()
    out = O.q8_matmul(q, s, 4, 4, np.zeros(4, np.float32))
    assert not out.any()
    q4, s4 = O.quantize4(np.zeros((3, 4), np.float32))
    assert all(b == 0x88 for b in q4[:6]) and not s4.any()  # s==0 -> nibble 8 (quant4.go:57-62)


def test_odd_columns_error():
    with pytest.raises(ValueError, match="tensai: quantize4 needs an even column count, got 3"):
        O.quantize4(np.zeros((4, 3), np.float32))


# ---- independent restatement -----------------------------------------------

@pytest.mark.parametrize("seed", range(6))
def test_quantizers_match_numpy_restatement(seed):
    rng = np.random.default_rng(seed)
    for rows, cols in [(1, 2), (3, 8), (64, 10), (65, 34), (130, 6), (200, 50)]:
        w = O.synth((rows, cols), seed, rows * 1000 + cols, float(rng.uniform(0.01, 3)))
        w[:, rng.integers(0, cols)] = 0  # one all-zero column
        w[rng.integers(0, rows), rng.integers(0, cols)] *= -1
        assert same_bits(O.quantize8(w)[0], refquant.quantize8(w)[0])
        assert same_bits(O.quantize8(w)[1], refquant.quantize8(w)[1])
        q4, s4 = O.quantize4(w)
        r4, rs4 = refquant.quantize4(w)
        assert same_bits(q4, r4) and same_bits(s4, rs4)


def test_golden_fixtures():
    d = np.load(GOLDEN)
    for name in d["names"]:
        name = str(name)
        w, bits = d[f"{name}.w"], int(d[f"{name}.bits"])
        q, s = (O.quantize8 if bits == 8 else O.quantize4)(w)
        assert same_bits(q, d[f"{name}.q"]), name
        assert same_bits(s, d[f"{name}.scale"]), name
        rows, cols = w.shape
        mm = O.q8_matmul if bits == 8 else O.q4_matmul
        want = d[f"{name}.want"]
        for v in (O.GENERIC, O.AVX2):
            got = mm(q, s, rows, cols, d[f"{name}.x"], v)[0]
            assert np.all(np.abs(got - want) <= 1e-3 * (1 + np.abs(want))), (name, v)


# ---- ports of the reference tests --------------------------------------------

@pytest.mark.parametrize("rows,cols", [(768, 2304), (16, 16), (7, 13), (1, 9)])
def test_quantize_matvec_port(rows, cols):
    """TestQuantizeMatVec (quant_test.go:9-70) against both kernel variants."""
    w = O.synth((rows, cols), 31, rows * 100000 + cols, O.glorot_sigma(rows, cols))
    q, s = O.quantize8(w)
    x = O.synth((rows,), 31, 1, 1.0)
    want = O.q8_exact(q, s, rows, cols, x)[0]
    for v in (O.GENERIC, O.AVX2):
        out = O.q8_matmul(q, s, rows, cols, x, v)[0]
        assert np.all(np.abs(out - want) <= 1e-3 * (1 + np.abs(want)))
    full = x.astype(np.float64) @ w.astype(np.float64)
    assert np.abs(want - full).max() <= 0.5


@pytest.mark.parametrize("rows,cols", [(768, 2304), (64, 32), (33, 10), (1, 2)])
def test_quantize4_matvec_port(rows, cols):
    """TestQuantize4MatVec (quant4_test.go:9-78) against both kernel variants."""
    w = O.synth((rows, cols), 41, rows * 100000 + cols, O.glorot_sigma(rows, cols))
    q, s = O.quantize4(w)
    x = O.synth((rows,), 41, 1, 1.0)
    want = O.q4_exact(q, s, rows, cols, x)[0]
    for v in (O.GENERIC, O.AVX2):
        out = O.q4_matmul(q, s, rows, cols, x, v)[0]
        assert np.all(np.abs(out - want) <= 1e-3 * (1 + np.abs(want)))
    full = x.astype(np.float64) @ w.astype(np.float64)
    assert np.abs(want - full).max() <= 1.0


def test_threaded_path_matches_single_thread():
    """The worker split (quant.go:82-101) never changes a result: chunks are
    independent column ranges computed by the same body."""
    rows, cols = 1024, 1032  # > 2^20 elements: parallel path, ragged last chunk
    w = O.synth((rows, cols), 3, 3, 0.02)
    x = O.synth((rows,), 3, 4, 1.0)
    q, s = O.quantize8(w)
    q4, s4 = O.quantize4(w)
    n = O.lib().tqo_get_threads()
    try:
        O.set_threads(1)
        a8, a4 = O.q8_matmul(q, s, rows, cols, x), O.q4_matmul(q4, s4, rows, cols, x)
        O.set_threads(max(n, 3))
        b8, b4 = O.q8_matmul(q, s, rows, cols, x), O.q4_matmul(q4, s4, rows, cols, x)
    finally:
        O.set_threads(n)
    assert same_bits(a8, b8) and same_bits(a4, b4)


def test_synth_is_deterministic_and_normalish():
    a = O.synth((1 << 16,), 9, 1, 1.0)
    b = O.synth((1 << 16,), 9, 1, 1.0)
    c = O.synth((1 << 16,), 9, 2, 1.0)
    assert same_bits(a, b) and not same_bits(a, c)
    assert abs(a.mean()) < 0.02 and abs(a.std() - 1) < 0.02
    s2 = O.synth((1 << 16,), 9, 1, 0.02)
    assert np.allclose(s2, a * np.float32(0.02), rtol=1e-6)
