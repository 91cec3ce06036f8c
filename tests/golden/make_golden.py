"""Generates tests/golden/quant_golden.npz: small quantization fixtures.

Inputs are constructed to hit the quantizers' edge cases (exact half-way
values k*s + s/2 on both signs, all-zero columns, +-maxAbs, a single row, a
partial final int4 group, two columns) plus seeded synthetic matrices at the
reference tests' small shapes (quant_test.go:11-16, quant4_test.go:11-16).

Expected codes and scales come from tests/refquant.py (a numpy float32
restatement of quant.go:37-72 / quant4.go:28-89); the script refuses to
write unless the C oracle produces the same bytes. Expected matvec outputs
are float64 recomputations over those codes (quant_test.go:30-39,
quant4_test.go:31-49).

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from oracle import oracle as O  # noqa: E402
import refquant  # noqa: E402


def halfway_matrix(rows, cols, rng, levels):
    """Columns whose values sit exactly on k*s + s/2 (s a power of two)."""
    w = np.zeros((rows, cols), dtype=np.float32)
    for j in range(cols):
        s = np.float32(2.0 ** rng.integers(-8, 2))
        k = rng.integers(-levels, levels, size=rows)
        w[:, j] = (k.astype(np.float32) + np.float32(0.5)) * s
        w[rng.integers(0, rows), j] = np.float32(levels) * s  # pin maxAbs so s is exact
    return w


def cases():
    rng = np.random.default_rng(2024)
    out = []
    out.append(("hand8", 8, np.array([[127, -63.5], [2.5, 1.0]], dtype=np.float32)))
    out.append(("hand4", 4, np.array([[7, -3.5], [-2.5, 1.75]], dtype=np.float32)))
    z = O.synth((5, 6), 7, 1, 0.3)
    z[:, 2] = 0
    out.append(("zerocol8", 8, z.copy()))
    out.append(("zerocol4", 4, z.copy()))
    out.append(("halfway8", 8, halfway_matrix(37, 24, rng, 127)))
    out.append(("halfway4", 4, halfway_matrix(130, 24, rng, 7)))
    out.append(("negmax8", 8, -np.abs(O.synth((9, 16), 9, 2, 1.0))))
    out.append(("row1_8", 8, O.synth((1, 9), 31, 3, 0.5)))
    out.append(("row1_4", 4, O.synth((1, 2), 41, 4, 0.5)))
    for r, c in [(16, 16), (7, 13)]:
        out.append((f"ref8_{r}x{c}", 8, O.synth((r, c), 31, r * 100000 + c, O.glorot_sigma(r, c))))
    for r, c in [(64, 32), (33, 10)]:
        out.append((f"ref4_{r}x{c}", 4, O.synth((r, c), 41, r * 100000 + c, O.glorot_sigma(r, c))))
    return out


def main():
    arrays = {}
    names = []
    for name, bits, w in cases():
        rows, cols = w.shape
        if bits == 8:
            q, s = refquant.quantize8(w)
            qo, so = O.quantize8(w)
        else:
            q, s = refquant.quantize4(w)
            qo, so = O.quantize4(w)
        if not (np.array_equal(q, qo) and np.array_equal(s.view(np.uint32), so.view(np.uint32))):
            raise SystemExit(f"{name}: C oracle disagrees with the numpy restatement; not writing fixtures")
        x = O.synth((rows,), 5, 77, 1.0)
        want = (O.q8_exact if bits == 8 else O.q4_exact)(q, s, rows, cols, x)[0]
        arrays[f"{name}.w"] = w
        arrays[f"{name}.q"] = q
        arrays[f"{name}.scale"] = s
        arrays[f"{name}.x"] = x
        arrays[f"{name}.want"] = want
        arrays[f"{name}.bits"] = np.array(bits)
        names.append(name)
    arrays["names"] = np.array(names)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "quant_golden.npz")
    np.savez_compressed(path, **arrays)
    print(f"wrote {path}: {len(names)} cases")


if __name__ == "__main__":
    main()
