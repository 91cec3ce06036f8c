"""Independent numpy restatement of tensai's quantizers, used only to cross-check
the C oracle (oracle/tq_oracle.c). Every step is a float32 numpy operation, so
each rounds once, as the Go code's float32 arithmetic does:

  QuantizeMatrix   quant.go:37-72
  QuantizeMatrix4  quant4.go:28-89
"""
import numpy as np

F = np.float32


def _round_away_trunc(v: np.ndarray) -> np.ndarray:
    # v >= 0 ? v + 0.5 : v - 0.5, then truncation toward zero (Go int8()/int()).
    v = np.where(v >= 0, v + F(0.5), v - F(0.5)).astype(np.float32)
    return np.trunc(v).astype(np.int64)


def quantize8(w: np.ndarray):
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    maxabs = np.max(np.abs(w), axis=0) if rows else np.zeros(cols, np.float32)
    s = (maxabs / F(127)).astype(np.float32)
    q = np.zeros((rows, cols), dtype=np.int8)
    nz = s != 0
    with np.errstate(divide="ignore"):
        inv = np.where(nz, F(1) / np.where(nz, s, F(1)), F(0)).astype(np.float32)
    v = (w * inv[None, :]).astype(np.float32)
    codes = _round_away_trunc(v)
    q[:, nz] = codes[:, nz].astype(np.int8)
    out = np.zeros(rows * cols + 16, dtype=np.int8)
    out[: rows * cols] = q.reshape(-1)
    return out, s


def quantize4(w: np.ndarray, group: int = 64):
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    assert cols % 2 == 0
    half = cols // 2
    groups = (rows + group - 1) // group
    scale = np.zeros((groups, cols), dtype=np.float32)
    nib = np.zeros((rows, cols), dtype=np.int64)
    for g in range(groups):
        lo, hi = g * group, min((g + 1) * group, rows)
        blk = w[lo:hi]
        s = (np.max(np.abs(blk), axis=0) / F(7)).astype(np.float32)
        scale[g] = s
        nz = s != 0
        inv = np.where(nz, F(1) / np.where(nz, s, F(1)), F(0)).astype(np.float32)
        n = np.clip(_round_away_trunc((blk * inv[None, :]).astype(np.float32)), -8, 7)
        nib[lo:hi] = np.where(nz[None, :], n + 8, 8)
    packed = (nib[:, :half] | (nib[:, half:] << 4)).astype(np.uint8)
    out = np.zeros(rows * half + 16, dtype=np.uint8)
    out[: rows * half] = packed.reshape(-1)
    return out, scale.reshape(-1)
