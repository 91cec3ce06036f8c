"""tensai_b200 — B200 (sm_100a) backend for tensai's weight-only quantized
inference path: int8 / int4 quantizers and dequantize-fused matvec/matmul,
served from libtensai_cuda.so (C ABI: include/tensai_cuda.h)."""
from .quant import (Matrix, NewMatrix, Q4Matrix, QMatrix, QuantizeMatrix, QuantizeMatrix4,  # noqa: F401
                    TensaiError)

__all__ = ["Matrix", "NewMatrix", "QMatrix", "Q4Matrix", "QuantizeMatrix", "QuantizeMatrix4", "TensaiError"]
