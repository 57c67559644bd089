"""mrun-b200: B200-native (sm_100a) kernels for mrun's quantized decode hot path.

The hot path lives in ``libmrun_b200.so`` (hand-written CUDA, C ABI in
``include/mrun_b200.h``). These modules mirror the reference's Python operator API so the
reference's engines can call them unchanged:

* ``dense_qstore_cuda`` — W8A16 projection, paired SwiGLU, RMSNorm, residual RMSNorm, head
* ``qstore_build``      — per-row int8 quantiser and dequantised row gathers
"""
from __future__ import annotations

__version__ = "0.1.0"
