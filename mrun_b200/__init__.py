"""mrun-b200: B200-native (sm_100a) kernels for mrun's quantized decode hot path.

The hot path lives in ``libmrun_b200.so`` (hand-written CUDA, C ABI in
``include/mrun_b200.h``). These modules mirror the reference's Python operator API so the
reference's engines can call them unchanged:

* ``dense_qstore_cuda``    — W8A16 projection, paired SwiGLU, RMSNorm, residual RMSNorm, head
* ``qstore_build``         — per-row int8 quantiser, dequantised row gathers, store writer
* ``qstore``               — on-disk QStore reader with the pinned prefetch ring
* ``w8a8``                 — W8A8 activation quantiser and int8 tensor-core GEMMs
* ``segmented_gqa_decode`` — paged decode / fused decode-step / prefill attention, RoPE + KV append
* ``paged_kv``             — the 16-token block-paged KV cache
* ``moe``                  — router, route compiler, grouped expert MLP, fixed-rank combine
* ``streaming``, ``page_policy`` — expert-page streaming and its residency policies
* ``expert_parallel``      — expert parallelism over NVLink peer memory or NCCL
* ``dense_engine``, ``moe_engine`` — the decode engines (prefill, CUDA-graph decode, greedy)
"""
from __future__ import annotations

__version__ = "0.1.0"
