"""p0pc0rn_b200: the B200 (sm_100a) implementation of p0pc0rn's 4-bit quantized matmul hot path.

The product is the C-ABI library libp0mm.so (include/p0mm.h; CUDA kernels under csrc/). This package loads it
and mirrors the reference's operator surface with the same argument objects and error messages:
  gemv / gemvM (engine/llm/lops.js, engine/llm/lops_spec.js) and gemm (engine/ops/gemm.js),
over Gpu buffers (engine/core/gpu.js), plus the q4g32a.t64 quantiser packQ4 (engine/kcheck.js:22-38) on the device.
"""
from .gpu import Buffer, Gpu, P0Error, createGpu, version  # noqa: F401
from .ops import argmax, argmaxM, dequant_f16, dhead, embed, gemm, gemv, gemvM, gemvM_noalloc, normadd, pack_q4, pack_q8  # noqa: F401
