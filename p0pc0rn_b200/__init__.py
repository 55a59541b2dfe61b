"""p0pc0rn_b200: the B200 (sm_100a) implementation of p0pc0rn's 4-bit quantized matmul hot path.

The product is the C-ABI library libp0mm.so (include/p0mm.h; CUDA kernels under csrc/). This package loads it
and mirrors the reference's operator surface with the same argument objects and error messages:
  gemv / gemvM (engine/llm/lops.js, engine/llm/lops_spec.js) and gemm (engine/ops/gemm.js),
over Gpu buffers (engine/core/gpu.js), plus the quantisers packQ4 / packQ8 (engine/kcheck.js:22-53) on the device;
the decode-path operators around the GEMV (embed, normadd, qkrope, attnDec, argmax / argmaxM, dhead); and the
weight-pack store (p0pc0rn_b200.store, engine/core/store.js) that uploads pack shards into device buffers.
"""
from .gpu import Buffer, Gpu, P0Error, createGpu, version  # noqa: F401
from .ops import (argmax, argmaxM, attnDec, dequant_f16, dhead, embed, gemm, gemv, gemvM, gemvM_noalloc, normadd, pack_q4,  # noqa: F401
                  pack_q8, qkrope)
