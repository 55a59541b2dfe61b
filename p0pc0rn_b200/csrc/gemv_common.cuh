// gemv_common.cuh -- what the GEMV kernels share: the launch parameters (the reference's uniform struct for
// lgemv / lgemvM), the prologue x'(m, k) of lops.js:49-53 / lops_spec.js:60-64, GELU in the reference's order, and
// the mma.sync / fp16 helpers of the tensor-core variants.
#pragma once
#include <cuda_fp16.h>

#include "internal.h"
#include "tc.cuh"

namespace p0gemv {


constexpr int kThreads = 256;   // 8 warps; a CTA = one 64-row tile x one k-split
constexpr int kWarps = kThreads / 32;

struct GemvParams {
  const float *X;    // x rows (f32)
  const uint8_t *W;  // the weight view's first byte (tile 0, group 0)
  float *Y;
  const float *NW;   // rms weights
  const float *EV;   // pleg per-layer vector
  const float *ST;   // rms rstd slots (gemv: the buffer lops.js:125 binds as MX)
  float *MX;         // softcap per-tile {max, idx}
  uint32_t M, N, K, wG, kPer, ldy, ldm, ldx, rowB, nOff, statOff, statLd, evOff, evLd, ldp, nsrc, ntile, xc;
  float cap;
  int pro, epi;
  uint32_t *err;
};

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg_u32(const void *p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// GELU as lops.js:26 writes it, in source order (no contraction)
__device__ __forceinline__ float gelu_l(float v) {
  float v3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
  float u = __fmul_rn(0.7978845608028654f, __fadd_rn(v, v3));
  u = fminf(15.0f, fmaxf(-15.0f, u));
  return __fmul_rn(__fmul_rn(v, 0.5f), __fadd_rn(1.0f, tanhf(u)));
}

// the prologue value x'(m, k) (lops.js:49-53 / lops_spec.js:60-64)
__device__ __forceinline__ float prologue(const GemvParams &p, uint32_t m, uint32_t k) {
  if (p.pro == P0_PRO_RAW) return p.X[m * p.ldx + p.rowB + k];
  if (p.pro == P0_PRO_RMS)
    return __fmul_rn(__fmul_rn(p.X[m * p.ldx + p.rowB + k], p.ST[p.statOff + m * p.statLd]), p.NW[p.nOff + k]);
  float s = 0.0f;
  for (uint32_t j = 0; j < p.nsrc; j++) s = __fadd_rn(s, p.X[j * p.ldp + m * p.ldx + k]);
  if (p.pro == P0_PRO_SUM) return s;
  return __fmul_rn(gelu_l(s), p.EV[p.evOff + m * p.evLd + k]);
}

// a pure function of its operands (not volatile): the scheduler may interleave independent MMAs with other work
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}


// the v3 (bulk-copy fed) kernels, in gemv_v3.cu
bool v3_fits(uint32_t M, uint32_t K, uint32_t nsplit, uint32_t ntile, int sms);
cudaError_t launch_v3(const GemvParams &p, int sms, cudaStream_t s);

}  // namespace p0gemv
