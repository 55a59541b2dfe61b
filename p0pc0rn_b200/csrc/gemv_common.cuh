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
  int overlap;       // the weights are not written by work ahead on the stream: copies may start before pdl_wait()
  int q8;            // q8g64s.t64 weights (4224-byte records of 64 k; only the v5 kernels take them)
  uint32_t *err;
};

// Programmatic dependent launch. Every GEMV is launched so that it may start while the kernel ahead of it on the
// stream is still running; it calls pdl_wait() before it touches anything an earlier kernel may write (x, the norm /
// stat / pleg vectors, its outputs, the workspace), and pdl_trigger() as soon as its own loads are under way, so that
// the next call can start too. Without such a launch both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// a kernel launch with the programmatic-dependent-launch attribute (and a cluster shape when cluster > 1)
template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t s, uint32_t cluster, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  unsigned n = 0;
  at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[n].val.programmaticStreamSerializationAllowed = 1;
  n++;
  if (cluster > 1) {
    at[n].id = cudaLaunchAttributeClusterDimension;
    at[n].val.clusterDim.x = cluster;
    at[n].val.clusterDim.y = 1;
    at[n].val.clusterDim.z = 1;
    n++;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

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

// packed f32 pairs (a 64-bit register pair) and the two-lane fused multiply-add of sm_100 (fma.rn.f32x2)
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float &a, float &b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
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


// ---------------------------------------------------------------- bulk-copy fed kernels (v3, v4)
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(tc::smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
               : "memory");
}
// shared loads stay ordered against the barrier waits and slot refills around them (volatile); the arithmetic between
// them is free to interleave
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
  return v;
}
// four 8x8 b16 matrices of 8 consecutive 16-byte rows each (lane l addresses row l): lane (g, c) receives b32 element
// (g, c) of each, i.e. code word c of rows g, g+8, g+16, g+24 of the 32 rows starting at the lane-0 address
__device__ __forceinline__ void ldsm_x4(uint32_t a, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];" : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a)
               : "memory");
}

// One group of one record (64 rows): its code words (two ldmatrix.x4) and (s, mn) words, loaded before any math
struct Rec {
  uint32_t w[4][2], t[4][2];
};
__device__ __forceinline__ void rec_load(Rec &q, uint32_t rec, uint32_t lane_row16, uint32_t tail_off) {
  ldsm_x4(rec + lane_row16, q.w[0][0], q.w[0][1], q.w[1][0], q.w[1][1]);
  ldsm_x4(rec + 512u + lane_row16, q.w[2][0], q.w[2][1], q.w[3][0], q.w[3][1]);
#pragma unroll
  for (int r = 0; r < 4; r++) {
    q.t[r][0] = lds32(rec + tail_off + r * 64);
    q.t[r][1] = lds32(rec + tail_off + r * 64 + 32);
  }
}
// the code MMAs and acc += s * D + mn * sum(x) for the 4 row-blocks (xs0 / xs1: this lane's x sums, 0 where they do
// not apply)
// (MT == 1: the odd D columns, tokens 1 and 3 in the packed layout, are empty for every lane; their updates are skipped)
template <int MT, bool PACK>
__device__ __forceinline__ void rec_math(float (&acc)[4][4], const Rec &q, const uint4 bh, const uint4 bl, float xs0, float xs1) {
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const uint32_t w0 = q.w[r][0], w1 = q.w[r][1];
    const uint32_t w0s = __umulhi(w0, 1u << 24), w1s = __umulhi(w1, 1u << 24);   // >> 8 on the multiplier pipe
    const uint32_t A0[4] = {w0 & 0x000F000Fu, w1 & 0x000F000Fu, w0 & 0x00F000F0u, w1 & 0x00F000F0u};
    const uint32_t A1[4] = {w0s & 0x000F000Fu, w1s & 0x000F000Fu, w0s & 0x00F000F0u, w1s & 0x00F000F0u};
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    mma16816(d, A0, bh.x, bh.y);
    mma16816(d, A1, bh.z, bh.w);
    if (!PACK) {
      mma16816(d, A0, bl.x, bl.y);
      mma16816(d, A1, bl.z, bl.w);
    }
    const __half2 h0 = *reinterpret_cast<const __half2 *>(&q.t[r][0]), h1 = *reinterpret_cast<const __half2 *>(&q.t[r][1]);
    const float s0 = __low2float(h0), m0 = __high2float(h0), s1 = __low2float(h1), m1 = __high2float(h1);
    // the same fused multiply-adds, two lanes of f32 per instruction (fma.rn.f32x2: each lane rounds as fmaf does)
    if (MT == 1) {
      uint64_t a = pk2(acc[r][0], acc[r][2]);
      a = ffma2(pk2(m0, m1), pk2(xs0, xs0), a);
      a = ffma2(pk2(s0, s1), pk2(d[0], d[2]), a);
      upk2(a, acc[r][0], acc[r][2]);
    } else {
      const uint64_t xs = pk2(xs0, xs1);
      uint64_t a = pk2(acc[r][0], acc[r][1]), b = pk2(acc[r][2], acc[r][3]);
      a = ffma2(pk2(m0, m0), xs, a);
      b = ffma2(pk2(m1, m1), xs, b);
      a = ffma2(pk2(s0, s0), pk2(d[0], d[1]), a);
      b = ffma2(pk2(s1, s1), pk2(d[2], d[3]), b);
      upk2(a, acc[r][0], acc[r][1]);
      upk2(b, acc[r][2], acc[r][3]);
    }
  }
}


// ---------------------------------------------------------------- q8g64s.t64 records (v5)
// A q8 record (64 rows x 64 k): int8 codes at r*64 + k, fp16 scales at 4096 + 2r; the weight is q*s (kcheck.js:40-53).
// Code word c (bytes 4c..4c+3) of a row's 16-k chunk j feeds the m16n8k16 A fragment: its first two codes are MMA-k
// 2c, 2c+1 and its last two MMA-k 2c+8, 2c+9, so x is staged in that order. Codes become exact fp16 by an xor with
// 0x80, a byte permute against 0x64 ((1024 + q + 128) in fp16) and an fp16 subtract of 1152.
struct Rec8 {
  uint32_t w[4][4][2];   // [row block][chunk][rows g, g+8]
  uint32_t s[4];         // [row block]: fp16 scales of rows g (low half) and g + 8 (high half)
};
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ void rec8_load(Rec8 &q, uint32_t rec, uint32_t lane) {
  const uint32_t g = lane >> 2, rl = (lane & 7u) + 8u * ((lane >> 3) & 1u), jl = lane >> 4;
#pragma unroll
  for (int r = 0; r < 4; r++) {
#pragma unroll
    for (int jp = 0; jp < 2; jp++)
      ldsm_x4(rec + (16u * r + rl) * 64u + 16u * (2u * jp + jl), q.w[r][2 * jp][0], q.w[r][2 * jp][1], q.w[r][2 * jp + 1][0],
              q.w[r][2 * jp + 1][1]);
    q.s[r] = lds16(rec + 4096u + 2u * (16u * r + g)) | (lds16(rec + 4096u + 2u * (16u * r + g + 8u)) << 16);
  }
}
__device__ __forceinline__ uint32_t q8_pair(uint32_t u, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(u), "r"(0x64646464u), "r"(sel));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(d), "r"(0x64806480u));
  return d;
}
// acc[r] += s_row * sum_k q x over the record; b[j] = this lane's staged x of chunk j (hi in .x/.y, lo in .z/.w)
template <int MT, bool PACK>
__device__ __forceinline__ void rec8_math(float (&acc)[4][4], const Rec8 &q, const uint4 (&b)[4], uint32_t bsel) {
#pragma unroll
  for (int r = 0; r < 4; r++) {
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint32_t u0 = q.w[r][j][0] ^ 0x80808080u, u1 = q.w[r][j][1] ^ 0x80808080u;
      const uint32_t A[4] = {q8_pair(u0, 0x4140u), q8_pair(u1, 0x4140u), q8_pair(u0, 0x4342u), q8_pair(u1, 0x4342u)};
      if (PACK) {
        mma16816(d, A, bsel ? b[j].z : b[j].x, bsel ? b[j].w : b[j].y);
      } else {
        mma16816(d, A, b[j].x, b[j].y);
        mma16816(d, A, b[j].z, b[j].w);
      }
    }
    const __half2 sh = *reinterpret_cast<const __half2 *>(&q.s[r]);
    const float s0 = __low2float(sh), s1 = __high2float(sh);
    acc[r][0] = fmaf(s0, d[0], acc[r][0]);
    acc[r][2] = fmaf(s1, d[2], acc[r][2]);
    if (MT > 1) {
      acc[r][1] = fmaf(s0, d[1], acc[r][1]);
      acc[r][3] = fmaf(s1, d[3], acc[r][3]);
    }
  }
}

// the v3 (bulk-copy fed, whole tiles per warp) kernels, in gemv_v3.cu
bool v3_fits(uint32_t M, uint32_t K, uint32_t nsplit, uint32_t ntile, int sms);
bool v3_split_fits(uint32_t M, uint32_t K, uint32_t nsplit, uint32_t ntile, int sms, bool pair);
cudaError_t launch_v3(const GemvParams &p, int sms, cudaStream_t s);

// the v4 (stream-K) kernels, in gemv_v4.cu
struct V4Plan {
  uint32_t R;       // records of the call: ntile * Gt
  uint32_t G;       // groups per tile = K / 32
  uint32_t Gt;      // records per tile in the stream: G, or 2G for geglu (the gate tile's G, then the up tile's G)
  uint32_t Gs;      // records per k-split (geglu: Gt, one unit per tile)
  uint32_t nsplit;
  uint32_t ntile;   // 64-row tiles of the output (geglu: the up tiles follow at tile + ntile)
  uint32_t NW;      // warps of the grid (a multiple of 16, <= R)
  uint32_t nslot;   // ring slots per warp
  uint32_t *cnt;    // workspace: [ntile * nsplit] arrival counters, zero between calls
  float *part;      // workspace: [ntile * nsplit + NW][halves][M][64] partial sums of shared units (geglu: 2 halves)
};
// false when the call does not fit v4 (weight columns < K, staged x too large, fewer records than warps);
// else fills the plan (without the workspace pointers) and the scratch bytes its partial sums need
bool v4_plan(const GemvParams &p, uint32_t nsplit, int sms, V4Plan *pl, size_t *scratch_bytes);
// bytes of arrival counters the plan needs (one u32 per unit)
size_t v4_counter_bytes(const V4Plan &pl);
cudaError_t launch_v4(const GemvParams &p, const V4Plan &pl, cudaStream_t s);
// the v5 (cluster) kernels, in gemv_v5.cu
struct V5Plan {
  uint32_t CS;      // CTAs per unit (thread-block cluster size, 1..8)
  uint32_t nsplit, Gs, G, ntile;
  uint32_t pair;    // geglu: ranks < CS/2 read the gate tile, the others the up tile
  uint32_t nmax;    // records per CTA at most
  uint32_t units;   // output units: tiles x k-splits (geglu: tiles)
};
// false when the call does not fit v5 (too many tiles for it to lead, weight columns < K, staged x or records too
// large for shared memory); else fills the plan
bool v5_plan(const GemvParams &p, uint32_t nsplit, int sms, V5Plan *pl);
cudaError_t launch_v5(const GemvParams &p, const V5Plan &pl, cudaStream_t s);

// the device address of the allocation-free entry point's fixed scratch (P0_NOALLOC_SCRATCH_BYTES) on the current
// device; looked up on a device's first call
cudaError_t v4_noalloc_scratch(uint8_t **out);

// the kernel choice and launch of one checked gemv / gemvM call (gemv.cu)
p0_status gemv_dispatch(p0_ctx *c, const char *op, const GemvParams &p, uint32_t nsplit, bool noalloc);

// the byte ranges a recorded call reads (x, norm, stat, ev) and writes (y, mx); {0, 0} = none
struct ChainRange {
  uintptr_t lo, hi;
};
struct ChainIO {
  ChainRange in[4], out[2];
};
// keeps a checked call in the chain being recorded on the context (chain.cu)
p0_status chain_record(p0_ctx *c, const char *op, const GemvParams &p, uint32_t nsplit, const ChainIO &io);

}  // namespace p0gemv
