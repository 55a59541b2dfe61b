// lops.cu -- the decode-path operators on either side of the GEMV: the token embedding gather (embed, engine/llm/
// lops.js:323-365), the residual add + RMS statistics (normadd, lops.js:143-180), the argmax over the head's per-tile
// maxima (argmax / argmaxM, lops.js:416-436, lops_spec.js:326-348) and the drafter's head over selected clusters
// (dhead, lops_spec.js:428-482), the decode step's q/k norm + RoPE + KV-cache write (qkrope, lops.js:183-233) and
// its split-key attention (attnDec + combine, lops.js:236-321). Small kernels: one CTA per output row, tile, head or
// key chunk, coalesced loads, warp-shuffle reductions; only attnDec uses scratch (the caller's `part` buffer).
#include <cuda_fp16.h>

#include "internal.h"

namespace {

constexpr int kT = 256;   // threads per CTA

// Programmatic dependent launch: every operator kernel is launched so that it may start while the kernel ahead of it is
// still running; it waits for that kernel (griddepcontrol.wait: all prerequisite grids complete, their writes visible)
// before it reads anything, then lets the kernel after it launch at once. Without such a launch both are no-ops.
__device__ __forceinline__ void dep_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float h2f(uint32_t h16) { return __half2float(__ushort_as_half((unsigned short)(h16 & 0xffffu))); }

// (value, index) pairs: the larger value wins, ties go to the lower index; NaN never wins
__device__ __forceinline__ void better(float &bv, uint32_t &bi, float v, uint32_t i) {
  if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}
__device__ __forceinline__ void warp_best(float &bv, uint32_t &bi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) better(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
}
// CTA sum of one float per thread (every thread gets the total)
__device__ __forceinline__ float cta_sum(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < kT / 32; i++) t += red[i];
  return t;
}

// ---------------------------------------------------------------- argmaxM: one CTA per row of n (max, bitcast index) pairs
__global__ void __launch_bounds__(kT) argmax_kernel(const float2 *__restrict__ MX, uint32_t n, uint32_t *__restrict__ out) {
  dep_enter();
  __shared__ float rv[kT / 32];
  __shared__ uint32_t ri[kT / 32];
  const uint32_t m = blockIdx.x;
  const float2 *row = MX + (size_t)m * n;
  float bv = -3.4e38f;
  uint32_t bi = 0xffffffffu;
  for (uint32_t i = threadIdx.x; i < n; i += kT) {
    const float2 e = row[i];
    better(bv, bi, e.x, __float_as_uint(e.y));
  }
  warp_best(bv, bi);
  if ((threadIdx.x & 31) == 0) { rv[threadIdx.x >> 5] = bv; ri[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kT / 32; w++) better(bv, bi, rv[w], ri[w]);
    out[2 * m] = bi;
    out[2 * m + 1] = __float_as_uint(bv);
  }
}

// ---------------------------------------------------------------- embed: one CTA per token; a thread per 8 (q4) / 4 (q8) k
// q4: v = (f32(q) * s + mn) * scale, q8: v = f32(q) * s * scale, each operation rounded as written (the oracle's order);
// an id beyond the table reads as a row of zeros (the WGSL's robust buffer access gives no defined value there)
template <bool Q8>
__global__ void __launch_bounds__(kT) embed_kernel(const uint8_t *__restrict__ W, uint32_t V, const uint32_t *__restrict__ ids,
                                                   uint32_t K, uint32_t wG, float scale, float eps, float *__restrict__ X,
                                                   uint32_t rowOut, float *__restrict__ ST, uint32_t statOff) {
  dep_enter();
  __shared__ float red[kT / 32];
  const uint32_t m = blockIdx.x, id = ids[m];
  const bool in = id < V;
  const uint32_t tile = in ? id >> 6 : 0u, r = id & 63u;
  float *x = X + (size_t)(rowOut + m) * K;
  float s2 = 0.0f;
  if (!Q8) {
    for (uint32_t u = threadIdx.x; u < K / 8; u += kT) {   // group u / 4, code word u % 4 (k = 8u .. 8u + 7)
      const uint8_t *rec = W + ((size_t)tile * wG + (u >> 2)) * 1280u;
      float v[8];
      if (in) {
        const uint32_t q = *reinterpret_cast<const uint32_t *>(rec + r * 16u + (u & 3u) * 4u);
        const uint32_t sm = *reinterpret_cast<const uint32_t *>(rec + 1024u + r * 4u);
        const float s = h2f(sm), mn = h2f(sm >> 16);
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = __fmul_rn(__fadd_rn(__fmul_rn((float)((q >> (4 * j)) & 15u), s), mn), scale);
      } else {
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = 0.0f;
      }
      *reinterpret_cast<float4 *>(x + 8u * u) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4 *>(x + 8u * u + 4u) = make_float4(v[4], v[5], v[6], v[7]);
#pragma unroll
      for (int j = 0; j < 8; j++) s2 = fmaf(v[j], v[j], s2);
    }
  } else {
    for (uint32_t u = threadIdx.x; u < K / 4; u += kT) {   // group u / 16, code word u % 16 (k = 4u .. 4u + 3)
      const uint8_t *rec = W + ((size_t)tile * wG + (u >> 4)) * 4224u;
      float v[4];
      if (in) {
        const uint32_t q = *reinterpret_cast<const uint32_t *>(rec + r * 64u + (u & 15u) * 4u);
        const float s = h2f(*reinterpret_cast<const uint16_t *>(rec + 4096u + r * 2u));
#pragma unroll
        for (int j = 0; j < 4; j++) v[j] = __fmul_rn(__fmul_rn((float)(int8_t)((q >> (8 * j)) & 255u), s), scale);
      } else {
#pragma unroll
        for (int j = 0; j < 4; j++) v[j] = 0.0f;
      }
      *reinterpret_cast<float4 *>(x + 4u * u) = make_float4(v[0], v[1], v[2], v[3]);
#pragma unroll
      for (int j = 0; j < 4; j++) s2 = fmaf(v[j], v[j], s2);
    }
  }
  const float tot = cta_sum(s2, red);
  if (threadIdx.x == 0) ST[statOff + m] = rsqrtf(__fadd_rn(__fdiv_rn(tot, (float)K), eps));
}

// ---------------------------------------------------------------- normadd: one CTA per row of D
// tv = sum over the nsrc partial rows (in order); rs = rsqrt(sum tv^2 / D + eps); mode 0: x = (x + tv * rs * w) * scale,
// mode 1: x = tv; ST = rsqrt(sum x^2 / D + eps). tv is kept in shared memory between the two passes.
__global__ void __launch_bounds__(kT) normadd_kernel(const float *__restrict__ T, uint32_t nsrc, uint64_t ldp, const float *__restrict__ Wn,
                                                     float *__restrict__ X, float *__restrict__ ST, uint32_t statOff, uint32_t D,
                                                     uint32_t mode, float eps, float scale, bool pre) {
  dep_enter();
  extern __shared__ float tv[];   // [D] summed partials; with pre, then [D] x and [D] w read in the same pass
  __shared__ float red[kT / 32];
  const uint32_t m = blockIdx.x;
  const size_t xb = (size_t)m * D;
  float *xv = tv + D, *wv = tv + 2 * (size_t)D;
  float s = 0.0f;
#pragma unroll 8
  for (uint32_t i = threadIdx.x; i < D; i += kT) {
    float v = 0.0f;
    for (uint32_t j = 0; j < nsrc; j++) v = __fadd_rn(v, T[j * ldp + xb + i]);
    if (pre) {   // x and w do not depend on the sum: their loads fly with the partials'
      xv[i] = X[xb + i];
      if (mode == 0) wv[i] = Wn[i];
    }
    tv[i] = v;
    s = fmaf(v, v, s);
  }
  const float rs = rsqrtf(__fadd_rn(__fdiv_rn(cta_sum(s, red), (float)D), eps));
  float s2 = 0.0f;
#pragma unroll 8
  for (uint32_t i = threadIdx.x; i < D; i += kT) {
    float x = pre ? xv[i] : X[xb + i];
    if (mode == 0) x = __fmul_rn(__fadd_rn(x, __fmul_rn(__fmul_rn(tv[i], rs), pre ? wv[i] : Wn[i])), scale);
    else x = tv[i];
    X[xb + i] = x;
    s2 = fmaf(x, x, s2);
  }
  const float tot = cta_sum(s2, red);
  if (threadIdx.x == 0) ST[statOff + m] = rsqrtf(__fadd_rn(__fdiv_rn(tot, (float)D), eps));
}

// ---------------------------------------------------------------- dhead: one CTA per selected tile, thread = (row, k quarter)
// Row r's dot runs in 4 lanes w (q4: k = 32g + 8w..+7, acc += s * (q . x) + mn * sum(x); q8: k = 64g + 16w..+15, acc +=
// s * (q . x)), each operation rounded in the oracle's order; the 4 lane sums are added in order, then the tile's max
// row (lowest row on ties) by shuffles and one shared-memory step. A tile beyond the head writes (-3.4e38, 0xffffffff),
// which never wins the argmax.
__device__ __forceinline__ float dot4r(const float *a, const float *b) {
  return __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(a[0], b[0]), __fmul_rn(a[1], b[1])), __fmul_rn(a[2], b[2])), __fmul_rn(a[3], b[3]));
}
template <bool Q8>
__global__ void __launch_bounds__(kT) dhead_kernel(const float *__restrict__ X, const uint8_t *__restrict__ W, uint32_t ntile,
                                                   const float *__restrict__ ST, const float *__restrict__ NW, const uint32_t *__restrict__ SEL,
                                                   uint32_t K, uint32_t wG, uint32_t tPer, float *__restrict__ MX) {
  dep_enter();
  __shared__ float xs[512];
  __shared__ float rv[kT / 32];
  __shared__ uint32_t ri[kT / 32];
  const uint32_t wt = blockIdx.x, tile = SEL[wt / tPer] * tPer + (wt % tPer);
  const float rs = ST[0];
  for (uint32_t k = threadIdx.x; k < K; k += kT) xs[k] = __fmul_rn(__fmul_rn(X[k], rs), NW[k]);
  __syncthreads();
  const uint32_t r = threadIdx.x >> 2, w = threadIdx.x & 3u;
  float acc = 0.0f;
  if (tile < ntile) {
    for (uint32_t g = 0; g < wG; g++) {
      if (Q8) {
        const uint8_t *rec = W + ((size_t)tile * wG + g) * 4224u;
        const float sc = h2f(*reinterpret_cast<const uint16_t *>(rec + 4096u + r * 2u));
        const uint4 q4 = *reinterpret_cast<const uint4 *>(rec + r * 64u + w * 16u);
        const uint32_t qw[4] = {q4.x, q4.y, q4.z, q4.w};
        float d = 0.0f;
#pragma unroll
        for (int u = 0; u < 4; u++) {
          float qv[4];
#pragma unroll
          for (int b = 0; b < 4; b++) qv[b] = (float)(int8_t)((qw[u] >> (8 * b)) & 255u);
          d = __fadd_rn(d, dot4r(qv, xs + g * 64u + w * 16u + u * 4u));
        }
        acc = __fadd_rn(acc, __fmul_rn(sc, d));
      } else {
        const uint8_t *rec = W + ((size_t)tile * wG + g) * 1280u;
        const uint32_t q = *reinterpret_cast<const uint32_t *>(rec + r * 16u + w * 4u);
        const uint32_t sm = *reinterpret_cast<const uint32_t *>(rec + 1024u + r * 4u);
        float qa[4], qb[4];
#pragma unroll
        for (int b = 0; b < 4; b++) { qa[b] = (float)((q >> (4 * b)) & 15u); qb[b] = (float)((q >> (16 + 4 * b)) & 15u); }
        const float *xv = xs + g * 32u + w * 8u;
        const float one[4] = {1.0f, 1.0f, 1.0f, 1.0f};
        const float dq = __fadd_rn(dot4r(qa, xv), dot4r(qb, xv + 4)), dx = __fadd_rn(dot4r(xv, one), dot4r(xv + 4, one));
        acc = __fadd_rn(__fadd_rn(acc, __fmul_rn(h2f(sm), dq)), __fmul_rn(h2f(sm >> 16), dx));
      }
    }
  }
  // the row total: lanes w = 0..3 of the row are consecutive threads; lane 0 adds them in order
  const float a1 = __shfl_down_sync(0xffffffffu, acc, 1), a2 = __shfl_down_sync(0xffffffffu, acc, 2), a3 = __shfl_down_sync(0xffffffffu, acc, 3);
  float bv = -3.4e38f;
  uint32_t bi = 0xffffffffu;
  if (w == 0 && tile < ntile) {
    bv = __fadd_rn(__fadd_rn(__fadd_rn(acc, a1), a2), a3);
    bi = tile * 64u + r;
  }
  warp_best(bv, bi);
  if ((threadIdx.x & 31) == 0) { rv[threadIdx.x >> 5] = bv; ri[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < kT / 32; i++) better(bv, bi, rv[i], ri[i]);
    MX[wt * 2] = bv;
    MX[wt * 2 + 1] = __uint_as_float(bi);
  }
}


// ---------------------------------------------------------------- qkrope (decode): one CTA per head of [q | k | v]
// the head's row = the sum of the split partials (in order), kept in shared memory; rs = rsqrt(mean square + eps);
// v heads -> f16(x * rs) into the value cache row; q / k heads: RMS-normed with their weights, rotate-half RoPE on the
// first npairs pairs (d, d + D/2), q -> f32 Q, k -> f16 key cache row (head-major [nkv][kvLen][D])
__global__ void __launch_bounds__(kT) qkrope_kernel(const float *__restrict__ S, uint32_t nsrc, uint64_t ldp, const float *__restrict__ NW,
                                                    const float *__restrict__ RP, float *__restrict__ Q, __half *__restrict__ KC,
                                                    __half *__restrict__ VC, uint32_t D, uint32_t nq, uint32_t nkv, uint32_t pos, float eps,
                                                    uint32_t qwOff, uint32_t kwOff, uint32_t npairs, uint32_t ropeOff, uint32_t kvRow,
                                                    uint32_t kvLen) {
  dep_enter();
  extern __shared__ float hv[];
  __shared__ float red[kT / 32];
  const uint32_t h = blockIdx.x, half = D / 2;
  const size_t base = (size_t)h * D;
  float s = 0.0f;
  for (uint32_t i = threadIdx.x; i < D; i += kT) {
    float v = 0.0f;
    for (uint32_t j = 0; j < nsrc; j++) v = __fadd_rn(v, S[j * ldp + base + i]);
    hv[i] = v;
    s = fmaf(v, v, s);
  }
  const float rs = rsqrtf(__fadd_rn(__fdiv_rn(cta_sum(s, red), (float)D), eps));
  const bool isV = h >= nq + nkv;
  const uint32_t kvh = isV ? h - nq - nkv : h - nq;
  const size_t cb = ((size_t)kvh * kvLen + kvRow) * D;
  if (isV) {
    for (uint32_t i = threadIdx.x; i < D; i += kT) VC[cb + i] = __float2half_rn(__fmul_rn(hv[i], rs));
    return;
  }
  const float *w = NW + (h >= nq ? kwOff : qwOff);
  for (uint32_t d = threadIdx.x; d < half; d += kT) {
    const float a = __fmul_rn(__fmul_rn(hv[d], rs), w[d]), b = __fmul_rn(__fmul_rn(hv[d + half], rs), w[d + half]);
    float c = 1.0f, sn = 0.0f;
    if (d < npairs) {
      const size_t rb = ropeOff + ((size_t)pos * npairs + d) * 2;
      c = RP[rb];
      sn = RP[rb + 1];
    }
    const float lo = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn)), hi = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, sn));
    if (h < nq) {
      Q[base + d] = lo;
      Q[base + d + half] = hi;
    } else {
      KC[cb + d] = __float2half_rn(lo);
      KC[cb + d + half] = __float2half_rn(hi);
    }
  }
}

// ---------------------------------------------------------------- attnDec (decode attention, split over 64-key chunks)
// One CTA per chunk. Scores: warp w takes keys 8w..8w+7 of the chunk at once; a lane holds 4 dims in each 128-dim
// step of those keys' rows (DV steps, coalesced 8-byte loads) and, per query head of the key's KV group, dots them
// with q from shared memory (q is read once per 8 keys), then a butterfly gives each key's score. Per head: m = max,
// p = exp(s - m), l = sum p. P.V: a thread owns a pair of dims, every query head's accumulator in registers, each V
// row read once per CTA. The chunk writes [nh] m | [nh] l | [nh][D] acc to the scratch; the combine merges chunks.
template <int DV>
__global__ void __launch_bounds__(kT) attn_chunk_kernel(const float *__restrict__ Q, const __half *__restrict__ KC,
                                                        const __half *__restrict__ VC, float *__restrict__ PT, uint32_t D, uint32_t nh,
                                                        uint32_t nkv, uint32_t kvLen, uint32_t kStart, uint32_t kEnd, uint32_t ring) {
  dep_enter();
  extern __shared__ float sm[];
  float *qs = sm, *sc = sm + (size_t)nh * D;   // q [nh][D] | scores [nh][64]
  __shared__ float mh[8];
  const uint32_t c = blockIdx.x, j0 = kStart + c * 64u, nk = kEnd - j0 < 64u ? kEnd - j0 : 64u;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, hpg = nh / nkv;
  for (uint32_t i = threadIdx.x; i < nh * D; i += kT) qs[i] = Q[i];
  for (uint32_t i = threadIdx.x; i < nh * 64u; i += kT) sc[i] = -3.0e38f;
  __syncthreads();
  for (uint32_t g = 0; g < nkv; g++) {
    float kf[8][DV * 4];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const uint32_t j = warp * 8u + i;
      const uint32_t row = ring ? (j0 + j) % ring : j0 + j;
      const __half *kr = KC + ((size_t)g * kvLen + (j < nk ? row : 0u)) * D;
#pragma unroll
      for (int v = 0; v < DV; v++) {
        const uint2 u = j < nk ? *reinterpret_cast<const uint2 *>(kr + 128u * v + 4u * lane) : make_uint2(0u, 0u);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x)), b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
        kf[i][4 * v] = a.x; kf[i][4 * v + 1] = a.y; kf[i][4 * v + 2] = b.x; kf[i][4 * v + 3] = b.y;
      }
    }
    for (uint32_t hh = g * hpg; hh < (g + 1) * hpg; hh++) {
      float qv[DV * 4];
#pragma unroll
      for (int v = 0; v < DV; v++) {
        const float4 q4 = *reinterpret_cast<const float4 *>(qs + (size_t)hh * D + 128u * v + 4u * lane);
        qv[4 * v] = q4.x; qv[4 * v + 1] = q4.y; qv[4 * v + 2] = q4.z; qv[4 * v + 3] = q4.w;
      }
      float part[8];
#pragma unroll
      for (int i = 0; i < 8; i++) {
        float t = 0.0f;
#pragma unroll
        for (int e = 0; e < DV * 4; e++) t = fmaf(kf[i][e], qv[e], t);
        part[i] = t;
      }
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part[i] += __shfl_xor_sync(0xffffffffu, part[i], o);
      if (lane < 8u && warp * 8u + lane < nk) {
        float v = part[0];
#pragma unroll
        for (int i = 1; i < 8; i++) v = lane == (uint32_t)i ? part[i] : v;
        sc[hh * 64u + warp * 8u + lane] = v;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < nh) {
    float m = -3.0e38f;
    for (uint32_t k = 0; k < nk; k++) m = fmaxf(m, sc[threadIdx.x * 64u + k]);
    mh[threadIdx.x] = m;
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < nh * 64u; i += kT) {
    const uint32_t hh = i >> 6, k = i & 63u;
    sc[i] = k < nk ? expf(sc[i] - mh[hh]) : 0.0f;
  }
  __syncthreads();
  const size_t pb = (size_t)c * nh * (2u + D);
  if (threadIdx.x < nh) {
    float l = 0.0f;
    for (uint32_t k = 0; k < nk; k++) l += sc[threadIdx.x * 64u + k];
    PT[pb + threadIdx.x] = mh[threadIdx.x];
    PT[pb + nh + threadIdx.x] = l;
  }
  // P.V: the chunk's V rows of one KV head are first staged in shared memory by every thread at once (16-byte loads, all
  // in flight together), then a thread per dim pair walks the keys from shared memory
  __half *vs = reinterpret_cast<__half *>(sc + (size_t)nh * 64u);   // [64][D]
  float2 acc[8];
#pragma unroll
  for (int hh = 0; hh < 8; hh++) acc[hh] = make_float2(0.0f, 0.0f);
  const uint32_t dpa = threadIdx.x;   // this thread's dim pair (D / 2 <= kT)
  for (uint32_t g = 0; g < nkv; g++) {
    __syncthreads();   // the previous head's rows are no longer read
    for (uint32_t i = threadIdx.x; i < nk * (D / 8u); i += kT) {
      const uint32_t k = i / (D / 8u), e = i - k * (D / 8u);
      const uint32_t row = ring ? (j0 + k) % ring : j0 + k;
      reinterpret_cast<uint4 *>(vs)[(size_t)k * (D / 8u) + e] = *reinterpret_cast<const uint4 *>(VC + ((size_t)g * kvLen + row) * D + 8u * e);
    }
    __syncthreads();
    if (dpa < D / 2) {
      for (uint32_t k = 0; k < nk; k++) {
        const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(vs + (size_t)k * D + 2u * dpa));
#pragma unroll
        for (int hh = 0; hh < 8; hh++)
          if ((uint32_t)hh >= g * hpg && (uint32_t)hh < (g + 1) * hpg) {
            const float p = sc[hh * 64u + k];
            acc[hh].x = fmaf(p, v.x, acc[hh].x);
            acc[hh].y = fmaf(p, v.y, acc[hh].y);
          }
      }
    }
  }
  if (dpa < D / 2) {
#pragma unroll
    for (int hh = 0; hh < 8; hh++)
      if ((uint32_t)hh < nh) *reinterpret_cast<float2 *>(PT + pb + 2u * nh + (size_t)hh * D + 2u * dpa) = acc[hh];
  }
}

// the chunks' merge, one CTA per head: M = max m_c, w_c = exp(m_c - M) / sum_c exp(m_c - M) l_c, O = sum_c w_c acc_c
__global__ void __launch_bounds__(kT) attn_combine_kernel(const float *__restrict__ PT, float *__restrict__ O, uint32_t D, uint32_t nh,
                                                          uint32_t nchunk) {
  dep_enter();
  __shared__ float wts[256];
  const uint32_t h = blockIdx.x;
  const size_t st = (size_t)nh * (2u + D);
  if (threadIdx.x == 0) {
    float M = -3.0e38f;
    for (uint32_t c = 0; c < nchunk; c++) M = fmaxf(M, PT[c * st + h]);
    float L = 0.0f;
    for (uint32_t c = 0; c < nchunk; c++) {
      const float e = expf(PT[c * st + h] - M);
      wts[c] = e;
      L = fmaf(e, PT[c * st + nh + h], L);
    }
    for (uint32_t c = 0; c < nchunk; c++) wts[c] = __fdiv_rn(wts[c], L);
  }
  __syncthreads();
  for (uint32_t d = threadIdx.x; d < D; d += kT) {
    float o = 0.0f;
    for (uint32_t c = 0; c < nchunk; c++) o = fmaf(wts[c], PT[c * st + 2u * nh + (size_t)h * D + d], o);
    O[(size_t)h * D + d] = o;
  }
}


// a kernel launch that lets the kernel start before the one ahead of it on the stream finishes (see dep_enter)
template <typename Kern, typename... Args>
cudaError_t launch_dep(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}
}  // namespace

extern "C" {

// argmax(g, a) (lops.js:434-436) is argmaxM with M = 1 (lops_spec.js:346-348)
p0_status p0_argmaxM(p0_ctx *c, p0_buf mx, uint32_t n, uint32_t M, p0_buf out) {
  if (!c) return P0_EINVAL;
  if (!M) return P0_OK;
  P0Range rm, ro;
  p0_status st;
  if ((st = p0_range(c, mx, 0, (uint64_t)M * n * 8, "argmax", "MX", &rm))) return st;
  if ((st = p0_range(c, out, 0, (uint64_t)M * 8, "argmax", "OUT", &ro))) return st;
  cudaSetDevice(c->device);
  launch_dep(argmax_kernel, dim3(M), dim3(kT), 0, c->stream, (const float2 *)rm.base, n, (uint32_t *)ro.base);
  return p0_launched(c, "argmax");
}

p0_status p0_embed(p0_ctx *c, const p0_embed_args *a) {
  if (!c || !a) return P0_EINVAL;
  const bool q8 = a->w.enc == P0_ENC_Q8G64S_T64;
  if (!q8 && a->w.enc != P0_ENC_Q4G32A_T64) return p0_fail(c, P0_EINVAL, "embed: encoding %u", a->w.enc);
  const uint32_t GK = q8 ? 64u : 32u, RB = q8 ? 4224u : 1280u, K = a->K;
  if (!a->n) return P0_OK;
  if (!K || K % GK) return p0_fail(c, P0_EINVAL, "embed: K must be a multiple of %u", GK);
  if (a->w.rows % 64 || a->w.cols != K) return p0_fail(c, P0_EINVAL, "embed: the table view must be [rows %% 64][K] (%ux%u)", a->w.rows, a->w.cols);
  const uint32_t wG = K / GK;
  P0Range rw, ri, rx, rs;
  p0_status st;
  if ((st = p0_range(c, a->w.buf, a->w.off, (uint64_t)(a->w.rows / 64) * wG * RB, "embed", "W", &rw))) return st;
  if ((uintptr_t)rw.base % 16) return p0_fail(c, P0_EALIGN, "embed: table offset must be 16-byte aligned");
  if ((st = p0_range(c, a->ids, 0, (uint64_t)a->n * 4, "embed", "IDS", &ri))) return st;
  if ((st = p0_range(c, a->x, 0, ((uint64_t)a->rowOut + a->n) * K * 4, "embed", "X", &rx))) return st;
  if ((st = p0_range(c, a->st, 0, ((uint64_t)a->st_off + a->n) * 4, "embed", "ST", &rs))) return st;
  const float eps = a->eps != 0.0f ? a->eps : 1e-6f;   // lops.js:364 `a.eps || 1e-6`
  cudaSetDevice(c->device);
  if (q8)
    launch_dep(embed_kernel<true>, dim3(a->n), dim3(kT), 0, c->stream, rw.base, a->w.rows, (const uint32_t *)ri.base, K, wG, a->scale, eps, (float *)rx.base,
                                                    a->rowOut, (float *)rs.base, a->st_off);
  else
    launch_dep(embed_kernel<false>, dim3(a->n), dim3(kT), 0, c->stream, rw.base, a->w.rows, (const uint32_t *)ri.base, K, wG, a->scale, eps, (float *)rx.base,
                                                     a->rowOut, (float *)rs.base, a->st_off);
  return p0_launched(c, "embed");
}

p0_status p0_normadd(p0_ctx *c, const p0_normadd_args *a) {
  if (!c || !a) return P0_EINVAL;
  const uint32_t D = a->D, M = a->M ? a->M : 1, nsrc = a->t_n ? a->t_n : 1;
  if (!D) return P0_OK;
  if (a->mode > 1) return p0_fail(c, P0_EINVAL, "normadd: mode %u", a->mode);
  if ((size_t)D * 4 > 200u * 1024u) return p0_fail(c, P0_EINVAL, "normadd: D %u exceeds the shared-memory row (51200)", D);
  const uint64_t ldp = a->t_ld ? a->t_ld : (uint64_t)D * M;
  P0Range rt, rw, rx, rs;
  p0_status st;
  if ((st = p0_range(c, a->t, 0, ((uint64_t)(nsrc - 1) * ldp + (uint64_t)M * D) * 4, "normadd", "T", &rt))) return st;
  if (a->mode == 0 && (st = p0_range(c, a->w, 0, ((uint64_t)a->w_off + D) * 4, "normadd", "W", &rw))) return st;
  if ((st = p0_range(c, a->x, 0, (uint64_t)M * D * 4, "normadd", "X", &rx))) return st;
  if ((st = p0_range(c, a->st, 0, ((uint64_t)a->st_off + M) * 4, "normadd", "ST", &rs))) return st;
  const float eps = a->eps != 0.0f ? a->eps : 1e-6f;   // lops.js:177 `a.eps || 1e-6`
  const bool pre = (size_t)D * 12 <= 200u * 1024u;   // room for x and w beside the sum: one pass of loads
  const size_t smem = (size_t)D * (pre ? 12 : 4);
  cudaSetDevice(c->device);
  // above the 48 KB default the kernel opts in (its static reduction array counts against the same limit)
  if (smem > 40u * 1024u) cudaFuncSetAttribute(normadd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_dep(normadd_kernel, dim3(M), dim3(kT), smem, c->stream, (const float *)rt.base, nsrc, ldp, a->mode == 0 ? (const float *)rw.base + a->w_off : nullptr,
                                             (float *)rx.base, (float *)rs.base, a->st_off, D, a->mode, eps, a->scale, pre);
  return p0_launched(c, "normadd");
}

p0_status p0_dhead(p0_ctx *c, const p0_dhead_args *a) {
  if (!c || !a) return P0_EINVAL;
  const bool q8 = a->w.enc == P0_ENC_Q8G64S_T64;
  if (!q8 && a->w.enc != P0_ENC_Q4G32A_T64) return p0_fail(c, P0_EINVAL, "dhead: encoding %u", a->w.enc);
  const uint32_t K = a->K, GK = q8 ? 64u : 32u, RB = q8 ? 4224u : 1280u;
  if (K > 512) return p0_fail(c, P0_EINVAL, "dhead: K > 512");
  if (!K || K % GK) return p0_fail(c, P0_EINVAL, "dhead: K must be a multiple of %u", GK);
  if (a->w.rows % 64 || a->w.cols != K) return p0_fail(c, P0_EINVAL, "dhead: the head view must be [rows %% 64][K] (%ux%u)", a->w.rows, a->w.cols);
  const uint32_t nblk = a->nsel * a->tPer, wG = K / GK;
  if (!nblk) return P0_OK;
  P0Range rx, rw, rs, rn, rsel, rm;
  p0_status st;
  if ((st = p0_range(c, a->x, 0, (uint64_t)K * 4, "dhead", "X", &rx))) return st;
  if ((st = p0_range(c, a->w.buf, a->w.off, (uint64_t)(a->w.rows / 64) * wG * RB, "dhead", "W", &rw))) return st;
  if ((uintptr_t)rw.base % 16) return p0_fail(c, P0_EALIGN, "dhead: head offset must be 16-byte aligned");
  if ((st = p0_range(c, a->stat, 0, ((uint64_t)a->stat_off + 1) * 4, "dhead", "ST", &rs))) return st;
  if ((st = p0_range(c, a->norm, 0, ((uint64_t)a->norm_off + K) * 4, "dhead", "NW", &rn))) return st;
  if ((st = p0_range(c, a->sel, 0, (uint64_t)a->nsel * 4, "dhead", "SEL", &rsel))) return st;
  if ((st = p0_range(c, a->mx, 0, (uint64_t)nblk * 8, "dhead", "MX", &rm))) return st;
  cudaSetDevice(c->device);
  const float *stp = (const float *)rs.base + a->stat_off, *nw = (const float *)rn.base + a->norm_off;
  if (q8)
    launch_dep(dhead_kernel<true>, dim3(nblk), dim3(kT), 0, c->stream, (const float *)rx.base, rw.base, a->w.rows / 64, stp, nw, (const uint32_t *)rsel.base, K,
                                                    wG, a->tPer, (float *)rm.base);
  else
    launch_dep(dhead_kernel<false>, dim3(nblk), dim3(kT), 0, c->stream, (const float *)rx.base, rw.base, a->w.rows / 64, stp, nw, (const uint32_t *)rsel.base, K,
                                                     wG, a->tPer, (float *)rm.base);
  return p0_launched(c, "dhead");
}

p0_status p0_qkrope(p0_ctx *c, const p0_qkrope_args *a) {
  if (!c || !a) return P0_EINVAL;
  const uint32_t D = a->D, nq = a->nq, nkv = a->nkv ? a->nkv : 1, nsrc = a->s_n ? a->s_n : 1;
  const uint32_t nh = nq + (a->hasKV ? 2 * nkv : 0);
  if (!nh || !D) return P0_OK;
  if (D % 2 || (size_t)D * 4 > 200u * 1024u) return p0_fail(c, P0_EINVAL, "qkrope: D %u must be even and at most 51200", D);
  if (a->npairs > D / 2) return p0_fail(c, P0_EINVAL, "qkrope: npairs %u > D/2", a->npairs);
  P0Range rs, rn, rr, rq, rk, rv;
  p0_status st;
  const uint64_t ldp = a->s_ld ? a->s_ld : (uint64_t)nh * D;
  if ((st = p0_range(c, a->s, 0, ((uint64_t)(nsrc - 1) * ldp + (uint64_t)nh * D) * 4, "qkrope", "S", &rs))) return st;
  const uint32_t wmax = (a->kw > a->qw ? a->kw : a->qw) + D;
  if ((st = p0_range(c, a->norm, 0, (uint64_t)wmax * 4, "qkrope", "NW", &rn))) return st;
  if ((st = p0_range(c, a->rope, 0, (a->npairs ? ((uint64_t)a->rope_off + ((uint64_t)a->pos + 1) * a->npairs * 2) : 1) * 4, "qkrope", "RP", &rr))) return st;
  if ((st = p0_range(c, a->q, 0, (uint64_t)nq * D * 4, "qkrope", "Q", &rq))) return st;
  if (a->hasKV) {
    if (a->kvRow >= a->kvLen) return p0_fail(c, P0_EINVAL, "qkrope: kvRow %u outside the cache of %u rows", a->kvRow, a->kvLen);
    if ((st = p0_range(c, a->kc, 0, (uint64_t)nkv * a->kvLen * D * 2, "qkrope", "KC", &rk))) return st;
    if ((st = p0_range(c, a->vc, 0, (uint64_t)nkv * a->kvLen * D * 2, "qkrope", "VC", &rv))) return st;
  }
  const float eps = a->eps != 0.0f ? a->eps : 1e-6f;   // lops.js:230 `a.eps || 1e-6`
  const size_t smem = (size_t)D * 4;
  cudaSetDevice(c->device);
  if (smem > 40u * 1024u) cudaFuncSetAttribute(qkrope_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_dep(qkrope_kernel, dim3(nh), dim3(kT), smem, c->stream, (const float *)rs.base, nsrc, ldp, (const float *)rn.base, (const float *)rr.base, (float *)rq.base,
                                             a->hasKV ? (__half *)rk.base : nullptr, a->hasKV ? (__half *)rv.base : nullptr, D, nq, nkv, a->pos,
                                             eps, a->qw, a->kw, a->npairs, a->rope_off, a->kvRow, a->kvLen);
  return p0_launched(c, "qkrope");
}

p0_status p0_attn_dec(p0_ctx *c, const p0_attn_dec_args *a) {
  if (!c || !a) return P0_EINVAL;
  const uint32_t D = a->D, nh = a->nh, nkv = a->nkv ? a->nkv : 1;
  if (a->kEnd <= a->kStart || !nh) return p0_fail(c, P0_EINVAL, "attnDec: no keys (kStart %u, kEnd %u) or heads", a->kStart, a->kEnd);
  const uint32_t nchunk = (a->kEnd - a->kStart + 63u) / 64u;
  if (nchunk > 256) return p0_fail(c, P0_EINVAL, "attnDec: context too long for one combine (%u chunks)", nchunk);
  if (nh > 8 || nh % nkv) return p0_fail(c, P0_EINVAL, "attnDec: %u query heads over %u KV heads (at most 8, a multiple)", nh, nkv);
  if (D % 128 || D > 512) return p0_fail(c, P0_EINVAL, "attnDec: D %u must be a multiple of 128, at most 512", D);
  const uint32_t rows = a->kvLen;
  if (a->ring ? a->ring > rows : a->kEnd > rows) return p0_fail(c, P0_EINVAL, "attnDec: keys beyond the cache of %u rows", rows);
  P0Range rq, rk, rv, rp, ro;
  p0_status st;
  if ((st = p0_range(c, a->q, 0, (uint64_t)nh * D * 4, "attnDec", "Q", &rq))) return st;
  if ((st = p0_range(c, a->kc, 0, (uint64_t)nkv * rows * D * 2, "attnDec", "KC", &rk))) return st;
  if ((st = p0_range(c, a->vc, 0, (uint64_t)nkv * rows * D * 2, "attnDec", "VC", &rv))) return st;
  if ((st = p0_range(c, a->part, 0, (uint64_t)nchunk * nh * (2 + D) * 4, "attnDec", "part", &rp))) return st;
  if ((st = p0_range(c, a->out, 0, (uint64_t)nh * D * 4, "attnDec", "O", &ro))) return st;
  const size_t smem = ((size_t)nh * D + (size_t)nh * 64) * 4 + (size_t)64 * D * 2;   // q | scores | a chunk's V rows
  cudaSetDevice(c->device);
  auto go = [&](auto kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_dep(kern, dim3(nchunk), dim3(kT), smem, c->stream, (const float *)rq.base, (const __half *)rk.base, (const __half *)rv.base, (float *)rp.base, D, nh, nkv,
                                          rows, a->kStart, a->kEnd, a->ring);
  };
  switch (D / 128) {
    case 1: go(attn_chunk_kernel<1>); break;
    case 2: go(attn_chunk_kernel<2>); break;
    case 3: go(attn_chunk_kernel<3>); break;
    default: go(attn_chunk_kernel<4>); break;
  }
  if ((st = p0_launched(c, "attnDec"))) return st;
  launch_dep(attn_combine_kernel, dim3(nh), dim3(kT), 0, c->stream, (const float *)rp.base, (float *)ro.base, D, nh, nchunk);
  return p0_launched(c, "attnDec combine");
}

}  // extern "C"
