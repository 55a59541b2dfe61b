// gemv.cu -- the decode / speculative-verify GEMV over q4g32a.t64 weights on sm_100a:
//   gemv  (engine/llm/lops.js:108-141, kernel lgemv :30-106)        one token
//   gemvM (engine/llm/lops_spec.js:159-191, kernel lgemvM :44-157)  M <= 8 tokens, each weight record read once
// Memory-bound: the weight stream is N*K*0.625 bytes; every record (64 rows x 32 k: 1024 B of codes + 256 B of
// fp16 scale/min) is read exactly once per call with 128-bit non-caching loads, dequantised in registers.
//
// Arithmetic (f32, the reference's factored form lops.js:67-71): per row and 32-k group
//   acc += s * sum_i(q_i * x_i) + mn * sum_i(x_i)
// sum_i(q_i x_i) is formed exactly from floats v_i = 1 + q_i/16, whose bits are 0x3F800000 | q_i << 19 (two
// integer ops per code, no int->float conversion): sum(v_i x_i) = sum(x_i) + sum(q_i x_i)/16, and the group's
// sum(x_i) is shared by every row of the CTA. The summation order differs from the WGSL's per-quarter order by
// f32 rounding only.
#include <cuda_fp16.h>

#include <cstdlib>
#include <cstring>

#include "gemv_common.cuh"

namespace {
using namespace p0gemv;

// 8 codes of one u32 word (k = 8w .. 8w+7, low nibble first) dotted with 8 staged x values, as v_i = 1 + q_i/16
__device__ __forceinline__ float dot8(uint32_t q, const float4 a, const float4 b, float acc) {
  const uint32_t E = 0x3F800000u, MSK = 0x00780000u;
  acc = fmaf(__uint_as_float(((q << 19) & MSK) | E), a.x, acc);
  acc = fmaf(__uint_as_float(((q << 15) & MSK) | E), a.y, acc);
  acc = fmaf(__uint_as_float(((q << 11) & MSK) | E), a.z, acc);
  acc = fmaf(__uint_as_float(((q << 7) & MSK) | E), a.w, acc);
  acc = fmaf(__uint_as_float(((q << 3) & MSK) | E), b.x, acc);
  acc = fmaf(__uint_as_float(((q >> 1) & MSK) | E), b.y, acc);
  acc = fmaf(__uint_as_float(((q >> 5) & MSK) | E), b.z, acc);
  acc = fmaf(__uint_as_float(((q >> 9) & MSK) | E), b.w, acc);
  return acc;
}

template <int MT, bool PAIR>
__global__ void __launch_bounds__(kThreads) gemv_q4_v1(const GemvParams p) {
  extern __shared__ __align__(16) float smem[];
  constexpr int NP = PAIR ? 2 : 1;
  const uint32_t XC = p.xc;                    // staged k per chunk (multiple of 32)
  float *xs = smem;                            // [MT][XC]
  float *xsum = smem + MT * XC;                // [MT][XC/32]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t tile = blockIdx.x, split = blockIdx.y;
  const uint32_t k0 = split * p.kPer, k1 = min(p.K, k0 + p.kPer);
  const uint8_t *tb[NP];
  tb[0] = p.W + (size_t)tile * p.wG * 1280u;
  if (PAIR) tb[NP - 1] = p.W + (size_t)(tile + p.N / 64u) * p.wG * 1280u;

  float acc[NP][2][MT];
#pragma unroll
  for (int a = 0; a < NP; a++)
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
      for (int m = 0; m < MT; m++) acc[a][r][m] = 0.0f;
  pdl_wait();
  pdl_trigger();

  for (uint32_t kc = k0; kc < k1; kc += XC) {
    const uint32_t kc1 = min(k1, kc + XC), len = kc1 - kc, ngr = len / 32;
    __syncthreads();
    for (uint32_t i = tid; i < MT * len; i += kThreads) {
      uint32_t m = i / len, k = i - m * len;
      xs[m * XC + k] = prologue(p, m, kc + k);
    }
    __syncthreads();
    for (uint32_t i = tid; i < MT * ngr; i += kThreads) {
      uint32_t m = i / ngr, gg = i - m * ngr;
      const float *xp = xs + m * XC + gg * 32;
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < 32; j++) s += xp[j];
      xsum[m * (XC / 32) + gg] = s;
    }
    __syncthreads();
    const uint32_t gbase = kc / 32;
    for (uint32_t gg = warp; gg < ngr; gg += kWarps) {
      const uint32_t g = gbase + gg;
#pragma unroll
      for (int a = 0; a < NP; a++) {
        const uint8_t *rec = tb[a] + (size_t)g * 1280u;
        uint4 c[2];
        uint32_t sm[2];
        c[0] = ldg_stream(rec + lane * 16);
        c[1] = ldg_stream(rec + (lane + 32) * 16);
        sm[0] = ldg_u32(rec + 1024 + lane * 4);
        sm[1] = ldg_u32(rec + 1024 + (lane + 32) * 4);
#pragma unroll
        for (int r = 0; r < 2; r++) {
          const float s = __half2float(__ushort_as_half((unsigned short)(sm[r] & 0xffffu)));
          const float mn = __half2float(__ushort_as_half((unsigned short)(sm[r] >> 16)));
          const float s16 = s * 16.0f;   // exact
#pragma unroll
          for (int m = 0; m < MT; m++) {
            const float4 *xv = reinterpret_cast<const float4 *>(xs + m * XC + gg * 32);
            float d = 0.0f;
            d = dot8(c[r].x, xv[0], xv[1], d);
            d = dot8(c[r].y, xv[2], xv[3], d);
            d = dot8(c[r].z, xv[4], xv[5], d);
            d = dot8(c[r].w, xv[6], xv[7], d);
            const float xsm = xsum[m * (XC / 32) + gg];
            // sum(q x) = 16 * (d - sum x); acc += s * sum(q x) + mn * sum(x)
            acc[a][r][m] = fmaf(s16, d - xsm, fmaf(mn, xsm, acc[a][r][m]));
          }
        }
      }
    }
  }
  // reduce the 8 warps' partials: red[warp][a][m][row]
  __syncthreads();
  float *red = smem;
#pragma unroll
  for (int a = 0; a < NP; a++)
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
      for (int m = 0; m < MT; m++) red[((warp * NP + a) * MT + m) * 64 + lane + 32 * r] = acc[a][r][m];
  __syncthreads();
  float *outv = smem + kWarps * NP * MT * 64;   // [MT][64] epilogue values (softcap)
  for (uint32_t i = tid; i < MT * 64; i += kThreads) {
    const uint32_t m = i / 64, r = i % 64, n = tile * 64 + r;
    float tot[NP];
#pragma unroll
    for (int a = 0; a < NP; a++) {
      float t = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; w++) t += red[((w * NP + a) * MT + m) * 64 + r];
      tot[a] = t;
    }
    if (p.epi == P0_EPI_STORE) {
      p.Y[(size_t)split * p.ldy + (size_t)m * p.ldm + n] = tot[0];
    } else if (p.epi == P0_EPI_GEGLU) {
      p.Y[(size_t)m * p.ldm + n] = __fmul_rn(gelu_l(tot[0]), tot[NP - 1]);
    } else {
      float t = fminf(15.0f, fmaxf(-15.0f, __fdiv_rn(tot[0], p.cap)));
      float v = __fmul_rn(p.cap, tanhf(t));
      p.Y[(size_t)m * p.ldm + n] = v;
      outv[m * 64 + r] = v;
    }
  }
  if (p.epi == P0_EPI_SOFTCAP) {
    __syncthreads();
    // per (row m, tile): the max and its lowest index (lops.js:96-102)
    for (uint32_t m = warp; m < MT; m += kWarps) {
      float v0 = outv[m * 64 + lane], v1 = outv[m * 64 + lane + 32];
      float bv = v0;
      uint32_t bi = lane;
      if (v1 > bv) { bv = v1; bi = lane + 32; }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) {
        const size_t o = ((size_t)m * p.ntile + tile) * 2;
        p.MX[o] = bv;
        p.MX[o + 1] = __uint_as_float(tile * 64 + bi);
      }
    }
  }
}

// ================================================================================================================ v2: tensor cores
// The same arithmetic on mma.sync.m16n8k16 (fp16 in, fp32 accumulate), whose cost does not grow with M <= 8:
//  * A (16 weight rows x 16 k): a thread (g = lane/4, c = lane%4) takes u32 word c of rows g and g+8 of a group's
//    record (8 codes each). One LOP3 turns two codes into an fp16x2 of EXACT subnormals: (w & 0x000F000F) is
//    (q0, q4) * 2^-24 and (w & 0x00F000F0) is (q1, q5) * 2^-20; (w >> 8) gives (q2, q6) and (q3, q7) alike.
//  * B (16 k x 8 tokens): x of the group for token g, arranged in shared memory in the same permuted k order, times a
//    per-split power of two sigma (keeps x*sigma inside fp16 range), the odd-code positions times 1/16, and split
//    into hi + lo fp16 halves (two MMAs): ~22 significant bits of each x.
//  * per group and row, in f32: acc += s * D + mn * sum(x) / f, with D the group's MMA sum and f = 2^24 / sigma;
//    the row total is acc * f. Summation order differs from the WGSL's by rounding only.
// Work item = RB row-blocks (16 rows each) x KS k-slices (RB * KS = 8 warps); k-slice partials are summed in
// shared memory in a fixed order. CTAs are persistent over items; x is staged once per CTA and k-split.
constexpr int kRedFloats = 8 * 2 * 4 * 32 * 4;   // [warp][pair][row-block][lane][4]

struct V2Plan {
  uint32_t RW;              // row-blocks (16 rows) per warp unit (template copy)
  uint32_t KS;              // k-slices per unit; 8 / KS units per CTA item
  uint32_t units_per_item, items_per_split, nitems, gmax;
};

// x of one split -> B fragments (hi/lo, permuted) + per-group sums; returns f = 2^24 / sigma
template <int MT>
__device__ float stage_x_v2(const GemvParams &p, uint32_t k0, uint32_t G, uint4 *xb, float *xsum, float *scratch) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t len = G * 32;
  // pass 1: the largest |x| of the split picks sigma
  float mx = 0.0f;
  for (uint32_t i = tid; i < MT * len; i += kThreads) {
    const uint32_t m = i / len, k = i - m * len;
    mx = fmaxf(mx, fabsf(prologue(p, m, k0 + k)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  __syncthreads();
  if (lane == 0) scratch[warp] = mx;
  __syncthreads();
  mx = scratch[0];
#pragma unroll
  for (int w = 1; w < kWarps; w++) mx = fmaxf(mx, scratch[w]);
  int e = 0;
  if (mx > 0.0f && mx < INFINITY) frexpf(mx, &e);            // mx < 2^e
  const float sigma = ldexpf(1.0f, 14 - e);                   // |x| * sigma < 2^14
  const float f = ldexpf(1.0f, 10 + e);                       // 2^24 / sigma
  const float finv = ldexpf(1.0f, -10 - e);
  // pass 2: units (group, token, c) of 8 consecutive k; lanes 4j..4j+3 hold one (group, token)
  const uint32_t units = G * MT * 4, ulim = (units + kThreads - 1) / kThreads * kThreads;
  for (uint32_t u = tid; u < ulim; u += kThreads) {
    float part = 0.0f;
    if (u < units) {
      const uint32_t gg = u / (MT * 4), rem = u - gg * (MT * 4), m = rem >> 2, c = rem & 3u;
      const uint32_t kb = k0 + gg * 32 + c * 8;
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; i++) {
        v[i] = prologue(p, m, kb + i);
        part += v[i];
      }
      float hv[8], lv[8];
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const float vs = v[i] * sigma * ((i & 1) ? 0.0625f : 1.0f);   // exact powers of two
        const float h = __half2float(__float2half_rn(vs));
        hv[i] = h;
        lv[i] = vs - h;
      }
      // MMA0: slots (2c, 2c+1) = k (0, 4), (2c+8, 2c+9) = k (1, 5); MMA1: (2, 6), (3, 7)
      xb[u * 2] = make_uint4(pack_h2(hv[0], hv[4]), pack_h2(hv[1], hv[5]), pack_h2(hv[2], hv[6]), pack_h2(hv[3], hv[7]));
      xb[u * 2 + 1] = make_uint4(pack_h2(lv[0], lv[4]), pack_h2(lv[1], lv[5]), pack_h2(lv[2], lv[6]), pack_h2(lv[3], lv[7]));
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    if (u < units && (u & 3u) == 0) xsum[u >> 2] = part * finv;   // sum(x) / f, exact scaling
  }
  __syncthreads();
  return f;
}

// one warp unit = RW row-blocks of 16 rows (RW = 4: a whole 64-row tile) over one k-slice
template <int MT, bool PAIR, int RW>
__global__ void __launch_bounds__(kThreads) gemv_q4_v2(const GemvParams p, const V2Plan plan) {
  extern __shared__ __align__(128) uint8_t smem8[];
  constexpr int NP = PAIR ? 2 : 1;
  uint4 *xb = reinterpret_cast<uint4 *>(smem8);                                        // [gmax][MT][4][2] uint4
  float *xsum = reinterpret_cast<float *>(smem8 + (size_t)plan.gmax * MT * 128);        // [gmax][MT]
  float *red = xsum + plan.gmax * MT;                                                   // kRedFloats
  float *scratch = red + kRedFloats;                                                    // 64 floats
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const uint32_t UPI = plan.units_per_item, KS = plan.KS, ui = warp % UPI, ksi = warp / UPI;
  uint32_t staged = 0xffffffffu;
  float f = 1.0f;
  uint32_t G = 0;
  const size_t pair_off = (size_t)(p.N / 64u) * p.wG * 1280u;   // geglu: the up rows' tiles follow the gate rows' tiles
  const bool tok_ok = (uint32_t)g < MT;                          // B column n = g is a real token
  pdl_wait();
  pdl_trigger();
  for (uint32_t item = blockIdx.x; item < plan.nitems; item += gridDim.x) {
    const uint32_t split = item / plan.items_per_split, it = item - split * plan.items_per_split;
    const uint32_t k0 = split * p.kPer, k1 = min(p.K, k0 + p.kPer);
    if (split != staged) {
      __syncthreads();
      G = (k1 - k0) / 32;
      f = stage_x_v2<MT>(p, k0, G, xb, xsum, scratch);
      staged = split;
    }
    const uint32_t R0 = (it * UPI + ui) * (RW * 16);          // first row of this warp's unit
    const uint32_t tile = R0 >> 6, rr = (R0 & 63u) + g;
    const uint8_t *base = p.W + (size_t)tile * p.wG * 1280u + (size_t)(k0 / 32) * 1280u;
    const uint8_t *pc = base + rr * 16 + c * 4;               // word c of row rr (+16j for row-block j, +8 rows: +128)
    const uint8_t *pt = base + 1024 + rr * 4;                 // (s, mn) of row rr
    float acc[NP][RW][4];
#pragma unroll
    for (int a = 0; a < NP; a++)
#pragma unroll
      for (int j = 0; j < RW; j++) acc[a][j][0] = acc[a][j][1] = acc[a][j][2] = acc[a][j][3] = 0.0f;
    uint32_t w[NP][RW][2], t[NP][RW][2];
    auto load = [&](uint32_t gg) {
#pragma unroll
      for (int a = 0; a < NP; a++)
#pragma unroll
        for (int j = 0; j < RW; j++) {
          const size_t o = (size_t)gg * 1280u + (a ? pair_off : 0);
          w[a][j][0] = ldg_u32(pc + o + j * 256);
          w[a][j][1] = ldg_u32(pc + o + j * 256 + 128);       // row + 8
          t[a][j][0] = ldg_u32(pt + o + j * 64);
          t[a][j][1] = ldg_u32(pt + o + j * 64 + 32);
        }
    };
    uint32_t gg = ksi;
    if (gg < G) load(gg);
    for (; gg < G; gg += KS) {
      uint32_t cw[NP][RW][2], ct[NP][RW][2];
#pragma unroll
      for (int a = 0; a < NP; a++)
#pragma unroll
        for (int j = 0; j < RW; j++) {
          cw[a][j][0] = w[a][j][0]; cw[a][j][1] = w[a][j][1]; ct[a][j][0] = t[a][j][0]; ct[a][j][1] = t[a][j][1];
        }
      if (gg + KS < G) load(gg + KS);
      // B fragments of this group (token g, slot set c), hi and lo, shared by every row-block of the unit
      uint4 bh = make_uint4(0, 0, 0, 0), bl = bh;
      if (tok_ok) {
        const uint4 *bp = xb + ((size_t)(gg * MT + g) * 4 + c) * 2;
        bh = bp[0];
        bl = bp[1];
      }
      const float xs0 = 2 * c < MT ? xsum[gg * MT + 2 * c] : 0.0f, xs1 = 2 * c + 1 < MT ? xsum[gg * MT + 2 * c + 1] : 0.0f;
#pragma unroll
      for (int a = 0; a < NP; a++)
#pragma unroll
        for (int j = 0; j < RW; j++) {
          const uint32_t w0 = cw[a][j][0], w1 = cw[a][j][1], w0s = w0 >> 8, w1s = w1 >> 8;
          const uint32_t A0[4] = {w0 & 0x000F000Fu, w1 & 0x000F000Fu, w0 & 0x00F000F0u, w1 & 0x00F000F0u};
          const uint32_t A1[4] = {w0s & 0x000F000Fu, w1s & 0x000F000Fu, w0s & 0x00F000F0u, w1s & 0x00F000F0u};
          float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          mma16816(d, A0, bh.x, bh.y);
          mma16816(d, A1, bh.z, bh.w);
          mma16816(d, A0, bl.x, bl.y);
          mma16816(d, A1, bl.z, bl.w);
          const float s0 = __half2float(__ushort_as_half((unsigned short)(ct[a][j][0] & 0xffffu)));
          const float m0 = __half2float(__ushort_as_half((unsigned short)(ct[a][j][0] >> 16)));
          const float s1 = __half2float(__ushort_as_half((unsigned short)(ct[a][j][1] & 0xffffu)));
          const float m1 = __half2float(__ushort_as_half((unsigned short)(ct[a][j][1] >> 16)));
          acc[a][j][0] = fmaf(s0, d[0], fmaf(m0, xs0, acc[a][j][0]));
          acc[a][j][1] = fmaf(s0, d[1], fmaf(m0, xs1, acc[a][j][1]));
          acc[a][j][2] = fmaf(s1, d[2], fmaf(m1, xs0, acc[a][j][2]));
          acc[a][j][3] = fmaf(s1, d[3], fmaf(m1, xs1, acc[a][j][3]));
        }
    }
    // k-slice partials -> the slice-0 warp of each unit, summed in slice order
    if (KS > 1) {
#pragma unroll
      for (int a = 0; a < NP; a++)
#pragma unroll
        for (int j = 0; j < RW; j++)
#pragma unroll
          for (int i = 0; i < 4; i++) red[(((warp * 2 + a) * 4 + j) * 32 + lane) * 4 + i] = acc[a][j][i];
      __syncthreads();
      if (ksi == 0) {
#pragma unroll
        for (int a = 0; a < NP; a++)
#pragma unroll
          for (int j = 0; j < RW; j++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
              float sum = 0.0f;
              for (uint32_t k = 0; k < KS; k++) sum += red[((((k * UPI + ui) * 2 + a) * 4 + j) * 32 + lane) * 4 + i];
              acc[a][j][i] = sum;
            }
      }
    }
    // ---- epilogue (slice-0 warps): row-block j rows R0+16j+g, +8; tokens 2c, 2c+1
    if (ksi == 0) {
      const uint32_t tk0 = 2u * c, tk1 = 2u * c + 1u;
      if (p.epi == P0_EPI_SOFTCAP) {
        // RW == 4: the unit is one whole tile; per token the max over its 64 rows, ties to the lowest row
        float bv0 = -INFINITY, bv1 = -INFINITY;
        uint32_t bi0 = 0xffffffffu, bi1 = 0xffffffffu;
#pragma unroll
        for (int j = 0; j < RW; j++)
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const uint32_t n = R0 + 16 * j + g + (i >= 2 ? 8 : 0), m = (i & 1) ? tk1 : tk0;
            const float v = __fmul_rn(p.cap, tanhf(fminf(15.0f, fmaxf(-15.0f, __fdiv_rn(acc[0][j][i] * f, p.cap)))));
            if (m < MT) p.Y[(size_t)m * p.ldm + n] = v;
            const uint32_t r = n & 63u;
            if (i & 1) { if (v > bv1 || (v == bv1 && r < bi1)) { bv1 = v; bi1 = r; } }
            else { if (v > bv0 || (v == bv0 && r < bi0)) { bv0 = v; bi0 = r; } }
          }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {   // over g: lanes with the same c hold the same tokens
          float ov = __shfl_xor_sync(0xffffffffu, bv0, o);
          uint32_t oi = __shfl_xor_sync(0xffffffffu, bi0, o);
          if (ov > bv0 || (ov == bv0 && oi < bi0)) { bv0 = ov; bi0 = oi; }
          ov = __shfl_xor_sync(0xffffffffu, bv1, o);
          oi = __shfl_xor_sync(0xffffffffu, bi1, o);
          if (ov > bv1 || (ov == bv1 && oi < bi1)) { bv1 = ov; bi1 = oi; }
        }
        if (g == 0) {
          if (tk0 < MT) { const size_t o = ((size_t)tk0 * p.ntile + tile) * 2; p.MX[o] = bv0; p.MX[o + 1] = __uint_as_float(tile * 64 + bi0); }
          if (tk1 < MT) { const size_t o = ((size_t)tk1 * p.ntile + tile) * 2; p.MX[o] = bv1; p.MX[o + 1] = __uint_as_float(tile * 64 + bi1); }
        }
      } else {
        const uint32_t split_off = p.epi == P0_EPI_STORE ? split * p.ldy : 0;
#pragma unroll
        for (int j = 0; j < RW; j++)
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const uint32_t n = R0 + 16 * j + g + (i >= 2 ? 8 : 0), m = (i & 1) ? tk1 : tk0;
            if (m >= MT) continue;
            float v = acc[0][j][i] * f;
            if (p.epi == P0_EPI_GEGLU) v = __fmul_rn(gelu_l(v), acc[NP - 1][j][i] * f);
            p.Y[(size_t)split_off + (size_t)m * p.ldm + n] = v;
          }
      }
    }
    if (KS > 1) __syncthreads();   // red is reused by the next item
  }
}

typedef void (*V2Kernel)(const GemvParams, const V2Plan);

template <int MT, bool PAIR>
V2Kernel v2_kernel(uint32_t RW) {
  return RW == 1 ? gemv_q4_v2<MT, PAIR, 1> : RW == 2 ? gemv_q4_v2<MT, PAIR, 2> : gemv_q4_v2<MT, PAIR, 4>;
}
template <int MT>
V2Kernel v2_kernel_m(bool pair, uint32_t RW) { return pair ? v2_kernel<MT, true>(RW) : v2_kernel<MT, false>(RW); }
V2Kernel v2_kernel_for(uint32_t M, bool pair, uint32_t RW) {
  switch (M) {
    case 1: return v2_kernel_m<1>(pair, RW);
    case 2: return v2_kernel_m<2>(pair, RW);
    case 3: return v2_kernel_m<3>(pair, RW);
    case 4: return v2_kernel_m<4>(pair, RW);
    case 5: return v2_kernel_m<5>(pair, RW);
    case 6: return v2_kernel_m<6>(pair, RW);
    case 7: return v2_kernel_m<7>(pair, RW);
    default: return v2_kernel_m<8>(pair, RW);
  }
}

size_t v2_smem(uint32_t M, uint32_t gmax) { return (size_t)gmax * M * 128 + (size_t)gmax * M * 4 + kRedFloats * 4 + 64 * 4; }

// v2 runs when the split's staged x fits in shared memory
bool v2_fits(uint32_t M, uint32_t kspan) { return v2_smem(M, (kspan + 31) / 32) <= 200u * 1024u; }

cudaError_t launch_v2(const GemvParams &p, uint32_t nsplit, int sms, cudaStream_t s) {
  const uint32_t nrb = p.N / 16;
  const bool pair = p.epi == P0_EPI_GEGLU;
  V2Plan pl{};
  pl.gmax = (min(p.kPer, p.K) + 31) / 32;
  const size_t smem = v2_smem(p.M, pl.gmax);
  // Unit = RW row-blocks over one k-slice; 8 / KS units per CTA item; CTAs persist over items. Pick the plan whose
  // items fill the resident CTA slots with the least wave-quantisation loss, preferring large units (more bytes in
  // flight per warp) and few k-slices. Softcap keeps a whole tile per unit (its argmax stays inside one warp).
  double best = -1.0;
  uint32_t bRW = 4, bKS = 8, bslots = 1;
  const uint32_t rws[3] = {4, 2, 1}, kss[4] = {1, 2, 4, 8};
  for (uint32_t a = 0; a < 3; a++) {
    const uint32_t RW = rws[a];
    if (p.epi == P0_EPI_SOFTCAP && RW != 4) continue;
    V2Kernel k = v2_kernel_for(p.M, pair, RW);
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kThreads, smem) != cudaSuccess || occ < 1) { cudaGetLastError(); occ = 1; }
    const uint32_t slots = (uint32_t)sms * (uint32_t)occ;
    for (uint32_t b = 0; b < 4; b++) {
      const uint32_t KS = kss[b], UPI = 8 / KS;
      if (nrb % (RW * UPI)) continue;
      const double items = (double)(nrb / (RW * UPI) * nsplit);
      const double waves = items / slots, eff = waves / ceil(waves);
      const double score = eff * (1.0 - 0.03 * b) * (1.0 - 0.02 * (2 - a));
      if (score > best) { best = score; bRW = RW; bKS = KS; bslots = slots; }
    }
  }
  pl.RW = bRW;
  pl.KS = bKS;
  pl.units_per_item = 8 / bKS;
  pl.items_per_split = nrb / (bRW * pl.units_per_item);
  pl.nitems = pl.items_per_split * nsplit;
  const uint32_t grid = bslots < pl.nitems ? bslots : pl.nitems;
  return launch_pdl(v2_kernel_for(p.M, pair, bRW), dim3(grid), dim3(kThreads), smem, s, 1, p, pl);
}

template <int MT>
cudaError_t launch_mt(const GemvParams &p, dim3 grid, size_t smem, cudaStream_t s) {
  if (p.epi == P0_EPI_GEGLU) {
    auto k = gemv_q4_v1<MT, true>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return launch_pdl(k, grid, dim3(kThreads), smem, s, 1, p);
  } else {
    auto k = gemv_q4_v1<MT, false>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return launch_pdl(k, grid, dim3(kThreads), smem, s, 1, p);
  }
}

cudaError_t launch_gemv(const GemvParams &p, uint32_t nsplit, cudaStream_t s) {
  const int NP = p.epi == P0_EPI_GEGLU ? 2 : 1;
  size_t stage = (size_t)p.M * p.xc * 4 + (size_t)p.M * (p.xc / 32) * 4;
  size_t red = (size_t)kWarps * NP * p.M * 64 * 4 + (size_t)p.M * 64 * 4;
  size_t smem = stage > red ? stage : red;
  dim3 grid(p.N / 64, nsplit);
  switch (p.M) {
    case 1: return launch_mt<1>(p, grid, smem, s);
    case 2: return launch_mt<2>(p, grid, smem, s);
    case 3: return launch_mt<3>(p, grid, smem, s);
    case 4: return launch_mt<4>(p, grid, smem, s);
    case 5: return launch_mt<5>(p, grid, smem, s);
    case 6: return launch_mt<6>(p, grid, smem, s);
    case 7: return launch_mt<7>(p, grid, smem, s);
    default: return launch_mt<8>(p, grid, smem, s);
  }
}

const char *epi_name(uint32_t e) { return e == P0_EPI_STORE ? "store" : e == P0_EPI_GEGLU ? "geglu" : e == P0_EPI_SOFTCAP ? "softcap" : "?"; }
const char *enc_name(uint32_t e) { return e == P0_ENC_Q4G32A_T64 ? "q4g32a.t64" : e == P0_ENC_Q8G64S_T64 ? "q8g64s.t64" : e == P0_ENC_F16 ? "f16" : "?"; }

// shared host path of gemv / gemvM once the reference's own argument checks have passed
p0_status run_gemv(p0_ctx *c, const char *op, const p0_wview &w, p0_buf xb, uint32_t rowB, uint32_t ldx, uint32_t M, uint32_t N,
                   uint32_t K, uint32_t kPer, uint32_t nsplit, uint32_t pro, uint32_t epi, p0_buf yb, uint32_t ldy, uint32_t ldm,
                   p0_buf stb, uint32_t stat_off, uint32_t stat_ld, p0_buf nb, uint32_t norm_off, p0_buf eb, uint32_t ev_off,
                   uint32_t ev_ld, uint32_t src_n, uint32_t src_ld, p0_buf mxb, float cap, bool noalloc = false) {
  p0_status st;
  const bool q8 = w.enc == P0_ENC_Q8G64S_T64;
  const uint32_t G = q8 ? 64u : 32u, RB = q8 ? 4224u : 1280u;   // k per record, bytes per record
  if (w.enc != P0_ENC_Q4G32A_T64 && !q8) return p0_fail(c, P0_EINVAL, "%s: encoding %s is not built in this library yet", op, enc_name(w.enc));
  if (K % G) return p0_fail(c, P0_EINVAL, "%s: K must be a multiple of %u", op, G);
  if (w.cols % G || w.cols < K) return p0_fail(c, P0_EINVAL, "%s: weight cols %u do not cover K %u", op, w.cols, K);
  if (pro > P0_PRO_PLEG || epi > P0_EPI_SOFTCAP) return p0_fail(c, P0_EINVAL, "%s: prologue/epilogue code", op);
  const uint32_t wG = w.cols / G, NT = N / 64, ntw = epi == P0_EPI_GEGLU ? 2 * NT : NT;
  // bind and bounds-check every view, as WebGPU validates bindings
  P0Range rw, rx, ry, rn, re, rs, rm;
  // the records the call reads: every tile's first K/G groups, tiles wG records apart (a view may start at a later
  // group of tile 0, as a k-slice of a wider weight does)
  uint64_t wneed = ((uint64_t)(ntw - 1) * wG + K / G) * RB;
  if (w.bytes && wneed > w.bytes) return p0_fail(c, P0_EINVAL, "%s: weight view of %llu bytes holds fewer than %u tiles", op, (unsigned long long)w.bytes, ntw);
  if ((st = p0_range(c, w.buf, w.off, wneed, op, "W", &rw))) return st;
  if ((uintptr_t)rw.base % 16) return p0_fail(c, P0_EALIGN, "%s: weight offset (16-byte aligned records needed)", op);
  uint64_t xneed;
  if (pro == P0_PRO_SUM || pro == P0_PRO_PLEG) {
    if (!src_n) return p0_fail(c, P0_EINVAL, "%s: %s needs src.n >= 1", op, pro == P0_PRO_SUM ? "sum" : "pleg");
    xneed = ((uint64_t)(src_n - 1) * src_ld + (uint64_t)(M - 1) * ldx + K) * 4;
  } else {
    xneed = ((uint64_t)(M - 1) * ldx + rowB + K) * 4;
  }
  if ((st = p0_range(c, xb, 0, xneed, op, "X", &rx))) return st;
  uint64_t yneed = epi == P0_EPI_STORE ? ((uint64_t)(nsplit - 1) * ldy + (uint64_t)(M - 1) * ldm + N) * 4 : ((uint64_t)(M - 1) * ldm + N) * 4;
  if ((st = p0_range(c, yb, 0, yneed, op, "Y", &ry))) return st;
  if (pro == P0_PRO_RMS) {
    if ((st = p0_range(c, nb, 0, ((uint64_t)norm_off + K) * 4, op, "norm", &rn))) return st;
    if ((st = p0_range(c, stb, 0, ((uint64_t)stat_off + (uint64_t)(M - 1) * stat_ld + 1) * 4, op, "stat", &rs))) return st;
  }
  if (pro == P0_PRO_PLEG && (st = p0_range(c, eb, 0, ((uint64_t)ev_off + (uint64_t)(M - 1) * ev_ld + K) * 4, op, "ev", &re))) return st;
  if (epi == P0_EPI_SOFTCAP && (st = p0_range(c, mxb, 0, (uint64_t)M * NT * 8, op, "mx", &rm))) return st;

  GemvParams p{};
  p.X = (const float *)rx.base; p.W = rw.base; p.Y = (float *)ry.base;
  p.NW = (const float *)rn.base; p.EV = (const float *)re.base; p.ST = (const float *)rs.base; p.MX = (float *)rm.base;
  p.M = M; p.N = N; p.K = K; p.wG = wG; p.kPer = kPer; p.ldy = ldy; p.ldm = ldm; p.ldx = ldx; p.rowB = rowB;
  p.nOff = norm_off; p.statOff = stat_off; p.statLd = stat_ld; p.evOff = ev_off; p.evLd = ev_ld; p.ldp = src_ld; p.nsrc = src_n;
  p.ntile = NT; p.cap = cap; p.pro = (int)pro; p.epi = (int)epi; p.err = c->d_err; p.overlap = c->overlap ? 1 : 0;
  p.q8 = q8 ? 1 : 0;
  // staged x per chunk: <= 32 KB of x rows, whole groups
  uint32_t xc = (8192u / M) / 32u * 32u;
  uint32_t span = kPer < K ? kPer : K;
  if (xc > span) xc = span;
  p.xc = xc;
  if (c->chain_rec) {
    // a chain is being recorded (p0_chain_begin): the checked call is kept, with the byte ranges it reads and
    // writes, instead of launched
    ChainIO io{};
    io.in[0] = {(uintptr_t)rx.base, (uintptr_t)rx.base + xneed};
    if (pro == P0_PRO_RMS) {
      io.in[1] = {(uintptr_t)rn.base, (uintptr_t)rn.base + (uint64_t)K * 4};
      io.in[2] = {(uintptr_t)rs.base, (uintptr_t)rs.base + ((uint64_t)(M - 1) * stat_ld + 1) * 4};
    }
    if (pro == P0_PRO_PLEG) io.in[3] = {(uintptr_t)re.base, (uintptr_t)re.base + ((uint64_t)(M - 1) * ev_ld + K) * 4};
    io.out[0] = {(uintptr_t)ry.base, (uintptr_t)ry.base + yneed};
    if (epi == P0_EPI_SOFTCAP) io.out[1] = {(uintptr_t)rm.base, (uintptr_t)rm.base + (uint64_t)M * NT * 8};
    return chain_record(c, op, p, nsplit, io);
  }
  return gemv_dispatch(c, op, p, nsplit, noalloc);
}

}  // namespace

namespace p0gemv {
// the kernel choice and launch of one checked gemv / gemvM call (also used for the calls of a recorded chain that do
// not run inside the chain kernel)
p0_status gemv_dispatch(p0_ctx *c, const char *op, const GemvParams &p, uint32_t nsplit, bool noalloc) {
  p0_status st;
  const uint32_t M = p.M, N = p.N, K = p.K, epi = (uint32_t)p.epi;
  const bool q8 = p.q8 != 0;
  const uint32_t span = p.kPer < K ? p.kPer : K;
  cudaSetDevice(c->device);
  cudaError_t e;
  // tuning override, read on every call: P0MM_GEMV=v2 | v3 | v4 | v5 runs that kernel wherever it fits
  const char *force = getenv("P0MM_GEMV");
  const int pick = force && force[0] == 'v' && force[1] >= '2' && force[1] <= '5' && !force[2] ? force[1] - '0' : 0;
  // Measured on B200 (config-2 sweep and the config-5 chain, graph-launched): v3 leads wherever it fits (the head);
  // v5 on the calls with few tiles it takes (N 2048: 5.8-7.0 us against v2's 8.0-15.6; N 16384: 9.1-20.5 against
  // 16.4-20.6); v4 next for M >= 5 on mid-sized calls (>= 8192 records, no geglu); v2 on the rest.
  V4Plan pl{};
  V5Plan p5{};
  size_t scratch_bytes = 0;
  if (q8) {
    // q8g64s.t64 weights run on the cluster kernel only
    if (noalloc) return p0_fail(c, P0_EINVAL, "%s: q8g64s.t64 weights are not built for the allocation-free entry point", op);
    if (!v5_plan(p, nsplit, c->sm_count, &p5))
      return p0_fail(c, P0_EINVAL, "%s: q8g64s.t64 with M %u x K %u (split %u) is not built in this library yet", op, M, K, p.kPer);
    if ((st = p0_cuda(c, launch_v5(p, p5, c->stream), op))) return st;
    return p0_launched(c, op);
  }
  if (noalloc) {
    // the allocation-free mode: the stream-K kernel with the fixed device array as its scratch
    if (!v4_plan(p, nsplit, c->sm_count, &pl, &scratch_bytes))
      return p0_fail(c, P0_EINVAL, "%s: this call does not fit the stream-K kernel (geglu with k-splits, weight columns < K, "
                     "M*K > 16384 or fewer than 16 records)", op);
    const size_t cnt_bytes = (v4_counter_bytes(pl) + 255) / 256 * 256;
    if (cnt_bytes > P0_NOALLOC_COUNTER_BYTES || scratch_bytes > (size_t)P0_NOALLOC_SCRATCH_BYTES - P0_NOALLOC_COUNTER_BYTES)
      return p0_fail(c, P0_EINVAL, "%s: needs %zu bytes of counters and %zu bytes of scratch; the fixed array holds %u and %u", op,
                     cnt_bytes, scratch_bytes, P0_NOALLOC_COUNTER_BYTES, P0_NOALLOC_SCRATCH_BYTES - P0_NOALLOC_COUNTER_BYTES);
    uint8_t *fixed = nullptr;
    if ((st = p0_cuda(c, v4_noalloc_scratch(&fixed), op))) return st;
    pl.cnt = (uint32_t *)fixed;
    pl.part = (float *)(fixed + P0_NOALLOC_COUNTER_BYTES);
    // No clearing pass: the counters start at zero (static device storage) and the kernel returns every counter it
    // uses to zero before it exits, on its give-up path too (v4_arrive_only), so a call leaves them as it found them.
    // A memset here would also sit between this launch and the kernel ahead and stop their programmatic overlap.
    if ((st = p0_cuda(c, launch_v4(p, pl, c->stream), op))) return st;
    return p0_launched(c, op);
  }
  const bool v3fit = v3_fits(M, K, nsplit, N / 64, c->sm_count);
  const bool v3sfit = v3_split_fits(M, K, nsplit, N / 64, c->sm_count, epi == P0_EPI_GEGLU);
  const bool v5fit = v5_plan(p, nsplit, c->sm_count, &p5);
  const bool v4fit = v4_plan(p, nsplit, c->sm_count, &pl, &scratch_bytes);
  bool v3ok, v4ok, v5ok;
  if (pick) {
    v3ok = pick == 3 && (v3fit || v3sfit);
    v4ok = pick == 4 && v4fit;
    v5ok = pick == 5 && v5fit;
  } else {
    // measured on B200 (graph-free back-to-back calls, weights beyond L2), including the column-split head shapes of
    // 2 / 4 / 8 ranks (2048 / 1024 / 512 tiles at K = 2048): at M >= 2 the cluster kernel loses once its units pass two
    // per SM (1024 tiles, M = 4: 68.9 us against v2's 41.2), and from 2048 tiles on the stream-K kernel is the fastest
    // at every M (M = 1: 51.5 us against 90.7)
    // and for the column-split head shapes (2048 / 1024 / 512 tiles at K = 2048), v3 with tiles cut into k-parts: at
    // 2048 tiles 50.4 / 50.2 / 49.8 / 57.7 us against stream-K's 51.2 / 55.2 / 62.6 / 70.0 at M = 1 / 2 / 4 / 8; at
    // 1024 and 512 tiles ahead from M = 2 on (33.4 against 42.1 us at 1024 tiles, M = 2), behind the cluster kernel at M = 1
    // and at 256 tiles (N = 16384, M = 2: 17.5 against 11.1 us)
    const uint32_t ntile_all = N / 64;
    v3ok = v3fit || (v3sfit && ntile_all >= 512u && (M >= 2 || ntile_all >= 2048u));
    v5ok = !v3ok && v5fit && (M == 1 || p.q8 || p5.units <= 2u * (uint32_t)c->sm_count);
    v4ok = !v3ok && !v5ok && v4fit && epi != P0_EPI_GEGLU && ((M >= 5 && pl.R >= 8192u) || ntile_all >= 2048u);
  }
  if (v5ok) {
    e = launch_v5(p, p5, c->stream);
  } else if (v4ok) {
    void *scratch = nullptr;
    if ((st = p0_workspace(c, v4_counter_bytes(pl), scratch_bytes, &pl.cnt, &scratch))) return st;
    pl.part = (float *)scratch;
    e = launch_v4(p, pl, c->stream);
  } else if (v3ok) e = launch_v3(p, c->sm_count, c->stream);
  else if (v2_fits(M, span)) e = launch_v2(p, nsplit, c->sm_count, c->stream);
  else e = launch_gemv(p, nsplit, c->stream);
  if ((st = p0_cuda(c, e, op))) return st;
  return p0_launched(c, op);
}
}  // namespace p0gemv

// the checks and call of gemvM (lops_spec.js:163-191), shared by p0_gemvM and p0_gemvM_noalloc
static p0_status gemvM_call(p0_ctx *c, const p0_gemvM_args *a, uint32_t *nsplit_out, bool noalloc) {
  if (!c || !a) return P0_EINVAL;
  const uint32_t enc = a->w.enc;
  if (enc != P0_ENC_Q4G32A_T64 && enc != P0_ENC_Q8G64S_T64) return p0_fail(c, P0_EINVAL, "gemvM: encoding %s", enc_name(enc));
  if (a->pro != P0_PRO_RAW && a->pro != P0_PRO_RMS && a->pro != P0_PRO_PLEG)
    return p0_fail(c, P0_EINVAL, "gemvM: prologue %s", a->pro == P0_PRO_SUM ? "sum" : "?");
  const uint32_t M = a->M, K = a->K, N = a->N, G = enc == P0_ENC_Q4G32A_T64 ? 32 : 64;
  if (M < 1 || M > 8) return p0_fail(c, P0_EINVAL, "gemvM: M %u (1..8)", M);
  const uint32_t kPer = a->kPer ? (a->kPer < 2048 ? a->kPer : 2048) : K;
  if (kPer == 0 || kPer % G) return p0_fail(c, P0_EINVAL, "gemvM: kPer must be a multiple of %u", G);
  const uint32_t nsplit = (K + kPer - 1) / kPer;
  if (a->epi != P0_EPI_STORE && nsplit > 1) return p0_fail(c, P0_EINVAL, "gemvM: %s needs one split", epi_name(a->epi));
  if (N % 64 || N == 0) return p0_fail(c, P0_EINVAL, "gemvM: N %% 64");
  if (a->w.off % 4) return p0_fail(c, P0_EINVAL, "gemvM: weight offset");
  const uint32_t ldm = a->ldm ? a->ldm : N, ldy = a->ldy ? a->ldy : M * ldm;
  p0_status st = run_gemv(c, noalloc ? "gemvM_noalloc" : "gemvM", a->w, a->x, a->x_rowB, a->x_ldx ? a->x_ldx : K, M, N, K, kPer, nsplit, a->pro, a->epi, a->y, ldy,
                          ldm, a->stat, a->stat_off, a->stat_ld ? a->stat_ld : 2, a->norm, a->norm_off, a->ev, a->ev_off, a->ev_ld,
                          a->src_n ? a->src_n : 1, a->src_ld, a->mx, a->cap != 0.0f ? a->cap : 30.0f, noalloc);
  if (st == P0_OK && nsplit_out) *nsplit_out = nsplit;
  return st;
}


extern "C" {

// gemv(g, a) (lops.js:111-141): the same checks, in the same order, with the same messages
p0_status p0_gemv(p0_ctx *c, const p0_gemv_args *a, uint32_t *nsplit_out) {
  if (!c || !a) return P0_EINVAL;
  const uint32_t enc = a->w.enc;
  if (enc != P0_ENC_Q4G32A_T64 && enc != P0_ENC_Q8G64S_T64) return p0_fail(c, P0_EINVAL, "gemv: encoding %s", enc_name(enc));
  const uint32_t K = a->K, N = a->N, G = enc == P0_ENC_Q4G32A_T64 ? 32 : 64;
  const uint32_t kch = (!a->kPer && K > 2048) ? (K + 255) / 256 * 256 : 2048;
  if (kch > 3072) return p0_fail(c, P0_EINVAL, "gemv: K %u needs a kPer", K);
  uint32_t kPer = a->kPer ? a->kPer : K;
  if (kPer > kch) kPer = kch;
  if (kPer == 0 || kPer % G) return p0_fail(c, P0_EINVAL, "gemv: kPer must be a multiple of %u", G);
  const uint32_t nsplit = (K + kPer - 1) / kPer;
  if (a->epi != P0_EPI_STORE && nsplit > 1) return p0_fail(c, P0_EINVAL, "gemv: %s needs one split", epi_name(a->epi));
  if (N % 64 || N == 0) return p0_fail(c, P0_EINVAL, "gemv: N %% 64");
  if (a->w.off % 4) return p0_fail(c, P0_EINVAL, "gemv: weight offset");
  // lops.js:125: the rms prologue reads its rstd from the buffer bound as MX: a.mx for softcap, else a.stat
  const p0_buf stb = a->epi == P0_EPI_SOFTCAP ? a->mx : a->stat;
  p0_status st = run_gemv(c, "gemv", a->w, a->x, a->x_rowB, K, 1, N, K, kPer, nsplit, a->pro, a->epi, a->y, a->ldy ? a->ldy : N, N,
                          stb, a->stat_off, 0, a->norm, a->norm_off, a->ev, a->ev_off, 0, a->src_n, a->src_ld, a->mx,
                          a->cap != 0.0f ? a->cap : 30.0f);
  if (st == P0_OK && nsplit_out) *nsplit_out = nsplit;
  return st;
}

// gemvM(g, a) (lops_spec.js:163-191)
p0_status p0_gemvM(p0_ctx *c, const p0_gemvM_args *a, uint32_t *nsplit_out) { return gemvM_call(c, a, nsplit_out, false); }

// gemvM for callers that cannot allocate device memory during a call (no counterpart in the reference; the header
// says why and what it costs): the stream-K kernel with its scratch in a fixed device array
p0_status p0_gemvM_noalloc(p0_ctx *c, const p0_gemvM_args *a, uint32_t *nsplit_out) { return gemvM_call(c, a, nsplit_out, true); }

}  // extern "C"
