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

#include "internal.h"

namespace {

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

template <int MT>
cudaError_t launch_mt(const GemvParams &p, dim3 grid, size_t smem, cudaStream_t s) {
  if (p.epi == P0_EPI_GEGLU) {
    auto k = gemv_q4_v1<MT, true>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, kThreads, smem, s>>>(p);
  } else {
    auto k = gemv_q4_v1<MT, false>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, kThreads, smem, s>>>(p);
  }
  return cudaGetLastError();
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
                   uint32_t ev_ld, uint32_t src_n, uint32_t src_ld, p0_buf mxb, float cap) {
  p0_status st;
  const uint32_t G = 32;
  if (w.enc != P0_ENC_Q4G32A_T64) return p0_fail(c, P0_EINVAL, "%s: encoding %s is not built in this library yet", op, enc_name(w.enc));
  if (K % G) return p0_fail(c, P0_EINVAL, "%s: K must be a multiple of %u", op, G);
  if (w.cols % G || w.cols < K) return p0_fail(c, P0_EINVAL, "%s: weight cols %u do not cover K %u", op, w.cols, K);
  if (pro > P0_PRO_PLEG || epi > P0_EPI_SOFTCAP) return p0_fail(c, P0_EINVAL, "%s: prologue/epilogue code", op);
  const uint32_t wG = w.cols / G, NT = N / 64, ntw = epi == P0_EPI_GEGLU ? 2 * NT : NT;
  // bind and bounds-check every view, as WebGPU validates bindings
  P0Range rw, rx, ry, rn, re, rs, rm;
  uint64_t wneed = (uint64_t)ntw * wG * 1280u;
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
  p.ntile = NT; p.cap = cap; p.pro = (int)pro; p.epi = (int)epi; p.err = c->d_err;
  // staged x per chunk: <= 32 KB of x rows, whole groups
  uint32_t xc = (8192u / M) / 32u * 32u;
  uint32_t span = kPer < K ? kPer : K;
  if (xc > span) xc = span;
  p.xc = xc;
  cudaSetDevice(c->device);
  return p0_cuda(c, launch_gemv(p, nsplit, c->stream), op) ?: p0_launched(c, op);
}

}  // namespace

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
p0_status p0_gemvM(p0_ctx *c, const p0_gemvM_args *a, uint32_t *nsplit_out) {
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
  p0_status st = run_gemv(c, "gemvM", a->w, a->x, a->x_rowB, a->x_ldx ? a->x_ldx : K, M, N, K, kPer, nsplit, a->pro, a->epi, a->y, ldy,
                          ldm, a->stat, a->stat_off, a->stat_ld ? a->stat_ld : 2, a->norm, a->norm_off, a->ev, a->ev_off, a->ev_ld,
                          a->src_n ? a->src_n : 1, a->src_ld, a->mx, a->cap != 0.0f ? a->cap : 30.0f);
  if (st == P0_OK && nsplit_out) *nsplit_out = nsplit;
  return st;
}

}  // extern "C"
