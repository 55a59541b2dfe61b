/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY. A CPU restatement of p0pc0rn's 4-bit quantized matmul path,
 * used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs as the
 * checker. Nothing in the product (p0pc0rn_b200/) links, imports or calls this file.
 *
 * The reference is JavaScript + WGSL (ArtistJoshHughes/p0pc0rn). It has no JS engine or WebGPU adapter
 * in this build environment, so every function below restates the cited JS/WGSL arithmetic in C:
 *   - data generation      engine/kcheck.js:10-11   (rng xorshift32, randn Box-Muller in f64 -> f32)
 *   - fp16 helpers         engine/core/gpu.js:274-295 (f2h: f64 -> f32 -> fp16 RNE; h2f)
 *   - quantisers           engine/kcheck.js:14,22-53 (rhe, packQ4 = q4g32a.t64, packQ8 = q8g64s.t64)
 *   - decode GEMV          engine/llm/lops.js:30-106 (lgemv: prologues raw/rms/sum/pleg, epilogues
 *                          store/geglu/softcap + per-tile max/argmax)
 *   - verify GEMV          engine/llm/lops_spec.js:44-157 (lgemvM: M rows, same per-row order)
 *   - DiT GEMM             engine/ops/gemm.js:25-253 (q4/q8/f16 weights, acc f32 or fp16 partials,
 *                          epilogues f16/f32/bias/resadd/swiglu) and engine/ops/misc.js:116 (ew gelu)
 * Each kernel restatement walks the WGSL's invocation structure (workgroup = 64-row tile x k-split,
 * thread = row x quarter) and sums in the order the WGSL source writes (f32, no contraction: build
 * with -ffp-contract=off). WGSL leaves dot() order and FMA contraction to the driver, so a GPU running
 * the reference may differ from this in the last bits; the parity tolerance covers that.
 *
 * Parity pin: the reference stores no golden vectors and cannot run here; the pins are its own
 * known-answer checks (kcheck.js:72-88, 129-135; tune/kshipped.js:17-45; tune/autotune.js:167-199)
 * restated in tests/test_oracle.py, plus hand-computed vectors for f2h/rng. Kernel outputs are
 * therefore "parity unpinned" against reference-produced numbers.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ data generation (kcheck.js:10-11) */

/* rng(seed): JS `s ^= s << 13; s >>>= 0; s ^= s >> 17; s ^= s << 5; s >>>= 0; return s / 4294967296`.
 * `s >> 17` is JS's signed (arithmetic) shift of the int32 view of s, so it is restated as such. */
typedef struct { uint32_t s; } or_rng;
static inline void rng_init(or_rng *r, uint32_t seed) { r->s = seed ? seed : 1u; }
static inline double rng_next(or_rng *r) {
  uint32_t s = r->s;
  s ^= s << 13;
  s ^= (uint32_t)(((int32_t)s) >> 17);
  s ^= s << 5;
  r->s = s;
  return (double)s / 4294967296.0;
}

/* randn(n, seed, scale) -> Float32Array (kcheck.js:11) */
void or_randn(float *o, int64_t n, uint32_t seed, double scale) {
  or_rng r; rng_init(&r, seed);
  for (int64_t i = 0; i < n; i += 2) {
    double u = rng_next(&r); if (u < 1e-9) u = 1e-9;   /* Math.max(1e-9, r()) */
    double v = rng_next(&r);
    double m = sqrt(-2.0 * log(u)) * scale;
    o[i] = (float)(m * cos(2.0 * M_PI * v));
    if (i + 1 < n) o[i + 1] = (float)(m * sin(2.0 * M_PI * v));
  }
}
uint32_t or_rng_u32(uint32_t seed, int64_t k) {   /* the k-th raw state (for pinning rng itself) */
  or_rng r; rng_init(&r, seed); double d = 0; for (int64_t i = 0; i <= k; i++) d = rng_next(&r); (void)d; return r.s;
}

/* ------------------------------------------------------------------ fp16 helpers (core/gpu.js:274-295) */

uint16_t or_f2h(double v) {
  float f = (float)v; uint32_t x; memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u, e = (x >> 23) & 0xffu, m = x & 0x7fffffu;
  if (e == 0xffu) return (uint16_t)(sign | 0x7c00u | (m ? 0x200u : 0u));
  int ne = (int)e - 112;
  if (ne >= 0x1f) return (uint16_t)(sign | 0x7c00u);
  if (ne <= 0) {
    if (ne < -10) return (uint16_t)sign;
    m |= 0x800000u; int sh = 14 - ne; uint32_t hm = m >> sh; uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
    if (rem > half || (rem == half && (hm & 1u))) hm++;
    return (uint16_t)(sign | hm);
  }
  uint32_t r = sign | ((uint32_t)ne << 10) | (m >> 13); uint32_t rem2 = m & 0x1fffu;
  if (rem2 > 0x1000u || (rem2 == 0x1000u && (r & 1u))) r++;
  return (uint16_t)r;
}
double or_h2f(uint16_t h) {
  double s = (h & 0x8000u) ? -1.0 : 1.0; uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  if (e == 0) return s * m * 5.960464477539063e-8;
  if (e == 31) return m ? NAN : s * INFINITY;
  return s * (1.0 + m / 1024.0) * ldexp(1.0, (int)e - 15);
}
static inline double rf16(double x) { return or_h2f(or_f2h(x)); }
static inline float h2f32(uint16_t h) { return (float)or_h2f(h); }

/* rhe: round half to even (kcheck.js:14) */
static inline double rhe(double x) { double f = floor(x), d = x - f; return d > 0.5 ? f + 1 : d < 0.5 ? f : (fmod(f, 2.0) == 0.0 ? f : f + 1); }

/* ------------------------------------------------------------------ packers (kcheck.js:22-53) */

/* packQ4 -> q4g32a.t64: record (t = n/64, g = k/32) of 1280 B at (t*G + g)*1280: byte r*16 + j = q[2j] | q[2j+1] << 4
 * for row r; u32 at 1024 + 4r = f16(s) | f16(mn) << 16. deq = q*s + mn rounded to f32. Requires N%64 == 0, K%32 == 0. */
void or_pack_q4(const float *W, int64_t N, int64_t K, uint8_t *out, float *deq) {
  int64_t NT = N / 64, G = K / 32;
  for (int64_t t = 0; t < NT; t++) for (int64_t g = 0; g < G; g++) {
    int64_t rec = (t * G + g) * 1280;
    for (int r = 0; r < 64; r++) {
      int64_t n = t * 64 + r, base = n * K + g * 32; double mnv = INFINITY, mxv = -INFINITY;
      for (int i = 0; i < 32; i++) { double v = W[base + i]; if (v < mnv) mnv = v; if (v > mxv) mxv = v; }
      double mn = rf16(mnv); double s = rf16((mxv - mn) / 15.0); if (s == 0.0) s = 1.0;
      for (int j = 0; j < 16; j++) {
        double q0 = fmin(15.0, fmax(0.0, rhe((W[base + 2 * j] - mn) / s)));
        double q1 = fmin(15.0, fmax(0.0, rhe((W[base + 2 * j + 1] - mn) / s)));
        out[rec + r * 16 + j] = (uint8_t)((int)q0 | ((int)q1 << 4));
        if (deq) { deq[base + 2 * j] = (float)(q0 * s + mn); deq[base + 2 * j + 1] = (float)(q1 * s + mn); }
      }
      uint32_t word = (uint32_t)or_f2h(s) | ((uint32_t)or_f2h(mn) << 16);
      memcpy(out + rec + 1024 + r * 4, &word, 4);   /* little-endian host, as DataView(..., true) */
    }
  }
}

/* packQ8 -> q8g64s.t64: record (t, g = k/64) of 4224 B: byte r*64 + i = int8 q; u16 at 4096 + 2r = f16(s). */
void or_pack_q8(const float *W, int64_t N, int64_t K, uint8_t *out, float *deq) {
  int64_t NT = N / 64, G = K / 64;
  for (int64_t t = 0; t < NT; t++) for (int64_t g = 0; g < G; g++) {
    int64_t rec = (t * G + g) * 4224;
    for (int r = 0; r < 64; r++) {
      int64_t n = t * 64 + r, base = n * K + g * 64; double am = 0;
      for (int i = 0; i < 64; i++) am = fmax(am, fabs((double)W[base + i]));
      double s = rf16(am / 127.0); if (s == 0.0) s = 1.0;
      for (int i = 0; i < 64; i++) {
        double q = fmin(127.0, fmax(-128.0, rhe(W[base + i] / s)));
        out[rec + r * 64 + i] = (uint8_t)(((int)q) & 255);
        if (deq) deq[base + i] = (float)(q * s);
      }
      uint16_t hs = or_f2h(s); memcpy(out + rec + 4096 + r * 2, &hs, 2);
    }
  }
}

/* the f16 weight each GEMM tile element carries: q4 ops/gemm.js:147-148 `vec4<f16>(cv*sc + mn)`, q8 :158-159 `vec4<f16>(cv*sc)` */
void or_deq16_q4(const uint8_t *w, int64_t N, int64_t K, uint16_t *out) {
  int64_t G = K / 32;
  for (int64_t n = 0; n < N; n++) for (int64_t k = 0; k < K; k++) {
    int64_t rec = ((n / 64) * G + k / 32) * 1280; int r = (int)(n % 64), kk = (int)(k % 32);
    uint8_t b = w[rec + r * 16 + kk / 2]; uint32_t q = (kk & 1) ? (b >> 4) : (b & 15u);
    uint32_t sm; memcpy(&sm, w + rec + 1024 + r * 4, 4);
    float s = h2f32((uint16_t)(sm & 0xffffu)), mn = h2f32((uint16_t)(sm >> 16));
    float f = (float)q * s + mn;    /* q*s is exact in f32, so contraction or not gives the same f32 */
    out[n * K + k] = or_f2h(f);
  }
}
void or_deq16_q8(const uint8_t *w, int64_t N, int64_t K, uint16_t *out) {
  int64_t G = K / 64;
  for (int64_t n = 0; n < N; n++) for (int64_t k = 0; k < K; k++) {
    int64_t rec = ((n / 64) * G + k / 64) * 4224; int r = (int)(n % 64), kk = (int)(k % 64);
    int8_t q = (int8_t)w[rec + r * 64 + kk]; uint16_t hs; memcpy(&hs, w + rec + 4096 + r * 2, 2);
    out[n * K + k] = or_f2h((float)q * h2f32(hs));
  }
}

/* ------------------------------------------------------------------ WGSL helpers */

/* GELU as lops.js:26 writes it (constant to 16 digits), f32 arithmetic in source order */
static inline float gelu_l(float v) {
  float u = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  u = fminf(15.0f, fmaxf(-15.0f, u));
  return v * 0.5f * (1.0f + tanhf(u));
}
/* GELU of ops/misc.js:116 / ops/gemm.js:204 (constant 0.7978845608) */
static inline float gelu_m(float x) {
  float u = 0.7978845608f * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.0f + tanhf(fminf(15.0f, fmaxf(-15.0f, u))));
}
static inline float gelu_g(float g) {   /* gemm.js:204 order: g * 0.5 * (1 + tanh(clamp(...))) */
  float u = fminf(15.0f, fmaxf(-15.0f, 0.7978845608f * (g + 0.044715f * g * g * g)));
  return g * 0.5f * (1.0f + tanhf(u));
}
static inline float silu_g(float g) { return g / (1.0f + expf(-g)); }
static inline float dot4(const float *a, const float *b) { return a[0] * b[0] + a[1] * b[1] + a[2] * b[2] + a[3] * b[3]; }
static inline float sum4(const float *a) { return a[0] * 1.0f + a[1] * 1.0f + a[2] * 1.0f + a[3] * 1.0f; }
static inline uint32_t fbits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bitsf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

enum { PRO_RAW = 0, PRO_RMS = 1, PRO_SUM = 2, PRO_PLEG = 3 };
enum { EPI_STORE = 0, EPI_GEGLU = 1, EPI_SOFTCAP = 2 };

/* the q4 record dot of one thread (lops.js:67-71 / lops_spec.js:102-107): quarter w of row r, group g */
static inline float q4_term(const uint32_t *W, uint32_t rec, uint32_t r, uint32_t w, const float *x8, float acc) {
  uint32_t q = W[rec + r * 4 + w], smw = W[rec + 256 + r];
  float sx = h2f32((uint16_t)(smw & 0xffffu)), sy = h2f32((uint16_t)(smw >> 16));
  float qa[4] = {(float)(q & 15u), (float)((q >> 4) & 15u), (float)((q >> 8) & 15u), (float)((q >> 12) & 15u)};
  float qb[4] = {(float)((q >> 16) & 15u), (float)((q >> 20) & 15u), (float)((q >> 24) & 15u), (float)((q >> 28) & 15u)};
  float d1 = dot4(qa, x8) + dot4(qb, x8 + 4);
  float d2 = sum4(x8) + sum4(x8 + 4);
  return acc + sx * d1 + sy * d2;
}
/* the q8 record dot of one thread (lops.js:72-81) */
static inline float q8_term(const uint32_t *W, uint32_t rec, uint32_t r, uint32_t w, const float *x16, float acc) {
  uint32_t s2 = W[rec + 1024 + (r >> 1)]; float sc = h2f32((uint16_t)((r & 1u) ? (s2 >> 16) : (s2 & 0xffffu)));
  float d = 0.0f;
  for (int u = 0; u < 4; u++) {
    uint32_t q = W[rec + r * 16 + w * 4 + u];
    float qv[4] = {(float)(int8_t)(q & 255u), (float)(int8_t)((q >> 8) & 255u), (float)(int8_t)((q >> 16) & 255u), (float)(int8_t)(q >> 24)};
    d = d + dot4(qv, x16 + u * 4);
  }
  return acc + sc * d;
}

/* ------------------------------------------------------------------ lgemv (lops.js:30-106) */
/* Buffers as the WGSL binds them: X, W (u32 words), Y, NW, EV, MX (the rms prologue's rstd lives in MX: lops.js:50,
 * bound to a.mx for softcap else a.stat: lops.js:125). Params = its uniform struct P. Grid [N/64 tiles, nsplit]. */
void or_gemv(int q8, int pro, int epi, const float *X, const uint32_t *W, float *Y, const float *NW, const float *EV, float *MX,
             uint32_t N, uint32_t K, uint32_t wG, uint32_t kPer, uint32_t nsplit, uint32_t ldy, uint32_t wOff, uint32_t nOff,
             uint32_t statOff, uint32_t rowB, uint32_t evOff, float cap, uint32_t ldp, uint32_t nsrc, uint32_t t0, uint32_t kch) {
  uint32_t NT = N / 64, G = q8 ? 64u : 32u, RW = q8 ? 1056u : 320u;
  float *xs = (float *)calloc(kch + 64, sizeof(float));
  for (uint32_t split = 0; split < nsplit; split++) {
    uint32_t k0 = split * kPer, k1 = k0 + kPer < K ? k0 + kPer : K;
    /* prologue: x chunk -> xs */
    float rs = pro == PRO_RMS ? MX[statOff] : 0.0f;
    for (uint32_t k = k0; k < k1; k++) {
      float v;
      if (pro == PRO_RAW) v = X[rowB + k];
      else if (pro == PRO_RMS) v = X[rowB + k] * rs * NW[nOff + k];
      else { float s = 0.0f; for (uint32_t j = 0; j < nsrc; j++) s = s + X[j * ldp + k]; v = pro == PRO_SUM ? s : gelu_l(s) * EV[evOff + k]; }
      xs[k - k0] = v;
    }
    uint32_t g0 = k0 / G, g1 = (k1 + G - 1) / G;
    /* tiles are independent (each writes its own Y rows and MX slot): spread over the host's threads, every tile's
     * arithmetic unchanged */
#ifdef _OPENMP
#pragma omp parallel for schedule(static) if (NT >= 16)
#endif
    for (uint32_t tile = 0; tile < NT; tile++) {
      float tot[2][64];
      int npair = epi == EPI_GEGLU ? 2 : 1;
      for (int ti = 0; ti < npair; ti++) {
        uint32_t tb = (ti == 0 ? tile : tile + N / 64) * wG;
        for (uint32_t r = 0; r < 64; r++) {
          float red[4];
          for (uint32_t w = 0; w < 4; w++) {
            float acc = 0.0f;
            for (uint32_t g = g0; g < g1; g++) {
              uint32_t rec = wOff + (tb + g) * RW;
              if (!q8) acc = q4_term(W, rec, r, w, xs + (g * 32 - k0 + w * 8), acc);
              else acc = q8_term(W, rec, r, w, xs + (g * 64 - k0 + w * 16), acc);
            }
            red[w] = acc;
          }
          tot[ti][r] = red[0] + red[1] + red[2] + red[3];
        }
      }
      uint32_t tg = tile + t0;
      if (epi == EPI_STORE) { for (uint32_t r = 0; r < 64; r++) Y[split * ldy + tg * 64 + r] = tot[0][r]; }
      else if (epi == EPI_GEGLU) { for (uint32_t r = 0; r < 64; r++) Y[tg * 64 + r] = gelu_l(tot[0][r]) * tot[1][r]; }
      else {
        float mxv[64]; uint32_t mxi[64];
        for (uint32_t r = 0; r < 64; r++) {
          float t = tot[0][r] / cap; t = fminf(15.0f, fmaxf(-15.0f, t));
          float v = cap * tanhf(t); Y[tg * 64 + r] = v; mxv[r] = v; mxi[r] = r;
        }
        for (uint32_t s = 32; s > 0; s >>= 1)
          for (uint32_t li = 0; li < s; li++) {
            float a = mxv[li], b = mxv[li + s];
            if (b > a || (b == a && mxi[li + s] < mxi[li])) { mxv[li] = b; mxi[li] = mxi[li + s]; }
          }
        MX[tg * 2] = mxv[0]; MX[tg * 2 + 1] = bitsf(tg * 64 + mxi[0]);
      }
    }
  }
  free(xs);
}

/* ------------------------------------------------------------------ lgemvM (lops_spec.js:44-157) */
void or_gemvM(int q8, int pro, int epi, uint32_t M, const float *X, const uint32_t *W, float *Y, const float *NW, const float *EV,
              const float *ST, float *MX, uint32_t N, uint32_t K, uint32_t wG, uint32_t kPer, uint32_t ldy, uint32_t ldm, uint32_t ldx,
              uint32_t wOff, uint32_t nOff, uint32_t statOff, uint32_t statLd, uint32_t rowB, uint32_t evOff, uint32_t evLd, float cap,
              uint32_t nsrc, uint32_t ldp, uint32_t t0, uint32_t ntile) {
  uint32_t NT = N / 64, G = q8 ? 64u : 32u, RW = q8 ? 1056u : 320u, nsplit = (K + kPer - 1) / kPer;
  int npair = epi == EPI_GEGLU ? 2 : 1;
  float *xs = (float *)malloc(sizeof(float) * (size_t)M * (K + 64));
  float *acc = (float *)malloc(sizeof(float) * (size_t)2 * M * 64 * 4);
  for (uint32_t split = 0; split < nsplit; split++) {
    uint32_t k0 = split * kPer, k1 = k0 + kPer < K ? k0 + kPer : K;
    /* pro(m, k), staged once for the split (the WGSL restages per xch sub-chunk with the same values) */
    for (uint32_t m = 0; m < M; m++) for (uint32_t k = k0; k < k1; k++) {
      float v;
      if (pro == PRO_RAW) v = X[m * ldx + rowB + k];
      else if (pro == PRO_RMS) v = X[m * ldx + rowB + k] * ST[statOff + m * statLd] * NW[nOff + k];
      else { float s = 0.0f; for (uint32_t j = 0; j < nsrc; j++) s = s + X[j * ldp + m * ldx + k]; v = gelu_l(s) * EV[evOff + m * evLd + k]; }
      xs[(size_t)m * (K + 64) + (k - k0)] = v;
    }
    uint32_t g0 = k0 / G, g1 = (k1 + G - 1) / G;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) if (NT >= 16)
#endif
    for (uint32_t tile = 0; tile < NT; tile++) {
      float tot[2][8][64];
      for (int ti = 0; ti < npair; ti++) {
        uint32_t tb = (ti == 0 ? tile : tile + N / 64) * wG;
        for (uint32_t r = 0; r < 64; r++) for (uint32_t m = 0; m < M; m++) {
          float red[4];
          for (uint32_t w = 0; w < 4; w++) {
            float a = 0.0f;
            for (uint32_t g = g0; g < g1; g++) {
              uint32_t rec = wOff + (tb + g) * RW; const float *xm = xs + (size_t)m * (K + 64);
              if (!q8) a = q4_term(W, rec, r, w, xm + (g * 32 - k0 + w * 8), a);
              else a = q8_term(W, rec, r, w, xm + (g * 64 - k0 + w * 16), a);
            }
            red[w] = a;
          }
          tot[ti][m][r] = red[0] + red[1] + red[2] + red[3];
        }
      }
      uint32_t tg = tile + t0;
      for (uint32_t m = 0; m < M; m++) {
        if (epi == EPI_STORE) { for (uint32_t r = 0; r < 64; r++) Y[split * ldy + m * ldm + tg * 64 + r] = tot[0][m][r]; }
        else if (epi == EPI_GEGLU) { for (uint32_t r = 0; r < 64; r++) Y[m * ldm + tg * 64 + r] = gelu_l(tot[0][m][r]) * tot[1][m][r]; }
        else {
          float mxv[64]; uint32_t mxi[64];
          for (uint32_t r = 0; r < 64; r++) {
            float t = fminf(15.0f, fmaxf(-15.0f, tot[0][m][r] / cap));
            float v = cap * tanhf(t); Y[m * ldm + tg * 64 + r] = v; mxv[r] = v; mxi[r] = r;
          }
          for (uint32_t s = 32; s > 0; s >>= 1)
            for (uint32_t li = 0; li < s; li++) {
              float a = mxv[li], b = mxv[li + s];
              if (b > a || (b == a && mxi[li + s] < mxi[li])) { mxv[li] = b; mxi[li] = mxi[li + s]; }
            }
          uint32_t o = (m * ntile + tg) * 2; MX[o] = mxv[0]; MX[o + 1] = bitsf(tg * 64 + mxi[0]);
        }
      }
    }
  }
  free(xs); free(acc);
}

/* ------------------------------------------------------------------ gemm (ops/gemm.js:25-253), x prologue 'f16' */
enum { GE_F16 = 0, GE_F32 = 1, GE_BIAS = 2, GE_RESADD = 3, GE_SWIGLU = 4 };
enum { WQ4 = 0, WQ8 = 1, WF16 = 2 };

/* f16 FMA with one rounding (the WGSL fma on vec4<f16>: acc 'f16' path, gemm.js:177) */
static inline uint16_t hfma(uint16_t a, uint16_t b, uint16_t c) {
  double r = or_h2f(a) * or_h2f(b) + or_h2f(c);   /* exact in f64: 11+11 bit product plus an fp16 */
  /* round the exact value straight to fp16 (not via f32) */
  double ar = fabs(r); if (!(ar == ar)) return 0x7e00;
  if (ar == 0) return (r < 0 || (r == 0 && signbit(r))) ? 0x8000 : 0;
  int e; frexp(ar, &e);                   /* ar = f * 2^e, f in [0.5,1) */
  int ulpe = (e - 1) - 10; if (ulpe < -24) ulpe = -24;
  double q = ar / ldexp(1.0, ulpe), fq = floor(q), d = q - fq;
  if (d > 0.5 || (d == 0.5 && fmod(fq, 2.0) != 0)) fq += 1;
  double v = fq * ldexp(1.0, ulpe);
  uint16_t h = or_f2h(r < 0 ? -v : v);    /* v is exactly representable (or overflows to inf) */
  return h;
}

/* hfma with a and b given as doubles (their fp16 values) and c through a table: the same value a*b + c and the same
 * rounding, by arithmetic instead of frexp / floor / fmod. For |r| < 2^(u + 52), (r + 1.5 * 2^(u + 52)) - 1.5 * 2^(u + 52)
 * is r rounded to a multiple of 2^u, ties to even (the sum's last bit is the parity of the multiple: 1.5 * 2^52 is
 * even), where u is the fp16 ulp exponent of r, as in hfma. h2d_init() fills the table; or_gemm calls it. */
static double h2d_tab[65536];
static int h2d_ready;
static void h2d_init(void) {
  if (h2d_ready) return;
  for (uint32_t i = 0; i < 65536u; i++) h2d_tab[i] = or_h2f((uint16_t)i);
  h2d_ready = 1;
}
static inline uint16_t hfma_d(double a, double b, uint16_t c) {
  double r = a * b + h2d_tab[c];
  if (!(r == r)) return 0x7e00;
  if (r == 0) return signbit(r) ? 0x8000 : 0;
  if (isinf(r)) return r < 0 ? 0xfc00 : 0x7c00;
  double ar = fabs(r);
  uint64_t bits; memcpy(&bits, &ar, 8);
  int ulpe = (int)((bits >> 52) & 0x7ffu) - 1033;        /* frexp's e - 11: ar = f * 2^e, f in [0.5, 1) */
  if (ulpe < -24) ulpe = -24;
  uint64_t sb = ((uint64_t)(ulpe + 52 + 1023) << 52) | 0x8000000000000ull;   /* 1.5 * 2^(ulpe + 52) */
  double sm; memcpy(&sm, &sb, 8);
  volatile double t = ar + sm;                             /* rounded once, to nearest even */
  double v = t - sm;
  return or_f2h(r < 0 ? -v : v);
}

/* the fp16 weight tile element (row, k) the WGSL dequantises into ws[] */
static inline uint16_t wtile(int wenc, const uint32_t *W, uint32_t row, uint32_t kabs, uint32_t wG) {
  if (wenc == WQ4) {
    uint32_t gi = kabs / 32, rec = ((row >> 6) * wG + gi) * 320, rr = row & 63, kk = kabs % 32;
    uint32_t q = W[rec + rr * 4 + kk / 8]; uint32_t cv = (q >> (4 * (kk % 8))) & 15u; uint32_t sm = W[rec + 256 + rr];
    float f = (float)cv * h2f32((uint16_t)(sm & 0xffffu)) + h2f32((uint16_t)(sm >> 16));
    return or_f2h(f);
  } else if (wenc == WQ8) {
    uint32_t gi = kabs / 64, rec = ((row >> 6) * wG + gi) * 1056, rr = row & 63, kk = kabs % 64;
    uint32_t q = W[rec + rr * 16 + kk / 4]; int8_t cv = (int8_t)((q >> (8 * (kk % 4))) & 255u);
    uint32_t s2 = W[rec + 1024 + (rr >> 1)]; float sc = h2f32((uint16_t)((rr & 1u) ? (s2 >> 16) : (s2 & 0xffffu)));
    return or_f2h((float)cv * sc);
  } else {
    const uint16_t *H = (const uint16_t *)W; return H[(size_t)row * wG + kabs];
  }
}

/* One GEMM call. Y is u16 (fp16) for f16/bias/swiglu epilogues, f32 for f32/resadd. post_gelu applies ew op 4 (misc.js:126,
 * `B = f16(gelu(f32(B)))` in place) after a 'bias' store, i.e. gemm(epi:'bias') -> ew(op:'gelu') as pocketflux-engine.js:3052-3053.
 * Threads: rows m of the 64-row M tile x columns of the BN tile, as gemm.js:170-211 with TM = TN = 8 (row/col independent). */
void or_gemm(int wenc, int epi, int acc16, int act_gelu, int res, int store, int gate, int bias, int post_gelu,
             const uint16_t *X, const uint32_t *W, void *Yv, const float *EV, const float *BV,
             uint32_t M, uint32_t N, uint32_t K, uint32_t ldx, uint32_t kx0, uint32_t wR0, uint32_t wR1, uint32_t wG, uint32_t wk0,
             uint32_t ldy, uint32_t ny0, uint32_t Nw, uint32_t evOff, uint32_t bvOff, uint32_t bvUp, int nthreads) {
  uint16_t *Yh = (uint16_t *)Yv; float *Yf = (float *)Yv;
  uint32_t BN = 128, ntiles = (N + BN - 1) / BN;
  const uint32_t ncol = ntiles * BN;
  (void)nthreads;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#endif
  /* The W tile of every column (gemm.js:96-160: the column's weight row, f16(q*s + mn) / f16(q*s)) and the X values,
   * dequantised and converted once per call instead of once per multiply: the same values, so every output's
   * arithmetic and summation order below are unchanged. */
  uint16_t *Wh = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)ncol * K);
#ifdef _OPENMP
#pragma omp parallel for schedule(static) if (nthreads != 1)
#endif
  for (int64_t nn = 0; nn < (int64_t)ncol; nn++) {
    const uint32_t n = (uint32_t)nn, cc = n % BN;
    const uint32_t row = epi == GE_SWIGLU ? (((cc & 1u) == 0u ? wR0 : wR1) + (n >> 1)) : (wR0 + n < Nw - 1 ? wR0 + n : Nw - 1);
    for (uint32_t k = 0; k < K; k++) Wh[(size_t)n * K + k] = wtile(wenc, W, row, wk0 + k, wG);
  }
  float *Wf = NULL, *Xf = NULL;
  double *Wd = NULL, *Xd = NULL;
  if (acc16) {
    h2d_init();
    Wd = (double *)malloc(sizeof(double) * (size_t)ncol * K);
    Xd = (double *)malloc(sizeof(double) * (size_t)M * K);
    for (size_t i = 0; i < (size_t)ncol * K; i++) Wd[i] = h2d_tab[Wh[i]];
    for (uint32_t m = 0; m < M; m++)
      for (uint32_t k = 0; k < K; k++) Xd[(size_t)m * K + k] = h2d_tab[X[(size_t)m * ldx + kx0 + k]];
  } else {
    Wf = (float *)malloc(sizeof(float) * (size_t)ncol * K);
    Xf = (float *)malloc(sizeof(float) * (size_t)M * K);
    for (size_t i = 0; i < (size_t)ncol * K; i++) Wf[i] = h2f32(Wh[i]);
    for (uint32_t m = 0; m < M; m++)
      for (uint32_t k = 0; k < K; k++) Xf[(size_t)m * K + k] = h2f32(X[(size_t)m * ldx + kx0 + k]);
  }
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) if (nthreads != 1)
#endif
  for (int64_t mm = 0; mm < (int64_t)M; mm++) {
    uint32_t m = (uint32_t)mm;
    float *a = (float *)malloc(sizeof(float) * ntiles * BN);
    for (uint32_t n = 0; n < ncol; n++) {
      float acc = 0.0f;
      for (uint32_t k0 = 0; k0 < K; k0 += 32) {
        if (acc16) {
          uint16_t h = 0;
          const double *wv = Wd + (size_t)n * K + k0, *xv = Xd + (size_t)m * K + k0;
          for (uint32_t k = 0; k < 32; k++) h = hfma_d(xv[k], wv[k], h);
          acc = acc + h2f32(h);
        } else {
          const float *wv = Wf + (size_t)n * K + k0, *xv = Xf + (size_t)m * K + k0;
          for (uint32_t k = 0; k < 32; k++) acc = fmaf(xv[k], wv[k], acc);
        }
      }
      a[n] = acc;
    }
    /* epilogues (gemm.js:190-211): columns in vec4 units, col < N checks per vec4 */
    if (epi == GE_SWIGLU) {
      for (uint32_t nt = 0; nt < ntiles; nt++) for (uint32_t j = 0; j < BN / 2; j++) {
        uint32_t nB = nt * BN, on = (nB >> 1) + j;
        float gB = bias ? BV[bvOff + on] : 0.0f, uB = bias ? BV[bvOff + bvUp + on] : 0.0f;
        float g = a[nB + 2 * j] + gB, u = a[nB + 2 * j + 1] + uB;
        float act = act_gelu ? gelu_g(g) : silu_g(g);
        Yh[(size_t)m * ldy + ny0 + on] = or_f2h(act * u);
      }
    } else {
      for (uint32_t col = 0; col < ntiles * BN; col += 4) {
        if (!(col < N)) continue;
        for (uint32_t i = 0; i < 4; i++) {
          uint32_t n = col + i; size_t yi = (size_t)m * ldy + ny0 + n; float v = a[n];
          if (epi == GE_F16) Yh[yi] = or_f2h(v);
          else if (epi == GE_F32) Yf[yi] = v;
          else if (epi == GE_BIAS) {
            float t = v + EV[evOff + n];
            if (res) t = t + h2f32(Yh[yi]);
            uint16_t h = or_f2h(t);
            if (post_gelu) h = or_f2h(gelu_m(h2f32(h)));
            Yh[yi] = h;
          } else {   /* resadd: Y = [Y +] g * (acc + c) */
            float g = gate ? EV[evOff + n] : 1.0f, c = bias ? BV[bvOff + n] : 0.0f;
            float t = g * (v + c);
            Yf[yi] = store ? t : Yf[yi] + t;
          }
        }
      }
    }
    free(a);
  }
  free(Wh);
  free(Wf);
  free(Xf);
  free(Wd);
  free(Xd);
}

/* ------------------------------------------------------------------ f64 references and the timed CPU baseline */

/* y[m][n] = sum_k deq[n][k] * x[m][k] in f64 (kcheck.js:133, kshipped.js:34 style) */
void or_dot64(const float *deq, const double *x, int64_t M, int64_t N, int64_t K, double *y) {
  for (int64_t m = 0; m < M; m++) for (int64_t n = 0; n < N; n++) {
    double s = 0; const float *w = deq + n * K; const double *xm = x + m * K;
    for (int64_t k = 0; k < K; k++) s += (double)w[k] * xm[k];
    y[m * N + n] = s;
  }
}

/* The CPU baseline: the same lgemvM arithmetic (per row: 4 quarter lanes over groups, then summed), threaded over
 * 64-row tiles with OpenMP. Prologue raw, epilogue store, q4. Returns nothing; writes Y[m*N + n]. */
void or_gemv_cpu_mt(const float *X, const uint32_t *W, float *Y, uint32_t M, uint32_t N, uint32_t K, uint32_t wG, int nthreads) {
  uint32_t NT = N / 64, G = K / 32;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
  for (int64_t t = 0; t < (int64_t)NT; t++) {
    for (uint32_t m = 0; m < M; m++) {
      const float *xm = X + (size_t)m * K;
      for (uint32_t r = 0; r < 64; r++) {
        float red[4];
        for (uint32_t w = 0; w < 4; w++) {
          float acc = 0.0f;
          for (uint32_t g = 0; g < G; g++) acc = q4_term(W, (uint32_t)((t * wG + g) * 320), r, w, xm + g * 32 + w * 8, acc);
          red[w] = acc;
        }
        Y[(size_t)m * N + t * 64 + r] = red[0] + red[1] + red[2] + red[3];
      }
    }
  }
}
int or_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------------ array helpers for the Python wrapper */
void or_f2h_arr(const double *x, int64_t n, uint16_t *o) { for (int64_t i = 0; i < n; i++) o[i] = or_f2h(x[i]); }
void or_h2f_arr(const uint16_t *h, int64_t n, double *o) { for (int64_t i = 0; i < n; i++) o[i] = or_h2f(h[i]); }
void or_hfma_arr(const uint16_t *a, const uint16_t *b, const uint16_t *c, int64_t n, uint16_t *o) { for (int64_t i = 0; i < n; i++) o[i] = hfma(a[i], b[i], c[i]); }
/* the table / add-and-subtract form the GEMM uses, for the check that it equals hfma */
void or_hfma_d_arr(const uint16_t *a, const uint16_t *b, const uint16_t *c, int64_t n, uint16_t *o) {
  h2d_init();
  for (int64_t i = 0; i < n; i++) o[i] = hfma_d(h2d_tab[a[i]], h2d_tab[b[i]], c[i]);
}

/* ------------------------------------------------------------------ GEMM x prologues (ops/gemm.js:55-63)
 * The fp16 X the reference's xload() yields for the f32 x modes: row m, k = 0..K-1 of X f32 [row * ldx + kx0 + k],
 * stats ST[(statOff + m) * 2] = {mean, rstd}, vectors PV (scale at pvOff, shift at pvOff + pvStride, indexed by
 * kx0 + k), in the WGSL's order of operations:
 *   lnmod: f16(((x - mean) * rstd) * (1 + PV[pvOff + k']) + PV[pvOff + pvStride + k'])
 *   rms:   f16((x * rstd) * PV[pvOff + k'])                                        (k' = kx0 + k) */
void or_gemm_xpro(int mode, const float *X, uint32_t M, uint32_t K, uint32_t ldx, uint32_t kx0, const float *ST, uint32_t statOff,
                  const float *PV, uint32_t pvOff, uint32_t pvStride, uint16_t *out) {
  for (uint32_t m = 0; m < M; m++) {
    const float mean = ST[(size_t)(statOff + m) * 2], rstd = ST[(size_t)(statOff + m) * 2 + 1];
    for (uint32_t k = 0; k < K; k++) {
      const uint32_t kk = kx0 + k;
      const float x = X[(size_t)m * ldx + kk];
      float v;
      if (mode == 1) {
        v = x - mean;
        v = v * rstd;
        v = v * (1.0f + PV[pvOff + kk]);
        v = v + PV[pvOff + pvStride + kk];
      } else {
        v = x * rstd;
        v = v * PV[pvOff + kk];
      }
      out[(size_t)m * K + k] = or_f2h((double)v);
    }
  }
}

/* ------------------------------------------------------------------ GEMM epilogues that reduce over one 128-wide head
 * (ops/gemm.js:212-250), applied to the f32 accumulators A[m * N + n] of one call (N % 128 == 0, one head per 128
 * columns, hd = n / 128). Per row and head, s = the sum of the 128 squared accumulators, summed as the WGSL does without
 * subgroups: 16 threads tx each take dot(a_0, a_0) + dot(a_1, a_1) over their 8 columns (rope 'half': columns
 * 4tx..4tx+3 and 64+4tx..; else 8tx..8tx+7), then one thread adds the 16 in order; inv = inverseSqrt(s / 128 + eps).
 *   onormgate (:223-229): Y[m*ldy + ny0 + n] = f16(a * inv * EV[evOff + c] / (1 + exp(-f32(GT[m*Ltot + ny0 + n])))), c = n % 128
 *     (the vec4 indices floor (m*Ltot + ny0 + n) / 4 like the WGSL's u32 division)
 *   heads (:231-249): section sec = 0 (q) for hd < Hq, 1 (k) for hd < Hq + Hkv, else 2 (v); row = rowOff + m.
 *     q / k: v = a * inv * EV[evOff + (sec ? 128 : 0) + c], then RoPE from RP (per row 128 floats):
 *       rope_half (rotate_half, pairs (d, d + 64)): cos = RP[row*128 + 2d], sin = RP[row*128 + 2d + 1],
 *         out[d] = v[d]*cos - v[d+64]*sin, out[d+64] = v[d+64]*cos + v[d]*sin   (d < 64)
 *       interleaved (pairs (2p, 2p+1)): cos = RP[row*128 + 2p], sin = RP[row*128 + 2p + 1],
 *         out[2p] = v[2p]*cos - v[2p+1]*sin, out[2p+1] = v[2p]*sin + v[2p+1]*cos
 *     v: out = a. Stored head-major: Y[(hd*Ltot + row)*128 + c] = f16(out[c]). */
void or_gemm_red128(int onormgate, int rope_half, const float *A, uint32_t M, uint32_t N, uint16_t *Y, const float *EV,
                    uint32_t evOff, const uint16_t *GT, const float *RP, uint32_t ldy, uint32_t ny0, uint32_t rowOff,
                    uint32_t Ltot, uint32_t Hq, uint32_t Hkv, float eps) {
  const int split = !onormgate && rope_half;
  for (uint32_t m = 0; m < M; m++) {
    for (uint32_t hd = 0; hd < N / 128; hd++) {
      const float *a = A + (size_t)m * N + hd * 128;
      float s = 0.0f;
      for (uint32_t tx = 0; tx < 16; tx++) {
        const uint32_t i0 = split ? tx * 4 : tx * 8, i1 = split ? 64 + tx * 4 : tx * 8 + 4;
        s = s + (dot4(a + i0, a + i0) + dot4(a + i1, a + i1));
      }
      const float inv = (float)(1.0 / sqrt((double)(s / 128.0f + eps)));
      if (onormgate) {
        const size_t gb = ((size_t)m * Ltot + ny0) & ~(size_t)3, yb = ((size_t)m * ldy + ny0) & ~(size_t)3;
        for (uint32_t c = 0; c < 128; c++) {
          const uint32_t n = hd * 128 + c;
          const float g = h2f32(GT[gb + n]);
          float v = a[c] * inv;
          v = v * EV[evOff + c];
          v = v / (1.0f + expf(-g));
          Y[yb + n] = or_f2h((double)v);
        }
        continue;
      }
      const uint32_t sec = hd < Hq ? 0u : hd < Hq + Hkv ? 1u : 2u, row = rowOff + m;
      uint16_t *yo = Y + ((size_t)hd * Ltot + row) * 128;
      if (sec == 2) {
        for (uint32_t c = 0; c < 128; c++) yo[c] = or_f2h((double)a[c]);
        continue;
      }
      float v[128];
      for (uint32_t c = 0; c < 128; c++) {
        const float t = a[c] * inv;
        v[c] = t * EV[evOff + (sec ? 128u : 0u) + c];
      }
      const float *rp = RP + (size_t)row * 128;
      if (split) {
        for (uint32_t d = 0; d < 64; d++) {
          const float cs = rp[2 * d], sn = rp[2 * d + 1];
          const float lo = v[d] * cs - v[d + 64] * sn, hi = v[d + 64] * cs + v[d] * sn;
          yo[d] = or_f2h((double)lo);
          yo[d + 64] = or_f2h((double)hi);
        }
      } else {
        for (uint32_t p = 0; p < 64; p++) {
          const float cs = rp[2 * p], sn = rp[2 * p + 1];
          const float x0 = v[2 * p], x1 = v[2 * p + 1];
          yo[2 * p] = or_f2h((double)(x0 * cs - x1 * sn));
          yo[2 * p + 1] = or_f2h((double)(x0 * sn + x1 * cs));
        }
      }
    }
  }
}

/* ------------------------------------------------------------------ decode-path operators around the GEMV
 * argmax / argmaxM (engine/llm/lops.js:416-436, lops_spec.js:326-348): for each row m of n (max, bitcast index) pairs,
 * OUT[2m] = the index of the largest max, ties to the lowest index, NaN maxima never win (start: -3.4e38, index
 * 0xffffffff); OUT[2m + 1] = the bits of that max. The tie rule makes the result independent of the scan order. */
void or_argmaxM(const float *MX, uint32_t n, uint32_t M, uint32_t *OUT) {
  for (uint32_t m = 0; m < M; m++) {
    float bv = -3.4e38f; uint32_t bi = 0xffffffffu;
    for (uint32_t i = 0; i < n; i++) {
      const float v = MX[2 * ((size_t)m * n + i)]; uint32_t id; memcpy(&id, &MX[2 * ((size_t)m * n + i) + 1], 4);
      if (v > bv || (v == bv && id < bi)) { bv = v; bi = id; }
    }
    OUT[2 * m] = bi; memcpy(&OUT[2 * m + 1], &bv, 4);
  }
}

/* the 256-thread tree sum of the WGSL reductions: red[t] partials, halving strides 128..1 */
static float tree256(float *red) {
  for (uint32_t k = 128; k > 0; k >>= 1) for (uint32_t t = 0; t < k; t++) red[t] = red[t] + red[t + k];
  return red[0];
}

/* embed (lops.js:323-365): x[(rowOut + m) * K + k] = dequant(E[ids[m]])[k] * scale, E a q4g32a.t64 / q8g64s.t64 table
 * [V][K] (word-indexed W); ST[statOff + m] = inverseSqrt(sum x^2 / K + eps), the sum as 256 strided thread partials
 * and the tree. q4: (f32(q) * s + mn) * scale; q8: f32(q) * s * scale. */
void or_embed(int q8, const uint32_t *W, const uint32_t *IDS, uint32_t n, uint32_t K, uint32_t wG, float scale, float eps,
              uint32_t statOff, uint32_t rowOut, float *X, float *ST) {
  float red[256];
  for (uint32_t m = 0; m < n; m++) {
    const uint32_t id = IDS[m], tile = id >> 6, r = id & 63u;
    for (uint32_t t = 0; t < 256; t++) {
      float s = 0.0f;
      for (uint32_t k = t; k < K; k += 256) {
        float v;
        if (q8) {
          const uint32_t gi = k >> 6, rec = (tile * wG + gi) * 1056u, kk = k & 63u;
          const uint32_t qb = (W[rec + r * 16u + (kk >> 2)] >> (8u * (kk & 3u))) & 255u;
          const float qs = (float)(int32_t)(int8_t)qb;
          const uint32_t s2 = W[rec + 1024u + (r >> 1)];
          const float sc = h2f32((uint16_t)((r & 1u) ? (s2 >> 16) : (s2 & 0xffffu)));
          v = qs * sc; v = v * scale;
        } else {
          const uint32_t gi = k >> 5, rec = (tile * wG + gi) * 320u, kk = k & 31u;
          const uint32_t q = (W[rec + r * 4u + (kk >> 3)] >> (4u * (kk & 7u))) & 15u, sm = W[rec + 256u + r];
          v = (float)q * h2f32((uint16_t)(sm & 0xffffu)); v = v + h2f32((uint16_t)(sm >> 16)); v = v * scale;
        }
        X[(size_t)(rowOut + m) * K + k] = v;
        s = s + v * v;
      }
      red[t] = s;
    }
    ST[statOff + m] = (float)(1.0 / sqrt((double)(tree256(red) / (float)K + eps)));
  }
}

/* normadd (lops.js:143-180): per row m < M of D: tv = sum over the nsrc partial rows T[j * ldp + m * D + i] (j in order);
 * rs = inverseSqrt(sum tv^2 / D + eps); mode 0: x = (x + tv * rs * W[wOff + i]) * scale, mode 1: x = tv;
 * ST[statOff + m] = inverseSqrt(sum x^2 / D + eps). Sums as 256 strided partials and the tree. */
void or_normadd(const float *T, uint32_t nsrc, uint32_t ldp, const float *W, uint32_t wOff, float *X, float *ST, uint32_t statOff,
                uint32_t D, uint32_t M, uint32_t mode, float eps, float scale) {
  float red[256];
  float *tv = (float *)malloc(sizeof(float) * D);
  for (uint32_t m = 0; m < M; m++) {
    const size_t xb = (size_t)m * D;
    for (uint32_t t = 0; t < 256; t++) {
      float s = 0.0f;
      for (uint32_t i = t; i < D; i += 256) {
        float v = 0.0f;
        for (uint32_t j = 0; j < nsrc; j++) v = v + T[(size_t)j * ldp + xb + i];
        tv[i] = v; s = s + v * v;
      }
      red[t] = s;
    }
    const float rs = (float)(1.0 / sqrt((double)(tree256(red) / (float)D + eps)));
    for (uint32_t t = 0; t < 256; t++) {
      float s2 = 0.0f;
      for (uint32_t i = t; i < D; i += 256) {
        float x = X[xb + i];
        if (mode == 0) { float u = tv[i] * rs; u = u * W[wOff + i]; x = (x + u) * scale; } else x = tv[i];
        X[xb + i] = x; s2 = s2 + x * x;
      }
      red[t] = s2;
    }
    ST[statOff + m] = (float)(1.0 / sqrt((double)(tree256(red) / (float)D + eps)));
  }
  free(tv);
}

/* dhead (lops_spec.js:428-482): the drafter's head over selected clusters. Workgroup wt < nsel * tPer scores tile
 * SEL[wt / tPer] * tPer + wt % tPer of a q4 / q8 head [rows][K] (K <= 512) against xs = X * ST[statOff] * NW[nOff + k]:
 * row r's dot in 4 k-quarter lanes w (q4: group g's k = 32g + 8w..+7, acc += s * (q . x) + mn * sum(x); q8: k = 64g +
 * 16w..+15, acc += s * (q . x)), lane sums in order w = 0..3, then the tile's max with the lowest row index winning ties:
 * MX[wt * 2] = max, MX[wt * 2 + 1] = bitcast(tile * 64 + row). */
void or_dhead(int q8, const float *X, const uint32_t *W, const float *ST, const float *NW, const uint32_t *SEL, uint32_t statOff,
              uint32_t nOff, uint32_t K, uint32_t wG, uint32_t tPer, uint32_t nsel, float *MX) {
  float xs[512];
  const float rs = ST[statOff];
  for (uint32_t k = 0; k < K; k++) { float v = X[k] * rs; xs[k] = v * NW[nOff + k]; }
  for (uint32_t wt = 0; wt < nsel * tPer; wt++) {
    const uint32_t tile = SEL[wt / tPer] * tPer + (wt % tPer), tb = tile * wG;
    float best = 0.0f; uint32_t bidx = 0;
    for (uint32_t r = 0; r < 64; r++) {
      float red[4];
      for (uint32_t w = 0; w < 4; w++) {
        float acc = 0.0f;
        for (uint32_t g = 0; g < wG; g++) {
          if (q8) {
            const uint32_t rec = (tb + g) * 1056u, s2 = W[rec + 1024u + (r >> 1)];
            const float sc = h2f32((uint16_t)((r & 1u) ? (s2 >> 16) : (s2 & 0xffffu)));
            float d = 0.0f;
            for (uint32_t u = 0; u < 4; u++) {
              const uint32_t q = W[rec + r * 16u + w * 4u + u], xb = g * 64u + w * 16u + u * 4u;
              float qv[4]; for (int b = 0; b < 4; b++) qv[b] = (float)(int32_t)(int8_t)((q >> (8 * b)) & 255u);
              d = d + dot4(qv, xs + xb);
            }
            acc = acc + sc * d;
          } else {
            const uint32_t rec = (tb + g) * 320u, q = W[rec + r * 4u + w], sm = W[rec + 256u + r], xb = g * 32u + w * 8u;
            float qa[4], qb[4];
            for (int b = 0; b < 4; b++) { qa[b] = (float)((q >> (4 * b)) & 15u); qb[b] = (float)((q >> (16 + 4 * b)) & 15u); }
            const float one[4] = {1.0f, 1.0f, 1.0f, 1.0f};
            const float s = h2f32((uint16_t)(sm & 0xffffu)), mn = h2f32((uint16_t)(sm >> 16));
            const float dq = dot4(qa, xs + xb) + dot4(qb, xs + xb + 4), dx = dot4(xs + xb, one) + dot4(xs + xb + 4, one);
            acc = acc + s * dq + mn * dx;
          }
        }
        red[w] = acc;
      }
      const float tot = red[0] + red[1] + red[2] + red[3];
      if (r == 0 || tot > best) { best = tot; bidx = tile * 64u + r; }
    }
    MX[wt * 2] = best; memcpy(&MX[wt * 2 + 1], &bidx, 4);
  }
}

/* qkrope (lops.js:183-233), decode: per head h of [q (nq) | k (nkv) | v (nkv)] (k and v only when hasKV): hv = the sum
 * of the nsrc partial rows S[j * ldp + h * D + i]; rs = inverseSqrt(sum hv^2 / D + eps) (256 strided partials, tree).
 * v heads: VC[(kvh * kvLen + kvRow) * D + i] = f16(hv[i] * rs). q / k heads, d < D/2: a = hv[d] * rs * NW[wo + d],
 * b = hv[d + D/2] * rs * NW[wo + d + D/2] (wo = qwOff or kwOff); (c, s) = RP[ropeOff + (pos * npairs + d) * 2 ..] for
 * d < npairs, else (1, 0); lo = a c - b s, hi = b c + a s: q -> Q[h * D + d] = lo, Q[h * D + d + D/2] = hi (f32);
 * k -> KC[(kvh * kvLen + kvRow) * D + d] = f16(lo), [.. + d + D/2] = f16(hi). */
void or_qkrope(const float *S, uint32_t nsrc, uint32_t ldp, const float *NW, const float *RP, float *Q, uint16_t *KC, uint16_t *VC,
               uint32_t D, uint32_t nq, uint32_t nkv, int hasKV, uint32_t pos, float eps, uint32_t qwOff, uint32_t kwOff,
               uint32_t npairs, uint32_t ropeOff, uint32_t kvRow, uint32_t kvLen) {
  float *hv = (float *)malloc(sizeof(float) * D);
  float red[256];
  const uint32_t nh = nq + (hasKV ? 2 * nkv : 0), half = D / 2;
  for (uint32_t h = 0; h < nh; h++) {
    const size_t base = (size_t)h * D;
    for (uint32_t t = 0; t < 256; t++) {
      float s = 0.0f;
      for (uint32_t i = t; i < D; i += 256) {
        float v = 0.0f;
        for (uint32_t j = 0; j < nsrc; j++) v = v + S[(size_t)j * ldp + base + i];
        hv[i] = v; s = s + v * v;
      }
      red[t] = s;
    }
    const float rs = (float)(1.0 / sqrt((double)(tree256(red) / (float)D + eps)));
    const int isV = h >= nq + nkv;
    const uint32_t kvh = isV ? h - nq - nkv : h - nq;
    const size_t cb = ((size_t)kvh * kvLen + kvRow) * D;
    if (isV) { for (uint32_t i = 0; i < D; i++) VC[cb + i] = or_f2h((double)(hv[i] * rs)); continue; }
    const uint32_t wo = h >= nq ? kwOff : qwOff;
    for (uint32_t d = 0; d < half; d++) {
      float a = hv[d] * rs; a = a * NW[wo + d];
      float b = hv[d + half] * rs; b = b * NW[wo + d + half];
      float c = 1.0f, sn = 0.0f;
      if (d < npairs) { const size_t rb = ropeOff + ((size_t)pos * npairs + d) * 2; c = RP[rb]; sn = RP[rb + 1]; }
      const float lo = a * c - b * sn, hi = b * c + a * sn;
      if (h < nq) { Q[base + d] = lo; Q[base + d + half] = hi; }
      else { KC[cb + d] = or_f2h((double)lo); KC[cb + d + half] = or_f2h((double)hi); }
    }
  }
  free(hv);
}

/* attnDec + its combine (lops.js:236-321), decode attention over keys [kStart, kEnd) in chunks of 64: Q f32 [nh][D];
 * KC / VC fp16 head-major [nkv][kvLen][D] (query head hh reads KV head hh / (nh / nkv)); cache row of key j is j % ring
 * when ring > 0. Per chunk: s[hh][j] = sum over d of f32(K) Q in 4-wide steps, m = max, p = exp(s - m), l = sum p,
 * acc[hh][d] = sum_k p V (keys in order); combine per head: M = max m_c, w_c = exp(m_c - M), L = sum w_c l_c,
 * O[hh][d] = sum_c (w_c / L) acc_c[hh][d]. No score scale (the callers fold it into q). */
void or_attn_dec(const float *Q, const uint16_t *KC, const uint16_t *VC, float *O, uint32_t D, uint32_t nh, uint32_t nkv,
                 uint32_t kvLen, uint32_t kStart, uint32_t kEnd, uint32_t ring) {
  const uint32_t nchunk = (kEnd - kStart + 63) / 64, hpg = nh / nkv;
  float *m = (float *)malloc(sizeof(float) * nchunk * nh), *l = (float *)malloc(sizeof(float) * nchunk * nh);
  float *acc = (float *)calloc((size_t)nchunk * nh * D, sizeof(float));
  float sc[64];
  for (uint32_t c = 0; c < nchunk; c++) {
    const uint32_t j0 = kStart + c * 64, nk = kEnd - j0 < 64 ? kEnd - j0 : 64;
    for (uint32_t hh = 0; hh < nh; hh++) {
      const uint32_t g = hh / hpg;
      float mx = -3.0e38f;
      for (uint32_t j = 0; j < nk; j++) {
        const uint32_t row = ring ? (j0 + j) % ring : j0 + j;
        const uint16_t *k = KC + ((size_t)g * kvLen + row) * D;
        float s = 0.0f;
        for (uint32_t d = 0; d < D; d += 4) {
          float t = h2f32(k[d]) * Q[(size_t)hh * D + d];
          for (uint32_t e = 1; e < 4; e++) t = t + h2f32(k[d + e]) * Q[(size_t)hh * D + d + e];
          s = s + t;
        }
        sc[j] = s; mx = s > mx ? s : mx;
      }
      float ls = 0.0f;
      for (uint32_t j = 0; j < nk; j++) { sc[j] = expf(sc[j] - mx); ls = ls + sc[j]; }
      m[c * nh + hh] = mx; l[c * nh + hh] = ls;
      float *a = acc + ((size_t)c * nh + hh) * D;
      for (uint32_t j = 0; j < nk; j++) {
        const uint32_t row = ring ? (j0 + j) % ring : j0 + j;
        const uint16_t *v = VC + ((size_t)g * kvLen + row) * D;
        for (uint32_t d = 0; d < D; d++) a[d] = a[d] + sc[j] * h2f32(v[d]);
      }
    }
  }
  for (uint32_t hh = 0; hh < nh; hh++) {
    float M = -3.0e38f;
    for (uint32_t c = 0; c < nchunk; c++) M = m[c * nh + hh] > M ? m[c * nh + hh] : M;
    float L = 0.0f;
    float *w = (float *)malloc(sizeof(float) * nchunk);
    for (uint32_t c = 0; c < nchunk; c++) { w[c] = expf(m[c * nh + hh] - M); L = L + w[c] * l[c * nh + hh]; }
    for (uint32_t c = 0; c < nchunk; c++) w[c] = w[c] / L;
    for (uint32_t d = 0; d < D; d++) {
      float o = 0.0f;
      for (uint32_t c = 0; c < nchunk; c++) o = o + w[c] * acc[((size_t)c * nh + hh) * D + d];
      O[(size_t)hh * D + d] = o;
    }
    free(w);
  }
  free(m); free(l); free(acc);
}
