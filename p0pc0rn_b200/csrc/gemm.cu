// gemm.cu -- the dequant-fused W4A16 GEMM on sm_100a tensor cores: gemm(gpu, a) of engine/ops/gemm.js:255-322 for
// q4g32a.t64 / q8g64s.t64 weights, the x prologues f16 / lnmod / rms, epilogues f16 / f32 / bias (+res, + the ew gelu
// that follows it) / resadd / swiglu (gemm.js:187-211) and the head-reducing heads / onormgate (gemm.js:212-250).
//
// Y[m, n] = sum_k X[m, k] * Wdq[n, k], Wdq[n, k] = f16(q * s + mn) (gemm.js:147-148), fp32 accumulation.
//
// A CTA owns 128 weight rows x BT tokens (BT = 64 / 128 / 256) and walks K in 64-wide stages through a 5-slot ring:
//   warp 0       producer: X tile [BT x 64] fp16 by TMA (128-byte swizzle, no multicast) and the stage's q4 records
//                (two 64-row tiles x two 32-k groups, 2 x 2560 contiguous bytes) by cp.async.bulk, on one mbarrier
//   warp 1       TMEM allocator and the single MMA-issuing thread: tcgen05.mma kind::f16, M = 128 weight rows,
//                N = BT tokens, K = 16, A (the dequantised weights) read from tensor memory, B (X) from shared
//                memory, D (fp32) in tensor memory
//   warps 2..17  dequantisers: thread = one weight row (its TMEM lane), a warp = one 32-k half of every other stage;
//                each reads its row's 16 code bytes and (s, mn) word from the ring, computes f16(fmaf(q, s, mn))
//                exactly and writes the 16 packed columns to the stage's TMEM slot with tcgen05.st. After the last
//                stage the same warps are the epilogue: tcgen05.ld -> bias / activation -> shared staging ->
//                coalesced vector stores.
// Orientation: D = Wdq . X^T, so TMEM lane = output column n and TMEM column = token m.
// A persistent form of the same GEMM (gemm_q4_ps, below) serves q4 calls with a store epilogue and short K: one CTA
// per SM walks the tiles with two accumulators in tensor memory and the dequantised weights in shared memory, so a
// tile's epilogue runs under the next tile's main loop.
#include <cuda.h>
#include <cstdlib>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "internal.h"
#include "tc.cuh"

namespace {

constexpr int kBW = 128;        // weight rows per CTA (TMEM lanes, MMA M)
constexpr int kBK = 64;         // k per stage
// Two shapes of the kernel, one source. Cfg1: 16 dequantiser warps (two stage parities), 5 stages, tiles of up to 256
// tokens, one CTA per SM, 512 TMEM columns. Cfg2: 8 dequantiser warps, 4 stages, tiles of up to 128 tokens, two CTAs
// per SM with 256 TMEM columns each, so that one CTA's epilogue runs while the other's main loop keeps the tensor
// cores busy. PAIR = 2: a CTA pair (a 2-CTA cluster) runs one tcgen05.mma.cta_group::2 of M = 256 weight rows: each
// CTA dequantises its own 128 rows into its tensor memory and loads half of the token tile's X (BT / 2 rows), and the
// even CTA's elected thread issues the pair's MMAs, which leave each CTA's 128 rows x BT tokens in its own tensor
// memory. Per SM that is the same dequantisation and MMA work per stage for half the X bytes out of L2.
// KS = 128: stages of 128 k (two 64-k X boxes, four q4 groups per row tile; q4 records by bulk copy only), so each
// stage hand-off carries twice the work.
template <int DQW, int STAGES, uint32_t MAXBT, int MINB, int PAIR = 1, int KS = 64>
struct GemmCfg {
  static constexpr int kPair = PAIR;
  static constexpr uint32_t kKS = KS;                  // k per stage
  static constexpr int kDqWarps = DQW;                 // warps 2 .. 2+DQW-1: (lane quarter) x (32-k half) x (parity)
  static constexpr int kPar = DQW / 8;                 // stage parities the dequantisers alternate over
  static constexpr int kStages = STAGES;
  static constexpr int kMinBlocks = MINB;
  static constexpr int kThreads = 32 * (2 + DQW);
  static constexpr uint32_t kMaxBT = MAXBT;
  static constexpr uint32_t kAcol = MAXBT;             // first TMEM column of the weight (A) stages; D holds [0, BT)
  static constexpr uint32_t kTmemCols = MAXBT + (KS / 2u) * STAGES <= 256u ? 256u : 512u;
  static constexpr size_t kXStage = (size_t)MAXBT / PAIR * KS * 2;   // X slot (1024-aligned); the ring is also the staging
  static constexpr size_t kRingBytes = (size_t)STAGES * kXStage;
};
using Cfg1 = GemmCfg<16, 5, 256, 1>;
using Cfg2 = GemmCfg<8, 4, 128, 2>;
using Cfg3 = GemmCfg<16, 6, 256, 1>;   // Cfg1 with a sixth stage (223 KB of shared memory, 448 TMEM columns)
using CfgH = GemmCfg<16, 4, 256, 1>;   // fp16 weights: 16 KB of weights per stage, so four stages fit
using Cfg4 = GemmCfg<24, 5, 256, 1>;   // Cfg1 with a third dequantiser parity (every third stage per warp; 832 threads)
using Cfg5 = GemmCfg<16, 8, 256, 1, 2>;
using Cfg7 = GemmCfg<16, 3, 256, 1, 1, 128>;   // 128-k stages: 3 x (64 KB X + 10 KB records), 448 TMEM columns   // CTA pairs: 16 KB X slots, so 8 stages (the ring still stages [256][128] f32)
constexpr int kDqPerStage = 8;  // dequant warps that fill one stage
// weights of a stage: q4 2 row tiles x 2 groups of 1280 B; q8 2 row tiles x 1 group of 4224 B (= the gathered layout's
// 128 rows x 2 halves x 32 code bytes + 128 scales x 2 B + 256 B)
// weight encodings of the kernel instances: q4g32a.t64, q8g64s.t64, fp16 row-major
enum { kWQ4 = 0, kWQ8 = 1, kWF16 = 2 };
// fp16: 128 rows x 64 k x 2 bytes, laid out [k half][16-byte chunk][row] so that a warp's rows are consecutive
template <int WE> __host__ __device__ constexpr uint32_t w_stage_e() { return WE == kWQ8 ? 2u * 4224u : WE == kWF16 ? 16384u : 2u * 2u * 1280u; }
template <bool Q8> __host__ __device__ constexpr uint32_t w_stage() { return w_stage_e<Q8 ? kWQ8 : kWQ4>(); }
constexpr uint32_t kWStage = w_stage<false>();

struct GemmParams {
  const uint8_t *W;   // weight view base
  uint8_t *Y;         // y buffer + y.off
  const float *EV, *BV;
  const float *RP;      // heads: rope (cos, sin) rows
  const uint16_t *GT;   // onormgate: the fp16 gate
  uint32_t M, N, K, wR0, wR1, wG, wk0, Nw, ldy, ny0, evOff, bvOff, bvUp;
  uint32_t Ltot, Hq, Hkv, rowOff;
  float eps;
  int rope_half;
  int epi, act, res, store, gate, bias, post_gelu;
  uint32_t BT, nk;
  uint32_t nkz;       // k split: stages per split (0: none); split z = blockIdx.z runs stages [z * nkz, (z + 1) * nkz)
  size_t zstride;     // k split: elements between the splits' f32 partial outputs
  int wtma;           // 1: the CTA's 128 rows are two whole 64-row tiles -> records arrive by bulk copy
  uint32_t *err;
};

// f16(fmaf(q, s, mn)) for the two codes of one byte (low nibble = even k), packed low/high: the GEMM's weight value
// (gemm.js:147-148 computes cv*sc + mn in f32 and converts to f16; q*s is exact in f32, so one fma is the same f32)
__device__ __forceinline__ uint32_t deq_pair(uint32_t byte, float s, float mn) {
  const float lo = __uint_as_float(0x4B000000u | (byte & 15u)) - 8388608.0f;
  const float hi = __uint_as_float(0x4B000000u | ((byte >> 4) & 15u)) - 8388608.0f;
  __half2 h = __floats2half2_rn(fmaf(lo, s, mn), fmaf(hi, s, mn));
  return *reinterpret_cast<uint32_t *>(&h);
}
// The same values on the fp16 pipe. q*s + mn rounded once to fp16 (HFMA2) equals the reference's f16(f32(q*s + mn))
// whenever q*s + mn is exact in f32, so that the f32 rounding is the identity. With s = S * 2^(Es-25) and
// mn = Mn * 2^(Em-25) (S, Mn < 2^11 integers; E = max(exponent field, 1)), q*s + mn is an integer multiple of
// 2^(min(Es,Em)-25) below 2^(16 + Es - Em) (Es >= Em) or 2^(12 + Em - Es) (Em > Es): exact in f32's 24 bits when
// -12 <= Es - Em <= 8. deq_fast_ok() checks that (and finiteness) per row-group; other groups take deq_pair().
__device__ __forceinline__ bool deq_fast_ok(uint32_t sm) {
  const int es = (int)((sm >> 10) & 31u), em = (int)((sm >> 26) & 31u);
  const int Es = es > 1 ? es : 1, Em = em > 1 ? em : 1, d = Es - Em;
  return es != 31 && em != 31 && d <= 8 && d >= -12;
}
__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ void deq_row16(const uint4 c, uint32_t sm, uint32_t (&r)[16]) {
  const uint32_t w[4] = {c.x, c.y, c.z, c.w};
  if (deq_fast_ok(sm)) {
    const uint32_t s2 = __byte_perm(sm, 0, 0x1010), mn2 = __byte_perm(sm, 0, 0x3232);   // (s, s), (mn, mn)
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint32_t w4 = w[i] >> 4;
#pragma unroll
      for (int b = 0; b < 4; b++) {
        // byte b of w (low code in bits 0-3) and byte b of w >> 4 (high code in bits 0-3) -> halves 0 and 1
        const uint32_t x = __byte_perm(w[i], w4, (uint32_t)(b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12)));
        const uint32_t q2 = hsub2_u32((x & 0x000F000Fu) | 0x64006400u, 0x64006400u);   // (1024 + q) - 1024, exact
        r[i * 4 + b] = hfma2_u32(q2, s2, mn2);
      }
    }
  } else {
    const float s = __half2float(__ushort_as_half((unsigned short)(sm & 0xffffu)));
    const float mn = __half2float(__ushort_as_half((unsigned short)(sm >> 16)));
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int b = 0; b < 4; b++) r[i * 4 + b] = deq_pair((w[i] >> (8 * b)) & 0xffu, s, mn);
  }
}

// q8 (gemm.js:150-160: f16(f32(q) * s)): 32 codes of one row (byte i = k i) -> 16 fp16 pairs. A code becomes exact fp16
// by an xor with 0x80, a byte permute against 0x64 ((1024 + q + 128) in fp16) and a subtract of 1152; q * s is exact
// in f32 (8 x 11 significant bits), so one fp16 multiply rounds it exactly as the reference's conversion does.
__device__ __forceinline__ uint32_t q8_pair_f16(uint32_t u, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(u), "r"(0x64646464u), "r"(sel));
  return hsub2_u32(d, 0x64806480u);
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ void deq_row16_q8(const uint4 c0, const uint4 c1, uint32_t sbits, uint32_t (&r)[16]) {
  const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  const uint32_t s2 = (sbits & 0xffffu) * 0x10001u;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const uint32_t u = w[i] ^ 0x80808080u;
    r[2 * i] = hmul2_u32(q8_pair_f16(u, 0x4140u), s2);
    r[2 * i + 1] = hmul2_u32(q8_pair_f16(u, 0x4342u), s2);
  }
}

__device__ __forceinline__ uint4 ldg_w(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg_w32(const void *p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// activations in the reference's source order (no contraction)
// tanh on the SFU (tanh.approx.f32): its error is far below an fp16 ulp of the GELU results the epilogue stores, and
// it takes one instruction where tanhf takes a sequence; the epilogue's GELU is the MLP-up GEMM's largest extra cost
__device__ __forceinline__ float tanh_sfu(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float gelu_g(float g) {   // gemm.js:204
  float u = __fmul_rn(0.7978845608f, __fadd_rn(g, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, g), g), g)));
  u = fminf(15.0f, fmaxf(-15.0f, u));
  return __fmul_rn(__fmul_rn(g, 0.5f), __fadd_rn(1.0f, tanh_sfu(u)));
}
__device__ __forceinline__ float gelu_m(float x) {   // ops/misc.js:116
  float u = __fmul_rn(0.7978845608f, __fadd_rn(x, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x)));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanh_sfu(fminf(15.0f, fmaxf(-15.0f, u)))));
}
__device__ __forceinline__ float silu_g(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

__device__ __forceinline__ uint32_t weight_row(const GemmParams &p, uint32_t nB, uint32_t cc) {
  uint32_t r = p.epi == P0_GEPI_SWIGLU ? ((cc & 1u) == 0u ? p.wR0 : p.wR1) + ((nB + cc) >> 1) : p.wR0 + nB + cc;
  return r < p.Nw - 1 ? r : p.Nw - 1;   // gemm.js:96 clamps to the last row
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(tc::smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
               : "memory");
}

// the two record-tiles a CTA's 128 TMEM lanes read (bulk-copy path): rows [nB, nB+128) map to tiles T0, T0+1, or for
// swiglu the gate tile (even lanes) and the up tile (odd lanes); a tile beyond the weight clamps to the last one
__device__ __forceinline__ void cta_tiles(const GemmParams &p, uint32_t nB, uint32_t &t0, uint32_t &t1) {
  const uint32_t nt = p.Nw / 64u;
  if (p.epi == P0_GEPI_SWIGLU) {
    t0 = (p.wR0 + (nB >> 1)) >> 6;
    t1 = (p.wR1 + (nB >> 1)) >> 6;
  } else {
    t0 = (p.wR0 + nB) >> 6;
    t1 = t0 + 1;
  }
  t0 = t0 < nt ? t0 : nt - 1;
  t1 = t1 < nt ? t1 : nt - 1;
}

__device__ __forceinline__ uint2 pack_h4(const float *v) {
  return make_uint2((uint32_t)__half_as_ushort(__float2half_rn(v[0])) | ((uint32_t)__half_as_ushort(__float2half_rn(v[1])) << 16),
                    (uint32_t)__half_as_ushort(__float2half_rn(v[2])) | ((uint32_t)__half_as_ushort(__float2half_rn(v[3])) << 16));
}

// the epilogues that reduce over one 128-wide head (gemm.js:212-250). The CTA's 128 columns are one head, staged as
// [BT][128] f32 accumulators; a warp takes a token row at a time, lane l columns 4l..4l+3, and the head's sum of
// squares comes from a butterfly over the warp. 'half' RoPE pairs dim d (lanes 0-15) with d + 64 (lane + 16).
__device__ __forceinline__ void store_red128(const GemmParams &p, const float *stg, uint32_t nB, uint32_t m0, uint32_t BT,
                                             uint32_t wi, uint32_t nwarps, uint32_t lane) {
  const uint32_t c = lane * 4u, hd = nB >> 7;
  const bool og = p.epi == P0_GEPI_ONORMGATE;
  const uint32_t sec = og ? 0u : hd < p.Hq ? 0u : hd < p.Hq + p.Hkv ? 1u : 2u;
  float w[4] = {1.0f, 1.0f, 1.0f, 1.0f};
  if (sec < 2u) {
    const float4 e = *reinterpret_cast<const float4 *>(p.EV + p.evOff + sec * 128u + c);
    w[0] = e.x; w[1] = e.y; w[2] = e.z; w[3] = e.w;
  }
  for (uint32_t ml = wi; ml < BT; ml += nwarps) {
    const uint32_t m = m0 + ml;
    if (m >= p.M) break;
    const float4 t = *reinterpret_cast<const float4 *>(stg + ml * 128u + c);
    float v[4] = {t.x, t.y, t.z, t.w}, out[4];
    if (sec < 2u) {
      float ss = __fmul_rn(v[0], v[0]);
#pragma unroll
      for (int i = 1; i < 4; i++) ss = fmaf(v[i], v[i], ss);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float inv = rsqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / 128.0f), p.eps));
#pragma unroll
      for (int i = 0; i < 4; i++) v[i] = __fmul_rn(__fmul_rn(v[i], inv), w[i]);
    }
    if (og) {
      const size_t gi = (size_t)m * p.Ltot + p.ny0 + nB + c;
      const uint2 g2 = *reinterpret_cast<const uint2 *>(p.GT + gi);
      const float g[4] = {__half2float(__ushort_as_half((unsigned short)(g2.x & 0xffffu))),
                          __half2float(__ushort_as_half((unsigned short)(g2.x >> 16))),
                          __half2float(__ushort_as_half((unsigned short)(g2.y & 0xffffu))),
                          __half2float(__ushort_as_half((unsigned short)(g2.y >> 16)))};
#pragma unroll
      for (int i = 0; i < 4; i++) out[i] = __fdiv_rn(v[i], __fadd_rn(1.0f, expf(-g[i])));
      *reinterpret_cast<uint2 *>(p.Y + ((size_t)m * p.ldy + p.ny0 + nB + c) * 2) = pack_h4(out);
      continue;
    }
    const uint32_t row = p.rowOff + m;
    if (sec == 2u) {
#pragma unroll
      for (int i = 0; i < 4; i++) out[i] = v[i];
    } else if (p.rope_half) {
      float o[4];
#pragma unroll
      for (int i = 0; i < 4; i++) o[i] = __shfl_xor_sync(0xffffffffu, v[i], 16);
      const float *rp = p.RP + (size_t)row * 128u + 2u * (c & 63u);
      const float4 a = *reinterpret_cast<const float4 *>(rp), b = *reinterpret_cast<const float4 *>(rp + 4);
      const float cs[4] = {a.x, a.z, b.x, b.z}, sn[4] = {a.y, a.w, b.y, b.w};
#pragma unroll
      for (int i = 0; i < 4; i++)
        out[i] = lane < 16u ? __fsub_rn(__fmul_rn(v[i], cs[i]), __fmul_rn(o[i], sn[i]))
                            : __fadd_rn(__fmul_rn(v[i], cs[i]), __fmul_rn(o[i], sn[i]));
    } else {
      const float4 r = *reinterpret_cast<const float4 *>(p.RP + (size_t)row * 128u + c);   // (cos, sin) of pairs c/2, c/2 + 1
      out[0] = __fsub_rn(__fmul_rn(v[0], r.x), __fmul_rn(v[1], r.y));
      out[1] = __fadd_rn(__fmul_rn(v[0], r.y), __fmul_rn(v[1], r.x));
      out[2] = __fsub_rn(__fmul_rn(v[2], r.z), __fmul_rn(v[3], r.w));
      out[3] = __fadd_rn(__fmul_rn(v[2], r.w), __fmul_rn(v[3], r.z));
    }
    *reinterpret_cast<uint2 *>(p.Y + (((size_t)hd * p.Ltot + row) * 128u + c) * 2) = pack_h4(out);
  }
}

template <class C, int WE>
__global__ void __launch_bounds__(C::kThreads, C::kMinBlocks) gemm_q4_tc(const __grid_constant__ CUtensorMap tmx, const GemmParams p) {
  constexpr bool Q8 = WE == kWQ8, F16 = WE == kWF16;
  constexpr int kStages = C::kStages, kDqWarps = C::kDqWarps;
  constexpr uint32_t kSK = C::kKS, kAC = kSK / 2u, kGS = kSK / 32u;   // k, TMEM A columns and q4 groups per stage
  static_assert(kSK == 64 || WE == kWQ4, "128-k stages are built for q4 records only");
  constexpr uint32_t kWStage = WE == kWQ4 ? 2u * kGS * 1280u : w_stage_e<WE>();
  constexpr uint32_t kAcol = C::kAcol, kTmemCols = C::kTmemCols;
  constexpr size_t kXStage = C::kXStage, kRingBytes = C::kRingBytes;
  static_assert((size_t)C::kMaxBT * 128 * 4 <= C::kRingBytes, "the epilogue stages [BT][128] f32 in the X ring");
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base by pointer arithmetic on the shared array (keeps shared-space loads and stores)
  uint8_t *smem = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t *xring = smem;
  uint8_t *wring = smem + kRingBytes;                  // kStages x kWStage
  uint64_t *full = (uint64_t *)(wring + (size_t)kStages * kWStage);
  uint64_t *full_a = full + kStages;
  uint64_t *empty = full_a + kStages;
  uint64_t *accf = empty + kStages;
  uint32_t *tmem_slot = (uint32_t *)(accf + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  constexpr bool PR = C::kPair == 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t BT = p.BT, nk = p.nk, nB = blockIdx.x * kBW, m0 = blockIdx.y * BT;
  // pairs: the CTA's rank in its cluster (= blockIdx.x & 1) picks its half of the token tile
  const uint32_t crank = PR ? tc::cluster_rank() : 0u, xrows = BT / C::kPair;
  const uint32_t xbytes = xrows * kSK * 2;
  const int32_t xm0 = (int32_t)(m0 + crank * xrows);
  const uint32_t g0 = p.wk0 / (Q8 ? 64u : 32u);
  // this CTA's stages: all of them, or its split's range (slots and phases count from the range's start)
  const uint32_t s0 = p.nkz ? blockIdx.z * p.nkz : 0u, nloc = p.nkz ? min(nk, s0 + p.nkz) - s0 : nk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&full_a[s], kDqPerStage * C::kPair);   // pairs: the even CTA's barrier counts both CTAs' warps
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(accf, 1);
    *abort_flag = 0u;
    tc::fence_mbar_init();
  }
  if (warp == 1) {
    if (PR) {
      tc::tmem_alloc_pair(tmem_slot, kTmemCols);
      tc::tmem_relinquish_pair();
    } else {
      tc::tmem_alloc(tmem_slot, kTmemCols);
      tc::tmem_relinquish();
    }
  }
  tc::fence_before();
  if (PR) tc::cluster_sync();   // both CTAs' barriers are initialised before either arrives on the other's
  else __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer: X by TMA, weight records by bulk copy
    uint32_t t0 = 0, t1 = 0;
    cta_tiles(p, nB, t0, t1);
    if (lane == 0) tc::prefetch_tmap(&tmx);
    uint32_t issued = 0;
    for (uint32_t sl = 0; sl < nloc; sl++) {
      const uint32_t s = s0 + sl, slot = sl % kStages, ph = (sl / kStages) & 1u;
      bool got = true;
      if (lane == 0) got = tc::mbar_wait(&empty[slot], ph ^ 1u, abort_flag, p.err, 0x101u, P0_SPIN_LIMIT);
      if (!__shfl_sync(0xffffffffu, (int)got, 0)) break;
      uint8_t *ws = wring + (size_t)slot * kWStage;
      const uint32_t ng = min(2u, (p.K - s * kBK) / 32u);   // groups in this stage (the last may hold one)
      if (F16) {
        // fp16 rows (any row mapping): each lane copies 4 rows' 64-byte halves as 16-byte chunks into [h][chunk][row]
        for (uint32_t i = 0; i < 4; i++) {
          const uint32_t nl = i * 32u + lane, row = weight_row(p, nB, nl);
          const uint8_t *src = p.W + ((size_t)row * p.wG + p.wk0 + s * kBK) * 2u;
          for (uint32_t h = 0; h < ng; h++)
#pragma unroll
            for (uint32_t j = 0; j < 4; j++)
              *reinterpret_cast<uint4 *>(ws + ((h * 4u + j) * 128u + nl) * 16u) = ldg_w(src + h * 64u + j * 16u);
        }
        __syncwarp();
        if (lane == 0) {
          tc::mbar_expect_tx(&full[slot], xbytes);
          tc::tma_load_2d(xring + (size_t)slot * kXStage, &tmx, &full[slot], (int32_t)(s * kBK), xm0);
        }
      } else if (p.wtma && Q8) {
        if (lane == 0) {   // one q8 record of each row tile: the stage's 64 k
          tc::mbar_expect_tx(&full[slot], xbytes + 2u * 4224u);
          tc::tma_load_2d(xring + (size_t)slot * kXStage, &tmx, &full[slot], (int32_t)(s * kBK), xm0);
          bulk_g2s(ws, p.W + ((size_t)t0 * p.wG + g0 + s) * 4224u, 4224u, &full[slot]);
          bulk_g2s(ws + 4224u, p.W + ((size_t)t1 * p.wG + g0 + s) * 4224u, 4224u, &full[slot]);
        }
      } else if (p.wtma || kSK != 64) {
        if (lane == 0) {
          const uint32_t ngs = min(kGS, (p.K - s * kSK) / 32u);   // groups in this stage (the last may hold fewer)
          tc::mbar_expect_tx(&full[slot], xbytes + 2u * ngs * 1280u);
#pragma unroll
          for (uint32_t bx = 0; bx < kSK / 64u; bx++)   // 64-k boxes (one 128-byte swizzle span each), stacked
            tc::tma_load_2d(xring + (size_t)slot * kXStage + bx * xrows * 128u, &tmx, &full[slot], (int32_t)(s * kSK + bx * 64u), xm0);
          bulk_g2s(ws, p.W + ((size_t)t0 * p.wG + g0 + kGS * s) * 1280u, ngs * 1280u, &full[slot]);
          bulk_g2s(ws + kGS * 1280u, p.W + ((size_t)t1 * p.wG + g0 + kGS * s) * 1280u, ngs * 1280u, &full[slot]);
        }
      } else if (Q8) {
        // q8 rows that are not whole tiles: [h][lane] 32 code bytes, then one scale per row
        for (uint32_t i = 0; i < 4; i++) {
          const uint32_t nl = i * 32u + lane, row = weight_row(p, nB, nl);
          const uint8_t *rec = p.W + ((size_t)(row >> 6) * p.wG + g0 + s) * 4224u;
          for (uint32_t h = 0; h < ng; h++) {
            const uint8_t *src = rec + (row & 63u) * 64u + h * 32u;
            *reinterpret_cast<uint4 *>(ws + (h * 128u + nl) * 32u) = ldg_w(src);
            *reinterpret_cast<uint4 *>(ws + (h * 128u + nl) * 32u + 16u) = ldg_w(src + 16);
          }
          *reinterpret_cast<uint16_t *>(ws + 8192u + nl * 2u) = *reinterpret_cast<const uint16_t *>(rec + 4096u + (row & 63u) * 2u);
        }
        __syncwarp();
        if (lane == 0) {
          tc::mbar_expect_tx(&full[slot], xbytes);
          tc::tma_load_2d(xring + (size_t)slot * kXStage, &tmx, &full[slot], (int32_t)(s * kBK), xm0);
        }
      } else {
        // rows that are not whole tiles: the warp gathers them into lane order ([h][lane] 16-byte codes, then tails)
        for (uint32_t i = 0; i < 4; i++) {
          const uint32_t nl = i * 32u + lane, row = weight_row(p, nB, nl);
          const uint8_t *rowrec = p.W + (size_t)(row >> 6) * p.wG * 1280u;
          for (uint32_t h = 0; h < ng; h++) {
            const uint8_t *rec = rowrec + (size_t)(g0 + 2u * s + h) * 1280u;
            *reinterpret_cast<uint4 *>(ws + (h * 128u + nl) * 16u) = ldg_w(rec + (row & 63u) * 16u);
            *reinterpret_cast<uint32_t *>(ws + 4096u + (h * 128u + nl) * 4u) = ldg_w32(rec + 1024u + (row & 63u) * 4u);
          }
        }
        __syncwarp();
        if (lane == 0) {
          tc::mbar_expect_tx(&full[slot], xbytes);
          tc::tma_load_2d(xring + (size_t)slot * kXStage, &tmx, &full[slot], (int32_t)(s * kBK), xm0);
        }
      }
      issued++;
    }
    // every issued copy has landed before the CTA can exit (bounded; no abort short-cut: copies always finish)
    if (lane == 0) {
      volatile uint32_t never = 0;
      for (uint32_t s = issued > (uint32_t)kStages ? issued - kStages : 0; s < issued; s++)
        tc::mbar_wait(&full[s % kStages], (s / kStages) & 1u, &never, p.err, 0x102u, P0_SPIN_LIMIT);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && crank == 0u) {   // pairs: the even CTA issues for both
      const uint32_t idesc = tc::idesc_f16_f32(kBW * C::kPair, BT);
      for (uint32_t sl = 0; sl < nloc; sl++) {
        const uint32_t slot = sl % kStages, ph = (sl / kStages) & 1u;
        // implies X landed (in both CTAs: each CTA's dequantisers waited for its stage before arriving)
        const bool got = PR ? tc::mbar_wait_cluster(&full_a[slot], ph, abort_flag, p.err, 0x202u, P0_SPIN_LIMIT)
                            : tc::mbar_wait(&full_a[slot], ph, abort_flag, p.err, 0x202u, P0_SPIN_LIMIT);
        if (!got) break;
        tc::fence_after();
        const uint32_t xs = tc::smem_u32(xring + (size_t)slot * kXStage);
#pragma unroll
        for (uint32_t kk = 0; kk < kSK / 16; kk++) {
          const uint64_t bd = tc::desc_sw128(xs + (kk >> 2) * xrows * 128u + (kk & 3u) * 32u);   // box kk / 4, k16 step kk % 4
          if (PR) tc::mma_ts_f16_pair(tmem, tmem + kAcol + slot * kAC + kk * 8u, bd, idesc, (sl | kk) != 0u);
          else tc::mma_ts_f16(tmem, tmem + kAcol + slot * kAC + kk * 8u, bd, idesc, (sl | kk) != 0u);
        }
        if (PR) tc::mma_commit_pair(&empty[slot]);   // frees the slot in both CTAs
        else tc::mma_commit(&empty[slot]);
      }
      if (PR) tc::mma_commit_pair(accf);
      else tc::mma_commit(accf);
      // the accumulator is complete (or the loop gave up) before TMEM can be released
      volatile uint32_t never = 0;
      tc::mbar_wait(accf, 0, &never, p.err, 0x203u, P0_SPIN_LIMIT);
    }
  } else {
    // ---------------------------------------------------------------- dequantisers, then the epilogue
    const uint32_t d = (uint32_t)warp - 2u, q = (uint32_t)warp & 3u, h = (d >> 2) & 1u, par = d >> 3;
    const uint32_t nl = q * 32u + lane;               // this thread's TMEM lane = weight row of the tile
    const uint32_t tq = tmem + ((q * 32u) << 16);
    // where this thread's 16 code bytes and (s, mn) word sit in a weight stage
    uint32_t code_off = 0, tail_off = 0;
    if (F16) {
      code_off = (h * 4u * 128u + nl) * 16u;   // chunk j of this row's half at code_off + j * 2048
    } else if (Q8) {
      if (p.wtma) {
        const uint32_t ts = p.epi == P0_GEPI_SWIGLU ? (nl & 1u) : (nl >> 6), r = p.epi == P0_GEPI_SWIGLU ? (nl >> 1) : (nl & 63u);
        code_off = ts * 4224u + r * 64u + h * 32u;
        tail_off = ts * 4224u + 4096u + r * 2u;
      } else {
        code_off = (h * 128u + nl) * 32u;
        tail_off = 8192u + nl * 2u;
      }
    } else if (p.wtma || kSK != 64) {
      // this thread's groups of a stage: h * kGS / 2 + j (j < kGS / 2), records 1280 bytes apart
      const uint32_t ts = p.epi == P0_GEPI_SWIGLU ? (nl & 1u) : (nl >> 6), r = p.epi == P0_GEPI_SWIGLU ? (nl >> 1) : (nl & 63u);
      code_off = ts * kGS * 1280u + h * (kGS / 2u) * 1280u + r * 16u;
      tail_off = ts * kGS * 1280u + h * (kGS / 2u) * 1280u + 1024u + r * 4u;
    } else {
      code_off = (h * 128u + nl) * 16u;
      tail_off = 4096u + (h * 128u + nl) * 4u;
    }
    bool ok = true;
    for (uint32_t sl = par; sl < nloc; sl += C::kPar) {   // this warp fills every kPar-th stage
      const uint32_t s = s0 + sl, slot = sl % kStages, ph = (sl / kStages) & 1u;
      const bool got = tc::mbar_wait(&full[slot], ph, abort_flag, p.err, 0x301u, P0_SPIN_LIMIT);
      if (!__all_sync(0xffffffffu, got)) { ok = false; break; }   // warp-uniform: tcgen05.st is .sync.aligned
#pragma unroll
      for (uint32_t j = 0; j < kGS / 2u; j++) {   // 64-k stages: one group (j = 0)
        const uint32_t gi = h * (kGS / 2u) + j;   // the group of the stage
        uint32_t r[16];
        if (s * kSK + gi * 32u < p.K) {
          const uint8_t *ws = wring + (size_t)slot * kWStage;
          if (F16) {
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
              const uint4 v = *reinterpret_cast<const uint4 *>(ws + code_off + jj * 2048u);
              r[4 * jj] = v.x; r[4 * jj + 1] = v.y; r[4 * jj + 2] = v.z; r[4 * jj + 3] = v.w;
            }
          } else if (Q8)
            deq_row16_q8(*reinterpret_cast<const uint4 *>(ws + code_off), *reinterpret_cast<const uint4 *>(ws + code_off + 16u),
                         *reinterpret_cast<const uint16_t *>(ws + tail_off), r);
          else
            deq_row16(*reinterpret_cast<const uint4 *>(ws + code_off + j * 1280u), *reinterpret_cast<const uint32_t *>(ws + tail_off + j * 1280u), r);
        } else {
#pragma unroll
          for (int i = 0; i < 16; i++) r[i] = 0u;   // k beyond K: zero weights (X is zero-filled there as well)
        }
        tc::tmem_st16(tq + kAcol + slot * kAC + gi * 16u, r);
      }
      tc::tmem_wait_st();
      tc::fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PR) tc::mbar_arrive_rank(&full_a[slot], 0u);   // the even CTA's barrier, which its MMA thread waits on
        else tc::mbar_arrive(&full_a[slot]);
      }
    }
    // ---- epilogue. Every epilogue thread passes both named barriers whatever happened (the loops above are
    // bounded), and the work between them is skipped warp-uniformly after a failed wait.
    asm volatile("bar.sync 1, %0;" ::"n"(kDqWarps * 32) : "memory");
    bool go = ok && !*abort_flag;
    if (go) go = tc::mbar_wait(accf, 0, abort_flag, p.err, 0x401u, P0_SPIN_LIMIT);
    go = __all_sync(0xffffffffu, go);
    float *stg = reinterpret_cast<float *>(xring);   // [BT][128] f32 (swiglu: [BT][64])
    const bool swi = p.epi == P0_GEPI_SWIGLU;
    if (go) {
      tc::fence_after();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      const uint32_t n = nB + nl;
      float pre_a = 1.0f, pre_b = 0.0f, gB = 0.0f, uB = 0.0f;   // per-row epilogue constants
      if (p.epi == P0_GEPI_BIAS) pre_b = n < p.N ? p.EV[p.evOff + n] : 0.0f;
      if (p.epi == P0_GEPI_RESADD && n < p.N) {
        pre_a = p.gate ? p.EV[p.evOff + n] : 1.0f;
        pre_b = p.bias ? p.BV[p.bvOff + n] : 0.0f;
      }
      if (swi && p.bias && nB + (nl & ~1u) < p.N) {
        const uint32_t o = (nB >> 1) + (nl >> 1);
        gB = p.BV[p.bvOff + o];
        uB = p.BV[p.bvOff + p.bvUp + o];
      }
      // warp: quarter q of the lanes, every (warps / 4)-th 16-column chunk of BT from chunk e
      const uint32_t e = d >> 2;
      for (uint32_t c0 = e * 16u; c0 < BT; c0 += (kDqWarps / 4) * 16u) {
        uint32_t r[16];
        tc::tmem_ld16(tq + c0, r);
        tc::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const float v = __uint_as_float(r[j]);
          const uint32_t ml = c0 + j;
          if (swi) {
            const float u = __shfl_down_sync(0xffffffffu, v, 1);
            if ((lane & 1) == 0) {
              const float g = __fadd_rn(v, gB), uu = __fadd_rn(u, uB);
              const float a = p.act == P0_ACT_GELU ? gelu_g(g) : silu_g(g);
              stg[ml * 64u + (nl >> 1)] = __fmul_rn(a, uu);
            }
          } else if (p.epi == P0_GEPI_BIAS) {
            stg[ml * 128u + nl] = __fadd_rn(v, pre_b);
          } else if (p.epi == P0_GEPI_RESADD) {
            stg[ml * 128u + nl] = __fmul_rn(pre_a, __fadd_rn(v, pre_b));
          } else {
            stg[ml * 128u + nl] = v;
          }
        }
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kDqWarps * 32) : "memory");
    if (nB >= p.N) {
      // a pair's odd CTA past the last weight row: nothing of its tile is stored
    } else if (go && !*abort_flag && (p.epi == P0_GEPI_HEADS || p.epi == P0_GEPI_ONORMGATE)) {
      store_red128(p, stg, nB, m0, BT, (threadIdx.x - 64u) >> 5, kDqWarps, lane);
    } else if (go && !*abort_flag) {
      // coalesced stores: 4 consecutive columns per thread per step (the reference's vec4 granularity)
      const uint32_t OC = swi ? 64u : 128u, q4 = OC / 4u, nOut0 = swi ? (nB >> 1) : nB;
      const uint32_t tid = threadIdx.x - 64u;   // 0 .. kDqWarps*32-1
      const bool f32y = p.epi == P0_GEPI_F32 || p.epi == P0_GEPI_RESADD;
      for (uint32_t idx = tid; idx < BT * q4; idx += kDqWarps * 32u) {
        const uint32_t ml = idx / q4, cq = idx - ml * q4, m = m0 + ml;
        const uint32_t colw = swi ? nB + cq * 8u : nB + cq * 4u;   // the ws column the vec4 starts at
        if (m >= p.M || colw >= p.N) continue;
        const float4 t = *reinterpret_cast<const float4 *>(stg + ml * OC + cq * 4u);
        const size_t e = (size_t)m * p.ldy + p.ny0 + nOut0 + cq * 4u + blockIdx.z * p.zstride;
        if (f32y) {
          float4 *yp = reinterpret_cast<float4 *>(p.Y + e * 4);
          float4 o = t;
          if (p.epi == P0_GEPI_RESADD && !p.store) {
            const float4 y0 = *yp;
            o = make_float4(__fadd_rn(y0.x, t.x), __fadd_rn(y0.y, t.y), __fadd_rn(y0.z, t.z), __fadd_rn(y0.w, t.w));
          }
          *yp = o;
        } else {
          uint2 *yp = reinterpret_cast<uint2 *>(p.Y + e * 2);
          float v[4] = {t.x, t.y, t.z, t.w};
          if (p.epi == P0_GEPI_BIAS && p.res) {
            const uint2 y0 = *yp;
            const __half2 a = *reinterpret_cast<const __half2 *>(&y0.x), b = *reinterpret_cast<const __half2 *>(&y0.y);
            v[0] = __fadd_rn(v[0], __low2float(a));
            v[1] = __fadd_rn(v[1], __high2float(a));
            v[2] = __fadd_rn(v[2], __low2float(b));
            v[3] = __fadd_rn(v[3], __high2float(b));
          }
          __half hv[4];
#pragma unroll
          for (int i = 0; i < 4; i++) {
            hv[i] = __float2half_rn(v[i]);
            if (p.epi == P0_GEPI_BIAS && p.post_gelu) hv[i] = __float2half_rn(gelu_m(__half2float(hv[i])));
          }
          uint2 o;
          o.x = (uint32_t)__half_as_ushort(hv[0]) | ((uint32_t)__half_as_ushort(hv[1]) << 16);
          o.y = (uint32_t)__half_as_ushort(hv[2]) | ((uint32_t)__half_as_ushort(hv[3]) << 16);
          *yp = o;
        }
      }
    }
  }
  // ---------------------------------------------------------------- teardown
  // (pairs: neither CTA frees its tensor memory or exits while the other may still arrive on its barriers or read it)
  tc::fence_before();
  if (PR) tc::cluster_sync();
  else __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    if (PR) tc::tmem_dealloc_pair(tmem, kTmemCols);
    else tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ================================================================================================ persistent form
// gemm_q4_ps: the same GEMM for q4 weights in whole 64-row tiles (the bulk-copy path) with the store epilogues
// (f16 / f32 / bias (+res, +post_gelu) / resadd / swiglu), as a persistent kernel: one CTA per SM walks the tiles
// t = blockIdx.x, blockIdx.x + gridDim.x, ... (row tile fastest, so the CTAs running at once share one or two token
// tiles' X in L2), its roles streaming through one ring across tile boundaries:
//   warp 0       producer: per stage the X tile by TMA and the two row tiles' q4 records by cp.async.bulk
//   warp 1       TMEM (512 columns: two accumulators of up to 256 tokens) and the MMA thread: tile i accumulates in
//                buffer i & 1, tcgen05.mma kind::f16 with A (the dequantised weights) and B (X) both from shared
//                memory, M = 128, N = BT
//   warps 2..17  dequantisers: f16(q*s + mn) of their row's 32 k into the stage's A slot, 128-byte swizzled K-major
//                (the layout TMA gives the X tile), then a proxy fence and an arrive
//   warps 18..25 epilogue: two per TMEM lane quarter, alternate 32-token chunks; waits for tile i's accumulator,
//                reads it 32 tokens at a time, applies the epilogue and stores straight to Y (a warp's 32 rows = 32
//                consecutive columns of Y per token), then frees the buffer for tile i + 2. Tile i's epilogue runs
//                under tile i + 1's main loop.
// Per tile the prologue (barrier set-up, TMEM allocation, pipeline fill) is paid once per CTA instead of per tile, and
// no epilogue leaves the tensor pipe idle.
constexpr int kPsStages = 4;
constexpr int kPsDq = 16;
constexpr int kPsEpi = 8;
constexpr int kPsThreads = 32 * (2 + kPsDq + kPsEpi);
constexpr size_t kPsX = (size_t)256 * kBK * 2;   // X slot: up to 256 tokens x 64 k fp16
constexpr size_t kPsA = (size_t)kBW * kBK * 2;   // A slot: 128 rows x 64 k fp16
constexpr size_t kPsW = 2u * 2u * 1280u;         // two row tiles x two q4 groups
constexpr size_t kPsSmem = (size_t)kPsStages * (kPsX + kPsA + kPsW) + 1024 + 256;

__global__ void __launch_bounds__(kPsThreads, 1) gemm_q4_ps(const __grid_constant__ CUtensorMap tmx, const GemmParams p, const uint32_t nrt,
                                                           const uint32_t ntiles) {
  constexpr int S = kPsStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t *xring = smem;
  uint8_t *aring = xring + S * kPsX;
  uint8_t *wring = aring + S * kPsA;
  uint64_t *full = (uint64_t *)(wring + S * kPsW);
  uint64_t *full_a = full + S;
  uint64_t *empty = full_a + S;
  uint64_t *acc_full = empty + S;     // [2]
  uint64_t *acc_empty = acc_full + 2; // [2]
  uint64_t *mdone = acc_empty + 2;
  uint32_t *tmem_slot = (uint32_t *)(mdone + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t BT = p.BT, nk = p.nk, xbytes = BT * kBK * 2, g0 = p.wk0 / 32u;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&full_a[s], kDqPerStage);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      tc::mbar_init(&acc_full[b], 1);
      tc::mbar_init(&acc_empty[b], kPsEpi);
    }
    tc::mbar_init(mdone, 1);
    *abort_flag = 0u;
    tc::fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) tc::prefetch_tmap(&tmx);
    uint32_t gs = 0;
    bool ok = true;
    for (uint32_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const uint32_t nB = (t % nrt) * kBW, m0 = (t / nrt) * BT;
      uint32_t t0 = 0, t1 = 0;
      cta_tiles(p, nB, t0, t1);
      for (uint32_t s = 0; s < nk; s++, gs++) {
        const uint32_t slot = gs % S, ph = (gs / S) & 1u;
        bool got = true;
        if (lane == 0) got = tc::mbar_wait(&empty[slot], ph ^ 1u, abort_flag, p.err, 0x111u, P0_SPIN_LIMIT);
        if (!__shfl_sync(0xffffffffu, (int)got, 0)) { ok = false; break; }
        if (lane == 0) {
          const uint32_t ng = min(2u, (p.K - s * kBK) / 32u);
          uint8_t *ws = wring + (size_t)slot * kPsW;
          tc::mbar_expect_tx(&full[slot], xbytes + 2u * ng * 1280u);
          tc::tma_load_2d(xring + (size_t)slot * kPsX, &tmx, &full[slot], (int32_t)(s * kBK), (int32_t)m0);
          bulk_g2s(ws, p.W + ((size_t)t0 * p.wG + g0 + 2u * s) * 1280u, ng * 1280u, &full[slot]);
          bulk_g2s(ws + 2560u, p.W + ((size_t)t1 * p.wG + g0 + 2u * s) * 1280u, ng * 1280u, &full[slot]);
        }
      }
    }
    // every issued copy has landed before the CTA can exit (bounded; copies always finish)
    if (lane == 0) {
      volatile uint32_t never = 0;
      for (uint32_t g = gs > (uint32_t)S ? gs - S : 0; g < gs; g++)
        tc::mbar_wait(&full[g % S], (g / S) & 1u, &never, p.err, 0x112u, P0_SPIN_LIMIT);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_f16_f32(kBW, BT);
      uint32_t gs = 0, i = 0;
      bool ok = true;
      for (uint32_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, i++) {
        const uint32_t b = i & 1u, u = i >> 1;
        // the epilogue has read this buffer's previous tile (the first use of each buffer passes at once)
        if (!tc::mbar_wait(&acc_empty[b], (u & 1u) ^ 1u, abort_flag, p.err, 0x211u, P0_SPIN_LIMIT)) break;
        tc::fence_after();
        const uint32_t dt = tmem + b * 256u;
        for (uint32_t s = 0; s < nk; s++, gs++) {
          const uint32_t slot = gs % S, ph = (gs / S) & 1u;
          if (!tc::mbar_wait(&full_a[slot], ph, abort_flag, p.err, 0x212u, P0_SPIN_LIMIT)) { ok = false; break; }   // implies X landed
          tc::fence_after();
          const uint32_t xs = tc::smem_u32(xring + (size_t)slot * kPsX), as = tc::smem_u32(aring + (size_t)slot * kPsA);
#pragma unroll
          for (uint32_t kk = 0; kk < kBK / 16; kk++)
            tc::mma_ss_f16(dt, tc::desc_sw128(as + kk * 32u), tc::desc_sw128(xs + kk * 32u), idesc, (s | kk) != 0u);
          tc::mma_commit(&empty[slot]);
        }
        if (ok) tc::mma_commit(&acc_full[b]);
      }
      // every MMA has completed before TMEM can be released
      tc::mma_commit(mdone);
      volatile uint32_t never = 0;
      tc::mbar_wait(mdone, 0, &never, p.err, 0x213u, P0_SPIN_LIMIT);
    }
  } else if (warp < 2 + kPsDq) {
    // ---------------------------------------------------------------- dequantisers
    const uint32_t d = (uint32_t)warp - 2u, q = (uint32_t)warp & 3u, h = (d >> 2) & 1u, par = d >> 3;
    const uint32_t nl = q * 32u + lane;   // this thread's weight row of the tile
    // its record tile and row (swiglu: even rows from the gate tile, odd rows from the up tile)
    const bool swi = p.epi == P0_GEPI_SWIGLU;
    const uint32_t ts = swi ? (nl & 1u) : (nl >> 6), rr = swi ? (nl >> 1) : (nl & 63u);
    const uint32_t code_off = ts * 2560u + h * 1280u + rr * 16u, tail_off = ts * 2560u + h * 1280u + 1024u + rr * 4u;
    const uint32_t arow = (nl >> 3) * 1024u + (nl & 7u) * 128u;   // the row's 128-byte line in the swizzled A slot
    uint32_t gs = 0;
    bool ok = true;
    for (uint32_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      for (uint32_t s = 0; s < nk; s++, gs++) {
        if ((gs & 1u) != par) continue;   // this warp fills every other stage of the ring's sequence
        const uint32_t slot = gs % S, ph = (gs / S) & 1u;
        const bool got = tc::mbar_wait(&full[slot], ph, abort_flag, p.err, 0x311u, P0_SPIN_LIMIT);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        uint32_t r[16];
        if (s * kBK + h * 32u < p.K) {
          const uint8_t *ws = wring + (size_t)slot * kPsW;
          deq_row16(*reinterpret_cast<const uint4 *>(ws + code_off), *reinterpret_cast<const uint32_t *>(ws + tail_off), r);
        } else {
#pragma unroll
          for (int j = 0; j < 16; j++) r[j] = 0u;   // k beyond K: zero weights (X is zero-filled there as well)
        }
        uint8_t *as = aring + (size_t)slot * kPsA + arow;
#pragma unroll
        for (uint32_t j = 0; j < 4; j++)   // 16-byte chunk 4h + j of the row at chunk position (4h + j) ^ (row % 8)
          *reinterpret_cast<uint4 *>(as + (((4u * h + j) ^ (nl & 7u)) * 16u)) = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the generic writes before the MMA's reads
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&full_a[slot]);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const uint32_t q = (uint32_t)warp & 3u, nl = q * 32u + lane, e = ((uint32_t)warp - 2u - kPsDq) >> 2;
    const bool swi = p.epi == P0_GEPI_SWIGLU, f32y = p.epi == P0_GEPI_F32 || p.epi == P0_GEPI_RESADD;
    uint32_t i = 0;
    for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x, i++) {
      const uint32_t b = i & 1u, u = i >> 1;
      const bool got = tc::mbar_wait(&acc_full[b], u & 1u, abort_flag, p.err, 0x411u, P0_SPIN_LIMIT);
      if (!__all_sync(0xffffffffu, got)) break;
      tc::fence_after();
      const uint32_t nB = (t % nrt) * kBW, m0 = (t / nrt) * BT, n = nB + nl;
      float pre_a = 1.0f, pre_b = 0.0f, gB = 0.0f, uB = 0.0f;   // per-row epilogue constants
      if (p.epi == P0_GEPI_BIAS) pre_b = n < p.N ? p.EV[p.evOff + n] : 0.0f;
      if (p.epi == P0_GEPI_RESADD && n < p.N) {
        pre_a = p.gate ? p.EV[p.evOff + n] : 1.0f;
        pre_b = p.bias ? p.BV[p.bvOff + n] : 0.0f;
      }
      const uint32_t o = (nB >> 1) + (nl >> 1);
      if (swi && p.bias && nB + (nl & ~1u) < p.N) {
        gB = p.BV[p.bvOff + o];
        uB = p.BV[p.bvOff + p.bvUp + o];
      }
      const bool col_ok = swi ? ((nl & 1u) == 0u && n < p.N) : n < p.N;
      const size_t col = swi ? (size_t)p.ny0 + o : (size_t)p.ny0 + n;
      const uint32_t dt = tmem + ((q * 32u) << 16) + b * 256u;
      for (uint32_t c0 = e * 32u; c0 < BT; c0 += 32u * (kPsEpi / 4)) {
        uint32_t r[32];
        tc::tmem_ld32(dt + c0, r);
        tc::tmem_wait_ld();
        if (c0 + 32u * (kPsEpi / 4) >= BT) {   // this warp's last chunk   // the accumulator is read: tile i + 2 may use it while these values are stored
          tc::fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&acc_empty[b]);
        }
#pragma unroll
        for (uint32_t j = 0; j < 32; j++) {
          const float v = __uint_as_float(r[j]);
          const uint32_t m = m0 + c0 + j;
          float w = v;
          if (swi) {
            const float up = __shfl_down_sync(0xffffffffu, v, 1);
            const float g = __fadd_rn(v, gB), uu = __fadd_rn(up, uB);
            w = __fmul_rn(p.act == P0_ACT_GELU ? gelu_g(g) : silu_g(g), uu);
          } else if (p.epi == P0_GEPI_BIAS) {
            w = __fadd_rn(v, pre_b);
          } else if (p.epi == P0_GEPI_RESADD) {
            w = __fmul_rn(pre_a, __fadd_rn(v, pre_b));
          }
          if (m >= p.M || !col_ok) continue;
          const size_t e = (size_t)m * p.ldy + col;
          if (f32y) {
            float *yp = reinterpret_cast<float *>(p.Y) + e;
            *yp = (p.epi == P0_GEPI_RESADD && !p.store) ? __fadd_rn(*yp, w) : w;
          } else {
            __half *yp = reinterpret_cast<__half *>(p.Y) + e;
            if (p.epi == P0_GEPI_BIAS && p.res) w = __fadd_rn(w, __half2float(*yp));
            __half hv = __float2half_rn(w);
            if (p.epi == P0_GEPI_BIAS && p.post_gelu) hv = __float2half_rn(gelu_m(__half2float(hv)));
            *yp = hv;
          }
        }
      }
    }
  }
  // ---------------------------------------------------------------- teardown
  tc::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// k split: the S f32 partial products P[z][m][n] of a call, summed in split order, then the call's store epilogue
// (f16 / bias (+res, +post_gelu) / f32 / resadd, the same arithmetic as the GEMM's store pass), 4 columns per thread
__global__ void gemm_ksplit_epilogue(const float *__restrict__ P, uint32_t S, size_t zstride, const GemmParams p) {
  const uint32_t q4 = p.N / 4u;
  const size_t total = (size_t)p.M * q4;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t m = (uint32_t)(i / q4), n = (uint32_t)(i - (size_t)m * q4) * 4u;
    float4 t = *reinterpret_cast<const float4 *>(P + (size_t)m * p.N + n);
    for (uint32_t z = 1; z < S; z++) {
      const float4 u = *reinterpret_cast<const float4 *>(P + z * zstride + (size_t)m * p.N + n);
      t = make_float4(__fadd_rn(t.x, u.x), __fadd_rn(t.y, u.y), __fadd_rn(t.z, u.z), __fadd_rn(t.w, u.w));
    }
    float v[4] = {t.x, t.y, t.z, t.w};
    const size_t e = (size_t)m * p.ldy + p.ny0 + n;
    if (p.epi == P0_GEPI_F32 || p.epi == P0_GEPI_RESADD) {
      float4 *yp = reinterpret_cast<float4 *>(p.Y + e * 4);
      if (p.epi == P0_GEPI_RESADD) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float pa = p.gate ? p.EV[p.evOff + n + j] : 1.0f, pb = p.bias ? p.BV[p.bvOff + n + j] : 0.0f;
          v[j] = __fmul_rn(pa, __fadd_rn(v[j], pb));
        }
        if (!p.store) {
          const float4 y0 = *yp;
          v[0] = __fadd_rn(y0.x, v[0]); v[1] = __fadd_rn(y0.y, v[1]); v[2] = __fadd_rn(y0.z, v[2]); v[3] = __fadd_rn(y0.w, v[3]);
        }
      }
      *yp = make_float4(v[0], v[1], v[2], v[3]);
    } else {
      uint2 *yp = reinterpret_cast<uint2 *>(p.Y + e * 2);
      if (p.epi == P0_GEPI_BIAS) {
#pragma unroll
        for (int j = 0; j < 4; j++) v[j] = __fadd_rn(v[j], p.EV[p.evOff + n + j]);
        if (p.res) {
          const uint2 y0 = *yp;
          const __half2 a = *reinterpret_cast<const __half2 *>(&y0.x), b = *reinterpret_cast<const __half2 *>(&y0.y);
          v[0] = __fadd_rn(v[0], __low2float(a));
          v[1] = __fadd_rn(v[1], __high2float(a));
          v[2] = __fadd_rn(v[2], __low2float(b));
          v[3] = __fadd_rn(v[3], __high2float(b));
        }
      }
      __half hv[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        hv[j] = __float2half_rn(v[j]);
        if (p.epi == P0_GEPI_BIAS && p.post_gelu) hv[j] = __float2half_rn(gelu_m(__half2float(hv[j])));
      }
      uint2 o;
      o.x = (uint32_t)__half_as_ushort(hv[0]) | ((uint32_t)__half_as_ushort(hv[1]) << 16);
      o.y = (uint32_t)__half_as_ushort(hv[2]) | ((uint32_t)__half_as_ushort(hv[3]) << 16);
      *yp = o;
    }
  }
}

// the dequantiser of the GEMM, dumped: out[row][k] = f16(q*s + mn) for a q4 view (bit-exactness checks)
__global__ void deq_dump_q4(const uint8_t *W, uint32_t rows, uint32_t cols, uint32_t wG, uint16_t *out) {
  const uint32_t G = cols / 32;
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)rows * G) return;
  const uint32_t row = (uint32_t)(idx / G), g = (uint32_t)(idx % G);
  const uint8_t *rec = W + ((size_t)(row >> 6) * wG + g) * 1280u;
  const uint4 c = *reinterpret_cast<const uint4 *>(rec + (row & 63u) * 16u);
  const uint32_t sm = *reinterpret_cast<const uint32_t *>(rec + 1024u + (row & 63u) * 4u);
  uint32_t r[16];
  deq_row16(c, sm, r);
  uint32_t *o = reinterpret_cast<uint32_t *>(out + (size_t)row * cols + (size_t)g * 32u);
#pragma unroll
  for (int i = 0; i < 16; i++) o[i] = r[i];
}

// The f32 x prologues of gemm.js:55-63, as a pass that writes the fp16 X [M][K] the GEMM's TMA then reads: one thread
// per 8 consecutive k of a row, the reference's order of operations (no contraction), round to nearest even.
__global__ void gemm_xpro_kernel(int mode, const float *__restrict__ X, uint32_t ldx, uint32_t kx0, const float *__restrict__ ST,
                                 uint32_t statOff, const float *__restrict__ PV, uint32_t pvOff, uint32_t pvStride, uint32_t M,
                                 uint32_t K, uint16_t *__restrict__ out) {
  const uint32_t K8 = K / 8;
  const uint64_t n8 = (uint64_t)M * K8;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t m = (uint32_t)(i / K8), k = (uint32_t)(i % K8) * 8u;
    const float mean = ST[(size_t)(statOff + m) * 2], rstd = ST[(size_t)(statOff + m) * 2 + 1];
    const float *x = X + (size_t)m * ldx + kx0 + k;
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      float v[2];
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const uint32_t kk = kx0 + k + j + h;
        float t;
        if (mode == P0_XPRO_LNMOD) {
          t = __fsub_rn(x[j + h], mean);
          t = __fmul_rn(t, rstd);
          t = __fmul_rn(t, __fadd_rn(1.0f, PV[pvOff + kk]));
          t = __fadd_rn(t, PV[pvOff + pvStride + kk]);
        } else {
          t = __fmul_rn(__fmul_rn(x[j + h], rstd), PV[pvOff + kk]);
        }
        v[h] = t;
      }
      o[j / 2] = (uint32_t)__half_as_ushort(__float2half_rn(v[0])) | ((uint32_t)__half_as_ushort(__float2half_rn(v[1])) << 16);
    }
    *reinterpret_cast<uint4 *>(out + (size_t)m * K + k) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// the q8 dequantiser of the GEMM, dumped: out[row][k] = f16(q*s) for a q8 view, one thread per (row, 32-k half group)
__global__ void deq_dump_q8(const uint8_t *W, uint32_t rows, uint32_t cols, uint32_t wG, uint16_t *out) {
  const uint32_t H = cols / 32;
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)rows * H) return;
  const uint32_t row = (uint32_t)(idx / H), hh = (uint32_t)(idx % H), g = hh / 2, h = hh % 2;
  const uint8_t *rec = W + ((size_t)(row >> 6) * wG + g) * 4224u;
  const uint8_t *src = rec + (row & 63u) * 64u + h * 32u;
  uint32_t r[16];
  deq_row16_q8(*reinterpret_cast<const uint4 *>(src), *reinterpret_cast<const uint4 *>(src + 16),
               *reinterpret_cast<const uint16_t *>(rec + 4096u + (row & 63u) * 2u), r);
  uint32_t *o = reinterpret_cast<uint32_t *>(out + (size_t)row * cols + (size_t)hh * 32u);
#pragma unroll
  for (int i = 0; i < 16; i++) o[i] = r[i];
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)f;
  }
  return fn;
}

const char *gepi_name(uint32_t e) {
  static const char *n[] = {"f16", "f32", "bias", "resadd", "swiglu", "heads", "onormgate"};
  return e < 7 ? n[e] : "?";
}

}  // namespace

extern "C" {

// gemm(gpu, a) (gemm.js:264-322): the reference's checks first, then the kernel's own layout needs
p0_status p0_gemm(p0_ctx *c, const p0_gemm_args *a, double *flops) {
  if (!c || !a) return P0_EINVAL;
  const char *op = "gemm";
  const uint32_t enc = a->w.enc;
  if (enc != P0_ENC_Q4G32A_T64 && enc != P0_ENC_Q8G64S_T64 && enc != P0_ENC_F16)
    return p0_fail(c, P0_EINVAL, "gemm: unsupported weight encoding %u", enc);
  const bool q8 = enc == P0_ENC_Q8G64S_T64, f16w = enc == P0_ENC_F16;
  const uint32_t GK = q8 ? 64u : f16w ? 1u : 32u, RB = q8 ? 4224u : 1280u;
  const uint32_t M = a->M, N = a->N, K = a->K;
  if (K % 32) return p0_fail(c, P0_EINVAL, "gemm: K must be a multiple of 32");
  if (a->epi > P0_GEPI_ONORMGATE) return p0_fail(c, P0_EINVAL, "gemm: epilogue %u is not built in this library yet", a->epi);
  // acc 1 ('f16', the DiT's default, pocketflux-engine.js:4095) asks for fp16 partial sums per 32-k tile
  // (gemm.js:172-183); the tensor cores accumulate every product in f32, which is at least as accurate, so both modes
  // run the same kernel. Values other than 0 / 1 fall back to f32 like the reference's `c.acc === 'f16'` test.
  if (a->post_gelu && a->epi != P0_GEPI_BIAS) return p0_fail(c, P0_EINVAL, "gemm: post_gelu applies to the 'bias' epilogue only");
  if (!M || !N || !K) return P0_OK;
  if (a->w.rows == 0 || a->w.cols % GK || a->wk0 % GK || a->wk0 + K > a->w.cols)
    return p0_fail(c, P0_EINVAL, "gemm: weight view %ux%u does not cover k [%u, %u) in whole %u-k groups", a->w.rows, a->w.cols, a->wk0,
                   a->wk0 + K, GK);
  if (!f16w && a->w.rows % 64) return p0_fail(c, P0_EINVAL, "gemm: %s rows must be a multiple of 64", q8 ? "q8g64s.t64" : "q4g32a.t64");
  // fp16 weights: rows of w.ld halves (0 = cols, gemm.js:271 `a.w.ld || Ktot`), read as 16-byte chunks
  const uint32_t wld = f16w ? (a->w.ld ? a->w.ld : a->w.cols) : 0u;
  if (f16w && wld < a->w.cols) return p0_fail(c, P0_EINVAL, "gemm: f16 weight row stride %u < cols %u", wld, a->w.cols);
  if (f16w && (wld % 8 || a->wk0 % 8)) return p0_fail(c, P0_EALIGN, "gemm: f16 weight rows must start on 16-byte boundaries (ld %% 8, wk0 %% 8)");
  if (N % 4) return p0_fail(c, P0_EALIGN, "gemm: N must be a multiple of 4 (the reference stores whole vec4s)");
  const uint32_t ldx = a->x_ld ? a->x_ld : K, ldy = a->y_ld ? a->y_ld : N, wG = f16w ? wld : a->w.cols / GK;
  const bool swi = a->epi == P0_GEPI_SWIGLU, f32y = a->epi == P0_GEPI_F32 || a->epi == P0_GEPI_RESADD;
  const uint32_t es = f32y ? 4 : 2, ncols_out = swi ? N / 2 : N;
  const uint32_t xmode = a->x_mode;
  if (xmode > P0_XPRO_RMS) return p0_fail(c, P0_EINVAL, "gemm: x prologue %u is not built in this library yet", xmode);
  if (xmode == P0_XPRO_F16 && (ldx % 8 || (a->x_off + 2ull * a->x_k0) % 16))
    return p0_fail(c, P0_EALIGN, "gemm: x rows must start on 16-byte boundaries (ld %% 8, off + 2*k0 %% 16)");
  if (xmode != P0_XPRO_F16 && a->x_off % 4) return p0_fail(c, P0_EALIGN, "gemm: f32 x must start on a 4-byte boundary");
  if (ldy % 4 || a->y_n0 % 4 || a->y_off % (4 * es)) return p0_fail(c, P0_EALIGN, "gemm: y must be vec4-aligned (ld %% 4, n0 %% 4, off)");
  p0_status st;
  P0Range rw, rx, ry, re, rb;
  const uint64_t wbytes = f16w ? ((uint64_t)(a->w.rows - 1) * wG + a->w.cols) * 2 : (uint64_t)(a->w.rows / 64) * wG * RB;
  if ((st = p0_range(c, a->w.buf, a->w.off, wbytes, op, "W", &rw))) return st;
  if ((uintptr_t)rw.base % 16) return p0_fail(c, P0_EALIGN, "gemm: weight offset must be 16-byte aligned");
  if ((st = p0_range(c, a->x, a->x_off, ((uint64_t)(M - 1) * ldx + a->x_k0 + K) * (xmode == P0_XPRO_F16 ? 2 : 4), op, "X", &rx)))
    return st;
  P0Range rst, rpv;
  if (xmode != P0_XPRO_F16) {
    if ((st = p0_range(c, a->stats, 0, ((uint64_t)a->stats_off + M) * 8, op, "stats", &rst))) return st;
    const uint64_t pvneed = (uint64_t)a->pv_off + (xmode == P0_XPRO_LNMOD ? a->pv_stride : 0) + a->x_k0 + K;
    if ((st = p0_range(c, a->pv, 0, pvneed * 4, op, "pv", &rpv))) return st;
  }
  // the head-reducing epilogues (gemm.js:212-250): whole 128-wide heads; the q / k heads read the norm weights and rope
  // rows, onormgate its gate (vec4 reads: Ltot % 4 keeps each row's gate on 8-byte boundaries)
  const bool heads = a->epi == P0_GEPI_HEADS, og = a->epi == P0_GEPI_ONORMGATE;
  const uint32_t nh = N / 128;
  const bool hq = heads && a->h_Hq > 0, hk = heads && nh > a->h_Hq && a->h_Hkv > 0;
  P0Range rrp, rgt;
  if ((heads || og) && N % 128) return p0_fail(c, P0_EINVAL, "gemm: the %s epilogue reduces over whole 128-wide heads (N %% 128)", gepi_name(a->epi));
  if (og && a->h_Ltot % 4) return p0_fail(c, P0_EALIGN, "gemm: onormgate reads the gate as vec4s (heads.Ltot %% 4)");
  const uint64_t ybytes = heads ? ((uint64_t)(nh - 1) * a->h_Ltot + a->h_rowOff + M) * 128 * 2
                                : ((uint64_t)(M - 1) * ldy + a->y_n0 + ncols_out) * es;
  if ((st = p0_range(c, a->y, a->y_off, ybytes, op, "Y", &ry))) return st;
  const bool need_ev = a->epi == P0_GEPI_BIAS || (a->epi == P0_GEPI_RESADD && a->ev.id) || og || hq || hk;
  const uint64_t evn = og || (hq && !hk) ? 128u : hk ? 256u : N;
  if (need_ev && (st = p0_range(c, a->ev, 0, ((uint64_t)a->ev_off + evn) * 4, op, "EV", &re))) return st;
  if ((heads || og) && a->ev_off % 4) return p0_fail(c, P0_EALIGN, "gemm: %s reads its norm weights as vec4s (ev.off %% 4)", gepi_name(a->epi));
  if ((hq || hk) && (st = p0_range(c, a->rope, 0, ((uint64_t)a->h_rowOff + M) * 128 * 4, op, "rope", &rrp))) return st;
  if (og && (st = p0_range(c, a->gt, 0, ((uint64_t)(M - 1) * a->h_Ltot + a->y_n0 + N) * 2, op, "gt", &rgt))) return st;
  const bool bias = a->bv.id != 0 && (a->epi == P0_GEPI_RESADD || swi);
  if (bias && (st = p0_range(c, a->bv, 0, ((uint64_t)a->bv_off + (swi ? a->bv_up + N / 2 : N)) * 4, op, "BV", &rb))) return st;
  if (swi && (a->wr0 + N / 2 > a->w.rows || a->wr1 + N / 2 > a->w.rows)) return p0_fail(c, P0_EINVAL, "gemm: swiglu rows beyond the weight");

  // Cfg1 everywhere: measured on B200 (configs 3 and 4), Cfg2's overlapped epilogue does not pay for halving the tokens
  // each dequantised stage feeds (804-899 against 937-1067 TFLOP/s). P0MM_GEMM=2 selects Cfg2 (tuning and tests).
  const char *gv = getenv("P0MM_GEMM");
  const bool cfg2 = gv && gv[0] == '2', cfg3 = gv && gv[0] == '3', cfg4 = gv && gv[0] == '4';
  uint32_t BT = M <= 64 ? 64u : (M <= 128 || cfg2) ? 128u : 256u;
  // tuning override, read on every call: P0MM_GEMM_BT=64|128|256 sets the token tile
  const char *btv = getenv("P0MM_GEMM_BT");
  if (btv && !cfg2) {
    const long b = strtol(btv, nullptr, 10);
    if (b == 64 || b == 128 || b == 256) BT = (uint32_t)b;
  }
  // CTA pairs (Cfg5, P0MM_GEMM=5) for q4 weights in 256-token tiles: half the X bytes per SM, measured at ~0.8x Cfg1
  // on the config-3/4 shapes (the pair's per-stage hand-off spans two SMs), so not the default
  const bool pair = gv && gv[0] == '5' && BT == 256u && !f16w && !q8;
  // bulk-copy weight path: every CTA's 128 lanes read two whole 64-row tiles
  const bool wtma = !f16w && (swi ? (a->wr0 % 64 == 0 && a->wr1 % 64 == 0 && (N / 2) % 64 == 0) : (a->wr0 % 64 == 0));
  dim3 grid((N + kBW - 1) / kBW, (M + BT - 1) / BT);
  // Which form (measured on B200, configs 3 and 4; the main loop of every form costs ~0.4-0.5 us per stage whatever
  // the stage's work, so the forms differ in work per stage and in per-tile fixed cost):
  //  * Cfg7, 128-k stages, for q4 records by bulk copy in 256-token tiles: +13-17 % over Cfg1 on all six shapes
  //    (1043-1097 against 957-968 TFLOP/s aggregate in the same runs);
  //  * else the persistent form for q4 records by bulk copy with a store epilogue, when the CTAs get more than one
  //    tile and K is at most 96 stages (it hides the per-tile fixed cost; its 4-stage ring loses on long K);
  //  * else Cfg1.
  // P0MM_GEMM=1..7 forces a form where it applies (tuning and tests): 1 Cfg1, 2..4 variants of it, 5 the CTA pair,
  // 6 the persistent form, 7 Cfg7.
  const bool q4bulk = !f16w && !q8 && wtma;
  const bool k128 = q4bulk && BT == 256u && (gv ? gv[0] == '7' : true);
  const bool ps_ok = q4bulk && a->epi != P0_GEPI_HEADS && a->epi != P0_GEPI_ONORMGATE;
  const uint32_t nk64 = (K + kBK - 1) / kBK, nk = k128 ? (K + 127u) / 128u : nk64;
  const bool persistent = !k128 && ps_ok && (gv ? gv[0] == '6' : (nk64 <= 96u && grid.x * grid.y > (uint32_t)c->sm_count));
  // k split, for grids that fill at most half the SMs (a row shard of few tokens; c3 down at 8 ranks is 48 CTAs):
  // split z runs stages [z * nkz, (z + 1) * nkz) and stores its f32 partial product to the workspace, a second pass
  // sums the splits in order and applies the store epilogue. P0MM_GEMM_KSPLIT=1..8 sets the split count (tuning, tests).
  uint32_t S = 1, nkz = 0;
  const bool split_epi = a->epi == P0_GEPI_F16 || a->epi == P0_GEPI_BIAS || a->epi == P0_GEPI_F32 || a->epi == P0_GEPI_RESADD;
  if (split_epi && !pair && !persistent) {
    const char *ksv = getenv("P0MM_GEMM_KSPLIT");
    const long want = ksv ? strtol(ksv, nullptr, 10) : 0;
    const uint32_t ctas = grid.x * grid.y, sms = (uint32_t)c->sm_count;
    if (want >= 1 && want <= 8) S = (uint32_t)want;
    else if (ctas * 2u <= sms && nk >= 16u) S = min(min(8u, sms / ctas), nk / 4u);
    if (S > nk) S = nk;
    if (S > 1u) {
      nkz = (nk + S - 1u) / S;
      S = (nk + nkz - 1u) / nkz;   // no empty split
    }
    if (S <= 1u) { S = 1u; nkz = 0u; }
  }
  auto enc_fn = tensor_map_encoder();
  if (!enc_fn) return p0_fail(c, P0_EDEVICE, "gemm: cuTensorMapEncodeTiled is unavailable");
  // the context workspace holds the prologue pass's fp16 X and the splits' partial products
  const size_t xws = xmode != P0_XPRO_F16 ? ((size_t)M * K * 2 + 255) / 256 * 256 : 0;
  const size_t pws = S > 1u ? (size_t)S * M * N * 4 : 0;
  uint8_t *wsp = nullptr;
  if (xws + pws) {
    uint32_t *unused_cnt = nullptr;
    void *scratch = nullptr;
    if ((st = p0_workspace(c, 0, xws + pws, &unused_cnt, &scratch))) return st;
    wsp = (uint8_t *)scratch;
  }
  // the fp16 X the GEMM reads: x itself, or the prologue pass's output in the context workspace
  const uint8_t *xbase = rx.base + 2ull * a->x_k0;
  uint32_t xld = ldx;
  if (xmode != P0_XPRO_F16) {
    void *scratch = wsp;
    cudaSetDevice(c->device);
    const uint64_t n8 = (uint64_t)M * (K / 8);
    const unsigned blocks = (unsigned)((n8 + 255) / 256 < (uint64_t)c->sm_count * 8 ? (n8 + 255) / 256 : (uint64_t)c->sm_count * 8);
    gemm_xpro_kernel<<<blocks, 256, 0, c->stream>>>((int)xmode, (const float *)rx.base, ldx, a->x_k0, (const float *)rst.base,
                                                    a->stats_off, (const float *)rpv.base, a->pv_off, a->pv_stride, M, K,
                                                    (uint16_t *)scratch);
    if ((st = p0_launched(c, "gemm x prologue"))) return st;
    xbase = (const uint8_t *)scratch;
    xld = K;
  }
  CUtensorMap tm;
  cuuint64_t dims[2] = {K, M};
  cuuint64_t strides[1] = {(cuuint64_t)xld * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, pair ? BT / 2u : BT};   // pairs: each CTA loads half of the token tile
  cuuint32_t estr[2] = {1, 1};
  CUresult cr = enc_fn(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)xbase, dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return p0_fail(c, P0_EDEVICE, "gemm: tensor map encode failed (%d)", (int)cr);

  GemmParams p{};
  p.W = rw.base; p.Y = (uint8_t *)ry.base; p.EV = (const float *)re.base; p.BV = (const float *)rb.base;
  p.M = M; p.N = N; p.K = K; p.wR0 = a->wr0; p.wR1 = a->wr1; p.wG = wG; p.wk0 = a->wk0; p.Nw = a->w.rows;
  p.ldy = ldy; p.ny0 = a->y_n0; p.evOff = a->ev_off; p.bvOff = a->bv_off; p.bvUp = a->bv_up;
  p.epi = (int)a->epi; p.act = (int)a->act; p.res = (int)a->res; p.store = (int)a->store; p.gate = a->ev.id != 0;
  p.bias = bias; p.post_gelu = (int)a->post_gelu;
  p.RP = (hq || hk) ? (const float *)rrp.base : nullptr; p.GT = og ? (const uint16_t *)rgt.base : nullptr;
  p.Ltot = a->h_Ltot; p.Hq = a->h_Hq; p.Hkv = a->h_Hkv; p.rowOff = a->h_rowOff;
  p.eps = a->h_eps != 0.0f ? a->h_eps : 1e-6f;   // gemm.js:309 `h.eps || 1e-6`
  p.rope_half = a->h_rope_mode == P0_ROPE_HALF;
  p.BT = BT; p.nk = nk; p.err = c->d_err;
  p.wtma = wtma;
  const GemmParams pe = p;   // the call's epilogue, for the k split's second pass
  if (S > 1u) {              // the splits store raw f32 partials [z][m][n]
    p.nkz = nkz;
    p.zstride = (size_t)M * N;
    p.Y = wsp + xws;
    p.epi = P0_GEPI_F32;
    p.ldy = N; p.ny0 = 0; p.res = 0; p.store = 1; p.post_gelu = 0;
    grid.z = S;
  }
  cudaSetDevice(c->device);
  if (f16w) {   // fp16 weights: four stages
    const size_t smem = CfgH::kRingBytes + (size_t)CfgH::kStages * w_stage_e<kWF16>() + 1024 + 256;
    cudaFuncSetAttribute(gemm_q4_tc<CfgH, kWF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    gemm_q4_tc<CfgH, kWF16><<<grid, CfgH::kThreads, smem, c->stream>>>(tm, p);
  } else if (q8) {   // q8 weights: Cfg1's shape
    const size_t smem = Cfg1::kRingBytes + (size_t)Cfg1::kStages * w_stage<true>() + 1024 + 256;
    cudaFuncSetAttribute(gemm_q4_tc<Cfg1, kWQ8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    gemm_q4_tc<Cfg1, kWQ8><<<grid, Cfg1::kThreads, smem, c->stream>>>(tm, p);
  } else if (k128) {
    const size_t smem = Cfg7::kRingBytes + (size_t)Cfg7::kStages * 2u * 4u * 1280u + 1024 + 256;
    cudaFuncSetAttribute(gemm_q4_tc<Cfg7, kWQ4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    gemm_q4_tc<Cfg7, kWQ4><<<grid, Cfg7::kThreads, smem, c->stream>>>(tm, p);
  } else if (persistent) {
    cudaFuncSetAttribute(gemm_q4_ps, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPsSmem);
    const uint32_t nrt = grid.x, ntiles = grid.x * grid.y;
    const uint32_t nctas = ntiles < (uint32_t)c->sm_count ? ntiles : (uint32_t)c->sm_count;
    gemm_q4_ps<<<nctas, kPsThreads, kPsSmem, c->stream>>>(tm, p, nrt, ntiles);
  } else if (pair) {
    const size_t smem = Cfg5::kRingBytes + (size_t)Cfg5::kStages * kWStage + 1024 + 256;
    cudaFuncSetAttribute(gemm_q4_tc<Cfg5, kWQ4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((grid.x + 1u) & ~1u, grid.y);   // whole pairs: an odd CTA past the last row tile stores nothing
    lc.blockDim = dim3(Cfg5::kThreads);
    lc.dynamicSmemBytes = smem;
    lc.stream = c->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    cudaLaunchKernelEx(&lc, gemm_q4_tc<Cfg5, kWQ4>, tm, p);
  } else if (cfg3) {
    const size_t smem = Cfg3::kRingBytes + (size_t)Cfg3::kStages * kWStage + 1024 + 256;
    cudaFuncSetAttribute(gemm_q4_tc<Cfg3, kWQ4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    gemm_q4_tc<Cfg3, kWQ4><<<grid, Cfg3::kThreads, smem, c->stream>>>(tm, p);
  } else if (cfg4) {
    const size_t smem = Cfg4::kRingBytes + (size_t)Cfg4::kStages * kWStage + 1024 + 256;
    cudaFuncSetAttribute(gemm_q4_tc<Cfg4, kWQ4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    gemm_q4_tc<Cfg4, kWQ4><<<grid, Cfg4::kThreads, smem, c->stream>>>(tm, p);
  } else if (cfg2) {
    const size_t smem = Cfg2::kRingBytes + (size_t)Cfg2::kStages * kWStage + 1024 + 256;
    cudaFuncSetAttribute(gemm_q4_tc<Cfg2, kWQ4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    gemm_q4_tc<Cfg2, kWQ4><<<grid, Cfg2::kThreads, smem, c->stream>>>(tm, p);
  } else {
    const size_t smem = Cfg1::kRingBytes + (size_t)Cfg1::kStages * kWStage + 1024 + 256;
    cudaFuncSetAttribute(gemm_q4_tc<Cfg1, kWQ4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    gemm_q4_tc<Cfg1, kWQ4><<<grid, Cfg1::kThreads, smem, c->stream>>>(tm, p);
  }
  if ((st = p0_launched(c, "gemm"))) return st;
  if (S > 1u) {
    const uint64_t n4 = (uint64_t)M * (N / 4);
    const unsigned blocks = (unsigned)((n4 + 255) / 256 < (uint64_t)c->sm_count * 8 ? (n4 + 255) / 256 : (uint64_t)c->sm_count * 8);
    gemm_ksplit_epilogue<<<blocks, 256, 0, c->stream>>>((const float *)(wsp + xws), S, (size_t)M * N, pe);
    if ((st = p0_launched(c, "gemm k-split epilogue"))) return st;
  }
  if (flops) *flops = 2.0 * M * N * K;
  return P0_OK;
}

p0_status p0_dequant_f16(p0_ctx *c, const p0_wview *w, p0_buf out) {
  if (!c || !w) return P0_EINVAL;
  const bool q8 = w->enc == P0_ENC_Q8G64S_T64;
  if (w->enc != P0_ENC_Q4G32A_T64 && !q8) return p0_fail(c, P0_EINVAL, "dequant: encoding %u is not built in this library yet", w->enc);
  const uint32_t GK = q8 ? 64u : 32u, RB = q8 ? 4224u : 1280u;
  if (w->rows % 64 || w->cols % GK) return p0_fail(c, P0_EINVAL, "dequant: needs rows %% 64 and cols %% %u", GK);
  p0_status st;
  P0Range rw, ro;
  const uint32_t wG = w->cols / GK;
  if ((st = p0_range(c, w->buf, w->off, (uint64_t)(w->rows / 64) * wG * RB, "dequant", "W", &rw))) return st;
  if ((uintptr_t)rw.base % 16) return p0_fail(c, P0_EALIGN, "dequant: weight offset must be 16-byte aligned");
  if ((st = p0_range(c, out, 0, (uint64_t)w->rows * w->cols * 2, "dequant", "out", &ro))) return st;
  const uint64_t n = (uint64_t)w->rows * (w->cols / 32);
  cudaSetDevice(c->device);
  if (q8) deq_dump_q8<<<(unsigned)((n + 255) / 256), 256, 0, c->stream>>>(rw.base, w->rows, w->cols, wG, (uint16_t *)ro.base);
  else deq_dump_q4<<<(unsigned)((n + 255) / 256), 256, 0, c->stream>>>(rw.base, w->rows, w->cols, wG, (uint16_t *)ro.base);
  return p0_launched(c, "dequant");
}

}  // extern "C"
