// gemv_v5.cu -- the cluster GEMV for calls with few tiles (the decode chain's QKV / O / FFN / down projections and the
// small config-2 calls), where the whole call is a few MB and its time is latency, not bandwidth.
//
// One output unit (a 64-row tile x k-split, or a geglu gate tile with its up tile) per thread-block cluster of CS CTAs.
// CTA `rank` of the cluster takes a contiguous slice of the unit's records (geglu: ranks < CS/2 slices of the gate
// tile, the others of the up tile). Every warp bulk-copies its share of the slice into shared memory at once (one
// DRAM round trip for the whole call), while the CTA stages its slice of x in one pass. The warps run the v2/v3
// arithmetic (codes as exact fp16 subnormals on mma.sync, x as fp16 hi/lo, acc += s * D + mn * sum(x) per group), sum
// their partials in shared memory in warp order, and rank 0 of the cluster sums the CTAs' partials through distributed
// shared memory in rank order and applies the epilogue. No global scratch, no atomics: the result does not depend on
// timing.
#include <cstdlib>

#include "gemv_common.cuh"

namespace p0gemv {
namespace {

constexpr int kV5Warps = 8;
constexpr int kV5Threads = 32 * kV5Warps;
constexpr uint32_t kV5XUnits = 4;   // staged x: units of 8 k per thread, kept in registers across the sigma reduction

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// every CTA of the cluster has arrived (its shared-memory writes before the arrive are visible to the others)
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// store a float into CTA `rank`'s shared memory at this CTA's shared address `saddr` (the layouts are the same)
__device__ __forceinline__ void st_dsmem(uint32_t saddr, uint32_t rank, float v) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(saddr), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}

// x of groups [gx, gx + n) of one slice, staged in one pass (the v4 staging): B fragments (fp16 hi / lo, permuted k
// order) and per-(group, token) sum(x) / f, indexed by the group's position in the slice. Returns f = 2^24 / sigma.
template <int MT>
__device__ float stage_x_v5(const GemvParams &p, uint32_t gx, uint32_t n, uint4 *xb, float *xsum, float *red) {
  constexpr uint32_t T = kV5Threads;
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  const uint32_t units = n * MT * 4;   // <= kV5XUnits * T (host-checked)
  float v[kV5XUnits][8];
  float mx = 0.0f;
#pragma unroll
  for (uint32_t j = 0; j < kV5XUnits; j++) {
    const uint32_t u = t + j * T;
#pragma unroll
    for (int i = 0; i < 8; i++) v[j][i] = 0.0f;
    if (u < units) {
      const uint32_t gg = u / (MT * 4), rem = u - gg * (MT * 4), m = rem >> 2, c = rem & 3u;
      const uint32_t kb = (gx + gg) * 32 + c * 8;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        v[j][i] = prologue(p, m, kb + i);
        mx = fmaxf(mx, fabsf(v[j][i]));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < kV5Warps; w++) mx = fmaxf(mx, red[w]);
  int e = 0;
  if (mx > 0.0f && mx < INFINITY) frexpf(mx, &e);
  const float sigma = ldexpf(1.0f, 14 - e), f = ldexpf(1.0f, 10 + e), finv = ldexpf(1.0f, -10 - e);
#pragma unroll
  for (uint32_t j = 0; j < kV5XUnits; j++) {
    const uint32_t u = t + j * T;
    float part = 0.0f;
    if (u < units) {
      float hv[8], lv[8];
#pragma unroll
      for (int i = 0; i < 8; i++) {
        part += v[j][i];
        const float vs = v[j][i] * sigma * ((i & 1) ? 0.0625f : 1.0f);
        const float h = __half2float(__float2half_rn(vs));
        hv[i] = h;
        lv[i] = vs - h;
      }
      xb[u * 2] = make_uint4(pack_h2(hv[0], hv[4]), pack_h2(hv[1], hv[5]), pack_h2(hv[2], hv[6]), pack_h2(hv[3], hv[7]));
      xb[u * 2 + 1] = make_uint4(pack_h2(lv[0], lv[4]), pack_h2(lv[1], lv[5]), pack_h2(lv[2], lv[6]), pack_h2(lv[3], lv[7]));
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    if (u < units && (u & 3u) == 0) xsum[u >> 2] = part * finv;
  }
  __syncthreads();
  return f;
}

// q8 slices: x of groups [gx, gx + n) (64 k each) as fp16 hi / lo in the order of the q8 A fragments (see Rec8):
// entry ((group * MT + token) * 4 + chunk) * 4 + c = {hi(k0, k1), hi(k2, k3), lo(k0, k1), lo(k2, k3)} for k = 16 chunk
// + 4c + 0..3. The codes are integers, so f = 1 / sigma.
template <int MT>
__device__ float stage_x_v5q8(const GemvParams &p, uint32_t gx, uint32_t n, uint4 *xb8, float *red) {
  constexpr uint32_t T = kV5Threads;
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  const uint32_t units = n * MT * 8;   // units of 8 consecutive k; <= kV5XUnits * T (host-checked)
  float v[kV5XUnits][8];
  float mx = 0.0f;
#pragma unroll
  for (uint32_t j = 0; j < kV5XUnits; j++) {
    const uint32_t u = t + j * T;
#pragma unroll
    for (int i = 0; i < 8; i++) v[j][i] = 0.0f;
    if (u < units) {
      const uint32_t gg = u / (MT * 8), rem = u - gg * (MT * 8), m = rem >> 3, cp = rem & 7u;
      const uint32_t kb = (gx + gg) * 64 + cp * 8;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        v[j][i] = prologue(p, m, kb + i);
        mx = fmaxf(mx, fabsf(v[j][i]));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < kV5Warps; w++) mx = fmaxf(mx, red[w]);
  int e = 0;
  if (mx > 0.0f && mx < INFINITY) frexpf(mx, &e);
  const float sigma = ldexpf(1.0f, 14 - e), f = ldexpf(1.0f, e - 14);
#pragma unroll
  for (uint32_t j = 0; j < kV5XUnits; j++) {
    const uint32_t u = t + j * T;
    if (u < units) {
      const uint32_t gg = u / (MT * 8), rem = u - gg * (MT * 8), m = rem >> 3, cp = rem & 7u;
#pragma unroll
      for (int hc = 0; hc < 2; hc++) {
        float hv[4], lv[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float vs = v[j][4 * hc + i] * sigma;   // exact power of two
          const float h = __half2float(__float2half_rn(vs));
          hv[i] = h;
          lv[i] = vs - h;
        }
        const uint32_t c = 2u * (cp & 1u) + hc;
        xb8[((gg * MT + m) * 4 + (cp >> 1)) * 4 + c] =
            make_uint4(pack_h2(hv[0], hv[1]), pack_h2(hv[2], hv[3]), pack_h2(lv[0], lv[1]), pack_h2(lv[2], lv[3]));
      }
    }
  }
  __syncthreads();
  return f;
}

// record bytes and x staging bytes per (group, token) of each encoding
__host__ __device__ constexpr uint32_t v5_rec_bytes(bool q8) { return q8 ? 4224u : 1280u; }
__host__ __device__ constexpr uint32_t v5_xb_bytes(bool q8) { return q8 ? 256u : 128u; }

size_t v5_smem(uint32_t M, uint32_t nmax, bool q8) {
  return (size_t)nmax * v5_rec_bytes(q8) + (size_t)nmax * M * v5_xb_bytes(q8) + (size_t)nmax * M * 4 + (size_t)kV5Warps * M * 64 * 4 +
         (size_t)8 * M * 64 * 4 + kV5Warps * 8 + 64 * 4;
}

template <int MT, bool PAIR, bool Q8>
__global__ void __launch_bounds__(kV5Threads, 2) gemv_q4_v5(const __grid_constant__ GemvParams p, const __grid_constant__ V5Plan pl) {
  constexpr bool PACK = MT <= 4;
  constexpr uint32_t RB = v5_rec_bytes(Q8), XB = v5_xb_bytes(Q8);
  extern __shared__ __align__(128) uint8_t smem8[];
  const uint32_t CS = pl.CS, rank = CS > 1u ? cluster_rank() : 0u, unit = blockIdx.x / CS;
  // ---- this CTA's slice: records [j0, j1) of tile `wt` (the weight tile it reads), groups gx.. of x
  uint32_t tile, split = 0, j0, j1, wt;
  if (PAIR) {
    const uint32_t hr = CS / 2u, half = rank / hr, rr = rank - half * hr;
    tile = unit;
    j0 = rr * pl.G / hr;
    j1 = (rr + 1u) * pl.G / hr;
    wt = tile + half * pl.ntile;
  } else {
    tile = unit / pl.nsplit;
    split = unit - tile * pl.nsplit;
    const uint32_t u0 = split * pl.Gs, nu = min(u0 + pl.Gs, pl.G) - u0;
    j0 = u0 + rank * nu / CS;
    j1 = u0 + (rank + 1u) * nu / CS;
    wt = tile;
  }
  const uint32_t n = j1 - j0;   // >= 1 (host-checked)
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem8);                        // [warps]
  float *misc = reinterpret_cast<float *>(bars + kV5Warps);                    // 64 floats
  volatile uint32_t *abort_flag = reinterpret_cast<volatile uint32_t *>(misc + 32);
  uint8_t *recs = reinterpret_cast<uint8_t *>(misc + 64);                      // [nmax] x RB (16-byte aligned)
  uint4 *xb = reinterpret_cast<uint4 *>(recs + (size_t)pl.nmax * RB);         // [nmax][MT] x XB
  float *xsum = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(xb) + (size_t)pl.nmax * MT * XB);   // [nmax][MT] (q4)
  float *red = xsum + (size_t)pl.nmax * MT;                                   // [warps][MT][64]
  float *gath = red + kV5Warps * MT * 64;   // [rank][MT][64]: in rank 0, every CTA's slice total
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t g = lane >> 2, c = lane & 3;
  // ---- every warp copies its share of the slice at once
  const uint32_t wa = warp * n / kV5Warps, wb = (warp + 1u) * n / kV5Warps, wn = wb - wa;
  if (lane == 0) {
    tc::mbar_init(&bars[warp], 1);
    tc::fence_mbar_init();
  }
  if (threadIdx.x == 0) *abort_flag = 0u;
  __syncwarp();
  if (!p.overlap) pdl_wait();
  if (lane == 0 && wn) {
    tc::mbar_expect_tx(&bars[warp], wn * RB);
    bulk_g2s(recs + (size_t)wa * RB, p.W + ((size_t)wt * p.wG + j0 + wa) * RB, wn * RB, &bars[warp]);
  }
  pdl_trigger();
  if (p.overlap) pdl_wait();
  // j0 is also the slice's first group of x
  const float f = Q8 ? stage_x_v5q8<MT>(p, j0, n, xb, misc) : stage_x_v5<MT>(p, j0, n, xb, xsum, misc);

  // ---- the warp's records: pairs, both loaded before the math (the v3 loop)
  const uint32_t btok = PACK ? (g & 3u) : g, bsel = PACK ? (g >> 2) : 0u;
  const bool tok_ok = btok < MT, xs_lane = !PACK || c < 2;
  const uint32_t rec_s = tc::smem_u32(recs), xb_s = tc::smem_u32(xb), xsum_s = tc::smem_u32(xsum);
  const uint32_t lane_row16 = (uint32_t)lane * 16u, tail_off = 1024u + g * 4u;
  const uint32_t xb_lane = xb_s + btok * 128u + c * 32u + bsel * 16u, xs_addr = xsum_s + 2u * c * 4u;
  float acc[2][4][4];
#pragma unroll
  for (int h = 0; h < 2; h++)
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int i = 0; i < 4; i++) acc[h][r][i] = 0.0f;
  bool ok = true;
  if (wn) {
    const bool got = tc::mbar_wait(&bars[warp], 0, abort_flag, p.err, 0x711u, P0_SPIN_LIMIT);
    ok = __all_sync(0xffffffffu, got);
    if (Q8) {
      // one 4224-byte record at a time (its 32 code words per lane fill the registers a second record would take)
      const uint32_t xb8_s = tc::smem_u32(xb);
      for (uint32_t k = 0; ok && k < wn; k++) {
        const uint32_t gA = wa + k;
        Rec8 q;
        rec8_load(q, rec_s + gA * RB, (uint32_t)lane);
        uint4 b[4];
#pragma unroll
        for (int j = 0; j < 4; j++)
          b[j] = tok_ok ? lds128(xb8_s + (((gA * MT + btok) * 4u + (uint32_t)j) * 4u + c) * 16u) : make_uint4(0, 0, 0, 0);
        rec8_math<MT, PACK>(acc[0], q, b, bsel);
      }
    }
    for (uint32_t k = 0; !Q8 && ok && k < wn; k += 2) {
      const uint32_t gA = wa + k, gB = k + 1u < wn ? gA + 1u : gA;   // positions in the slice
      const bool two = k + 1u < wn;
      Rec q0, q1;
      rec_load(q0, rec_s + gA * 1280u, lane_row16, tail_off);
      if (two) rec_load(q1, rec_s + gB * 1280u, lane_row16, tail_off);
      uint4 bh0 = make_uint4(0, 0, 0, 0), bl0 = bh0, bh1 = bh0, bl1 = bh0;
      float x00 = 0.0f, x01 = 0.0f, x10 = 0.0f, x11 = 0.0f;
      if (tok_ok) {
        bh0 = lds128(xb_lane + gA * MT * 128u);
        if (!PACK) bl0 = lds128(xb_lane + gA * MT * 128u + 16u);
        bh1 = lds128(xb_lane + gB * MT * 128u);
        if (!PACK) bl1 = lds128(xb_lane + gB * MT * 128u + 16u);
      }
      if (xs_lane) {
        if (2 * c < MT) { x00 = __uint_as_float(lds32(xs_addr + gA * MT * 4u)); x10 = __uint_as_float(lds32(xs_addr + gB * MT * 4u)); }
        if (2 * c + 1 < MT) { x01 = __uint_as_float(lds32(xs_addr + gA * MT * 4u + 4u)); x11 = __uint_as_float(lds32(xs_addr + gB * MT * 4u + 4u)); }
      }
      rec_math<MT, PACK>(acc[0], q0, bh0, bl0, x00, x01);
      if (two) rec_math<MT, PACK>(acc[1], q1, bh1, bl1, x10, x11);
    }
  }
  // ---- the warp's totals (x f; PACK: hi + lo columns) -> red[warp][m][row]
  const bool holder = !PACK || c < 2u;
#pragma unroll
  for (int r = 0; r < 4; r++)
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float v = (acc[0][r][i] + acc[1][r][i]) * f;
      if (PACK) v += __shfl_xor_sync(0xffffffffu, v, 2);
      const uint32_t row = 16u * r + g + (i >= 2 ? 8u : 0u), m = 2u * c + (i & 1);
      if (holder && m < MT) red[(warp * MT + m) * 64u + row] = v;
    }
  __syncthreads();
  // the CTA's slice total, summed in warp order, pushed into rank 0's gath[rank] (remote stores, no round trips)
  const uint32_t gath_s = tc::smem_u32(gath) + rank * (MT * 64u) * 4u;
  for (uint32_t idx = threadIdx.x; idx < MT * 64u; idx += kV5Threads) {
    float sum = 0.0f;
#pragma unroll
    for (int w = 0; w < kV5Warps; w++) sum += red[w * MT * 64u + idx];
    if (CS > 1u) st_dsmem(gath_s + idx * 4u, 0u, sum);
    else gath[idx] = sum;
  }
  if (CS > 1u) cluster_sync();   // the release / acquire pair makes every rank's stores visible in rank 0
  else __syncthreads();
  // ---- rank 0: the unit's total (the ranks' parts in rank order; geglu: gate ranks, then up ranks) and the epilogue;
  // warp m takes token m, lane l rows l and l + 32
  if (rank == 0u && warp < MT && ok && !*abort_flag) {
    const uint32_t m = warp;
    float t[2], u2[2] = {0.0f, 0.0f};
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const uint32_t idx = m * 64u + lane + 32u * h;
      const uint32_t hr = PAIR ? CS / 2u : CS;
      float a = 0.0f, b = 0.0f;
      for (uint32_t r = 0; r < hr; r++) a += gath[r * MT * 64u + idx];
      if (PAIR)
        for (uint32_t r = hr; r < CS; r++) b += gath[r * MT * 64u + idx];
      t[h] = a;
      u2[h] = b;
    }
    const uint32_t R0 = tile * 64u;
    if (PAIR) {
#pragma unroll
      for (int h = 0; h < 2; h++) p.Y[(size_t)m * p.ldm + R0 + lane + 32u * h] = __fmul_rn(gelu_l(t[h]), u2[h]);
    } else if (p.epi == P0_EPI_SOFTCAP) {
      float bv = -INFINITY;
      uint32_t bi = 0xffffffffu;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const float v = __fmul_rn(p.cap, tanhf(fminf(15.0f, fmaxf(-15.0f, __fdiv_rn(t[h], p.cap)))));
        p.Y[(size_t)m * p.ldm + R0 + lane + 32u * h] = v;
        if (v > bv) { bv = v; bi = lane + 32u * h; }   // h = 0 first: ties keep the lower row
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) {
        const size_t o = ((size_t)m * p.ntile + tile) * 2;
        p.MX[o] = bv;
        p.MX[o + 1] = __uint_as_float(R0 + bi);
      }
    } else {
#pragma unroll
      for (int h = 0; h < 2; h++) p.Y[(size_t)split * p.ldy + (size_t)m * p.ldm + R0 + lane + 32u * h] = t[h];
    }
  }
  // a copy whose wait gave up lands before the CTA exits (bounded)
  if (!ok && lane == 0 && wn) {
    volatile uint32_t never = 0;
    tc::mbar_wait(&bars[warp], 0, &never, p.err, 0x712u, P0_SPIN_LIMIT);
  }
}

typedef void (*V5Kernel)(const GemvParams, const V5Plan);
template <int MT>
V5Kernel v5_kernel_m(bool pair, bool q8) {
  return q8 ? (pair ? gemv_q4_v5<MT, true, true> : gemv_q4_v5<MT, false, true>)
            : (pair ? gemv_q4_v5<MT, true, false> : gemv_q4_v5<MT, false, false>);
}
V5Kernel v5_kernel_for(uint32_t M, bool pair, bool q8) {
  switch (M) {
    case 1: return v5_kernel_m<1>(pair, q8);
    case 2: return v5_kernel_m<2>(pair, q8);
    case 3: return v5_kernel_m<3>(pair, q8);
    case 4: return v5_kernel_m<4>(pair, q8);
    case 5: return v5_kernel_m<5>(pair, q8);
    case 6: return v5_kernel_m<6>(pair, q8);
    case 7: return v5_kernel_m<7>(pair, q8);
    default: return v5_kernel_m<8>(pair, q8);
  }
}
}  // namespace

bool v5_plan(const GemvParams &p, uint32_t nsplit, int sms, V5Plan *pl) {
  const bool q8 = p.q8 != 0;
  const uint32_t GK = q8 ? 64u : 32u, G = p.K / GK;
  const bool pair = p.epi == P0_EPI_GEGLU;
  if (G == 0 || p.wG < G || (pair && nsplit != 1)) return false;
  const uint32_t ntile = p.N / 64, Gs = p.kPer / GK < G ? p.kPer / GK : G;
  const uint64_t units = pair ? ntile : (uint64_t)ntile * nsplit;
  const uint32_t nu = pair ? G : Gs;   // records per unit (per half for geglu)
  // the smallest cluster that reaches a CTA count, within the staging and shared-memory limits: one CTA per SM for
  // M <= 2, two for M >= 4 (measured on B200: at M = 4 the per-CTA x staging and math gain from the spread, N = 16384
  // 14.2 against 15.8 us; at M = 1 the extra cluster traffic costs, 11.3 against 8.2 us). P0MM_V5_CTAS, a tuning
  // override, sets the CTA count instead.
  const char *tv = getenv("P0MM_V5_CTAS");
  const long tn = tv ? strtol(tv, nullptr, 10) : 0;
  const uint64_t target = tn > 0 && tn < 100000 ? (uint64_t)tn : (uint64_t)sms * (p.M >= 4 ? 2u : 1u);
  uint32_t best = 0;
  for (uint32_t CS = pair ? 2u : 1u; CS <= 8u; CS *= 2u) {
    const uint32_t parts = pair ? CS / 2u : CS;
    if (parts > nu) break;
    const uint32_t nmax = (nu + parts - 1) / parts;
    if (nmax * p.M * (q8 ? 8u : 4u) > kV5XUnits * kV5Threads || v5_smem(p.M, nmax, q8) > 200u * 1024u) continue;
    best = CS;
    if (units * CS >= target) break;
  }
  // many tiles: the streaming kernels take q4 calls; q8 calls have only this kernel, in as many waves as they need
  if (!best || (!q8 && units * best > (uint64_t)sms * 8)) return false;
  const uint32_t parts = pair ? best / 2u : best;
  pl->CS = best; pl->nsplit = nsplit; pl->Gs = Gs; pl->G = G; pl->ntile = ntile; pl->pair = pair;
  pl->nmax = (nu + parts - 1) / parts;
  pl->units = (uint32_t)units;
  return true;
}

cudaError_t launch_v5(const GemvParams &p, const V5Plan &pl, cudaStream_t s) {
  V5Kernel k = v5_kernel_for(p.M, pl.pair != 0, p.q8 != 0);
  const size_t smem = v5_smem(p.M, pl.nmax, p.q8 != 0);
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return launch_pdl(k, dim3(pl.units * pl.CS), dim3(kV5Threads), smem, s, pl.CS, p, pl);
}

}  // namespace p0gemv
