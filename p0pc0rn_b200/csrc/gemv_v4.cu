// gemv_v4.cu -- the stream-K GEMV: every warp of the grid gets an equal, contiguous range of weight records.
//
// The records of a q4g32a.t64 weight (tile t, group g at (t*wG + g) * 1280 bytes; wG = the view's columns / 32, G = K / 32
// of them per tile used) form one stream in (tile, group) order. Warp w of NW takes records [w*R/NW, (w+1)*R/NW) of
// the R = ntile * G records, streams them through a private ring of shared-memory slots (two records per slot, refilled
// by its lane 0 with cp.async.bulk as soon as the slot is in registers) and runs the arithmetic of the v2/v3 kernels
// (codes as exact fp16 subnormals on mma.sync, x as fp16 hi/lo, per group acc += s * D + mn * sum(x) in f32).
//
// An output unit is (tile, k-split): rows t*64 .. t*64+63 of split s, whose records are the unit's groups. A warp
// that holds every record of a unit applies the epilogue itself. A unit shared by several warps (its records cross a
// range boundary) is combined through a workspace: each warp writes its compact partial [M][64] to slot (unit + w),
// then increments the unit's arrival counter; the warp that arrives last sums the parts in warp order (fixed, so the
// result does not depend on arrival order), applies the epilogue and sets the counter back to zero for the next call.
// No warp waits for another: a warp that is not last simply moves on.
//
// Unlike the whole-tile-per-warp v3 kernel, no warp idles while others finish a last tile (4096 head tiles over 2368
// warps leave v3 a 1.73 : 2 load balance), and calls with few tiles still spread over many SMs.
#include <cstdlib>
#include <mutex>

#include "gemv_common.cuh"

namespace p0gemv {
namespace {

constexpr int kV4Warps = 16;
constexpr int kV4Threads = 32 * kV4Warps;
constexpr uint32_t kV4Slot = 2560;
constexpr uint32_t kV4MaxSlots = 4;
constexpr uint32_t kV4XUnits = 4;   // staged x: units of 8 k per thread (registers hold them between the two passes)

// the warp that owns record j: the largest w with floor(w * R / NW) <= j
__device__ __forceinline__ uint32_t v4_owner(uint32_t j, uint32_t R, uint32_t NW) {
  return (uint32_t)((((uint64_t)j + 1u) * NW - 1u) / R);
}

// x staging in one pass over x: each thread keeps its (at most kV4XUnits) units of 8 values in registers while the
// block agrees on sigma, then writes the B fragments (fp16 hi / lo, permuted k order) and the per-(group, token)
// sum(x) / f. Returns f = 2^24 / sigma.
template <int MT>
__device__ float stage_x_v4(const GemvParams &p, uint32_t G, uint4 *xb, float *xsum, float *red) {
  constexpr uint32_t T = kV4Threads;
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  const uint32_t units = G * MT * 4;   // <= kV4XUnits * T (host-checked)
  float v[kV4XUnits][8];
  float mx = 0.0f;
#pragma unroll
  for (uint32_t j = 0; j < kV4XUnits; j++) {
    const uint32_t u = t + j * T;
#pragma unroll
    for (int i = 0; i < 8; i++) v[j][i] = 0.0f;
    if (u < units) {
      const uint32_t gg = u / (MT * 4), rem = u - gg * (MT * 4), m = rem >> 2, c = rem & 3u;
      const uint32_t kb = gg * 32 + c * 8;
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
  for (int w = 1; w < kV4Warps; w++) mx = fmaxf(mx, red[w]);
  int e = 0;
  if (mx > 0.0f && mx < INFINITY) frexpf(mx, &e);             // mx < 2^e
  const float sigma = ldexpf(1.0f, 14 - e), f = ldexpf(1.0f, 10 + e), finv = ldexpf(1.0f, -10 - e);
#pragma unroll
  for (uint32_t j = 0; j < kV4XUnits; j++) {
    const uint32_t u = t + j * T;
    float part = 0.0f;
    if (u < units) {
      float hv[8], lv[8];
#pragma unroll
      for (int i = 0; i < 8; i++) {
        part += v[j][i];
        const float vs = v[j][i] * sigma * ((i & 1) ? 0.0625f : 1.0f);   // exact powers of two
        const float h = __half2float(__float2half_rn(vs));
        hv[i] = h;
        lv[i] = vs - h;
      }
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

// a unit's row totals in the mma D-fragment layout of the warp: lane (g, c), row-block r, element i -> row
// 16r + g + 8*(i >= 2), token 2c + (i & 1) (PACK: lanes c < 2 hold the tokens)
struct V4Tot {
  float v[4][4];
};

// the first and last record (in the call's record stream) of unit u
__device__ __forceinline__ void v4_unit_range(const V4Plan &pl, uint32_t u, uint32_t &rf, uint32_t &rl) {
  const uint32_t tile = u / pl.nsplit, split = u - tile * pl.nsplit;
  rf = tile * pl.Gt + split * pl.Gs;
  rl = min(rf + pl.Gs, tile * pl.Gt + pl.Gt) - 1u;
}

// completes unit u for this warp: the epilogue directly when the warp holds the whole unit, else the workspace
// hand-off described at the top of the file. PAIR (geglu): `a` holds the gate rows' totals, `b` the up rows' (zeros for
// a half this warp has no records of); else `a` holds the unit's totals.
template <int MT, bool PAIR>
__device__ __noinline__ void v4_flush(const GemvParams &p, const V4Plan &pl, V4Tot a, V4Tot b, uint32_t u, bool whole, uint32_t w) {
  constexpr bool PACK = MT <= 4;
  constexpr uint32_t H = PAIR ? 2u : 1u;
  const uint32_t lane = threadIdx.x & 31u, g = lane >> 2, c = lane & 3u;
  const bool holder = !PACK || c < 2u;   // lanes whose values are the unit's (PACK: c = 2, 3 hold copies)
  const uint32_t tile = u / pl.nsplit, split = u - tile * pl.nsplit;
  if (!whole) {
    float *ps = pl.part + (size_t)(u + w) * (H * MT * 64u);
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t n = 16u * r + g + (i >= 2 ? 8u : 0u), m = 2u * c + (i & 1);
        if (holder && m < MT) {
          ps[m * 64u + n] = a.v[r][i];
          if (PAIR) ps[MT * 64u + m * 64u + n] = b.v[r][i];
        }
      }
    __threadfence();
    __syncwarp();
    uint32_t old = 0;
    if (lane == 0) old = atomicAdd(&pl.cnt[u], 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    uint32_t rf, rl;
    v4_unit_range(pl, u, rf, rl);
    const uint32_t wf = v4_owner(rf, pl.R, pl.NW), nparts = v4_owner(rl, pl.R, pl.NW) - wf + 1u;
    if (old + 1u != nparts) return;   // another warp completes the unit
    __threadfence();
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int i = 0; i < 4; i++) a.v[r][i] = b.v[r][i] = 0.0f;
    for (uint32_t k = 0; k < nparts; k++) {
      const float *pk = pl.part + (size_t)(u + wf + k) * (H * MT * 64u);
#pragma unroll
      for (int r = 0; r < 4; r++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const uint32_t n = 16u * r + g + (i >= 2 ? 8u : 0u), m = 2u * c + (i & 1);
          if (holder && m < MT) {
            a.v[r][i] += __ldcg(pk + m * 64u + n);
            if (PAIR) b.v[r][i] += __ldcg(pk + MT * 64u + m * 64u + n);
          }
        }
    }
    if (lane == 0) pl.cnt[u] = 0u;   // every part has arrived: the counter is free for the next call
  }
  // ---- epilogue of the unit (the v2 / v3 contract)
  const uint32_t R0 = tile * 64u, tk0 = 2u * c, tk1 = 2u * c + 1u;
  if (!PAIR && p.epi == P0_EPI_SOFTCAP) {
    float bv0 = -INFINITY, bv1 = -INFINITY;
    uint32_t bi0 = 0xffffffffu, bi1 = 0xffffffffu;
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t n = R0 + 16u * r + g + (i >= 2 ? 8u : 0u), m = (i & 1) ? tk1 : tk0;
        const float v = __fmul_rn(p.cap, tanhf(fminf(15.0f, fmaxf(-15.0f, __fdiv_rn(a.v[r][i], p.cap)))));
        if (m < MT) p.Y[(size_t)m * p.ldm + n] = v;
        const uint32_t rr = n & 63u;
        if (i & 1) { if (v > bv1 || (v == bv1 && rr < bi1)) { bv1 = v; bi1 = rr; } }
        else { if (v > bv0 || (v == bv0 && rr < bi0)) { bv0 = v; bi0 = rr; } }
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
      if (tk0 < MT) { const size_t o = ((size_t)tk0 * p.ntile + tile) * 2; p.MX[o] = bv0; p.MX[o + 1] = __uint_as_float(R0 + bi0); }
      if (tk1 < MT) { const size_t o = ((size_t)tk1 * p.ntile + tile) * 2; p.MX[o] = bv1; p.MX[o + 1] = __uint_as_float(R0 + bi1); }
    }
  } else {
    const size_t so = (size_t)split * p.ldy;
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t n = R0 + 16u * r + g + (i >= 2 ? 8u : 0u), m = (i & 1) ? tk1 : tk0;
        if (m >= MT) continue;
        if (PAIR) p.Y[(size_t)m * p.ldm + n] = __fmul_rn(gelu_l(a.v[r][i]), b.v[r][i]);
        else p.Y[so + (size_t)m * p.ldm + n] = a.v[r][i];
      }
  }
}

// after a failed wait: the warp still arrives on every shared unit of its range (from unit u0 on), so that every
// counter returns to zero; the results of the call are void (its error is reported)
__device__ __noinline__ void v4_arrive_only(const V4Plan &pl, uint32_t u0, uint32_t r1) {
  if ((threadIdx.x & 31u) != 0u) return;
  const uint32_t tl = (r1 - 1u) / pl.Gt, gl = (r1 - 1u) - tl * pl.Gt;
  const uint32_t ulast = tl * pl.nsplit + (pl.nsplit > 1u ? gl / pl.Gs : 0u);
  for (uint32_t u = u0; u <= ulast; u++) {
    uint32_t rf, rl;
    v4_unit_range(pl, u, rf, rl);
    const uint32_t nparts = v4_owner(rl, pl.R, pl.NW) - v4_owner(rf, pl.R, pl.NW) + 1u;
    if (nparts > 1u && atomicAdd(&pl.cnt[u], 1u) + 1u == nparts) pl.cnt[u] = 0u;
  }
}

// The warp's range is walked as segments: maximal runs of records inside one unit and (geglu) one half of it. Within a
// segment the records are consecutive groups of one tile, so the per-slot work is the same as v3's; the unit
// bookkeeping runs only where a segment ends.
// seg_end(rec, r1): the end (exclusive) of the segment that starts at stream record rec
__device__ __forceinline__ uint32_t v4_seg_end(const V4Plan &pl, uint32_t rec, uint32_t r1) {
  const uint32_t t = rec / pl.Gt, j = rec - t * pl.Gt;
  uint32_t e = (t + 1u) * pl.Gt;                                       // tile end
  if (pl.Gt != pl.G) { if (j < pl.G) e = t * pl.Gt + pl.G; }          // geglu: end of the gate half
  else if (pl.nsplit > 1u) e = min(e, t * pl.Gt + (j / pl.Gs + 1u) * pl.Gs);   // end of the k-split
  return min(e, r1);
}

template <int MT, bool PAIR>
__global__ void __launch_bounds__(kV4Threads, 1) gemv_q4_v4(const __grid_constant__ GemvParams p, const __grid_constant__ V4Plan pl) {
  constexpr bool PACK = MT <= 4;
  extern __shared__ __align__(128) uint8_t smem8[];
  const uint32_t nslot = pl.nslot, G = pl.G, Gt = pl.Gt;
  uint8_t *ring = smem8;                                                              // [warp][slot] x 2560 B
  uint64_t *full = reinterpret_cast<uint64_t *>(ring + (size_t)kV4Warps * nslot * kV4Slot);
  float *red = reinterpret_cast<float *>(full + kV4Warps * kV4MaxSlots);              // 32 floats
  volatile uint32_t *abort_flag = reinterpret_cast<volatile uint32_t *>(red + 24);
  uint4 *xb = reinterpret_cast<uint4 *>(red + 32);                                    // [G][MT][4][2]
  float *xsum = reinterpret_cast<float *>(xb + (size_t)G * MT * 8);                   // [G][MT]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t g = lane >> 2, c = lane & 3;
  const uint32_t w = blockIdx.x * kV4Warps + warp;
  const uint32_t r0 = (uint32_t)((uint64_t)w * pl.R / pl.NW), r1 = (uint32_t)((uint64_t)(w + 1u) * pl.R / pl.NW);
  uint8_t *myring = ring + (size_t)warp * nslot * kV4Slot;
  uint64_t *myfull = full + warp * kV4MaxSlots;
  if (lane == 0) {
    for (uint32_t i = 0; i < nslot; i++) tc::mbar_init(&myfull[i], 1);
    tc::fence_mbar_init();
  }
  if (threadIdx.x == 0) *abort_flag = 0u;
  __syncwarp();
  // ---- the issue side (lane 0 only): the same segments, one or two records per slot (a slot never crosses a
  // segment). Stream record (t, j) sits at (t * wG + j) * 1280; geglu: j >= G is record j - G of up tile t + ntile.
  // Incremental: the address advances by 1280 per record inside a segment; divisions run only at segment starts.
  auto seg_src = [&](uint32_t rec) -> const uint8_t * {
    uint32_t t = rec / Gt, j = rec - t * Gt;
    if (PAIR && j >= G) { t += pl.ntile; j -= G; }
    return p.W + ((size_t)t * p.wG + j) * 1280u;
  };
  uint32_t i_rec = r0, i_left = v4_seg_end(pl, r0, r1) - r0, issued = 0;
  const uint8_t *i_src = seg_src(r0);
  auto issue_next = [&](uint32_t slot) {
    const uint32_t n = i_left >= 2u ? 2u : 1u;
    tc::mbar_expect_tx(&myfull[slot], n * 1280u);
    bulk_g2s(myring + (size_t)slot * kV4Slot, i_src, n * 1280u, &myfull[slot]);
    i_rec += n;
    i_left -= n;
    i_src += n * 1280u;
    if (i_left == 0u && i_rec < r1) {
      i_left = v4_seg_end(pl, i_rec, r1) - i_rec;
      i_src = seg_src(i_rec);
    }
    issued++;
  };
  if (!p.overlap) pdl_wait();
  if (lane == 0)
    for (uint32_t k = 0; k < nslot && i_rec < r1; k++) issue_next(k);   // these fly while x is staged
  pdl_trigger();
  if (p.overlap) pdl_wait();
  const float f = stage_x_v4<MT>(p, G, xb, xsum, red);

  const uint32_t btok = PACK ? (g & 3u) : g, bsel = PACK ? (g >> 2) : 0u;   // B column of this lane
  const bool tok_ok = btok < MT, xs_lane = !PACK || c < 2;
  const uint32_t ring_s = tc::smem_u32(myring), xb_s = tc::smem_u32(xb), xsum_s = tc::smem_u32(xsum);
  const uint32_t lane_row16 = (uint32_t)lane * 16u, tail_off = 1024u + g * 4u;
  const uint32_t xb_lane = xb_s + btok * 128u + c * 32u + bsel * 16u, xs_addr = xsum_s + 2u * c * 4u;

  float acc[2][4][4];   // [record parity]: independent FMA chains for the two records of a slot
  V4Tot gate;           // geglu: the gate half's totals once the warp has moved on to the up half
  auto zero = [&]() {
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
      for (int r = 0; r < 4; r++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[h][r][i] = 0.0f;
  };
  auto totals = [&]() {
    V4Tot t;
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        float v = (acc[0][r][i] + acc[1][r][i]) * f;
        if (PACK) v += __shfl_xor_sync(0xffffffffu, v, 2);
        t.v[r][i] = v;
      }
    return t;
  };
  auto clear = [&](V4Tot &t) {
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int i = 0; i < 4; i++) t.v[r][i] = 0.0f;
  };
  zero();
  clear(gate);
  uint32_t cs = 0, cph = 0, consumed = 0;
  bool ok = true, from_start = false, in_up = false;
  uint32_t rec = r0;
  while (rec < r1 && ok) {
    const uint32_t e = v4_seg_end(pl, rec, r1);
    const uint32_t t = rec / Gt, j = rec - t * Gt;
    const uint32_t u = t * pl.nsplit + (pl.nsplit > 1u ? j / pl.Gs : 0u);
    const bool ustart = j == 0u || (pl.nsplit > 1u && j % pl.Gs == 0u);
    if (ustart || rec == r0) { from_start = ustart; in_up = PAIR && j >= G; }
    const uint32_t g0 = PAIR && j >= G ? j - G : j, len = e - rec;
    for (uint32_t k = 0; 2u * k < len; k++) {
      const bool got = tc::mbar_wait(&myfull[cs], cph, abort_flag, p.err, 0x611u, P0_SPIN_LIMIT);
      if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
      consumed++;
      const uint32_t sl = ring_s + cs * kV4Slot;
      const bool two = 2u * k + 1u < len;
      const uint32_t gA = g0 + 2u * k, gB = two ? gA + 1u : gA;
      // all shared loads of the slot first
      Rec q0, q1;
      rec_load(q0, sl, lane_row16, tail_off);
      if (two) rec_load(q1, sl + 1280u, lane_row16, tail_off);
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
      // every lane has read the slot: lane 0 refills it (generic reads before the async-proxy write: warp sync, then a
      // proxy fence); the math below uses registers only
      __syncwarp();
      if (lane == 0 && i_rec < r1) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue_next(cs);
      }
      if (++cs == nslot) { cs = 0; cph ^= 1u; }
      rec_math<MT, PACK>(acc[0], q0, bh0, bl0, x00, x01);
      if (two) rec_math<MT, PACK>(acc[1], q1, bh1, bl1, x10, x11);
    }
    if (!ok) break;
    rec = e;
    // the segment ends at the end of its unit, at the end of the range, or (geglu) at the end of the gate half
    uint32_t rf, rl;
    v4_unit_range(pl, u, rf, rl);
    if (PAIR && !in_up && e <= rl && e < r1) {   // gate half done, the up half follows in this warp
      gate = totals();
      zero();
      in_up = true;
      continue;
    }
    const bool whole = from_start && e == rl + 1u;
    if (PAIR) {
      V4Tot z;
      clear(z);
      if (in_up) v4_flush<MT, PAIR>(p, pl, gate, totals(), u, whole, w);
      else v4_flush<MT, PAIR>(p, pl, totals(), z, u, whole, w);
      clear(gate);
    } else {
      const V4Tot tt = totals();
      v4_flush<MT, PAIR>(p, pl, tt, tt, u, whole, w);
    }
    zero();
  }
  if (!ok) {
    const uint32_t t = rec / Gt, j = rec - t * Gt;
    v4_arrive_only(pl, t * pl.nsplit + (pl.nsplit > 1u ? j / pl.Gs : 0u), r1);
    // copies this warp issued but did not consume land before the CTA exits (bounded)
    if (lane == 0) {
      volatile uint32_t never = 0;
      uint32_t slot = cs, ph = cph;
      for (uint32_t k = consumed; k < issued; k++) {
        tc::mbar_wait(&myfull[slot], ph, &never, p.err, 0x612u, P0_SPIN_LIMIT);
        if (++slot == nslot) { slot = 0; ph ^= 1u; }
      }
    }
  }
}

typedef void (*V4Kernel)(const GemvParams, const V4Plan);
template <int MT>
V4Kernel v4_kernel_m(bool pair) { return pair ? gemv_q4_v4<MT, true> : gemv_q4_v4<MT, false>; }
V4Kernel v4_kernel_for(uint32_t M, bool pair) {
  switch (M) {
    case 1: return v4_kernel_m<1>(pair);
    case 2: return v4_kernel_m<2>(pair);
    case 3: return v4_kernel_m<3>(pair);
    case 4: return v4_kernel_m<4>(pair);
    case 5: return v4_kernel_m<5>(pair);
    case 6: return v4_kernel_m<6>(pair);
    case 7: return v4_kernel_m<7>(pair);
    default: return v4_kernel_m<8>(pair);
  }
}
size_t v4_smem(uint32_t M, uint32_t G, uint32_t nslot) {
  return (size_t)kV4Warps * nslot * kV4Slot + kV4Warps * kV4MaxSlots * 8 + 32 * 4 + (size_t)G * M * 128 + (size_t)G * M * 4;
}
uint32_t v4_min_records() {
  static const uint32_t v = [] {
    const char *s = getenv("P0MM_V4_MINREC");   // tuning override: fewest records per warp before the grid shrinks
    const long n = s ? strtol(s, nullptr, 10) : 0;
    return n >= 1 && n <= 4096 ? (uint32_t)n : 8u;
  }();
  return v;
}
// The allocation-free entry point's scratch (p0_gemvM_noalloc): counters first, then partial sums. Static device
// storage starts zeroed when the library's module loads; each call still clears the counters it uses.
static __device__ __align__(256) uint8_t g_noalloc_scratch[P0_NOALLOC_SCRATCH_BYTES];
}  // namespace

// The device address of g_noalloc_scratch on the current device. The name is only a host-side stand-in for the
// array, so the address comes from cudaGetSymbolAddress, called once per device (with that device current) and cached.
cudaError_t v4_noalloc_scratch(uint8_t **out) {
  static std::mutex mu;
  static uint8_t *addr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void *ptr = nullptr;
    e = cudaGetSymbolAddress((void **)&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    addr[dev] = (uint8_t *)ptr;
  }
  *out = addr[dev];
  return cudaSuccess;
}

bool v4_plan(const GemvParams &p, uint32_t nsplit, int sms, V4Plan *pl, size_t *scratch_bytes) {
  const uint32_t G = p.K / 32;
  const bool pair = p.epi == P0_EPI_GEGLU;
  if (p.wG < G || G == 0 || (pair && nsplit != 1)) return false;
  if ((uint64_t)G * p.M * 4 > (uint64_t)kV4XUnits * kV4Threads) return false;
  const uint32_t ntile = p.N / 64, Gt = pair ? 2 * G : G, Gs = pair ? Gt : (p.kPer / 32 < G ? p.kPer / 32 : G);
  const uint64_t R = (uint64_t)ntile * Gt;
  if (R == 0 || R > 0x7fffffffull) return false;
  // warps: one per v4_min_records() records, at most 16 per SM, whole CTAs
  uint64_t nw = R / v4_min_records();
  const uint64_t cap = (uint64_t)sms * kV4Warps;
  if (nw > cap) nw = cap;
  nw = nw / kV4Warps * kV4Warps;
  if (nw < (uint64_t)kV4Warps) nw = kV4Warps;
  if (nw > R) return false;   // fewer records than one CTA's warps: v2 handles it
  const uint32_t per = (uint32_t)((R + nw - 1) / nw), stages = (per + 1) / 2 + 2;   // + segment ends
  uint32_t nslot = 0;
  for (uint32_t n = kV4MaxSlots; n >= 2; n--)
    if (v4_smem(p.M, G, n) <= 220u * 1024u) { nslot = n; break; }
  if (!nslot) return false;
  if (nslot > stages) nslot = stages;
  const uint32_t nunit = ntile * nsplit;
  pl->R = (uint32_t)R; pl->G = G; pl->Gt = Gt; pl->Gs = Gs; pl->nsplit = nsplit; pl->ntile = ntile; pl->NW = (uint32_t)nw;
  pl->nslot = nslot;
  pl->cnt = nullptr;
  pl->part = nullptr;
  *scratch_bytes = ((size_t)nunit + nw) * (pair ? 2 : 1) * p.M * 64 * 4;
  return true;
}

size_t v4_counter_bytes(const V4Plan &pl) { return (size_t)pl.ntile * pl.nsplit * 4; }

cudaError_t launch_v4(const GemvParams &p, const V4Plan &pl, cudaStream_t s) {
  V4Kernel k = v4_kernel_for(p.M, pl.Gt != pl.G);
  const size_t smem = v4_smem(p.M, pl.G, pl.nslot);
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return launch_pdl(k, dim3(pl.NW / kV4Warps), dim3(kV4Threads), smem, s, 1, p, pl);
}

}  // namespace p0gemv
