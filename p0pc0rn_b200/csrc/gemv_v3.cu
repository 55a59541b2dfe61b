// gemv_v3.cu -- the bulk-copy fed tensor-core GEMV (see the v3 notes below) and its launcher.
#include <cstdlib>

#include "gemv_common.cuh"

namespace p0gemv {
namespace {

// ================================================================================================================ v3: TMA-fed
// The v2 arithmetic fed by bulk copies, for one k-split (nsplit == 1) and many tiles (the vocabulary head and other
// wide projections). Each of 16 warps owns whole 64-row tiles (units) of its CTA's contiguous share and a private ring of
// shared-memory slots (a slot = two consecutive groups of its tile, 2560 contiguous bytes; geglu: one group of the gate
// tile and the same group of the up tile). Lane 0 keeps the ring full with cp.async.bulk: when the warp has read a slot
// it refills it with the stage nslot ahead. Up to 160 KB of weights are in flight per SM; no warp waits on another.
// Per group the warp fetches each lane's code words with two ldmatrix.x4 (word c of rows g, g+8, ... of 32 rows each)
// and runs v2's arithmetic: code MMAs (A = codes as fp16 subnormals, B = x hi/lo), then acc += s * D + mn * sum(x) in
// f32. Both groups of a slot are loaded before any math and accumulate separately (summed per tile), so their MMA and
// FMA chains interleave.
// For M <= 4 the B operands' 8 columns carry the x-hi parts of tokens 0..3 (columns 0..3) and the x-lo parts (columns
// 4..7): one MMA per k16 instead of two; lanes c = 2, 3 then hold the lo parts, added to lanes c = 0, 1 once per tile.
constexpr int kV3Warps = 16;
constexpr int kV3Threads = 32 * kV3Warps;
constexpr uint32_t kV3Slot = 2560;
constexpr uint32_t kV3MaxSlots = 4;
// G4 (M = 1, whole tiles, no geglu pair): a slot holds four consecutive groups of a tile, each record 1312 bytes after
// the previous one (1280 + 32: the four records' rows then fall in different shared-memory banks)
constexpr uint32_t kG4Rec = 1312;
constexpr uint32_t kG4Slot = 4u * kG4Rec;

// x staging (v2's): B fragments of x * sigma as fp16 hi / lo in the permuted k order, and per (group, token) sum(x) / f
// in f32. Returns f = 2^24 / sigma.
template <int MT>
__device__ float stage_x_v3(const GemvParams &p, uint32_t G, uint4 *xb, float *xsum, float *scratch) {
  constexpr uint32_t T = kV3Threads;
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5, len = G * 32;
  float mx = 0.0f;
  for (uint32_t i = t; i < MT * len; i += T) {
    const uint32_t m = i / len, k = i - m * len;
    mx = fmaxf(mx, fabsf(prologue(p, m, k)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) scratch[warp] = mx;
  __syncthreads();
  mx = scratch[0];
#pragma unroll
  for (int w = 1; w < kV3Warps; w++) mx = fmaxf(mx, scratch[w]);
  int e = 0;
  if (mx > 0.0f && mx < INFINITY) frexpf(mx, &e);
  const float sigma = ldexpf(1.0f, 14 - e), f = ldexpf(1.0f, 10 + e), finv = ldexpf(1.0f, -10 - e);
  const uint32_t units = G * MT * 4, ulim = (units + T - 1) / T * T;
  for (uint32_t u = t; u < ulim; u += T) {
    float part = 0.0f;
    if (u < units) {
      const uint32_t gg = u / (MT * 4), rem = u - gg * (MT * 4), m = rem >> 2, c = rem & 3u;
      const uint32_t kb = gg * 32 + c * 8;
      float v[8], hv[8], lv[8];
#pragma unroll
      for (int i = 0; i < 8; i++) {
        v[i] = prologue(p, m, kb + i);
        part += v[i];
      }
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const float vs = v[i] * sigma * ((i & 1) ? 0.0625f : 1.0f);
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

// SPLIT (calls with fewer tiles than warps, e.g. a column-split head on several GPUs): each tile is cut into S k-parts
// (runs of stages), and the parts are the units dealt to the warps; a warp writes its part's row totals to shared memory
// and, after the CTA's barrier, the warps sum each tile's parts in part order and run the epilogue.
//
// G4: the M = 1 form with one group per lane of a quad. The MMA's 16 k slots hold four groups (the slots of lane c,
// 2c, 2c+1, 2c+8, 2c+9, carry group c's codes, four per MMA), and B's column n holds group n / 2's x (hi for even n,
// lo for odd n) in the slots of that group and zeros elsewhere, so D's columns 2c, 2c+1 are group c's hi and lo sums
// for the lane's two rows: each lane converts only its own group's (s, mn) and scales only its own sums (a quarter of
// the generic form's conversions and FMAs at M = 1, where six of the eight D columns are empty). Eight MMAs per row
// block walk the group's four code words; the row totals are summed over the quad's lanes at the end of the tile.
// At M = 2 (G2) an MMA holds two groups: lanes c = 0, 1 carry group 2p's code words 0-1 and 2-3, lanes 2, 3 group
// 2p + 1's; B's column n is token (n / 2) % 2 of group n / 4 (hi / lo by n's parity). D's columns 2c, 2c+1 are then
// group c / 2's hi and lo sums for token c % 2: a lane converts and scales one group and token per MMA pair (half of
// the generic form's work); per tile, the token's total is the sum of lanes c and c ^ 2.
template <int MT, bool PAIR, bool SPLIT, bool G4 = false>
__global__ void __launch_bounds__(kV3Threads, 1) gemv_q4_v3(const GemvParams p, const uint32_t gx, const uint32_t nslot, const uint32_t S_arg) {
  static_assert(!G4 || ((MT == 1 || MT == 2) && !PAIR && !SPLIT), "G4 is the whole-tile form for M = 1 and 2");
  constexpr uint32_t kSlotB = G4 ? kG4Slot : kV3Slot;
  const uint32_t S = SPLIT ? S_arg : 1u;   // whole tiles fold every part computation away
  constexpr bool PACK = MT <= 4;
  constexpr int NP = PAIR ? 2 : 1;
  extern __shared__ __align__(128) uint8_t smem8[];
  uint8_t *ring = smem8;                                                              // [warp][slot] x 2560 B
  uint64_t *full = reinterpret_cast<uint64_t *>(ring + (size_t)kV3Warps * nslot * kSlotB);
  float *scratch = reinterpret_cast<float *>(full + kV3Warps * kV3MaxSlots);          // 32 floats
  volatile uint32_t *abort_flag = reinterpret_cast<volatile uint32_t *>(scratch + 24);
  uint4 *xb = reinterpret_cast<uint4 *>(scratch + 32);                                // [G][MT][4][2]
  const uint32_t G = p.K / 32;
  float *xsum = reinterpret_cast<float *>(xb + (size_t)G * MT * 8);                   // [G][MT]
  float *pbuf = xsum + (size_t)G * MT;                                                // S > 1: [unit][lane][16] totals
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t g = lane >> 2, c = lane & 3;
  const uint32_t ntile = p.N / 64, spt = G4 ? (G + 3) / 4 : PAIR ? G : (G + 1) / 2;   // stages per tile
  const size_t tile_bytes = (size_t)p.wG * 1280u, pair_off = (size_t)ntile * tile_bytes;
  // CTA b owns the contiguous tiles [b*ntile/gx, (b+1)*ntile/gx) (27 or 28 of the head's 4096 on 148 SMs), dealt to its
  // warps round-robin: every SM gets the same share of the work
  const uint32_t T0 = (uint32_t)((uint64_t)blockIdx.x * ntile / gx), T1 = (uint32_t)((uint64_t)(blockIdx.x + 1u) * ntile / gx);
  // units: (tile, part) for the CTA's tiles, part-minor; part k of a tile runs stages [k*spt/S, (k+1)*spt/S)
  const uint32_t U0 = T0 * S, U1 = T1 * S;
  const uint32_t unit0 = U0 + warp, ustride = kV3Warps;
  const uint32_t nunits = unit0 < U1 ? (U1 - unit0 + ustride - 1) / ustride : 0;
  uint32_t nstage = 0;
  for (uint32_t k = 0; k < nunits; k++) {
    const uint32_t part = (unit0 + k * ustride) % S;
    nstage += (part + 1u) * spt / S - part * spt / S;
  }
  uint8_t *myring = ring + (size_t)warp * nslot * kSlotB;
  uint64_t *myfull = full + warp * kV3MaxSlots;
  if (lane == 0) {
    for (uint32_t i = 0; i < nslot; i++) tc::mbar_init(&myfull[i], 1);
    tc::fence_mbar_init();
  }
  if (threadIdx.x == 0) *abort_flag = 0u;
  __syncwarp();
  // the issue side: next stage ni_s (of the tile) of the warp's unit ni_k, which ends at stage ni_e (lane 0 only)
  uint32_t ni_k = 0, ni_s = 0, ni_e = 0, issued = 0;
  const uint8_t *ni_src = p.W;
  auto unit_begin = [&](uint32_t k) {
    const uint32_t u = unit0 + k * ustride, part = u % S;
    ni_src = p.W + (size_t)(u / S) * tile_bytes;
    ni_s = part * spt / S;
    ni_e = (part + 1u) * spt / S;
  };
  if (nunits) unit_begin(0);
  auto issue_next = [&](uint32_t slot) {
    uint8_t *dst = myring + (size_t)slot * kSlotB;
    if (G4) {
      const uint32_t gs = 4u * ni_s, cnt = G - gs < 4u ? G - gs : 4u;
      tc::mbar_expect_tx(&myfull[slot], cnt * 1280u);
      for (uint32_t i = 0; i < cnt; i++) bulk_g2s(dst + i * kG4Rec, ni_src + (size_t)(gs + i) * 1280u, 1280u, &myfull[slot]);
    } else if (PAIR) {
      tc::mbar_expect_tx(&myfull[slot], 2560u);
      bulk_g2s(dst, ni_src + (size_t)ni_s * 1280u, 1280u, &myfull[slot]);
      bulk_g2s(dst + 1280u, ni_src + pair_off + (size_t)ni_s * 1280u, 1280u, &myfull[slot]);
    } else {
      const uint32_t bytes = 2u * ni_s + 1u < G ? 2560u : 1280u;
      tc::mbar_expect_tx(&myfull[slot], bytes);
      bulk_g2s(dst, ni_src + (size_t)ni_s * 2560u, bytes, &myfull[slot]);
    }
    issued++;
    if (++ni_s == ni_e && ++ni_k < nunits) unit_begin(ni_k);
  };
  // the first copies fly while x is staged (and, when the weights are static, while the call ahead finishes)
  if (!p.overlap) pdl_wait();
  if (lane == 0)
    for (uint32_t j = 0; j < nslot && j < nstage; j++) issue_next(j);
  pdl_trigger();
  if (p.overlap) pdl_wait();
  const float f = stage_x_v3<MT>(p, G, xb, xsum, scratch);

  const uint32_t btok = PACK ? (g & 3u) : g, bsel = PACK ? (g >> 2) : 0u;   // B column of this lane
  const bool tok_ok = btok < MT, xs_lane = !PACK || c < 2;   // PACK: the x-sum term belongs to the hi columns
  const uint32_t ring_s = tc::smem_u32(myring), xb_s = tc::smem_u32(xb), xsum_s = tc::smem_u32(xsum);
  const uint32_t lane_row16 = (uint32_t)lane * 16u, tail_off = 1024u + g * 4u;
  // this lane's addresses for group gg: B fragments at xb_lane + gg * MT * 128, x sums at xs_addr + gg * MT * 4
  const uint32_t xb_lane = xb_s + btok * 128u + c * 32u + bsel * 16u, xs_addr = xsum_s + 2u * c * 4u;
  uint32_t cs = 0, cph = 0, consumed = 0;   // consumed slot and its phase; slots consumed so far
  bool ok = true;
  // ---- epilogue of a tile from its row totals (same contract as v2); PACK: lanes c < 2 hold the tokens
  auto tile_epilogue = [&](const uint32_t tile, const float (&tot)[NP][4][4]) {
    const uint32_t R0 = tile * 64, tk0 = 2u * c, tk1 = 2u * c + 1u;
    if (p.epi == P0_EPI_SOFTCAP) {
      float bv0 = -INFINITY, bv1 = -INFINITY;
      uint32_t bi0 = 0xffffffffu, bi1 = 0xffffffffu;
#pragma unroll
      for (int r = 0; r < 4; r++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const uint32_t n = R0 + 16 * r + g + (i >= 2 ? 8 : 0), m = (i & 1) ? tk1 : tk0;
          const float v = __fmul_rn(p.cap, tanhf(fminf(15.0f, fmaxf(-15.0f, __fdiv_rn(tot[0][r][i], p.cap)))));
          if (m < MT) p.Y[(size_t)m * p.ldm + n] = v;
          const uint32_t rr = n & 63u;
          if (i & 1) { if (v > bv1 || (v == bv1 && rr < bi1)) { bv1 = v; bi1 = rr; } }
          else { if (v > bv0 || (v == bv0 && rr < bi0)) { bv0 = v; bi0 = rr; } }
        }
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
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
#pragma unroll
      for (int r = 0; r < 4; r++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const uint32_t n = R0 + 16 * r + g + (i >= 2 ? 8 : 0), m = (i & 1) ? tk1 : tk0;
          if (m >= MT) continue;
          float v = tot[0][r][i];
          if (PAIR) v = __fmul_rn(gelu_l(v), tot[NP - 1][r][i]);
          p.Y[(size_t)m * p.ldm + n] = v;
        }
    }
  };
  if constexpr (G4 && MT == 2) {
    // ---- G2 main loop (M = 2): per stage, pairs p = 0, 1 of groups; lane (g, c) takes group 4 * st + 2p + c / 2,
    // its code words 2 (c % 2) and 2 (c % 2) + 1, token c % 2; rows 16r + 8j + g of the tile
    const uint32_t half = c >> 1u, tk = c & 1u, wofs = 8u * (c & 1u);   // word pair of the lane: bytes 8 (c % 2)
    // B: this lane supplies column g for its own slots, nonzero when column g's group (g / 4) is the lane's (c / 2)
    const bool bcol = half == (g >> 2u);
    const uint32_t btk = (g >> 1u) & 1u, blo = g & 1u;
    for (uint32_t ui = 0; ui < nunits && ok; ui++) {
      const uint32_t tile = unit0 + ui * ustride;
      float acc[4][2];
#pragma unroll
      for (int r = 0; r < 4; r++) acc[r][0] = acc[r][1] = 0.0f;
      for (uint32_t st = 0; st < spt; st++) {
        const bool got = tc::mbar_wait(&myfull[cs], cph, abort_flag, p.err, 0x511u, P0_SPIN_LIMIT);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        consumed++;
        uint2 cw[2][4][2];
        uint32_t tl[2][4][2];
        uint4 bx[2][2];
        float xs[2] = {0.0f, 0.0f};
        bool live[2];
#pragma unroll
        for (int q = 0; q < 2; q++) {
          const uint32_t ri = 2u * q + half, gg = 4u * st + ri;
          live[q] = gg < G;
          const uint32_t rec = ring_s + cs * kSlotB + ri * kG4Rec;
#pragma unroll
          for (int r = 0; r < 4; r++)
#pragma unroll
            for (int j = 0; j < 2; j++) {
              const uint32_t row = 16u * r + 8u * j + g;
              asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(cw[q][r][j].x), "=r"(cw[q][r][j].y) : "r"(rec + row * 16u + wofs));
              tl[q][r][j] = lds32(rec + 1024u + row * 4u);
            }
          bx[q][0] = bx[q][1] = make_uint4(0, 0, 0, 0);
          if (live[q]) {
            xs[q] = __uint_as_float(lds32(xsum_s + (gg * 2u + tk) * 4u));
            const uint32_t gb = 4u * st + 2u * q + (g >> 2u);   // column g's group
            if (bcol) {
#pragma unroll
              for (int w = 0; w < 2; w++) bx[q][w] = lds128(xb_s + ((gb * 8u + btk * 4u + 2u * (c & 1u) + w) * 2u + blo) * 16u);
            }
          }
        }
        __syncwarp();
        if (lane == 0 && issued < nstage) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issue_next(cs);
        }
        if (++cs == nslot) { cs = 0; cph ^= 1u; }
#pragma unroll
        for (int q = 0; q < 2; q++)
#pragma unroll
          for (int r = 0; r < 4; r++) {
            float d0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, d1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const uint32_t wa[2] = {cw[q][r][0].x, cw[q][r][0].y}, wb[2] = {cw[q][r][1].x, cw[q][r][1].y};
#pragma unroll
            for (int w = 0; w < 2; w++) {
              const uint32_t a = wa[w], b = wb[w];
              const uint32_t as = __umulhi(a, 1u << 24), bs = __umulhi(b, 1u << 24);
              const uint32_t A0[4] = {a & 0x000F000Fu, b & 0x000F000Fu, a & 0x00F000F0u, b & 0x00F000F0u};
              const uint32_t A1[4] = {as & 0x000F000Fu, bs & 0x000F000Fu, as & 0x00F000F0u, bs & 0x00F000F0u};
              float(&dd)[4] = w ? d1 : d0;
              mma16816(dd, A0, bx[q][w].x, bx[q][w].y);
              mma16816(dd, A1, bx[q][w].z, bx[q][w].w);
            }
            if (live[q]) {
              const float vg = __fadd_rn(__fadd_rn(d0[0], d1[0]), __fadd_rn(d0[1], d1[1]));
              const float vg8 = __fadd_rn(__fadd_rn(d0[2], d1[2]), __fadd_rn(d0[3], d1[3]));
              const __half2 h0 = *reinterpret_cast<const __half2 *>(&tl[q][r][0]), h1 = *reinterpret_cast<const __half2 *>(&tl[q][r][1]);
              uint64_t av = pk2(acc[r][0], acc[r][1]);
              av = ffma2(pk2(__high2float(h0), __high2float(h1)), pk2(xs[q], xs[q]), av);
              av = ffma2(pk2(__low2float(h0), __low2float(h1)), pk2(vg, vg8), av);
              upk2(av, acc[r][0], acc[r][1]);
            }
          }
      }
      if (!ok) break;
      // token totals: lanes c and c ^ 2 hold the two halves of the groups; lane c = 0 takes token 0 and token 1 (lane 1)
      float tot[NP][4][4];
#pragma unroll
      for (int r = 0; r < 4; r++)
#pragma unroll
        for (int j = 0; j < 2; j++) {
          float v = acc[r][j];
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          const float o = __shfl_xor_sync(0xffffffffu, v, 1);
          tot[0][r][2 * j] = v * f;
          tot[0][r][2 * j + 1] = o * f;
        }
      tile_epilogue(tile, tot);
    }
  } else if constexpr (G4) {
    // ---- G4 main loop (M = 1): lane (g, c) takes group 4 * st + c of every stage, rows 16r + 8j + g of the tile
    const uint32_t rec_off = c * kG4Rec;
    const bool bcol = c == (g >> 1u);      // this lane's B column n = g belongs to its own group: x (hi / lo), else 0
    const uint32_t blo = g & 1u;
    for (uint32_t ui = 0; ui < nunits && ok; ui++) {
      const uint32_t tile = unit0 + ui * ustride;
      float acc[4][2];
#pragma unroll
      for (int r = 0; r < 4; r++) acc[r][0] = acc[r][1] = 0.0f;
      for (uint32_t st = 0; st < spt; st++) {
        const bool got = tc::mbar_wait(&myfull[cs], cph, abort_flag, p.err, 0x511u, P0_SPIN_LIMIT);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        consumed++;
        const uint32_t gg = 4u * st + c;
        const bool live = gg < G;          // the tile's last stage may hold fewer than four groups
        const uint32_t rec = ring_s + cs * kSlotB + rec_off;
        uint4 cw[4][2];
        uint32_t tl[4][2];
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
          for (int j = 0; j < 2; j++) {
            const uint32_t row = 16u * r + 8u * j + g;
            cw[r][j] = lds128(rec + row * 16u);
            tl[r][j] = lds32(rec + 1024u + row * 4u);
          }
        uint4 bx[4];
        float xs = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; w++) bx[w] = make_uint4(0, 0, 0, 0);
        if (live) {
          xs = __uint_as_float(lds32(xsum_s + gg * 4u));
          if (bcol) {
#pragma unroll
            for (int w = 0; w < 4; w++) bx[w] = lds128(xb_s + ((gg * 4u + w) * 2u + blo) * 16u);
          }
        }
        // every lane has read the slot: lane 0 refills it with the stage nslot ahead
        __syncwarp();
        if (lane == 0 && issued < nstage) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issue_next(cs);
        }
        if (++cs == nslot) { cs = 0; cph ^= 1u; }
#pragma unroll
        for (int r = 0; r < 4; r++) {
          float d0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, d1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          const uint32_t wa[4] = {cw[r][0].x, cw[r][0].y, cw[r][0].z, cw[r][0].w};
          const uint32_t wb[4] = {cw[r][1].x, cw[r][1].y, cw[r][1].z, cw[r][1].w};
#pragma unroll
          for (int w = 0; w < 4; w++) {
            const uint32_t a = wa[w], b = wb[w];
            const uint32_t as = __umulhi(a, 1u << 24), bs = __umulhi(b, 1u << 24);   // >> 8 on the multiplier pipe
            const uint32_t A0[4] = {a & 0x000F000Fu, b & 0x000F000Fu, a & 0x00F000F0u, b & 0x00F000F0u};
            const uint32_t A1[4] = {as & 0x000F000Fu, bs & 0x000F000Fu, as & 0x00F000F0u, bs & 0x00F000F0u};
            if (w & 1) {
              mma16816(d1, A0, bx[w].x, bx[w].y);
              mma16816(d1, A1, bx[w].z, bx[w].w);
            } else {
              mma16816(d0, A0, bx[w].x, bx[w].y);
              mma16816(d0, A1, bx[w].z, bx[w].w);
            }
          }
          if (live) {
            // D columns 2c, 2c+1: this group's hi and lo sums for rows g (d[0], d[1]) and g + 8 (d[2], d[3])
            const float vg = __fadd_rn(__fadd_rn(d0[0], d1[0]), __fadd_rn(d0[1], d1[1]));
            const float vg8 = __fadd_rn(__fadd_rn(d0[2], d1[2]), __fadd_rn(d0[3], d1[3]));
            const __half2 h0 = *reinterpret_cast<const __half2 *>(&tl[r][0]), h1 = *reinterpret_cast<const __half2 *>(&tl[r][1]);
            uint64_t av = pk2(acc[r][0], acc[r][1]);
            av = ffma2(pk2(__high2float(h0), __high2float(h1)), pk2(xs, xs), av);
            av = ffma2(pk2(__low2float(h0), __low2float(h1)), pk2(vg, vg8), av);
            upk2(av, acc[r][0], acc[r][1]);
          }
        }
      }
      if (!ok) break;
      // row totals: the quad's four groups (lanes c), then f; the epilogue reads token 0 from lanes c = 0
      float tot[NP][4][4];
#pragma unroll
      for (int r = 0; r < 4; r++)
#pragma unroll
        for (int j = 0; j < 2; j++) {
          float v = acc[r][j];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          tot[0][r][2 * j] = v * f;
          tot[0][r][2 * j + 1] = 0.0f;
        }
      tile_epilogue(tile, tot);
    }
  } else {
    for (uint32_t ui = 0; ui < nunits && ok; ui++) {
      const uint32_t u = unit0 + ui * ustride, tile = u / S, part = u % S;
      const uint32_t st0 = part * spt / S, st1 = (part + 1u) * spt / S;
      float acc[2][NP][4][4];   // [group parity] -> independent FMA chains for the two groups of a slot
  #pragma unroll
      for (int h = 0; h < 2; h++)
  #pragma unroll
        for (int a = 0; a < NP; a++)
  #pragma unroll
          for (int r = 0; r < 4; r++)
  #pragma unroll
            for (int i = 0; i < 4; i++) acc[h][a][r][i] = 0.0f;
      for (uint32_t st = st0; st < st1; st++) {
        const bool got = tc::mbar_wait(&myfull[cs], cph, abort_flag, p.err, 0x511u, P0_SPIN_LIMIT);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        consumed++;
        const uint32_t sl = ring_s + cs * kV3Slot;
        const bool two = PAIR || 2u * st + 1u < G;   // PAIR: gate and up records of one group; else two groups
        const uint32_t gg0 = PAIR ? st : 2u * st, gg1 = PAIR ? st : gg0 + 1u;
        // all shared loads of the slot first
        Rec q0, q1;
        rec_load(q0, sl, lane_row16, tail_off);
        if (two) rec_load(q1, sl + 1280u, lane_row16, tail_off);
        uint4 bh0 = make_uint4(0, 0, 0, 0), bl0 = bh0, bh1 = bh0, bl1 = bh0;
        float x00 = 0.0f, x01 = 0.0f, x10 = 0.0f, x11 = 0.0f;
        if (tok_ok) {
          bh0 = lds128(xb_lane + gg0 * MT * 128u);
          if (!PACK) bl0 = lds128(xb_lane + gg0 * MT * 128u + 16u);
          if (!PAIR && two) {
            bh1 = lds128(xb_lane + gg1 * MT * 128u);
            if (!PACK) bl1 = lds128(xb_lane + gg1 * MT * 128u + 16u);
          }
        }
        if (xs_lane) {
          if (2 * c < MT) { x00 = __uint_as_float(lds32(xs_addr + gg0 * MT * 4u)); x10 = __uint_as_float(lds32(xs_addr + gg1 * MT * 4u)); }
          if (2 * c + 1 < MT) { x01 = __uint_as_float(lds32(xs_addr + gg0 * MT * 4u + 4u)); x11 = __uint_as_float(lds32(xs_addr + gg1 * MT * 4u + 4u)); }
        }
        // every lane has read the slot: lane 0 refills it with the stage nslot ahead (generic reads before the
        // async-proxy write: warp sync, then a proxy fence); the math below uses registers only
        __syncwarp();
        if (lane == 0 && issued < nstage) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issue_next(cs);
        }
        if (++cs == nslot) { cs = 0; cph ^= 1u; }
        if (PAIR) {
          rec_math<MT, PACK>(acc[0][0], q0, bh0, bl0, x00, x01);
          rec_math<MT, PACK>(acc[1][NP - 1], q1, bh0, bl0, x00, x01);
        } else {
          rec_math<MT, PACK>(acc[0][0], q0, bh0, bl0, x00, x01);
          if (two) rec_math<MT, PACK>(acc[1][0], q1, bh1, bl1, x10, x11);
        }
      }
      if (!ok) break;
      // row totals: f * (the two parities' sums); PACK: add the x-lo lanes c = 2, 3
      float tot[NP][4][4];
  #pragma unroll
      for (int a = 0; a < NP; a++)
  #pragma unroll
        for (int r = 0; r < 4; r++)
  #pragma unroll
          for (int i = 0; i < 4; i++) {
            float v = PAIR ? acc[a][a][r][i] * f : (acc[0][a][r][i] + acc[1][a][r][i]) * f;
            if (PACK) v += __shfl_xor_sync(0xffffffffu, v, 2);
            tot[a][r][i] = v;
          }
      if (!SPLIT) {
        tile_epilogue(tile, tot);
      } else {
        float *pb = pbuf + ((size_t)(u - U0) * 32u + lane) * 16u;
  #pragma unroll
        for (int r = 0; r < 4; r++)
  #pragma unroll
          for (int i = 0; i < 4; i++) pb[r * 4 + i] = tot[0][r][i];
      }
    }
  }
  // copies this warp issued but did not consume (only after a failed wait) land before the CTA exits (bounded)
  if (lane == 0 && !ok) {
    volatile uint32_t never = 0;
    uint32_t slot = cs, ph = cph;
    for (uint32_t k = consumed; k < issued; k++) {
      tc::mbar_wait(&myfull[slot], ph, &never, p.err, 0x512u, P0_SPIN_LIMIT);
      if (++slot == nslot) { slot = 0; ph ^= 1u; }
    }
  }
  if (SPLIT) {
    // every part is in shared memory: each tile's parts summed in part order, then its epilogue (warps take tiles
    // round-robin). After a failed wait the results are void (the error word reports it), the stores still bounded.
    __syncthreads();
    for (uint32_t tile = T0 + warp; tile < T1; tile += kV3Warps) {
      float tot[NP][4][4];
#pragma unroll
      for (int r = 0; r < 4; r++)
#pragma unroll
        for (int i = 0; i < 4; i++) tot[0][r][i] = 0.0f;
      for (uint32_t k = 0; k < S; k++) {
        const float *pb = pbuf + ((size_t)((tile - T0) * S + k) * 32u + lane) * 16u;
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
          for (int i = 0; i < 4; i++) tot[0][r][i] += pb[r * 4 + i];
      }
      tile_epilogue(tile, tot);
    }
  }
}

typedef void (*V3Kernel)(const GemvParams, const uint32_t, const uint32_t, const uint32_t);
V3Kernel v3_kernel_g4(uint32_t M) { return M == 1 ? gemv_q4_v3<1, false, false, true> : gemv_q4_v3<2, false, false, true>; }
template <int MT>
V3Kernel v3_kernel_m(bool pair, bool split) {
  return pair ? gemv_q4_v3<MT, true, false> : split ? gemv_q4_v3<MT, false, true> : gemv_q4_v3<MT, false, false>;
}
V3Kernel v3_kernel_for(uint32_t M, bool pair, bool split) {
  switch (M) {
    case 1: return v3_kernel_m<1>(pair, split);
    case 2: return v3_kernel_m<2>(pair, split);
    case 3: return v3_kernel_m<3>(pair, split);
    case 4: return v3_kernel_m<4>(pair, split);
    case 5: return v3_kernel_m<5>(pair, split);
    case 6: return v3_kernel_m<6>(pair, split);
    case 7: return v3_kernel_m<7>(pair, split);
    default: return v3_kernel_m<8>(pair, split);
  }
}
size_t v3_smem(uint32_t M, uint32_t G, uint32_t nslot, uint32_t slotb = kV3Slot) {
  return (size_t)kV3Warps * nslot * slotb + kV3Warps * kV3MaxSlots * 8 + 32 * 4 + (size_t)G * M * 128 + (size_t)G * M * 4;
}
uint32_t v3_slots(uint32_t M, uint32_t G) {
  for (uint32_t n = kV3MaxSlots; n >= 2; n--)
    if (v3_smem(M, G, n) <= 220u * 1024u) return n;
  return 0;
}
}  // namespace

// whole tiles per warp: when every warp of the grid gets one, or, for M <= 4, from 13 tiles per SM (measured on B200 at
// 2048 tiles, the 2-rank column-split head, whole tiles against k-parts: 37.8 / 44.7 / 45.2 against 48.8 / 46.7 / 46.4 us
// at M = 1 / 2 / 4, M = 8 even (56.4 against 55.8); at 1024 tiles the k-parts lead by 10 us from M = 2 on)
bool v3_whole(uint32_t M, uint32_t ntile, int sms) {
  return ntile >= (uint32_t)sms * kV3Warps || (M <= 4u && ntile >= (uint32_t)sms * 13u);
}
// the parts per tile: 1 for whole tiles (or for geglu pairs); else enough parts for about 27 units per CTA (whole-tile
// v3 runs the head at 27-28 tiles per CTA), at most 8 and at most a part per stage
uint32_t v3_parts(uint32_t K, uint32_t ntile, int sms, bool pair, uint32_t M) {
  const uint32_t spt = (K / 32 + 1) / 2;
  // tuning override, read on every call: P0MM_V3_PARTS=n (1..8) cuts every non-geglu v3 call's tiles into n parts
  const char *ov = getenv("P0MM_V3_PARTS");
  const long nov = ov ? strtol(ov, nullptr, 10) : 0;
  if (!pair && nov >= 1 && nov <= 8) return (uint32_t)nov < spt ? (uint32_t)nov : spt;
  if (pair || v3_whole(M, ntile, sms)) return 1;
  uint32_t S = ((uint32_t)sms * 27u + ntile - 1) / ntile;
  if (S > 8) S = 8;
  if (S > spt) S = spt;
  return S < 1 ? 1 : S;
}
size_t v3_pbuf(uint32_t ntile, int sms, uint32_t S) {
  if (S == 1) return 0;
  const uint32_t gx = ntile < (uint32_t)sms ? ntile : (uint32_t)sms;
  return (size_t)((ntile + gx - 1) / gx) * S * 32u * 16u * 4u;
}
uint32_t v3_slots_with(uint32_t M, uint32_t G, size_t extra) {
  for (uint32_t n = kV3MaxSlots; n >= 2; n--)
    if (v3_smem(M, G, n) + extra <= 220u * 1024u) return n;
  return 0;
}

// v3: one split and a ring of >= 2 slots; whole tiles per warp (v3_whole), else (not geglu, at least one tile per
// SM) tiles cut into k-parts
bool v3_fits(uint32_t M, uint32_t K, uint32_t nsplit, uint32_t ntile, int sms) {
  return nsplit == 1 && v3_slots(M, K / 32) >= 2 && v3_whole(M, ntile, sms);
}
bool v3_split_fits(uint32_t M, uint32_t K, uint32_t nsplit, uint32_t ntile, int sms, bool pair) {
  if (nsplit != 1 || pair || ntile < (uint32_t)sms || v3_whole(M, ntile, sms)) return false;
  const uint32_t S = v3_parts(K, ntile, sms, pair, M);
  return S > 1 && v3_slots_with(M, K / 32, v3_pbuf(ntile, sms, S)) >= 2;
}
cudaError_t launch_v3(const GemvParams &p, int sms, cudaStream_t s) {
  const bool pair = p.epi == P0_EPI_GEGLU;
  const uint32_t G = p.K / 32, ntile = p.N / 64;
  uint32_t S = v3_parts(p.K, ntile, sms, pair, p.M);
  if (S > 1 && v3_slots_with(p.M, G, v3_pbuf(ntile, sms, S)) < 2) S = 1;   // the parts' totals do not fit beside a ring
  V3Kernel k = v3_kernel_for(p.M, pair, S > 1);
  const size_t pb = v3_pbuf(ntile, sms, S);
  uint32_t nslot = v3_slots_with(p.M, G, pb);
  size_t smem = v3_smem(p.M, G, nslot) + pb;
  // M = 1 / 2 whole tiles: the grouped forms (two 4-group slots per warp, the same bytes in flight) when they fit;
  // P0MM_V3_G4=0, a tuning override read on every call, keeps the generic form
  const char *g4v = getenv("P0MM_V3_G4");
  if (p.M <= 2 && !pair && S == 1 && !(g4v && g4v[0] == '0') && v3_smem(p.M, G, 2, kG4Slot) <= 220u * 1024u) {
    k = v3_kernel_g4(p.M);
    nslot = 2;
    smem = v3_smem(p.M, G, 2, kG4Slot);
  }
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const uint32_t need = S == 1 ? (ntile + kV3Warps - 1) / kV3Warps : ntile;
  uint32_t gx = (uint32_t)sms;
  if (gx > need) gx = need;
  return launch_pdl(k, dim3(gx), dim3(kV3Threads), smem, s, 1, p, gx, nslot, S);
}


}  // namespace p0gemv
