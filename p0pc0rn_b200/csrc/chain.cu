// chain.cu -- recorded GEMV chains: the decode step's sequence of gemv / gemvM calls run as one persistent kernel.
//
// The reference records one decode token's ~500 dispatches into one command buffer and replays it (DecodeRunner,
// engine/llm/drunner.js:1-8, begin :36): the ops keep calling gemv / gemvM as always while g.runner points at the
// recorder. p0_chain_begin / p0_chain_end do the same here: between them every p0_gemv / p0_gemvM call on the context is
// checked exactly as it would be, and kept instead of launched. p0_chain_run then enqueues the whole sequence.
//
// On B200 a decode step's GEMVs are 2.6-21 MB each: alone, each pays a launch, an HBM round trip before its first
// bytes arrive and a reduction tail, and the chain of 105 calls of config 5 ran at a quarter of HBM bandwidth. The
// chain kernel removes those gaps. It is cooperative (one CTA of 16 warps per SM, all resident) and walks the calls in
// order; between a call and one that reads what the earlier calls of the kernel wrote (or writes what they read or
// wrote) it waits at a grid barrier. Every warp keeps a ring of bulk copies of its own next weight records, and that
// sequence runs on across calls and barriers: while a CTA waits for the call ahead to finish, the weights of its share
// of the next calls are already arriving (weights are constant while a chain runs: p0mm.h says so).
//
// Work split of a call: its output units (a unit = one 64-row tile x k-split, or a geglu gate tile with its up tile)
// are dealt to the CTAs round-robin, continuing across calls where the previous call's units ended, so that every call
// starts on different SMs. A CTA computes each of its units whole: the unit's records are split evenly over its 16
// warps, whose per-row partials are summed in shared memory in warp order, and it writes the outputs itself. No unit
// is shared between CTAs, so a call's critical path after its barrier is one read of x, the unit's records (already in
// the rings), one CTA reduction and the stores. The per-record arithmetic is the library's tensor-core GEMV
// (gemv_common.cuh: exact fp16-subnormal codes, x as fp16 hi + lo, acc += s * D + mn * sum(x)).
#include <algorithm>
#include <vector>

#include "gemv_common.cuh"

namespace p0gemv {

constexpr int kCW = 16;                 // warps per CTA
constexpr int kCT = 32 * kCW;
constexpr uint32_t kCMaxSlots = 8;      // ring slots (one 1280-byte record each) per warp
constexpr uint32_t kCMaxGroups = 64;    // x groups one segment stages (K per split <= 2048)
// bounded waits: a record copy lands within microseconds and a barrier within the call ahead's time, so these limits
// (polls, each at most a short suspend) only end a chain that has already failed
constexpr uint32_t kCSpin = 1u << 20;

// one recorded call as the chain kernel sees it
// Index math is 32-bit throughout: a call the chain kernel takes has at most 4 x SMs units of at most 128 records, so
// R * NB < 2^32.
struct ChainCall {
  GemvParams p;
  uint32_t nsplit, Gs, Glast, units, pair, barrier;
  uint32_t ubase;      // the CTA that takes unit 0 (units u go to CTA (ubase + u) % NB)
  uint32_t pad;
};

struct ChainRun {
  const ChainCall *calls;
  uint32_t ncalls, nslot;
  uint32_t *bar;       // grid barrier arrivals (zeroed before each launch)
  uint32_t *gabort;    // set by a CTA that gave up a wait: every CTA stops at its next wait
  uint32_t *err;
};

__device__ __forceinline__ uint32_t unit_len(const ChainCall &cc, uint32_t u) {
  if (cc.pair) return 2u * cc.Gs;
  return u / cc.p.ntile == cc.nsplit - 1u ? cc.Glast : cc.Gs;
}
// this CTA's first unit of a call (>= units: none), its units step by NB
__device__ __forceinline__ uint32_t first_unit(const ChainCall &cc, uint32_t b, uint32_t NB) { return (b + NB - cc.ubase % NB) % NB; }
// the record j of unit u: its address, and the x group it multiplies
__device__ __forceinline__ const uint8_t *rec_addr(const ChainCall &cc, uint32_t u, uint32_t j) {
  uint32_t tile, grp;
  if (cc.pair) {
    const bool up = j >= cc.Gs;
    tile = u + (up ? cc.p.ntile : 0u);
    grp = up ? j - cc.Gs : j;
  } else {
    const uint32_t s = u / cc.p.ntile;
    tile = u - s * cc.p.ntile;
    grp = s * cc.Gs + j;
  }
  return cc.p.W + ((size_t)tile * cc.p.wG + grp) * 1280u;
}
__device__ __forceinline__ uint32_t rec_xgroup(const ChainCall &cc, uint32_t u, uint32_t j) {
  if (cc.pair) return j >= cc.Gs ? j - cc.Gs : j;
  return (u / cc.p.ntile) * cc.Gs + j;
}

// One warp's record sequence over the whole chain: for every call, every unit of its CTA, the warp's even share of
// the unit's records. The producer (lane 0) walks it ahead of the consumer to keep the ring full.
struct WarpSeq {
  uint32_t ci, u, j, jend;   // call, unit, next record (unit-relative), end of the share
  bool done;
};
__device__ __forceinline__ void seq_share(const ChainCall &cc, uint32_t u, uint32_t w, uint32_t &ja, uint32_t &jb) {
  const uint32_t len = unit_len(cc, u);
  ja = w * len / kCW;
  jb = (w + 1u) * len / kCW;
}
// moves to the first record at or after the current position (the current call's unit u, or later); false when the
// chain is done
__device__ bool seq_settle(const ChainRun &run, WarpSeq &q, uint32_t w) {
  while (!q.done && q.j >= q.jend) {
    const ChainCall &cc = run.calls[q.ci];
    if (q.u + gridDim.x < cc.units) {   // the CTA's next unit of this call
      q.u += gridDim.x;
      seq_share(cc, q.u, w, q.j, q.jend);
      continue;
    }
    for (;;) {                           // the next call with a unit for this CTA
      if (++q.ci >= run.ncalls) { q.done = true; return false; }
      const ChainCall &nc = run.calls[q.ci];
      q.u = first_unit(nc, blockIdx.x, gridDim.x);
      if (q.u < nc.units) {
        seq_share(nc, q.u, w, q.j, q.jend);
        break;
      }
    }
  }
  return !q.done;
}

// x staging of a segment (the library's tensor-core layout): B fragments of x * sigma as fp16 hi / lo in the permuted
// k order for groups [xg0, xg0 + ng) and tokens m < MT, plus per (group, token) sum(x) / f. x, stat, norm and ev are
// read through L2 (ld.cg): calls earlier in the kernel may have written them. Returns f = 2^24 / sigma.
__device__ __forceinline__ float ldcg_f(const float *p) { return __ldcg(p); }
__device__ __forceinline__ float chain_prologue(const GemvParams &p, uint32_t m, uint32_t k) {
  if (p.pro == P0_PRO_RAW) return ldcg_f(p.X + m * p.ldx + p.rowB + k);
  if (p.pro == P0_PRO_RMS)
    return __fmul_rn(__fmul_rn(ldcg_f(p.X + m * p.ldx + p.rowB + k), ldcg_f(p.ST + p.statOff + m * p.statLd)), ldcg_f(p.NW + p.nOff + k));
  float s = 0.0f;
  for (uint32_t j = 0; j < p.nsrc; j++) s = __fadd_rn(s, ldcg_f(p.X + j * p.ldp + m * p.ldx + k));
  if (p.pro == P0_PRO_SUM) return s;
  return __fmul_rn(gelu_l(s), ldcg_f(p.EV + p.evOff + m * p.evLd + k));
}
template <int MT>
__device__ float stage_x_seg(const GemvParams &p, uint32_t xg0, uint32_t ng, uint4 *xb, float *xsum, float *scratch) {
  // one read of x: each thread loads its (group, token, quarter) units' 8 values into registers (at most 4 units:
  // ng * MT * 4 <= 64 * 8 * 4 = 4 * 512), takes the CTA's max |x| from them, then converts them
  constexpr uint32_t kUPT = (kCMaxGroups * MT * 4 + kCT - 1) / kCT;
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5, k0 = xg0 * 32;
  const uint32_t units = ng * MT * 4;
  float v[kUPT][8];
  float mx = 0.0f;
#pragma unroll
  for (uint32_t q = 0; q < kUPT; q++) {
    const uint32_t u = t + q * kCT;
    if (u < units) {
      const uint32_t gg = u / (MT * 4), rem = u - gg * (MT * 4), m = rem >> 2, c = rem & 3u;
      const uint32_t kb = k0 + gg * 32 + c * 8;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        v[q][i] = chain_prologue(p, m, kb + i);
        mx = fmaxf(mx, fabsf(v[q][i]));
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; i++) v[q][i] = 0.0f;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) scratch[warp] = mx;
  __syncthreads();
  mx = scratch[0];
#pragma unroll
  for (int w = 1; w < kCW; w++) mx = fmaxf(mx, scratch[w]);
  int e = 0;
  if (mx > 0.0f && mx < INFINITY) frexpf(mx, &e);
  const float sigma = ldexpf(1.0f, 14 - e), f = ldexpf(1.0f, 10 + e), finv = ldexpf(1.0f, -10 - e);
#pragma unroll
  for (uint32_t q = 0; q < kUPT; q++) {
    const uint32_t u = t + q * kCT;
    if (q * kCT >= units) break;   // CTA-uniform: every lane of a warp takes the shuffles below together
    float part = 0.0f, hv[8], lv[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      part += v[q][i];
      const float vs = v[q][i] * sigma * ((i & 1) ? 0.0625f : 1.0f);
      const float h = __half2float(__float2half_rn(vs));
      hv[i] = h;
      lv[i] = vs - h;
    }
    if (u < units) {
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

// Release / acquire at GPU scope by one thread: the CTA barrier ahead of the release orders every thread's writes before
// it, the one after the acquire orders every thread's reads after it (fence.acq_rel, lighter than a __threadfence's
// sequentially consistent fence, which every thread would otherwise pay)
__device__ __forceinline__ void fence_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// grid barrier number k (1, 2, ...) of this launch: every CTA arrives once; bounded wait; false when the chain gives up
__device__ bool grid_barrier(const ChainRun &run, uint32_t k, volatile uint32_t *abort_flag) {
  __syncthreads();
  if (threadIdx.x == 0 && !*abort_flag) {
    fence_gpu();
    atomicAdd(run.bar, 1u);
    const uint32_t target = k * gridDim.x;
    for (uint32_t i = 0;; i++) {
      uint32_t v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(run.bar) : "memory");
      if (v >= target) break;
      if (*(volatile uint32_t *)run.gabort) { *abort_flag = 1u; break; }
      if (i >= kCSpin) {
        atomicOr(run.err, 0x7c1u);
        atomicExch(run.gabort, 1u);
        *abort_flag = 1u;
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  return *abort_flag == 0u;
}

// the epilogue of unit u from its final totals tot[h][m][row] (shared memory, f32): the contract of gemv / gemvM
template <int MT>
__device__ void unit_epilogue(const ChainCall &cc, uint32_t u, const float *tot, float *vals) {
  const GemvParams &p = cc.p;
  const uint32_t t = threadIdx.x;
  const uint32_t s = cc.pair ? 0u : u / p.ntile, tile = cc.pair ? u : u - s * p.ntile;
  if (t < MT * 64u) {
    const uint32_t m = t / 64u, r = t % 64u, n = tile * 64u + r;
    const float v0 = tot[m * 64u + r];
    if (p.epi == P0_EPI_STORE) {
      p.Y[(size_t)s * p.ldy + (size_t)m * p.ldm + n] = v0;
    } else if (p.epi == P0_EPI_GEGLU) {
      p.Y[(size_t)m * p.ldm + n] = __fmul_rn(gelu_l(v0), tot[(MT + m) * 64u + r]);
    } else {
      const float v = __fmul_rn(p.cap, tanhf(fminf(15.0f, fmaxf(-15.0f, __fdiv_rn(v0, p.cap)))));
      p.Y[(size_t)m * p.ldm + n] = v;
      vals[m * 64u + r] = v;
    }
  }
  if (p.epi == P0_EPI_SOFTCAP) {
    __syncthreads();
    const uint32_t warp = t >> 5, lane = t & 31u;
    if (warp < (uint32_t)MT) {
      const uint32_t m = warp;
      const float v0 = vals[m * 64u + lane], v1 = vals[m * 64u + lane + 32u];
      float bv = v0;
      uint32_t bi = lane;
      if (v1 > bv) { bv = v1; bi = lane + 32u; }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) {
        const size_t o = ((size_t)m * p.ntile + tile) * 2;
        p.MX[o] = bv;
        p.MX[o + 1] = __uint_as_float(tile * 64u + bi);
      }
    }
  }
}

template <int MT>
__global__ void __launch_bounds__(kCT, 1) gemv_chain(const ChainRun run) {
  constexpr bool PACK = MT <= 4;
  extern __shared__ __align__(128) uint8_t smem8[];
  const uint32_t nslot = run.nslot;
  uint8_t *ring = smem8;                                                                  // [warp][slot] x 1280 B
  uint64_t *full = reinterpret_cast<uint64_t *>(ring + (size_t)kCW * nslot * 1280u);       // [warp][kCMaxSlots]
  float *scratch = reinterpret_cast<float *>(full + kCW * kCMaxSlots);                    // 32 floats
  volatile uint32_t *abort_flag = reinterpret_cast<volatile uint32_t *>(scratch + 24);
  volatile uint32_t *last_flag = reinterpret_cast<volatile uint32_t *>(scratch + 25);
  float *ctot = scratch + 32;                                                             // [2][MT][64]
  float *vals = ctot + 2 * MT * 64;                                                       // [MT][64]
  uint8_t *xarea = reinterpret_cast<uint8_t *>(vals + MT * 64);
  uint4 *xb = reinterpret_cast<uint4 *>(xarea);                                           // [64][MT][4][2]
  float *xsum = reinterpret_cast<float *>(xb + (size_t)kCMaxGroups * MT * 8);             // [64][MT]
  float *wpart = reinterpret_cast<float *>(xarea);                                        // [warp][2][MT][64] (after the math)
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t g = lane >> 2, c = lane & 3u;
  uint8_t *myring = ring + (size_t)warp * nslot * 1280u;
  uint64_t *myfull = full + warp * kCMaxSlots;
  if (lane == 0) {
    for (uint32_t i = 0; i < nslot; i++) tc::mbar_init(&myfull[i], 1);
    tc::fence_mbar_init();
  }
  if (threadIdx.x == 0) { *abort_flag = 0u; *last_flag = 0u; }
  __syncthreads();

  // ---- the producer: lane 0 keeps the ring full with the warp's next records, across calls and barriers
  WarpSeq pq{};
  pq.ci = 0;
  pq.done = run.ncalls == 0;
  if (!pq.done) {
    pq.u = first_unit(run.calls[0], blockIdx.x, gridDim.x);
    if (pq.u < run.calls[0].units) seq_share(run.calls[0], pq.u, warp, pq.j, pq.jend);
    else { pq.u = 0xffffffffu - gridDim.x; pq.j = pq.jend = 0; }   // seq_settle moves on to the next call
  }
  uint32_t issued = 0;
  auto issue_next = [&](uint32_t slot) {
    if (!seq_settle(run, pq, warp)) return;
    const uint8_t *src = rec_addr(run.calls[pq.ci], pq.u, pq.j);
    pq.j++;
    tc::mbar_expect_tx(&myfull[slot], 1280u);
    bulk_g2s(myring + (size_t)slot * 1280u, src, 1280u, &myfull[slot]);
    issued++;
  };
  if (lane == 0)
    for (uint32_t j = 0; j < nslot; j++) issue_next(j);

  const uint32_t btok = PACK ? (g & 3u) : g, bsel = PACK ? (g >> 2) : 0u;
  const bool tok_ok = btok < (uint32_t)MT, xs_lane = !PACK || c < 2;
  const uint32_t ring_s = tc::smem_u32(myring), xb_s = tc::smem_u32(xb), xsum_s = tc::smem_u32(xsum);
  const uint32_t lane_row16 = lane * 16u, tail_off = 1024u + g * 4u;
  const uint32_t xb_lane = xb_s + btok * 128u + c * 32u + bsel * 16u, xs_addr = xsum_s + 2u * c * 4u;
  uint32_t cs = 0, cph = 0, consumed = 0, nbar = 0;
  bool ok = true;

  __shared__ ChainCall s_cc;   // the current call's descriptor, read once per call
  for (uint32_t ci = 0; ci < run.ncalls && ok; ci++) {
    __syncthreads();
    if (threadIdx.x < sizeof(ChainCall) / 4u)
      reinterpret_cast<uint32_t *>(&s_cc)[threadIdx.x] = reinterpret_cast<const uint32_t *>(run.calls + ci)[threadIdx.x];
    __syncthreads();
    const ChainCall &cc = s_cc;
    if (ci > 0 && cc.barrier && !grid_barrier(run, ++nbar, abort_flag)) { ok = false; break; }
    const uint32_t NP = cc.pair ? 2u : 1u;
    for (uint32_t u = first_unit(cc, blockIdx.x, gridDim.x); u < cc.units; u += gridDim.x) {
      const uint32_t ulen = unit_len(cc, u);
      // the unit's x groups: its k-split (geglu: all of K, for the gate and the up records)
      const uint32_t xg0 = cc.pair ? 0u : (u / cc.p.ntile) * cc.Gs, ng = cc.pair ? cc.Gs : ulen;
      const float f = stage_x_seg<MT>(cc.p, xg0, ng, xb, xsum, scratch);
      const uint32_t wa = warp * ulen / kCW, wb = (warp + 1u) * ulen / kCW;
      float acc[2][4][4];
#pragma unroll
      for (int h = 0; h < 2; h++)
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
          for (int i = 0; i < 4; i++) acc[h][r][i] = 0.0f;
      for (uint32_t j = wa; j < wb; j++) {
        const bool got = tc::mbar_wait(&myfull[cs], cph, abort_flag, run.err, 0x7c2u, kCSpin);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        consumed++;
        const uint32_t sl = ring_s + cs * 1280u;
        const uint32_t gx = rec_xgroup(cc, u, j) - xg0;
        Rec q;
        rec_load(q, sl, lane_row16, tail_off);
        uint4 bh = make_uint4(0, 0, 0, 0), bl = bh;
        float x0 = 0.0f, x1 = 0.0f;
        if (tok_ok) {
          bh = lds128(xb_lane + gx * MT * 128u);
          if (!PACK) bl = lds128(xb_lane + gx * MT * 128u + 16u);
        }
        if (xs_lane) {
          if (2 * c < (uint32_t)MT) x0 = __uint_as_float(lds32(xs_addr + gx * MT * 4u));
          if (2 * c + 1 < (uint32_t)MT) x1 = __uint_as_float(lds32(xs_addr + gx * MT * 4u + 4u));
        }
        __syncwarp();
        if (lane == 0) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issue_next(cs);
        }
        if (++cs == nslot) { cs = 0; cph ^= 1u; }
        if (cc.pair && j >= cc.Gs) rec_math<MT, PACK>(acc[1], q, bh, bl, x0, x1);
        else rec_math<MT, PACK>(acc[0], q, bh, bl, x0, x1);
      }
      // a failed wait anywhere in the CTA ends the chain for it and, through the global flag, for every CTA at its
      // next barrier
      __syncthreads();
      if (!ok || *abort_flag) {
        if (threadIdx.x == 0) atomicExch(run.gabort, 1u);
        ok = false;
        break;
      }
      // warp partials in true scale -> shared memory [warp][h][m][row] (the x staging area is free now); a warp with
      // no records adds zeros
      for (uint32_t h = 0; h < NP; h++)
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
          for (int i = 0; i < 4; i++) {
            float v = acc[h][r][i] * f;
            if (PACK) v += __shfl_xor_sync(0xffffffffu, v, 2);
            const uint32_t row = 16u * r + g + (i >= 2 ? 8u : 0u), m = (i & 1) ? 2u * c + 1u : 2u * c;
            if (m < (uint32_t)MT && (!PACK || c < 2)) wpart[((warp * 2u + h) * MT + m) * 64u + row] = v;
          }
      __syncthreads();
      for (uint32_t i = threadIdx.x; i < NP * MT * 64u; i += kCT) {
        float tsum = 0.0f;
        for (uint32_t w = 0; w < (uint32_t)kCW; w++) tsum += wpart[(w * 2u) * MT * 64u + i];   // i = (h * MT + m) * 64 + row
        ctot[i] = tsum;
      }
      __syncthreads();
      unit_epilogue<MT>(cc, u, ctot, vals);
      __syncthreads();
    }
  }
  // copies this warp issued but did not consume (only after a failed wait) land before the CTA exits (bounded)
  if (lane == 0 && consumed < issued) {
    volatile uint32_t never = 0;
    uint32_t slot = cs, ph = cph;
    for (uint32_t k = consumed; k < issued; k++) {
      tc::mbar_wait(&myfull[slot], ph, &never, run.err, 0x7c3u, kCSpin);
      if (++slot == nslot) { slot = 0; ph ^= 1u; }
    }
  }
}

size_t chain_smem(uint32_t M, uint32_t nslot) {
  const size_t xa = std::max((size_t)kCMaxGroups * M * 128 + (size_t)kCMaxGroups * M * 4, (size_t)kCW * 2 * M * 64 * 4);
  return (size_t)kCW * nslot * 1280 + kCW * kCMaxSlots * 8 + 32 * 4 + (size_t)2 * M * 64 * 4 + (size_t)M * 64 * 4 + xa;
}
typedef void (*ChainKernel)(const ChainRun);
ChainKernel chain_kernel_for(uint32_t M) {
  switch (M) {
    case 1: return gemv_chain<1>;
    case 2: return gemv_chain<2>;
    case 3: return gemv_chain<3>;
    case 4: return gemv_chain<4>;
    case 5: return gemv_chain<5>;
    case 6: return gemv_chain<6>;
    case 7: return gemv_chain<7>;
    default: return gemv_chain<8>;
  }
}

}  // namespace p0gemv

using namespace p0gemv;

// ------------------------------------------------------------------------------------------------ host side
namespace {
struct Recorded {
  GemvParams p;
  uint32_t nsplit;
  ChainIO io;
  std::string op;
};
// a run of the chain: calls [i0, i1) as one chain-kernel launch, or one call launched as it would be alone
struct Piece {
  bool kernel;
  uint32_t i0, i1;
  ChainCall *d_calls = nullptr;   // device descriptors of the piece
  uint32_t nslot = 0;
  size_t state_off = 0;          // offset of its [bar, abort] words in the chain's device memory
  size_t state_bytes = 0;
  uint32_t nbar = 0;             // grid barriers inside the launch
};
}  // namespace

struct p0_chain {
  std::vector<Recorded> rec;
  std::vector<Piece> pieces;
  uint32_t M = 0;
  void *d_mem = nullptr;          // descriptors, then state
  size_t d_bytes = 0;
  int device = 0;
};

namespace p0gemv {
p0_status chain_record(p0_ctx *c, const char *op, const GemvParams &p, uint32_t nsplit, const ChainIO &io) {
  auto *ch = static_cast<p0_chain *>(c->chain_rec);
  ch->rec.push_back(Recorded{p, nsplit, io, op});
  return P0_OK;
}
}  // namespace p0gemv

namespace {
bool overlaps(const ChainRange &a, const ChainRange &b) { return a.hi > a.lo && b.hi > b.lo && a.lo < b.hi && b.lo < a.hi; }
bool any_overlap(const ChainRange *a, int na, const std::vector<ChainRange> &set) {
  for (int i = 0; i < na; i++)
    for (const auto &r : set)
      if (overlaps(a[i], r)) return true;
  return false;
}
// the chain kernel takes q4 calls with one M for the whole chain, K per split <= 2048 (geglu: K <= 2048), and few
// enough units that every CTA meets at most a handful (wider calls, the vocabulary head, stream whole tiles per warp
// faster on their own kernels)
bool chain_fits(const GemvParams &p, uint32_t nsplit, uint32_t M, int sms) {
  if (p.q8 || p.M != M) return false;
  const uint32_t G = p.K / 32, Gs = (p.kPer < p.K ? p.kPer : p.K) / 32;
  if (p.wG < G) return false;
  if (p.epi == P0_EPI_GEGLU ? (nsplit != 1 || G > kCMaxGroups) : Gs > kCMaxGroups) return false;
  const uint64_t units = (uint64_t)p.ntile * (p.epi == P0_EPI_GEGLU ? 1u : nsplit);
  return units <= 4ull * (uint64_t)sms;
}
}  // namespace

extern "C" {

p0_status p0_chain_begin(p0_ctx *c) {
  if (!c) return P0_EINVAL;
  if (c->chain_rec) return p0_fail(c, P0_EINVAL, "chain: a chain is already being recorded");
  c->chain_rec = new p0_chain();
  return P0_OK;
}

p0_status p0_chain_end(p0_ctx *c, p0_chain **out) {
  if (!c || !out) return P0_EINVAL;
  *out = nullptr;
  auto *ch = static_cast<p0_chain *>(c->chain_rec);
  if (!ch) return p0_fail(c, P0_EINVAL, "chain: no chain is being recorded");
  c->chain_rec = nullptr;
  ch->device = c->device;
  const int sms = c->sm_count;
  const uint32_t n = (uint32_t)ch->rec.size();
  // the chain kernel's M: the M of the first call it can take
  for (const auto &r : ch->rec)
    if (!r.p.q8) { ch->M = r.p.M; break; }
  // pieces: maximal runs of calls the chain kernel takes; every other call on its own
  for (uint32_t i = 0; i < n;) {
    if (ch->M && chain_fits(ch->rec[i].p, ch->rec[i].nsplit, ch->M, sms)) {
      uint32_t j = i;
      while (j < n && chain_fits(ch->rec[j].p, ch->rec[j].nsplit, ch->M, sms)) j++;
      ch->pieces.push_back(Piece{true, i, j});
      i = j;
    } else {
      ch->pieces.push_back(Piece{false, i, i + 1});
      i++;
    }
  }
  // device memory: per kernel piece its descriptors and its state (barrier arrivals, abort flag)
  const uint32_t M = ch->M ? ch->M : 1;
  std::vector<std::vector<ChainCall>> descs(ch->pieces.size());
  size_t desc_bytes = 0, state_bytes = 0;
  for (size_t pi = 0; pi < ch->pieces.size(); pi++) {
    Piece &pc = ch->pieces[pi];
    if (!pc.kernel) continue;
    std::vector<ChainRange> wr, rd;
    uint32_t dealt = 0;   // units dealt so far in the piece: the next call starts on the CTA after the last one
    for (uint32_t i = pc.i0; i < pc.i1; i++) {
      const Recorded &r = ch->rec[i];
      ChainCall cc{};
      cc.p = r.p;
      cc.nsplit = r.nsplit;
      const uint32_t G = r.p.K / 32, kp = r.p.kPer < r.p.K ? r.p.kPer : r.p.K;
      cc.Gs = r.p.epi == P0_EPI_GEGLU ? G : kp / 32;
      cc.Glast = r.p.epi == P0_EPI_GEGLU ? G : G - (r.nsplit - 1) * cc.Gs;
      cc.pair = r.p.epi == P0_EPI_GEGLU ? 1u : 0u;
      cc.units = r.p.ntile * (cc.pair ? 1u : r.nsplit);
      cc.ubase = dealt % (uint32_t)sms;
      dealt += cc.units;
      // a barrier before this call when it reads what the kernel has written since the last barrier, or writes what
      // it has read or written since then
      const bool dep = i > pc.i0 && (any_overlap(r.io.in, 4, wr) || any_overlap(r.io.out, 2, wr) || any_overlap(r.io.out, 2, rd));
      cc.barrier = dep ? 1u : 0u;
      pc.nbar += cc.barrier;
      if (dep) { wr.clear(); rd.clear(); }
      for (const auto &x : r.io.out) if (x.hi > x.lo) wr.push_back(x);
      for (const auto &x : r.io.in) if (x.hi > x.lo) rd.push_back(x);
      descs[pi].push_back(cc);
    }
    pc.state_off = state_bytes;
    pc.state_bytes = 8 * 4;
    state_bytes += (pc.state_bytes + 255) / 256 * 256;
    desc_bytes += (descs[pi].size() * sizeof(ChainCall) + 255) / 256 * 256;
    uint32_t nslot = kCMaxSlots;
    while (nslot > 2 && chain_smem(M, nslot) > 226u * 1024u) nslot--;   // + the static descriptor copy
    pc.nslot = nslot;
  }
  ch->d_bytes = desc_bytes + state_bytes;
  if (ch->d_bytes) {
    cudaSetDevice(c->device);
    cudaError_t e = cudaMalloc(&ch->d_mem, ch->d_bytes);
    if (e != cudaSuccess) {
      cudaGetLastError();
      const size_t want = ch->d_bytes;
      delete ch;
      return p0_fail(c, P0_ENOMEM, "chain: %zu bytes of device state: %s", want, cudaGetErrorString(e));
    }
    uint8_t *base = (uint8_t *)ch->d_mem;
    size_t doff = 0;
    for (size_t pi = 0; pi < ch->pieces.size(); pi++) {
      Piece &pc = ch->pieces[pi];
      if (!pc.kernel) continue;
      pc.d_calls = (ChainCall *)(base + doff);
      e = cudaMemcpy(base + doff, descs[pi].data(), descs[pi].size() * sizeof(ChainCall), cudaMemcpyHostToDevice);
      if (e != cudaSuccess) { p0_status st = p0_cuda(c, e, "chain"); cudaFree(ch->d_mem); delete ch; return st; }
      doff += (descs[pi].size() * sizeof(ChainCall) + 255) / 256 * 256;
    }
    // state zeroed once here and before every launch
    e = cudaMemset(base + desc_bytes, 0, state_bytes);
    // those copies and the memset run on the legacy stream and may still be in flight when the calls return; the
    // context's stream (non-blocking) does not wait for it, so finish them before a run can be enqueued
    if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamLegacy);
    if (e != cudaSuccess) { p0_status st = p0_cuda(c, e, "chain"); cudaFree(ch->d_mem); delete ch; return st; }
    for (auto &pc : ch->pieces) pc.state_off += desc_bytes;
  }
  *out = ch;
  return P0_OK;
}

p0_status p0_chain_run(p0_ctx *c, p0_chain *ch) {
  if (!c || !ch) return P0_EINVAL;
  if (c->chain_rec) return p0_fail(c, P0_EINVAL, "chain: p0_chain_run while a chain is being recorded");
  if (ch->device != c->device) return p0_fail(c, P0_EINVAL, "chain: recorded on device %d, run on %d", ch->device, c->device);
  cudaSetDevice(c->device);
  p0_status st;
  const int sms = c->sm_count;
  uint8_t *base = (uint8_t *)ch->d_mem;
  for (const Piece &pc : ch->pieces) {
    if (!pc.kernel) {
      const Recorded &r = ch->rec[pc.i0];
      GemvParams p = r.p;
      p.overlap = c->overlap ? 1 : 0;
      if ((st = gemv_dispatch(c, r.op.c_str(), p, r.nsplit, false))) return st;
      continue;
    }
    uint32_t *state = (uint32_t *)(base + pc.state_off);
    if ((st = p0_cuda(c, cudaMemsetAsync(state, 0, pc.state_bytes, c->stream), "chain"))) return st;
    ChainRun run{};
    run.calls = pc.d_calls;
    run.ncalls = pc.i1 - pc.i0;
    run.nslot = pc.nslot;
    run.bar = state;
    run.gabort = state + 1;
    run.err = c->d_err;
    ChainKernel k = chain_kernel_for(ch->M);
    const size_t smem = chain_smem(ch->M, pc.nslot);
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kCT, smem) != cudaSuccess || occ < 1) {
      cudaGetLastError();
      return p0_fail(c, P0_EDEVICE, "chain: the chain kernel does not fit an SM (%zu bytes of shared memory)", smem);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(kCT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;   // every CTA resident: the grid barriers cannot wait on an unscheduled CTA
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if ((st = p0_cuda(c, cudaLaunchKernelEx(&cfg, k, run), "chain"))) return st;
    if ((st = p0_launched(c, "chain"))) return st;
  }
  return P0_OK;
}

p0_status p0_chain_info(p0_ctx *c, const p0_chain *ch, uint32_t *calls, uint32_t *kernel_calls, uint32_t *launches, uint32_t *barriers) {
  if (!c || !ch) return P0_EINVAL;
  uint32_t kc = 0, bars = 0;
  for (const Piece &pc : ch->pieces)
    if (pc.kernel) { kc += pc.i1 - pc.i0; bars += pc.nbar; }
  if (calls) *calls = (uint32_t)ch->rec.size();
  if (kernel_calls) *kernel_calls = kc;
  if (launches) *launches = (uint32_t)ch->pieces.size();
  if (barriers) *barriers = bars;
  return P0_OK;
}

p0_status p0_chain_free(p0_ctx *c, p0_chain *ch) {
  if (!c || !ch) return P0_EINVAL;
  if (ch->d_mem) {
    cudaSetDevice(ch->device);
    cudaStreamSynchronize(c->stream);   // a run in flight may still read the descriptors
    cudaFree(ch->d_mem);
  }
  delete ch;
  return P0_OK;
}

}  // extern "C"
