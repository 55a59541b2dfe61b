// pack.cu -- the quantisers on the device, bit for bit: packQ4 (q4g32a.t64, engine/kcheck.js:22-38) and packQ8
// (q8g64s.t64, engine/kcheck.js:39-52).
// One thread per (row, 32-k group): mn = f16(min), s = f16((max - mn) / 15) (s == 0 -> 1), q = clamp(rhe((w - mn) / s),
// 0, 15), bytes r*16 + j = q[2j] | q[2j+1] << 4, word 1024 + 4r = f16(s) | f16(mn) << 16. The reference computes in
// f64 and converts f64 -> f32 -> f16 with round-to-nearest-even (core/gpu.js:274-289); so does this kernel.
#include <cuda_fp16.h>

#include "internal.h"

namespace {

__device__ __forceinline__ double rf16(double x) { return (double)__half2float(__float2half_rn((float)x)); }
__device__ __forceinline__ uint32_t f2h(double x) { return __half_as_ushort(__float2half_rn((float)x)); }

__global__ void pack_q4_kernel(const float *__restrict__ W, uint64_t ldw, uint32_t N, uint32_t K, uint8_t *__restrict__ out) {
  const uint32_t G = K / 32;
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)N * G) return;
  // consecutive threads take consecutive rows of one group: their 16-byte code stores are contiguous
  const uint32_t g = (uint32_t)(idx / N), n = (uint32_t)(idx % N);
  const uint32_t t = n / 64, r = n % 64;
  const float *w = W + (uint64_t)n * ldw + (uint64_t)g * 32;
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = w[i];
  double mnv = v[0], mxv = v[0];
#pragma unroll
  for (int i = 1; i < 32; i++) { mnv = v[i] < mnv ? v[i] : mnv; mxv = v[i] > mxv ? v[i] : mxv; }
  const double mn = rf16(mnv);
  double s = rf16((mxv - mn) / 15.0);
  if (s == 0.0) s = 1.0;
  uint32_t words[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < 32; i++) {
    double q = rint(((double)v[i] - mn) / s);   // rhe: round half to even
    q = q < 0.0 ? 0.0 : (q > 15.0 ? 15.0 : q);
    words[i / 8] |= (uint32_t)q << (4 * (i % 8));
  }
  uint8_t *rec = out + ((uint64_t)t * G + g) * 1280u;
  *reinterpret_cast<uint4 *>(rec + r * 16) = make_uint4(words[0], words[1], words[2], words[3]);
  *reinterpret_cast<uint32_t *>(rec + 1024 + r * 4) = f2h(s) | (f2h(mn) << 16);
}

// packQ8 (kcheck.js:39-52), one thread per (row, 64-k group): s = f16(max|w| / 127) (s == 0 -> 1), q = clamp(rhe(w / s),
// -128, 127); bytes r*64 + i = q & 255 of record (t, g) (4224 B), u16 at 4096 + 2r = f16(s).
__global__ void pack_q8_kernel(const float *__restrict__ W, uint64_t ldw, uint32_t N, uint32_t K, uint8_t *__restrict__ out) {
  const uint32_t G = K / 64;
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)N * G) return;
  const uint32_t g = (uint32_t)(idx / N), n = (uint32_t)(idx % N);
  const uint32_t t = n / 64, r = n % 64;
  const float *w = W + (uint64_t)n * ldw + (uint64_t)g * 64;
  double am = 0.0;
  for (int i = 0; i < 64; i++) { const double a = fabs((double)w[i]); am = a > am ? a : am; }
  double s = rf16(am / 127.0);
  if (s == 0.0) s = 1.0;
  uint8_t *rec = out + ((uint64_t)t * G + g) * 4224u;
  for (int c = 0; c < 4; c++) {
    uint32_t words[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 16; i++) {
      double q = rint((double)w[c * 16 + i] / s);   // rhe: round half to even
      q = q < -128.0 ? -128.0 : (q > 127.0 ? 127.0 : q);
      words[i / 4] |= ((uint32_t)(int32_t)q & 255u) << (8 * (i % 4));
    }
    *reinterpret_cast<uint4 *>(rec + r * 64 + c * 16) = make_uint4(words[0], words[1], words[2], words[3]);
  }
  *reinterpret_cast<uint16_t *>(rec + 4096 + r * 2) = (uint16_t)f2h(s);
}

}  // namespace

extern "C" {

p0_status p0_pack_q8(p0_ctx *c, p0_buf w, uint64_t w_off, uint32_t ldw, uint32_t N, uint32_t K, p0_buf out, uint64_t out_off) {
  if (!c) return P0_EINVAL;
  if (N % 64 || K % 64 || !N || !K) return p0_fail(c, P0_EINVAL, "packQ8: N must be a multiple of 64 and K of 64");
  const uint32_t ld = ldw ? ldw : K;
  if (ld < K) return p0_fail(c, P0_EINVAL, "packQ8: row stride %u < K %u", ld, K);
  P0Range rw, ro;
  p0_status st;
  if ((st = p0_range(c, w, w_off, ((uint64_t)(N - 1) * ld + K) * 4, "packQ8", "W", &rw))) return st;
  if ((st = p0_range(c, out, out_off, (uint64_t)N * K / 64 * 66, "packQ8", "out", &ro))) return st;
  if ((uintptr_t)rw.base % 4 || (uintptr_t)ro.base % 16) return p0_fail(c, P0_EALIGN, "packQ8: W 4-byte and out 16-byte alignment");
  const uint64_t n = (uint64_t)N * (K / 64);
  cudaSetDevice(c->device);
  pack_q8_kernel<<<(unsigned)((n + 255) / 256), 256, 0, c->stream>>>((const float *)rw.base, ld, N, K, (uint8_t *)ro.base);
  return p0_launched(c, "packQ8");
}

p0_status p0_pack_q4(p0_ctx *c, p0_buf w, uint64_t w_off, uint32_t ldw, uint32_t N, uint32_t K, p0_buf out, uint64_t out_off) {
  if (!c) return P0_EINVAL;
  if (N % 64 || K % 32 || !N || !K) return p0_fail(c, P0_EINVAL, "packQ4: N must be a multiple of 64 and K of 32");
  const uint32_t ld = ldw ? ldw : K;
  if (ld < K) return p0_fail(c, P0_EINVAL, "packQ4: row stride %u < K %u", ld, K);
  P0Range rw, ro;
  p0_status st;
  if ((st = p0_range(c, w, w_off, ((uint64_t)(N - 1) * ld + K) * 4, "packQ4", "W", &rw))) return st;
  if ((st = p0_range(c, out, out_off, (uint64_t)N * K / 32 * 20, "packQ4", "out", &ro))) return st;
  if ((uintptr_t)rw.base % 4 || (uintptr_t)ro.base % 16) return p0_fail(c, P0_EALIGN, "packQ4: W 4-byte and out 16-byte alignment");
  const uint64_t n = (uint64_t)N * (K / 32);
  cudaSetDevice(c->device);
  pack_q4_kernel<<<(unsigned)((n + 255) / 256), 256, 0, c->stream>>>((const float *)rw.base, ld, N, K, (uint8_t *)ro.base);
  return p0_launched(c, "packQ4");
}

}  // extern "C"
