// context.cu -- device context, buffers and synchronisation: the replacement of the WebGPU buffer path in
// engine/core/gpu.js (createGpu :18-23, Gpu.buffer :81-88, free :89-94, upload :98-117, _readback :118-140,
// done :141-147) for the matmul operators. One context per device; all work goes on one CUDA stream in order.
#include <chrono>
#include <cstring>
#include <thread>

#include "internal.h"
#include "tc.cuh"

namespace {
// One warp waits on an mbarrier phase that nothing completes (one expected arrival, none made), through the same
// bounded wait the GEMV / GEMM kernels use for their copies. The wait gives up after `polls` tries, records `code`
// in the context's error word and the kernel returns: the failure path of an in-kernel wait, with no fault.
__global__ void wait_selftest_kernel(uint32_t *err, uint32_t polls, uint32_t code) {
  __shared__ uint64_t bar;
  __shared__ uint32_t abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    abort_flag = 0u;
    tc::fence_mbar_init();
  }
  __syncthreads();
  tc::mbar_wait(&bar, 0u, &abort_flag, err, code, polls);
  __syncthreads();
}
}  // namespace

p0_status p0_workspace(p0_ctx *c, size_t cnt_bytes, size_t scratch_bytes, uint32_t **cnt, void **scratch) {
  const size_t MB = (size_t)1 << 20;
  cnt_bytes = (cnt_bytes + 255) / 256 * 256;
  if (cnt_bytes > c->ws_cnt_bytes || c->ws_cnt_bytes + scratch_bytes > c->ws_bytes) {
    const size_t ncnt = cnt_bytes > c->ws_cnt_bytes ? (cnt_bytes < 65536 ? 65536 : cnt_bytes) : c->ws_cnt_bytes;
    size_t want = ncnt + scratch_bytes;
    want = want < MB ? MB : (want + MB - 1) / MB * MB;
    if (want < c->ws_bytes) want = c->ws_bytes;
    if (c->ws) {
      p0_status st = p0_cuda(c, cudaStreamSynchronize(c->stream), "workspace");   // queued kernels may still use it
      if (st) return st;
      cudaFree(c->ws);
      c->ws = nullptr;
      c->ws_bytes = c->ws_cnt_bytes = 0;
    }
    cudaError_t e = cudaMalloc(&c->ws, want);
    if (e != cudaSuccess) { cudaGetLastError(); c->ws = nullptr; return p0_fail(c, P0_ENOMEM, "workspace %zu B: %s", want, cudaGetErrorString(e)); }
    if ((e = cudaMemsetAsync(c->ws, 0, want, c->stream)) != cudaSuccess) return p0_cuda(c, e, "workspace zero-fill");
    c->ws_bytes = want;
    c->ws_cnt_bytes = ncnt;
  }
  *cnt = (uint32_t *)c->ws;
  *scratch = (uint8_t *)c->ws + c->ws_cnt_bytes;
  return P0_OK;
}

extern "C" {

p0_status p0_init(int device, p0_ctx **out) {
  if (!out) return P0_EINVAL;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return P0_EDEVICE;
  if (device < 0 || device >= n) return P0_EINVAL;
  p0_ctx *c = new p0_ctx();
  c->device = device;
  p0_status st;
  // a failed step releases what the earlier steps made (p0_destroy takes a partly built context)
  if ((st = p0_cuda(c, cudaSetDevice(device), "p0_init")) != P0_OK) { p0_destroy(c); return st; }
  if ((st = p0_cuda(c, cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device), "p0_init SM count")) != P0_OK ||
      c->sm_count <= 0) {
    p0_destroy(c);
    return st != P0_OK ? st : P0_EDEVICE;
  }
  if ((st = p0_cuda(c, cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking), "p0_init stream")) != P0_OK) { p0_destroy(c); return st; }
  c->stream = c->own_stream;
  if ((st = p0_cuda(c, cudaMalloc(&c->d_err, 16), "p0_init error word")) != P0_OK) { p0_destroy(c); return st; }
  if ((st = p0_cuda(c, cudaMemset(c->d_err, 0, 16), "p0_init error word")) != P0_OK) { p0_destroy(c); return st; }
  if ((st = p0_cuda(c, cudaMallocHost(&c->h_err, 16), "p0_init pinned word")) != P0_OK) { p0_destroy(c); return st; }
  memset(c->h_err, 0, 16);
  if ((st = p0_cuda(c, cudaDeviceSynchronize(), "p0_init")) != P0_OK) { p0_destroy(c); return st; }
  *out = c;
  return P0_OK;
}

p0_status p0_destroy(p0_ctx *c) {
  if (!c) return P0_EINVAL;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  for (auto &kv : c->bufs)
    if (kv.second.owned) cudaFree(kv.second.ptr);
  c->bufs.clear();
  if (c->ws) cudaFree(c->ws);
  if (c->d_err) cudaFree(c->d_err);
  if (c->h_err) cudaFreeHost(c->h_err);
  for (int i = 0; i < 2; i++) {
    if (c->io_stage[i]) cudaFreeHost(c->io_stage[i]);
    if (c->io_done[i]) cudaEventDestroy(c->io_done[i]);
  }
  if (c->own_stream) cudaStreamDestroy(c->own_stream);
  delete c;
  return P0_OK;
}

p0_status p0_set_stream(p0_ctx *c, void *s) {
  if (!c) return P0_EINVAL;
  // NULL selects the context's own stream; CUDA's legacy default stream is cudaStreamLegacy
  c->stream = s ? (cudaStream_t)s : c->own_stream;
  return P0_OK;
}

p0_status p0_set_overlap(p0_ctx *c, uint32_t flags) {
  if (!c) return P0_EINVAL;
  if (flags & ~(uint32_t)P0_OVERLAP_WEIGHTS) return p0_fail(c, P0_EINVAL, "set_overlap: unknown flags 0x%x", flags);
  c->overlap = (flags & P0_OVERLAP_WEIGHTS) != 0;
  return P0_OK;
}

p0_status p0_last_error(p0_ctx *c, char *msg, size_t cap) {
  if (!c || !msg || !cap) return P0_EINVAL;
  snprintf(msg, cap, "%s", c->last_error.c_str());
  return P0_OK;
}

p0_status p0_stats(p0_ctx *c, uint64_t *alive, uint64_t *peak, uint64_t *disp) {
  if (!c) return P0_EINVAL;
  if (alive) *alive = c->alive;
  if (peak) *peak = c->peak;
  if (disp) *disp = c->dispatches;
  return P0_OK;
}

p0_status p0_buffer(p0_ctx *c, size_t bytes, const char *label, p0_buf *out) {
  if (!c || !out) return P0_EINVAL;
  out->id = 0;
  size_t size = bytes < 16 ? 16 : (bytes + 15) / 16 * 16;   // Math.max(16, ceil(size / 16) * 16), gpu.js:82
  cudaSetDevice(c->device);
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, size);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return p0_fail(c, P0_ENOMEM, "buffer %s %zu B: %s", label ? label : "", size, cudaGetErrorString(e));
  }
  // WebGPU buffers start zero-filled
  if ((e = cudaMemsetAsync(p, 0, size, c->stream)) != cudaSuccess) { cudaFree(p); return p0_cuda(c, e, "buffer zero-fill"); }
  P0Buffer b;
  b.ptr = p; b.bytes = size; b.owned = true; b.label = label ? label : "";
  out->id = c->next_id++;
  c->bufs.emplace(out->id, b);
  c->alive += size;
  if (c->alive > c->peak) c->peak = c->alive;
  return P0_OK;
}

p0_status p0_wrap(p0_ctx *c, void *ptr, size_t bytes, const char *label, p0_buf *out) {
  if (!c || !out) return P0_EINVAL;
  out->id = 0;
  if (!ptr) return p0_fail(c, P0_EINVAL, "wrap: null device pointer");
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, ptr) != cudaSuccess || at.type != cudaMemoryTypeDevice) {
    cudaGetLastError();
    return p0_fail(c, P0_EINVAL, "wrap: %s is not device memory", label ? label : "");
  }
  // the kernels read and write a context's buffers as this device's own memory
  if (at.device != c->device)
    return p0_fail(c, P0_EINVAL, "wrap: %s is memory of device %d, the context's device is %d", label ? label : "", at.device, c->device);
  P0Buffer b;
  b.ptr = ptr; b.bytes = bytes; b.owned = false; b.label = label ? label : "";
  out->id = c->next_id++;
  c->bufs.emplace(out->id, b);
  return P0_OK;
}

p0_status p0_free(p0_ctx *c, p0_buf b) {
  if (!c) return P0_EINVAL;
  auto it = c->bufs.find(b.id);
  if (it == c->bufs.end()) return P0_OK;   // Gpu.free ignores unknown buffers (gpu.js:90)
  if (it->second.owned) {
    cudaStreamSynchronize(c->stream);     // no queued kernel may still read it
    cudaFree(it->second.ptr);
    c->alive -= it->second.bytes;
  }
  c->bufs.erase(it);
  return P0_OK;
}

p0_status p0_upload(p0_ctx *c, p0_buf b, size_t off, const void *src, size_t n) {
  if (!c) return P0_EINVAL;
  P0Range r;
  p0_status st = p0_range(c, b, off, n, "upload", "dst", &r);
  if (st) return st;
  if (!n) return P0_OK;
  return p0_cuda(c, cudaMemcpyAsync((void *)r.base, src, n, cudaMemcpyHostToDevice, c->stream), "upload");
}

p0_status p0_copy(p0_ctx *c, p0_buf src, size_t src_off, p0_buf dst, size_t dst_off, size_t n) {
  if (!c) return P0_EINVAL;
  P0Range rs, rd;
  p0_status st = p0_range(c, src, src_off, n, "copy", "src", &rs);
  if (st) return st;
  if ((st = p0_range(c, dst, dst_off, n, "copy", "dst", &rd))) return st;
  if (!n) return P0_OK;
  return p0_cuda(c, cudaMemcpyAsync((void *)rd.base, rs.base, n, cudaMemcpyDeviceToDevice, c->stream), "copy");
}

p0_status p0_read(p0_ctx *c, p0_buf b, size_t off, size_t n, void *dst) {
  if (!c) return P0_EINVAL;
  P0Range r;
  p0_status st = p0_range(c, b, off, n, "read", "src", &r);
  if (st) return st;
  if (n && (st = p0_cuda(c, cudaMemcpyAsync(dst, r.base, n, cudaMemcpyDeviceToHost, c->stream), "read"))) return st;
  return p0_cuda(c, cudaStreamSynchronize(c->stream), "read sync");
}

p0_status p0_done(p0_ctx *c, uint32_t timeout_ms) {
  if (!c) return P0_EINVAL;
  // bounded wait: poll the stream rather than block on it
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaStreamQuery(c->stream);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return p0_cuda(c, e, "done");
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms && ms > (long long)timeout_ms) return p0_fail(c, P0_ETIMEOUT, "done: the device did not finish within %u ms", timeout_ms);
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  // in-kernel bounded waits that ran out leave a code in the error word
  p0_status st = p0_cuda(c, cudaMemcpy(c->h_err, c->d_err, 4, cudaMemcpyDeviceToHost), "done error word");
  if (st) return st;
  if (c->h_err[0]) {
    uint32_t code = c->h_err[0];
    // the resets go on the context's stream, so the next call's kernels run after them (a plain cudaMemset would run
    // on the legacy stream, which the context's non-blocking stream does not wait for)
    if ((st = p0_cuda(c, cudaMemsetAsync(c->d_err, 0, 4, c->stream), "done error word"))) return st;
    // a kernel that gave up may have left workspace counters mid-count: start the next call from zero
    if (c->ws && (st = p0_cuda(c, cudaMemsetAsync(c->ws, 0, c->ws_bytes, c->stream), "done workspace"))) return st;
    return p0_fail(c, P0_ETIMEOUT, "done: a kernel gave up a bounded wait (code 0x%x)", code);
  }
  return P0_OK;
}

p0_status p0_device_ptr(p0_ctx *c, p0_buf b, uint64_t *out) {
  if (!c || !out) return P0_EINVAL;
  const P0Buffer *B = p0_lookup(c, b);
  if (!B) return p0_fail(c, P0_EINVAL, "device_ptr: not a live buffer");
  *out = (uint64_t)(uintptr_t)B->ptr;
  return P0_OK;
}

p0_status p0_wait_selftest(p0_ctx *c, uint32_t polls) {
  if (!c) return P0_EINVAL;
  if (polls == 0 || polls > (1u << 20)) return p0_fail(c, P0_EINVAL, "wait_selftest: polls must be in [1, 2^20]");
  wait_selftest_kernel<<<1, 32, 0, c->stream>>>(c->d_err, polls, 0x7e1u);
  return p0_launched(c, "wait_selftest");
}

const char *p0_version(void) { return "p0mm sm_100a gemv-v5 gemm-tc-v2 lops-v1 io-v1"; }

}  // extern "C"
