// internal.h -- shared state of the p0mm library: the context, buffer table and the error plumbing.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/p0mm.h"

struct P0Buffer {
  void *ptr = nullptr;
  size_t bytes = 0;
  bool owned = true;
  std::string label;
};

struct p0_ctx {
  int device = 0;
  int sm_count = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  std::unordered_map<uint64_t, P0Buffer> bufs;
  uint64_t next_id = 1;
  uint64_t alive = 0, peak = 0, dispatches = 0;
  std::string last_error;
  uint32_t *d_err = nullptr;     // device word: kernels record a bounded-wait timeout here (never trap)
  uint32_t *h_err = nullptr;     // pinned mirror read by p0_done
  // kernel workspace, grown on demand: [counters: ws_cnt_bytes][scratch: the rest]. The counter region never moves
  // or shrinks while the workspace lives, so one call's scratch never lands on another call's counters.
  void *ws = nullptr;
  size_t ws_bytes = 0, ws_cnt_bytes = 0;
  void *chain_rec = nullptr;     // p0_chain_begin .. p0_chain_end: gemv / gemvM calls are recorded into this chain
  bool overlap = false;          // p0_set_overlap: weights are static, GEMVs may fetch them before the call ahead ends
  // p0_upload_file: two pinned staging chunks and the events that say when the copy out of each has finished
  void *io_stage[2] = {nullptr, nullptr};
  cudaEvent_t io_done[2] = {nullptr, nullptr};
  std::mutex mu;
};

// the context's workspace with at least `cnt_bytes` of counters (zero between calls) and `scratch_bytes` of scratch
// after them. Zero-filled when (re)allocated; kernels that use it leave every counter at zero when they finish, so it
// is never cleared between calls. Growing it waits for the stream first.
p0_status p0_workspace(p0_ctx *c, size_t cnt_bytes, size_t scratch_bytes, uint32_t **cnt, void **scratch);

// records the message and returns the status (message wording follows the reference's `throw new Error(...)`)
inline p0_status p0_fail(p0_ctx *c, p0_status st, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (c) c->last_error = buf;
  return st;
}

inline p0_status p0_cuda(p0_ctx *c, cudaError_t e, const char *what) {
  if (e == cudaSuccess) return P0_OK;
  return p0_fail(c, e == cudaErrorMemoryAllocation ? P0_ENOMEM : P0_EDEVICE, "%s: %s", what, cudaGetErrorString(e));
}

// resolves a buffer handle; id 0 -> nullptr with size 0 (an absent optional binding)
inline const P0Buffer *p0_lookup(p0_ctx *c, p0_buf b) {
  if (b.id == 0) return nullptr;
  auto it = c->bufs.find(b.id);
  return it == c->bufs.end() ? nullptr : &it->second;
}

// a bound range [off, off + bytes) of a buffer, checked like a WebGPU binding (offset + size <= buffer size)
struct P0Range {
  const uint8_t *base = nullptr;
  size_t bytes = 0;
};
inline p0_status p0_range(p0_ctx *c, p0_buf b, uint64_t off, uint64_t need, const char *op, const char *name, P0Range *out,
                          bool optional = false) {
  if (b.id == 0) {
    if (optional) { *out = P0Range{}; return P0_OK; }
    return p0_fail(c, P0_EINVAL, "%s: missing binding %s", op, name);
  }
  const P0Buffer *B = p0_lookup(c, b);
  if (!B) return p0_fail(c, P0_EINVAL, "%s: %s is not a live buffer", op, name);
  if (off > B->bytes || need > B->bytes - off)
    return p0_fail(c, P0_EINVAL, "%s: %s range [%llu, +%llu) exceeds its buffer of %llu bytes", op, name, (unsigned long long)off,
                   (unsigned long long)need, (unsigned long long)B->bytes);
  out->base = (const uint8_t *)B->ptr + off;
  out->bytes = B->bytes - off;
  return P0_OK;
}

// launch bookkeeping: counts dispatches and turns launch errors into statuses
inline p0_status p0_launched(p0_ctx *c, const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return p0_cuda(c, e, what);
  c->dispatches++;
  return P0_OK;
}

// in-kernel bounded waits give up after this many polls and record P0_ETIMEOUT in the context's error word
#define P0_SPIN_LIMIT (1u << 26)
