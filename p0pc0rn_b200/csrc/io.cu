// io.cu -- shard upload straight from a pack file (the reference's WeightStore.upload, engine/core/store.js:222-245):
// the file is read in 16 MiB chunks with pread into two pinned staging buffers that alternate, each chunk copied to
// the device buffer with cudaMemcpyAsync on the context's stream, so the next chunk's disk read overlaps the last
// chunk's PCIe copy. A staging buffer is refilled only after the event recorded behind its previous copy has fired.
#include <fcntl.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>

#include "internal.h"

namespace {
constexpr size_t kChunk = 16u << 20;   // the reference's CH (store.js:226)
}

extern "C" {

p0_status p0_upload_file(p0_ctx *c, p0_buf dst, uint64_t dst_off, const char *path, uint64_t file_off, uint64_t bytes) {
  if (!c || !path) return P0_EINVAL;
  P0Range r;
  p0_status st = p0_range(c, dst, dst_off, bytes, "upload", "dst", &r);
  if (st) return st;
  if (!bytes) return P0_OK;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return p0_fail(c, P0_EINVAL, "upload: cannot open %s: %s", path, strerror(errno));
  cudaSetDevice(c->device);
  for (int i = 0; i < 2; i++) {
    if (!c->io_stage[i] && (st = p0_cuda(c, cudaHostAlloc(&c->io_stage[i], kChunk, cudaHostAllocDefault), "upload staging"))) {
      close(fd);
      return st;
    }
    if (!c->io_done[i] && (st = p0_cuda(c, cudaEventCreateWithFlags(&c->io_done[i], cudaEventDisableTiming), "upload event"))) {
      close(fd);
      return st;
    }
  }
  uint8_t *out = (uint8_t *)r.base;
  uint64_t done = 0;
  for (uint64_t i = 0; done < bytes; i++) {
    const int b = (int)(i & 1);
    const size_t len = (size_t)((bytes - done) < kChunk ? (bytes - done) : kChunk);
    // the buffer's previous copy (chunk i - 2) must have left it before the disk read overwrites it
    if ((st = p0_cuda(c, cudaEventSynchronize(c->io_done[b]), "upload wait"))) break;
    size_t got = 0;
    while (got < len) {
      const ssize_t n = pread(fd, (uint8_t *)c->io_stage[b] + got, len - got, (off_t)(file_off + done + got));
      if (n < 0 && errno == EINTR) continue;
      if (n <= 0) {
        st = p0_fail(c, P0_EINVAL, "upload: %s: read of %zu bytes at %llu failed (%s)", path, len - got,
                     (unsigned long long)(file_off + done + got), n < 0 ? strerror(errno) : "end of file");
        break;
      }
      got += (size_t)n;
    }
    if (st) break;
    if ((st = p0_cuda(c, cudaMemcpyAsync(out + done, c->io_stage[b], len, cudaMemcpyHostToDevice, c->stream), "upload copy"))) break;
    if ((st = p0_cuda(c, cudaEventRecord(c->io_done[b], c->stream), "upload record"))) break;
    done += len;
  }
  close(fd);
  return st;
}

}  // extern "C"
