/*
 * p0mm.h -- C ABI of the B200 (sm_100a) 4-bit quantized matmul library for p0pc0rn.
 *
 * This is the drop-in boundary for p0pc0rn's three matmul operators and the buffer calls they ride on.
 * The reference binds these as JavaScript functions over WebGPU buffers; each entry point below names the
 * reference interface it replaces (paths are inside the reference repository ArtistJoshHughes/p0pc0rn).
 * Plain pointers and sizes only; every call returns a p0_status and never traps. A non-zero status is
 * returned where the reference throws; p0_last_error() gives the message in the reference's wording.
 *
 * Units follow the reference: weight / x / y byte offsets where the reference uses bytes (ops/gemm.js:300-302),
 * f32-element offsets where it uses elements (llm/lops.js:127-128: x.rowB, norm.off, stat.off, ev.off).
 * All work is enqueued on the context's stream and is asynchronous; p0_read() and p0_done() synchronise.
 * A context is used by one thread at a time (as the reference's Gpu object lives on JavaScript's one thread): calls
 * on the same context from several threads at once must be serialised by the caller. Separate contexts, one per
 * thread, may be used concurrently.
 */
#ifndef P0MM_H
#define P0MM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct p0_ctx p0_ctx;
/* an opaque device allocation; id 0 means "no buffer" (an absent optional binding) */
typedef struct { uint64_t id; } p0_buf;

typedef enum {
  P0_OK = 0,
  P0_EINVAL = 1,    /* argument error: the reference throws `new Error(...)` */
  P0_EALIGN = 2,    /* offset / stride alignment the kernels need */
  P0_ENOMEM = 3,
  P0_EDEVICE = 4,   /* CUDA error; the device may be lost (reference: GpuError / GPU_LOST, core/gpu.js:141-147) */
  P0_ETIMEOUT = 5,  /* a bounded wait ran out (host poll or an in-kernel wait) */
  P0_ECOMM = 6
} p0_status;

/* weight encodings: engine/kcheck.js:22-53 (q4g32a.t64: 1280 B per 64-row x 32-k record; q8g64s.t64: 4224 B per
 * 64-row x 64-k record); 'f16' = row-major fp16 with a row stride */
enum { P0_ENC_Q4G32A_T64 = 1, P0_ENC_Q8G64S_T64 = 2, P0_ENC_F16 = 3 };

/* ---------------------------------------------------------------------------------------------- device context */
/* createGpu (engine/core/gpu.js:18-23): one context per device; owns a CUDA stream and every buffer */
p0_status p0_init(int device, p0_ctx **out);
/* Gpu.freeAll (engine/core/gpu.js:95) + device.destroy: frees every buffer, the stream and the context */
p0_status p0_destroy(p0_ctx *ctx);
/* run subsequent work on an external cudaStream_t (NULL = the context's own stream; pass cudaStreamLegacy for CUDA's
 * legacy default stream, whose handle 0 would otherwise mean "own stream"). No counterpart in the reference, whose
 * device has one queue. */
p0_status p0_set_stream(p0_ctx *ctx, void *cuda_stream);
/* Consecutive GEMV calls on the context's stream always overlap their launch with the call ahead (programmatic
 * dependent launch: a call waits for the work ahead before it reads x or writes anything). With P0_OVERLAP_WEIGHTS set
 * a call also starts fetching its weights before the work ahead has finished; the caller then guarantees that no work
 * still in flight on the stream writes a weight buffer a later GEMV reads (weights written once, then the stream
 * synchronised, as a loaded model's are). No counterpart in the reference, whose WebGPU queue runs dispatches in
 * order. Default: 0. */
enum { P0_OVERLAP_WEIGHTS = 1 };
p0_status p0_set_overlap(p0_ctx *ctx, uint32_t flags);
/* the message of the last failed call, in the reference's wording (e.g. "gemv: N % 64", the Error that
 * engine/llm/lops.js:122 throws); the reference hands its messages over as thrown errors instead */
p0_status p0_last_error(p0_ctx *ctx, char *msg, size_t cap);
/* byte accounting (gpu.js:28, 81-96) and dispatch counter (Runner, gpu.js:177-179) */
p0_status p0_stats(p0_ctx *ctx, uint64_t *alive_bytes, uint64_t *peak_bytes, uint64_t *dispatches);

/* ---------------------------------------------------------------------------------------------- buffers */
/* Gpu.buffer(bytes, label) (gpu.js:81-96): device allocation rounded up to 16 B, zero-filled, accounted */
p0_status p0_buffer(p0_ctx *ctx, size_t bytes, const char *label, p0_buf *out);
/* register caller-owned device memory (e.g. a torch tensor) as a buffer; p0_free() only unregisters it. No
 * counterpart in the reference (WebGPU buffers are always created by the device). */
p0_status p0_wrap(p0_ctx *ctx, void *device_ptr, size_t bytes, const char *label, p0_buf *out);
/* Gpu.upload / queue.writeBuffer (gpu.js:98-117): host -> device, ordered on the stream */
p0_status p0_upload(p0_ctx *ctx, p0_buf buf, size_t dst_off, const void *src, size_t n);
/* WeightStore.upload's copy loop (core/store.js:222-245) from a pack file: bytes at file_off of the file at path ->
 * buf at dst_off, in 16 MiB chunks through two pinned staging buffers (disk reads overlap the copies). Returns with the
 * last copies in flight on the stream; the staging buffers are reused only after their copies have finished. */
p0_status p0_upload_file(p0_ctx *ctx, p0_buf buf, uint64_t dst_off, const char *path, uint64_t file_off, uint64_t bytes);
/* Runner.copy(src, srcOff, dst, dstOff, size) (gpu.js:237): device -> device, ordered on the stream */
p0_status p0_copy(p0_ctx *ctx, p0_buf src, size_t src_off, p0_buf dst, size_t dst_off, size_t n);
/* Gpu.read(buf, off, n) -> Gpu._readback (gpu.js:118-140): flushes the stream, then device -> host */
p0_status p0_read(p0_ctx *ctx, p0_buf buf, size_t off, size_t n, void *dst);
/* Gpu.free (gpu.js:89-94) */
p0_status p0_free(p0_ctx *ctx, p0_buf buf);
/* Gpu.done (gpu.js:141-147): wait for the stream with a bound; reports in-kernel wait timeouts */
p0_status p0_done(p0_ctx *ctx, uint32_t timeout_ms);
/* the device address of a buffer (for NCCL / interop); the address is valid until p0_free. No counterpart in the
 * reference (WebGPU hides buffer addresses). */
p0_status p0_device_ptr(p0_ctx *ctx, p0_buf buf, uint64_t *out);

/* a weight tensor view: WeightStore h.t(name) -> {buf, off (bytes), bytes, enc, rows, cols} (core/store.js:249-253) */
typedef struct {
  p0_buf buf;
  uint64_t off;    /* bytes */
  uint64_t bytes;  /* 0 = to the end of the buffer */
  uint32_t enc;    /* P0_ENC_* */
  uint32_t rows;   /* Nw */
  uint32_t cols;   /* Ktot (for f16: also the row stride in halves unless ld is set) */
  uint32_t ld;     /* f16 only: row stride in halves (0 = cols) */
} p0_wview;

/* ---------------------------------------------------------------------------------------------- GEMV */
enum { P0_PRO_RAW = 0, P0_PRO_RMS = 1, P0_PRO_SUM = 2, P0_PRO_PLEG = 3 };
enum { P0_EPI_STORE = 0, P0_EPI_GEGLU = 1, P0_EPI_SOFTCAP = 2 };

/* gemv(g, a) -> nsplit (engine/llm/lops.js:108-141): y = x W^T for one token.
 * Fields mirror `a`: w; x {buf, rowB}; N; K; kPer (0 = none); pro; epi; y {buf}; ldy (0 = N); stat {buf, off}
 * (rms rstd slot; bound as in lops.js:125: the mx buffer when epi is softcap); norm {buf, off}; ev {buf, off};
 * src {n, ld} (sum / pleg partials); mx {buf}; cap (0 = 30). Output contract: store -> Y[split*ldy + n];
 * geglu -> Y[n] = gelu(gate n) * up n (W rows [gate 0..N) | up N..2N)); softcap -> Y[n] and MX[tile*2] =
 * {max, bitcast idx} per 64-row tile, ties to the lowest index. */
typedef struct {
  p0_wview w;
  p0_buf x;    uint32_t x_rowB;
  uint32_t N, K, kPer;
  uint32_t pro, epi;
  p0_buf y;    uint32_t ldy;
  p0_buf stat; uint32_t stat_off;
  p0_buf norm; uint32_t norm_off;
  p0_buf ev;   uint32_t ev_off;
  uint32_t src_n, src_ld;
  p0_buf mx;
  float cap;
} p0_gemv_args;
p0_status p0_gemv(p0_ctx *ctx, const p0_gemv_args *a, uint32_t *nsplit);

/* gemvM(g, a) -> nsplit (engine/llm/lops_spec.js:159-191): M <= 8 rows at once, each weight record read once.
 * Adds x.ldx (0 = K), y.ldm (0 = N) and y.ldy (0 = M*ldm), stat.ld (0 = 2), ev.ld. Prologues raw | rms | pleg.
 * store -> Y[split*ldy + m*ldm + n]; softcap -> MX[(m*ntile + tile)*2], ntile = N/64. */
typedef struct {
  p0_wview w;
  p0_buf x;    uint32_t x_rowB, x_ldx;
  uint32_t M, N, K, kPer;
  uint32_t pro, epi;
  p0_buf y;    uint32_t ldy, ldm;
  p0_buf stat; uint32_t stat_off, stat_ld;
  p0_buf norm; uint32_t norm_off;
  p0_buf ev;   uint32_t ev_off, ev_ld;
  uint32_t src_n, src_ld;
  p0_buf mx;
  float cap;
} p0_gemvM_args;
p0_status p0_gemvM(p0_ctx *ctx, const p0_gemvM_args *a, uint32_t *nsplit);

/* gemvM without any device allocation. No counterpart in the reference (its WebGPU runtime has no such constraint).
 * Same arguments, checks, outputs and error messages as p0_gemvM, always computed by the stream-K GEMV kernel.
 * p0_gemvM keeps that kernel's counters and partial sums in a context workspace that it allocates on first use and
 * re-allocates (cudaFree, which waits for the whole device, then cudaMalloc) when a larger call needs more. Callers
 * that cannot allocate device memory in the middle of their work use this entry point instead: a decode loop with a
 * latency budget that a device-wide wait would break, or a process whose device memory is all owned by another
 * allocator (for example a framework's caching allocator that has reserved the HBM). The scratch lives in a
 * file-scope device array of P0_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until the process
 * exits: P0_NOALLOC_COUNTER_BYTES of per-unit arrival counters (one u32 per 64-row tile x k-split; zero at load, and
 * every call's kernel returns each counter it uses to zero before it exits, also when one of its waits gives up), then
 * the partial sums ((tiles x splits + warps of the grid) x halves x M x 64 floats, halves = 2 for geglu). A call that needs more returns P0_EINVAL and says how much; so does a call the stream-K kernel does
 * not take (geglu with k-splits, weight columns < K, M*K > 16384, fewer than 16 weight records).
 * The first call on each device looks up the array's device address and keeps it for the life of the process; make
 * that first call before any stream capture, and do not reset the device (cudaDeviceReset) after it: a new primary
 * context would leave the kept address stale. Every call on a device shares the one array and keeps the last call's contents: calls whose kernels can
 * overlap on the GPU (other streams, contexts or threads on the same device) race and give wrong results. */
#define P0_NOALLOC_SCRATCH_BYTES (16u << 20)
#define P0_NOALLOC_COUNTER_BYTES (64u << 10)
p0_status p0_gemvM_noalloc(p0_ctx *ctx, const p0_gemvM_args *a, uint32_t *nsplit);

/* ---------------------------------------------------------------------------------------------- recorded chains */
/* The decode loop's dispatch recorder (DecodeRunner, engine/llm/drunner.js:1-8, begin :36): between p0_chain_begin and
 * p0_chain_end every p0_gemv / p0_gemvM call on the context is checked exactly as it would be (same statuses and
 * messages) and recorded instead of launched; p0_chain_run enqueues the recorded calls on the context's stream, in
 * order, with the results they would have had one by one (within the GEMV tolerance: partial sums combine in another
 * order). Runs of q4 calls with the chain's M (the M of its first q4 call), K per split <= 2048 and at most 4 x SMs
 * output units run as ONE cooperative kernel: each output unit (64-row tile x k-split) is computed whole by one CTA,
 * units dealt round-robin over the SMs across calls; every warp streams its share of its CTA's records through a ring
 * of bulk copies that runs on across calls, and a grid barrier sits only before a call that reads what earlier calls
 * of the kernel wrote (or writes what they read or wrote), by the byte ranges each call binds. Other calls (the
 * vocabulary head, q8 weights) run between them on their own kernels. p0_chain_end allocates the chain's device state
 * (descriptors, barrier words); p0_chain_run allocates nothing. The chain keeps the device addresses of every
 * buffer its calls bound, so those buffers must outlive it, and the weights must not change while a run is in flight
 * (they are fetched ahead of the barriers). Runs of one chain on one stream are ordered; two runs of one chain must
 * not overlap on the GPU (they share the counters). A barrier wait that runs out sets the context's error word
 * (p0_done reports P0_ETIMEOUT). p0_chain_info reports the recorded calls, those the chain kernel takes, the launches
 * of a run and the grid barriers. */
typedef struct p0_chain p0_chain;
p0_status p0_chain_begin(p0_ctx *ctx);
p0_status p0_chain_end(p0_ctx *ctx, p0_chain **out);
p0_status p0_chain_run(p0_ctx *ctx, p0_chain *chain);
p0_status p0_chain_info(p0_ctx *ctx, const p0_chain *chain, uint32_t *calls, uint32_t *kernel_calls, uint32_t *launches,
                        uint32_t *barriers);
p0_status p0_chain_free(p0_ctx *ctx, p0_chain *chain);

/* ---------------------------------------------------------------------------------------------- GEMM */
enum { P0_GEPI_F16 = 0, P0_GEPI_F32 = 1, P0_GEPI_BIAS = 2, P0_GEPI_RESADD = 3, P0_GEPI_SWIGLU = 4, P0_GEPI_HEADS = 5, P0_GEPI_ONORMGATE = 6 };
enum { P0_ACT_SILU = 0, P0_ACT_GELU = 1 };

/* gemm(gpu, a) -> flops (engine/ops/gemm.js:255-322): Y[m, n] = sum_k X[m, k] * W[n, k], W dequantised in-kernel
 * to fp16 (q4: f16(q*s + mn), gemm.js:147-148; q8: f16(q*s); f16 weights as they are, rows of w.ld halves, ld % 8 and
 * wk0 % 8 for 16-byte row reads), fp32 accumulation on the tensor cores.
 * Fields mirror `a`: w; x {buf, off (bytes), ld (halves, 0 = K), k0}; M, N, K; wr0, wr1, wk0; epi; act;
 * y {buf, off (bytes), ld (0 = N), n0}; ev {buf, off (floats)} (bias vector for 'bias', gate for 'resadd');
 * bv {buf, off (floats), up} (resadd / swiglu bias); res; store.
 * post_gelu (bias epilogue only) applies engine/ops/misc.js ew op 'gelu' to the fp16 result in the same pass:
 * the pair gemm(epi:'bias') -> ew(op:'gelu') of pocketflux-engine.js:3052-3053 as one call.
 * acc: 0 = 'f32', 1 = 'f16' (gemm.js:172-183: fp16 partial sums over each 32-k tile, folded into f32; the default of
 * the DiT's calls, pocketflux-engine.js:4095). Both compute on the tensor cores with every product accumulated in f32:
 * the 'f16' mode's results are the f32 ones, closer to the exact sum than the reference's fp16 partials (whose extra
 * rounding error is up to about 2^-11 of each 32-term partial's magnitude).
 * The f32 x prologues run as a pass that writes the fp16 X into the context's workspace (M*K*2 bytes), then the GEMM.
 * A call whose grid fills at most half the SMs (few tokens and few weight rows), with at least 16 k-stages and a store
 * epilogue (f16 / bias / f32 / resadd), splits K: the splits' f32 partial products go to the same workspace (S*M*N*4 bytes,
 * S <= 8, after the prologue's X), and a second pass sums them in split order and applies the epilogue. A call that
 * has to grow the workspace waits for the context's stream first (as the x prologues do), so the first such call of a
 * size should not sit inside a stream capture. */
typedef struct {
  p0_wview w;
  p0_buf x;  uint64_t x_off; uint32_t x_ld, x_k0;
  uint32_t M, N, K;
  uint32_t wr0, wr1, wk0;
  uint32_t epi, act, acc;
  p0_buf y;  uint64_t y_off; uint32_t y_ld, y_n0;
  p0_buf ev; uint32_t ev_off;
  p0_buf bv; uint32_t bv_off, bv_up;
  uint32_t res, store, post_gelu;
  /* x prologue (gemm.js:55-63): P0_XPRO_F16 (x fp16, the default), or an f32 x turned into fp16 per element:
   * P0_XPRO_LNMOD f16(((x - mean) * rstd) * (1 + pv[k]) + pv[pv_stride + k]), P0_XPRO_RMS f16((x * rstd) * pv[k]), with
   * {mean, rstd} = stats[(stats_off + m) * 2 ..] (rows of ops/misc.js rowstats) and k counted from x.k0; x.ld in floats */
  uint32_t x_mode;
  p0_buf stats; uint32_t stats_off;
  p0_buf pv;    uint32_t pv_off, pv_stride;
  /* epilogues that reduce over one 128-wide head (gemm.js:212-250; N % 128 == 0, head hd = column / 128), fields of
   * a.heads {Ltot, Hq, Hkv, rowOff, eps (0 = 1e-6), ropeMode, rope} and a.gt; inv = 1/sqrt(sum of the head's 128 squared
   * accumulators / 128 + eps), c = column % 128:
   * P0_GEPI_HEADS (QK-RMSNorm + RoPE + head-major write): heads hd < Hq are q, hd < Hq + Hkv k, the rest v. q / k:
   *   v = a * inv * ev[ev_off + (k ? 128 : 0) + c], rotated by the (cos, sin) pairs of rope row rowOff + m (128 f32 per
   *   row): P0_ROPE_HALF pairs dims (d, d + 64) with pair d (rotate_half), P0_ROPE_INTER pairs (2p, 2p + 1) with pair p.
   *   v heads: the accumulator. Y fp16 head-major: Y[((hd * Ltot) + rowOff + m) * 128 + c]; y.ld and y.n0 unused.
   * P0_GEPI_ONORMGATE: Y[m * ld + n0 + n] = f16(a * inv * ev[ev_off + c] / (1 + exp(-gt[m * Ltot + n0 + n]))), gt fp16.
   * rope and gt are read from the start of their buffers, as the reference binds them whole. */
  uint32_t h_Ltot, h_Hq, h_Hkv, h_rowOff;
  float h_eps;
  uint32_t h_rope_mode;
  p0_buf rope;
  p0_buf gt;
} p0_gemm_args;
enum { P0_XPRO_F16 = 0, P0_XPRO_LNMOD = 1, P0_XPRO_RMS = 2 };
enum { P0_ROPE_INTER = 0, P0_ROPE_HALF = 1 };
p0_status p0_gemm(p0_ctx *ctx, const p0_gemm_args *a, double *flops);

/* ---------------------------------------------------------------------------------------------- decode-path operators */
/* argmax(g, a) (engine/llm/lops.js:416-436) / argmaxM(g, a) (lops_spec.js:326-348): for each of M rows of n
 * (max, bitcast index) pairs, mx f32 [M][n][2] (the GEMV's softcap MX), out[2m] = the index of the largest max (ties:
 * the lowest index; NaN maxima never win; none: 0xffffffff with -3.4e38), out[2m + 1] = the bits of that max.
 * argmax is M = 1. Both buffers are read from their start, as the reference binds them. */
p0_status p0_argmaxM(p0_ctx *ctx, p0_buf mx, uint32_t n, uint32_t M, p0_buf out);

/* embed(g, a) (lops.js:323-365): x[(rowOut + m) * K + k] = dequant(E[ids[m]])[k] * scale for m < n, E a q4g32a.t64 /
 * q8g64s.t64 table view [rows][K] (the lm_head's records); st[st_off + m] = 1 / sqrt(sum_k x^2 / K + eps) (eps 0 =
 * 1e-6). ids, x and st are read from their start (st_off in floats). An id >= w.rows reads as a row of zeros. */
typedef struct {
  p0_wview w;
  p0_buf ids, x, st;
  uint32_t st_off, K, n, rowOut;
  float scale, eps;
} p0_embed_args;
p0_status p0_embed(p0_ctx *ctx, const p0_embed_args *a);

/* normadd(g, a) (lops.js:143-180): for rows m < M (0 = 1) of D: tv = the sum of the t_n (0 = 1) partial rows
 * t[j * t_ld + m * D + i] (t_ld floats, 0 = D * M); mode 0: x = (x + tv * rsqrt(mean tv^2 + eps) * w[w_off + i]) *
 * scale, mode 1: x = tv; st[st_off + m] = rsqrt(mean x^2 + eps). eps 0 = 1e-6; scale has no default here (the
 * reference's is 1). Buffers from their start; D * 4 bytes <= 200 KB. */
typedef struct {
  p0_buf t; uint32_t t_n, t_ld;
  p0_buf w; uint32_t w_off;
  p0_buf x, st; uint32_t st_off;
  uint32_t D, M, mode;
  float eps, scale;
} p0_normadd_args;
p0_status p0_normadd(p0_ctx *ctx, const p0_normadd_args *a);

/* dhead(g, a) (lops_spec.js:428-482): the drafter's head over selected clusters. Block b < nsel * tPer scores tile
 * sel[b / tPer] * tPer + b % tPer of a q4 / q8 head view [rows][K] (K <= 512) against x * stat[stat_off] *
 * norm[norm_off + k]: mx[2b] = the tile's largest row dot, mx[2b + 1] = bitcast(tile * 64 + row) (lowest row on
 * ties). A tile beyond the head gives (-3.4e38, 0xffffffff). x, stat, norm, sel, mx from their start. */
typedef struct {
  p0_wview w;
  p0_buf x, stat; uint32_t stat_off;
  p0_buf norm; uint32_t norm_off;
  p0_buf sel, mx;
  uint32_t K, tPer, nsel;
} p0_dhead_args;
p0_status p0_dhead(p0_ctx *ctx, const p0_dhead_args *a);

/* qkrope(g, a) (lops.js:183-233), one decode token: heads of s (the sum of s_n (0 = 1) partial rows of s_ld floats,
 * 0 = (nq + 2 nkv) * D) laid out [q (nq heads) | k (nkv) | v (nkv)] of D each (k and v only when hasKV).
 * rs = rsqrt(mean square + eps) (eps 0 = 1e-6). v: vc[(kvh * kvLen + kvRow) * D + i] = f16(x * rs). q / k: a = x[d] rs
 * norm[w + d], b = x[d + D/2] rs norm[w + d + D/2] (w = qw or kw), rotated by (cos, sin) = rope[rope_off + (pos *
 * npairs + d) * 2 ..] for d < npairs (else unrotated): q -> q[h * D + d], q[h * D + d + D/2] (f32); k -> kc (fp16,
 * head-major [nkv][kvLen][D], row kvRow). Buffers from their start. */
typedef struct {
  p0_buf s; uint32_t s_n, s_ld;
  p0_buf norm; uint32_t qw, kw;
  p0_buf rope; uint32_t rope_off, npairs, pos;
  p0_buf q, kc, vc;
  uint32_t D, nq, nkv, hasKV, kvRow, kvLen;
  float eps;
} p0_qkrope_args;
p0_status p0_qkrope(p0_ctx *ctx, const p0_qkrope_args *a);

/* attnDec(g, a) + its combine (lops.js:236-321): decode attention of nh <= 8 query heads (q f32 [nh][D], D % 128 == 0,
 * D <= 512) over keys [kStart, kEnd) of the fp16 caches kc / vc (head-major [nkv][kvLen][D]; query head h reads KV
 * head h / (nh / nkv); key j is row j % ring when ring > 0), in chunks of 64 keys (at most 256 chunks): softmax(q . k)
 * . v per head, no score scale -> out f32 [nh][D]. part: scratch of >= nchunk * nh * (2 + D) floats. */
typedef struct {
  p0_buf q, kc, vc, part, out;
  uint32_t D, nh, nkv, kvLen, kStart, kEnd, ring;
} p0_attn_dec_args;
p0_status p0_attn_dec(p0_ctx *ctx, const p0_attn_dec_args *a);

/* ---------------------------------------------------------------------------------------------- quantiser */
/* packQ4 (engine/kcheck.js:22-38) on the device, bit for bit: W f32 [N][ldw] at w_off (bytes) -> q4g32a.t64 records
 * (N*K*5/8 bytes) at out_off. N % 64 == 0, K % 32 == 0. The dequantised value of code q is q*s + mn. */
p0_status p0_pack_q4(p0_ctx *ctx, p0_buf w, uint64_t w_off, uint32_t ldw, uint32_t N, uint32_t K, p0_buf out, uint64_t out_off);

/* packQ8 (engine/kcheck.js:39-52) on the device, bit for bit: W f32 [N][ldw] -> q8g64s.t64 records (N*K*66/64 bytes:
 * 64 rows x 64 int8 codes + 64 fp16 scales per record). N % 64 == 0, K % 64 == 0. The dequantised value is q*s. */
p0_status p0_pack_q8(p0_ctx *ctx, p0_buf w, uint64_t w_off, uint32_t ldw, uint32_t N, uint32_t K, p0_buf out, uint64_t out_off);

/* ---------------------------------------------------------------------------------------------- testing aids */
/* writes the fp16 weight the GEMM tile holds for rows [0, rows) x k [0, cols) of a q4/q8 view, row-major,
 * into out_f16 (a buffer of rows*cols*2 bytes): the in-kernel dequantisation (gemm.js:139-160), dumped for bit-exact
 * checks; no entry point of its own in the reference */
p0_status p0_dequant_f16(p0_ctx *ctx, const p0_wview *w, p0_buf out_f16);
/* failure-path check, no counterpart in the reference: enqueues one small kernel whose warp waits on an mbarrier
 * phase that nothing completes, through the same bounded in-kernel wait as the matmul kernels, giving up after `polls`
 * tries (1 .. 2^20). It records its code (0x7e1) in the context's error word and returns, so the next p0_done reports
 * P0_ETIMEOUT (the reference's GpuError at done(), core/gpu.js:141-147) and the context stays usable. */
p0_status p0_wait_selftest(p0_ctx *ctx, uint32_t polls);
/* the library build tag (kernel versions), e.g. "p0mm sm_100a gemv-v1 gemm-tc-v1"; no counterpart in the reference */
const char *p0_version(void);

#ifdef __cplusplus
}
#endif
#endif /* P0MM_H */
