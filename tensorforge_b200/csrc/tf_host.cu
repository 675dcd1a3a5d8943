// tf_host.cu -- tforge_gemm_host: the GEMM operators on host buffers, with the host->device
// copies, the kernels and the device->host copies overlapped across streams.
//
// The reference's GPU runner moves data in three serial steps around one launch: cudaMemcpy
// of A, B and bias to the device, the kernel, cudaMemcpy of C back
// (runners/gpu/tforge-gpu-bench.cu:198-207,292-302,327).  Over PCIe the copies cost far more
// than the kernel (2048^3 fp32: 50 MB of copies against ~75 us of compute), so here:
//
//   * B (and bias) go first on a copy stream; A (and C_res) follow in row chunks.
//   * Chunk i's kernel runs on compute stream i % 4 as soon as its rows have landed (an
//     event), so kernels of neighbouring chunks overlap each other and the next copies.
//   * Chunk i's rows of out go back on a second copy stream once its kernel is done, so the
//     two PCIe directions run at the same time.
//   * In BF16 mode with f32 B, B is rounded to bf16 once on the device and every chunk reads
//     that copy.
//
// Staging memory comes from the library's stream-ordered pool on the caller's stream and is
// returned on it after the last copy, so the call never blocks the host.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>

#include "tf_internal.h"
#include "tforge.h"

namespace {

constexpr int kMaxDev = 64;
constexpr int kComputeStreams = 4;
constexpr int64_t kMaxChunks = 64;
constexpr int64_t kAutoChunks = 8;

struct HostCtx {
  std::mutex mu;
  bool ready = false;
  cudaStream_t h2d = nullptr, d2h = nullptr, comp[kComputeStreams] = {};
  cudaEvent_t start = nullptr, done = nullptr, join[kComputeStreams + 1] = {};
  cudaEvent_t landed[kMaxChunks] = {}, computed[kMaxChunks] = {};
};
HostCtx g_ctx[kMaxDev];

int fail(cudaError_t e, const char *what) {
  const std::string msg = std::string(what) + ": " + cudaGetErrorString(e);
  tf::set_last_error(msg.c_str());
  return TFORGE_ERR_CUDA;
}

// Streams and events of the current device, created on first use (caller holds ctx.mu).
int init_ctx(HostCtx &c) {
  if (c.ready) return TFORGE_OK;
  cudaError_t e = cudaStreamCreateWithFlags(&c.h2d, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c.d2h, cudaStreamNonBlocking);
  for (int i = 0; i < kComputeStreams && e == cudaSuccess; ++i)
    e = cudaStreamCreateWithFlags(&c.comp[i], cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c.start, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c.done, cudaEventDisableTiming);
  for (int j = 0; j <= kComputeStreams && e == cudaSuccess; ++j)
    e = cudaEventCreateWithFlags(&c.join[j], cudaEventDisableTiming);
  for (int64_t i = 0; i < kMaxChunks && e == cudaSuccess; ++i) {
    e = cudaEventCreateWithFlags(&c.landed[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c.computed[i], cudaEventDisableTiming);
  }
  if (e != cudaSuccess) return fail(e, "tforge_gemm_host: stream/event creation");
  c.ready = true;
  return TFORGE_OK;
}

size_t round256(size_t b) { return (b + 255) & ~size_t(255); }

}  // namespace

extern "C" int tforge_gemm_host(const tforge_gemm_args *a, int64_t chunk_rows, void *stream) {
  int64_t lda, ldb, ldc;
  int rc = tf::check_gemm_args(a, &lda, &ldb, &ldc);
  if (rc) return rc;
  if (a->out_dtype != TFORGE_F32) return TFORGE_ERR_MODE;  // host buffers: f32 output only
  if (a->M == 0 || a->N == 0) return TFORGE_OK;
  const int64_t M = a->M, N = a->N, K = a->K;
  const size_t ea = a->a_dtype == TFORGE_BF16 ? 2 : 4, eb = a->b_dtype == TFORGE_BF16 ? 2 : 4;
  const bool mbr = a->workload == TFORGE_MBR, add = a->workload == TFORGE_MATMUL_ADD;
  const bool b16 = a->mode == TFORGE_MODE_BF16 && a->b_dtype == TFORGE_F32 && K > 0 && N % 8 == 0;

  // Rows per chunk: automatic = at most 8 chunks of a multiple of 128 rows, at least 512
  // rows each (a chunk's kernel costs the whole K loop however few rows it has; 2048^3 on a
  // B200: 512-row chunks 0.85 ms, 256-row 0.88, 1024-row 0.89); never more than 64 chunks.
  int64_t rows = chunk_rows;
  if (rows <= 0) {
    const int64_t chunks = std::min(kAutoChunks, std::max<int64_t>(1, M / 512));
    rows = ((M + chunks - 1) / chunks + 127) / 128 * 128;
  }
  rows = std::max(rows, (M + kMaxChunks - 1) / kMaxChunks);
  const int64_t nchunks = (M + rows - 1) / rows;

  // Device staging: B [, B as bf16], bias, A, C_res, out -- contiguous rows, 256-aligned.
  const size_t oB = 0, oB16 = oB + round256((size_t)K * N * eb);
  const size_t oBias = oB16 + (b16 ? round256((size_t)K * N * 2) : 0);
  const size_t oA = oBias + (mbr ? round256((size_t)N * 4) : 0);
  const size_t oC = oA + round256((size_t)M * K * ea);
  const size_t oOut = oC + (add ? round256((size_t)M * N * 4) : 0);
  const size_t total = oOut + round256((size_t)M * N * 4);

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDev) return TFORGE_ERR_UNSUPPORTED;
  HostCtx &c = g_ctx[dev];
  std::lock_guard<std::mutex> lk(c.mu);
  rc = init_ctx(c);
  if (rc) return rc;
  cudaMemPool_t pool = nullptr;
  rc = tf::device_pool(&pool);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char *base = nullptr;
  e = cudaMallocFromPoolAsync(reinterpret_cast<void **>(&base), total, pool, st);
  if (e != cudaSuccess) return fail(e, "tforge_gemm_host: staging allocation");

  // Everything below is ordered after the caller's earlier work and the allocation.
  e = cudaEventRecord(c.start, st);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(c.h2d, c.start, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(c.d2h, c.start, 0);
  const char *hA = static_cast<const char *>(a->A), *hB = static_cast<const char *>(a->B);
  if (e == cudaSuccess && K > 0)
    e = cudaMemcpy2DAsync(base + oB, N * eb, hB, ldb * eb, N * eb, K, cudaMemcpyHostToDevice, c.h2d);
  if (e == cudaSuccess && b16)
    e = tf::launch_convert_bf16(reinterpret_cast<const float *>(base + oB),
                                reinterpret_cast<uint16_t *>(base + oB16), K * N, c.h2d);
  if (e == cudaSuccess && mbr) e = cudaMemcpyAsync(base + oBias, a->bias, N * 4, cudaMemcpyHostToDevice, c.h2d);
  if (e != cudaSuccess) rc = fail(e, "tforge_gemm_host: B/bias staging");

  for (int64_t i = 0; i < nchunks && rc == TFORGE_OK; ++i) {
    const int64_t r0 = i * rows, nr = std::min(rows, M - r0);
    if (K > 0)
      e = cudaMemcpy2DAsync(base + oA + (size_t)r0 * K * ea, K * ea, hA + (size_t)r0 * lda * ea, lda * ea,
                            K * ea, nr, cudaMemcpyHostToDevice, c.h2d);
    if (e == cudaSuccess && add)
      e = cudaMemcpy2DAsync(base + oC + (size_t)r0 * N * 4, N * 4, a->C_res + (size_t)r0 * ldc, ldc * 4, N * 4,
                            nr, cudaMemcpyHostToDevice, c.h2d);
    if (e == cudaSuccess) e = cudaEventRecord(c.landed[i], c.h2d);
    cudaStream_t cs = c.comp[i % kComputeStreams];
    if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, c.landed[i], 0);
    if (e != cudaSuccess) {
      rc = fail(e, "tforge_gemm_host: A staging");
      break;
    }
    tforge_gemm_args g = *a;
    g.A = base + oA + (size_t)r0 * K * ea;
    g.B = b16 ? static_cast<const void *>(base + oB16) : static_cast<const void *>(base + oB);
    g.b_dtype = b16 ? TFORGE_BF16 : a->b_dtype;
    g.bias = mbr ? reinterpret_cast<const float *>(base + oBias) : nullptr;
    g.C_res = add ? reinterpret_cast<const float *>(base + oC) + r0 * N : nullptr;
    g.out = reinterpret_cast<float *>(base + oOut) + r0 * N;
    g.M = nr;
    g.lda = K;
    g.ldb = N;
    g.ldc = N;
    rc = tforge_gemm(&g, cs);
    if (rc) break;
    e = cudaEventRecord(c.computed[i], cs);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(c.d2h, c.computed[i], 0);
    if (e == cudaSuccess)
      e = cudaMemcpy2DAsync(static_cast<float *>(a->out) + (size_t)r0 * ldc, ldc * 4, base + oOut + (size_t)r0 * N * 4, N * 4, N * 4,
                            nr, cudaMemcpyDeviceToHost, c.d2h);
    if (e != cudaSuccess) rc = fail(e, "tforge_gemm_host: out copy-back");
  }
  // Join: the copy-back stream waits for the copy stream and every compute stream (which
  // covers the chunks that were enqueued before a failure), the caller's stream waits for
  // the copy-back stream, and the staging then returns to the pool on the caller's stream.
  for (int j = 0; j <= kComputeStreams; ++j) {
    cudaStream_t s = j < kComputeStreams ? c.comp[j] : c.h2d;
    if (cudaEventRecord(c.join[j], s) == cudaSuccess) cudaStreamWaitEvent(c.d2h, c.join[j], 0);
  }
  e = cudaEventRecord(c.done, c.d2h);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(st, c.done, 0);
  if (e != cudaSuccess && rc == TFORGE_OK) rc = fail(e, "tforge_gemm_host: join");
  cudaFreeAsync(base, st);
  return rc;
}
