// tf_noalloc.cu -- fused relu(A @ B + bias) in BF16 mode that allocates nothing.
//
// tforge_mbr in TFORGE_MODE_BF16 first rounds its f32 operands to bf16 into scratch it takes
// from a stream-ordered memory pool, so a call can allocate device memory.  Some callers
// cannot allow that: a serving loop that pre-reserves all of its device memory at start-up
// and must not see an out-of-memory failure (or an allocator's device-wide
// synchronisation) in the middle of a request, a host framework that owns every byte of
// device memory through its own allocator and forbids libraries to allocate behind its
// back, or a process whose memory is capped and fully committed.  This file gives them
// tforge_mbr_bf16_noalloc: the same conversion and the same tensor-core kernel, with the
// scratch in a file-scope device array instead of allocated memory.
//
//   * The array holds kScratchBytes (16 MiB) of bf16 operand copies plus a 256-byte tail
//     whose first word is the kernel's bounded-wait status.  Every GPU that loads this
//     library keeps the array for the lifetime of the process.
//   * A problem fits when bytes(A as bf16), rounded up to 256, plus bytes(B as bf16) is at
//     most 16 MiB, e.g. M = N = K = 2048.  Larger problems are rejected with
//     TFORGE_ERR_SHAPE and a message in tforge_last_error(); nothing is allocated instead.
//   * All calls share the array and each call overwrites it, so calls that overlap on the
//     GPU (on different streams without ordering between them) race.
//   * The kernels' bounded waits honour tforge_set_wait_limit_ns and tforge_debug_skip_load
//     like every other GEMM entry.  A wait that expires writes TFORGE_ERR_TIMEOUT into the
//     status word; tforge_device_status reports it (and clears it) with the other entries'
//     status, so a call whose output is incomplete never goes unnoticed.  The word is
//     cleared only when it is read.
//   * In host code the array's name does not denote a device address.  The first call on
//     each device resolves the address with cudaGetSymbolAddress (with that device
//     current), clears the status word and caches the address; make that first call before
//     any stream capture.
//   * No cudaMalloc, cudaFree, pool or other allocating routine is called on this path.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "tf_internal.h"
#include "tforge.h"

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;
constexpr size_t kTailBytes = 256;

__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes + kTailBytes];

constexpr int kMaxDevices = 64;
std::mutex g_addr_mu;
void *g_addr[kMaxDevices] = {};

// Device address of the static scratch on the current device (resolved once per device).
int scratch_address(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    tf::set_last_error(cudaGetErrorString(e));
    return TFORGE_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    tf::set_last_error("tforge_mbr_bf16_noalloc: device index beyond the 64 this library tracks");
    return TFORGE_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lk(g_addr_mu);
  if (!g_addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      tf::set_last_error(e != cudaSuccess ? cudaGetErrorString(e) : "cudaGetSymbolAddress returned NULL");
      return TFORGE_ERR_CUDA;
    }
    // Set-up: the status word starts at zero (cudaMemset allocates nothing).
    e = cudaMemset(static_cast<unsigned char *>(p) + kScratchBytes, 0, sizeof(uint32_t));
    if (e != cudaSuccess) {
      tf::set_last_error(cudaGetErrorString(e));
      return TFORGE_ERR_CUDA;
    }
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return TFORGE_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool overlap(const void *a, size_t an, const void *b, size_t bn) {
  const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return x < y + bn && y < x + an;
}

}  // namespace

namespace tf {

int noalloc_take_status(uint32_t *v) {
  *v = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return TFORGE_OK;
  }
  void *base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_addr_mu);
    base = g_addr[dev];
  }
  if (!base) return TFORGE_OK;  // never set up on this device: nothing can have been written
  uint32_t *w = reinterpret_cast<uint32_t *>(static_cast<unsigned char *>(base) + kScratchBytes);
  cudaError_t e = cudaMemcpy(v, w, sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && *v) e = cudaMemset(w, 0, sizeof(uint32_t));
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return TFORGE_ERR_CUDA;
  }
  return TFORGE_OK;
}

}  // namespace tf

extern "C" int tforge_mbr_bf16_noalloc(const float *A, const float *B, const float *bias, float *out,
                                       int64_t M, int64_t N, int64_t K, void *stream) {
  if (M < 0 || N < 0 || K < 0) return TFORGE_ERR_SHAPE;
  if (M == 0 || N == 0) return TFORGE_OK;
  if (!A || !B || !bias || !out) return TFORGE_ERR_NULL;
  // Only the tensor-core path: bf16 rows must be 16-byte multiples and every pointer
  // 16-byte aligned; K == 0 has no tensor-core work.
  if (K == 0 || K % 8 || N % 8) return TFORGE_ERR_UNSUPPORTED;
  if (!aligned16(A) || !aligned16(B) || !aligned16(bias) || !aligned16(out)) return TFORGE_ERR_ALIGN;
  const size_t abytes = (size_t)M * (size_t)K * 2, bbytes = (size_t)K * (size_t)N * 2;
  const size_t boff = (abytes + 255) & ~size_t(255);
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || boff + bbytes > kScratchBytes) {
    tf::set_last_error("tforge_mbr_bf16_noalloc: bf16 copies of A and B exceed the 16 MiB static scratch");
    return TFORGE_ERR_SHAPE;
  }
  const size_t ob = (size_t)M * N * 4;
  if (overlap(out, ob, A, (size_t)M * K * 4) || overlap(out, ob, B, (size_t)K * N * 4) ||
      overlap(out, ob, bias, (size_t)N * 4))
    return TFORGE_ERR_ALIAS;

  tf::TcConfig cfg{};
  if (!tf::select_tc_config(TFORGE_MODE_BF16, M, N, K, &cfg)) return TFORGE_ERR_UNSUPPORTED;
  void *base = nullptr;
  int rc = scratch_address(&base);
  if (rc) return rc;
  uint16_t *sa = static_cast<uint16_t *>(base);
  uint16_t *sb = reinterpret_cast<uint16_t *>(static_cast<unsigned char *>(base) + boff);
  uint32_t *status = reinterpret_cast<uint32_t *>(static_cast<unsigned char *>(base) + kScratchBytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  cudaError_t e = tf::launch_convert_bf16(A, sa, M * K, st);
  if (e == cudaSuccess) e = tf::launch_convert_bf16(B, sb, K * N, st);
  if (e != cudaSuccess) {
    tf::set_last_error(cudaGetErrorString(e));
    return TFORGE_ERR_CUDA;
  }
  CUtensorMap tmA, tmB;
  rc = tf::encode_operand_map(&tmA, sa, true, M, K, K, 64, 128, false);
  if (!rc) rc = tf::encode_operand_map(&tmB, sb, true, K, N, N, 64, 64, false);
  if (rc) return rc;
  tf::TcParams p{};
  p.bias = bias;
  p.cres = nullptr;
  p.out = out;
  p.M = (int32_t)M;
  p.N = (int32_t)N;
  p.K = (int32_t)K;
  p.ldc = N;
  p.status = status;
  p.limit_ns = tf::wait_limit_ns();
  p.debug_skip = tf::debug_skip_load();
  p.pdl = 1;  // the conversions above wrote A and B: the GEMM sets up while they finish
  if (cfg.pair) {
    CUtensorMap tmO;
    rc = tf::encode_operand_map(&tmO, out, false, M, N, N, 32, 128, false);
    if (rc) return rc;
    e = cfg.persist ? tf::launch_gemm_pair_persistent(cfg.prec, cfg.stages, tf::EPI_MBR, tmA, tmB, tmO, p, st)
                    : tf::launch_gemm_pair(cfg.prec, cfg.stages, cfg.bn, tf::EPI_MBR, tmA, tmB, tmO, tmO, p, st);
  } else {
    e = tf::launch_gemm_tc(cfg, tf::EPI_MBR, tmA, tmB, p, st);
  }
  if (e != cudaSuccess) {
    tf::set_last_error(cudaGetErrorString(e));
    return TFORGE_ERR_CUDA;
  }
  return TFORGE_OK;
}
