/*
 * tforge.h -- C-ABI of the B200 (sm_100a) TensorForge operator library.
 *
 * Drop-in for the kernel that TensorForge's `--tforge-gpu-pipeline` generates and that
 * runners/gpu/tforge-gpu-bench.cu launches with cuLaunchKernel. The argument order is
 * the MLIR host entry's out-param order, `entry(A, B, bias, out)`:
 *   matmul:   A (M x K), B (K x N), out (M x N)            runners/gpu/tforge-gpu-bench.cu:20-24
 *   mbr:      A, B, bias (N), out                          runners/gpu/tforge-gpu-bench.cu:209-213
 *   bias_add: X (M x N), bias (N), Y                       python/tforge_cpu.py:3-8
 *   relu:     X, Y
 * All tensors are row-major contiguous f32 in device memory, owned by the caller,
 * distinct and non-overlapping (the reference marks every kernel pointer `noalias`,
 * lib/Transforms/Gpu.cpp:453-457). The library allocates no input or output buffers
 * and never copies them. Every call is asynchronous on `stream` (a cudaStream_t; NULL
 * is the legacy default stream) and returns a status code; it never exits the process
 * (the reference runner's die() + exit(1), tforge-gpu-bench.cu:52-70, becomes a code).
 *
 * Op semantics (include/TensorForge/Dialect/TForge/TForgeOps.td:37-113):
 *   matmul   C[m,n] = sum_k A[m,k] * B[k,n], accumulator starts at +0.0, K order unspecified
 *   bias_add Y[m,n] = X[m,n] + bias[n]            (one IEEE add)
 *   relu     Y = maximum(X, +0.0)                  (IEEE-2019: NaN -> NaN, -0.0 -> +0.0)
 *   add      Z = X + Y                             (one IEEE add)
 *   mbr      relu(bias_add(matmul(A, B), bias))    fused in one kernel
 *   matmul_add  matmul(A, B) + C_res               fused in one kernel
 */
#ifndef TFORGE_H
#define TFORGE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
enum tforge_status {
  TFORGE_OK = 0,
  TFORGE_ERR_SHAPE = 1,       /* M, N or K negative, or a pitch smaller than its row */
  TFORGE_ERR_ALIGN = 2,       /* a pointer not 4-byte aligned (f32) */
  TFORGE_ERR_ALIAS = 3,       /* the output overlaps an input */
  TFORGE_ERR_MODE = 4,        /* unknown precision mode or workload */
  TFORGE_ERR_CUDA = 5,        /* a CUDA runtime/driver call failed; see tforge_last_error() */
  TFORGE_ERR_TIMEOUT = 6,     /* a bounded device-side wait expired (reported by tforge_device_status) */
  TFORGE_ERR_NULL = 7,        /* a required pointer is NULL */
  TFORGE_ERR_UNSUPPORTED = 8, /* no kernel for this combination (e.g. a forced config that cannot run) */
  TFORGE_ERR_NOMEM = 9        /* the library's own workspace could not be allocated */
};

/* Precision modes of the GEMM kernels. */
enum tforge_mode {
  TFORGE_MODE_FP32 = 0,       /* fp32-accurate: 3xTF32 split products on tcgen05 (default) */
  TFORGE_MODE_TF32 = 1,       /* one TF32 product on tcgen05 (inputs rounded to 10-bit mantissa) */
  TFORGE_MODE_BF16 = 2,       /* inputs rounded to bf16, fp32 accumulation on tcgen05 */
  TFORGE_MODE_FP32_EXACT = 3  /* SIMT FFMA, sequential k from +0.0: bitwise equal to the reference's
                                 generated kernels (docs/numerics.md:3,53) */
};

/* Workloads (python/tforge_cpu.py:3-8 plus matmul_add). */
enum tforge_workload {
  TFORGE_MATMUL = 0,
  TFORGE_MBR = 1,
  TFORGE_MATMUL_ADD = 2,
  TFORGE_BIAS_ADD = 3,
  TFORGE_RELU = 4,
  TFORGE_ADD = 5
};

/* Element types accepted for A and B by tforge_gemm. */
enum tforge_dtype { TFORGE_F32 = 0, TFORGE_BF16 = 1 };

/* Fused GEMM.  out = epilogue(A @ B).  Replaces the generated `entry_kernel` of the
 * tforge-gpu-pipeline (lib/Transforms/Gpu.cpp:219-316) launched at
 * runners/gpu/tforge-gpu-bench.cu:292-302.  Pitches are in elements; 0 means packed
 * (lda = K, ldb = N, ldc = N; C_res shares ldc).  BF16 A/B are accepted only in
 * TFORGE_MODE_BF16 (inputs already converted, e.g. a weight converted once).
 * out_dtype TFORGE_BF16 (TFORGE_MODE_BF16 only; not in tforge_gemm_host): out holds M x N
 * bf16 values, the f32 results rounded to nearest even -- the same values tforge_convert_bf16
 * of the f32 output gives, written without the f32 round trip (a hidden layer feeding a
 * BF16-mode layer, e.g. the MLP chain's H). */
typedef struct tforge_gemm_args {
  int32_t workload;      /* TFORGE_MATMUL, TFORGE_MBR or TFORGE_MATMUL_ADD */
  int32_t mode;          /* enum tforge_mode */
  int32_t a_dtype;       /* enum tforge_dtype */
  int32_t b_dtype;       /* enum tforge_dtype */
  const void *A;         /* M x K */
  const void *B;         /* K x N */
  const float *bias;     /* N        (mbr) */
  const float *C_res;    /* M x N    (matmul_add) */
  void *out;             /* M x N, f32 (or bf16, see out_dtype) */
  int64_t M, N, K;
  int64_t lda, ldb, ldc;
  int32_t out_dtype;     /* enum tforge_dtype; 0 = TFORGE_F32 */
} tforge_gemm_args;

int tforge_gemm(const tforge_gemm_args *args, void *stream);

/* tforge_gemm on HOST buffers: args->A, B, bias / C_res and out are host pointers (pitches as in
 * tforge_gemm).  Replaces the GPU runner's host flow -- cudaMalloc, cudaMemcpy of A, B and bias
 * to the device, the launch, cudaMemcpy of C back (runners/gpu/tforge-gpu-bench.cu:198-207,
 * 292-302,327) -- with an overlapped one: device staging comes from the library's pool; B and
 * bias are copied first, then A (and C_res) in chunks of `chunk_rows` rows (0: automatic, at
 * most 8 chunks of at least 512 rows); each chunk's kernel starts on its own stream once its
 * rows have landed, and each chunk of out is copied back while later chunks compute.
 * Asynchronous with respect to the host: out is complete once `stream` has synchronized.  Copies overlap only
 * with page-locked host memory; pageable memory gives the same results without overlap.
 * Results equal tforge_gemm's on each chunk of rows (the kernel is chosen per chunk). */
int tforge_gemm_host(const tforge_gemm_args *args, int64_t chunk_rows, void *stream);

/* The three operator entries, in the reference's host-entry argument order. */
int tforge_matmul(const float *A, const float *B, float *out, int64_t M, int64_t N, int64_t K,
                  int mode, void *stream);
int tforge_mbr(const float *A, const float *B, const float *bias, float *out, int64_t M, int64_t N,
               int64_t K, int mode, void *stream);
int tforge_matmul_add(const float *A, const float *B, const float *C_res, float *out, int64_t M,
                      int64_t N, int64_t K, int mode, void *stream);

/* Elementwise ops, bit-exact (one IEEE operation per element): the GPU runner's
 * bias_add / relu workloads (runners/gpu/tforge-gpu-bench.cu:127-130) and the CPU
 * runner's add (runners/cpu/tforge-cpu-bench.cpp:214-219). */
int tforge_bias_add(const float *X, const float *bias, float *Y, int64_t M, int64_t N, void *stream);
int tforge_relu(const float *X, float *Y, int64_t M, int64_t N, void *stream);
int tforge_add(const float *X, const float *Y, float *Z, int64_t M, int64_t N, void *stream);

/* Round f32 to bf16 (round to nearest even), n elements: converts a weight once for
 * repeated TFORGE_MODE_BF16 calls with b_dtype = TFORGE_BF16. */
int tforge_convert_bf16(const float *x, uint16_t *y, int64_t n, void *stream);

/* relu(A @ B + bias) in TFORGE_MODE_BF16 without allocating anything.  No counterpart in
 * the reference.  For callers that must not allocate device memory during a call (a
 * serving loop that reserves all of its memory up front and cannot risk an out-of-memory
 * error or an allocator synchronisation mid-request, or a host framework that owns every
 * device byte).  The f32 -> bf16 operand copies go to a 16 MiB static device array that
 * every GPU loading this library keeps until exit: bf16(A) (rounded up to 256 bytes) plus
 * bf16(B) must fit in 16 MiB (e.g. M = N = K = 2048), else TFORGE_ERR_SHAPE.  Needs K and
 * N multiples of 8 and 16-byte-aligned pointers (else TFORGE_ERR_UNSUPPORTED /
 * TFORGE_ERR_ALIGN).  Calls share the array: calls that overlap on the GPU race.  The
 * first call on a device resolves the array's address; make it before any stream capture. */
int tforge_mbr_bf16_noalloc(const float *A, const float *B, const float *bias, float *out, int64_t M,
                            int64_t N, int64_t K, void *stream);

/* Launch description: replaces the `tforge.launch = {kernel, grid, block, args}`
 * module attribute (lib/Transforms/Gpu.cpp:449-457,572-577) that python/tforge_gpu.py
 * parses into launch.json (:42-51,88-90).  Filled for the kernel the dispatch table
 * picks for (workload, M, N, K, mode) without launching anything. */
typedef struct tforge_launch {
  char kernel[64];       /* kernel family name */
  int32_t grid[3];
  int32_t block[3];
  int32_t cluster[3];
  int32_t smem_bytes;    /* dynamic shared memory per CTA */
  int32_t tile[3];       /* BM, BN, BK (K elements per pipeline stage) */
  int32_t stages;
  int32_t tmem_cols;     /* tensor-memory columns per CTA (0 for SIMT kernels) */
  int32_t mode;          /* the precision mode that will run */
  int32_t persistent;    /* 1 if CTAs loop over tiles */
  int32_t split_k;
  int32_t regs;          /* registers per thread (-1 without a device) */
  int32_t static_smem;   /* static shared memory per CTA (-1 without a device) */
  int32_t blocks_per_sm; /* resident CTAs per SM from the occupancy API (-1 without a device) */
} tforge_launch;

int tforge_describe(int workload, int64_t M, int64_t N, int64_t K, int mode, tforge_launch *out);

/* Force a kernel configuration (offline tuning sweeps); NULL restores the table. */
typedef struct tforge_config {
  int32_t kernel;        /* 0 = table, 1 = tcgen05 one CTA per tile, 2 = SIMT, 3 = tcgen05 CTA pair */
  int32_t bn;            /* 64, 128 or 256 (one-CTA kernel); 256 or 240 (CTA pair) */
  int32_t stages;
  int32_t persistent;    /* 1 with kernel = 3: persistent CTA-pair kernel (TF32 / BF16 modes,
                            256x256 tiles, two TMEM accumulators, no split-K) */
  int32_t split_k;       /* CTA-pair kernel in fp32 / TF32 mode: 0 = automatic, 1 = no split,
                            S = 2..8 pairs per tile, each over K / S */
  int32_t b_layout;      /* TF32 mode, 256-wide pair and persistent pair kernels: 0 or 1 = B as
                            given, loaded as k-group-major tiles (one 4-D box per tile) when N is
                            a multiple of 32 and K of 4, else in 128-byte column blocks; 2 = a
                            transposed, K-major copy of B (one extra pass over B); 3 = B as given
                            in column blocks.  Every form gives the same bits. */
} tforge_config;

int tforge_set_config(const tforge_config *cfg);

/* Synchronizes `stream`, then returns and clears the current device's status words that
 * bounded waits write on expiry (TFORGE_OK or TFORGE_ERR_TIMEOUT): the one of the GEMM
 * entries and the one of tforge_mbr_bf16_noalloc.  Allocates nothing.  TFORGE_ERR_CUDA if
 * the synchronization itself failed. */
int tforge_device_status(void *stream);

/* Device-side wait limit in nanoseconds (default 1e9); 0 restores the default. */
int tforge_set_wait_limit_ns(uint64_t ns);

/* Test hook: 1 makes the next GEMM launches' producer skip its first stage's load, so
 * the consumer's bounded wait expires and reports TFORGE_ERR_TIMEOUT; 0 clears. */
int tforge_debug_skip_load(int on);

/* Test hook: bytes of the library's scratch pool in use now and the high-water mark since
 * the last reset (reset_high = 1 resets it after reading).  Creates the pool if the
 * device has none yet. */
int tforge_debug_pool_usage(uint64_t *used_now, uint64_t *used_high, int reset_high);

const char *tforge_status_string(int status);
const char *tforge_last_error(void);   /* text of the last TFORGE_ERR_CUDA, per thread */
const char *tforge_version(void);

/* Minimal device-memory helpers for callers without a CUDA binding (the ctypes shim). */
int tforge_malloc(void **ptr, uint64_t bytes);
int tforge_free(void *ptr);
int tforge_memcpy_h2d(void *dst, const void *src, uint64_t bytes, void *stream);
int tforge_memcpy_d2h(void *dst, const void *src, uint64_t bytes, void *stream);
int tforge_memset(void *dst, int byte, uint64_t bytes, void *stream);
int tforge_stream_sync(void *stream);
int tforge_device_count(int *n);
int tforge_set_device(int dev);

#ifdef __cplusplus
}
#endif

#endif /* TFORGE_H */
