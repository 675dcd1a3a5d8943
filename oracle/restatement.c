/*
 * oracle/restatement.c -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * CPU restatement of TensorForge's CPU kernel for the fused dense layer
 * relu(A @ B + bias) and its siblings, written from the reference's pass
 * pipeline and numerics study:
 *
 *   - lib/Pipelines/Pipelines.cpp:47-121  `--tforge-cpu-pipeline` with
 *     `fuse-elementwise=1 reg-tile=6,16,4 vectorize=1` (the BASELINE CPU config).
 *   - lib/Transforms/TileAndFuse.cpp:133-231  M and N tiled by 6 x 16, K by 4,
 *     every loop peeled so full tiles have static shapes; the epilogue is fused
 *     into the producer's init (EpilogueIntoProducerInit, :78-131), so no M x N
 *     temporary exists.
 *   - lib/Transforms/Vectorize.cpp:43-81, docs/stage6.md:9-18,81-103  the
 *     accumulator is a 6x16 vector started at +0.0 (TForgeToLinalg.cpp:31-35)
 *     and updated by one FMA per k, in sequential k order.
 *   - include/TensorForge/Dialect/TForge/TForgeOps.td:37-113, docs/dialect.md:19-30
 *     op semantics: bias_add is one IEEE add, relu is IEEE-2019 maximum(x, +0)
 *     (NaN propagates, -0 -> +0), add is one IEEE add.
 *   - docs/numerics.md:3,34,38,53  every FMA variant with sequential k (CPU
 *     vectorized, GPU naive, GPU staged) is bitwise identical; the unfused
 *     `cpu-scalar` pipeline (separate multiply and add) is the other variant.
 *
 * Exports:
 *   _mlir_ciface_entry(...)  the reference harness ABI (runners/cpu/tforge-cpu-bench.cpp:91-97,
 *                            211-239), one workload per build (-DTF_WORKLOAD_*), so the reference's
 *                            own harness can drive this file unchanged; allocates nothing.
 *   oracle_gemm(...)         matmul / mbr / matmul_add on plain pointers (ctypes entry).
 *   oracle_elementwise(...)  add / relu / bias_add.
 *
 * Compiled with -ffp-contract=off: the only fused multiply-adds are the explicit
 * ones (fmaf and _mm256_fmadd_ps, both single-rounding), so the FMA path is the
 * reference's sequential-k FMA order and the scalar path is its unfused order.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>
#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#define TF_HAVE_AVX2 1
#endif

enum { OR_MATMUL = 0, OR_MBR = 1, OR_MATMUL_ADD = 2 };
enum { OR_ADD = 0, OR_RELU = 1, OR_BIAS_ADD = 2 };

/* IEEE-2019 maximum(x, +0.0): NaN -> NaN, -0.0 -> +0.0, negatives -> +0.0. */
static inline float ieee_relu(float x) {
  if (x != x) return x;
  return x > 0.0f ? x : 0.0f;
}

static inline float epilogue(int workload, float acc, const float *aux, int64_t m, int64_t n,
                             int64_t ldc) {
  if (workload == OR_MBR) return ieee_relu(acc + aux[n]);
  if (workload == OR_MATMUL_ADD) return acc + aux[m * ldc + n];
  return acc;
}

/* One mr x nr register tile (mr <= 6, nr <= 16): accumulators from +0.0, one
 * single-rounding FMA per k in sequential k order, K stepped by 4 like the
 * reference's reg-tile K extent (the order per element is sequential either way). */
static void tile_fma(int workload, const float *A, const float *B, const float *aux, float *C,
                     int64_t m0, int mr, int64_t n0, int nr, int64_t N, int64_t K) {
  float acc[6][16];
  for (int i = 0; i < 6; ++i)
    for (int j = 0; j < 16; ++j) acc[i][j] = 0.0f;
#ifdef TF_HAVE_AVX2
  if (mr == 6 && nr == 16) {
    __m256 c[6][2];
    for (int i = 0; i < 6; ++i) c[i][0] = c[i][1] = _mm256_setzero_ps();
    for (int64_t k0 = 0; k0 < K; k0 += 4) {
      int64_t kr = K - k0 < 4 ? K - k0 : 4;
      for (int64_t kk = 0; kk < kr; ++kk) {
        const float *brow = B + (k0 + kk) * N + n0;
        __m256 b0 = _mm256_loadu_ps(brow), b1 = _mm256_loadu_ps(brow + 8);
        for (int i = 0; i < 6; ++i) {
          __m256 a = _mm256_broadcast_ss(A + (m0 + i) * K + k0 + kk);
          c[i][0] = _mm256_fmadd_ps(a, b0, c[i][0]);
          c[i][1] = _mm256_fmadd_ps(a, b1, c[i][1]);
        }
      }
    }
    for (int i = 0; i < 6; ++i) {
      _mm256_storeu_ps(acc[i], c[i][0]);
      _mm256_storeu_ps(acc[i] + 8, c[i][1]);
    }
  } else
#endif
  {
    for (int64_t k0 = 0; k0 < K; k0 += 4) {
      int64_t kr = K - k0 < 4 ? K - k0 : 4;
      for (int64_t kk = 0; kk < kr; ++kk)
        for (int i = 0; i < mr; ++i) {
          float a = A[(m0 + i) * K + k0 + kk];
          for (int j = 0; j < nr; ++j) acc[i][j] = fmaf(a, B[(k0 + kk) * N + n0 + j], acc[i][j]);
        }
    }
  }
  for (int i = 0; i < mr; ++i)
    for (int j = 0; j < nr; ++j)
      C[(m0 + i) * N + n0 + j] = epilogue(workload, acc[i][j], aux, m0 + i, n0 + j, N);
}

/* The reference's unfused scalar pipeline (`--tforge-cpu-pipeline` with no
 * options): acc = acc + a*b with two roundings, sequential k, from +0.0. */
static void gemm_scalar(int workload, const float *A, const float *B, const float *aux, float *C,
                        int64_t M, int64_t N, int64_t K) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        float p = A[m * K + k] * B[k * N + n];
        acc = acc + p;
      }
      C[m * N + n] = epilogue(workload, acc, aux, m, n, N);
    }
}

/* workload: 0 matmul, 1 mbr (aux = bias[N]), 2 matmul_add (aux = C_res[M x N]).
 * fma: 1 = reference BASELINE CPU kernel (6x16 register tiles, sequential-k FMA),
 *      0 = reference cpu-scalar (separate multiply and add). Returns 0 on success. */
int oracle_gemm(int workload, const float *A, const float *B, const float *aux, float *C,
                int64_t M, int64_t N, int64_t K, int fma) {
  if (M < 0 || N < 0 || K < 0 || workload < 0 || workload > 2) return 1;
  if (!fma) {
    gemm_scalar(workload, A, B, aux, C, M, N, K);
    return 0;
  }
  for (int64_t m0 = 0; m0 < M; m0 += 6) {
    int mr = M - m0 < 6 ? (int)(M - m0) : 6;
    for (int64_t n0 = 0; n0 < N; n0 += 16) {
      int nr = N - n0 < 16 ? (int)(N - n0) : 16;
      tile_fma(workload, A, B, aux, C, m0, mr, n0, nr, N, K);
    }
  }
  return 0;
}

/* Scalar sequential-k fmaf loop: the bitwise target the tiled kernel must equal. */
int oracle_gemm_fma_naive(int workload, const float *A, const float *B, const float *aux, float *C,
                          int64_t M, int64_t N, int64_t K) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k) acc = fmaf(A[m * K + k], B[k * N + n], acc);
      C[m * N + n] = epilogue(workload, acc, aux, m, n, N);
    }
  return 0;
}

/* op: 0 add (Z = X + Y, Y is M x N), 1 relu (Z = maximum(X, +0)), 2 bias_add (Z = X + bias[n]). */
int oracle_elementwise(int op, const float *X, const float *Y, float *Z, int64_t M, int64_t N) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      float x = X[m * N + n];
      if (op == OR_ADD) Z[m * N + n] = x + Y[m * N + n];
      else if (op == OR_RELU) Z[m * N + n] = ieee_relu(x);
      else if (op == OR_BIAS_ADD) Z[m * N + n] = x + Y[n];
      else return 1;
    }
  return 0;
}

/* ---- the reference harness ABI (runners/cpu/tforge-cpu-bench.cpp:91-97) ---- */
typedef struct { float *allocated, *aligned; int64_t offset, sizes[2], strides[2]; } MemRef2;
typedef struct { float *allocated, *aligned; int64_t offset, sizes[1], strides[1]; } MemRef1;

#define DATA(d) ((d)->aligned + (d)->offset)

#if defined(TF_WORKLOAD_MBR)
void _mlir_ciface_entry(MemRef2 *a, MemRef2 *b, MemRef1 *bias, MemRef2 *out) {
  oracle_gemm(OR_MBR, DATA(a), DATA(b), DATA(bias), DATA(out), a->sizes[0], b->sizes[1], a->sizes[1], 1);
}
#elif defined(TF_WORKLOAD_MATMUL)
void _mlir_ciface_entry(MemRef2 *a, MemRef2 *b, MemRef2 *out) {
  oracle_gemm(OR_MATMUL, DATA(a), DATA(b), NULL, DATA(out), a->sizes[0], b->sizes[1], a->sizes[1], 1);
}
#elif defined(TF_WORKLOAD_ADD)
void _mlir_ciface_entry(MemRef2 *a, MemRef2 *b, MemRef2 *out) {
  oracle_elementwise(OR_ADD, DATA(a), DATA(b), DATA(out), a->sizes[0], a->sizes[1]);
}
#elif defined(TF_WORKLOAD_RELU)
void _mlir_ciface_entry(MemRef2 *a, MemRef2 *out) {
  oracle_elementwise(OR_RELU, DATA(a), NULL, DATA(out), a->sizes[0], a->sizes[1]);
}
#endif
