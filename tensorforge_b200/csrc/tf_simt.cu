// tf_simt.cu -- SIMT kernels: the bit-exact FFMA GEMM and the elementwise ops.
//
// gemm_simt_kernel: each output element is one accumulator that starts at +0.0 and takes
// one FFMA per k in sequential k order, then the fused epilogue.  That is the evaluation
// order of every kernel TensorForge generates with FMA contraction (CPU vectorized, GPU
// naive and staged), which docs/numerics.md:3,34,38,53 measured to be bitwise identical,
// so this kernel reproduces the reference's GPU results bit for bit.  It serves
// TFORGE_MODE_FP32_EXACT, K == 0, very small K in the fp32 mode, and shapes whose row
// pitches are not 16-byte multiples (which TMA cannot address).  Loads are scalar and
// bounds-checked, so any M, N, K and any 4-byte-aligned pointer works.
//
// Elementwise kernels: one IEEE operation per element (bit-exact against NumPy float32,
// python/tforge_gpu.py:116-126), 16-byte accesses when the pointers allow.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "tf_internal.h"

namespace tf {

namespace {

constexpr int SBM = 128, SBN = 128, SBK = 8, STM = 8, STN = 8;

// IEEE-2019 maximum(x, +0.0) with the NaN payload kept, on the bit pattern (a float
// compare-and-select may be contracted into a max that canonicalizes NaN).
__device__ __forceinline__ float relu_max(float x) {
  const uint32_t u = __float_as_uint(x);
  const bool keep = static_cast<int32_t>(u) > 0 || (u & 0x7FFFFFFFu) > 0x7F800000u;  // > +0 or NaN
  return __uint_as_float(keep ? u : 0u);
}

template <int EPI>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const float *__restrict__ A,
                                                        const float *__restrict__ B,
                                                        const float *__restrict__ aux,
                                                        float *__restrict__ C, int64_t M, int64_t N,
                                                        int64_t K, int64_t lda, int64_t ldb,
                                                        int64_t ldc) {
  __shared__ float As[2][SBK][SBM];
  __shared__ float Bs[2][SBK][SBN];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * SBM, n0 = (int64_t)blockIdx.x * SBN;
  float acc[STM][STN];
#pragma unroll
  for (int i = 0; i < STM; ++i)
#pragma unroll
    for (int j = 0; j < STN; ++j) acc[i][j] = 0.0f;

  // Each thread stages 4 elements of A (column k = tid % 8, rows tid / 8 + 32 i) and
  // 4 of B (row k = tid / 32, columns tid % 32 + 32 j) per K tile.
  auto load = [&](int buf, int64_t k0) {
    const int ak = tid & 7, ar = tid >> 3;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t m = m0 + ar + 32 * i, k = k0 + ak;
      As[buf][ak][ar + 32 * i] = (m < M && k < K) ? A[m * lda + k] : 0.0f;
    }
    const int bk = tid >> 5, bc = tid & 31;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t k = k0 + bk, n = n0 + bc + 32 * j;
      Bs[buf][bk][bc + 32 * j] = (k < K && n < N) ? B[k * ldb + n] : 0.0f;
    }
  };

  const int64_t ntiles = (K + SBK - 1) / SBK;
  if (ntiles > 0) load(0, 0);
  __syncthreads();
  for (int64_t t = 0; t < ntiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < ntiles) load(buf ^ 1, (t + 1) * SBK);
    const int64_t kleft = K - t * SBK;
    const int kmax = kleft < SBK ? (int)kleft : SBK;  // never add a padded 0*0: -0 must stay -0
#pragma unroll
    for (int kk = 0; kk < SBK; ++kk) {
      if (kk < kmax) {
        float a[STM], b[STN];
#pragma unroll
        for (int i = 0; i < STM; ++i) a[i] = As[buf][kk][ty + 16 * i];
#pragma unroll
        for (int j = 0; j < STN; ++j) b[j] = Bs[buf][kk][tx + 16 * j];
#pragma unroll
        for (int i = 0; i < STM; ++i)
#pragma unroll
          for (int j = 0; j < STN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < STM; ++i) {
    const int64_t m = m0 + ty + 16 * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < STN; ++j) {
      const int64_t n = n0 + tx + 16 * j;
      if (n >= N) continue;
      float v = acc[i][j];
      if (EPI == EPI_MBR) v = relu_max(__fadd_rn(v, aux[n]));
      else if (EPI == EPI_ADD) v = __fadd_rn(v, aux[m * ldc + n]);
      C[m * ldc + n] = v;
    }
  }
}

__global__ void elementwise_vec4(int op, const float4 *__restrict__ X, const float4 *__restrict__ Y,
                                 float4 *__restrict__ Z, int64_t n4, int64_t N4) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 x = X[i], r;
    if (op == 1) {
      r.x = relu_max(x.x); r.y = relu_max(x.y); r.z = relu_max(x.z); r.w = relu_max(x.w);
    } else {
      const float4 y = op == 0 ? Y[i] : Y[i % N4];
      r.x = __fadd_rn(x.x, y.x); r.y = __fadd_rn(x.y, y.y);
      r.z = __fadd_rn(x.z, y.z); r.w = __fadd_rn(x.w, y.w);
    }
    Z[i] = r;
  }
}

__global__ void elementwise_scalar(int op, const float *__restrict__ X, const float *__restrict__ Y,
                                   float *__restrict__ Z, int64_t n, int64_t N) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float x = X[i];
    Z[i] = op == 1 ? relu_max(x) : __fadd_rn(x, op == 0 ? Y[i] : Y[i % N]);
  }
}

__global__ void convert_bf16_kernel(const float *__restrict__ x, __nv_bfloat16 *__restrict__ y,
                                    int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}

int grid_for(int64_t work, int threads) {
  // Grid-stride loops: enough CTAs to fill 148 SMs several times over.
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = 148 * 16;
  if (g > cap) g = cap;
  return g < 1 ? 1 : (int)g;
}

}  // namespace

void simt_launch_shape(int64_t M, int64_t N, int grid[3], int block[3], int *smem) {
  grid[0] = (int)((N + SBN - 1) / SBN);
  grid[1] = (int)((M + SBM - 1) / SBM);
  grid[2] = 1;
  block[0] = 256;
  block[1] = block[2] = 1;
  *smem = 0;
}

cudaError_t launch_gemm_simt(int epi, const float *A, const float *B, const float *aux, float *C,
                             int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                             int64_t ldc, cudaStream_t stream) {
  if (M == 0 || N == 0) return cudaSuccess;
  dim3 grid((unsigned)((N + SBN - 1) / SBN), (unsigned)((M + SBM - 1) / SBM));
  if (epi == EPI_MATMUL)
    gemm_simt_kernel<EPI_MATMUL><<<grid, 256, 0, stream>>>(A, B, aux, C, M, N, K, lda, ldb, ldc);
  else if (epi == EPI_MBR)
    gemm_simt_kernel<EPI_MBR><<<grid, 256, 0, stream>>>(A, B, aux, C, M, N, K, lda, ldb, ldc);
  else
    gemm_simt_kernel<EPI_ADD><<<grid, 256, 0, stream>>>(A, B, aux, C, M, N, K, lda, ldb, ldc);
  return cudaGetLastError();
}

cudaError_t simt_func_attributes(int epi, cudaFuncAttributes *a, int *blocks) {
  const void *f = epi == EPI_MBR   ? reinterpret_cast<const void *>(gemm_simt_kernel<EPI_MBR>)
                  : epi == EPI_ADD ? reinterpret_cast<const void *>(gemm_simt_kernel<EPI_ADD>)
                                   : reinterpret_cast<const void *>(gemm_simt_kernel<EPI_MATMUL>);
  cudaError_t e = cudaFuncGetAttributes(a, f);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, f, 256, 0);
}

cudaError_t launch_elementwise(int op, const float *X, const float *Y, float *Z, int64_t M,
                               int64_t N, cudaStream_t stream) {
  const int64_t n = M * N;
  if (n == 0) return cudaSuccess;
  const bool vec = (N % 4 == 0) && ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(Z) |
                                     (op == 1 ? 0 : reinterpret_cast<uintptr_t>(Y))) % 16 == 0);
  if (vec) {
    const int64_t n4 = n / 4;
    elementwise_vec4<<<grid_for(n4, 256), 256, 0, stream>>>(
        op, reinterpret_cast<const float4 *>(X), reinterpret_cast<const float4 *>(Y),
        reinterpret_cast<float4 *>(Z), n4, N / 4);
  } else {
    elementwise_scalar<<<grid_for(n, 256), 256, 0, stream>>>(op, X, Y, Z, n, N);
  }
  return cudaGetLastError();
}

cudaError_t launch_convert_bf16(const float *x, uint16_t *y, int64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  convert_bf16_kernel<<<grid_for(n, 256), 256, 0, stream>>>(
      x, reinterpret_cast<__nv_bfloat16 *>(y), n);
  return cudaGetLastError();
}

}  // namespace tf

namespace tf {
namespace {

// Split-K epilogue, one float4 per thread step: the S partial sums in slice order, then the
// operator's epilogue (one IEEE add for bias / C_res, IEEE maximum for relu).
__global__ void splitk_reduce_kernel(int epi, const float4 *__restrict__ ws, int splits, int64_t slice4, int64_t M,
                                     int64_t n4, const float4 *__restrict__ bias, const float *__restrict__ cres,
                                     float *__restrict__ out, int64_t ldc) {
  const int64_t total = M * n4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / n4, c = i - m * n4;
    float4 acc = ws[i];
    for (int s = 1; s < splits; ++s) {
      const float4 v = ws[s * slice4 + i];
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z);
      acc.w = __fadd_rn(acc.w, v.w);
    }
    if (epi == EPI_MBR) {
      const float4 b = bias[c];
      acc.x = relu_max(__fadd_rn(acc.x, b.x));
      acc.y = relu_max(__fadd_rn(acc.y, b.y));
      acc.z = relu_max(__fadd_rn(acc.z, b.z));
      acc.w = relu_max(__fadd_rn(acc.w, b.w));
    } else if (epi == EPI_ADD) {
      const float4 r = *reinterpret_cast<const float4 *>(cres + m * ldc + 4 * c);
      acc.x = __fadd_rn(acc.x, r.x);
      acc.y = __fadd_rn(acc.y, r.y);
      acc.z = __fadd_rn(acc.z, r.z);
      acc.w = __fadd_rn(acc.w, r.w);
    }
    *reinterpret_cast<float4 *>(out + m * ldc + 4 * c) = acc;
  }
}

}  // namespace

cudaError_t launch_splitk_reduce(int epi, const float *ws, int splits, int64_t slice, int64_t M, int64_t N,
                                 const float *bias, const float *cres, float *out, int64_t ldc,
                                 cudaStream_t stream) {
  const int64_t n4 = N / 4, total = M * n4;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  splitk_reduce_kernel<<<(unsigned)blocks, 256, 0, stream>>>(epi, reinterpret_cast<const float4 *>(ws), splits,
                                                             slice / 4, M, n4, reinterpret_cast<const float4 *>(bias),
                                                             cres, out, ldc);
  return cudaGetLastError();
}

}  // namespace tf
