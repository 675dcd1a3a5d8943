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
#include "tf_ptx.cuh"

namespace tf {

namespace {

constexpr int SBK = 8;  // K per shared-memory stage

// IEEE-2019 maximum(x, +0.0) with the NaN payload kept, on the bit pattern (a float
// compare-and-select may be contracted into a max that canonicalizes NaN).
__device__ __forceinline__ float relu_max(float x) {
  const uint32_t u = __float_as_uint(x);
  const bool keep = static_cast<int32_t>(u) > 0 || (u & 0x7FFFFFFFu) > 0x7F800000u;  // > +0 or NaN
  return __uint_as_float(keep ? u : 0u);
}

// BM x BN tile (128 or 64 each) on 256 threads.  Thread (tx, ty) = (tid % 16, tid / 16) owns
// rows 64 h + 4 ty + i and columns 64 g + 4 tx + j (h < BM / 64, g < BN / 64, i, j < 4): per k
// it reads BM / 64 float4 of A and BN / 64 of B from shared memory (128x128: 4 loads for 64
// FMAs).  Every output keeps one accumulator updated by one fmaf per k in increasing k from
// +0.0, so the result is the reference's bit for bit.  The next K tile is fetched into
// registers while this one is consumed (vector global loads when the pointers and pitches
// allow, VEC), then stored into the other shared-memory buffer.
template <int EPI, bool VEC, int BM, int BN>
__global__ void __launch_bounds__(256, BM == 128 ? 2 : 4) gemm_simt_kernel(
    const float *__restrict__ A, const float *__restrict__ B, const float *__restrict__ aux, float *__restrict__ C,
    int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc) {
  constexpr int HM = BM / 64, HN = BN / 64;
  constexpr int EA = BM / 32, EB = BN / 32;  // elements each thread stages per K tile
  constexpr int TPR = SBK / EA;              // threads per A row
  // A tile transposed (As[k][m]); 4 floats of padding put the k sub-rows a thread group
  // stores into different banks, and keep every row 16-byte aligned.
  __shared__ __align__(16) float As[2][SBK][BM + 4];
  __shared__ __align__(16) float Bs[2][SBK][BN];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  float acc[4 * HM][4 * HN];
#pragma unroll
  for (int i = 0; i < 4 * HM; ++i)
#pragma unroll
    for (int j = 0; j < 4 * HN; ++j) acc[i][j] = 0.0f;

  // Staging of one K tile: A row ar, k ak .. ak + EA - 1; B row bk, columns bc .. bc + EB - 1.
  // Out-of-range elements read as 0.
  const int ar = tid / TPR, ak = (tid % TPR) * EA, bk = tid >> 5, bc = (tid & 31) * EB;
  float ra[EA], rb[EB];
  auto gload = [&](int64_t k0) {
    const int64_t m = m0 + ar, k = k0 + ak;
    if (VEC && m < M && k + EA - 1 < K) {
      if constexpr (EA == 4) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(A + m * lda + k));
        ra[0] = v.x; ra[1] = v.y; ra[2] = v.z; ra[3] = v.w;
      } else {
        const float2 v = __ldg(reinterpret_cast<const float2 *>(A + m * lda + k));
        ra[0] = v.x; ra[1] = v.y;
      }
    } else {
#pragma unroll
      for (int c = 0; c < EA; ++c) ra[c] = (m < M && k + c < K) ? __ldg(A + m * lda + k + c) : 0.0f;
    }
    const int64_t kb = k0 + bk, n = n0 + bc;
    if (VEC && kb < K && n + EB - 1 < N) {
      if constexpr (EB == 4) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(B + kb * ldb + n));
        rb[0] = v.x; rb[1] = v.y; rb[2] = v.z; rb[3] = v.w;
      } else {
        const float2 v = __ldg(reinterpret_cast<const float2 *>(B + kb * ldb + n));
        rb[0] = v.x; rb[1] = v.y;
      }
    } else {
#pragma unroll
      for (int c = 0; c < EB; ++c) rb[c] = (kb < K && n + c < N) ? __ldg(B + kb * ldb + n + c) : 0.0f;
    }
  };
  auto sstore = [&](int buf) {
#pragma unroll
    for (int c = 0; c < EA; ++c) As[buf][ak + c][ar] = ra[c];
#pragma unroll
    for (int c = 0; c < EB; ++c) Bs[buf][bk][bc + c] = rb[c];
  };
  auto step = [&](int buf, int kk) {
    float a[4 * HM], b[4 * HN];
#pragma unroll
    for (int h = 0; h < HM; ++h) {
      const float4 v = *reinterpret_cast<const float4 *>(&As[buf][kk][64 * h + 4 * ty]);
      a[4 * h] = v.x; a[4 * h + 1] = v.y; a[4 * h + 2] = v.z; a[4 * h + 3] = v.w;
    }
#pragma unroll
    for (int g = 0; g < HN; ++g) {
      const float4 v = *reinterpret_cast<const float4 *>(&Bs[buf][kk][64 * g + 4 * tx]);
      b[4 * g] = v.x; b[4 * g + 1] = v.y; b[4 * g + 2] = v.z; b[4 * g + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 4 * HM; ++i)
#pragma unroll
      for (int j = 0; j < 4 * HN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
  };

  const int64_t ntiles = (K + SBK - 1) / SBK;
  if (ntiles > 0) {
    gload(0);
    sstore(0);
  }
  __syncthreads();
  for (int64_t t = 0; t < ntiles; ++t) {
    const int buf = (int)(t & 1);
    const bool more = t + 1 < ntiles;
    if (more) gload((t + 1) * SBK);
    if (more || K - t * SBK == SBK) {
#pragma unroll
      for (int kk = 0; kk < SBK; ++kk) step(buf, kk);
    } else {
      // Last, partial tile: never add a padded 0 * 0 (-0 must stay -0).
      const int kmax = (int)(K - t * SBK);
#pragma unroll
      for (int kk = 0; kk < SBK; ++kk)
        if (kk < kmax) step(buf, kk);
    }
    if (more) sstore(buf ^ 1);
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 4 * HM; ++i) {
    const int64_t m = m0 + 64 * (i / 4) + 4 * ty + (i % 4);
    if (m >= M) continue;
#pragma unroll
    for (int g = 0; g < HN; ++g) {
      const int64_t n = n0 + 64 * g + 4 * tx;
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t nn = n + j;
        v[j] = acc[i][4 * g + j];
        if (nn < N) {
          if (EPI == EPI_MBR) v[j] = relu_max(__fadd_rn(v[j], aux[nn]));
          else if (EPI == EPI_ADD) v[j] = __fadd_rn(v[j], aux[m * ldc + nn]);
        }
      }
      if (VEC && n + 3 < N) {
        *reinterpret_cast<float4 *>(C + m * ldc + n) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (n + j < N) C[m * ldc + n + j] = v[j];
      }
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
  grid_launch_dependents();  // a GEMM launched as this kernel's dependent may start setting up
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}

// Eight elements per step (x and y 16-byte aligned): two 16-byte loads, one 16-byte store;
// the same round-to-nearest-even per element as __float2bfloat16_rn.
__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&v);
}
__device__ __forceinline__ uint4 bf16x8(const float4 a, const float4 b) {
  return make_uint4(bf16x2_bits(a.x, a.y), bf16x2_bits(a.z, a.w), bf16x2_bits(b.x, b.y), bf16x2_bits(b.z, b.w));
}
__global__ void convert_bf16_vec8_kernel(const float4 *__restrict__ x, uint4 *__restrict__ y, int64_t n8) {
  grid_launch_dependents();  // a GEMM launched as this kernel's dependent may start setting up
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = bf16x8(__ldg(x + 2 * i), __ldg(x + 2 * i + 1));
}

// dst[c * ldd + r] = src[r * lds + c]: 32 x 32 tiles through shared memory (padded against
// bank conflicts), coalesced reads along c and writes along r; 32 x 8 threads, 4 rows each.
__global__ void transpose_f32_kernel(const float *__restrict__ src, int64_t lds, float *__restrict__ dst, int64_t ldd,
                                     int64_t rows, int64_t cols) {
  grid_launch_dependents();  // a GEMM launched as this kernel's dependent may start setting up
  __shared__ float t[32][33];
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int64_t r = r0 + threadIdx.y + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) t[threadIdx.y + i][threadIdx.x] = __ldg(src + r * lds + c);
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int64_t c = c0 + threadIdx.y + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[c * ldd + r] = t[threadIdx.x][threadIdx.y + i];
  }
}

// Two packed arrays in one launch (A and B of a BF16-mode call), eight elements per step.
__global__ void convert_bf16_two_vec8_kernel(const float4 *__restrict__ x1, uint4 *__restrict__ y1, int64_t n1_8,
                                             const float4 *__restrict__ x2, uint4 *__restrict__ y2, int64_t n2_8) {
  grid_launch_dependents();  // a GEMM launched as this kernel's dependent may start setting up
  const int64_t total = n1_8 + n2_8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    if (i < n1_8) y1[i] = bf16x8(__ldg(x1 + 2 * i), __ldg(x1 + 2 * i + 1));
    else {
      const int64_t j = i - n1_8;
      y2[j] = bf16x8(__ldg(x2 + 2 * j), __ldg(x2 + 2 * j + 1));
    }
  }
}

// Pitched rows, eight elements per step (N, both pitches multiples of 8, bases aligned).
__global__ void convert_rows_bf16_vec8_kernel(const float *__restrict__ x, int64_t lds, uint16_t *__restrict__ y,
                                              int64_t ldd, int64_t M, int64_t n8) {
  grid_launch_dependents();  // a GEMM launched as this kernel's dependent may start setting up
  const int64_t total = M * n8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / n8, c = (i - r * n8) * 8;
    const float4 *src = reinterpret_cast<const float4 *>(x + r * lds + c);
    *reinterpret_cast<uint4 *>(y + r * ldd + c) = bf16x8(__ldg(src), __ldg(src + 1));
  }
}

// Pitched f32 -> bf16 rows (one element per thread step; the general bf16-output path).
__global__ void convert_rows_bf16_kernel(const float *__restrict__ x, int64_t lds, __nv_bfloat16 *__restrict__ y,
                                         int64_t ldd, int64_t M, int64_t N) {
  grid_launch_dependents();  // a GEMM launched as this kernel's dependent may start setting up
  const int64_t total = M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / N, c = i - r * N;
    y[r * ldd + c] = __float2bfloat16_rn(x[r * lds + c]);
  }
}

int grid_for(int64_t work, int threads) {
  // Grid-stride loops: enough CTAs to fill 148 SMs several times over.
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = 148 * 16;
  if (g > cap) g = cap;
  return g < 1 ? 1 : (int)g;
}

}  // namespace

// 128x128 tiles, or 64x64 when there are fewer 128x128 tiles than SMs (4x the CTAs).
static int simt_tile(int64_t M, int64_t N) {
  const int64_t tiles = ((M + 127) / 128) * ((N + 127) / 128);
  return tiles < 148 ? 64 : 128;
}

void simt_launch_shape(int64_t M, int64_t N, int grid[3], int block[3], int *smem) {
  const int t = simt_tile(M, N);
  grid[0] = (int)((N + t - 1) / t);
  grid[1] = (int)((M + t - 1) / t);
  grid[2] = 1;
  block[0] = 256;
  block[1] = block[2] = 1;
  *smem = 0;
}

int simt_tile_size(int64_t M, int64_t N) { return simt_tile(M, N); }

// Vector global access needs 16-byte-aligned bases and pitches (C_res shares ldc).
static bool simt_vec_ok(const float *A, const float *B, const float *aux, const float *C, int64_t lda, int64_t ldb,
                        int64_t ldc, int epi) {
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return lda % 4 == 0 && ldb % 4 == 0 && ldc % 4 == 0 && al(A) && al(B) && al(C) &&
         (epi != EPI_ADD || al(aux));
}

template <int EPI, int T>
static void launch_simt_tile(bool vec, cudaStream_t stream, const float *A, const float *B, const float *aux,
                             float *C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc) {
  const dim3 grid((unsigned)((N + T - 1) / T), (unsigned)((M + T - 1) / T));
  if (vec) gemm_simt_kernel<EPI, true, T, T><<<grid, 256, 0, stream>>>(A, B, aux, C, M, N, K, lda, ldb, ldc);
  else gemm_simt_kernel<EPI, false, T, T><<<grid, 256, 0, stream>>>(A, B, aux, C, M, N, K, lda, ldb, ldc);
}

template <int EPI>
static void launch_simt_epi(bool vec, int tile, cudaStream_t stream, const float *A, const float *B,
                            const float *aux, float *C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                            int64_t ldc) {
  if (tile == 64) launch_simt_tile<EPI, 64>(vec, stream, A, B, aux, C, M, N, K, lda, ldb, ldc);
  else launch_simt_tile<EPI, 128>(vec, stream, A, B, aux, C, M, N, K, lda, ldb, ldc);
}

cudaError_t launch_gemm_simt(int epi, const float *A, const float *B, const float *aux, float *C,
                             int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                             int64_t ldc, cudaStream_t stream) {
  if (M == 0 || N == 0) return cudaSuccess;
  const bool vec = simt_vec_ok(A, B, aux, C, lda, ldb, ldc, epi);
  const int tile = simt_tile(M, N);
  if (epi == EPI_MATMUL) launch_simt_epi<EPI_MATMUL>(vec, tile, stream, A, B, aux, C, M, N, K, lda, ldb, ldc);
  else if (epi == EPI_MBR) launch_simt_epi<EPI_MBR>(vec, tile, stream, A, B, aux, C, M, N, K, lda, ldb, ldc);
  else launch_simt_epi<EPI_ADD>(vec, tile, stream, A, B, aux, C, M, N, K, lda, ldb, ldc);
  return cudaGetLastError();
}

cudaError_t simt_func_attributes(int epi, cudaFuncAttributes *a, int *blocks) {
  const void *f = epi == EPI_MBR   ? reinterpret_cast<const void *>(gemm_simt_kernel<EPI_MBR, true, 128, 128>)
                  : epi == EPI_ADD ? reinterpret_cast<const void *>(gemm_simt_kernel<EPI_ADD, true, 128, 128>)
                                   : reinterpret_cast<const void *>(gemm_simt_kernel<EPI_MATMUL, true, 128, 128>);
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

cudaError_t launch_convert_rows_bf16(const float *src, int64_t lds, uint16_t *dst, int64_t ldd, int64_t M,
                                     int64_t N, cudaStream_t stream) {
  if (M == 0 || N == 0) return cudaSuccess;
  const bool vec = N % 8 == 0 && lds % 8 == 0 && ldd % 8 == 0 && ((uintptr_t)src % 16) == 0 && ((uintptr_t)dst % 16) == 0;
  if (vec)
    convert_rows_bf16_vec8_kernel<<<grid_for(M * N / 8, 256), 256, 0, stream>>>(src, lds, dst, ldd, M, N / 8);
  else
    convert_rows_bf16_kernel<<<grid_for(M * N, 256), 256, 0, stream>>>(src, lds, reinterpret_cast<__nv_bfloat16 *>(dst),
                                                                       ldd, M, N);
  return cudaGetLastError();
}

cudaError_t launch_transpose_f32(const float *src, int64_t lds, float *dst, int64_t ldd, int64_t rows, int64_t cols,
                                 cudaStream_t stream) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  if ((cols + 31) / 32 > 0x7FFFFFFF || (rows + 31) / 32 > 65535) return cudaErrorInvalidValue;
  transpose_f32_kernel<<<dim3((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32)), dim3(32, 8), 0, stream>>>(
      src, lds, dst, ldd, rows, cols);
  return cudaGetLastError();
}

cudaError_t launch_convert_bf16_two(const float *x1, uint16_t *y1, int64_t n1, const float *x2, uint16_t *y2,
                                    int64_t n2, cudaStream_t stream) {
  const bool vec = n1 % 8 == 0 && n2 % 8 == 0 && ((uintptr_t)x1 % 16) == 0 && ((uintptr_t)y1 % 16) == 0 &&
                   ((uintptr_t)x2 % 16) == 0 && ((uintptr_t)y2 % 16) == 0;
  if (!vec || n1 + n2 == 0) {
    cudaError_t e = launch_convert_bf16(x1, y1, n1, stream);
    return e == cudaSuccess ? launch_convert_bf16(x2, y2, n2, stream) : e;
  }
  convert_bf16_two_vec8_kernel<<<grid_for((n1 + n2) / 8, 256), 256, 0, stream>>>(
      reinterpret_cast<const float4 *>(x1), reinterpret_cast<uint4 *>(y1), n1 / 8, reinterpret_cast<const float4 *>(x2),
      reinterpret_cast<uint4 *>(y2), n2 / 8);
  return cudaGetLastError();
}

cudaError_t launch_convert_bf16(const float *x, uint16_t *y, int64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  if (((uintptr_t)x % 16) == 0 && ((uintptr_t)y % 16) == 0 && n >= 8) {
    // Aligned bulk in 8-element steps, the remaining n % 8 elements one by one.
    const int64_t n8 = n / 8;
    convert_bf16_vec8_kernel<<<grid_for(n8, 256), 256, 0, stream>>>(reinterpret_cast<const float4 *>(x),
                                                                    reinterpret_cast<uint4 *>(y), n8);
    if (n % 8)
      convert_bf16_kernel<<<1, 32, 0, stream>>>(x + n8 * 8, reinterpret_cast<__nv_bfloat16 *>(y) + n8 * 8, n % 8);
    return cudaGetLastError();
  }
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
