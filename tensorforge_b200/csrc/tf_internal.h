// tf_internal.h -- declarations shared by the library's translation units (not public).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "tforge.h"

namespace tf {

enum Epi : int { EPI_MATMUL = 0, EPI_MBR = 1, EPI_ADD = 2 };
// Tensor-core precision paths: one TF32 product, the 3xTF32 split, or bf16 operands.
enum Prec : int { PREC_TF32 = 0, PREC_X3 = 1, PREC_BF16 = 2 };

#ifndef TF_PAIR_SPLIT
#define TF_PAIR_SPLIT 1
#endif
// 3xTF32 operand split of the pair kernel: 1 = truncation split, 0 = round split.
constexpr int kPairSplit = TF_PAIR_SPLIT;

#ifndef TF_PAIR_X3_LAND
#define TF_PAIR_X3_LAND (TF_PAIR_SPLIT ? 5 : 4)
#endif
// Landing-ring depth of the 3xTF32 pair kernel (its instantiated "stages").
constexpr int kPairX3Land = TF_PAIR_X3_LAND;

#ifndef TF_RASTER_GROUP
#define TF_RASTER_GROUP 8
#endif
// Tile rows per raster group of the pair kernels' tile order.
constexpr int kRasterGroup = TF_RASTER_GROUP;

// Parameters of the tcgen05 kernel besides the two tensor maps.
struct TcParams {
  const float *bias;   // N (mbr)
  const float *cres;   // M x N, pitch ldc (matmul_add)
  float *out;          // M x N, pitch ldc
  int32_t M, N, K;
  int64_t ldc;
  uint32_t *status;    // device status word
  uint64_t limit_ns;   // bounded-wait limit
  int32_t debug_skip;  // test hook: skip the first stage's loads
  // Split-K (CTA-pair kernel): `splits` > 1 CTA pairs per tile (grid z) each take an equal
  // k-range and store raw partial sums into slice z of the output map, at row offset
  // z * split_rows; 0 or 1 = no split.
  int32_t splits;
  int32_t split_rows;
  // 1: out holds bf16 (RNE of the f32 results), tmO is a bf16 map (box 32 columns x 128
  // rows, 64-B swizzle).  BF16 precision, mbr epilogue, 256-wide pair tiles or the
  // persistent pair kernel only.
  int32_t out_bf16;
  // 1 (TF32, 256-wide pair tiles or the persistent pair kernel): tmB maps a transposed copy
  // of B (N x K, K-major tiles of 128 columns x 32 k); the MMAs read both operands K-major.
  int32_t b_kmajor;
  // 1 (TF32, B as given, 256-wide pair tiles or the persistent pair kernel, N a multiple of 32
  // and K of 4): tmB is the 4-D map of the k-group-major B tiling (BTileMN, tf_ptx.cuh) and the
  // kernel instantiation reads that tiling; 0: the 2-D map of 128-B column blocks.
  int32_t b_atoms;
  // 1: the launch is a programmatic dependent of the kernel just before it on the stream (the
  // operand conversion or B transpose that wrote what tmA / tmB read): the CTAs set up while
  // that kernel finishes, and the TMA producer waits for it (griddepcontrol.wait) before its
  // first operand load.  Nothing else in the GEMM reads what that kernel writes.
  int32_t pdl;
};

// Launch attribute of a programmatic dependent launch (TcParams::pdl).
inline void pdl_attr(cudaLaunchAttribute &a) {
  a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a.val.programmaticStreamSerializationAllowed = 1;
}

struct TcConfig {
  int prec;    // Prec
  int bn;      // 64, 128, 256 (output tile width; 256 for the CTA-pair kernel)
  int stages;
  int pair;    // 1: CTA-pair kernel (cta_group::2, 256 x bn tiles), 0: one CTA per 128 x bn tile
  int persist;  // 1 (pair, TF32 / BF16, bn 256): persistent pair kernel, two TMEM accumulators
};

// Dynamic shared memory the tcgen05 kernel needs for a configuration.
int tc_smem_bytes(const TcConfig &cfg);
// True when a kernel instantiation exists for the configuration.
bool tc_config_supported(const TcConfig &cfg);
// Launches the tcgen05 kernel.  tmA / tmB are encoded by the caller.
cudaError_t launch_gemm_tc(const TcConfig &cfg, int epi, const CUtensorMap &tmA,
                           const CUtensorMap &tmB, const TcParams &p, cudaStream_t stream);

// Registers / static shared memory of an instantiation and resident CTAs per SM
// (needs a device).
cudaError_t tc_func_attributes(const TcConfig &cfg, int epi, cudaFuncAttributes *attr,
                               int *blocks_per_sm);
cudaError_t simt_func_attributes(int epi, cudaFuncAttributes *attr, int *blocks_per_sm);

// CTA-pair (cta_group::2) kernel: 256-row x bn-column output tiles (bn 256 or 240),
// clusters of two CTAs.
int pair_smem_bytes(int prec, int stages);
int pair_tmem_cols(int prec);
// True when the pair kernel for (prec, bn) accumulates the transposed tile (TF32, 256 wide):
// its output / C_res maps then use 32-row x 128-column boxes without swizzle.
bool pair_transposed(int prec, int bn);
// tmO / tmC: f32 maps of the output and of C_res (box 32 columns x 128 rows, 128-B
// swizzle) for the TMA-store epilogue; tmC is read only by matmul_add.  bn 240 takes no
// split-K (p.splits <= 1).
cudaError_t launch_gemm_pair(int prec, int stages, int bn, int epi, const CUtensorMap &tmA,
                             const CUtensorMap &tmB, const CUtensorMap &tmO, const CUtensorMap &tmC,
                             const TcParams &p, cudaStream_t stream);
cudaError_t pair_func_attributes(int prec, int stages, int bn, int epi, cudaFuncAttributes *attr,
                                 int *blocks_per_sm);

// Persistent CTA-pair kernel (TF32 / BF16 modes, 256 x 256 tiles, no split-K): clusters
// loop over tiles with two TMEM accumulators.  tmO as for launch_gemm_pair; matmul_add reads
// p.cres directly.  persist_grid_pairs: clusters it launches for M x N (-1 without a device).
int persist_smem_bytes(int prec, int stages);
cudaError_t launch_gemm_pair_persistent(int prec, int stages, int epi, const CUtensorMap &tmA,
                                        const CUtensorMap &tmB, const CUtensorMap &tmO, const TcParams &p,
                                        cudaStream_t stream);
cudaError_t persist_func_attributes(int prec, int stages, int epi, cudaFuncAttributes *attr,
                                    int *blocks_per_sm);
int persist_grid_pairs(int prec, int stages, int epi, int64_t M, int64_t N);
// True when the persistent kernel for `prec` accumulates the transposed tile (TF32 reading B as
// given): its output map then uses 32-row x 128-column boxes without swizzle.
bool persist_transposed(int prec);

// The dispatch table's tensor-core choice (false when it would not use tcgen05), the
// TMA operand map encoder, and the per-thread error text (all defined in tf_api.cu).
bool select_tc_config(int mode, int64_t M, int64_t N, int64_t K, TcConfig *out);
// dst[r * ldd + c] = bf16_rn(src[r * lds + c]) for r < M, c < N.
cudaError_t launch_convert_rows_bf16(const float *src, int64_t lds, uint16_t *dst, int64_t ldd, int64_t M,
                                     int64_t N, cudaStream_t stream);
int encode_operand_map(CUtensorMap *m, const void *base, bool bf16, int64_t rows, int64_t cols,
                       int64_t ld, uint32_t box_cols, uint32_t box_rows, bool atom32);
void set_last_error(const char *msg);
// tforge_gemm's argument checks (pointers are only compared, never dereferenced) and the
// library's per-device stream-ordered memory pool.
int check_gemm_args(const tforge_gemm_args *a, int64_t *lda, int64_t *ldb, int64_t *ldc);
int device_pool(cudaMemPool_t *out);
// The bounded-wait limit (tforge_set_wait_limit_ns) and the skip-load test hook
// (tforge_debug_skip_load) every GEMM launch passes to its kernel.
uint64_t wait_limit_ns();
int debug_skip_load();
// Reads and clears the allocation-free entry's status word on the current device (tf_noalloc.cu);
// *v = 0 when that entry was never set up on it.
int noalloc_take_status(uint32_t *v);

// SIMT sequential-k FFMA GEMM (bitwise equal to the reference's generated kernels).
cudaError_t launch_gemm_simt(int epi, const float *A, const float *B, const float *aux, float *C,
                             int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                             int64_t ldc, cudaStream_t stream);
void simt_launch_shape(int64_t M, int64_t N, int grid[3], int block[3], int *smem);
int simt_tile_size(int64_t M, int64_t N);  // 128 or 64 (square tiles)

// Elementwise ops: op 0 add, 1 relu, 2 bias_add.
cudaError_t launch_elementwise(int op, const float *X, const float *Y, float *Z, int64_t M,
                               int64_t N, cudaStream_t stream);
cudaError_t launch_convert_bf16(const float *x, uint16_t *y, int64_t n, cudaStream_t stream);
// dst (cols x rows, pitch ldd) = transpose of src (rows x cols, pitch lds); rows < 2^21.
cudaError_t launch_transpose_f32(const float *src, int64_t lds, float *dst, int64_t ldd, int64_t rows, int64_t cols,
                                 cudaStream_t stream);
// Both conversions in one launch when both arrays are 16-byte aligned multiples of 8 elements.
cudaError_t launch_convert_bf16_two(const float *x1, uint16_t *y1, int64_t n1, const float *x2, uint16_t *y2,
                                    int64_t n2, cudaStream_t stream);
// Split-K epilogue: out[m, n] = epi(sum over s = 0..S-1, in order, of ws[s * slice + m * N + n]);
// N a multiple of 4, 16-byte-aligned rows.
cudaError_t launch_splitk_reduce(int epi, const float *ws, int splits, int64_t slice, int64_t M, int64_t N,
                                 const float *bias, const float *cres, float *out, int64_t ldc,
                                 cudaStream_t stream);

}  // namespace tf
