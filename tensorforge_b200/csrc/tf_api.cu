// tf_api.cu -- the C-ABI (include/tforge.h): argument checks, the per-shape dispatch
// table, TMA tensor-map encoding, the device status word and small device helpers.
//
// The dispatch table replaces the reference's analytical cost model and autotuner
// (python/costmodel.py:49-97, bench/stage9_costmodel.py:63-154): the tile choice is a
// function of (mode, M, N, K) over the instantiated tcgen05 configurations -- the measured
// winner of the offline sweep (tf_tune_table.inc) near a measured shape, an analytic wave
// model elsewhere.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "tforge.h"
#include "tf_internal.h"

using namespace tf;

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_wait_limit_ns{1000000000ull};
std::atomic<int> g_debug_skip{0};
std::mutex g_cfg_mu;
tforge_config g_cfg{};  // kernel == 0: use the table

int cuda_fail(cudaError_t e, const char *what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return TFORGE_ERR_CUDA;
}

// ---- cuTensorMapEncodeTiled through the runtime's driver entry point -----------------
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// 2-D row-major tensor [rows x cols] with pitch `ld` elements; box = {box_cols, box_rows};
// 128-byte swizzle (16-byte atoms, or 32-byte atoms with `atom32`, the layout the tensor
// cores require for N-contiguous 32-bit operands); out-of-range elements read as zero.
// Shared-memory layouts of a tile map: 128-B swizzle, its 32-B-atom form (MN-major TF32
// operands), 64-B swizzle (bf16 output boxes), none (transposed output boxes).
enum Swz { SW128 = 0, SW128_A32 = 1, SW64 = 2, SWNONE = 3 };

int make_tmap(CUtensorMap *m, const void *base, bool bf16, int64_t rows, int64_t cols, int64_t ld,
              uint32_t box_cols, uint32_t box_rows, int swz = SW128) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    g_last_error = "cuTensorMapEncodeTiled unavailable";
    return TFORGE_ERR_CUDA;
  }
  const int esz = bf16 ? 2 : 4;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * esz)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                   const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swz == SW64        ? CU_TENSOR_MAP_SWIZZLE_64B
                   : swz == SWNONE    ? CU_TENSOR_MAP_SWIZZLE_NONE
                   : swz == SW128_A32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                      : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    g_last_error = "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
    return TFORGE_ERR_CUDA;
  }
  return TFORGE_OK;
}

// TF32 B (K x N f32, row pitch ldb elements) as a 4-D map whose box is one CTA's 128-column B
// tile in the k-group-major tiling of BTileMN<4> (tf_ptx.cuh): dims (32 columns of a 128-B
// block, 4 rows of a k-group, column blocks, k-groups) with byte strides (-, 4 ldb, 128,
// 16 ldb); the box is one block wide, one group high, the tile's 4 blocks and a stage's 8 groups
// deep.  Needs N % 32 == 0 and K % 4 == 0, so that no element of a box lies outside B (the
// per-dimension bounds cannot see a partial block or group); k-groups past K read as zero.
int make_tmap_b_atoms(CUtensorMap *m, const void *B, int64_t K, int64_t N, int64_t ldb) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    g_last_error = "cuTensorMapEncodeTiled unavailable";
    return TFORGE_ERR_CUDA;
  }
  cuuint64_t dims[4] = {32, 4, (cuuint64_t)(N / 32), (cuuint64_t)(K / 4)};
  cuuint64_t strides[3] = {(cuuint64_t)(ldb * 4), 128, (cuuint64_t)(16 * ldb)};
  cuuint32_t box[4] = {32, 4, 4, 8};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void *>(B), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    g_last_error = "cuTensorMapEncodeTiled failed for the 4-D B map (" + std::to_string((int)r) + ")";
    return TFORGE_ERR_CUDA;
  }
  return TFORGE_OK;
}

// ---- per-device status word ------------------------------------------------------------
constexpr int kMaxDev = 64;
uint32_t *g_status[kMaxDev] = {};
std::mutex g_status_mu;

// The status word of the current device if a GEMM has created it, else nullptr (no allocation).
uint32_t *existing_status_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_status_mu);
  return g_status[dev];
}

int status_word(uint32_t **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDev) return TFORGE_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (!g_status[dev]) {
    void *p = nullptr;
    e = cudaMalloc(&p, 256);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(status)");
    e = cudaMemset(p, 0, 256);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(status)");
    g_status[dev] = static_cast<uint32_t *>(p);
  }
  *out = g_status[dev];
  return TFORGE_OK;
}

// ---- per-device scratch pool -------------------------------------------------------------
// Stream-ordered scratch (bf16 copies of f32 operands) comes from a pool the library owns,
// so concurrent streams never share a buffer and freed memory stays mapped for reuse
// (the release threshold is unlimited); the caller's default pool is left untouched.
cudaMemPool_t g_pool[kMaxDev] = {};

int scratch_pool(cudaMemPool_t *out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDev) return TFORGE_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (!g_pool[dev]) {
    cudaMemPoolProps props{};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    e = cudaMemPoolCreate(&pool, &props);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemPoolCreate");
    uint64_t keep = UINT64_MAX;
    e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemPoolSetAttribute");
    g_pool[dev] = pool;
  }
  *out = g_pool[dev];
  return TFORGE_OK;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

bool overlaps(const void *a, size_t abytes, const void *b, size_t bbytes) {
  if (!a || !b || !abytes || !bbytes) return false;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  return a0 < b0 + bbytes && b0 < a0 + abytes;
}

size_t span_bytes(int64_t rows, int64_t cols, int64_t ld, int esz) {
  if (rows <= 0 || cols <= 0) return 0;
  return (size_t)((rows - 1) * ld + cols) * esz;
}

// ---- dispatch table ------------------------------------------------------------------------
enum KernelKind { K_TC = 1, K_SIMT = 2 };

struct Choice {
  int kind;
  TcConfig tc;
};

// Stages per instantiated configuration: [prec][bn index] for one CTA; pair kernel.
constexpr int kStages1[3][3] = {{4, 6, 8}, {2, 3, 4}, {4, 6, 8}};  // bn = 256, 128, 64
constexpr int kStagesPair[3] = {6, kPairX3Land, 6};                // TF32, X3, BF16

// Relative throughput per busy SM of each kernel shape (pair, bn 256, 128, 64): wider
// tiles read fewer operand bytes per FLOP, and the pair halves B per SM.
constexpr double kKernelEff[4] = {1.0, 0.6, 0.5, 0.4};

// Estimated time units of a configuration: waves of CTAs (148 SMs, one CTA each) over
// the useful fraction of the tile area, divided by the per-SM throughput factor.
double est_cost(int64_t M, int64_t N, int tile_m, int tile_n, int ctas_per_tile, double eff) {
  const int64_t tiles = ((M + tile_m - 1) / tile_m) * ((N + tile_n - 1) / tile_n);
  const int64_t ctas = tiles * ctas_per_tile;
  const double waves = (double)((ctas + 147) / 148);
  const double area = (double)tiles * tile_m * tile_n;  // MMA work incl. padding
  const double per_wave_area = 148.0 / ctas_per_tile * tile_m * tile_n;
  return (waves * per_wave_area > area ? waves * per_wave_area : area) / eff;
}

bool config_supported(const TcConfig &c) {
  if (c.persist) return c.pair && c.bn == 256 && c.prec != PREC_X3 && persist_smem_bytes(c.prec, c.stages) > 0;
  if (c.pair) return (c.bn == 256 || c.bn == 240) && pair_smem_bytes(c.prec, c.stages) > 0;
  return tc_config_supported(c);
}

// Measured choices of the offline sweep (python -m tensorforge_b200.autotune on a B200):
// the fastest instantiated configuration that passed the FP64 check, per (prec, M, N, K).
// pair: 0 one-CTA kernel, 1 CTA-pair kernel, 2 persistent CTA-pair kernel.
struct TuneEntry {
  int prec;
  int64_t m, n, k;
  int pair, bn, stages;
  double tflops;
};
const TuneEntry kTune[] = {
#include "tf_tune_table.inc"
    {-1, 1, 1, 1, 0, 0, 0, 0.0}};

// The measured entry nearest to (M, N, K) in summed |log2| distance, provided each
// dimension lies within a factor of two of it; false when none does.
bool tuned_tc(int prec, int64_t M, int64_t N, int64_t K, TcConfig *out) {
  const TuneEntry *hit = nullptr;
  double best = 1e30;
  for (const TuneEntry &e : kTune) {
    if (e.prec != prec) continue;
    const double dm = std::fabs(std::log2((double)M / (double)e.m));
    const double dn = std::fabs(std::log2((double)N / (double)e.n));
    const double dk = std::fabs(std::log2((double)K / (double)e.k));
    if (dm > 1.0 || dn > 1.0 || dk > 1.0) continue;
    if (dm + dn + dk < best) {
      best = dm + dn + dk;
      hit = &e;
    }
  }
  if (!hit) return false;
  // The pair kernel has one instantiated depth per precision; the table says pair or not.
  const TcConfig c{prec, hit->bn, hit->pair ? kStagesPair[prec] : hit->stages, hit->pair ? 1 : 0, hit->pair == 2};
  if (!config_supported(c)) return false;
  *out = c;
  return true;
}

int device_pairs();
int auto_pair_splits(int prec, int64_t M, int64_t N, int64_t K);

// Tile width of the pair kernel without split-K: 240 instead of 256 columns when that takes
// no more waves of SM pairs, so each wave's tiles are 1/16 narrower (2048 x 2048: 72 tiles
// of 256 x 240 on 74 pairs instead of 64 tiles of 256 x 256, 86 % of the pairs busy).
int pair_width(int prec, int64_t M, int64_t N, int64_t K) {
  if (auto_pair_splits(prec, M, N, K) > 1) return 256;
  const int64_t pairs = device_pairs(), tm = (M + 255) / 256;
  const int64_t w256 = (tm * ((N + 255) / 256) + pairs - 1) / pairs;
  const int64_t w240 = (tm * ((N + 239) / 240) + pairs - 1) / pairs;
  return w240 * 240 < w256 * 256 ? 240 : 256;
}

// Analytic fallback outside the measured range: the fewest waves over the tile area.  The
// pair kernel takes 256x240 tiles when they help (3xTF32, pair_width), or -- TF32 and BF16
// with more tiles than SM pairs -- its persistent form, which overlaps each tile's epilogue
// with the next tile's MMAs (it won every such shape of the tuning sweep but one, by 1 %).
// Not beyond 32 tiles per pair: on a 131072 x 8192 x 8192 TF32 call (221 tiles per pair,
// 30 ms under the power cap) the persistent kernel ran at a lower clock and 13 % slower.
TcConfig model_tc(int prec, int64_t M, int64_t N, int64_t K) {
  TcConfig best{prec, 256, kStagesPair[prec], 1, 0};
  const int64_t tiles = ((M + 255) / 256) * ((N + 255) / 256), pairs = device_pairs();
  if (prec == PREC_X3)
    best.bn = pair_width(prec, M, N, K);
  else if (tiles > pairs && tiles <= 32 * pairs)
    best.persist = 1;
  double best_cost = est_cost(M, N, 256, 256, 2, kKernelEff[0]);
  const int bns[3] = {256, 128, 64};
  for (int i = 0; i < 3; ++i) {
    const double c = est_cost(M, N, 128, bns[i], 1, kKernelEff[i + 1]);
    if (c < best_cost * (1 - 1e-9)) {
      best_cost = c;
      best = TcConfig{prec, bns[i], kStages1[prec][i], 0};
    }
  }
  return best;
}

TcConfig table_tc(int prec, int64_t M, int64_t N, int64_t K) {
  TcConfig c{};
  if (tuned_tc(prec, M, N, K, &c)) return c;
  return model_tc(prec, M, N, K);
}

Choice choose(int mode, int64_t M, int64_t N, int64_t K, bool tma_ok) {
  Choice c{K_SIMT, {}};
  if (mode == TFORGE_MODE_FP32_EXACT || K == 0 || !tma_ok) return c;
  // 3xTF32 carries about 2^-20 relative error per product independent of K, while the
  // fp32 bound gamma_{K+1} shrinks with K; below K = 16 the exact kernel is used instead.
  if (mode == TFORGE_MODE_FP32 && K < 16) return c;
  const int prec = mode == TFORGE_MODE_FP32 ? PREC_X3 : (mode == TFORGE_MODE_TF32 ? PREC_TF32 : PREC_BF16);
  c.kind = K_TC;
  c.tc = table_tc(prec, M, N, K);
  std::lock_guard<std::mutex> lk(g_cfg_mu);
  if (g_cfg.kernel == 2) {
    c.kind = K_SIMT;
  } else if (g_cfg.kernel == 1 || g_cfg.kernel == 3) {
    const int pair = g_cfg.kernel == 3;
    TcConfig f{prec, pair ? (g_cfg.bn == 240 ? 240 : 256) : (g_cfg.bn ? g_cfg.bn : (c.tc.pair ? 256 : c.tc.bn)), 0,
               pair, pair && g_cfg.persistent ? 1 : 0};
    f.stages = g_cfg.stages ? g_cfg.stages
                            : (pair ? kStagesPair[prec] : kStages1[prec][f.bn == 256 ? 0 : (f.bn == 128 ? 1 : 2)]);
    if (config_supported(f) && !(pair && (f.bn == 240 || f.persist) && g_cfg.split_k > 1)) c.tc = f;
    else c.kind = -1;
  }
  return c;
}

int check_gemm(const tforge_gemm_args *a, int64_t *lda, int64_t *ldb, int64_t *ldc) {
  if (!a) return TFORGE_ERR_NULL;
  if (a->workload < TFORGE_MATMUL || a->workload > TFORGE_MATMUL_ADD) return TFORGE_ERR_MODE;
  if (a->mode < TFORGE_MODE_FP32 || a->mode > TFORGE_MODE_FP32_EXACT) return TFORGE_ERR_MODE;
  if ((a->a_dtype != TFORGE_F32 && a->a_dtype != TFORGE_BF16) ||
      (a->b_dtype != TFORGE_F32 && a->b_dtype != TFORGE_BF16))
    return TFORGE_ERR_MODE;
  if ((a->a_dtype == TFORGE_BF16 || a->b_dtype == TFORGE_BF16) && a->mode != TFORGE_MODE_BF16)
    return TFORGE_ERR_MODE;
  if (a->out_dtype != TFORGE_F32 && !(a->out_dtype == TFORGE_BF16 && a->mode == TFORGE_MODE_BF16))
    return TFORGE_ERR_MODE;
  if (a->M < 0 || a->N < 0 || a->K < 0) return TFORGE_ERR_SHAPE;
  if (a->M > INT32_MAX || a->N > INT32_MAX || a->K > INT32_MAX) return TFORGE_ERR_SHAPE;
  *lda = a->lda ? a->lda : a->K;
  *ldb = a->ldb ? a->ldb : a->N;
  *ldc = a->ldc ? a->ldc : a->N;
  if (*lda < a->K || *ldb < a->N || *ldc < a->N) return TFORGE_ERR_SHAPE;
  if (a->M == 0 || a->N == 0) return TFORGE_OK;
  if (!a->out) return TFORGE_ERR_NULL;
  if (a->K > 0 && (!a->A || !a->B)) return TFORGE_ERR_NULL;
  if (a->workload == TFORGE_MBR && !a->bias) return TFORGE_ERR_NULL;
  if (a->workload == TFORGE_MATMUL_ADD && !a->C_res) return TFORGE_ERR_NULL;
  const int ea = a->a_dtype == TFORGE_BF16 ? 2 : 4, eb = a->b_dtype == TFORGE_BF16 ? 2 : 4;
  const int eo = a->out_dtype == TFORGE_BF16 ? 2 : 4;
  if (!aligned(a->A, ea) || !aligned(a->B, eb) || !aligned(a->out, eo) || !aligned(a->bias, 4) ||
      !aligned(a->C_res, 4))
    return TFORGE_ERR_ALIGN;
  const size_t ob = span_bytes(a->M, a->N, *ldc, eo), cb = span_bytes(a->M, a->N, *ldc, 4);
  if (overlaps(a->out, ob, a->A, span_bytes(a->M, a->K, *lda, ea)) ||
      overlaps(a->out, ob, a->B, span_bytes(a->K, a->N, *ldb, eb)) ||
      (a->workload == TFORGE_MBR && overlaps(a->out, ob, a->bias, (size_t)a->N * 4)) ||
      (a->workload == TFORGE_MATMUL_ADD && overlaps(a->out, ob, a->C_res, cb)))
    return TFORGE_ERR_ALIAS;
  return TFORGE_OK;
}

// TMA needs 16-byte-aligned bases and pitches; the vector epilogue needs 16-byte rows.  In
// BF16 mode an f32 operand is read once into a packed bf16 copy, so only its f32 rows need
// 16 bytes; a bf16 operand's own rows are checked with its element size.
bool tma_compatible(const tforge_gemm_args *a, int64_t lda, int64_t ldb, int64_t ldc) {
  const int ea = a->a_dtype == TFORGE_BF16 ? 2 : 4, eb = a->b_dtype == TFORGE_BF16 ? 2 : 4;
  const int eo = a->out_dtype == TFORGE_BF16 ? 2 : 4;
  if ((lda * ea) % 16 || (ldb * eb) % 16 || (ldc * eo) % 16) return false;
  if (!aligned(a->A, 16) || !aligned(a->B, 16) || !aligned(a->out, 16)) return false;
  if (a->workload == TFORGE_MBR && !aligned(a->bias, 16)) return false;
  if (a->workload == TFORGE_MATMUL_ADD && !aligned(a->C_res, 16)) return false;
  if (a->N % 4) return false;
  return true;
}

// SM pairs of the current device (148 SMs on a B200 when no device is visible).
int device_pairs() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    cudaGetLastError();
    return 74;
  }
  return sms / 2;
}

// Split-K factor of the CTA-pair kernel: tforge_config.split_k when set, else (fp32 and TF32
// modes) as many pairs per tile as fit one wave of SM pairs, at most 8 and at least 4
// k-blocks each.  BF16 never splits, forced or not (so the allocation-free BF16 entry, which
// has no workspace for partial sums, gives the same bits as tforge_mbr).
int pair_splits(const TcConfig &c, int64_t M, int64_t N, int64_t K) {
  if (!c.pair || c.prec == PREC_BF16) return 1;
  {
    std::lock_guard<std::mutex> lk(g_cfg_mu);
    if (g_cfg.kernel == 3 && g_cfg.split_k > 0) return g_cfg.split_k;
  }
  return c.bn == 256 && !c.persist ? auto_pair_splits(c.prec, M, N, K) : 1;
}

int auto_pair_splits(int prec, int64_t M, int64_t N, int64_t K) {
  if (prec == PREC_BF16) return 1;
  const int64_t tiles = ((M + 255) / 256) * ((N + 255) / 256);
  const int64_t kb = (K + 31) / 32;
  const int64_t pairs = device_pairs();
  if (tiles * 2 > pairs) return 1;
  int64_t sk = pairs / tiles;
  if (sk > kb / 4) sk = kb / 4;
  if (sk > 8) sk = 8;
  return sk >= 2 ? (int)sk : 1;
}

int run_tc(const tforge_gemm_args *a, const TcConfig &cfg, const void *A, const void *B,
           bool bf16, int64_t lda, int64_t ldb, int64_t ldc, cudaStream_t st, bool after_conversion = false) {
  const int esz = bf16 ? 2 : 4;
  const uint32_t bk = 128 / esz;  // K elements per stage
  CUtensorMap tmA, tmB;
  int rc = make_tmap(&tmA, A, bf16, a->M, a->K, lda, bk, 128);
  if (rc) return rc;
  rc = make_tmap(&tmB, B, bf16, a->K, a->N, ldb, 128 / esz, bk, bf16 ? SW128 : SW128_A32);
  if (rc) return rc;
  TcParams p{};
  p.bias = a->bias;
  p.cres = a->C_res;
  p.out = static_cast<float *>(a->out);  // bf16 output (out_bf16) is written through tmO only
  p.out_bf16 = a->out_dtype == TFORGE_BF16;
  const bool ob16 = p.out_bf16 != 0;
  p.M = (int32_t)a->M;
  p.N = (int32_t)a->N;
  p.K = (int32_t)a->K;
  p.ldc = ldc;
  rc = status_word(&p.status);
  if (rc) return rc;
  p.limit_ns = g_wait_limit_ns.load();
  p.debug_skip = g_debug_skip.load();
  // The operand conversion just launched on this stream wrote A and B: overlap this launch's
  // set-up with its tail (programmatic dependent launch).
  p.pdl = after_conversion ? 1 : 0;
  const int epi = a->workload == TFORGE_MBR ? EPI_MBR : (a->workload == TFORGE_MATMUL_ADD ? EPI_ADD : EPI_MATMUL);
  cudaError_t e;
  const int splits = pair_splits(cfg, a->M, a->N, a->K);
  // TF32, b_layout = 2 only: the MMAs read a transposed (K-major) copy of B made by one pass
  // over B.  It used to be the default from M = 16384 rows, when B as given was read in column
  // blocks; read as k-group-major tiles, B as given is as fast or faster at every size measured
  // (16384 x 8192 x 8192 618.5 vs 576.9 TFLOP/s, 16384 x 16384 x 4096 638.1 vs 602.3,
  // 32768 x 8192 x 8192 even; same box, interleaved) and needs no scratch.
  int b_layout = 0;
  {
    std::lock_guard<std::mutex> lk(g_cfg_mu);
    b_layout = g_cfg.b_layout;
  }
  bool bkm = !bf16 && cfg.prec == PREC_TF32 && ((cfg.pair && cfg.bn == 256) || cfg.persist) && a->K % 4 == 0 &&
             a->K <= 65535 * 32 &&  // the transpose kernel's grid
             b_layout == 2;
  void *bt = nullptr;
  if (bkm) {
    cudaMemPool_t pool = nullptr;
    rc = scratch_pool(&pool);
    if (rc) return rc;
    cudaError_t e2 = cudaMallocFromPoolAsync(&bt, sizeof(float) * (size_t)a->N * a->K, pool, st);
    if (e2 != cudaSuccess) {  // no room for the copy: read B as given
      cudaGetLastError();
      bt = nullptr;
      bkm = false;
    }
  }
  if (bkm) {
    cudaError_t e2 = launch_transpose_f32(static_cast<const float *>(B), ldb, static_cast<float *>(bt), a->K, a->K, a->N, st);
    if (e2 == cudaSuccess) rc = make_tmap(&tmB, bt, false, a->N, a->K, a->K, bk, 128);
    if (e2 != cudaSuccess || rc) {
      cudaFreeAsync(bt, st);
      return rc ? rc : cuda_fail(e2, "B transpose");
    }
    p.b_kmajor = 1;
    p.pdl = 1;  // the GEMM sets up while the transpose finishes
  }
  // TF32, B as given, on the 256-wide pair tiles or the persistent pair kernel: B is read
  // through the k-group-major tiling when its shape allows it (one 4-D box per tile; same
  // results), which the tensor core takes faster for a 32-bit MN-major operand.  The same
  // tiling measured 4-6 % slower for BF16 and even for 3xTF32, which keep column blocks, as does
  // tforge_config.b_layout = 3.
  if (!bkm && cfg.prec == PREC_TF32 && ((cfg.pair && cfg.bn == 256) || cfg.persist) && b_layout != 3 &&
      a->N % 32 == 0 && a->K % 4 == 0) {
    rc = make_tmap_b_atoms(&tmB, B, a->K, a->N, ldb);
    if (rc) return rc;
    p.b_atoms = 1;
  }
  // The copy is released (stream-ordered) after the launches below, on every return path.
  struct PoolRelease {
    void *ptr;
    cudaStream_t stream;
    ~PoolRelease() {
      if (ptr) cudaFreeAsync(ptr, stream);
    }
  } bt_release{bt, st};
  // Pair kernels that accumulate the transposed tile store 32-row x 128-column boxes.
  const bool swapped = cfg.pair && !cfg.persist && !bkm && pair_transposed(cfg.prec, cfg.bn);
  if (cfg.pair && splits > 1) {
    // Split-K: raw partial sums of each k-range into slice z of a pooled workspace (rows
    // padded to whole tiles so no tile crosses a slice), then one pass sums the slices in
    // order and applies the epilogue.
    const int64_t mp = (a->M + 255) / 256 * 256;
    cudaMemPool_t pool = nullptr;
    rc = scratch_pool(&pool);
    if (rc) return rc;
    void *ws = nullptr;
    cudaError_t e2 = cudaMallocFromPoolAsync(&ws, sizeof(float) * (size_t)splits * mp * a->N, pool, st);
    if (e2 != cudaSuccess) return cuda_fail(e2, "cudaMallocFromPoolAsync(split-K workspace)");
    CUtensorMap tmW;
    rc = swapped ? make_tmap(&tmW, ws, false, splits * mp, a->N, a->N, 128, 32, SWNONE)
                 : make_tmap(&tmW, ws, false, splits * mp, a->N, a->N, 32, 128);
    if (rc) {
      cudaFreeAsync(ws, st);
      return rc;
    }
    p.splits = splits;
    p.split_rows = (int32_t)mp;
    e = launch_gemm_pair(cfg.prec, cfg.stages, cfg.bn, EPI_MATMUL, tmA, tmB, tmW, tmW, p, st);
    if (e == cudaSuccess)
      e = launch_splitk_reduce(epi, static_cast<const float *>(ws), splits, mp * a->N, a->M, a->N, a->bias, a->C_res,
                               static_cast<float *>(a->out), ldc, st);
    cudaFreeAsync(ws, st);
  } else if (cfg.persist) {
    CUtensorMap tmO;
    rc = !bkm && persist_transposed(cfg.prec) ? make_tmap(&tmO, a->out, false, a->M, a->N, ldc, 128, 32, SWNONE)
                                               : make_tmap(&tmO, a->out, ob16, a->M, a->N, ldc, 32, 128, ob16 ? SW64 : SW128);
    if (rc) return rc;
    e = launch_gemm_pair_persistent(cfg.prec, cfg.stages, epi, tmA, tmB, tmO, p, st);
  } else if (cfg.pair) {
    CUtensorMap tmO, tmC;
    rc = swapped ? make_tmap(&tmO, a->out, false, a->M, a->N, ldc, 128, 32, SWNONE)
                 : make_tmap(&tmO, a->out, ob16, a->M, a->N, ldc, 32, 128, ob16 ? SW64 : SW128);
    if (rc) return rc;
    tmC = tmO;
    if (a->workload == TFORGE_MATMUL_ADD) {
      rc = swapped ? make_tmap(&tmC, a->C_res, false, a->M, a->N, ldc, 128, 32, SWNONE)
                   : make_tmap(&tmC, a->C_res, false, a->M, a->N, ldc, 32, 128);
      if (rc) return rc;
    }
    e = launch_gemm_pair(cfg.prec, cfg.stages, cfg.bn, epi, tmA, tmB, tmO, tmC, p, st);
  } else {
    e = launch_gemm_tc(cfg, epi, tmA, tmB, p, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 GEMM launch");
  return TFORGE_OK;
}

}  // namespace

namespace tf {

// The tensor-core configuration tforge_gemm picks for (mode, M, N, K) with TMA-compatible
// operands, or false when it would not use a tensor-core kernel.
bool select_tc_config(int mode, int64_t M, int64_t N, int64_t K, TcConfig *out) {
  const Choice c = choose(mode, M, N, K, true);
  if (c.kind != K_TC) return false;
  *out = c.tc;
  return true;
}

int encode_operand_map(CUtensorMap *m, const void *base, bool bf16, int64_t rows, int64_t cols,
                       int64_t ld, uint32_t box_cols, uint32_t box_rows, bool atom32) {
  return make_tmap(m, base, bf16, rows, cols, ld, box_cols, box_rows, atom32 ? SW128_A32 : SW128);
}

void set_last_error(const char *msg) { g_last_error = msg; }

int check_gemm_args(const tforge_gemm_args *a, int64_t *lda, int64_t *ldb, int64_t *ldc) {
  return check_gemm(a, lda, ldb, ldc);
}

int device_pool(cudaMemPool_t *out) { return scratch_pool(out); }

uint64_t wait_limit_ns() { return g_wait_limit_ns.load(); }
int debug_skip_load() { return g_debug_skip.load(); }

}  // namespace tf

namespace {

// bf16 output on a path without a bf16-output epilogue: the f32 result goes to pooled scratch
// (packed), then one pass rounds it into out with the same conversion the epilogues use.
int gemm_bf16_out_via_f32(const tforge_gemm_args *a, int64_t ldc, cudaStream_t st) {
  cudaMemPool_t pool = nullptr;
  int rc = scratch_pool(&pool);
  if (rc) return rc;
  void *tmp = nullptr;
  cudaError_t e = cudaMallocFromPoolAsync(&tmp, sizeof(float) * (size_t)a->M * a->N, pool, st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMallocFromPoolAsync(f32 output scratch)");
  tforge_gemm_args t = *a;
  t.out = tmp;
  t.ldc = a->N;
  t.out_dtype = TFORGE_F32;
  rc = tforge_gemm(&t, st);
  if (rc == TFORGE_OK) {
    e = launch_convert_rows_bf16(static_cast<const float *>(tmp), a->N, static_cast<uint16_t *>(a->out), ldc, a->M,
                                 a->N, st);
    if (e != cudaSuccess) rc = cuda_fail(e, "bf16 output conversion");
  }
  cudaFreeAsync(tmp, st);
  return rc;
}

}  // namespace

extern "C" {

int tforge_gemm(const tforge_gemm_args *a, void *stream) {
  int64_t lda, ldb, ldc;
  int rc = check_gemm(a, &lda, &ldb, &ldc);
  if (rc) return rc;
  if (a->M == 0 || a->N == 0) return TFORGE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int epi = a->workload == TFORGE_MBR ? EPI_MBR : (a->workload == TFORGE_MATMUL_ADD ? EPI_ADD : EPI_MATMUL);
  const bool f32_in = a->a_dtype == TFORGE_F32 && a->b_dtype == TFORGE_F32;
  const Choice c = choose(a->mode, a->M, a->N, a->K, tma_compatible(a, lda, ldb, ldc));
  if (c.kind < 0) return TFORGE_ERR_UNSUPPORTED;
  if (a->out_dtype == TFORGE_BF16) {
    // Direct bf16 stores from the mbr epilogue of the 256-wide and persistent BF16 pair
    // kernels (K and N multiples of 8 keep the bf16 operand rows TMA-aligned).
    const bool direct = c.kind == K_TC && c.tc.prec == PREC_BF16 && epi == EPI_MBR &&
                        (c.tc.persist || (c.tc.pair && c.tc.bn == 256)) && a->K % 8 == 0 && a->N % 8 == 0 &&
                        pair_splits(c.tc, a->M, a->N, a->K) <= 1;  // a forced split-K reduces in f32
    if (!direct) return gemm_bf16_out_via_f32(a, ldc, st);
  }
  if (c.kind == K_SIMT) {
    if (!f32_in) return TFORGE_ERR_UNSUPPORTED;  // bf16 operands need the tensor-core path
    const float *aux = a->workload == TFORGE_MBR ? a->bias : a->C_res;
    cudaError_t e = launch_gemm_simt(epi, static_cast<const float *>(a->A),
                                     static_cast<const float *>(a->B), aux, static_cast<float *>(a->out), a->M, a->N, a->K,
                                     lda, ldb, ldc, st);
    return e == cudaSuccess ? TFORGE_OK : cuda_fail(e, "SIMT GEMM launch");
  }
  if (c.tc.prec != PREC_BF16) return run_tc(a, c.tc, a->A, a->B, false, lda, ldb, ldc, st);

  // BF16 mode: f32 operands are rounded to bf16 into stream-ordered scratch first.
  const void *A = a->A, *B = a->B;
  void *scratch = nullptr;
  int64_t la = lda, lb = ldb;
  const size_t abytes = a->a_dtype == TFORGE_F32 ? (size_t)a->M * a->K * 2 : 0;
  const size_t bbytes = a->b_dtype == TFORGE_F32 ? (size_t)a->K * a->N * 2 : 0;
  if (abytes + bbytes) {
    cudaMemPool_t pool = nullptr;
    rc = scratch_pool(&pool);
    if (rc) return rc;
    cudaError_t e = cudaMallocFromPoolAsync(&scratch, abytes + bbytes + 256, pool, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMallocFromPoolAsync(bf16 scratch)");
    uint16_t *sa = static_cast<uint16_t *>(scratch);
    uint16_t *sb = reinterpret_cast<uint16_t *>(static_cast<char *>(scratch) + ((abytes + 255) & ~size_t(255)));
    if (abytes && bbytes && lda == a->K && ldb == a->N) {
      // Both operands packed: one launch converts both.
      e = launch_convert_bf16_two(static_cast<const float *>(a->A), sa, a->M * a->K, static_cast<const float *>(a->B), sb,
                                  a->K * a->N, st);
      A = sa;
      la = a->K;
      B = sb;
      lb = a->N;
    } else if (abytes) {
      // Packed bf16 copy of a possibly pitched A (one launch either way).
      e = lda == a->K ? launch_convert_bf16(static_cast<const float *>(a->A), sa, a->M * a->K, st)
                      : launch_convert_rows_bf16(static_cast<const float *>(a->A), lda, sa, a->K, a->M, a->K, st);
      A = sa;
      la = a->K;
    }
    if (bbytes && B != sb && e == cudaSuccess) {
      e = ldb == a->N ? launch_convert_bf16(static_cast<const float *>(a->B), sb, a->K * a->N, st)
                      : launch_convert_rows_bf16(static_cast<const float *>(a->B), ldb, sb, a->N, a->K, a->N, st);
      B = sb;
      lb = a->N;
    }
    if (e != cudaSuccess) {
      cudaFreeAsync(scratch, st);
      return cuda_fail(e, "bf16 conversion");
    }
  }
  if ((la * 2) % 16 || (lb * 2) % 16) {
    if (scratch) cudaFreeAsync(scratch, st);
    // bf16 rows must be 16-byte multiples for TMA: K and N multiples of 8.
    const float *aux = a->workload == TFORGE_MBR ? a->bias : a->C_res;
    if (!f32_in) return TFORGE_ERR_UNSUPPORTED;
    cudaError_t e = launch_gemm_simt(epi, static_cast<const float *>(a->A),
                                     static_cast<const float *>(a->B), aux, static_cast<float *>(a->out), a->M, a->N,
                                     a->K, lda, ldb, ldc, st);
    return e == cudaSuccess ? TFORGE_OK : cuda_fail(e, "SIMT GEMM launch");
  }
  rc = run_tc(a, c.tc, A, B, true, la, lb, ldc, st, scratch != nullptr);
  if (scratch) cudaFreeAsync(scratch, st);
  return rc;
}

int tforge_matmul(const float *A, const float *B, float *out, int64_t M, int64_t N, int64_t K,
                  int mode, void *stream) {
  tforge_gemm_args a{TFORGE_MATMUL, mode, TFORGE_F32, TFORGE_F32, A, B, nullptr, nullptr, out, M, N, K, 0, 0, 0};
  return tforge_gemm(&a, stream);
}

int tforge_mbr(const float *A, const float *B, const float *bias, float *out, int64_t M, int64_t N,
               int64_t K, int mode, void *stream) {
  tforge_gemm_args a{TFORGE_MBR, mode, TFORGE_F32, TFORGE_F32, A, B, bias, nullptr, out, M, N, K, 0, 0, 0};
  return tforge_gemm(&a, stream);
}

int tforge_matmul_add(const float *A, const float *B, const float *C_res, float *out, int64_t M,
                      int64_t N, int64_t K, int mode, void *stream) {
  tforge_gemm_args a{TFORGE_MATMUL_ADD, mode, TFORGE_F32, TFORGE_F32, A, B, nullptr, C_res, out, M, N, K, 0, 0, 0};
  return tforge_gemm(&a, stream);
}

static int elementwise(int op, const float *X, const float *Y, float *Z, int64_t M, int64_t N,
                       void *stream) {
  if (M < 0 || N < 0) return TFORGE_ERR_SHAPE;
  if (M == 0 || N == 0) return TFORGE_OK;
  if (!X || !Z || (op != 1 && !Y)) return TFORGE_ERR_NULL;
  if (!aligned(X, 4) || !aligned(Z, 4) || !aligned(Y, 4)) return TFORGE_ERR_ALIGN;
  const size_t zb = (size_t)M * N * 4;
  if (overlaps(Z, zb, X, zb) || (op == 0 && overlaps(Z, zb, Y, zb)) ||
      (op == 2 && overlaps(Z, zb, Y, (size_t)N * 4)))
    return TFORGE_ERR_ALIAS;
  cudaError_t e = launch_elementwise(op, X, Y, Z, M, N, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TFORGE_OK : cuda_fail(e, "elementwise launch");
}

int tforge_bias_add(const float *X, const float *bias, float *Y, int64_t M, int64_t N, void *stream) {
  return elementwise(2, X, bias, Y, M, N, stream);
}
int tforge_relu(const float *X, float *Y, int64_t M, int64_t N, void *stream) {
  return elementwise(1, X, nullptr, Y, M, N, stream);
}
int tforge_add(const float *X, const float *Y, float *Z, int64_t M, int64_t N, void *stream) {
  return elementwise(0, X, Y, Z, M, N, stream);
}

int tforge_convert_bf16(const float *x, uint16_t *y, int64_t n, void *stream) {
  if (n < 0) return TFORGE_ERR_SHAPE;
  if (n == 0) return TFORGE_OK;
  if (!x || !y) return TFORGE_ERR_NULL;
  if (!aligned(x, 4) || !aligned(y, 2)) return TFORGE_ERR_ALIGN;
  if (overlaps(x, (size_t)n * 4, y, (size_t)n * 2)) return TFORGE_ERR_ALIAS;
  cudaError_t e = launch_convert_bf16(x, y, n, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TFORGE_OK : cuda_fail(e, "bf16 conversion");
}

int tforge_describe(int workload, int64_t M, int64_t N, int64_t K, int mode, tforge_launch *out) {
  if (!out) return TFORGE_ERR_NULL;
  if (M < 0 || N < 0 || K < 0) return TFORGE_ERR_SHAPE;
  if (mode < TFORGE_MODE_FP32 || mode > TFORGE_MODE_FP32_EXACT) return TFORGE_ERR_MODE;
  std::memset(out, 0, sizeof(*out));
  out->cluster[0] = out->cluster[1] = out->cluster[2] = 1;
  out->mode = mode;
  out->split_k = 1;
  out->regs = out->static_smem = out->blocks_per_sm = -1;
  const int epi = workload == TFORGE_MBR ? EPI_MBR : (workload == TFORGE_MATMUL_ADD ? EPI_ADD : EPI_MATMUL);
  int ndev = 0;
  const bool have_dev = cudaGetDeviceCount(&ndev) == cudaSuccess && ndev > 0;
  auto fill_attrs = [&](cudaError_t e, const cudaFuncAttributes &fa, int blocks) {
    if (e != cudaSuccess) {
      cudaGetLastError();
      return;
    }
    out->regs = fa.numRegs;
    out->static_smem = (int)fa.sharedSizeBytes;
    out->blocks_per_sm = blocks;
  };
  if (workload >= TFORGE_BIAS_ADD && workload <= TFORGE_ADD) {
    std::snprintf(out->kernel, sizeof(out->kernel), "tf_elementwise");
    out->block[0] = 256;
    out->block[1] = out->block[2] = 1;
    const int64_t n4 = (M * N + 3) / 4;
    int64_t g = (n4 + 255) / 256;
    out->grid[0] = (int)(g > 148 * 16 ? 148 * 16 : (g < 1 ? 1 : g));
    out->grid[1] = out->grid[2] = 1;
    return TFORGE_OK;
  }
  if (workload < TFORGE_MATMUL || workload > TFORGE_MATMUL_ADD) return TFORGE_ERR_MODE;
  const bool tma_ok = (K % 4 == 0) && (N % 4 == 0) && (mode != TFORGE_MODE_BF16 || (K % 8 == 0 && N % 8 == 0));
  const Choice c = choose(mode, M, N, K, tma_ok);
  if (c.kind < 0) return TFORGE_ERR_UNSUPPORTED;
  if (c.kind == K_SIMT) {
    std::snprintf(out->kernel, sizeof(out->kernel), "tf_gemm_simt_ffma");
    int smem = 0;
    simt_launch_shape(M, N, out->grid, out->block, &smem);
    out->smem_bytes = smem;
    out->tile[0] = out->tile[1] = simt_tile_size(M, N);
    out->tile[2] = 8;
    out->stages = 2;
    out->mode = TFORGE_MODE_FP32_EXACT;
    if (have_dev) {
      cudaFuncAttributes fa{};
      int blocks = 0;
      cudaError_t e = simt_func_attributes(epi, &fa, &blocks);
      fill_attrs(e, fa, blocks);
    }
    return TFORGE_OK;
  }
  static const char *names[3] = {"tf_gemm_tcgen05_tf32", "tf_gemm_tcgen05_3xtf32", "tf_gemm_tcgen05_bf16"};
  std::snprintf(out->kernel, sizeof(out->kernel), "%s%s", names[c.tc.prec],
                c.tc.persist ? "_pair_persistent" : (c.tc.pair ? "_pair" : ""));
  const int tm = c.tc.pair ? 256 : 128;
  out->grid[0] = (int)((N + c.tc.bn - 1) / c.tc.bn) * (c.tc.pair ? 2 : 1);
  out->grid[1] = (int)((M + tm - 1) / tm);
  out->grid[2] = 1;
  if (c.tc.persist) {  // one cluster per co-resident pair, each looping over tiles
    const int64_t tiles = (int64_t)out->grid[0] / 2 * out->grid[1];
    int pairs = have_dev ? persist_grid_pairs(c.tc.prec, c.tc.stages, epi, M, N) : -1;
    if (pairs <= 0) pairs = (int)(tiles < device_pairs() ? tiles : device_pairs());
    out->grid[0] = 2 * pairs;
    out->grid[1] = 1;
    out->persistent = 1;
  }
  out->block[0] = c.tc.pair && c.tc.prec == PREC_X3 ? 384 : 256;  // 3xTF32 pair: 12 warps
  out->split_k = pair_splits(c.tc, M, N, K);
  out->grid[2] = out->split_k;
  out->block[1] = out->block[2] = 1;
  out->cluster[0] = c.tc.pair ? 2 : 1;
  out->smem_bytes = c.tc.persist ? persist_smem_bytes(c.tc.prec, c.tc.stages)
                                  : (c.tc.pair ? pair_smem_bytes(c.tc.prec, c.tc.stages) : tc_smem_bytes(c.tc));
  out->tile[0] = tm;
  out->tile[1] = c.tc.bn;
  out->tile[2] = c.tc.prec == PREC_BF16 ? 64 : 32;
  out->stages = c.tc.stages;
  out->tmem_cols = c.tc.persist ? 512 : (c.tc.pair ? pair_tmem_cols(c.tc.prec) : c.tc.bn);
  if (have_dev) {
    cudaFuncAttributes fa{};
    int blocks = 0;
    cudaError_t e = c.tc.persist ? persist_func_attributes(c.tc.prec, c.tc.stages, epi, &fa, &blocks)
                    : c.tc.pair  ? pair_func_attributes(c.tc.prec, c.tc.stages, c.tc.bn, epi, &fa, &blocks)
                                 : tc_func_attributes(c.tc, epi, &fa, &blocks);
    fill_attrs(e, fa, blocks);
  }
  return TFORGE_OK;
}

int tforge_set_config(const tforge_config *cfg) {
  std::lock_guard<std::mutex> lk(g_cfg_mu);
  if (!cfg) {
    g_cfg = tforge_config{};
    return TFORGE_OK;
  }
  if (cfg->kernel < 0 || cfg->kernel > 3 || cfg->split_k < 0 || cfg->split_k > 8 || cfg->persistent < 0 ||
      cfg->persistent > 1 || cfg->b_layout < 0 || cfg->b_layout > 3)
    return TFORGE_ERR_MODE;
  g_cfg = *cfg;
  return TFORGE_OK;
}

int tforge_device_status(void *stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  // Two words per device: the one tforge_gemm's kernels write (created by the first GEMM; a
  // device without one has nothing to report, and nothing is allocated here) and the one in
  // the allocation-free entry's static array.  Both are read and cleared.
  uint32_t v = 0;
  if (uint32_t *w = existing_status_word()) {
    e = cudaMemcpy(&v, w, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(status)");
    if (v) {
      e = cudaMemset(w, 0, 4);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(status)");
    }
  }
  uint32_t v2 = 0;
  const int rc = noalloc_take_status(&v2);
  if (rc) return rc;
  return (int)(v ? v : v2);
}

int tforge_set_wait_limit_ns(uint64_t ns) {
  g_wait_limit_ns.store(ns ? ns : 1000000000ull);
  return TFORGE_OK;
}

int tforge_debug_skip_load(int on) {
  g_debug_skip.store(on ? 1 : 0);
  return TFORGE_OK;
}

int tforge_debug_pool_usage(uint64_t *used_now, uint64_t *used_high, int reset_high) {
  if (!used_now || !used_high) return TFORGE_ERR_NULL;
  cudaMemPool_t pool = nullptr;
  int rc = scratch_pool(&pool);
  if (rc) return rc;
  cudaError_t e = cudaMemPoolGetAttribute(pool, cudaMemPoolAttrUsedMemCurrent, used_now);
  if (e == cudaSuccess) e = cudaMemPoolGetAttribute(pool, cudaMemPoolAttrUsedMemHigh, used_high);
  if (e == cudaSuccess && reset_high) {
    uint64_t zero = 0;
    e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrUsedMemHigh, &zero);
  }
  return e == cudaSuccess ? TFORGE_OK : cuda_fail(e, "cudaMemPoolGetAttribute");
}

const char *tforge_status_string(int s) {
  switch (s) {
    case TFORGE_OK: return "ok";
    case TFORGE_ERR_SHAPE: return "invalid shape or pitch";
    case TFORGE_ERR_ALIGN: return "misaligned pointer";
    case TFORGE_ERR_ALIAS: return "output overlaps an input";
    case TFORGE_ERR_MODE: return "unknown mode, workload or dtype";
    case TFORGE_ERR_CUDA: return "CUDA error";
    case TFORGE_ERR_TIMEOUT: return "device-side wait timed out";
    case TFORGE_ERR_NULL: return "null pointer";
    case TFORGE_ERR_UNSUPPORTED: return "unsupported configuration";
    case TFORGE_ERR_NOMEM: return "out of memory";
  }
  return "unknown status";
}

const char *tforge_last_error(void) { return g_last_error.c_str(); }
const char *tforge_version(void) { return "tforge-b200 0.1 (sm_100a)"; }

int tforge_malloc(void **ptr, uint64_t bytes) {
  if (!ptr) return TFORGE_ERR_NULL;
  cudaError_t e = cudaMalloc(ptr, bytes ? bytes : 1);
  return e == cudaSuccess ? TFORGE_OK : cuda_fail(e, "cudaMalloc");
}
int tforge_free(void *ptr) {
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? TFORGE_OK : cuda_fail(e, "cudaFree");
}
int tforge_memcpy_h2d(void *dst, const void *src, uint64_t bytes, void *stream) {
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TFORGE_OK : cuda_fail(e, "cudaMemcpyAsync(H2D)");
}
int tforge_memcpy_d2h(void *dst, const void *src, uint64_t bytes, void *stream) {
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TFORGE_OK : cuda_fail(e, "cudaMemcpyAsync(D2H)");
}
int tforge_memset(void *dst, int byte, uint64_t bytes, void *stream) {
  cudaError_t e = cudaMemsetAsync(dst, byte, bytes, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TFORGE_OK : cuda_fail(e, "cudaMemsetAsync");
}
int tforge_stream_sync(void *stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TFORGE_OK : cuda_fail(e, "cudaStreamSynchronize");
}
int tforge_device_count(int *n) {
  if (!n) return TFORGE_ERR_NULL;
  cudaError_t e = cudaGetDeviceCount(n);
  if (e != cudaSuccess) {
    *n = 0;
    return cuda_fail(e, "cudaGetDeviceCount");
  }
  return TFORGE_OK;
}
int tforge_set_device(int dev) {
  cudaError_t e = cudaSetDevice(dev);
  return e == cudaSuccess ? TFORGE_OK : cuda_fail(e, "cudaSetDevice");
}

}  // extern "C"
