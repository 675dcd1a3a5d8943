// tforge-gpu-bench (B200 build): run, check and time a TensorForge operator.
//
// Same command line and JSON object as the reference runner
// (runners/gpu/tforge-gpu-bench.cu:8-27,370-382), with `--mode lib` in place of
// `--mode kernel`: instead of loading a generated cubin and marshalling `--args`, it calls
// the library's C-ABI (include/tforge.h), which picks and launches the sm_100a kernel.
//
//   tforge-gpu-bench --mode lib --workload mbr --m M --n N --k K [--precision fp32|tf32|bf16|fp32_exact]
//       [--kernel pair|cta|simt --bn 256 --stages 4 --split S --persistent --b-layout L] [--warmup 10 --reps 100 --flush]
//       [--in-dir d --out o.bin] [--seed S] [--operands bf16]
//     --operands bf16 (BF16 precision): A and B rounded to bf16 once before timing and passed
//     as bf16 (tforge_gemm, a_dtype = b_dtype = TFORGE_BF16), so only the GEMM is timed.
//   tforge-gpu-bench --mode cublas --workload mbr --m M --n N --k K
//       [--math default|tf32|bf16|bf16x9|lt|lt_tf32|lt_bf16]
//     default: cublasSgemm (FP32 FMA) + separate bias/relu -- the reference's comparator;
//     tf32 / bf16: TF32 tensor-op math / bf16 inputs with f32 accumulation;
//     bf16x9: FP32 emulated on bf16 tensor cores (CUBLAS_COMPUTE_32F_EMULATED_16BFX9, eager);
//     lt / lt_tf32: cuBLASLt FP32 / TF32 with the bias + relu fused into its epilogue;
//     lt_bf16: cuBLASLt on bf16 copies of A and B made once before timing (f32 accumulate and
//     output, fused bias + relu) -- the counterpart of `--mode lib --precision bf16 --operands bf16`.
//   tforge-gpu-bench ... --info-only        (launch description and occupancy, no run)
//
// Buffers follow the host entry's argument order (runners/gpu/tforge-gpu-bench.cu:20-24):
//   matmul: A B C; mbr: A B bias C; matmul_add: A B C_res C; bias_add: X bias Y; relu: X Y;
//   add: X Y Z.  Inputs are read from --in-dir/<a|b|bias|c|y>.bin or drawn from
// mt19937(seed) U[-1,1] in the reference's order.  Timing: CUDA events around each rep
// on one stream, warm-up reps untimed, optional 256 MiB L2 flush outside the timed
// region, NVML SM clock and power sampled after every rep (loaded at run time).
#include <cublasLt.h>
#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <random>
#include <sstream>
#include <string>
#include <vector>

#include "tforge.h"

namespace {

void die(const std::string &m) {
  std::fprintf(stderr, "tforge-gpu-bench: %s\n", m.c_str());
  std::exit(1);
}
void cuda_ok(cudaError_t r, const char *what) {
  if (r != cudaSuccess) die(std::string(what) + ": " + cudaGetErrorString(r));
}
void tf_ok(int rc, const char *what) {
  if (rc != TFORGE_OK)
    die(std::string(what) + ": " + tforge_status_string(rc) +
        (rc == TFORGE_ERR_CUDA ? std::string(" (") + tforge_last_error() + ")" : ""));
}
void blas_ok(cublasStatus_t r, const char *what) {
  if (r != CUBLAS_STATUS_SUCCESS) die(std::string(what) + ": cuBLAS status " + std::to_string(r));
}

struct Args {
  std::string mode = "lib", workload, inDir, out, precision = "fp32", math = "default", kernel,
              operands = "f32";
  long m = 0, n = 0, k = 0;
  int warmup = 10, reps = 100, bn = 0, stages = 0, split = 0, persistent = 0, b_layout = 0;
  bool flush = false, infoOnly = false;
  unsigned seed = 1234;
};

Args parse(int argc, char **argv) {
  Args a;
  for (int i = 1; i < argc; ++i) {
    std::string f = argv[i];
    auto next = [&]() -> std::string {
      if (i + 1 >= argc) die("missing value for " + f);
      return argv[++i];
    };
    if (f == "--mode") a.mode = next();
    else if (f == "--workload") a.workload = next();
    else if (f == "--m") a.m = std::stol(next());
    else if (f == "--n") a.n = std::stol(next());
    else if (f == "--k") a.k = std::stol(next());
    else if (f == "--precision") a.precision = next();
    else if (f == "--math") a.math = next();
    else if (f == "--bn") a.bn = std::stoi(next());
    else if (f == "--kernel") a.kernel = next();
    else if (f == "--operands") a.operands = next();
    else if (f == "--stages") a.stages = std::stoi(next());
    else if (f == "--split") a.split = std::stoi(next());
    else if (f == "--persistent") a.persistent = 1;
    else if (f == "--b-layout") a.b_layout = std::stoi(next());
    else if (f == "--warmup") a.warmup = std::stoi(next());
    else if (f == "--reps") a.reps = std::stoi(next());
    else if (f == "--flush") a.flush = true;
    else if (f == "--info-only") a.infoOnly = true;
    else if (f == "--in-dir") a.inDir = next();
    else if (f == "--out") a.out = next();
    else if (f == "--seed") a.seed = std::stoul(next());
    else die("unknown flag " + f);
  }
  static const char *wl[] = {"matmul", "mbr", "matmul_add", "bias_add", "relu", "add"};
  if (std::find(std::begin(wl), std::end(wl), a.workload) == std::end(wl))
    die("--workload matmul|mbr|matmul_add|bias_add|relu|add");
  const bool gemm = a.workload == "matmul" || a.workload == "mbr" || a.workload == "matmul_add";
  if (a.m <= 0 || a.n <= 0 || (gemm && a.k < 0)) die("need --m --n (and --k)");
  if (!gemm) a.k = 1;
  if (a.mode != "lib" && a.mode != "cublas") die("--mode lib|cublas");
  if (!gemm && a.mode == "cublas") die("cublas mode needs matmul, mbr or matmul_add");
  return a;
}

int precision_mode(const std::string &p) {
  if (p == "fp32") return TFORGE_MODE_FP32;
  if (p == "tf32") return TFORGE_MODE_TF32;
  if (p == "bf16") return TFORGE_MODE_BF16;
  if (p == "fp32_exact") return TFORGE_MODE_FP32_EXACT;
  die("--precision fp32|tf32|bf16|fp32_exact");
  return 0;
}

int workload_id(const std::string &w) {
  if (w == "matmul") return TFORGE_MATMUL;
  if (w == "mbr") return TFORGE_MBR;
  if (w == "matmul_add") return TFORGE_MATMUL_ADD;
  if (w == "bias_add") return TFORGE_BIAS_ADD;
  if (w == "relu") return TFORGE_RELU;
  return TFORGE_ADD;
}

// relu(C + bias) as a separate kernel after cuBLAS: the reference's unfused baseline
// (runners/gpu/tforge-gpu-bench.cu:143-146) with fmaxf, which maps NaN to 0.
__global__ void bias_relu(float *c, const float *bias, long m, long n) {
  long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i < m * n) c[i] = fmaxf(c[i] + bias[i % n], 0.0f);
}
__global__ void add_inplace(float *c, const float *r, long total) {
  long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i < total) c[i] = c[i] + r[i];
}
__global__ void to_bf16(const float *x, __nv_bfloat16 *y, long n) {
  long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2bfloat16_rn(x[i]);
}

// Per-rep samples reduced to the JSON's figures: median (mean of the two middle samples when
// the count is even), minimum, mean and sample standard deviation (Welford's running update);
// all -1 for no samples.
struct Summary {
  double median = -1, min = -1, mean = -1, sd = -1;
};
Summary summarize(const std::vector<double> &samples) {
  Summary r;
  const size_t n = samples.size();
  if (n == 0) return r;
  std::vector<double> work(samples);
  auto mid = work.begin() + n / 2;
  std::nth_element(work.begin(), mid, work.end());
  r.median = (n & 1) ? *mid : 0.5 * (*mid + *std::max_element(work.begin(), mid));
  r.min = *std::min_element(samples.begin(), samples.end());
  double mean = 0, m2 = 0;
  size_t count = 0;
  for (double x : samples) {
    ++count;
    const double d = x - mean;
    mean += d / count;
    m2 += d * (x - mean);
  }
  r.mean = mean;
  r.sd = n > 1 ? std::sqrt(m2 / (n - 1)) : 0.0;
  return r;
}

void fill(std::vector<float> &v, const Args &a, const char *name, std::mt19937 &rng) {
  if (!a.inDir.empty()) {
    std::ifstream f(a.inDir + "/" + name + ".bin", std::ios::binary);
    if (!f) die(std::string("cannot read ") + name);
    f.read(reinterpret_cast<char *>(v.data()), v.size() * sizeof(float));
    if ((size_t)f.gcount() != v.size() * sizeof(float)) die(std::string("short read ") + name);
    return;
  }
  std::uniform_real_distribution<float> d(-1.0f, 1.0f);
  for (float &x : v) x = d(rng);
}

// NVML through dlopen: the runner works (without clocks) where NVML is absent.
struct Nvml {
  void *h = nullptr, *dev = nullptr;
  int (*clock)(void *, int, unsigned *) = nullptr;
  int (*power)(void *, unsigned *) = nullptr;
  bool ok = false;
  Nvml() {
    h = dlopen("libnvidia-ml.so.1", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
    auto init = reinterpret_cast<int (*)()>(dlsym(h, "nvmlInit_v2"));
    auto get = reinterpret_cast<int (*)(unsigned, void **)>(dlsym(h, "nvmlDeviceGetHandleByIndex_v2"));
    clock = reinterpret_cast<int (*)(void *, int, unsigned *)>(dlsym(h, "nvmlDeviceGetClockInfo"));
    power = reinterpret_cast<int (*)(void *, unsigned *)>(dlsym(h, "nvmlDeviceGetPowerUsage"));
    int cur = 0;
    cudaGetDevice(&cur);
    ok = init && get && clock && power && init() == 0 && get((unsigned)cur, &dev) == 0;
  }
};

}  // namespace

int main(int argc, char **argv) {
  Args a = parse(argc, argv);
  const long M = a.m, N = a.n, K = a.k;
  const int wl = workload_id(a.workload);
  const int mode = precision_mode(a.precision);
  const bool gemm = wl <= TFORGE_MATMUL_ADD;

  if (a.bn || a.stages || a.split || a.persistent || a.b_layout || !a.kernel.empty()) {
    // --kernel pair|cta|simt forces a kernel family (offline tuning); --bn/--stages refine it;
    // --split S sets the pair kernel's split-K factor and --persistent picks the persistent
    // pair kernel (both imply --kernel pair).
    int kind = 1;
    if (a.kernel == "pair" || ((a.split || a.persistent) && a.kernel.empty())) kind = 3;
    else if (a.kernel.empty() && !a.bn && !a.stages) kind = 0;  // --b-layout alone: the table's kernel
    else if (a.kernel == "simt") kind = 2;
    else if (!a.kernel.empty() && a.kernel != "cta") die("--kernel pair|cta|simt");
    tforge_config cfg{kind, a.bn, a.stages, a.persistent, a.split, a.b_layout};
    tf_ok(tforge_set_config(&cfg), "tforge_set_config");
  }
  tforge_launch L{};
  tf_ok(tforge_describe(wl, M, N, K, mode, &L), "tforge_describe");
  if (a.infoOnly) {
    std::printf("{\"kernel\": \"%s\", \"grid\": \"%dx%dx%d\", \"block\": \"%dx%dx%d\", "
                "\"regs\": %d, \"local_bytes\": 0, \"static_smem\": %d, \"dyn_smem\": %d, "
                "\"blocks_per_sm\": %d, \"theo_occupancy\": %.3f, \"threads\": %d, \"tile\": \"%dx%dx%d\", "
                "\"stages\": %d, \"tmem_cols\": %d}\n",
                L.kernel, L.grid[0], L.grid[1], L.grid[2], L.block[0], L.block[1], L.block[2], L.regs,
                L.static_smem, L.smem_bytes, L.blocks_per_sm,
                L.blocks_per_sm > 0 ? L.blocks_per_sm * (L.block[0] / 32) / 64.0 : -1.0, L.block[0],
                L.tile[0], L.tile[1], L.tile[2], L.stages, L.tmem_cols);
    return 0;
  }

  cuda_ok(cudaSetDevice(0), "cudaSetDevice");
  cudaDeviceProp prop{};
  cuda_ok(cudaGetDeviceProperties(&prop, 0), "cudaGetDeviceProperties");

  // Host inputs in the reference's draw order (a, b, bias), then c for matmul_add.
  std::mt19937 rng(a.seed);
  const bool elementwise = !gemm;
  std::vector<float> hA(elementwise ? M * N : M * K), hB, hBias, hC(M * N), hRes;
  fill(hA, a, "a", rng);
  if (gemm) {
    hB.resize(K * N);
    fill(hB, a, "b", rng);
  }
  if (wl == TFORGE_MBR || wl == TFORGE_BIAS_ADD) {
    hBias.resize(N);
    fill(hBias, a, "bias", rng);
  }
  if (wl == TFORGE_MATMUL_ADD) {
    hRes.resize(M * N);
    fill(hRes, a, "c", rng);
  }
  if (wl == TFORGE_ADD) {
    hB.resize(M * N);
    fill(hB, a, "b", rng);
  }
  auto upload = [](const std::vector<float> &h) -> float * {
    if (h.empty()) return nullptr;
    float *d = nullptr;
    cuda_ok(cudaMalloc(&d, h.size() * 4), "cudaMalloc");
    cuda_ok(cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice), "cudaMemcpy");
    return d;
  };
  float *dA = upload(hA), *dB = upload(hB), *dBias = upload(hBias), *dRes = upload(hRes), *dC = nullptr;
  cuda_ok(cudaMalloc(&dC, hC.size() * 4), "cudaMalloc(C)");

  cudaStream_t stream;
  cuda_ok(cudaStreamCreate(&stream), "cudaStreamCreate");
  std::function<void()> run;
  cublasHandle_t blas = nullptr;
  __nv_bfloat16 *abf = nullptr, *bbf = nullptr;
  cublasLtHandle_t lt = nullptr;
  cublasLtMatmulDesc_t ltDesc = nullptr;
  cublasLtMatrixLayout_t ltA = nullptr, ltB = nullptr, ltC = nullptr;
  cublasLtMatmulHeuristicResult_t ltHeur{};
  void *ltWs = nullptr;
  std::string kernel = L.kernel;

  // --operands bf16 (lib mode, BF16 precision, GEMM workloads): A and B are rounded to bf16
  // once, before timing, and each call passes the bf16 copies (tforge_gemm with a_dtype =
  // b_dtype = TFORGE_BF16), so only the GEMM is timed; the output is the same bits as the
  // call on f32 operands.
  if (a.operands != "f32" && a.operands != "bf16") die("--operands f32|bf16");
  const bool bf16_ops = a.operands == "bf16";
  if (bf16_ops && (a.mode != "lib" || !gemm || mode != TFORGE_MODE_BF16))
    die("--operands bf16 needs --mode lib, a GEMM workload and --precision bf16");
  if (bf16_ops) {
    cuda_ok(cudaMalloc(&abf, M * K * 2), "cudaMalloc(A bf16)");
    cuda_ok(cudaMalloc(&bbf, K * N * 2), "cudaMalloc(B bf16)");
    tf_ok(tforge_convert_bf16(dA, reinterpret_cast<uint16_t *>(abf), M * K, stream), "tforge_convert_bf16(A)");
    tf_ok(tforge_convert_bf16(dB, reinterpret_cast<uint16_t *>(bbf), K * N, stream), "tforge_convert_bf16(B)");
    cuda_ok(cudaStreamSynchronize(stream), "convert");
    kernel = L.kernel;
  }

  if (a.mode == "lib" && bf16_ops) {
    run = [&] {
      tforge_gemm_args g{};
      g.workload = wl;
      g.mode = mode;
      g.a_dtype = TFORGE_BF16;
      g.b_dtype = TFORGE_BF16;
      g.A = abf;
      g.B = bbf;
      g.bias = dBias;
      g.C_res = dRes;
      g.out = dC;
      g.M = M;
      g.N = N;
      g.K = K;
      tf_ok(tforge_gemm(&g, stream), "tforge_gemm (bf16 operands)");
    };
  } else if (a.mode == "lib") {
    run = [&] {
      int rc = TFORGE_OK;
      switch (wl) {
        case TFORGE_MATMUL: rc = tforge_matmul(dA, dB, dC, M, N, K, mode, stream); break;
        case TFORGE_MBR: rc = tforge_mbr(dA, dB, dBias, dC, M, N, K, mode, stream); break;
        case TFORGE_MATMUL_ADD: rc = tforge_matmul_add(dA, dB, dRes, dC, M, N, K, mode, stream); break;
        case TFORGE_BIAS_ADD: rc = tforge_bias_add(dA, dBias, dC, M, N, stream); break;
        case TFORGE_RELU: rc = tforge_relu(dA, dC, M, N, stream); break;
        case TFORGE_ADD: rc = tforge_add(dA, dB, dC, M, N, stream); break;
      }
      tf_ok(rc, "library call");
    };
  } else {
    blas_ok(cublasCreate(&blas), "cublasCreate");
    blas_ok(cublasSetStream(blas, stream), "cublasSetStream");
    const float one = 1.0f, zero = 0.0f;
    if (a.math == "default") {
      // The reference's comparator: FP32 FMA, no TF32 (runners/gpu/tforge-gpu-bench.cu:306-307).
      blas_ok(cublasSetMathMode(blas, CUBLAS_DEFAULT_MATH), "cublasSetMathMode");
      kernel = "cublasSgemm(default math)";
    } else if (a.math == "tf32") {
      blas_ok(cublasSetMathMode(blas, CUBLAS_TF32_TENSOR_OP_MATH), "cublasSetMathMode");
      kernel = "cublasSgemm(TF32 tensor op)";
    } else if (a.math == "bf16") {
      cuda_ok(cudaMalloc(&abf, M * K * 2), "cudaMalloc");
      cuda_ok(cudaMalloc(&bbf, K * N * 2), "cudaMalloc");
      kernel = "cublasGemmEx(bf16 in, f32 acc)";
    } else if (a.math == "bf16x9") {
      blas_ok(cublasSetEmulationStrategy(blas, CUBLAS_EMULATION_STRATEGY_EAGER), "cublasSetEmulationStrategy");
      kernel = "cublasGemmEx(f32, COMPUTE_32F_EMULATED_16BFX9)";
    } else if (a.math == "lt" || a.math == "lt_tf32" || a.math == "lt_bf16") {
      if (wl == TFORGE_MATMUL_ADD) die("--math lt* covers matmul and mbr");
      blas_ok(cublasLtCreate(&lt), "cublasLtCreate");
      const bool ltb = a.math == "lt_bf16";
      if (ltb) {
        cuda_ok(cudaMalloc(&abf, M * K * 2), "cudaMalloc");
        cuda_ok(cudaMalloc(&bbf, K * N * 2), "cudaMalloc");
        to_bf16<<<(unsigned)((M * K + 255) / 256), 256, 0, stream>>>(dA, abf, M * K);
        to_bf16<<<(unsigned)((K * N + 255) / 256), 256, 0, stream>>>(dB, bbf, K * N);
        cuda_ok(cudaStreamSynchronize(stream), "bf16 copies");
      }
      const cublasComputeType_t ct = a.math == "lt_tf32" ? CUBLAS_COMPUTE_32F_FAST_TF32 : CUBLAS_COMPUTE_32F;
      blas_ok(cublasLtMatmulDescCreate(&ltDesc, ct, CUDA_R_32F), "cublasLtMatmulDescCreate");
      const cublasOperation_t opN = CUBLAS_OP_N;
      blas_ok(cublasLtMatmulDescSetAttribute(ltDesc, CUBLASLT_MATMUL_DESC_TRANSA, &opN, sizeof(opN)), "TRANSA");
      blas_ok(cublasLtMatmulDescSetAttribute(ltDesc, CUBLASLT_MATMUL_DESC_TRANSB, &opN, sizeof(opN)), "TRANSB");
      if (wl == TFORGE_MBR) {
        // Column-major view C^T (N x M): the bias runs along its rows, i.e. our columns.
        const cublasLtEpilogue_t epi = CUBLASLT_EPILOGUE_RELU_BIAS;
        blas_ok(cublasLtMatmulDescSetAttribute(ltDesc, CUBLASLT_MATMUL_DESC_EPILOGUE, &epi, sizeof(epi)), "EPILOGUE");
        blas_ok(cublasLtMatmulDescSetAttribute(ltDesc, CUBLASLT_MATMUL_DESC_BIAS_POINTER, &dBias, sizeof(dBias)),
                "BIAS_POINTER");
      }
      blas_ok(cublasLtMatrixLayoutCreate(&ltB, ltb ? CUDA_R_16BF : CUDA_R_32F, N, K, N), "layout B");
      blas_ok(cublasLtMatrixLayoutCreate(&ltA, ltb ? CUDA_R_16BF : CUDA_R_32F, K, M, K), "layout A");
      blas_ok(cublasLtMatrixLayoutCreate(&ltC, CUDA_R_32F, N, M, N), "layout C");
      cublasLtMatmulPreference_t pref;
      blas_ok(cublasLtMatmulPreferenceCreate(&pref), "pref");
      const size_t wsBytes = size_t(64) << 20;
      blas_ok(cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &wsBytes,
                                                   sizeof(wsBytes)),
              "pref workspace");
      cuda_ok(cudaMalloc(&ltWs, wsBytes), "cudaMalloc(lt workspace)");
      int found = 0;
      blas_ok(cublasLtMatmulAlgoGetHeuristic(lt, ltDesc, ltB, ltA, ltC, ltC, pref, 1, &ltHeur, &found), "heuristic");
      if (!found) die("cuBLASLt: no algorithm");
      cublasLtMatmulPreferenceDestroy(pref);
      const char *prec = a.math == "lt" ? "f32" : a.math == "lt_tf32" ? "tf32" : "bf16 operands";
      kernel = std::string("cublasLtMatmul(") + prec + (wl == TFORGE_MBR ? ", RELU_BIAS epilogue)" : ")");
    } else {
      die("--math default|tf32|bf16|bf16x9|lt|lt_tf32|lt_bf16");
    }
    run = [&, one, zero] {
      if (a.math == "lt" || a.math == "lt_tf32" || a.math == "lt_bf16") {
        const void *lb = a.math == "lt_bf16" ? static_cast<const void *>(bbf) : dB;
        const void *la = a.math == "lt_bf16" ? static_cast<const void *>(abf) : dA;
        blas_ok(cublasLtMatmul(lt, ltDesc, &one, lb, ltB, la, ltA, &zero, dC, ltC, dC, ltC, &ltHeur.algo, ltWs,
                               size_t(64) << 20, stream),
                "cublasLtMatmul");
        if (wl == TFORGE_MATMUL_ADD) add_inplace<<<(unsigned)((M * N + 255) / 256), 256, 0, stream>>>(dC, dRes, M * N);
        cuda_ok(cudaGetLastError(), "epilogue launch");
        return;
      }
      if (a.math == "bf16x9") {
        blas_ok(cublasGemmEx(blas, CUBLAS_OP_N, CUBLAS_OP_N, (int)N, (int)M, (int)K, &one, dB, CUDA_R_32F, (int)N,
                             dA, CUDA_R_32F, (int)K, &zero, dC, CUDA_R_32F, (int)N,
                             CUBLAS_COMPUTE_32F_EMULATED_16BFX9, CUBLAS_GEMM_DEFAULT),
                "cublasGemmEx(bf16x9)");
      } else if (a.math == "bf16") {
        to_bf16<<<(unsigned)((M * K + 255) / 256), 256, 0, stream>>>(dA, abf, M * K);
        to_bf16<<<(unsigned)((K * N + 255) / 256), 256, 0, stream>>>(dB, bbf, K * N);
        blas_ok(cublasGemmEx(blas, CUBLAS_OP_N, CUBLAS_OP_N, (int)N, (int)M, (int)K, &one, bbf,
                             CUDA_R_16BF, (int)N, abf, CUDA_R_16BF, (int)K, &zero, dC, CUDA_R_32F,
                             (int)N, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT),
                "cublasGemmEx");
      } else {
        // Row-major C = A B as column-major C^T = B^T A^T.
        blas_ok(cublasSgemm(blas, CUBLAS_OP_N, CUBLAS_OP_N, (int)N, (int)M, (int)K, &one, dB,
                            (int)N, dA, (int)K, &zero, dC, (int)N),
                "cublasSgemm");
      }
      const long total = M * N;
      if (wl == TFORGE_MBR) bias_relu<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(dC, dBias, M, N);
      if (wl == TFORGE_MATMUL_ADD) add_inplace<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(dC, dRes, total);
      cuda_ok(cudaGetLastError(), "epilogue launch");
    };
  }

  // Correctness run: output pre-filled with NaN (0xFF bytes) so unwritten elements show.
  cuda_ok(cudaMemset(dC, 0xFF, hC.size() * 4), "cudaMemset");
  run();
  cuda_ok(cudaStreamSynchronize(stream), "correctness run");
  if (a.mode == "lib") tf_ok(tforge_device_status(stream), "device status");
  cuda_ok(cudaMemcpy(hC.data(), dC, hC.size() * 4, cudaMemcpyDeviceToHost), "cudaMemcpy(C)");
  if (!a.out.empty()) {
    std::ofstream o(a.out, std::ios::binary);
    o.write(reinterpret_cast<const char *>(hC.data()), hC.size() * 4);
  }

  Nvml nv;
  void *flushBuf = nullptr;
  const size_t flushBytes = size_t(256) << 20;
  if (a.flush) cuda_ok(cudaMalloc(&flushBuf, flushBytes), "cudaMalloc(flush)");
  unsigned flushVal = 0;
  cudaEvent_t e0, e1;
  cuda_ok(cudaEventCreate(&e0), "cudaEventCreate");
  cuda_ok(cudaEventCreate(&e1), "cudaEventCreate");
  for (int i = 0; i < a.warmup; ++i) run();
  cuda_ok(cudaStreamSynchronize(stream), "warm-up");
  std::vector<double> ms(a.reps), clk, pwr;
  for (int i = 0; i < a.reps; ++i) {
    if (a.flush) cuda_ok(cudaMemsetAsync(flushBuf, (int)(++flushVal & 0xFF), flushBytes, stream), "flush");
    cuda_ok(cudaEventRecord(e0, stream), "cudaEventRecord");
    run();
    cuda_ok(cudaEventRecord(e1, stream), "cudaEventRecord");
    cuda_ok(cudaEventSynchronize(e1), "cudaEventSynchronize");
    float t = 0;
    cuda_ok(cudaEventElapsedTime(&t, e0, e1), "cudaEventElapsedTime");
    ms[i] = t;
    unsigned c = 0, p = 0;
    if (nv.ok && nv.clock(nv.dev, 1 /* NVML_CLOCK_SM */, &c) == 0) clk.push_back(c);
    if (nv.ok && nv.power(nv.dev, &p) == 0) pwr.push_back(p / 1000.0);
  }
  if (a.mode == "lib") tf_ok(tforge_device_status(stream), "device status");
  const Summary s = summarize(ms), c = summarize(clk), p = summarize(pwr);
  double clkMax = clk.empty() ? -1 : *std::max_element(clk.begin(), clk.end());
  int driver = 0;
  cudaDriverGetVersion(&driver);
  const double flops = gemm ? 2.0 * M * N * K : 0.0;
  const double tflops = s.median > 0 ? flops / (s.median * 1e-3) / 1e12 : 0.0;

  std::printf(
      "{\"gpu\": \"%s\", \"mode\": \"%s\", \"workload\": \"%s\", \"m\": %ld, \"n\": %ld, \"k\": %ld, "
      "\"padded\": \"%ldx%ldx%ld\", \"precision\": \"%s\", \"kernel\": \"%s\", "
      "\"grid\": \"%dx%dx%d\", \"block\": \"%dx%dx%d\", \"regs\": %d, \"local_bytes\": 0, "
      "\"static_smem\": %d, \"dyn_smem\": %d, \"blocks_per_sm\": %d, \"theo_occupancy\": %.3f, "
      "\"tile\": \"%dx%dx%d\", \"stages\": %d, "
      "\"warmup\": %d, \"reps\": %d, \"l2_flush\": %d, \"median_ms\": %.6f, \"min_ms\": %.6f, "
      "\"std_ms\": %.6f, \"tflops\": %.3f, \"sm_clock_median_mhz\": %.0f, \"sm_clock_min_mhz\": %.0f, "
      "\"sm_clock_max_mhz\": %.0f, \"power_median_w\": %.1f, \"cuda_driver\": %d}\n",
      prop.name, a.mode.c_str(), a.workload.c_str(), M, N, K, M, N, K,
      a.mode == "lib" ? a.precision.c_str() : a.math.c_str(), kernel.c_str(), L.grid[0], L.grid[1],
      L.grid[2], L.block[0], L.block[1], L.block[2], L.regs, L.static_smem, L.smem_bytes,
      L.blocks_per_sm, L.blocks_per_sm > 0 ? L.blocks_per_sm * (L.block[0] / 32) / 64.0 : -1.0,
      L.tile[0], L.tile[1], L.tile[2], L.stages, a.warmup, a.reps, a.flush ? 1 : 0, s.median, s.min,
      s.sd, tflops, c.median, c.min, clkMax, p.median, driver);
  return 0;
}
