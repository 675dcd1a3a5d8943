// tf_gemm_2sm_persist.cu -- persistent CTA-pair GEMM for the TF32 and BF16 modes: each
// cluster of two CTAs loops over 256 x 256 output tiles and keeps two accumulators in
// tensor memory, so the epilogue of one tile runs while the MMAs of the next one do.
//
// Per tile the operand layout, k-block order and MMA sequence are those of
// gemm_pair_kernel (tf_gemm_2sm.cu), so every output element is computed by the same
// instructions in the same order and the two kernels agree bit for bit.  What changes:
//
//   * grid = 2 x min(tiles, co-resident clusters); pair g takes tiles g, g + pairs, ...
//     of the grouped raster order, and one TMA -> MMA ring of STAGES slots runs across
//     all of them (ring position = k-blocks issued so far).
//   * TMEM: 512 columns; tile i of a pair accumulates into columns [256 (i % 2), +256).
//     The leader's MMA thread waits acce[b] (both CTAs' epilogues have read accumulator b)
//     before the first MMA of a tile into b, and a multicast tcgen05.commit signals accf[b]
//     in both CTAs after the tile's last k-block.
//   * epilogue (warps 4..7 of each CTA): 32-column chunks, tcgen05.ld -> +bias / +C_res,
//     relu -> one of two dedicated 128 x 32 staging boxes (128-B swizzle) -> TMA store.
//     The ring cannot lend its memory to the output here, since the next tile's loads
//     are already in it.  matmul_add reads C_res with plain global loads.
//   * TF32 with B as given (SWAP): the MMA's operands are exchanged as in the pair kernel --
//     B's tile (MN-major, which for 32-bit elements the tensor core reads through the
//     128B_BASE32B swizzle) is the M side, local to each CTA, and A's tile the N side shared
//     by the pair -- so CTA r accumulates the transposed tile: TMEM lane = output column
//     n0 + 128 r + lane, TMEM column j = output row (pair's first row) + j.  Each 32-column
//     chunk is 32 output rows x 128 columns, staged row-major without swizzle (a warp writes
//     128 consecutive bytes per row) and stored as one 32-row x 128-column TMA box.
//
// 256 threads: warp 0 TMA producer (both CTAs), warp 1 MMA issuer (leader), warps 4..7
// epilogue.  Every wait is bounded (tf_ptx.cuh); on a timeout each role stops, the MMA
// issuer and the producer drain what they issued (bounded), and both CTAs meet at a
// cluster barrier before TMEM is freed.
#include <cuda.h>
#include <cuda_runtime.h>

#include "tf_internal.h"
#include "tf_ptx.cuh"

namespace tf {

namespace {

#ifndef TF_PERSIST_SWAP
#define TF_PERSIST_SWAP 1
#endif
// TF32 with B as given: exchange the MMA's operands (see the kernel's header comment).
constexpr bool kPersistSwap = TF_PERSIST_SWAP;

template <int PREC, int STAGES>
struct PersistLayout {
  static constexpr int kThreads = 256;
  static constexpr int kElem = PREC == PREC_BF16 ? 2 : 4;
  static constexpr int kBK = 128 / kElem;           // K elements per stage (one 128-B row)
  static constexpr int kUmmaK = 32 / kElem;         // K per MMA instruction
  static constexpr int kKSteps = kBK / kUmmaK;      // 4
  static constexpr int kNBlk = 128 / kElem;         // B columns per 128-B MN block
  static constexpr int kBBlocks = 128 / kNBlk;      // TMA boxes per B half
  static constexpr int kABytes = 128 * 128;         // this CTA's 128 A rows
  static constexpr int kBBytes = 128 * kBK * kElem;  // this CTA's 128 B columns
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBoxBytes = 128 * 128;       // 128 rows x 32 f32 columns
  static constexpr int kBoxOff = STAGES * kStageBytes;
  static constexpr int kBarOff = kBoxOff + 2 * kBoxBytes;
  // Barriers: full[STAGES], empty[STAGES], accf[2], acce[2], drain; then the TMEM slot,
  // the abort flag, the epilogue's go/no-go word and a spare word.
  static constexpr int kNumBars = 2 * STAGES + 5;
  static constexpr int kBarBytes = (8 * kNumBars + 16 + 15) / 16 * 16;
  static constexpr int kBiasOff = kBarOff + kBarBytes;  // the tile's 256 bias values
  static constexpr int kSmemBytes = 1024 + kBiasOff + 256 * 4;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// Bounded pause (abort drains of loads this CTA cannot observe).
__device__ __forceinline__ void pause_ns(uint64_t ns) {
  const uint64_t t0 = globaltimer();
  while (globaltimer() - t0 < ns) __nanosleep(1000);
}

template <int PREC, int STAGES, int EPI, bool OUTB, bool BKM, bool BAT = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 1)
    gemm_pair_persistent_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                const __grid_constant__ CUtensorMap tmO, const TcParams p) {
  using L = PersistLayout<PREC, STAGES>;
  constexpr bool kTF32 = PREC == PREC_TF32;
  // TF32 with B as given: operands exchanged, transposed accumulator and epilogue.
  constexpr bool kSwap = kTF32 && !BKM && kPersistSwap;
  // BKM (TF32): B is a transposed copy, loaded and read K-major like A.
  constexpr uint32_t kIdesc = kSwap  ? instr_desc_a_mn(2u, 256, 256)
                              : BKM ? (instr_desc(2u, 256, 256) & ~(1u << 16))
                                    : instr_desc(kTF32 ? 2u : 1u, 256, 256);
  // bf16 output (OUTB): BF16 precision and the mbr epilogue only.
  static_assert(!OUTB || (PREC == PREC_BF16 && EPI == EPI_MBR), "bf16 output configuration");
  static_assert(!BKM || PREC == PREC_TF32, "K-major B configuration");
  // B as given (TF32): its tile in the k-group-major tiling (BAT, one 4-D box,
  // TcParams::b_atoms) or in column blocks; a compile-time choice, as in gemm_pair_kernel.
  using BT = BTileMN<L::kElem>;
  static_assert(!BAT || (kTF32 && !BKM && !OUTB), "k-group-major B configuration");
  constexpr bool b_atoms = BAT;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  // full[s]: both CTAs' bytes of ring slot s landed (leader's barrier); empty[s]: the pair
  // MMAs reading slot s are done (both CTAs); accf[b]: accumulator b holds a finished tile
  // (both CTAs); acce[b] (leader): both CTAs' epilogues have read accumulator b; drain: the
  // MMA issuer's in-flight MMAs after an abort.
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * STAGES, accf0 = empty0 + 8 * STAGES,
                 acce0 = accf0 + 16, drainf = acce0 + 16;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + L::kNumBars);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  volatile uint32_t *epi_ok = tmem_slot + 2;
  float4 *bias_s = reinterpret_cast<float4 *>(smem + L::kBiasOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int tiles_m = (p.M + 255) / 256, tiles_n = (p.N + 255) / 256;
  const int tiles = tiles_m * tiles_n;
  const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);
  const int my_tiles = pair < tiles ? (tiles - 1 - pair) / npairs + 1 : 0;
  const int nkb = (p.K + L::kBK - 1) / L::kBK;
  const WaitCtl wc{abort_flag, p.status, p.limit_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, 8);  // lane 0 of the 4 epilogue warps of both CTAs
    }
    mbar_init(drainf, 1);
    *abort_flag = 0u;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers are initialised before any remote arrive or TMA
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    grid_dependency_wait();  // operands written by the kernel before this launch (TcParams::pdl)
    // Loads complete on the LEADER's full[s], which expects both CTAs' bytes; slot s is
    // reused once the pair MMAs that read it are done (empty[s], committed to both CTAs).
    const uint32_t lead_full0 = map_to_cta(full0, 0);
    int g = 0;  // k-blocks issued so far
    bool ok = true;
    for (int i = 0; i < my_tiles && ok; ++i) {
      int tm, tn;
      raster_tile(pair + i * npairs, tiles_m, tiles_n, kRasterGroup, tm, tn);
      const int m0 = tm * 256 + (int)rank * 128, nb = tn * 256 + (int)rank * 128;
      for (int kb = 0; kb < nkb; ++kb, ++g) {
        const int s = g % STAGES, round = g / STAGES;
        if (round > 0 && !mbar_wait_cluster(empty0 + 8 * s, (round - 1) & 1, wc)) {
          ok = false;
          break;
        }
        if (p.debug_skip && g == 0) continue;  // test hook: this stage never fills
        const int kc = kb * L::kBK;
        const uint32_t slot = sbase + s * L::kStageBytes;
        if (rank == 0) mbar_arrive_expect_tx(full0 + 8 * s, 2 * L::kStageBytes);
        tma_load_2d_pair(slot, &tmA, kc, m0, lead_full0 + 8 * s);
        if constexpr (BKM) {
          tma_load_2d_pair(slot + L::kABytes, &tmB, kc, nb, lead_full0 + 8 * s);  // 128 n-rows x 32 k
        } else if constexpr (b_atoms) {
          tma_load_4d_pair(slot + L::kABytes, &tmB, 0, 0, nb / L::kNBlk, kc / BT::kRows, lead_full0 + 8 * s);
        } else {
#pragma unroll
          for (int j = 0; j < L::kBBlocks; ++j)
            tma_load_2d_pair(slot + L::kABytes + j * (L::kBK * 128), &tmB, nb + j * L::kNBlk, kc, lead_full0 + 8 * s);
        }
      }
    }
    if (*abort_flag) {
      if (rank == 0) {
#pragma unroll 1
        for (int s = 0; s < STAGES; ++s) {
          if (g - 1 < s) continue;
          const int last = g - 1 - ((g - 1 - s) % STAGES);
          if (p.debug_skip && last == 0) continue;
          mbar_wait_drain_cluster(full0 + 8 * s, (last / STAGES) & 1, p.limit_ns);
        }
      } else {
        pause_ns(200000);  // the peer's loads complete on the leader's barrier
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ---------------- pair MMA issuer (leader CTA) ----------------
    // Ring slot s and its phase are kept incrementally, and the descriptors are the slot-0 ones
    // plus constant offsets (16-B units): this thread's loop is on the critical path.
    bool ok = true;
    const uint64_t a_d0 = smem_desc(sbase, 16, 1024, 2);
    const uint64_t b_d0 = BKM ? smem_desc(sbase + L::kABytes, 16, 1024, 2) : BT::desc(sbase + L::kABytes, 0, b_atoms);
    constexpr uint32_t kBStep = BKM ? 2u : BT::step(b_atoms) >> 4;
    int s = 0;
    uint32_t phase = 0, bar = full0;
    uint64_t so = 0;
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int b = i & 1;
      const uint32_t acc = tmem + 256u * b;
      // Use u = i / 2 of accumulator b needs the epilogues' release of use u - 1.
      if (i >= 2 && !mbar_wait_cluster(acce0 + 8 * b, ((i >> 1) - 1) & 1, wc)) break;
      tc_fence_after();
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait_cluster(bar, phase, wc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = a_d0 + so, bd = b_d0 + so;
#pragma unroll
        for (int ks = 0; ks < L::kKSteps; ++ks) {
          if constexpr (kSwap)
            mma_ss_pair<kTF32>(acc, bd + ks * kBStep, ad + 2 * ks, kIdesc, (kb | ks) ? 1u : 0u);
          else
            mma_ss_pair<kTF32>(acc, ad + 2 * ks, bd + ks * kBStep, kIdesc, (kb | ks) ? 1u : 0u);
        }
        mma_commit_pair(bar + 8 * STAGES, 0x3);
        if (++s == STAGES) {
          s = 0;
          phase ^= 1u;
          bar = full0;
          so = 0;
        } else {
          bar += 8;
          so += L::kStageBytes >> 4;
        }
      }
      if (!ok) break;
      mma_commit_pair(accf0 + 8 * b, 0x3);
    }
    if (*abort_flag) {
      mma_commit_pair(drainf, 0x1);
      mbar_wait_drain_cluster(drainf, 0, p.limit_ns);
    }
  } else if (warp >= 4) {
    // ---------------- epilogue (both CTAs, warps 4..7) ----------------
    // Warp w reads TMEM lanes 32 (w % 4) .. +31: row r of this CTA's 128 rows.  Chunk c
    // (32 columns) goes through staging box c % 2; before a box is rewritten the store
    // issued from it two chunks earlier must have finished reading it.
    const int q = warp & 3, r = q * 32 + lane, et = threadIdx.x - 128;
    const uint32_t lead_acce0 = map_to_cta(acce0, 0);
    uint8_t *boxes = smem + L::kBoxOff;
#pragma unroll 1
    for (int i = 0; i < my_tiles; ++i) {
      const int b = i & 1;
      int tm, tn;
      raster_tile(pair + i * npairs, tiles_m, tiles_n, kRasterGroup, tm, tn);
      const int m0 = tm * 256 + (int)rank * 128, n0 = tn * 256;
      if constexpr (EPI == EPI_MBR) {
        // The previous tile's reads of bias_s all happened before its last chunk barrier.
        if (et < 64) {
          const int col = n0 + 4 * et;
          bias_s[et] = col < p.N ? __ldg(reinterpret_cast<const float4 *>(p.bias + col))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      // One thread waits (bounded) and publishes the outcome, so all four warps take the
      // same branch and no named barrier below waits for a warp that gave up.
      if (et == 0) *epi_ok = mbar_wait_cluster(accf0 + 8 * b, (i >> 1) & 1, wc, 128) ? 1u : 0u;
      named_barrier(1, 128);
      if (!*epi_ok) break;
      tc_fence_after();
      const bool cta_rows = m0 < p.M;
      const uint32_t tacc = tmem + 256u * b + ((uint32_t)(q * 32) << 16);
      if constexpr (kSwap) {
        // Transposed accumulator: thread r holds output column nb + r for the pair's 256 rows
        // mp0 .., 32 per chunk; chunk c goes through box c % 2 (32 rows x 128 columns).
        const int mp0 = tm * 256, nb = n0 + (int)rank * 128, col = nb + r;
        const bool cta_cols = nb < p.N;
        const float bcol = EPI == EPI_MBR ? reinterpret_cast<const float *>(bias_s)[(int)rank * 128 + r] : 0.f;
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          const int row0 = mp0 + 32 * c;
          const bool live = cta_cols && row0 < p.M;
          uint32_t rr[32];
          tmem_ld_32x32b_x32(tacc + c * 32, rr);
          float cr[32];
          if constexpr (EPI == EPI_ADD) {
            const bool col_ok = live && col < p.N;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              cr[i] = col_ok && row0 + i < p.M ? __ldg(p.cres + (int64_t)(row0 + i) * p.ldc + col) : 0.f;
          }
          tmem_ld_wait(rr);
          float *box = reinterpret_cast<float *>(boxes + (c & 1) * L::kBoxBytes);
          if (et == 0) bulk_wait_group_read1();
          named_barrier(2, 128);
          if (live) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              float v = __uint_as_float(rr[i]);
              if constexpr (EPI == EPI_MBR) v = relu_ieee(__fadd_rn(v, bcol));
              else if constexpr (EPI == EPI_ADD) v = __fadd_rn(v, cr[i]);
              box[i * 128 + r] = v;
            }
          }
          fence_proxy_async_smem();
          named_barrier(3, 128);
          if (et == 0 && live) {
            tma_store_2d(&tmO, smem_u32(box), nb, row0);
            bulk_commit_group();
          }
        }
      } else {
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        const int col0 = n0 + c * 32;
        const bool live = cta_rows && col0 < p.N;
        uint32_t rr[32];
        tmem_ld_32x32b_x32(tacc + c * 32, rr);
        float4 cr[8];
        if constexpr (EPI == EPI_ADD) {
          const bool row_ok = live && m0 + r < p.M;
          const float4 *src = reinterpret_cast<const float4 *>(p.cres + (int64_t)(m0 + r) * p.ldc + col0);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            cr[j] = row_ok && col0 + 4 * j < p.N ? __ldg(src + j) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        tmem_ld_wait(rr);
        uint8_t *box = boxes + (c & 1) * L::kBoxBytes;
        if (et == 0) bulk_wait_group_read1();
        named_barrier(2, 128);
        if (OUTB && live) {
          // bf16 output: 64 B per row in the box's first 8 KB (64-B swizzle: 16-B unit u of
          // row r at unit u ^ ((r >> 1) & 3)), matching the bf16 output map.
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint32_t pk[4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const float4 bb = bias_s[c * 8 + 2 * u + h];
              const int e = 8 * u + 4 * h;
              pk[2 * h] = pack_bf16x2(relu_ieee(__fadd_rn(__uint_as_float(rr[e]), bb.x)),
                                      relu_ieee(__fadd_rn(__uint_as_float(rr[e + 1]), bb.y)));
              pk[2 * h + 1] = pack_bf16x2(relu_ieee(__fadd_rn(__uint_as_float(rr[e + 2]), bb.z)),
                                          relu_ieee(__fadd_rn(__uint_as_float(rr[e + 3]), bb.w)));
            }
            *reinterpret_cast<uint4 *>(box + r * 64 + ((u ^ ((r >> 1) & 3)) << 4)) =
                make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
        } else if (live) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float4 v = make_float4(__uint_as_float(rr[4 * j]), __uint_as_float(rr[4 * j + 1]),
                                   __uint_as_float(rr[4 * j + 2]), __uint_as_float(rr[4 * j + 3]));
            if constexpr (EPI == EPI_MBR) {
              const float4 bb = bias_s[c * 8 + j];
              v.x = relu_ieee(__fadd_rn(v.x, bb.x));
              v.y = relu_ieee(__fadd_rn(v.y, bb.y));
              v.z = relu_ieee(__fadd_rn(v.z, bb.z));
              v.w = relu_ieee(__fadd_rn(v.w, bb.w));
            } else if constexpr (EPI == EPI_ADD) {
              v.x = __fadd_rn(v.x, cr[j].x);
              v.y = __fadd_rn(v.y, cr[j].y);
              v.z = __fadd_rn(v.z, cr[j].z);
              v.w = __fadd_rn(v.w, cr[j].w);
            }
            *reinterpret_cast<float4 *>(box + r * 128 + ((j ^ (r & 7)) << 4)) = v;
          }
        }
        fence_proxy_async_smem();
        named_barrier(3, 128);
        if (et == 0 && live) {
          tma_store_2d(&tmO, smem_u32(box), col0, m0);
          bulk_commit_group();
        }
      }
      }
      // Every tcgen05.ld of accumulator b has completed (tmem_ld_wait): release it.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(lead_acce0 + 8 * b);
    }
    if (et == 0) bulk_wait_group_read0();  // staging stays valid until read
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while the pair MMA may still read its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// Co-resident clusters of one instantiation on the current device (0 on failure).
template <int PREC, int STAGES, int EPI, bool OUTB = false, bool BKM = false, bool BAT = false>
int persist_clusters() {
  using L = PersistLayout<PREC, STAGES>;
  auto kern = gemm_pair_persistent_kernel<PREC, STAGES, EPI, OUTB, BKM, BAT>;
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  int *slot = &cached[dev & 63];
  int v = __atomic_load_n(slot, __ATOMIC_ACQUIRE);
  if (v > 0) return v;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes) != cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cfg.gridDim = dim3(2 * (sms / 2 > 0 ? sms / 2 : 1), 1, 1);
  cfg.blockDim = dim3(L::kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kSmemBytes;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    cfg.numAttrs = 0;  // the compile-time cluster shape alone
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      return 0;
    }
  }
  __atomic_store_n(slot, n, __ATOMIC_RELEASE);
  return n;
}

template <int PREC, int STAGES, int EPI, bool OUTB, bool BKM = false, bool BAT = false>
cudaError_t launch_persist_kern(const CUtensorMap &tmA, const CUtensorMap &tmB, const CUtensorMap &tmO,
                                const TcParams &p, cudaStream_t stream) {
  using L = PersistLayout<PREC, STAGES>;
  const int clusters = persist_clusters<PREC, STAGES, EPI, OUTB, BKM, BAT>();
  if (clusters <= 0) return cudaErrorInvalidConfiguration;
  const int64_t tiles = (int64_t)((p.M + 255) / 256) * ((p.N + 255) / 256);
  const int pairs = tiles < clusters ? (int)tiles : clusters;
  auto kern = gemm_pair_persistent_kernel<PREC, STAGES, EPI, OUTB, BKM, BAT>;
  if (p.pdl) {
    cudaLaunchAttribute attr[1];
    pdl_attr(attr[0]);
    cudaLaunchConfig_t cfg = {dim3(2 * pairs), dim3(L::kThreads), (size_t)L::kSmemBytes, stream, attr, 1};
    return cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmO, p);
  }
  kern<<<2 * pairs, L::kThreads, L::kSmemBytes, stream>>>(tmA, tmB, tmO, p);
  return cudaGetLastError();
}

template <int PREC, int STAGES, int EPI>
cudaError_t launch_persist_one(const CUtensorMap &tmA, const CUtensorMap &tmB, const CUtensorMap &tmO,
                               const TcParams &p, cudaStream_t stream) {
  if (p.splits > 1) return cudaErrorInvalidValue;
  if (p.b_kmajor) {
    if constexpr (PREC == PREC_TF32)
      return p.out_bf16 ? cudaErrorInvalidValue : launch_persist_kern<PREC, STAGES, EPI, false, true>(tmA, tmB, tmO, p, stream);
    return cudaErrorInvalidValue;
  }
  if (p.out_bf16) {
    if constexpr (PREC == PREC_BF16 && EPI == EPI_MBR)
      return launch_persist_kern<PREC, STAGES, EPI, true>(tmA, tmB, tmO, p, stream);
    return cudaErrorInvalidValue;
  }
  if (p.b_atoms) {
    if constexpr (PREC == PREC_TF32) return launch_persist_kern<PREC, STAGES, EPI, false, false, true>(tmA, tmB, tmO, p, stream);
    return cudaErrorInvalidValue;
  }
  return launch_persist_kern<PREC, STAGES, EPI, false>(tmA, tmB, tmO, p, stream);
}

template <int PREC, int STAGES>
cudaError_t launch_persist_epi(int epi, const CUtensorMap &tmA, const CUtensorMap &tmB, const CUtensorMap &tmO,
                               const TcParams &p, cudaStream_t stream) {
  switch (epi) {
    case EPI_MATMUL: return launch_persist_one<PREC, STAGES, EPI_MATMUL>(tmA, tmB, tmO, p, stream);
    case EPI_MBR: return launch_persist_one<PREC, STAGES, EPI_MBR>(tmA, tmB, tmO, p, stream);
    case EPI_ADD: return launch_persist_one<PREC, STAGES, EPI_ADD>(tmA, tmB, tmO, p, stream);
  }
  return cudaErrorInvalidValue;
}

template <int PREC, int STAGES>
cudaError_t persist_attrs(int epi, cudaFuncAttributes *a, int *blocks) {
  using L = PersistLayout<PREC, STAGES>;
  const void *f = epi == EPI_MBR   ? reinterpret_cast<const void *>(gemm_pair_persistent_kernel<PREC, STAGES, EPI_MBR, false, false>)
                  : epi == EPI_ADD ? reinterpret_cast<const void *>(gemm_pair_persistent_kernel<PREC, STAGES, EPI_ADD, false, false>)
                                   : reinterpret_cast<const void *>(gemm_pair_persistent_kernel<PREC, STAGES, EPI_MATMUL, false, false>);
  cudaError_t e = cudaFuncGetAttributes(a, f);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, f, L::kThreads, L::kSmemBytes);
}

}  // namespace

// Instantiated persistent configurations: (precision, stages).
#define TF_PERSIST_CONFIGS(X) X(PREC_TF32, 6) X(PREC_BF16, 6)

bool persist_transposed(int prec) { return prec == PREC_TF32 && kPersistSwap; }

int persist_smem_bytes(int prec, int stages) {
#define TF_PSMEM(P, S) \
  if (prec == P && stages == S) return PersistLayout<P, S>::kSmemBytes;
  TF_PERSIST_CONFIGS(TF_PSMEM)
#undef TF_PSMEM
  return -1;
}

cudaError_t launch_gemm_pair_persistent(int prec, int stages, int epi, const CUtensorMap &tmA,
                                        const CUtensorMap &tmB, const CUtensorMap &tmO, const TcParams &p,
                                        cudaStream_t stream) {
#define TF_PLAUNCH(P, S) \
  if (prec == P && stages == S) return launch_persist_epi<P, S>(epi, tmA, tmB, tmO, p, stream);
  TF_PERSIST_CONFIGS(TF_PLAUNCH)
#undef TF_PLAUNCH
  return cudaErrorInvalidValue;
}

cudaError_t persist_func_attributes(int prec, int stages, int epi, cudaFuncAttributes *a, int *blocks) {
#define TF_PATTR(P, S) \
  if (prec == P && stages == S) return persist_attrs<P, S>(epi, a, blocks);
  TF_PERSIST_CONFIGS(TF_PATTR)
#undef TF_PATTR
  return cudaErrorInvalidValue;
}

int persist_grid_pairs(int prec, int stages, int epi, int64_t M, int64_t N) {
  int clusters = 0;
#define TF_PCL(P, S)                                                             \
  if (prec == P && stages == S)                                                  \
    clusters = epi == EPI_MBR   ? persist_clusters<P, S, EPI_MBR>()              \
               : epi == EPI_ADD ? persist_clusters<P, S, EPI_ADD>()              \
                                : persist_clusters<P, S, EPI_MATMUL>();
  TF_PERSIST_CONFIGS(TF_PCL)
#undef TF_PCL
  const int64_t tiles = ((M + 255) / 256) * ((N + 255) / 256);
  if (clusters <= 0) return -1;
  return (int)(tiles < clusters ? tiles : clusters);
}

}  // namespace tf
