// tf_gemm_2sm.cu -- fused GEMM on a CTA pair (tcgen05 cta_group::2), 256 x 256 or 256 x 240 output tiles.
//
// Same operator and epilogue as tf_gemm_tc.cu (matmul, mbr = relu(A @ B + bias),
// matmul_add), for large problems.  Two CTAs on two SMs form a cluster; CTA r of the pair
// loads A rows [m0 + 128 r, +128) and B columns [n0 + (BN / 2) r, +128) into its own shared
// memory (plain TMA tile loads, no multicast), and one pair MMA (M = 256, N = BN) reads A
// from both CTAs and B from both halves, so each SM reads only half of B per FLOP.
//
// fp32-accurate mode (3xTF32): per K step the MMA issues lo*hi, hi*lo and hi*hi.  The
// split of A goes to tensor memory (tcgen05.st), so the MMAs read only B from shared
// memory.  Two rings: TMA lands raw A and B in a landing ring (kLand slots); converters
// load a slot and write the split operands into an operand ring (kOps slots: B lo in
// shared memory, A hi and lo in TMEM), which the MMAs free.  B hi is the raw B of the
// landing slot (truncation split), which the MMAs read in place, so a landing slot is
// free once its converters have loaded it and the MMAs reading its B are done.
// 384 threads per CTA:
//
//   warp 0       TMA producer (each CTA): A tile and B half of k-block kb -> landing slot
//                l = kb % kLand (full[l]) once slot l is free (lempty[l]).
//   warps 2..11  converters (each CTA): load the landing slot, arrive lempty[l], wait
//                until operand slot o = kb % kOps is free (empty[o]), write B lo there;
//                warps 4..11 also split A: warp w takes rows 32 (w % 4) .. +31 (its TMEM
//                lane quadrant) and K half (w - 4) / 4, into TMEM columns [256 + 64 o, +32)
//                (hi) and [+32, +32) (lo).  Then each warp arrives on this CTA's conv[o].
//   warp 1       leader CTA: issues the pair MMAs into TMEM columns [0, BN) of both CTAs
//                once its conv[o] and ready[o] (the peer's) completed; multicast
//                tcgen05.commits free operand slot o (empty[o]) and landing slot l
//                (lempty[l]) in both CTAs, a last one signals accf in both.  Peer CTA:
//                relays its conv[o] to the leader's ready[o] with one st.async token per
//                k-block.
//   warps 0..11  epilogue (each CTA), once the accumulator is complete: its 128 rows x BN
//                columns from its own TMEM, in three groups of four warps (one per TMEM
//                lane quadrant) taking the 32-column chunks in turn.
//
// The split (kPairSplit): the tensor core reads an f32 operand as TF32 by dropping its low
// 13 mantissa bits, so the truncation split keeps hi = x and computes only
// lo = x - trunc(x), exact in f32.  The round split (cvt.rna) is kept as an alternative;
// it writes B hi into the operand slot as well.
//
// Tile width BN: 256, or 240 when that needs no more waves of SM pairs (each CTA's MMA
// half is then the first 120 of the 128 B columns it loads).
//
// TF32 with 256-wide tiles (kTf32Swap) exchanges the MMA's operands: B's tile (MN-major,
// which for 32-bit elements the tensor core reads through the 128B_BASE32B swizzle) is the M
// side, local to each CTA, and A's tile the N side shared by the pair, so CTA r accumulates
// the transposed tile: TMEM lane = output column n0 + 128 r + lane, TMEM column j = output
// row (pair's first row) + j.  The loads are unchanged; the epilogue stores 32-row x
// 128-column boxes.  (Measured on cuBLAS as well: its TF32 GEMM with the MN-major operand on
// the N side ran 690 TFLOP/s at 8192^3 against 808 with it on the M side.)
//
// TF32 / BF16 modes have no converters: each CTA's TMA (.cta_group::2 form) completes on
// the LEADER's full[s], which expects both CTAs' bytes, and the MMA reads A and B from
// shared memory.
//
// Every wait is bounded (tf_ptx.cuh); both CTAs meet at a cluster barrier before TMEM is
// freed, so no CTA exits while the pair MMA may still read its shared or tensor memory.
#include <cuda.h>
#include <cuda_runtime.h>

#include "tf_internal.h"
#include "tf_ptx.cuh"

namespace tf {


namespace {

#ifndef TF_PAIR_OPS
#define TF_PAIR_OPS 3
#endif
// 3xTF32: depth of the operand ring (B lo in shared memory, A hi/lo in TMEM).
constexpr int kPairOps = TF_PAIR_OPS;
// Truncation split: B hi is the raw f32 B as TMA landed it (the tensor core drops the low
// 13 bits itself), so the MMAs read it from the landing slot and only B lo is written.
constexpr bool kPairHiDirect = kPairSplit == 1;

// bf16-output epilogue staging box: 128 rows x 32 bf16 columns.
constexpr int kEpiBoxBytesB = 128 * 64;

#ifndef TF_TF32_SWAP
#define TF_TF32_SWAP 1
#endif
constexpr bool kTf32Swap = TF_TF32_SWAP;

template <int PREC, int STAGES>
struct PairLayout {
  // 3xTF32: warps 0 producer, 1 MMA (leader) / relay (peer), 2..11 converters.
  static constexpr bool kX3 = PREC == PREC_X3;
  static constexpr int kThreads = kX3 ? 384 : 256;
  // Epilogue warps kEpiWarp0 .. + kEpiWarps - 1.  3xTF32: all twelve -- the producer, MMA and
  // B-only converter warps (0..3) are idle once the accumulator is complete, and three groups
  // of four take the eight 32-column chunks in turn (at most three each).  TF32 / BF16: 4..7.
  static constexpr int kEpiWarp0 = kX3 ? 0 : 4;
  static constexpr int kEpiWarps = kX3 ? 12 : 4;
  static constexpr int kElem = PREC == PREC_BF16 ? 2 : 4;
  static constexpr int kBK = 128 / kElem;              // K elements per stage (one 128-B row)
  static constexpr int kUmmaK = 32 / kElem;            // K per MMA instruction
  static constexpr int kKSteps = kBK / kUmmaK;         // 4
  static constexpr int kNBlk = 128 / kElem;            // N elements per 128-B MN block
  static constexpr int kBNHalf = 128;                  // B columns loaded by each CTA
  static constexpr int kBBlocks = kBNHalf / kNBlk;     // TMA boxes per B half
  static constexpr int kABytes = 128 * 128;            // this CTA's 128 A rows
  static constexpr int kBBytes = kBNHalf * kBK * kElem;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // Landing ring (TMA destination): kLand slots of A + B.  TF32/BF16: the MMA reads them
  // in place.  3xTF32: the converters load a slot into the operand ring of kOps slots --
  // B lo in shared memory, A hi and lo in TMEM -- which the MMAs empty; the MMAs read
  // B hi from the landing slot itself.
  static constexpr int kLand = STAGES;
  static constexpr int kOps = kX3 ? kPairOps : STAGES;
  // Operand slot: B lo (and B hi unless the MMAs read it from the landing slot).
  static constexpr int kOpBytes = kX3 ? (kPairHiDirect ? kBBytes : 2 * kBBytes) : 0;
  static constexpr int kRingBytes = kLand * kStageBytes + kOps * kOpBytes;
  // Barriers: full[kLand], lempty[kLand] (3xTF32: converters + MMAs -> producer), conv[kOps],
  // ready[kOps], empty[kOps] (MMA commit), accf, resf.
  static constexpr int kNumBars = 2 * kLand + 3 * kOps + 3;
  // barriers, then tmem slot, abort flag, epilogue flag, spare, and one mailbox word per
  // operand stage (the peer's st.async tokens land there).
  static constexpr int kBarBytes = 8 * kNumBars + 16 + 4 * kOps;
  // The tile's 256 bias values, staged during the mainloop for the epilogue.
  static constexpr int kBiasBytes = 256 * 4;
  __host__ __device__ static constexpr int bias_off() { return kRingBytes + (kBarBytes + 15) / 16 * 16; }
  static constexpr int kSmemBytes = 1024 + kRingBytes + (kBarBytes + 15) / 16 * 16 + kBiasBytes;
  static constexpr uint32_t kAccCols = 256;
  static constexpr uint32_t kTmemCols = kX3 ? 512u : 256u;
  static constexpr int kConvWarps = 10;                // warps 2..11 (3xTF32)
  __host__ __device__ static constexpr int a_off(int l) { return l * kStageBytes; }
  __host__ __device__ static constexpr int b_off(int l) { return l * kStageBytes + kABytes; }
  __host__ __device__ static constexpr int lo_off(int o) { return kLand * kStageBytes + o * kOpBytes; }
  __host__ __device__ static constexpr int hi_off(int o) { return lo_off(o) + kBBytes; }  // copy only
  __host__ __device__ static constexpr int bar_off() { return kRingBytes; }
  __host__ __device__ static constexpr uint32_t a_tmem_col(int o) { return kAccCols + 64u * o; }
  static_assert(!kX3 || kAccCols + 64u * kOps <= 512u, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  // Epilogue staging: eight 128-row x 32-column f32 boxes (16 KB each) reuse the ring.
  static constexpr int kEpiBoxBytes = 128 * 128;
  static_assert(8 * kEpiBoxBytes <= kRingBytes, "epilogue staging fits in the ring");
};

// Bounded pause (abort drains of loads this CTA cannot observe).
__device__ __forceinline__ void pause_ns(uint64_t ns) {
  const uint64_t t0 = globaltimer();
  while (globaltimer() - t0 < ns) __nanosleep(1000);
}

// 3xTF32 split of four f32 values into hi + lo.  SPLIT 1 (truncation): the tensor core
// reads an f32 operand as TF32 by dropping the low 13 mantissa bits, so hi = x as stored
// and lo = x - trunc(x) (exact); non-finite inputs take the per-element path.  SPLIT 0
// (round): hi = rna(x), lo = rna(x - hi).
template <int SPLIT>
__device__ __forceinline__ void split4(const float4 x, float4 &hi, float4 &lo) {
  if constexpr (SPLIT == 1) {
    bool special;
    lo = split_lo_trunc4(x, special);
    hi = x;
    if (special) {
      lo = make_float4(split_lo_trunc(x.x), split_lo_trunc(x.y), split_lo_trunc(x.z), split_lo_trunc(x.w));
      hi = make_float4(__uint_as_float(split_hi_trunc_bits(__float_as_uint(x.x))),
                       __uint_as_float(split_hi_trunc_bits(__float_as_uint(x.y))),
                       __uint_as_float(split_hi_trunc_bits(__float_as_uint(x.z))),
                       __uint_as_float(split_hi_trunc_bits(__float_as_uint(x.w))));
    }
  } else {
    hi = make_float4(to_tf32(x.x), to_tf32(x.y), to_tf32(x.z), to_tf32(x.w));
    lo.x = isfinite(hi.x) ? to_tf32(x.x - hi.x) : 0.f;
    lo.y = isfinite(hi.y) ? to_tf32(x.y - hi.y) : 0.f;
    lo.z = isfinite(hi.z) ? to_tf32(x.z - hi.z) : 0.f;
    lo.w = isfinite(hi.w) ? to_tf32(x.w - hi.w) : 0.f;
  }
}

// Peer CTA of a 3xTF32 pair: forwards "this CTA's converters finished stage kb" (local
// conv[s]) to the leader: an st.async of a 4-byte token into the leader's mailbox word for
// stage s completes the leader's ready[s] (which its MMA thread armed with expect_tx(4)).
template <int STAGES>
__device__ __forceinline__ void relay_stages(uint32_t conv0, uint32_t ready0, uint32_t mailbox0, int nkb,
                                             const WaitCtl &wc) {
  const uint32_t lead_ready0 = map_to_cta(ready0, 0), lead_mail0 = map_to_cta(mailbox0, 0);
  for (int kb = 0; kb < nkb; ++kb) {
    const int s = kb % STAGES, round = kb / STAGES;
    if (!mbar_wait(conv0 + 8 * s, round & 1, wc)) break;
    st_async_signal(lead_mail0 + 4 * s, (uint32_t)kb, lead_ready0 + 8 * s);
  }
}

template <int PREC, int STAGES, int EPI, int SPLIT, int BN, bool OUTB, bool BKM, bool BAT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairLayout<PREC, STAGES>::kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmC,
                     const TcParams p) {
  using L = PairLayout<PREC, STAGES>;
  constexpr bool kX3 = PREC == PREC_X3;
  constexpr bool kTF32 = PREC != PREC_BF16;
  // BKM (TF32, 256-wide tiles): B is a transposed copy, loaded and read K-major like A.
  static_assert(!BKM || (PREC == PREC_TF32 && BN == 256 && !OUTB), "K-major B configuration");
  // TF32, 256-wide tiles, B as given: operands exchanged (B's MN-major tile on the M side),
  // transposed epilogue.
  constexpr bool kSwap = PREC == PREC_TF32 && BN == 256 && kTf32Swap && !BKM;
  // B as given (TF32, 256-wide tiles): its tile in the k-group-major tiling (BAT, one 4-D box,
  // TcParams::b_atoms) or in column blocks.  A compile-time choice: the MMA issuer's loop is
  // on the critical path, and selecting descriptor strides at run time measured 6-8 % slower.
  using BT = BTileMN<L::kElem>;
  static_assert(!BAT || (PREC == PREC_TF32 && BN == 256 && !BKM && !OUTB), "k-group-major B configuration");
  constexpr bool b_atoms = BAT;
  constexpr uint32_t kIdesc = kSwap  ? instr_desc_a_mn(2u, 256, 256)
                              : BKM ? (instr_desc(2u, 256, 256) & ~(1u << 16))  // B K-major
                                    : instr_desc(kTF32 ? 2u : 1u, 256, BN);
  // BN = 240: each CTA's MMA half is 120 B columns (the first 120 of the 128 it loads), and
  // the accumulator's last 32-column chunk holds only 16 output columns.
  static_assert(BN == 256 || BN == 240, "pair tile width");
  // bf16 output (OUTB): BF16 precision, mbr epilogue, 256-wide tiles.
  static_assert(!OUTB || (PREC == PREC_BF16 && EPI == EPI_MBR && BN == 256), "bf16 output configuration");
  constexpr int kHalfN = BN / 2;
  constexpr bool kHalfChunk = BN % 32 != 0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::bar_off());
  // full[l]: TMA bytes of landing slot l arrived (3xTF32: this CTA's; otherwise the
  // leader's barrier counts both CTAs' bytes); lempty[l] (3xTF32): this CTA's converters
  // have loaded slot l; conv[o]: this CTA's converters filled operand slot o; ready[o]
  // (leader): the peer's converters did; empty[o]: the pair MMAs reading operand slot o
  // are done (TF32/BF16: operand slot = landing slot); accf: accumulator done; resf: C_res
  // boxes landed; biasf: the tile's bias is staged in shared memory.
  constexpr int kL = L::kLand, kO = L::kOps;
  const uint32_t full0 = smem_u32(bars), lempty0 = full0 + 8 * kL, conv0 = lempty0 + 8 * kL,
                 ready0 = conv0 + 8 * kO, empty0 = ready0 + 8 * kO, accf = empty0 + 8 * kO, resf = accf + 8,
                 biasf = resf + 8;
  float4 *bias_s = reinterpret_cast<float4 *>(smem + L::bias_off());
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + L::kNumBars);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  const uint32_t mailbox0 = smem_u32(tmem_slot + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  // Grouped raster: launch order walks kRasterGroup tile rows at a time, column by column,
  // so the tiles of one wave share a few A row panels and B column panels in L2.
  const int tiles_n = (int)(gridDim.x >> 1), tiles_m = (int)gridDim.y;
  int tile_m, tile_n;
  raster_tile((int)blockIdx.y * tiles_n + (int)(blockIdx.x >> 1), tiles_m, tiles_n, kRasterGroup, tile_m, tile_n);
  const int n0 = tile_n * BN, m0 = tile_m * 256 + (int)rank * 128;
  // Split-K: this pair takes k-blocks [kb0, kb0 + nkb) of the tile's K and stores raw
  // partial sums at row offset blockIdx.z * split_rows of the output map.
  const int nkb_all = (p.K + L::kBK - 1) / L::kBK;
  const int splits = p.splits > 1 ? p.splits : 1;
  const int kb0 = (int)((int64_t)blockIdx.z * nkb_all / splits);
  const int nkb = (int)((int64_t)(blockIdx.z + 1) * nkb_all / splits) - kb0;
  const int out_row0 = m0 + (int)blockIdx.z * p.split_rows;
  const WaitCtl wc{abort_flag, p.status, p.limit_ns};

  if (threadIdx.x == 0) {
    for (int l = 0; l < kL; ++l) {
      mbar_init(full0 + 8 * l, 1);
      // 3xTF32 with B hi read in place: the pair MMAs' commit also frees the slot.
      mbar_init(lempty0 + 8 * l, L::kConvWarps + (kPairHiDirect ? 1 : 0));
    }
    for (int o = 0; o < kO; ++o) {
      mbar_init(conv0 + 8 * o, L::kConvWarps);
      mbar_init(ready0 + 8 * o, 1);
      mbar_init(empty0 + 8 * o, 1);
    }
    mbar_init(accf, 1);
    mbar_init(resf, 1);
    mbar_init(biasf, 2);  // warps 2 and 3
    *abort_flag = 0u;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmO);
    if constexpr (EPI == EPI_ADD) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers are initialised before any remote arrive or TMA
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if constexpr (EPI == EPI_MBR) {
    // Warps 2 and 3 stage this tile's 256 bias values (64 float4; N is a multiple of 4 and
    // bias 16-byte aligned on this path) while the first loads are in flight, so the
    // epilogue reads bias from shared memory instead of waiting on global loads per chunk.
    if (warp == 2 || warp == 3) {
      const int i = threadIdx.x - 64, col = n0 + 4 * i;
      bias_s[i] = col < p.N ? __ldg(reinterpret_cast<const float4 *>(p.bias + col)) : make_float4(0.f, 0.f, 0.f, 0.f);
      __syncwarp();
      if (lane == 0) mbar_arrive(biasf);
    }
  }

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    grid_dependency_wait();  // operands written by the kernel before this launch (TcParams::pdl)
    // 3xTF32: loads complete on this CTA's full[l]; the slot is reused once this CTA's
    // converters have loaded it (lempty[l]).  TF32/BF16: loads complete on the LEADER's
    // full[l], which expects both CTAs' bytes; the slot is reused once the pair MMAs that
    // read it are done (empty[l], committed to both CTAs).
    const uint32_t lead_full0 = map_to_cta(full0, 0);
    int kb = 0;
    for (; kb < nkb; ++kb) {
      const int s = kb % kL, round = kb / kL;
      if (round > 0) {
        const bool ok = kX3 ? mbar_wait(lempty0 + 8 * s, (round - 1) & 1, wc)
                            : mbar_wait_cluster(empty0 + 8 * s, (round - 1) & 1, wc);
        if (!ok) break;
      }
      if (p.debug_skip && kb == 0) continue;  // test hook: this stage never fills
      const int kc = (kb0 + kb) * L::kBK;
      const int nb = n0 + (int)rank * kHalfN;
      if constexpr (kX3) {
        mbar_arrive_expect_tx(full0 + 8 * s, L::kStageBytes);
        tma_load_2d(sbase + L::a_off(s), &tmA, kc, m0, full0 + 8 * s);
#pragma unroll
        for (int j = 0; j < L::kBBlocks; ++j)
          tma_load_2d(sbase + L::b_off(s) + j * (L::kBK * 128), &tmB, nb + j * L::kNBlk, kc, full0 + 8 * s);
      } else {
        if (rank == 0) mbar_arrive_expect_tx(full0 + 8 * s, 2 * L::kStageBytes);
        tma_load_2d_pair(sbase + L::a_off(s), &tmA, kc, m0, lead_full0 + 8 * s);
        if constexpr (BKM) {
          tma_load_2d_pair(sbase + L::b_off(s), &tmB, kc, nb, lead_full0 + 8 * s);  // 128 n-rows x 32 k
        } else if constexpr (b_atoms) {
          tma_load_4d_pair(sbase + L::b_off(s), &tmB, 0, 0, nb / L::kNBlk, kc / BT::kRows, lead_full0 + 8 * s);
        } else {
#pragma unroll
          for (int j = 0; j < L::kBBlocks; ++j)
            tma_load_2d_pair(sbase + L::b_off(s) + j * (L::kBK * 128), &tmB, nb + j * L::kNBlk, kc,
                             lead_full0 + 8 * s);
        }
      }
    }
    if (*abort_flag) {
      if (kX3 || rank == 0) {
#pragma unroll 1
        for (int s = 0; s < kL; ++s) {
          if (kb - 1 < s) continue;
          const int last = kb - 1 - ((kb - 1 - s) % kL);
          if (p.debug_skip && last == 0) continue;
          mbar_wait_drain_cluster(full0 + 8 * s, (last / kL) & 1, p.limit_ns);
        }
      } else {
        pause_ns(200000);  // the peer's loads complete on the leader's barrier
      }
    }
  } else if (warp == 1 && lane == 0) {
    if (rank == 0) {
      // ---------------- pair MMA issuer (leader CTA) ----------------
      // This thread's loop is on the critical path: ring positions are kept incrementally
      // (slot s of kO with phase ph; 3xTF32 landing slot land of kL) and the descriptors are the
      // slot-0 ones plus constant offsets in 16-B units.
      uint32_t accum = 0, ph = 0;
      int s = 0, land = 0;
      uint32_t s_off = 0, land_off = 0;  // 16-B units: slot s, landing slot land
      constexpr uint32_t kSlot16 = (kX3 ? L::kOpBytes : L::kStageBytes) >> 4, kLand16 = L::kStageBytes >> 4;
      constexpr uint32_t kBStep = BKM ? 2u : BT::step(b_atoms) >> 4;
      const uint64_t a_d0 = smem_desc(sbase + L::a_off(0), 16, 1024, 2);
      const uint64_t b_d0 = BKM ? smem_desc(sbase + L::b_off(0), 16, 1024, 2) : BT::desc(sbase + L::b_off(0), 0, b_atoms);
      const uint64_t lo_d0 = BT::desc(sbase + L::lo_off(0), 0, false);  // 3xTF32 B lo (operand slot)
      const uint64_t hi_d0 = BT::desc(sbase + (kPairHiDirect ? L::b_off(0) : L::hi_off(0)), 0, false);
      for (int kb = 0; kb < nkb; ++kb) {
        if constexpr (kX3) {
          if (!mbar_wait(conv0 + 8 * s, ph, wc)) break;
          mbar_arrive_expect_tx(ready0 + 8 * s, 4);  // the peer's token for this round
          if (!mbar_wait_cluster(ready0 + 8 * s, ph, wc)) break;
        } else {
          if (!mbar_wait_cluster(full0 + 8 * s, ph, wc)) break;
        }
        tc_fence_after();
        // 3xTF32: landing slot `land` holds this k-block's raw B (= B hi).
        const uint64_t bl = lo_d0 + s_off, bh = hi_d0 + (kPairHiDirect ? land_off : s_off);
        const uint64_t ad = a_d0 + s_off, bd = b_d0 + s_off;
        const uint32_t a_hi0 = tmem + L::a_tmem_col(s);
#pragma unroll
        for (int ks = 0; ks < L::kKSteps; ++ks) {
          if constexpr (kX3) {
            const uint32_t a_hi = a_hi0 + 8 * ks, a_lo = a_hi + 32;
            mma_ts_pair_tf32(tmem, a_lo, bh + ks * kBStep, kIdesc, accum);
            mma_ts_pair_tf32(tmem, a_hi, bl + ks * kBStep, kIdesc, 1u);
            mma_ts_pair_tf32(tmem, a_hi, bh + ks * kBStep, kIdesc, 1u);
          } else {
            if constexpr (kSwap)
              mma_ss_pair<kTF32>(tmem, bd + ks * kBStep, ad + 2 * ks, kIdesc, accum);
            else
              mma_ss_pair<kTF32>(tmem, ad + 2 * ks, bd + ks * kBStep, kIdesc, accum);
          }
          accum = 1u;
        }
        mma_commit_pair(empty0 + 8 * s, 0x3);
        if constexpr (kX3 && kPairHiDirect) mma_commit_pair(lempty0 + 8 * land, 0x3);
        if (++s == kO) {
          s = 0;
          s_off = 0;
          ph ^= 1u;
        } else {
          s_off += kSlot16;
        }
        if constexpr (kX3) {
          if (++land == kL) {
            land = 0;
            land_off = 0;
          } else {
            land_off += kLand16;
          }
        }
      }
      mma_commit_pair(accf, 0x3);
      if (*abort_flag) mbar_wait_drain_cluster(accf, 0, p.limit_ns);
    } else if constexpr (kX3) {
      relay_stages<kO>(conv0, ready0, mailbox0, nkb, wc);
    }
  } else if (kX3 && warp >= 2) {
    // ---------------- 3xTF32 converters (both CTAs, warps 2..11) ----------------
    // k-block kb: landing slot l = kb % kLand, operand slot o = kb % kOps.  Each thread
    // loads its B chunks (t + 320 i) and, in warps 4..11, four 16-B chunks of A row r (K
    // half h), and arrives on lempty[l] before it splits.  It then waits until the MMAs of
    // k-block kb - kOps have finished with operand slot o (empty[o]) and writes B lo there
    // at the offsets TMA used (same swizzle), and A hi and lo into the TMEM columns of
    // slot o.
    const int t = threadIdx.x - 64;
    constexpr int kChunks = L::kBBytes / 16;
    const int q = warp & 3, h = (warp - 4) >> 2, r = q * 32 + lane;
    for (int kb = 0; kb < nkb; ++kb) {
      const int l = kb % kL, o = kb % kO;
      if (!mbar_wait(full0 + 8 * l, (kb / kL) & 1, wc)) break;
      const float4 *braw = reinterpret_cast<const float4 *>(smem + L::b_off(l));
      // Row r of the A tile: 128 B at r * 128, 16-B chunk j stored at j ^ (r % 8).
      const uint8_t *arow = smem + L::a_off(l) + r * 128;
      float4 xb[4], xa[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (t + 320 * i < kChunks) xb[i] = braw[t + 320 * i];
      if (warp >= 4) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          xa[jj] = *reinterpret_cast<const float4 *>(arow + (((4 * h + jj) ^ (r & 7)) << 4));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(lempty0 + 8 * l);
      if (kb >= kO && !mbar_wait_cluster(empty0 + 8 * o, ((kb / kO) - 1) & 1, wc)) break;
      float4 *bhi = reinterpret_cast<float4 *>(smem + L::hi_off(o));
      float4 *blo = reinterpret_cast<float4 *>(smem + L::lo_off(o));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = t + 320 * i;
        if (c < kChunks) {
          if constexpr (kPairHiDirect) {
            // B hi stays in the landing slot; a non-finite chunk (rare) gets its hi patched
            // there (NaN kept quiet after the tensor core drops the low 13 bits).
            bool special;
            float4 ll = split_lo_trunc4(xb[i], special);
            if (special) {
              float4 hh;
              split4<SPLIT>(xb[i], hh, ll);
              reinterpret_cast<float4 *>(smem + L::b_off(l))[c] = hh;
            }
            blo[c] = ll;
          } else {
            float4 hh, ll;
            split4<SPLIT>(xb[i], hh, ll);
            bhi[c] = hh;
            blo[c] = ll;
          }
        }
      }
      fence_proxy_async_smem();
      if (warp >= 4) {
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          float4 hh, ll;
          split4<SPLIT>(xa[jj], hh, ll);
          hi[4 * jj + 0] = __float_as_uint(hh.x);
          hi[4 * jj + 1] = __float_as_uint(hh.y);
          hi[4 * jj + 2] = __float_as_uint(hh.z);
          hi[4 * jj + 3] = __float_as_uint(hh.w);
          lo[4 * jj + 0] = __float_as_uint(ll.x);
          lo[4 * jj + 1] = __float_as_uint(ll.y);
          lo[4 * jj + 2] = __float_as_uint(ll.z);
          lo[4 * jj + 3] = __float_as_uint(ll.w);
        }
        const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + L::a_tmem_col(o) + 16 * h;
        tmem_st_32x32b_x16(ta, hi);
        tmem_st_32x32b_x16(ta + 32, lo);
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(conv0 + 8 * o);
    }
  }

  // ---------------- epilogue: TMEM -> registers -> smem -> TMA store (both CTAs) ----------------
  // Column chunk c (32 columns) of this CTA's 128 rows: the warp of TMEM lane quadrant q
  // takes rows 32 q .. +31, applies the epilogue and writes them into staging box c
  // (128-B swizzle: 16-B unit j of row r at unit j ^ (r % 8), matching the output tensor
  // map); after the four quadrant warps of chunk c meet at named barrier 1 + c, one thread
  // stores the box with TMA, which clips rows >= M and columns >= N.  The ring is free:
  // every load was consumed before accf.  matmul_add first brings its C_res boxes in the
  // same way (TMA loads into the boxes, then in-place update).
  if (warp >= L::kEpiWarp0 && warp < L::kEpiWarp0 + L::kEpiWarps) {
    // One thread waits (bounded) for the accumulator and publishes the outcome, so every
    // epilogue warp takes the same branch and the named barriers below cannot be left
    // waiting for a warp that gave up.
    constexpr int kEpiThreads = 32 * L::kEpiWarps;
    volatile uint32_t *epi_ok = tmem_slot + 2;
    if (warp == 4 && lane == 0)
      *epi_ok = (mbar_wait_cluster(accf, 0, wc, 128) && (EPI != EPI_MBR || mbar_wait(biasf, 0, wc))) ? 1u : 0u;
    named_barrier(9, kEpiThreads);
    if (kSwap && *epi_ok) {
      // Transposed accumulator: thread (q, lane) holds output column nb + r for the 256 rows
      // mp0 .. mp0 + 255, 32 per chunk c; chunk c goes through box c (32 rows x 128 columns,
      // row-major, no swizzle: a warp writes 128 consecutive bytes per row) and one TMA store.
      tc_fence_after();
      const int q = warp & 3, r = q * 32 + lane;
      const int mp0 = m0 - (int)rank * 128, nb = n0 + (int)rank * 128;
      const bool cta_cols = nb < p.N;
      const int split_off = (int)blockIdx.z * p.split_rows;
      const float *bias_f = reinterpret_cast<const float *>(bias_s);
      const float bcol = EPI == EPI_MBR ? bias_f[(int)rank * 128 + r] : 0.f;  // 0 beyond N
      bool res_ok = true;
      if constexpr (EPI == EPI_ADD) {
        if (warp == 4 && lane == 0 && cta_cols) {
          mbar_arrive_expect_tx(resf, 8 * L::kEpiBoxBytes);
#pragma unroll 1
          for (int c = 0; c < 8; ++c) tma_load_2d(sbase + c * L::kEpiBoxBytes, &tmC, nb, mp0 + 32 * c, resf);
        }
        res_ok = !cta_cols || mbar_wait_cluster(resf, 0, wc);
      }
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t rr[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, rr);
        tmem_ld_wait(rr);
        const int row0 = mp0 + 32 * c;
        float *box = reinterpret_cast<float *>(smem + c * L::kEpiBoxBytes);
        const bool live = res_ok && cta_cols && row0 < p.M;
        if (live) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float v = __uint_as_float(rr[i]);
            if constexpr (EPI == EPI_MBR) v = relu_ieee(__fadd_rn(v, bcol));
            else if constexpr (EPI == EPI_ADD) v = __fadd_rn(v, box[i * 128 + r]);
            box[i * 128 + r] = v;
          }
        }
        fence_proxy_async_smem();
        named_barrier(1 + c, 128);
        if (q == 0 && lane == 0 && live) {
          tma_store_2d(&tmO, sbase + c * L::kEpiBoxBytes, nb, row0 + split_off);
          bulk_commit_group();
        }
      }
      if (q == 0 && lane == 0) bulk_wait_group_read0();  // staging stays valid until read
    } else if (*epi_ok) {
      tc_fence_after();
      constexpr int kGroups = L::kEpiWarps / 4;  // group g takes column chunks g, g + kGroups, ...
      const int q = warp & 3;
      const int g = (warp - L::kEpiWarp0) >> 2;
      const int r = q * 32 + lane;  // row within this CTA's 128 rows
      const bool cta_rows = m0 < p.M;
      bool res_ok = true;
      if constexpr (EPI == EPI_ADD) {
        if (warp == 4 && lane == 0 && cta_rows) {
          mbar_arrive_expect_tx(resf, 8 * L::kEpiBoxBytes);
#pragma unroll 1
          for (int c = 0; c < 8; ++c)
            tma_load_2d(sbase + c * L::kEpiBoxBytes, &tmC, n0 + c * 32, m0, resf);
        }
        res_ok = !cta_rows || mbar_wait_cluster(resf, 0, wc);
      }
#pragma unroll 1
      for (int c = g; c < 8; c += kGroups) {
        uint32_t rr[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, rr);
        tmem_ld_wait(rr);
        const int col0 = n0 + c * 32;
        uint8_t *box = smem + c * L::kEpiBoxBytes + r * 128;
        // Epilogue of columns col0 + 4 j .. + 3 (matmul_add: the residual sits in the box).
        auto finish = [&](int j) {
          float4 v = make_float4(__uint_as_float(rr[4 * j]), __uint_as_float(rr[4 * j + 1]),
                                 __uint_as_float(rr[4 * j + 2]), __uint_as_float(rr[4 * j + 3]));
          if constexpr (EPI == EPI_MBR) {
            const float4 b = bias_s[c * 8 + j];
            v.x = relu_ieee(__fadd_rn(v.x, b.x));
            v.y = relu_ieee(__fadd_rn(v.y, b.y));
            v.z = relu_ieee(__fadd_rn(v.z, b.z));
            v.w = relu_ieee(__fadd_rn(v.w, b.w));
          } else if constexpr (EPI == EPI_ADD) {
            const float4 cr = *reinterpret_cast<const float4 *>(box + ((j ^ (r & 7)) << 4));
            v.x = __fadd_rn(v.x, cr.x);
            v.y = __fadd_rn(v.y, cr.y);
            v.z = __fadd_rn(v.z, cr.z);
            v.w = __fadd_rn(v.w, cr.w);
          }
          return v;
        };
        if (kHalfChunk && c == 7) {
          // The last 16 columns of a 240-wide tile: the other half of a 32-column box
          // belongs to the next tile, so each thread stores its row's 16 values directly
          // (no split-K on this width: out_row0 == m0).
          if (res_ok && m0 + r < p.M && col0 < p.N) {
            float *orow = p.out + (int64_t)(m0 + r) * p.ldc;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 v = finish(j);
              const int col = col0 + 4 * j;
              if (col + 3 < p.N) {
                *reinterpret_cast<float4 *>(orow + col) = v;
              } else {
                if (col < p.N) orow[col] = v.x;
                if (col + 1 < p.N) orow[col + 1] = v.y;
                if (col + 2 < p.N) orow[col + 2] = v.z;
              }
            }
          }
          continue;  // every warp of this chunk takes this branch: no named barrier
        }
        if constexpr (OUTB) {
          // bf16 output: the chunk's 32 values of row r become 64 B in box c of 128 rows x
          // 64 B (64-B swizzle: 16-B unit u of row r at unit u ^ ((r >> 1) & 3), matching the
          // bf16 output map), stored by TMA like the f32 boxes.
          uint8_t *bbox = smem + c * kEpiBoxBytesB + r * 64;
          if (res_ok && cta_rows && col0 < p.N) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float4 v0 = finish(2 * u), v1 = finish(2 * u + 1);
              uint4 pk;
              pk.x = pack_bf16x2(v0.x, v0.y);
              pk.y = pack_bf16x2(v0.z, v0.w);
              pk.z = pack_bf16x2(v1.x, v1.y);
              pk.w = pack_bf16x2(v1.z, v1.w);
              *reinterpret_cast<uint4 *>(bbox + ((u ^ ((r >> 1) & 3)) << 4)) = pk;
            }
          }
          fence_proxy_async_smem();
          named_barrier(1 + c, 128);
          if (q == 0 && lane == 0 && res_ok && cta_rows && col0 < p.N) {
            tma_store_2d(&tmO, sbase + c * kEpiBoxBytesB, col0, out_row0);
            bulk_commit_group();
          }
          continue;
        }
        if (res_ok && cta_rows && col0 < p.N) {
#pragma unroll
          for (int j = 0; j < 8; ++j) *reinterpret_cast<float4 *>(box + ((j ^ (r & 7)) << 4)) = finish(j);
        }
        fence_proxy_async_smem();
        named_barrier(1 + c, 128);
        if (q == 0 && lane == 0 && res_ok && cta_rows && col0 < p.N) {
          tma_store_2d(&tmO, sbase + c * L::kEpiBoxBytes, col0, out_row0);
          bulk_commit_group();
        }
      }
      if (q == 0 && lane == 0) bulk_wait_group_read0();  // staging stays valid until read
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while the pair MMA may still read its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, L::kTmemCols);
  }
}

template <int PREC, int STAGES, int EPI, int BN, bool OUTB, bool BKM = false, bool BAT = false>
cudaError_t launch_pair_kern(const CUtensorMap &tmA, const CUtensorMap &tmB, const CUtensorMap &tmO,
                             const CUtensorMap &tmC, const TcParams &p, cudaStream_t stream) {
  using L = PairLayout<PREC, STAGES>;
  auto kern = gemm_pair_kernel<PREC, STAGES, EPI, kPairSplit, BN, OUTB, BKM, BAT>;
  static unsigned long long configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(__atomic_load_n(&configured, __ATOMIC_ACQUIRE) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
    if (e != cudaSuccess) return e;
    __atomic_fetch_or(&configured, bit, __ATOMIC_RELEASE);
  }
  dim3 grid(2 * ((p.N + BN - 1) / BN), (p.M + 255) / 256, p.splits > 1 ? p.splits : 1);
  if (p.pdl) {
    cudaLaunchAttribute attr[1];
    pdl_attr(attr[0]);
    cudaLaunchConfig_t cfg = {grid, dim3(L::kThreads), (size_t)L::kSmemBytes, stream, attr, 1};
    return cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmO, tmC, p);
  }
  kern<<<grid, L::kThreads, L::kSmemBytes, stream>>>(tmA, tmB, tmO, tmC, p);
  return cudaGetLastError();
}

template <int PREC, int STAGES, int EPI, int BN>
cudaError_t launch_pair_one(const CUtensorMap &tmA, const CUtensorMap &tmB, const CUtensorMap &tmO,
                            const CUtensorMap &tmC, const TcParams &p, cudaStream_t stream) {
  // The 240-wide tile stores its last 16 columns through p.out, so it takes no split-K.
  if (BN != 256 && p.splits > 1) return cudaErrorInvalidValue;
  if (p.b_kmajor) {
    if constexpr (PREC == PREC_TF32 && BN == 256)
      return p.out_bf16 ? cudaErrorInvalidValue
                        : launch_pair_kern<PREC, STAGES, EPI, BN, false, true>(tmA, tmB, tmO, tmC, p, stream);
    return cudaErrorInvalidValue;
  }
  if (p.out_bf16) {
    if constexpr (PREC == PREC_BF16 && EPI == EPI_MBR && BN == 256)
      return p.splits > 1 ? cudaErrorInvalidValue
                          : launch_pair_kern<PREC, STAGES, EPI, BN, true>(tmA, tmB, tmO, tmC, p, stream);
    return cudaErrorInvalidValue;
  }
  if (p.b_atoms) {
    if constexpr (PREC == PREC_TF32 && BN == 256)
      return launch_pair_kern<PREC, STAGES, EPI, BN, false, false, true>(tmA, tmB, tmO, tmC, p, stream);
    return cudaErrorInvalidValue;
  }
  return launch_pair_kern<PREC, STAGES, EPI, BN, false>(tmA, tmB, tmO, tmC, p, stream);
}

template <int PREC, int STAGES, int BN>
cudaError_t launch_pair_epi(int epi, const CUtensorMap &tmA, const CUtensorMap &tmB, const CUtensorMap &tmO,
                            const CUtensorMap &tmC, const TcParams &p, cudaStream_t stream) {
  switch (epi) {
    case EPI_MATMUL: return launch_pair_one<PREC, STAGES, EPI_MATMUL, BN>(tmA, tmB, tmO, tmC, p, stream);
    case EPI_MBR: return launch_pair_one<PREC, STAGES, EPI_MBR, BN>(tmA, tmB, tmO, tmC, p, stream);
    case EPI_ADD: return launch_pair_one<PREC, STAGES, EPI_ADD, BN>(tmA, tmB, tmO, tmC, p, stream);
  }
  return cudaErrorInvalidValue;
}

template <int PREC, int STAGES, int BN>
cudaError_t pair_attrs(int epi, cudaFuncAttributes *a, int *blocks) {
  using L = PairLayout<PREC, STAGES>;
  const void *f = epi == EPI_MBR   ? reinterpret_cast<const void *>(gemm_pair_kernel<PREC, STAGES, EPI_MBR, kPairSplit, BN, false, false, false>)
                  : epi == EPI_ADD ? reinterpret_cast<const void *>(gemm_pair_kernel<PREC, STAGES, EPI_ADD, kPairSplit, BN, false, false, false>)
                                   : reinterpret_cast<const void *>(gemm_pair_kernel<PREC, STAGES, EPI_MATMUL, kPairSplit, BN, false, false, false>);
  cudaError_t e = cudaFuncGetAttributes(a, f);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, f, L::kThreads, L::kSmemBytes);
}

}  // namespace

// Instantiated pair configurations: (precision, stages).
#define TF_PAIR_CONFIGS(X) X(PREC_X3, kPairX3Land) X(PREC_TF32, 6) X(PREC_BF16, 6)

int pair_smem_bytes(int prec, int stages) {
#define TF_PSMEM(P, S) \
  if (prec == P && stages == S) return PairLayout<P, S>::kSmemBytes;
  TF_PAIR_CONFIGS(TF_PSMEM)
#undef TF_PSMEM
  return -1;
}

int pair_tmem_cols(int prec) { return prec == PREC_X3 ? 512 : 256; }

bool pair_transposed(int prec, int bn) { return prec == PREC_TF32 && bn == 256 && kTf32Swap; }

cudaError_t launch_gemm_pair(int prec, int stages, int bn, int epi, const CUtensorMap &tmA,
                             const CUtensorMap &tmB, const CUtensorMap &tmO, const CUtensorMap &tmC,
                             const TcParams &p, cudaStream_t stream) {
#define TF_PLAUNCH(P, S)                                                                              \
  if (prec == P && stages == S && bn == 256) return launch_pair_epi<P, S, 256>(epi, tmA, tmB, tmO, tmC, p, stream); \
  if (prec == P && stages == S && bn == 240) return launch_pair_epi<P, S, 240>(epi, tmA, tmB, tmO, tmC, p, stream);
  TF_PAIR_CONFIGS(TF_PLAUNCH)
#undef TF_PLAUNCH
  return cudaErrorInvalidValue;
}

cudaError_t pair_func_attributes(int prec, int stages, int bn, int epi, cudaFuncAttributes *a, int *blocks) {
#define TF_PATTR(P, S)                                                               \
  if (prec == P && stages == S && bn == 256) return pair_attrs<P, S, 256>(epi, a, blocks); \
  if (prec == P && stages == S && bn == 240) return pair_attrs<P, S, 240>(epi, a, blocks);
  TF_PAIR_CONFIGS(TF_PATTR)
#undef TF_PATTR
  return cudaErrorInvalidValue;
}

}  // namespace tf
