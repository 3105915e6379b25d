// phi GEMM on the sm_100a tensor cores: out = act(x W^T + bias) [* temp].
//
// The feature map of the default FA-KLA configuration is one nn.Linear over
// the full H*Dk projected row followed by elu+1 (LearnablePositiveMap,
// ultra_rwka/kernels/feature_maps.py:224,248,259-268); at B=8, T=4096,
// H*Dk=2048 it is ~90% of the FA-KLA FLOPs. This kernel computes it for up to
// two row sets in one launch (q rows and k rows share W), with the bias,
// the activation and the k-side temperature (k~ = phi(k) * temp,
// cpu_kernels.cpp:121-123) fused into the epilogue, and writes bf16. The
// activation is a template parameter: elu+1 for FA-KLA, and the other
// FAKLA_ACT_* forms for the rest of the feature-map family (LearnablePositive
// Map's relu/softplus/gelu, MLP hidden layers, gate logits, and the cos/sin
// pairs of random Fourier features, written to columns n and N + n).
//
// Structure: persistent CTAs (one per SM), 10 warps:
//   warp 0      TMA producer: 128x64 x-tile + 256x64 W-tile per stage (4 stages)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (128x256x16)
//   warps 2..9  epilogue, two warps per TMEM lane quadrant (each takes 128 of
//               the 256 columns): TMEM -> registers -> bias/elu+1/temp ->
//               bf16 -> 128B-swizzled staging -> TMA store (32 rows x 64 cols)
// The 128x256 fp32 accumulator is double-buffered in TMEM (2 x 256 columns),
// so the epilogue of tile i overlaps the MMAs of tile i+1. The epilogue is
// sized to keep up with the tensor pipe: with it skipped the main loop was
// measured at 98% of the bf16 peak, and a 4-warp epilogue with an accurate
// exp cost 80% on top of that.
//
// Large GEMMs run the same kernel as CTA pairs (clusters of two): a pair
// computes a 256x256 tile with cta_group::2 MMAs (256x256x16) issued by rank
// 0; each CTA loads its 128 x rows and 128 of the tile's 256 W rows for two
// 64-wide K slabs per stage (3 stages of 64 KB), so each SM moves a third
// fewer operand bytes per FLOP through L2 and shared memory. Rank 0's commits arrive on both CTAs'
// barriers; each CTA runs the epilogue of its own 128 rows from its own TMEM.
//
// A persistent grid gives every pair the tiles tile0, tile0 + pairs, ...; when
// the tile count leaves a last wave less than half full (e.g. 256 tiles on 74
// pairs: 3 waves + 34 tiles), those last tiles run as two 256x128 halves each
// (N=128 MMAs, a W map with a 64-row box), so the tail takes half a tile's time
// on twice as many pairs instead of a whole tile's time on a few.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "fakla_common.cuh"
#include "fakla_kernels.h"
#include "sm100_umma.cuh"

namespace fakla {
namespace {

using namespace sm100;

constexpr int BM = 128;   // rows of a tile per CTA
constexpr int BN = 256;   // N tile; 128 (BNT below) when 256-wide tiles would not fill the GPU
constexpr int BK = 64;
constexpr int kABytes = BM * BK * 2;                 // 16 KB
// Per CTA: a single CTA holds all BNT rows of the W tile; a CTA pair splits them.
template <int BNT, bool PAIR> constexpr int kBRowsT = PAIR ? BNT / 2 : BNT;
template <int BNT, bool PAIR> constexpr int kBBytesT = kBRowsT<BNT, PAIR> * BK * 2;
// K slabs of BK per pipeline stage. One thread issues every MMA, and each
// MMA instruction takes it about 70 cycles to issue while each stage adds a
// barrier wait and a commit (about 300 cycles): with one slab a CTA pair's
// four 256x256x16 MMAs (128 cycles of tensor pipe each) could not be issued
// as fast as the pipe ran them. Two slabs put eight MMAs behind each round
// trip. Single CTAs and the MN-major forms keep one slab.
template <int BNT, bool PAIR, bool AMN, bool BMN>
constexpr int kSlabsT = (PAIR && !AMN && !BMN) ? 2 : 1;
template <int BNT, bool PAIR, int SL> constexpr int kStageBytesT = SL * (kABytes + kBBytesT<BNT, PAIR>);
// 4 stages of 48 KB (single CTA, BNT 256), 6 of 32 KB (pair, one slab) or
// 3 of 64 KB (pair, two slabs)
template <int BNT, bool PAIR, int SL> constexpr int kStagesT = PAIR ? (SL == 2 ? 3 : 6) : 4;
constexpr int kEpiWarps = 8;
constexpr int kOutWarpBytes = 32 * 128;              // 32 rows x 64 bf16
constexpr int kOutBytes = kEpiWarps * kOutWarpBytes;  // 32 KB (one buffer per warp)
constexpr int kThreads = 64 + 32 * kEpiWarps;        // 320
constexpr uint32_t kEpiBarrier = 1;                  // named barrier of the epilogue warps
template <int BNT> constexpr uint32_t kTmemColsT = 2 * BNT;  // 512 (BNT = 256)
constexpr uint64_t kWaitNs = 2000000000ull;          // 2 s per wait
// Suspend-time hint of the pipeline's barrier polls: a waiting thread sleeps
// until the phase completes (or this long) instead of spinning, so the
// producer, the MMA issuer and the epilogue's poller spend few issue slots.
constexpr uint32_t kSleepNs = 50000;

template <int BNT, bool PAIR, int SL = 1>
constexpr size_t kSmemBytesT = 1024 /*align slack*/ +
                               (size_t)kStagesT<BNT, PAIR, SL> * kStageBytesT<BNT, PAIR, SL> + kOutBytes + 256;

// x - 2 pi k with k = round(x / (2 pi)): the cos/sin argument brought into
// [-pi, pi] (Cody-Waite reduction with 2 pi split into a float head and the
// remainder, both subtracted by fma), where the hardware sin/cos are accurate
// to about 2^-21 absolute, far below the bf16 rounding of the output (the
// output is rounded to bf16; fp32 maps use sincosf on the CUDA cores).
__device__ __forceinline__ float reduce_2pi(float x) {
  constexpr float kInv2Pi = 0.159154943091895336f;
  constexpr float k2PiHi = 6.28318548202514648f;    // float(2 pi)
  constexpr float k2PiLo = -1.7484556025237907e-07f;  // 2 pi - float(2 pi)
  const float k = rintf(x * kInv2Pi);
  return fmaf(-k, k2PiLo, fmaf(-k, k2PiHi, x));
}

// 2^x by the MUFU's approximation (relative error far below the bf16
// rounding applied to the output); as raw bits.
__device__ __forceinline__ uint32_t ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return __float_as_uint(r);
}

struct PhiArgs {
  const __nv_bfloat16* bias;   // [N] or null
  float scale;                 // FAKLA_ACT_COSSIN output scale
  const __nv_bfloat16* temp0;  // [rows, heads] or null (row set 0)
  const __nv_bfloat16* temp1;  // [rows, heads] or null (row set 1)
  int rows, N, K, heads, nsets;
  int m;                       // features per head (temperature index = (col - tcol0) / m)
  int ident_from;              // columns >= ident_from skip the activation (N: none)
  int tcol0, tcol1;            // temperature applies to columns [tcol0, tcol1)
  int n_full;                  // tiles [0, n_full) run whole, the rest as two column halves
  int a_rows;                  // rows of x per A box (BM, or fewer when a row set has fewer
                               // than BM rows: the rest of each A stage stays zero)
  int* status;
};

// PAIR: launched in clusters of two CTAs on neighbouring SMs that compute a
// 256 x BNT tile together with cta_group::2 MMAs (rank 0 issues them; each
// CTA loads its 128 rows of x and half of the W tile and runs the epilogue of
// its 128 rows), so each SM streams a third fewer operand bytes per FLOP.
// AMN / BMN: the A (x) / B (W) operand is stored MN-major, i.e. as (K, M) /
// (K, N) row-major matrices (the transposed operands of a linear layer's
// input and weight gradients); each stage then holds 64-row K slabs of 64-wide
// MN atoms (kMnAtom bytes apart) loaded as 64 x 64 boxes.
constexpr int kMnAtom = BK * 128;  // 8 KB: 64 K rows x 64 MN elements
template <int ACT, int BNT, bool PAIR, bool AMN = false, bool BMN = false>
__global__ void __launch_bounds__(kThreads, 1) phi_gemm_sm100_kernel(
    const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
    const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmBh,
    const __grid_constant__ CUtensorMap tmC0, const __grid_constant__ CUtensorMap tmC1,
    const PhiArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int SL = kSlabsT<BNT, PAIR, AMN, BMN>;
  constexpr int kStages = kStagesT<BNT, PAIR, SL>;
  constexpr int kBBytes = kBBytesT<BNT, PAIR>;
  constexpr int kAStage = SL * kABytes;  // A bytes per stage (SL slabs of kABytes)
  constexpr int kBStage = SL * kBBytes;
  constexpr uint32_t kTmemCols = kTmemColsT<BNT>;
  constexpr int kTileRows = PAIR ? 2 * BM : BM;
  uint8_t* sA = smem;                                  // kStages x kAStage
  uint8_t* sB = smem + kStages * kAStage;              // kStages x kBStage
  uint8_t* sOut = sB + kStages * kBStage;              // 32 KB (1024-aligned)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + kOutBytes);
  uint64_t* full = bars;                  // [kStages]
  uint64_t* empty = bars + kStages;       // [kStages]
  uint64_t* tfull = bars + 2 * kStages;   // [2]
  uint64_t* tempty = tfull + 2;           // [2]
  uint64_t* drain = tempty + 2;           // [1] MMAs in flight after an abort
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;  // 0 issues the MMAs
  const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tile_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  const int row_tiles = (args.rows + kTileRows - 1) / kTileRows;
  const int col_tiles = args.N / BNT;
  const int tiles_per_set = row_tiles * col_tiles;
  const int total_tiles = tiles_per_set * args.nsets;
  // stages of SL * BK along K; a ragged last one reads zeros past K
  const int kblocks = (args.K + SL * BK - 1) / (SL * BK);
  // work units: whole tiles [0, n_full), then each remaining tile as two
  // halves of BNT / 2 columns (CTA pairs only; the host passes n_full =
  // total_tiles otherwise)
  const int n_full = args.n_full;
  const int total_units = n_full + 2 * (total_tiles - n_full);
  struct Unit {
    int set, r;   // row set and tile within it
    bool whole;
    int coff;     // column offset of the unit within its tile (0 or BNT / 2)
  };
  auto unit_at = [&](int u) {
    Unit t;
    const bool whole = u < n_full;
    const int tile = whole ? u : n_full + ((u - n_full) >> 1);
    t.set = tile / tiles_per_set;
    t.r = tile % tiles_per_set;
    t.whole = whole;
    t.coff = whole ? 0 : ((u - n_full) & 1) * (BNT / 2);
    return t;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], PAIR ? 2 * kEpiWarps : kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA0);
    tma_prefetch_desc(&tmA1);
    tma_prefetch_desc(&tmB);
    if (n_full < total_tiles) tma_prefetch_desc(&tmBh);
    tma_prefetch_desc(&tmC0);
    tma_prefetch_desc(&tmC1);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  // A row set of fewer than BM rows (a decode step of few sequences) loads only
  // its rows: the TMA would otherwise move the zero fill of a whole BM-row box
  // through the crossbar on every stage. The rows past a_rows are zeroed once
  // here and never written again, so the MMAs read zeros there.
  if constexpr (!PAIR && !AMN) {
    if (args.a_rows < BM) {
      const int from = args.a_rows * 128 / 16, to = BM * 128 / 16;  // uint4 offsets within a stage
      for (int s = 0; s < kStages; ++s) {
        uint4* dst = reinterpret_cast<uint4*>(sA + s * kAStage);  // one slab (single CTAs)
        for (int o = from + (int)threadIdx.x; o < to; o += kThreads) dst[o] = make_uint4(0u, 0u, 0u, 0u);
      }
      fence_proxy_async_smem();
    }
  }
  tc_fence_before();
  __syncthreads();
  // a pair's barriers must be initialised before the other CTA signals them
  if constexpr (PAIR) cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // set-up done: from here on the kernel reads inputs earlier work may write
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Single CTA: waits for a free stage, loads the x tile and the W tile.
    // Pair: each CTA loads its 128 x rows and its half of the W tile into its
    // own stage, counted against rank 0's `full` barrier; rank 0's MMA
    // commits release the stage in both CTAs' `empty` barriers.
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long it = 0;
      for (int u = tile0; u < total_units && !*abort_flag; u += tile_step) {
        const Unit t = unit_at(u);
        const int row0 = (t.r / col_tiles) * kTileRows + (int)rank * BM;
        // this CTA's rows of the unit's W tile (all of them for a single CTA)
        const int brows = t.whole ? kBRowsT<BNT, PAIR> : kBRowsT<BNT, PAIR> / 2;
        const int col0 = (t.r % col_tiles) * BNT + t.coff + (int)rank * brows;
        const CUtensorMap* mapA = t.set == 0 ? &tmA0 : &tmA1;
        const CUtensorMap* mapB = t.whole ? &tmB : &tmBh;
        const uint32_t stage_tx = (uint32_t)((AMN ? BM : args.a_rows) * BK * 2 + brows * BK * 2);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const bool free = rank == 0 ? mbar_wait_hint(&empty[stage], phase ^ 1u, kWaitNs, kSleepNs)
                                      : mbar_wait_cluster_hint(&empty[stage], phase ^ 1u, kWaitNs, kSleepNs);
          if (!free) {
            report_status(args.status, FAKLA_ERR_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          uint8_t* dA = sA + stage * kAStage;
          uint8_t* dB = sB + stage * kBStage;
          if constexpr (PAIR) {
            const uint32_t fb = mapa_shared(&full[stage], 0);
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * SL * stage_tx);
            if constexpr (AMN) {
              for (int a = 0; a < BM / 64; ++a) tma_load_2d_pair(dA + a * kMnAtom, mapA, fb, row0 + 64 * a, kb * BK);
            } else {
#pragma unroll
              for (int sl = 0; sl < SL; ++sl)
                tma_load_2d_pair(dA + sl * kABytes, mapA, fb, (kb * SL + sl) * BK, row0);
            }
            if constexpr (BMN) {
              for (int a = 0; a < brows / 64; ++a) tma_load_2d_pair(dB + a * kMnAtom, mapB, fb, col0 + 64 * a, kb * BK);
            } else {
#pragma unroll
              for (int sl = 0; sl < SL; ++sl)
                tma_load_2d_pair(dB + sl * kBBytes, mapB, fb, (kb * SL + sl) * BK, col0);
            }
          } else {
            mbar_arrive_expect_tx(&full[stage], stage_tx);
            if constexpr (AMN) {
              for (int a = 0; a < BM / 64; ++a) tma_load_2d(dA + a * kMnAtom, mapA, &full[stage], row0 + 64 * a, kb * BK);
            } else {
              tma_load_2d(dA, mapA, &full[stage], kb * BK, row0);
            }
            if constexpr (BMN) {
              for (int a = 0; a < brows / 64; ++a) tma_load_2d(dB + a * kMnAtom, mapB, &full[stage], col0 + 64 * a, kb * BK);
            } else {
              tma_load_2d(dB, mapB, &full[stage], kb * BK, col0);
            }
          }
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (*abort_flag && rank == 0) {
        // Let the copies in flight land before the CTA exits (rank 1's
        // copies count against rank 0's barriers, which it cannot wait on;
        // the cluster barrier at the end holds it until rank 0 is done).
        for (long i = it - kStages; i < it; ++i)
          if (i >= 0) (void)mbar_wait(&full[i % kStages], (uint32_t)(i / kStages) & 1u, kWaitNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc_whole = idesc_bf16_f32(kTileRows, BNT, AMN, BMN);
      constexpr uint32_t idesc_half = idesc_bf16_f32(kTileRows, BNT / 2, AMN, BMN);
      // descriptor steps per 16-element K slice: 32 bytes inside a K-major
      // atom row, 16 K rows (2048 bytes) of an MN-major atom; LBO = the MN
      // atom stride for MN-major operands
      constexpr uint64_t kStepA = AMN ? 2048 >> 4 : 32 >> 4;
      constexpr uint64_t kStepB = BMN ? 2048 >> 4 : 32 >> 4;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int u = tile0; u < total_units && !*abort_flag; u += tile_step) {
        const uint32_t idesc = u < n_full ? idesc_whole : idesc_half;
        const bool drained = PAIR ? mbar_wait_cluster_hint(&tempty[acc], acc_phase ^ 1u, kWaitNs, kSleepNs)
                                  : mbar_wait_hint(&tempty[acc], acc_phase ^ 1u, kWaitNs, kSleepNs);
        if (!drained) {
          report_status(args.status, FAKLA_ERR_TIMEOUT);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BNT);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_hint(&full[stage], phase, kWaitNs, kSleepNs)) {
            report_status(args.status, FAKLA_ERR_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int sl = 0; sl < SL; ++sl) {
            const uint64_t da =
                smem_desc_sw128(smem_u32(sA + stage * kAStage + sl * kABytes), AMN ? kMnAtom : 16, 1024);
            const uint64_t db =
                smem_desc_sw128(smem_u32(sB + stage * kBStage + sl * kBBytes), BMN ? kMnAtom : 16, 1024);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint32_t accum = (kb | sl | k) != 0 ? 1u : 0u;
              if constexpr (PAIR)
                mma_ss_pair(d_tmem, da + kStepA * k, db + kStepB * k, idesc, accum);
              else
                mma_ss(d_tmem, da + kStepA * k, db + kStepB * k, idesc, accum);
            }
          }
          if constexpr (PAIR)
            mma_commit_pair(&empty[stage]);
          else
            mma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if constexpr (PAIR)
          mma_commit_pair(&tfull[acc]);
        else
          mma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (*abort_flag) {
        // Let the MMAs already issued finish before TMEM is freed (and, for a
        // pair, before the other CTA's shared memory goes away).
        if constexpr (PAIR)
          mma_commit_pair(drain);
        else
          mma_commit(drain);
        (void)mbar_wait(drain, 0u, kWaitNs);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;          // TMEM lane quadrant this warp may access
    const int ew = warp - 2;         // epilogue warp index (staging buffer owner)
    const int half = ew >> 2;        // which half of the tile's BNT columns
    constexpr int kWarpCols = BNT / 2;  // 128 or 64 columns per warp
    uint8_t* buf = sOut + ew * kOutWarpBytes;
    const int m = args.m;  // features per head
    int acc = 0;
    uint32_t acc_phase = 0;
    bool stored = false;
    for (int u = tile0; u < total_units; u += tile_step) {
      // One epilogue warp polls the accumulator barrier (and the abort flag);
      // the other seven sleep in a named barrier, which takes no issue slots.
      // Eight polling warps spent most of the kernel's instructions, and under
      // the power cap that cost clock. The barrier also hands every warp the
      // same stop decision, so none leaves the loop while others wait in it.
      bool stop = false;
      if (ew == 0) {
        stop = *abort_flag != 0;
        if (!stop) {
          // Pair: rank 0's commit lands on both CTAs' `tfull`.
          const bool ready = rank == 0 ? mbar_wait_hint(&tfull[acc], acc_phase, kWaitNs, kSleepNs)
                                       : mbar_wait_cluster_hint(&tfull[acc], acc_phase, kWaitNs, kSleepNs);
          if (!ready) {
            if (lane == 0) report_status(args.status, FAKLA_ERR_TIMEOUT);
            *abort_flag = 1;
            stop = true;
          }
        }
      }
      if (named_barrier_or(kEpiBarrier, 32 * kEpiWarps, stop)) break;
      const Unit t = unit_at(u);
      // columns of this warp: half of the unit's (BNT or BNT / 2)
      const int wcols = t.whole ? kWarpCols : kWarpCols / 2;
      const int row0 = (t.r / col_tiles) * kTileRows + (int)rank * BM;  // this CTA's 128 rows
      const int col0 = (t.r % col_tiles) * BNT + t.coff + half * wcols;
      const CUtensorMap* mapC = t.set == 0 ? &tmC0 : &tmC1;
      const __nv_bfloat16* temp = t.set == 0 ? args.temp0 : args.temp1;
      const int grow = row0 + 32 * q + lane;  // this thread's output row
      tc_fence_after();
      const uint32_t t_row =
          tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * BNT + half * wcols);
      const int nj = wcols / 64;
#pragma unroll 1
      for (int j = 0; j < nj; ++j) {
        uint32_t v0[32], v1[32];
        tmem_ld32(t_row + (uint32_t)(j * 64), v0);
        tmem_ld32(t_row + (uint32_t)(j * 64 + 32), v1);
        tmem_ld_wait();
        if (j == nj - 1) {
          // this warp's share of the accumulator is in registers: release it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (rank == 0)
              mbar_arrive(&tempty[acc]);
            else
              mbar_arrive_cluster(mapa_shared(&tempty[acc], 0));
          }
        }
        const int c0 = col0 + j * 64;
        const bool ident = c0 >= args.ident_from;  // identity columns (the v block of a q/k/v GEMM)
        // temperature on this chunk's columns (warp-uniform; rows past the end
        // keep 1)
        const bool scaled = temp != nullptr && c0 >= args.tcol0 && c0 < args.tcol1;
        float tscale = 1.f;
        if (scaled && grow < args.rows)
          tscale = __bfloat162float(temp[(int64_t)grow * args.heads + (c0 - args.tcol0) / m]);
        uint32_t bw[32];  // bias of the 64 columns as bf16 pairs (same for all lanes)
        if (args.bias != nullptr) {
          const uint4* bp = reinterpret_cast<const uint4*>(args.bias + c0);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 u = __ldg(bp + i);
            bw[4 * i] = u.x;
            bw[4 * i + 1] = u.y;
            bw[4 * i + 2] = u.z;
            bw[4 * i + 3] = u.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) bw[i] = 0u;
        }
        // Two passes for FAKLA_ACT_COSSIN (cos to column c0, sin to column
        // N + c0), one for every other activation.
        constexpr int kPasses = ACT == FAKLA_ACT_COSSIN ? 2 : 1;
#pragma unroll 1
        for (int pass = 0; pass < kPasses; ++pass) {
          uint32_t packed[32];
          const uint64_t tscale2 = f2_splat(tscale);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const uint32_t raw_a = i < 16 ? v0[2 * i] : v1[2 * i - 32];
            const uint32_t raw_b = i < 16 ? v0[2 * i + 1] : v1[2 * i + 1 - 32];
            // columns 2i, 2i+1 as an fp32 pair (paired FP32 pipe; each lane
            // rounds as the scalar operation would)
            const uint64_t x = f2_add(f2_make(raw_a, raw_b), f2_from_bf16x2(bw[i]));
            const float2 ab = f2_split(x);
            const float a = ab.x, b = ab.y;
            if constexpr (ACT == FAKLA_ACT_COSSIN) {
              const float ra = reduce_2pi(a), rb = reduce_2pi(b);
              const float fa = pass == 0 ? __cosf(ra) : __sinf(ra);
              const float fb = pass == 0 ? __cosf(rb) : __sinf(rb);
              packed[i] = pack_bf16x2(fa * args.scale * tscale, fb * args.scale * tscale);
            } else if (ident) {
              packed[i] = pack_bf16x2(x);
            } else {
              uint64_t y;
              if constexpr (ACT == FAKLA_ACT_ELU1) {
                // elu(x) + 1 = x + 1 for x > 0, e^x = 2^(x log2 e) otherwise: the
                // pair's x + 1 and x log2 e one paired op each, the two powers of
                // two on the MUFU (ex2.approx; the result is rounded to bf16), and
                // the choice by the sign bit in one bitwise select each (x = -0
                // takes 2^-0 = 1 = 0 + 1). The epilogue shares issue slots with the
                // producer and MMA threads, so its instruction count shows in the
                // tensor pipe's activity.
                const float2 p1 = f2_split(f2_add(x, f2_splat(1.f)));
                const float2 t = f2_split(f2_mul(x, f2_splat(1.4426950408889634f)));
                const uint32_t ma = (uint32_t)((int32_t)__float_as_uint(a) >> 31);
                const uint32_t mb = (uint32_t)((int32_t)__float_as_uint(b) >> 31);
                y = f2_make((ex2_approx(t.x) & ma) | (__float_as_uint(p1.x) & ~ma),
                            (ex2_approx(t.y) & mb) | (__float_as_uint(p1.y) & ~mb));
              } else {
                y = f2_make(__float_as_uint(activate<ACT, true>(a)), __float_as_uint(activate<ACT, true>(b)));
              }
              packed[i] = pack_bf16x2(scaled ? f2_mul(y, tscale2) : y);
            }
          }
          // single staging buffer per warp: the previous store must have read it
          if (lane == 0 && stored) bulk_wait_group_read<0>();
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint4 val = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2],
                                   packed[4 * c + 3]);
            *reinterpret_cast<uint4*>(buf + sw128_offset((uint32_t)lane, (uint32_t)(c * 8))) = val;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && row0 + 32 * q < args.rows) {
            tma_store_2d(mapC, buf, c0 + pass * args.N, row0 + 32 * q);
            bulk_commit_group();
          }
          stored = true;
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  // a pair's CTAs exit together: rank 0's MMAs read rank 1's shared memory and
  // write its TMEM, and rank 1 arrives on rank 0's barriers
  if constexpr (PAIR) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, kTmemCols);
    else
      tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static bool make_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                        uint32_t box_inner, uint32_t box_outer) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return encode_tensor_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base),
                           dims, strides, box, estr, CU_TENSOR_MAP_SWIZZLE_128B);
}

bool phi_sm100_supported(int64_t rows, int64_t K, int64_t N, int64_t heads) {
  if (rows < 1 || K < BK || N < 128) return false;
  if (K % BK != 0 || N % 128 != 0) return false;
  if (heads < 1 || N % heads != 0 || (N / heads) % 64 != 0) return false;
  if (rows > (int64_t)INT32_MAX || K > (int64_t)INT32_MAX / 2 || N > (int64_t)INT32_MAX / 2)
    return false;
  return true;
}

// Tile shapes: 0 = single CTA, 128 x 256; 1 = single CTA, 128 x 128;
// 2 = CTA pair, 256 x 256.
enum PhiTiling { kTile256 = 0, kTile128 = 1, kTilePair = 2 };

// Pairs of CTAs that can be resident at once (a pair needs two SMs of one
// GPC), per device; 0 if the query failed.
static int pair_slots() {
  static std::atomic<int> cached[64];  // 0: not queried yet; else count + 1
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  int known = cached[dev].load(std::memory_order_relaxed);
  if (known == 0) {
    int n = 0;
    const auto kern = phi_gemm_sm100_kernel<FAKLA_ACT_ELU1, BN, true>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemBytesT<BN, true, kSlabsT<BN, true, false, false>>) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(2 * fakla_sm_count());
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = kSmemBytesT<BN, true, kSlabsT<BN, true, false, false>>;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    (void)cudaGetLastError();
    known = n + 1;  // the same value from any thread that gets here first
    cached[dev].store(known, std::memory_order_relaxed);
  }
  return known - 1;
}

// CTA pairs when N allows 256-wide tiles and there are enough 256 x 256
// tiles to occupy every pair; otherwise single CTAs with 256-wide tiles, or
// 128-wide ones when N is an odd multiple of 128 or when 256-wide tiles would
// leave SMs idle (few rows, e.g. a decode step).
static int pick_tiling(int64_t rows, int64_t N, int nsets) {
  if (N % BN == 0) {
    const int slots = pair_slots();
    if (slots > 0 && ((rows + 2 * BM - 1) / (2 * BM)) * (N / BN) * nsets >= slots) return kTilePair;
  }
  const int64_t row_tiles = (rows + BM - 1) / BM;
  if (N % BN != 0 || row_tiles * (N / BN) * nsets < fakla_sm_count()) return kTile128;
  return kTile256;
}

static int tiling_bn(int tiling) { return tiling == kTile128 ? 128 : BN; }
// rows of W per CTA per stage (the TMA box height of the W map)
static int tiling_b_rows(int tiling) { return tiling == kTilePair ? BN / 2 : tiling_bn(tiling); }
// rows of x per A box: a single-CTA launch whose row sets have fewer than BM
// rows loads only those (rounded up to 8), not a whole BM-row box
static int a_box_rows(int64_t rows, int tiling) {
  return (tiling != kTilePair && rows < BM) ? (int)((rows + 7) / 8 * 8) : BM;
}

// Tensor maps of one launch: x rows of both row sets, W (box of a CTA's rows
// of a whole tile, and of half a tile for the split tail), outputs.
struct PhiMaps {
  CUtensorMap A0, A1, B, Bh, C0, C1;
};

// Tiles that run whole: all but a last wave that would leave more than half
// the pairs idle, which runs as twice as many half tiles instead.
static int64_t whole_tiles(int64_t tiles, int tiling) {
  if (tiling != kTilePair) return tiles;
  const int64_t slots = pair_slots();
  const int64_t pairs = tiles < slots ? tiles : slots;
  if (pairs < 1) return tiles;
  const int64_t rem = tiles % pairs;
  return (rem == 0 || 2 * rem > pairs) ? tiles : tiles - rem;
}

template <int ACT, int BNT, bool PAIR, bool AMN = false, bool BMN = false>
static cudaError_t launch_act_t(const PhiMaps& m, const PhiArgs& a, int64_t units, cudaStream_t stream) {
  const auto kern = phi_gemm_sm100_kernel<ACT, BNT, PAIR, AMN, BMN>;
  constexpr size_t smem = kSmemBytesT<BNT, PAIR, kSlabsT<BNT, PAIR, AMN, BMN>>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if constexpr (PAIR) {
    const int64_t pairs = units < pair_slots() ? units : pair_slots();
    return launch_chained(kern, dim3((unsigned)(2 * pairs)), dim3(kThreads), smem, stream,
                          2u, m.A0, m.A1, m.B, m.Bh, m.C0, m.C1, a);
  } else {
    const int sms = fakla_sm_count();
    const int grid = units < sms ? (int)units : sms;
    return launch_chained(kern, dim3((unsigned)grid), dim3(kThreads), smem, stream, 1u,
                          m.A0, m.A1, m.B, m.Bh, m.C0, m.C1, a);
  }
}

static int64_t tile_count(int64_t rows, int64_t N, int nsets, int tiling) {
  const int64_t tile_rows = tiling == kTilePair ? 2 * BM : BM;
  return ((rows + tile_rows - 1) / tile_rows) * (N / tiling_bn(tiling)) * nsets;
}

// Fills a.n_full for the chosen tiling and launches.
template <int ACT, bool AMN = false, bool BMN = false>
static cudaError_t launch_act(const PhiMaps& m, PhiArgs a, int64_t rows, int64_t N, int tiling,
                              cudaStream_t stream) {
  const int64_t tiles = tile_count(rows, N, a.nsets, tiling);
  const int64_t whole = whole_tiles(tiles, tiling);
  a.n_full = (int)whole;
  const int64_t units = whole + 2 * (tiles - whole);
  switch (tiling) {
    case kTilePair: return launch_act_t<ACT, BN, true, AMN, BMN>(m, a, units, stream);
    case kTile128: return launch_act_t<ACT, 128, false, AMN, BMN>(m, a, units, stream);
    default: return launch_act_t<ACT, BN, false, AMN, BMN>(m, a, units, stream);
  }
}

// W maps: a CTA's rows of a whole tile and of a half tile (the half-tile map
// is only read by the split tail of CTA-pair launches).
static bool make_w_maps(PhiMaps* m, const void* W, int64_t K, int64_t N, int tiling) {
  const uint32_t brows = (uint32_t)tiling_b_rows(tiling);
  return make_map_2d(&m->B, W, (uint64_t)K, (uint64_t)N, BK, brows) &&
         make_map_2d(&m->Bh, W, (uint64_t)K, (uint64_t)N, BK, tiling == kTilePair ? brows / 2 : brows);
}

cudaError_t launch_phi_sm100(const void* x0, const void* x1, const void* W, const void* bias,
                             const void* temp0, const void* temp1, void* out0, void* out1,
                             int64_t rows, int64_t K, int64_t N, int64_t heads, int act,
                             float scale, cudaStream_t stream, int* status, bool* encoded) {
  PhiMaps m;
  const int nsets = x1 != nullptr ? 2 : 1;
  const int tiling = pick_tiling(rows, N, nsets);
  const uint64_t out_cols = (uint64_t)N * (act == FAKLA_ACT_COSSIN ? 2 : 1);
  const int a_rows = a_box_rows(rows, tiling);
  bool ok = make_map_2d(&m.A0, x0, (uint64_t)K, (uint64_t)rows, BK, (uint32_t)a_rows) &&
            make_w_maps(&m, W, K, N, tiling) && make_map_2d(&m.C0, out0, out_cols, (uint64_t)rows, 64, 32);
  if (ok && nsets == 2)
    ok = make_map_2d(&m.A1, x1, (uint64_t)K, (uint64_t)rows, BK, (uint32_t)a_rows) &&
         make_map_2d(&m.C1, out1, out_cols, (uint64_t)rows, 64, 32);
  else {
    m.A1 = m.A0;
    m.C1 = m.C0;
  }
  *encoded = ok;
  if (!ok) return cudaErrorInvalidValue;
  PhiArgs a;
  a.bias = (const __nv_bfloat16*)bias;
  a.scale = scale;
  a.temp0 = (const __nv_bfloat16*)temp0;
  a.temp1 = (const __nv_bfloat16*)temp1;
  a.rows = (int)rows;
  a.N = (int)N;
  a.K = (int)K;
  a.heads = (int)heads;
  a.nsets = nsets;
  a.m = (int)(N / heads);
  a.ident_from = (int)N;
  a.tcol0 = 0;
  a.tcol1 = (int)N;
  a.a_rows = a_rows;
  a.status = status;
  switch (act) {
    case FAKLA_ACT_ELU1: return launch_act<FAKLA_ACT_ELU1>(m, a, rows, N, tiling, stream);
    case FAKLA_ACT_RELU: return launch_act<FAKLA_ACT_RELU>(m, a, rows, N, tiling, stream);
    case FAKLA_ACT_SOFTPLUS: return launch_act<FAKLA_ACT_SOFTPLUS>(m, a, rows, N, tiling, stream);
    case FAKLA_ACT_GELU: return launch_act<FAKLA_ACT_GELU>(m, a, rows, N, tiling, stream);
    case FAKLA_ACT_IDENTITY: return launch_act<FAKLA_ACT_IDENTITY>(m, a, rows, N, tiling, stream);
    case FAKLA_ACT_SIGMOID: return launch_act<FAKLA_ACT_SIGMOID>(m, a, rows, N, tiling, stream);
    case FAKLA_ACT_ABS: return launch_act<FAKLA_ACT_ABS>(m, a, rows, N, tiling, stream);
    case FAKLA_ACT_COSSIN: return launch_act<FAKLA_ACT_COSSIN>(m, a, rows, N, tiling, stream);
    default: return cudaErrorInvalidValue;
  }
}

bool gemm_sm100_supported(int64_t M, int64_t N, int64_t K, bool a_mn, bool b_mn) {
  if (M < 1 || N < 128 || K < 1 || N % 128 != 0) return false;
  if (M > (int64_t)INT32_MAX / 2 || N > (int64_t)INT32_MAX / 2 || K > (int64_t)INT32_MAX / 2) return false;
  // row strides of the operands (16-byte multiples for TMA): K-major rows hold
  // K elements, MN-major rows M or N
  if (!a_mn && K % 8 != 0) return false;
  if (a_mn && M % 8 != 0) return false;
  // B's rows hold K (K-major) or N (MN-major) elements; N % 128 == 0 covers the
  // latter. The innermost extent of every operand spans at least one 64-wide
  // box (the boxes may run past the outer extents, which read as zeros).
  if ((!a_mn || !b_mn) && K < 64) return false;
  if (a_mn && M < 64) return false;
  return true;
}

cudaError_t launch_gemm_sm100(const void* A, bool a_mn, const void* B, bool b_mn, void* D, int64_t M,
                              int64_t N, int64_t K, cudaStream_t stream, int* status, bool* encoded) {
  if (!b_mn && K % 8 != 0) {
    *encoded = false;
    return cudaErrorInvalidValue;
  }
  PhiMaps m;
  const int tiling = pick_tiling(M, N, 1);
  const uint32_t brows = (uint32_t)tiling_b_rows(tiling);
  const int a_rows = a_mn ? BM : a_box_rows(M, tiling);
  bool ok = a_mn ? make_map_2d(&m.A0, A, (uint64_t)M, (uint64_t)K, 64, BK)
                 : make_map_2d(&m.A0, A, (uint64_t)K, (uint64_t)M, BK, (uint32_t)a_rows);
  if (b_mn)
    ok = ok && make_map_2d(&m.B, B, (uint64_t)N, (uint64_t)K, 64, BK) &&
         make_map_2d(&m.Bh, B, (uint64_t)N, (uint64_t)K, 64, BK);
  else
    ok = ok && make_map_2d(&m.B, B, (uint64_t)K, (uint64_t)N, BK, brows) &&
         make_map_2d(&m.Bh, B, (uint64_t)K, (uint64_t)N, BK, tiling == kTilePair ? brows / 2 : brows);
  ok = ok && make_map_2d(&m.C0, D, (uint64_t)N, (uint64_t)M, 64, 32);
  *encoded = ok;
  if (!ok) return cudaErrorInvalidValue;
  m.A1 = m.A0;
  m.C1 = m.C0;
  PhiArgs a;
  a.bias = nullptr;
  a.scale = 1.f;
  a.temp0 = nullptr;
  a.temp1 = nullptr;
  a.rows = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.heads = 1;
  a.nsets = 1;
  a.m = (int)N;
  a.ident_from = 0;
  a.tcol0 = 0;
  a.tcol1 = 0;
  a.a_rows = a_rows;
  a.status = status;
  if (a_mn && b_mn) return launch_act<FAKLA_ACT_IDENTITY, true, true>(m, a, M, N, tiling, stream);
  if (a_mn) return launch_act<FAKLA_ACT_IDENTITY, true, false>(m, a, M, N, tiling, stream);
  if (b_mn) return launch_act<FAKLA_ACT_IDENTITY, false, true>(m, a, M, N, tiling, stream);
  return launch_act<FAKLA_ACT_IDENTITY, false, false>(m, a, M, N, tiling, stream);
}

bool qkv_sm100_supported(int64_t rows, int64_t K, int64_t feat, int64_t vdim, int64_t heads) {
  const int64_t N = 2 * feat + vdim;
  return rows >= 1 && K >= BK && K % BK == 0 && N % 128 == 0 && feat % 64 == 0 && heads >= 1 &&
         feat % heads == 0 && (feat / heads) % 64 == 0 && rows <= (int64_t)INT32_MAX &&
         K <= (int64_t)INT32_MAX / 2 && N <= (int64_t)INT32_MAX / 2;
}

cudaError_t launch_qkv_sm100(const void* x, const void* W, const void* bias, const void* temp,
                             void* out, int64_t rows, int64_t K, int64_t feat, int64_t vdim,
                             int64_t heads, cudaStream_t stream, int* status, bool* encoded) {
  const int64_t N = 2 * feat + vdim;
  const int tiling = pick_tiling(rows, N, 1);
  PhiMaps m;
  const int a_rows = a_box_rows(rows, tiling);
  const bool ok = make_map_2d(&m.A0, x, (uint64_t)K, (uint64_t)rows, BK, (uint32_t)a_rows) &&
                  make_w_maps(&m, W, K, N, tiling) && make_map_2d(&m.C0, out, (uint64_t)N, (uint64_t)rows, 64, 32);
  m.A1 = m.A0;
  m.C1 = m.C0;
  *encoded = ok;
  if (!ok) return cudaErrorInvalidValue;
  PhiArgs a;
  a.bias = (const __nv_bfloat16*)bias;
  a.scale = 1.f;
  a.temp0 = (const __nv_bfloat16*)temp;
  a.temp1 = nullptr;
  a.rows = (int)rows;
  a.N = (int)N;
  a.K = (int)K;
  a.heads = (int)heads;
  a.nsets = 1;
  a.m = (int)(feat / heads);
  a.ident_from = (int)(2 * feat);  // [phi(q) | phi(k) * temp | v]
  a.tcol0 = (int)feat;
  a.tcol1 = (int)(2 * feat);
  a.a_rows = a_rows;
  a.status = status;
  return launch_act<FAKLA_ACT_ELU1>(m, a, rows, N, tiling, stream);
}

}  // namespace fakla
