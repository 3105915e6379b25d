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
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fakla_common.cuh"
#include "fakla_kernels.h"
#include "sm100_umma.cuh"

namespace fakla {
namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr int BN = 256;  // N tile; 128 (BNT below) when 256-wide tiles would not fill the GPU
constexpr int BK = 64;
constexpr int kStages = 4;
constexpr int kABytes = BM * BK * 2;                 // 16 KB
template <int BNT> constexpr int kBBytesT = BNT * BK * 2;             // 32 KB (BNT = 256)
template <int BNT> constexpr int kStageBytesT = kABytes + kBBytesT<BNT>;  // 48 KB
constexpr int kEpiWarps = 8;
constexpr int kOutWarpBytes = 32 * 128;              // 32 rows x 64 bf16
constexpr int kOutBytes = kEpiWarps * kOutWarpBytes;  // 32 KB (one buffer per warp)
constexpr int kThreads = 64 + 32 * kEpiWarps;        // 320
template <int BNT> constexpr uint32_t kTmemColsT = 2 * BNT;  // 512 (BNT = 256)
constexpr uint64_t kWaitNs = 2000000000ull;          // 2 s per wait

template <int BNT>
constexpr size_t kSmemBytesT = 1024 /*align slack*/ + (size_t)kStages * kStageBytesT<BNT> + kOutBytes + 256;

struct PhiArgs {
  const __nv_bfloat16* bias;   // [N] or null
  float scale;                 // FAKLA_ACT_COSSIN output scale
  const __nv_bfloat16* temp0;  // [rows, heads] or null (row set 0)
  const __nv_bfloat16* temp1;  // [rows, heads] or null (row set 1)
  int rows, N, K, heads, nsets;
  int m;                       // features per head (temperature index = (col - tcol0) / m)
  int ident_from;              // columns >= ident_from skip the activation (N: none)
  int tcol0, tcol1;            // temperature applies to columns [tcol0, tcol1)
  int* status;
};

template <int ACT, int BNT>
__global__ void __launch_bounds__(kThreads, 1) phi_gemm_sm100_kernel(
    const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
    const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmC0,
    const __grid_constant__ CUtensorMap tmC1, const PhiArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;                                  // kStages x 16 KB
  uint8_t* sB = smem + kStages * kABytes;              // kStages x 32 KB
  constexpr int kBBytes = kBBytesT<BNT>;
  constexpr int kStageBytes = kStageBytesT<BNT>;
  constexpr uint32_t kTmemCols = kTmemColsT<BNT>;
  uint8_t* sOut = sB + kStages * kBBytes;              // 32 KB (1024-aligned)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + kOutBytes);
  uint64_t* full = bars;                  // [kStages]
  uint64_t* empty = bars + kStages;       // [kStages]
  uint64_t* tfull = bars + 2 * kStages;   // [2]
  uint64_t* tempty = tfull + 2;           // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int row_tiles = (args.rows + BM - 1) / BM;
  const int col_tiles = args.N / BNT;
  const int tiles_per_set = row_tiles * col_tiles;
  const int total_tiles = tiles_per_set * args.nsets;
  const int kblocks = args.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA0);
    tma_prefetch_desc(&tmA1);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC0);
    tma_prefetch_desc(&tmC1);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long it = 0;
      for (int tile = blockIdx.x; tile < total_tiles && !*abort_flag; tile += gridDim.x) {
        const int set = tile / tiles_per_set;
        const int r = tile % tiles_per_set;
        const int row0 = (r / col_tiles) * BM;
        const int col0 = (r % col_tiles) * BNT;
        const CUtensorMap* mapA = set == 0 ? &tmA0 : &tmA1;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, kWaitNs)) {
            report_status(args.status, FAKLA_ERR_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          tma_load_2d(sA + stage * kABytes, mapA, &full[stage], kb * BK, row0);
          tma_load_2d(sB + stage * kBBytes, &tmB, &full[stage], kb * BK, col0);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (*abort_flag) {
        // Let this CTA's copies in flight land before it exits.
        for (long i = it - kStages; i < it; ++i)
          if (i >= 0) (void)mbar_wait(&full[i % kStages], (uint32_t)(i / kStages) & 1u, kWaitNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BNT, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = blockIdx.x; tile < total_tiles && !*abort_flag; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, kWaitNs)) {
          report_status(args.status, FAKLA_ERR_TIMEOUT);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BNT);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, kWaitNs)) {
            report_status(args.status, FAKLA_ERR_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_sw128(smem_u32(sA + stage * kABytes), 16, 1024);
          const uint64_t db = smem_desc_sw128(smem_u32(sB + stage * kBBytes), 16, 1024);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // advance 16 bf16 = 32 bytes along K inside the 128-byte swizzle atom
            mma_ss(d_tmem, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc,
                   (kb | k) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        mma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
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
    for (int tile = blockIdx.x; tile < total_tiles && !*abort_flag; tile += gridDim.x) {
      const int set = tile / tiles_per_set;
      const int r = tile % tiles_per_set;
      const int row0 = (r / col_tiles) * BM;
      const int col0 = (r % col_tiles) * BNT + half * kWarpCols;
      const CUtensorMap* mapC = set == 0 ? &tmC0 : &tmC1;
      const __nv_bfloat16* temp = set == 0 ? args.temp0 : args.temp1;
      const int grow = row0 + 32 * q + lane;  // this thread's output row
      if (!mbar_wait(&tfull[acc], acc_phase, kWaitNs)) {
        report_status(args.status, FAKLA_ERR_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t t_row =
          tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * BNT + half * kWarpCols);
#pragma unroll 1
      for (int j = 0; j < kWarpCols / 64; ++j) {
        uint32_t v0[32], v1[32];
        tmem_ld32(t_row + (uint32_t)(j * 64), v0);
        tmem_ld32(t_row + (uint32_t)(j * 64 + 32), v1);
        tmem_ld_wait();
        if (j == kWarpCols / 64 - 1) {
          // this warp's share of the accumulator is in registers: release it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
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
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const uint32_t raw_a = i < 16 ? v0[2 * i] : v1[2 * i - 32];
            const uint32_t raw_b = i < 16 ? v0[2 * i + 1] : v1[2 * i + 1 - 32];
            const float a = __uint_as_float(raw_a) + __uint_as_float(bw[i] << 16);
            const float b = __uint_as_float(raw_b) + __uint_as_float(bw[i] & 0xffff0000u);
            if constexpr (ACT == FAKLA_ACT_COSSIN) {
              const float fa = pass == 0 ? cosf(a) : sinf(a);
              const float fb = pass == 0 ? cosf(b) : sinf(b);
              packed[i] = pack_bf16x2(fa * args.scale * tscale, fb * args.scale * tscale);
            } else if (ident) {
              packed[i] = pack_bf16x2(a, b);
            } else if (scaled) {
              packed[i] = pack_bf16x2(activate<ACT, true>(a) * tscale, activate<ACT, true>(b) * tscale);
            } else {
              packed[i] = pack_bf16x2(activate<ACT, true>(a), activate<ACT, true>(b));
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
          if (lane == 0) {
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
  if (warp == 1) {
    tc_fence_after();
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

template <int ACT, int BNT>
static cudaError_t launch_act_t(const CUtensorMap& mA0, const CUtensorMap& mA1, const CUtensorMap& mB,
                                const CUtensorMap& mC0, const CUtensorMap& mC1, const PhiArgs& a,
                                int grid, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(phi_gemm_sm100_kernel<ACT, BNT>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBytesT<BNT>);
  if (e != cudaSuccess) return e;
  phi_gemm_sm100_kernel<ACT, BNT><<<grid, kThreads, kSmemBytesT<BNT>, stream>>>(mA0, mA1, mB, mC0, mC1, a);
  return cudaGetLastError();
}

template <int ACT>
static cudaError_t launch_act(const CUtensorMap& mA0, const CUtensorMap& mA1, const CUtensorMap& mB,
                              const CUtensorMap& mC0, const CUtensorMap& mC1, const PhiArgs& a,
                              int grid, int bn, cudaStream_t stream) {
  return bn == 128 ? launch_act_t<ACT, 128>(mA0, mA1, mB, mC0, mC1, a, grid, stream)
                   : launch_act_t<ACT, BN>(mA0, mA1, mB, mC0, mC1, a, grid, stream);
}

// The N tile: 256, or 128 when N is an odd multiple of 128 or when 256-wide
// tiles would leave SMs idle (few rows, e.g. a decode step).
static int pick_bn(int64_t rows, int64_t N, int nsets) {
  const int64_t row_tiles = (rows + BM - 1) / BM;
  if (N % BN != 0 || row_tiles * (N / BN) * nsets < fakla_sm_count()) return 128;
  return BN;
}

cudaError_t launch_phi_sm100(const void* x0, const void* x1, const void* W, const void* bias,
                             const void* temp0, const void* temp1, void* out0, void* out1,
                             int64_t rows, int64_t K, int64_t N, int64_t heads, int act,
                             float scale, cudaStream_t stream, int* status, bool* encoded) {
  CUtensorMap mA0, mA1, mB, mC0, mC1;
  const int nsets = x1 != nullptr ? 2 : 1;
  const int bn = pick_bn(rows, N, nsets);
  const uint64_t out_cols = (uint64_t)N * (act == FAKLA_ACT_COSSIN ? 2 : 1);
  bool ok = make_map_2d(&mA0, x0, (uint64_t)K, (uint64_t)rows, BK, BM) &&
            make_map_2d(&mB, W, (uint64_t)K, (uint64_t)N, BK, (uint32_t)bn) &&
            make_map_2d(&mC0, out0, out_cols, (uint64_t)rows, 64, 32);
  if (ok && nsets == 2)
    ok = make_map_2d(&mA1, x1, (uint64_t)K, (uint64_t)rows, BK, BM) &&
         make_map_2d(&mC1, out1, out_cols, (uint64_t)rows, 64, 32);
  else {
    mA1 = mA0;
    mC1 = mC0;
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
  a.status = status;
  const int row_tiles = (int)((rows + BM - 1) / BM);
  const int total = row_tiles * (int)(N / bn) * nsets;
  const int grid = total < fakla_sm_count() ? total : fakla_sm_count();
  switch (act) {
    case FAKLA_ACT_ELU1: return launch_act<FAKLA_ACT_ELU1>(mA0, mA1, mB, mC0, mC1, a, grid, bn, stream);
    case FAKLA_ACT_RELU: return launch_act<FAKLA_ACT_RELU>(mA0, mA1, mB, mC0, mC1, a, grid, bn, stream);
    case FAKLA_ACT_SOFTPLUS: return launch_act<FAKLA_ACT_SOFTPLUS>(mA0, mA1, mB, mC0, mC1, a, grid, bn, stream);
    case FAKLA_ACT_GELU: return launch_act<FAKLA_ACT_GELU>(mA0, mA1, mB, mC0, mC1, a, grid, bn, stream);
    case FAKLA_ACT_IDENTITY: return launch_act<FAKLA_ACT_IDENTITY>(mA0, mA1, mB, mC0, mC1, a, grid, bn, stream);
    case FAKLA_ACT_SIGMOID: return launch_act<FAKLA_ACT_SIGMOID>(mA0, mA1, mB, mC0, mC1, a, grid, bn, stream);
    case FAKLA_ACT_ABS: return launch_act<FAKLA_ACT_ABS>(mA0, mA1, mB, mC0, mC1, a, grid, bn, stream);
    case FAKLA_ACT_COSSIN: return launch_act<FAKLA_ACT_COSSIN>(mA0, mA1, mB, mC0, mC1, a, grid, bn, stream);
    default: return cudaErrorInvalidValue;
  }
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
  const int bn = pick_bn(rows, N, 1);
  CUtensorMap mA, mB, mC;
  const bool ok = make_map_2d(&mA, x, (uint64_t)K, (uint64_t)rows, BK, BM) &&
                  make_map_2d(&mB, W, (uint64_t)K, (uint64_t)N, BK, (uint32_t)bn) &&
                  make_map_2d(&mC, out, (uint64_t)N, (uint64_t)rows, 64, 32);
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
  a.status = status;
  const int row_tiles = (int)((rows + BM - 1) / BM);
  const int total = row_tiles * (int)(N / bn);
  const int grid = total < fakla_sm_count() ? total : fakla_sm_count();
  return launch_act<FAKLA_ACT_ELU1>(mA, mA, mB, mC, mC, a, grid, bn, stream);
}

}  // namespace fakla
