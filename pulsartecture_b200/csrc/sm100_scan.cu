// Chunked causal FA-KLA scan on the sm_100a tensor cores (Df = Dv = 128, bf16
// activations, fp32 state). One CTA per (b, h) sequence walks its T tokens in
// chunks of C = 128. For chunk c with rows Q = phi(q), K = phi(k)*temp, V:
//
//   P   = Q K^T                     (128x128, fp32 in TMEM)        [MMA1]
//   Pm  = causal_mask_inclusive(P)  (s <= t), split hi+lo bf16 into TMEM
//   O   = Q S_{<c}                  (S_{<c} as bf16 in smem)       [MMA2]
//   O  += Pm_hi V + Pm_lo V         (A operand straight from TMEM)  [MMA3]
//   S  += K^T V                     (fp32 accumulator kept in TMEM) [MMA4]
//   den = rowsum(Pm) + Q . z_{<c};  z += colsum(K)   (fp32, CUDA cores)
//   out = O / (den + 1e-12)
//
// This is the chunk-parallel form of the reference recurrence
// (ultra_rwka/backend/cpp/cpu/cpu_kernels.cpp:107-164): out_t sums k~_s v_s
// over s <= t, exactly as the per-token loop does, with the state carried
// across chunks.
//
// Warp roles (192 threads): warp 0 TMA producer (Q, K, V tiles, 2 stages);
// warp 1 TMEM allocator + MMA issuer; warps 2..5 (128 threads, thread r owns
// TMEM lane r: token r for P/O, feature r for S) mask/split P, refresh the
// bf16 copy of S, update z, normalise and store the output.
// Every wait is bounded; on expiry the kernel records FAKLA_ERR_TIMEOUT in the
// device status word and winds down.
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

constexpr int C = 128;                       // tokens per chunk
constexpr int D = 128;                       // Df = Dv
constexpr int kAtom = C * 128;               // 16 KB: 128 rows x 64 bf16
constexpr int kTile = 2 * kAtom;             // 32 KB: 128 rows x 128 bf16
constexpr int kStages = 2;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColP = 0, kColO = 128, kColS = 256, kColPh = 384, kColPl = 448;
constexpr uint64_t kWaitNs = 2000000000ull;

// smem: Q[2] K[2] V[2] Sb | z[128] f32 | barriers
constexpr size_t kOffQ = 0;
constexpr size_t kOffK = kOffQ + kStages * kTile;
constexpr size_t kOffV = kOffK + kStages * kTile;
constexpr size_t kOffSb = kOffV + kStages * kTile;
constexpr size_t kOffZ = kOffSb + kTile;
constexpr size_t kOffBar = kOffZ + D * sizeof(float);
constexpr size_t kSmemBytes = 1024 + kOffBar + 128;

enum Bar {
  kFull0 = 0,
  kEmpty0 = kFull0 + kStages,
  kBarP = kEmpty0 + kStages,
  kBarS,
  kBarO,
  kE1Done,
  kSReady,
  kOFree,
  kKReady,
  kNumBars
};
static_assert(kNumBars * 8 + 8 <= 128, "barrier area");

struct ScanArgs {
  const __nv_bfloat16* temp;  // (B,T,H) or null
  __nv_bfloat16* out;         // (B,T,H,D)
  float* S;                   // (B,H,D,D) or null
  float* z;                   // (B,H,D) or null
  int T, H;
  unsigned flags;
  int* status;
};

__device__ __forceinline__ uint64_t kdesc(uint32_t tile_addr, int j) {
  // K-major operand, K step j (16 elements): atom j/4, +32 B per step inside.
  return smem_desc_sw128(tile_addr + (uint32_t)((j >> 2) * kAtom + (j & 3) * 32), 16, 1024);
}
__device__ __forceinline__ uint64_t mndesc(uint32_t tile_addr, int j) {
  // MN-major operand, K step j: 16 K rows (2048 B) further; MN atoms 16 KB apart.
  return smem_desc_sw128(tile_addr + (uint32_t)(j * 2048), kAtom, 1024);
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__global__ void __launch_bounds__(kThreads, 1) scan_sm100_kernel(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
    const __grid_constant__ CUtensorMap tmV, const ScanArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem + kOffQ;
  uint8_t* sK = smem + kOffK;
  uint8_t* sV = smem + kOffV;
  uint8_t* sSb = smem + kOffSb;
  float* zs = reinterpret_cast<float*>(smem + kOffZ);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.x / args.H;
  const int h = blockIdx.x % args.H;
  const int nchunks = (args.T + C - 1) / C;
  const bool has_temp = args.temp != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[kFull0 + s], 1);
      mbar_init(&bars[kEmpty0 + s], 1);
    }
    mbar_init(&bars[kBarP], 1);
    mbar_init(&bars[kBarS], 1);
    mbar_init(&bars[kBarO], 1);
    mbar_init(&bars[kE1Done], 4);
    mbar_init(&bars[kSReady], 4);
    mbar_init(&bars[kOFree], 4);
    mbar_init(&bars[kKReady], 4);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      for (int c = 0; c < nchunks && !*abort_flag; ++c) {
        const int st = c & 1;
        const uint32_t ph = (uint32_t)(c >> 1) & 1u;
        if (!mbar_wait(&bars[kEmpty0 + st], ph ^ 1u, kWaitNs)) {
          report_status(args.status, FAKLA_ERR_TIMEOUT);
          *abort_flag = 1;
          break;
        }
        uint64_t* fb = &bars[kFull0 + st];
        mbar_arrive_expect_tx(fb, 3 * kTile);
        for (int a = 0; a < 2; ++a) {
          tma_load_4d(sQ + st * kTile + a * kAtom, &tmQ, fb, a * 64, h, c * C, b);
          tma_load_4d(sK + st * kTile + a * kAtom, &tmK, fb, a * 64, h, c * C, b);
          tma_load_4d(sV + st * kTile + a * kAtom, &tmV, fb, a * 64, h, c * C, b);
        }
      }
      if (*abort_flag) {
        // Let this CTA's own copies in flight land before the CTA exits.
        for (int c = nchunks - 2; c < nchunks; ++c)
          if (c >= 0) (void)mbar_wait(&bars[kFull0 + (c & 1)], (uint32_t)(c >> 1) & 1u, kWaitNs);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idP = idesc_bf16_f32(128, 128, false, false);   // Q . K^T
      constexpr uint32_t idOi = idesc_bf16_f32(128, 128, false, true);   // Q . S
      constexpr uint32_t idOt = idesc_bf16_f32(128, 128, false, true);   // Pm . V
      constexpr uint32_t idS = idesc_bf16_f32(128, 128, true, true);     // K^T . V
      const uint32_t aSb = smem_u32(sSb);
      bool ok = true;
      for (int c = 0; c < nchunks && ok && !*abort_flag; ++c) {
        const int st = c & 1;
        const uint32_t ph = (uint32_t)(c >> 1) & 1u;
        const uint32_t par = (uint32_t)c & 1u, prev = (uint32_t)(c - 1) & 1u;
        ok = mbar_wait(&bars[kFull0 + st], ph, kWaitNs);
        if (ok && has_temp) ok = mbar_wait(&bars[kKReady], par, kWaitNs);
        if (ok && c > 0) ok = mbar_wait(&bars[kE1Done], prev, kWaitNs);
        if (!ok) break;
        tc_fence_after();
        const uint32_t aQ = smem_u32(sQ + st * kTile);
        const uint32_t aK = smem_u32(sK + st * kTile);
        const uint32_t aV = smem_u32(sV + st * kTile);
        // MMA1: P = Q K^T
#pragma unroll
        for (int j = 0; j < 8; ++j) mma_ss(tmem + kColP, kdesc(aQ, j), kdesc(aK, j), idP, j > 0);
        mma_commit(&bars[kBarP]);
        ok = mbar_wait(&bars[kSReady], par, kWaitNs);
        if (ok && c > 0) ok = mbar_wait(&bars[kOFree], prev, kWaitNs);
        if (!ok) break;
        tc_fence_after();
        // MMA2: O = Q S_{<c}   (B = bf16 S in smem, MN-major: rows f, dv contiguous)
#pragma unroll
        for (int j = 0; j < 8; ++j) mma_ss(tmem + kColO, kdesc(aQ, j), mndesc(aSb, j), idOi, j > 0);
        // MMA4: S += K^T V   (A = K as M=f x K=s, MN-major; B = V MN-major)
#pragma unroll
        for (int j = 0; j < 8; ++j) mma_ss(tmem + kColS, mndesc(aK, j), mndesc(aV, j), idS, 1u);
        mma_commit(&bars[kBarS]);
        ok = mbar_wait(&bars[kE1Done], par, kWaitNs);
        if (!ok) break;
        tc_fence_after();
        // MMA3: O += Pm_hi V + Pm_lo V   (A from TMEM: 16 bf16 = 8 columns per K step)
#pragma unroll
        for (int j = 0; j < 8; ++j)
          mma_ts(tmem + kColO, tmem + kColPh + (uint32_t)(8 * j), mndesc(aV, j), idOt, 1u);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          mma_ts(tmem + kColO, tmem + kColPl + (uint32_t)(8 * j), mndesc(aV, j), idOt, 1u);
        mma_commit(&bars[kBarO]);
        mma_commit(&bars[kEmpty0 + st]);
      }
      if (!ok) {
        report_status(args.status, FAKLA_ERR_TIMEOUT);
        *abort_flag = 1;
      }
    }
  } else {
    // ---------------------------------------------------------------- compute
    const int q4 = warp & 3;
    const int r = 32 * q4 + lane;  // TMEM lane: token r (P, O) / feature r (S)
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q4) << 16);
    const int64_t bh = (int64_t)b * args.H + h;

    // ---- initial state: S into TMEM (fp32) and smem (bf16), z into smem
    {
      const bool load = (args.flags & FAKLA_STATE_IN) && args.S != nullptr;
      const float* srow = load ? args.S + (bh * D + r) * D : nullptr;
#pragma unroll 1
      for (int cc = 0; cc < D; cc += 16) {
        uint32_t v[16];
        float f[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          f[i] = load ? srow[cc + i] : 0.f;
          v[i] = __float_as_uint(f[i]);
        }
        tmem_st16(lane_addr + kColS + (uint32_t)cc, v);
        uint32_t p[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) p[i] = pack_bf16x2(f[2 * i], f[2 * i + 1]);
        uint8_t* atom = sSb + (cc >= 64 ? kAtom : 0);
        const int col = cc & 63;
        *reinterpret_cast<uint4*>(atom + sw128_offset(r, col)) = make_uint4(p[0], p[1], p[2], p[3]);
        *reinterpret_cast<uint4*>(atom + sw128_offset(r, col + 8)) = make_uint4(p[4], p[5], p[6], p[7]);
      }
      zs[r] = load ? args.z[bh * D + r] : 0.f;
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kSReady]);
    }

    bool ok = true;
    for (int c = 0; c < nchunks && !*abort_flag; ++c) {
      const int st = c & 1;
      const uint32_t ph = (uint32_t)(c >> 1) & 1u;
      const uint32_t par = (uint32_t)c & 1u;
      uint8_t* tQ = sQ + st * kTile;
      uint8_t* tK = sK + st * kTile;
      const int t_glob = c * C + r;
      const bool t_valid = t_glob < args.T;

      ok = mbar_wait(&bars[kFull0 + st], ph, kWaitNs);
      if (!ok) break;
      named_barrier_sync(1, 128);  // z of the previous chunk complete everywhere

      if (has_temp) {
        // k~ = k * temp: scale row r (token) of the K tile in place
        const float tv = t_valid
                             ? __bfloat162float(args.temp[((int64_t)b * args.T + t_glob) * args.H + h])
                             : 0.f;
#pragma unroll
        for (int a = 0; a < 2; ++a) {
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            uint4* p = reinterpret_cast<uint4*>(tK + a * kAtom + r * 128 + ch * 16);
            uint4 u = *p;
            float f[8];
            bf16x8_to_f32(u, f);
            u = make_uint4(pack_bf16x2(f[0] * tv, f[1] * tv), pack_bf16x2(f[2] * tv, f[3] * tv),
                           pack_bf16x2(f[4] * tv, f[5] * tv), pack_bf16x2(f[6] * tv, f[7] * tv));
            *p = u;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kKReady]);
        named_barrier_sync(1, 128);
      }

      // den_inter = q_t . z_{<c}   (row r of Q; chunks are position-permuted
      // inside a row by the swizzle, so read physical chunk p = logical p^(r&7))
      float dinter = 0.f;
#pragma unroll
      for (int a = 0; a < 2; ++a) {
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const uint4 u = *reinterpret_cast<const uint4*>(tQ + a * kAtom + r * 128 + p * 16);
          const int lc = p ^ (r & 7);
          float f[8];
          bf16x8_to_f32(u, f);
#pragma unroll
          for (int i = 0; i < 8; ++i) dinter = fmaf(f[i], zs[a * 64 + lc * 8 + i], dinter);
        }
      }
      named_barrier_sync(1, 128);  // all reads of z_{<c} done
      {
        // z += colsum(K): feature r, all 128 tokens of the chunk
        const int a = r >> 6, col = r & 63;
        const uint8_t* base = tK + a * kAtom;
        float zsum = 0.f;
#pragma unroll 8
        for (int s = 0; s < C; ++s) {
          const __nv_bfloat16 x =
              *reinterpret_cast<const __nv_bfloat16*>(base + sw128_offset((uint32_t)s, (uint32_t)col));
          zsum += __bfloat162float(x);
        }
        zs[r] += zsum;
      }

      // ---- E1: P row r -> inclusive causal mask -> hi/lo bf16 into TMEM
      ok = mbar_wait(&bars[kBarP], par, kWaitNs);
      if (!ok) break;
      tc_fence_after();
      float dintra = 0.f;
#pragma unroll 1
      for (int cc = 0; cc < C; cc += 32) {
        uint32_t v[32];
        tmem_ld32(lane_addr + kColP + (uint32_t)cc, v);
        tmem_ld_wait();
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int s0 = cc + 2 * i;
          float x0 = s0 <= r ? __uint_as_float(v[2 * i]) : 0.f;
          float x1 = s0 + 1 <= r ? __uint_as_float(v[2 * i + 1]) : 0.f;
          dintra += x0 + x1;
          const __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
          const float l0 = x0 - __bfloat162float(h0), l1 = x1 - __bfloat162float(h1);
          hi[i] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
          lo[i] = pack_bf16x2(l0, l1);
        }
        tmem_st16(lane_addr + kColPh + (uint32_t)(cc / 2), hi);
        tmem_st16(lane_addr + kColPl + (uint32_t)(cc / 2), lo);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kE1Done]);

      // ---- E2: S row r (fp32, TMEM) -> bf16 copy in smem (+ final state out)
      ok = mbar_wait(&bars[kBarS], par, kWaitNs);
      if (!ok) break;
      tc_fence_after();
      const bool last = (c == nchunks - 1);
      const bool sout = last && (args.flags & FAKLA_STATE_OUT) && args.S != nullptr;
#pragma unroll 1
      for (int cc = 0; cc < D; cc += 32) {
        uint32_t v[32];
        tmem_ld32(lane_addr + kColS + (uint32_t)cc, v);
        tmem_ld_wait();
        uint32_t p[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          p[i] = pack_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
        uint8_t* atom = sSb + (cc >= 64 ? kAtom : 0);
        const int col = cc & 63;
#pragma unroll
        for (int g = 0; g < 4; ++g)
          *reinterpret_cast<uint4*>(atom + sw128_offset(r, col + 8 * g)) =
              make_uint4(p[4 * g], p[4 * g + 1], p[4 * g + 2], p[4 * g + 3]);
        if (sout) {
          float4* dst = reinterpret_cast<float4*>(args.S + (bh * D + r) * D + cc);
#pragma unroll
          for (int g = 0; g < 8; ++g)
            dst[g] = make_float4(__uint_as_float(v[4 * g]), __uint_as_float(v[4 * g + 1]),
                                 __uint_as_float(v[4 * g + 2]), __uint_as_float(v[4 * g + 3]));
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kSReady]);

      // ---- E3: out row r = O / (den + eps)
      ok = mbar_wait(&bars[kBarO], par, kWaitNs);
      if (!ok) break;
      tc_fence_after();
      const float inv = 1.f / (dintra + dinter + kEps);
      __nv_bfloat16* orow = args.out + (((int64_t)b * args.T + t_glob) * args.H + h) * D;
#pragma unroll 1
      for (int cc = 0; cc < D; cc += 32) {
        uint32_t v[32];
        tmem_ld32(lane_addr + kColO + (uint32_t)cc, v);
        tmem_ld_wait();
        if (t_valid) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(v[8 * g + 0]) * inv, __uint_as_float(v[8 * g + 1]) * inv);
            u.y = pack_bf16x2(__uint_as_float(v[8 * g + 2]) * inv, __uint_as_float(v[8 * g + 3]) * inv);
            u.z = pack_bf16x2(__uint_as_float(v[8 * g + 4]) * inv, __uint_as_float(v[8 * g + 5]) * inv);
            u.w = pack_bf16x2(__uint_as_float(v[8 * g + 6]) * inv, __uint_as_float(v[8 * g + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + cc + 8 * g) = u;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kOFree]);
    }
    if (!ok) {
      report_status(args.status, FAKLA_ERR_TIMEOUT);
      *abort_flag = 1;
    }
    if (ok && (args.flags & FAKLA_STATE_OUT) && args.z != nullptr) args.z[bh * D + r] = zs[r];
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static bool make_map_bthd(CUtensorMap* map, const void* base, int64_t B, int64_t T, int64_t H) {
  // (B, T, H, 128) bf16 viewed as 4-D {d, h, t, b}; box = 64 d x 1 h x 128 t x 1 b.
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)H * D * 2,
                                 (cuuint64_t)T * H * D * 2};
  const cuuint32_t box[4] = {64, 1, (cuuint32_t)C, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return encode_tensor_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base),
                           dims, strides, box, estr, CU_TENSOR_MAP_SWIZZLE_128B);
}

bool scan_sm100_supported(int64_t B, int64_t T, int64_t H, int64_t Df, int64_t Dv) {
  return Df == D && Dv == D && B >= 1 && T >= 1 && H >= 1 && B * H <= (int64_t)INT32_MAX &&
         T <= (int64_t)INT32_MAX - C;
}

cudaError_t launch_scan_sm100(const void* q, const void* k, const void* v, const void* temp,
                              void* out, float* S, float* z, int64_t B, int64_t T, int64_t H,
                              unsigned flags, cudaStream_t stream, int* status, bool* encoded) {
  CUtensorMap mQ, mK, mV;
  const bool ok = make_map_bthd(&mQ, q, B, T, H) && make_map_bthd(&mK, k, B, T, H) &&
                  make_map_bthd(&mV, v, B, T, H);
  *encoded = ok;
  if (!ok) return cudaErrorInvalidValue;
  ScanArgs a;
  a.temp = (const __nv_bfloat16*)temp;
  a.out = (__nv_bfloat16*)out;
  a.S = S;
  a.z = z;
  a.T = (int)T;
  a.H = (int)H;
  a.flags = flags;
  a.status = status;
  cudaError_t e = cudaFuncSetAttribute(scan_sm100_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  scan_sm100_kernel<<<(unsigned)(B * H), kThreads, kSmemBytes, stream>>>(mQ, mK, mV, a);
  return cudaGetLastError();
}

}  // namespace fakla
