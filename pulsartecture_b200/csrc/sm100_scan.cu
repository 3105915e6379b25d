// Chunked causal FA-KLA scan on the sm_100a tensor cores (Df = Dv = 128, bf16
// activations, fp32 state). A CTA walks the tokens of one (b, h) sequence, or
// of one segment of it, in chunks of C = 128. For chunk c with rows
// Q = phi(q), K = phi(k)*temp, V:
//
//   P   = Q K^T                      (128x128 fp32, TMEM)            [MMA1]
//   Pm  = causal_mask_inclusive(P)   as bf16 in place in TMEM (the backward
//                                    modes: bf16 hi + lo residual)
//   O   = Q S_{<c}                   (S_{<c} as bf16 in smem)        [MMA2]
//   Dz  = Q [z_hi z_lo]              (z_{<c} split hi/lo, N = 16)    [MMA2b]
//   S  += K^T V                      (fp32, lives in TMEM)           [MMA4]
//   z  += K^T 1                      (fp32, N = 16, column 0)        [MMA4b]
//   O  += Pm V  (backward: Pm_hi V + Pm_lo V; A straight from TMEM) [MMA3]
//   out = O / (rowsum(Pm) + Dz[0] + Dz[1] + 1e-12), the row sum in fp32
//
// This is the chunk-parallel form of the reference recurrence
// (ultra_rwka/backend/cpp/cpu/cpu_kernels.cpp:107-164): out_t sums k~_s v_s
// (and k~_s for the denominator) over s <= t, exactly as the per-token loop
// does, with the state carried across chunks.
//
// Warp roles (448 threads): warp 0 TMA producer (Q, K, V tiles, 2 stages);
// warp 1 TMEM allocator + single-thread MMA issuer; three warpgroups, each
// thread owning one TMEM lane (token r for P/O, feature r for S/z):
//   warps 2-5   (P)  inclusive mask, bf16 P (and its residual), row sums
//   warps 6-9   (S)  state refresh: S (TMEM fp32) -> bf16 smem operand,
//                    z -> hi/lo operand; initial state in, final state out
//   warps 10-13 (O)  normalise O into a dead tile of the chunk and TMA-store
//                    it. The forward stages in the V tile (its readers MMA4
//                    and MMA3 are done at barO): Q and K of a stage come on
//                    one barrier and are refilled once MMA4 has read them, V
//                    on its own and refilled once the stores have read it;
//                    with heads of 128 the S warps, idle between refreshes,
//                    normalise and store columns 64-127. The backward modes
//                    stage in the Q tile (or, mode 3, the V tile) and refill
//                    Q after the stores, K/V after MMA3.
// so the mask of chunk c+1 overlaps the normalisation of chunk c and the
// state refresh, and the tensor pipe sees MMA2/MMA4 of one chunk between
// MMA1 and MMA3 of the next.
//
// Long sequences with few (b, h) pairs are split into G segments of whole
// chunks: scan_delta_sm100_kernel sums K^T V and K^T 1 over each segment but
// the last, scan_prefix_kernel turns those into each segment's initial state
// (plus the caller's initial state), and the main kernel runs one CTA per
// (b, h, segment).
//
// Every wait is bounded; on expiry the kernel records FAKLA_ERR_TIMEOUT in the
// device status word and winds down (copies and MMAs in flight are drained
// before TMEM is freed).
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
constexpr int kThreads = 448;
constexpr uint32_t kTmemCols = 512;
// TMEM columns: P (hi/lo written in place), O, S, z accumulator, Q.z result,
// and the two parity slots of the per-row sum of the masked P.
constexpr uint32_t kColP = 0, kColO = 128, kColS = 256, kColZ = 384, kColDz = 400, kColRs = 416;
constexpr uint64_t kWaitNs = 2000000000ull;
// Longest sleep per poll of a barrier wait (the thread wakes when the phase
// completes): waiting warps then take fewer issue slots from the working
// warps of their scheduler.
constexpr uint32_t kSleepNs = 20000;
constexpr int64_t kStateFloats = (int64_t)D * D + D;  // one (S, z) record

// Shared memory. Barriers sit in the first 256 bytes of the dynamic window;
// the operand region starts at the next 1024-byte boundary:
//   Q[2] K[2] V[2] (32 KB each) | M0 | M1 | Sb (32 KB)
// M0/M1 are two 1 KB swizzle atoms holding the N=16 K-major operands:
//   ZK (z_{<c} as bf16 hi in row 0, lo in row 1; features 0-63 in M0, 64-127
//   in M1) and ONES (rows 4 and 5 of M0 all 1.0). Only those rows feed result
//   columns that are read; the other rows of the 16-row operands fall on
//   whatever lies there (M0/M1/Sb) and only produce columns nobody reads.
constexpr size_t kOffQ = 0;
constexpr size_t kOffK = kOffQ + kStages * kTile;
constexpr size_t kOffV = kOffK + kStages * kTile;
constexpr size_t kOffM0 = kOffV + kStages * kTile;
constexpr size_t kOffM1 = kOffM0 + 1024;
constexpr size_t kOffSb = kOffM1 + 1024;
constexpr size_t kOperandBytes = kOffSb + kTile;
// The unnormalised modes keep one K tile (stage 0) and use the second K slot
// for Sb_lo: their state enters MMA2 as bf16 hi + lo (the backward's
// products cancel to small results, where one bf16 rounding of S shows).
constexpr size_t kHeadBytes = 256;
constexpr size_t kSmemBytes = 1024 + kOperandBytes;  // 232448 = the sm_100 per-CTA maximum
constexpr uint32_t kSmallSbo = 2048;                 // rows 8-15 of the N=16 operands

enum Bar {
  kFull0 = 0,
  kEmpty0 = kFull0 + kStages,   // K, V tiles of a stage free (MMA3 done)
  kEmptyQ0 = kEmpty0 + kStages, // Q tile of a stage free (output stored from it)
  kBarP = kEmptyQ0 + kStages,
  kBarS,
  kBarO,
  kE1Done,
  kSReady,
  kOFree,
  kKReady,
  kDrain,
  kKFree,   // unnormalised modes: the single K tile read by MMA4
  kRow0,    // (4) per output warp: its 32 rows of the epilogue's row tensor landed
  kFullV0 = kRow0 + 4,  // (kStages) forward: the V tile of a stage landed (Q, K: kFull0)
  kNumBars = kFullV0 + kStages
};
static_assert(kNumBars * 8 + 8 <= kHeadBytes, "barrier area");

struct ScanArgs {
  const __nv_bfloat16* temp;  // (B,T,H) or null
  float* S;                   // (B,H,D,D) or null
  float* z;                   // (B,H,D) or null
  const float* seg_init;      // (B*H, G) records of (S, z): each segment's initial state; or null
  int T, H;
  int G;                      // segments per sequence
  int seg_chunks;             // chunks per segment
  unsigned flags;
  int* status;
  int hd;  // head size: 128, or 64 (features and values in the first 64 columns of
           // each tile, whose second 64-column atom stays zero)
  // backward passes (modes below)
  const __nv_bfloat16* grad_rows;  // kScanNormalGrad: (B,T,H,D) output gradient -> dden_out
  float* dden_out;                 // (B,T,H): -(bf16(g/den) . out) (g = grad_rows)
  int dnum_store;                  // kScanNormalGrad: the output rows are bf16(g/den)
  const float* add;           // (B,T,H) per-token term added to the kept P entries, or null
  float* den_out;             // (B,T,H) denominators of the normalised mode, or null
  int state_in_T;             // the initial state is given transposed (S[dv][f])
  // backward epilogues: out = (o + coef * vec_c + sigma_t mvec) * row_scale, vec_c =
  // vec_init + the sums of the chunks walked before chunk c,
  // coef = add[t] in kScanRowAdd and 1 in kScanRevCol, sigma_t = the row's
  // kept q'.k' + term summed over all chunks so far (the centring term of
  // v' = v - mvec); dot_out[t] = sum(that unscaled row * dot_rows[t])
  const float* vec;           // (B*H, nchunks, hd) per-chunk sums, or null
  const float* vec_init;      // (B*H, hd): the vector before the first chunk walked, or null (0)
  float* vec_total;           // (B*H, hd): vec_init + every chunk's sum, or null
  int vec_mma;                // kScanRevCol: the chunk sums are v'^T add, on the tensor cores
  const float* mvec;          // (B*H, D), or null
  const __nv_bfloat16* row_scale;  // (B,T,H), or null
  const __nv_bfloat16* dot_rows;   // (B,T,H,D) with dot_out, or null
  __nv_bfloat16* dot_out;          // (B,T,H), or null
};

// Modes of scan_sm100_kernel. The backward of FA-KLA is three unnormalised
// scans of the same shape as the forward one (simt_backward.cu gives the
// formulas; sm100_backward.cu runs them):
//   kScanNormal  out = (q S_{<c} + (M o Q K^T) V) / den        (the forward)
//   kScanNormalGrad  the forward, also writing den and dden (backward's first pass)
//   kScanRowAdd  out = q S_{<c} + (M o (Q K^T + a 1^T)) V       (dq: a = dden)
//   kScanRevRaw  out = q S_{>c} + (M' o Q K^T) V                (dv, reversed time)
//   kScanRevCol  out = q S_{>c} + (M' o (Q K^T + 1 b^T)) V      (dk~, reversed: b = dden)
// M keeps s <= t; M' keeps s >= t and the chunks are walked from the end.
enum { kScanNormal = 0, kScanRowAdd = 1, kScanRevRaw = 2, kScanRevCol = 3, kScanNormalGrad = 4 };

__device__ __forceinline__ uint64_t kdesc(uint32_t tile_addr, int j) {
  // K-major operand, K step j (16 elements): atom j/4, +32 B per step inside.
  return smem_desc_sw128(tile_addr + (uint32_t)((j >> 2) * kAtom + (j & 3) * 32), 16, 1024);
}
__device__ __forceinline__ uint64_t mndesc(uint32_t tile_addr, int j) {
  // MN-major operand, K step j: 16 K rows (2048 B) further; MN atoms 16 KB apart.
  return smem_desc_sw128(tile_addr + (uint32_t)(j * 2048), kAtom, 1024);
}
// N=16 K-major operands: ZK atoms are the two 1 KB blocks M0, M1; ONES rows
// 4 and 5 of M0 serve as row 0 of atoms 0 and 1 (a uniform row reads the
// same under any swizzle phase).
__device__ __forceinline__ uint64_t zkdesc(uint32_t m0_addr, int j) {
  return smem_desc_sw128(m0_addr + (uint32_t)((j >> 2) * 1024 + (j & 3) * 32), 16, kSmallSbo);
}
__device__ __forceinline__ uint64_t onesdesc(uint32_t m0_addr, int j) {
  return smem_desc_sw128(m0_addr + 512u + (uint32_t)((j >> 2) * 128 + (j & 3) * 32), 16, kSmallSbo);
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// k~ = k * temp on row r (one token) of a K tile in shared memory. Rows are
// 128 bytes (all 32 banks), so the 16-byte pieces are visited in an order
// rotated by the row: the 32 rows of a warp then touch 8 different bank
// groups per access instead of one.
__device__ __forceinline__ void scale_k_row(uint8_t* tK, int r, float tv) {
  const __nv_bfloat162 t2 = __floats2bfloat162_rn(tv, tv);
#pragma unroll
  for (int a = 0; a < 2; ++a) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int ch = (c + r) & 7;
      uint4* p = reinterpret_cast<uint4*>(tK + a * kAtom + r * 128 + ch * 16);
      uint4 u = *p;
      // bf16 pair products, rounded once (tv is a bf16 value): the same bits
      // as rounding the fp32 product k * temp
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) h[e] = __hmul2(h[e], t2);
      *p = u;
    }
  }
}

__device__ __forceinline__ float temp_at(const __nv_bfloat16* temp, int b, int T, int H, int h, int t) {
  return t < T ? __bfloat162float(temp[((int64_t)b * T + t) * H + h]) : 0.f;
}

// Per-token fp32 term of the backward scans (0 past the end of the sequence).
__device__ __forceinline__ float add_at(const float* add, int b, int T, int H, int h, int t) {
  return t < T ? add[((int64_t)b * T + t) * H + h] : 0.f;
}

// Write z_f as bf16 hi (row 0) and lo (row 1) of the ZK operand.
__device__ __forceinline__ void put_zk(uint8_t* m0, int f, float zf) {
  const __nv_bfloat16 hi = __float2bfloat16_rn(zf);
  const __nv_bfloat16 lo = __float2bfloat16_rn(zf - __bfloat162float(hi));
  uint8_t* blk = m0 + (f >= 64 ? 1024 : 0);
  *reinterpret_cast<__nv_bfloat16*>(blk + sw128_offset(0, (uint32_t)(f & 63))) = hi;
  *reinterpret_cast<__nv_bfloat16*>(blk + sw128_offset(1, (uint32_t)(f & 63))) = lo;
}

// Tokens [sbase, sbase+32) of row r of P (fp32 bits in v), split into bf16
// hi + lo and stored in place: hi in columns sbase + [0,16), lo in sbase +
// [16,32) (two tokens per column). kMask: 0 keeps the whole group, 1 keeps
// s <= r (causal diagonal group), 2 keeps s >= r (reversed diagonal group).
// The kept values first get `arow` (a per-row term) and bcol[s - sbase] (a
// per-column term: 32 floats in shared memory, the same for every row).
// Returns the sum of the kept values.
template <int kMask, bool kCol, bool kRow, bool kLo = true>
__device__ __forceinline__ float split_group(const uint32_t (&v)[32], int sbase, int r,
                                             uint32_t p_addr, float arow, const float* bcol) {
  uint32_t hi[16], lo[16];
  float rs = 0.f;
  const uint64_t arow2 = f2_splat(arow);
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    // token pair (2e, 2e+1) as an fp32 pair on the paired FP32 pipe
    uint64_t x = f2_make(v[2 * e], v[2 * e + 1]);
    if (kRow) x = f2_add(x, arow2);  // (x + 0 is not folded away: keep the add out of the other modes)
    if (kCol) x = f2_add(x, reinterpret_cast<const uint64_t*>(bcol)[e]);
    if (kMask != 0) {
      float2 xf = f2_split(x);
      if (kMask == 1) {
        xf.x = sbase + 2 * e <= r ? xf.x : 0.f;
        xf.y = sbase + 2 * e + 1 <= r ? xf.y : 0.f;
      } else {
        xf.x = sbase + 2 * e >= r ? xf.x : 0.f;
        xf.y = sbase + 2 * e + 1 >= r ? xf.y : 0.f;
      }
      x = f2_make(__float_as_uint(xf.x), __float_as_uint(xf.y));
    }
    const float2 xf = f2_split(x);
    rs += xf.x + xf.y;
    hi[e] = pack_bf16x2(xf.x, xf.y);
    if (kLo) lo[e] = pack_bf16x2(f2_sub(x, f2_from_bf16x2(hi[e])));
  }
  tmem_st16(p_addr + (uint32_t)sbase, hi);
  if (kLo) tmem_st16(p_addr + (uint32_t)(sbase + 16), lo);
  return rs;
}

// Row r of P, token group g (32 tokens) of a warp whose rows are the group
// q4. Causal: groups below the diagonal are kept whole, the diagonal one is
// masked. Reversed: groups above the diagonal are kept whole.
template <bool kRev, bool kCol, bool kRow, bool kLo = true>
__device__ __forceinline__ float split_group_at(const uint32_t (&v)[32], int g, int q4, int r,
                                                uint32_t p_addr, float arow, const float* bcol) {
  return g == q4 ? split_group<kRev ? 2 : 1, kCol, kRow, kLo>(v, 32 * g, r, p_addr, arow, bcol)
                 : split_group<0, kCol, kRow, kLo>(v, 32 * g, r, p_addr, arow, bcol);
}

// Outside the kept triangle the whole group is masked: hi = lo = 0.
__device__ __forceinline__ void zero_group(int g, uint32_t p_addr) {
  uint32_t zz[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) zz[e] = 0u;
  tmem_st16(p_addr + (uint32_t)(32 * g), zz);
  tmem_st16(p_addr + (uint32_t)(32 * g + 16), zz);
}

// State row r, columns [c, c+8) into the MN-major bf16 operand Sb (and, with
// kLo, the residual S - bf16(S) into Sb_lo).
template <bool kLo>
__device__ __forceinline__ void put_sb8(uint8_t* sb, uint8_t* sb_lo, int r, int c, const float* f) {
  uint32_t hi[4], lo[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    hi[e] = pack_bf16x2(f[2 * e], f[2 * e + 1]);
    if (kLo)
      lo[e] = pack_bf16x2(f2_sub(f2_make(__float_as_uint(f[2 * e]), __float_as_uint(f[2 * e + 1])),
                                 f2_from_bf16x2(hi[e])));
  }
  const uint32_t off = (c >= 64 ? kAtom : 0) + sw128_offset((uint32_t)r, (uint32_t)(c & 63));
  *reinterpret_cast<uint4*>(sb + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  if (kLo) *reinterpret_cast<uint4*>(sb_lo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

// 32 fp32 values (bits in v) times inv, written as bf16 into row r, columns
// [col0, col0+32) of a 128-row x 128-column 128B-swizzled staging tile.
__device__ __forceinline__ void stage_scaled_32(const uint32_t (&v)[32], float inv, uint8_t* tile,
                                                int r, int col0) {
  uint8_t* atom = tile + (col0 >= 64 ? kAtom : 0);
  const uint64_t inv2 = f2_splat(inv);
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint4 u;
    u.x = pack_bf16x2(f2_mul(f2_make(v[8 * g + 0], v[8 * g + 1]), inv2));
    u.y = pack_bf16x2(f2_mul(f2_make(v[8 * g + 2], v[8 * g + 3]), inv2));
    u.z = pack_bf16x2(f2_mul(f2_make(v[8 * g + 4], v[8 * g + 5]), inv2));
    u.w = pack_bf16x2(f2_mul(f2_make(v[8 * g + 6], v[8 * g + 7]), inv2));
    *reinterpret_cast<uint4*>(atom + sw128_offset((uint32_t)r, (uint32_t)((col0 & 63) + 8 * g))) = u;
  }
}

// Half a row (64 bf16 from column c0) of a 128-row x 128-column 128B-swizzled
// tile in shared memory.
__device__ __forceinline__ void load_row_smem(const uint8_t* tile, int r, int c0, uint4 (&u)[8]) {
  const uint8_t* atom = tile + (c0 >= 64 ? kAtom : 0);
#pragma unroll
  for (int k = 0; k < 8; ++k)
    u[k] = *reinterpret_cast<const uint4*>(atom + sw128_offset((uint32_t)r, (uint32_t)((c0 & 63) + 8 * k)));
}

// Half a row (64 bf16 from column c0) into a 128-row x 128-column
// 128B-swizzled tile in shared memory (the layout load_row_smem reads).
__device__ __forceinline__ void store_row_smem(uint8_t* tile, int r, int c0, const uint4 (&u)[8]) {
  uint8_t* atom = tile + (c0 >= 64 ? kAtom : 0);
#pragma unroll
  for (int k = 0; k < 8; ++k)
    *reinterpret_cast<uint4*>(atom + sw128_offset((uint32_t)r, (uint32_t)((c0 & 63) + 8 * k))) = u[k];
}

// sum over 32 columns of bf16(g * inv) * (x * inv): x = out * den (fp32 bits
// in v), g = 32 bf16 of the output gradient row (4 uint4). g is replaced by
// bf16(g * inv) (dnum, rounded as bf16 pairs), the value the sum uses.
__device__ __forceinline__ float dden_dot_32(const uint32_t (&v)[32], float inv, uint4* g) {
  const uint64_t inv2 = f2_splat(inv);
  uint64_t acc = f2_splat(0.f);  // even columns in the low half, odd in the high half
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint32_t* w = reinterpret_cast<uint32_t*>(&g[k]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      w[e] = pack_bf16x2(f2_mul(f2_from_bf16x2(w[e]), inv2));
      acc = f2_fma(f2_from_bf16x2(w[e]), f2_make(v[8 * k + 2 * e], v[8 * k + 2 * e + 1]), acc);
    }
  }
  const float2 a = f2_split(acc);
  return (a.x + a.y) * inv;
}

// Backward epilogue of one row: y = (x + coef * vec + sig * mv) * scale over
// columns [col0, col0+32), written as bf16 like stage_scaled_32. vec and mv
// (32 floats each from column col0, shared memory, the same for every row;
// mv only with kM) are read as broadcasts. With kDot the return value is
// sum(x + coef * vec + sig * mv) * k over these columns, k = 32 bf16 of this
// row (4 uint4), else 0.
// Columns are processed as fp32 pairs on the paired FP32 pipe (each element
// rounded as the scalar fmaf/multiply would round it); the dot keeps the
// even and odd columns in the two halves of one accumulator pair.
template <bool kDot, bool kM>
__device__ __forceinline__ float stage_affine_32(const uint32_t (&v)[32], float coef, const float* vec,
                                                 float sig, const float* mv, float scale,
                                                 const uint4* krow, uint8_t* tile, int r, int col0) {
  uint8_t* atom = tile + (col0 >= 64 ? kAtom : 0);
  const uint64_t coef2 = f2_splat(coef), sig2 = f2_splat(sig), scale2 = f2_splat(scale);
  const bool scaled = scale != 1.f;  // multiplying by 1 changes nothing
  uint64_t dot2 = f2_splat(0.f);
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const ulonglong2 w01 = reinterpret_cast<const ulonglong2*>(vec)[2 * g];
    const ulonglong2 w23 = reinterpret_cast<const ulonglong2*>(vec)[2 * g + 1];
    const uint64_t w[4] = {w01.x, w01.y, w23.x, w23.y};
    uint64_t y[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) y[e] = f2_fma(coef2, w[e], f2_make(v[8 * g + 2 * e], v[8 * g + 2 * e + 1]));
    if (kM) {
      const ulonglong2 m01 = reinterpret_cast<const ulonglong2*>(mv)[2 * g];
      const ulonglong2 m23 = reinterpret_cast<const ulonglong2*>(mv)[2 * g + 1];
      const uint64_t m[4] = {m01.x, m01.y, m23.x, m23.y};
#pragma unroll
      for (int e = 0; e < 4; ++e) y[e] = f2_fma(sig2, m[e], y[e]);
    }
    if (kDot) {
      const uint32_t kw[4] = {krow[g].x, krow[g].y, krow[g].z, krow[g].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) dot2 = f2_fma(y[e], f2_make(kw[e] << 16, kw[e] & 0xffff0000u), dot2);
    }
    if (scaled) {
#pragma unroll
      for (int e = 0; e < 4; ++e) y[e] = f2_mul(y[e], scale2);
    }
    uint4 u;
    u.x = pack_bf16x2(y[0]);
    u.y = pack_bf16x2(y[1]);
    u.z = pack_bf16x2(y[2]);
    u.w = pack_bf16x2(y[3]);
    *reinterpret_cast<uint4*>(atom + sw128_offset((uint32_t)r, (uint32_t)((col0 & 63) + 8 * g))) = u;
  }
  const float2 d = f2_split(dot2);
  return d.x + d.y;
}

// The bounded wait with a suspend-time hint.
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  return mbar_wait_hint(bar, parity, limit_ns, kSleepNs);
}

// Warp-uniform forms of the bounded wait and of the abort check, for warps
// that go on to issue .sync.aligned tcgen05 loads and stores.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, bar_wait(bar, parity, kWaitNs));
}
__device__ __forceinline__ bool warp_aborted(volatile int* abort_flag) {
  return __any_sync(0xffffffffu, *abort_flag != 0);
}

__device__ __forceinline__ uint8_t* operand_base(uint8_t* raw) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + kHeadBytes + 1023) &
                                    ~uintptr_t(1023));
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) scan_sm100_kernel(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
    const __grid_constant__ CUtensorMap tmR, const ScanArgs args) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* smem = operand_base(smem_raw);
  // The operand region must end inside the allocation (true unless the
  // dynamic window starts more than 768 bytes past a 1 KB boundary).
  if (smem + kOperandBytes > smem_raw + kSmemBytes) {
    if (threadIdx.x == 0) report_status(args.status, FAKLA_ERR_ALIGNMENT);
    return;
  }
  uint8_t* sQ = smem + kOffQ;
  uint8_t* sK = smem + kOffK;
  uint8_t* sV = smem + kOffV;
  uint8_t* sM0 = smem + kOffM0;
  uint8_t* sSb = smem + kOffSb;
  uint8_t* sSbLo = smem + kOffK + kTile;  // unnormalised modes only

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh_idx = blockIdx.x / args.G;
  const int seg = blockIdx.x % args.G;
  const int b = bh_idx / args.H;
  const int h = bh_idx % args.H;
  const int nchunks_total = (args.T + C - 1) / C;
  const int c0 = seg * args.seg_chunks;
  const int c1 = min(nchunks_total, c0 + args.seg_chunks);
  const int nch = c1 - c0;
  const bool has_temp = args.temp != nullptr;
  const bool last_seg = seg == args.G - 1;
  constexpr bool kGrad = MODE == kScanNormalGrad;
  constexpr bool kRaw = MODE != kScanNormal && !kGrad;  // no normaliser: q.z, z, den not formed
  constexpr bool kRev = MODE == kScanRevRaw || MODE == kScanRevCol;  // chunks from the end, s >= t kept
  // the k' row sum z (MMA4b) and q'.z (MMA2b): the normaliser of the forward,
  // the centring term of kScanRowAdd
  constexpr bool kZ = MODE != kScanRevRaw && MODE != kScanRevCol;
  // The epilogue's per-row tensor (the output gradient of kScanNormalGrad,
  // the dot rows of kScanRevCol) comes by TMA into the chunk's Q tile once
  // the MMAs have read it; kScanRevCol then stages its output in the V tile,
  // which its output warps (not MMA3's commit) hand back to the producer.
  constexpr bool kRowTile = kGrad || MODE == kScanRevCol;
  constexpr bool kStageInV = MODE == kScanRevCol;
  // The forward loads Q and K (needed first, by MMA1 and MMA2) apart from V
  // (needed from MMA4 on) and stages its output in the V tile: the Q and K
  // tiles of a stage are refilled as soon as MMA4 has read them, and only V
  // waits for the output stores of the chunk two back, so those stores stay
  // off the path to the next MMA1.
  constexpr bool kSplitV = MODE == kScanNormal;
  // P enters MMA3 as bf16 hi + lo (the residual) in the backward modes, whose
  // products cancel to small results, and as bf16 alone in the forward: one
  // MMA3 per K step and no residual in the split (the split's instructions sit
  // on the chunk's critical chain). The forward's error against the oracle
  // stays within the bf16 bar: 2.4e-3 rel-L2 at config 2 against 1.6e-3 with
  // the residual (bar 5e-3), max-abs 1e-3 (bar 2e-2).
  constexpr bool kPLo = MODE != kScanNormal;
  // Vectors shared by every row of a chunk, broadcast from shared memory in
  // the unused rows of the two 1 KB N=16 operand atoms (with kZ, rows 0-1 of
  // both hold ZK and rows 4-5 of M0 ONES; the other rows only feed result
  // columns nobody reads): the epilogue's vector, the centring vector
  // (kScanRowAdd: m[0:64] in rows 6-7 of M0, m[64:128] in rows 6-7 of M1) and
  // the per-column terms of kScanRevCol.
  constexpr bool kAffine = MODE == kScanRowAdd || MODE == kScanRevCol;
  float* vec_sm = reinterpret_cast<float*>(sM0 + 1024 + (kZ ? 256 : 0));
  float* mlo_sm = reinterpret_cast<float*>(sM0 + 768);
  float* mhi_sm = reinterpret_cast<float*>(sM0 + 1024 + 768);
  float* bcol_sm = reinterpret_cast<float*>(sM0);
  auto k_tile = [&](int st) { return sK + (kRaw ? 0 : st * kTile); };
  // The forward's output epilogue is split by columns: the output warps take
  // columns 0-63 of each chunk and the state warps, idle between their state
  // refreshes, columns 64-127 (128-wide heads), which shortens the chain
  // output -> OFree -> next chunk's MMA2 that sets the chunk period.
  const bool split_o = MODE == kScanNormal && args.hd == 128;
  // first token of this CTA's chunk i
  auto chunk_t0 = [&](int i) {
    const int ci = c0 + i;
    return (kRev ? nchunks_total - 1 - ci : ci) * C;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[kFull0 + s], 1);
      mbar_init(&bars[kEmpty0 + s], kSplitV ? (split_o ? 8 : 4) : (kStageInV ? 4 : 1));
      mbar_init(&bars[kEmptyQ0 + s], kSplitV ? 1 : 4);
      mbar_init(&bars[kFullV0 + s], 1);
    }
    mbar_init(&bars[kBarP], 1);
    mbar_init(&bars[kBarS], 1);
    mbar_init(&bars[kBarO], 1);
    mbar_init(&bars[kE1Done], 4);
    mbar_init(&bars[kSReady], 4);
    mbar_init(&bars[kOFree], split_o ? 8 : 4);
    mbar_init(&bars[kKReady], 4);
    mbar_init(&bars[kDrain], 1);
    mbar_init(&bars[kKFree], 1);
    for (int w = 0; w < 4; ++w) mbar_init(&bars[kRow0 + w], 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
    if (kRowTile) tma_prefetch_desc(&tmR);
  }
  // ONES: rows 4-5 of M0 (256 bytes of bf16 1.0).
  if (threadIdx.x < 64)
    reinterpret_cast<uint32_t*>(sM0 + 512)[threadIdx.x] = 0x3F803F80u;
  // 64-wide heads: the second atom of every Q, K and V tile is zero for the
  // whole kernel (no load writes it; the output is staged in the first atom
  // only), so the MMAs see zero features and values past column 64.
  const int na = args.hd == 64 ? 1 : 2;  // 64-column atoms loaded per tile
  if (na == 1) {
    constexpr int kPer = kAtom / 16;
    for (int o = threadIdx.x; o < 3 * kStages * kPer; o += kThreads) {
      const int t = o / kPer;  // Q0 Q1 K0 K1 V0 V1
      // the unnormalised modes keep one K tile (the second K slot is Sb_lo)
      if (kRaw && t == 3) continue;
      uint8_t* base = (t < 2 ? sQ : (t < 4 ? sK : sV)) + (t & 1) * kTile + kAtom;
      reinterpret_cast<uint4*>(base)[o % kPer] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  // set-up of shared memory done: from here on the kernel reads inputs
  // earlier work may write
  griddep_wait();
  griddep_launch_dependents();
  // kScanRowAdd's centring vector, read by the output warps: m[0:64] in rows
  // 6-7 of M0, m[64:128] in rows 6-7 of M1 (zero without centring, so that
  // sigma * m is 0 whatever those rows held before)
  if (MODE == kScanRowAdd && threadIdx.x < 128) {
    const int f = threadIdx.x;
    const float mf = (args.mvec != nullptr && f < args.hd) ? args.mvec[(int64_t)bh_idx * args.hd + f] : 0.f;
    (f < 64 ? mlo_sm[f] : mhi_sm[f - 64]) = mf;
  }
  fence_proxy_async_smem();
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
      int issued = 0, issued_v = 0;
      for (int i = 0; i < nch && !*abort_flag; ++i) {
        const int st = i & 1;
        const uint32_t ph = (uint32_t)(i >> 1) & 1u;
        if constexpr (kSplitV) {
          const int t0 = chunk_t0(i);
          // Q, K of chunk i: MMA1-MMA4 of chunk i-2 have read the stage
          if (!bar_wait(&bars[kEmptyQ0 + st], ph ^ 1u, kWaitNs)) {
            report_status(args.status, FAKLA_ERR_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          uint64_t* fb = &bars[kFull0 + st];
          mbar_arrive_expect_tx(fb, 2 * na * kAtom);
          for (int a = 0; a < na; ++a) {
            tma_load_4d(sQ + st * kTile + a * kAtom, &tmQ, fb, a * 64, h, t0, b);
            tma_load_4d(sK + st * kTile + a * kAtom, &tmK, fb, a * 64, h, t0, b);
          }
          ++issued;
          // V of chunk i: the stores of chunk i-2's output (staged in this
          // V tile) have read it
          if (!bar_wait(&bars[kEmpty0 + st], ph ^ 1u, kWaitNs)) {
            report_status(args.status, FAKLA_ERR_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          uint64_t* fv = &bars[kFullV0 + st];
          mbar_arrive_expect_tx(fv, na * kAtom);
          for (int a = 0; a < na; ++a) tma_load_4d(sV + st * kTile + a * kAtom, &tmV, fv, a * 64, h, t0, b);
          ++issued_v;
          continue;
        }
        if (!bar_wait(&bars[kEmpty0 + st], ph ^ 1u, kWaitNs)) {
          report_status(args.status, FAKLA_ERR_TIMEOUT);
          *abort_flag = 1;
          break;
        }
        uint64_t* fb = &bars[kFull0 + st];
        mbar_arrive_expect_tx(fb, 3 * na * kAtom);
        const int t0 = chunk_t0(i);
        if constexpr (kRaw) {
          for (int a = 0; a < na; ++a) tma_load_4d(sV + st * kTile + a * kAtom, &tmV, fb, a * 64, h, t0, b);
          ++issued;
          // one K tile: MMA4 of the previous chunk must have read it
          if (i > 0 && !bar_wait(&bars[kKFree], (uint32_t)(i - 1) & 1u, kWaitNs)) {
            report_status(args.status, FAKLA_ERR_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          for (int a = 0; a < na; ++a) tma_load_4d(sK + a * kAtom, &tmK, fb, a * 64, h, t0, b);
        } else {
          for (int a = 0; a < na; ++a) {
            tma_load_4d(sK + st * kTile + a * kAtom, &tmK, fb, a * 64, h, t0, b);
            tma_load_4d(sV + st * kTile + a * kAtom, &tmV, fb, a * 64, h, t0, b);
          }
          ++issued;
        }
        // The Q tile doubles as the output staging of chunk i-2: wait for
        // that store to have read it.
        if (!bar_wait(&bars[kEmptyQ0 + st], ph ^ 1u, kWaitNs)) {
          report_status(args.status, FAKLA_ERR_TIMEOUT);
          *abort_flag = 1;
          break;
        }
        for (int a = 0; a < na; ++a)
          tma_load_4d(sQ + st * kTile + a * kAtom, &tmQ, fb, a * 64, h, t0, b);
      }
      if (*abort_flag) {
        // Let this CTA's own copies in flight land before the CTA exits.
        for (int i = issued - kStages; i < issued; ++i)
          if (i >= 0) (void)bar_wait(&bars[kFull0 + (i & 1)], (uint32_t)(i >> 1) & 1u, kWaitNs);
        for (int i = issued_v - kStages; i < issued_v; ++i)
          if (i >= 0) (void)bar_wait(&bars[kFullV0 + (i & 1)], (uint32_t)(i >> 1) & 1u, kWaitNs);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idP = idesc_bf16_f32(128, 128, false, false);   // Q . K^T
      constexpr uint32_t idQS = idesc_bf16_f32(128, 128, false, true);   // Q . S
      constexpr uint32_t idQZ = idesc_bf16_f32(128, 16, false, false);   // Q . [z_hi z_lo]
      constexpr uint32_t idPV = idesc_bf16_f32(128, 128, false, true);   // Pm . V
      constexpr uint32_t idKV = idesc_bf16_f32(128, 128, true, true);    // K^T . V
      constexpr uint32_t idK1 = idesc_bf16_f32(128, 16, true, false);    // K^T . 1
      const uint32_t aSb = smem_u32(sSb);
      const uint32_t aSbLo = smem_u32(sSbLo);
      const uint32_t aM0 = smem_u32(sM0);
      bool ok = true;
      bool issued_any = false;
      for (int i = 0; i < nch && ok && !*abort_flag; ++i) {
        const int st = i & 1;
        const uint32_t ph = (uint32_t)(i >> 1) & 1u;
        const uint32_t par = (uint32_t)i & 1u, prev = (uint32_t)(i - 1) & 1u;
        ok = bar_wait(&bars[kFull0 + st], ph, kWaitNs);
        if (ok && has_temp) ok = bar_wait(&bars[kKReady], par, kWaitNs);
        if (!ok) break;
        tc_fence_after();
        const uint32_t aQ = smem_u32(sQ + st * kTile);
        const uint32_t aK = smem_u32(k_tile(st));
        const uint32_t aV = smem_u32(sV + st * kTile);
        issued_any = true;
        // MMA1: P = Q K^T (overwrites the hi/lo of the previous chunk, which
        // MMA3 of that chunk, issued earlier, has consumed: MMAs run in order)
#pragma unroll
        for (int j = 0; j < 8; ++j) mma_ss(tmem + kColP, kdesc(aQ, j), kdesc(aK, j), idP, j > 0);
        mma_commit(&bars[kBarP]);
        ok = bar_wait(&bars[kSReady], par, kWaitNs);
        if (ok && i > 0) ok = bar_wait(&bars[kOFree], prev, kWaitNs);
        if (!ok) break;
        tc_fence_after();
        // MMA2 / MMA2b: O = Q S_{<c}, Dz = Q [z_hi z_lo]
#pragma unroll
        for (int j = 0; j < 8; ++j) mma_ss(tmem + kColO, kdesc(aQ, j), mndesc(aSb, j), idQS, j > 0);
        if constexpr (kRaw) {
#pragma unroll
          for (int j = 0; j < 8; ++j) mma_ss(tmem + kColO, kdesc(aQ, j), mndesc(aSbLo, j), idQS, 1u);
        }
        if constexpr (kZ) {
#pragma unroll
          for (int j = 0; j < 8; ++j) mma_ss(tmem + kColDz, kdesc(aQ, j), zkdesc(aM0, j), idQZ, j > 0);
        }
        if constexpr (kSplitV) {
          ok = bar_wait(&bars[kFullV0 + st], ph, kWaitNs);
          if (!ok) break;
          tc_fence_after();
        }
        // MMA4 / MMA4b: S += K^T V, z += K^T 1 (A = K as M=f x K=s, MN-major)
#pragma unroll
        for (int j = 0; j < 8; ++j) mma_ss(tmem + kColS, mndesc(aK, j), mndesc(aV, j), idKV, 1u);
        if constexpr (kZ) {
#pragma unroll
          for (int j = 0; j < 8; ++j) mma_ss(tmem + kColZ, mndesc(aK, j), onesdesc(aM0, j), idK1, 1u);
        }
        // the last reader of the single K tile of the unnormalised modes
        if constexpr (kRaw) mma_commit(&bars[kKFree]);
        mma_commit(&bars[kBarS]);
        if constexpr (kSplitV) mma_commit(&bars[kEmptyQ0 + st]);  // Q, K of this stage read
        ok = bar_wait(&bars[kE1Done], par, kWaitNs);
        if (!ok) break;
        tc_fence_after();
        // MMA3: O += Pm_hi V (+ Pm_lo V in the backward modes). Hi/lo of
        // tokens [32g, 32g+32) sit in columns 32g + [0,16) and 32g + [16,32);
        // K step j = 16 tokens.
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t col = kColP + (uint32_t)(32 * (j >> 1) + 8 * (j & 1));
          mma_ts(tmem + kColO, tmem + col, mndesc(aV, j), idPV, 1u);
          if constexpr (kPLo) mma_ts(tmem + kColO, tmem + col + 16u, mndesc(aV, j), idPV, 1u);
        }
        if constexpr (MODE == kScanRevCol) {
          if (args.vec_mma) {
            // MMA-W: sum over the chunk's tokens of v'_t add_t, one N=16 slot per
            // chunk parity (columns 0 and 1: the hi and lo parts of add)
            const uint32_t slot = tmem + kColZ + 16u * ((uint32_t)i & 1u);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              mma_ss(slot, mndesc(aV, j),
                     smem_desc_sw128(aM0 + 768u + (uint32_t)((j >> 2) * 1024 + (j & 3) * 32), 16, kSmallSbo),
                     idK1, j > 0 ? 1u : 0u);
          }
        }
        mma_commit(&bars[kBarO]);
        if constexpr (!kStageInV && !kSplitV) mma_commit(&bars[kEmpty0 + st]);
      }
      if (!ok) {
        report_status(args.status, FAKLA_ERR_TIMEOUT);
        *abort_flag = 1;
        if (issued_any) {
          // Drain the MMAs in flight before TMEM and smem are released.
          mma_commit(&bars[kDrain]);
          (void)bar_wait(&bars[kDrain], 0, kWaitNs);
        }
      }
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------------- P: mask + split
    const int q4 = warp & 3;
    const int r = 32 * q4 + lane;  // token r of the chunk
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q4) << 16);
    bool ok = true;
    constexpr bool kCol = MODE == kScanRevCol;
    // kScanRevCol's four P warps share the column terms through shared memory
    // and stop together (a named barrier that ORs their wait results; every
    // wait before it is bounded).
    for (int i = 0; i < nch && (kCol || !warp_aborted(abort_flag)); ++i) {
      const uint32_t par = (uint32_t)i & 1u;
      // the per-row / per-column terms, loaded before the wait so that their
      // latency overlaps it
      const int t0 = chunk_t0(i);
      const float arow = MODE == kScanRowAdd ? add_at(args.add, b, args.T, args.H, h, t0 + r) : 0.f;
      const float bval = kCol ? add_at(args.add, b, args.T, args.H, h, t0 + r) : 0.f;
      ok = warp_wait(&bars[kBarP], par);
      if constexpr (kCol) {
        if (named_barrier_or(2, 128, !ok || *abort_flag != 0)) break;
        bcol_sm[r] = bval;  // the previous chunk's readers passed the barrier above
        if (args.vec_mma) {
          // the column terms as the B operand of MMA-W: bf16 hi in row 6, lo in
          // row 7 of M0 (tokens 0-63) and M1 (tokens 64-127); MMA-W of the
          // previous chunk completed before barP
          const __nv_bfloat16 bh16 = __float2bfloat16_rn(bval);
          const __nv_bfloat16 bl16 = __float2bfloat16_rn(bval - __bfloat162float(bh16));
          uint8_t* blk = sM0 + (r >= 64 ? 1024 : 0);
          *reinterpret_cast<__nv_bfloat16*>(blk + sw128_offset(6, (uint32_t)(r & 63))) = bh16;
          *reinterpret_cast<__nv_bfloat16*>(blk + sw128_offset(7, (uint32_t)(r & 63))) = bl16;
          fence_proxy_async_smem();
        }
        named_barrier_sync(2, 128);
      } else if (!ok) {
        break;
      }
      tc_fence_after();
      // Token groups of 32: this warp's rows are group q4, so group g is
      // whole, diagonal or empty for every lane (causal: whole below the
      // diagonal; reversed: whole above it).
      const uint32_t p_addr = lane_addr + kColP;
      float rs = 0.f;
#pragma unroll 1
      for (int g0 = 0; g0 < 4; g0 += 2) {
        const bool k0 = kRev ? g0 >= q4 : g0 <= q4;
        const bool k1 = kRev ? g0 + 1 >= q4 : g0 + 1 <= q4;
        if (!k0 && !k1) {
          zero_group(g0, p_addr);
          zero_group(g0 + 1, p_addr);
          continue;
        }
        uint32_t va[32], vb[32];
        if (k0) tmem_ld32(p_addr + (uint32_t)(32 * g0), va);
        if (k1) tmem_ld32(p_addr + (uint32_t)(32 * g0 + 32), vb);
        tmem_ld_wait();
        if (k0)
          rs += split_group_at<kRev, kCol, MODE == kScanRowAdd, kPLo>(va, g0, q4, r, p_addr, arow, bcol_sm + 32 * g0);
        else
          zero_group(g0, p_addr);
        if (k1)
          rs += split_group_at<kRev, kCol, MODE == kScanRowAdd, kPLo>(vb, g0 + 1, q4, r, p_addr, arow, bcol_sm + 32 * g0 + 32);
        else
          zero_group(g0 + 1, p_addr);
      }
      tmem_st1(lane_addr + kColRs + par, __float_as_uint(rs));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kE1Done]);
    }
    if (!ok) {
      report_status(args.status, FAKLA_ERR_TIMEOUT);
      *abort_flag = 1;
    }
  } else if (warp < 10) {
    // ---------------------------------------------------------------- S: state refresh
    const int q4 = warp & 3;
    const int r = 32 * q4 + lane;  // feature r
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q4) << 16);
    const int64_t bh = (int64_t)b * args.H + h;
    {
      // initial state: the segment's record, else the caller's state (by rows,
      // or transposed: column r), else 0
      const float* srow = nullptr;
      const float* scol = nullptr;
      int srow_len = D;  // columns of srow (the caller's S of a 64-wide head has 64)
      float z0 = 0.f;
      if (args.seg_init != nullptr) {
        const float* rec = args.seg_init + (bh * args.G + seg) * kStateFloats;
        srow = rec + (int64_t)r * D;
        z0 = rec[(int64_t)D * D + r];
      } else if ((args.flags & FAKLA_STATE_IN) && args.S != nullptr && r < args.hd) {
        const int hd = args.hd;
        if (args.state_in_T)
          scol = args.S + bh * hd * hd + r;
        else
          srow = args.S + (bh * hd + r) * hd;
        srow_len = hd;
        if (!kRaw) z0 = args.z[bh * hd + r];
      }
      // 32 values per round trip to global memory (the loads of a piece are
      // all issued before any is used): this load sits on the first chunk's
      // path to MMA2, which short segments feel
#pragma unroll 1
      for (int c32 = 0; c32 < D; c32 += 32) {
        float f[32];
        if (srow != nullptr && c32 < srow_len) {
          // srow_len is 128 or 64, so a 32-wide piece is whole
          const float4* s4 = reinterpret_cast<const float4*>(srow + c32);
          float4 x[8];
#pragma unroll
          for (int g = 0; g < 8; ++g) x[g] = s4[g];
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            f[4 * g] = x[g].x;
            f[4 * g + 1] = x[g].y;
            f[4 * g + 2] = x[g].z;
            f[4 * g + 3] = x[g].w;
          }
        } else if (scol != nullptr) {
#pragma unroll
          for (int e = 0; e < 32; ++e) f[e] = c32 + e < srow_len ? scol[(int64_t)(c32 + e) * srow_len] : 0.f;
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) f[e] = 0.f;
        }
#pragma unroll
        for (int h16 = 0; h16 < 32; h16 += 16) {
          const int cc = c32 + h16;
          uint32_t v[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = __float_as_uint(f[h16 + e]);
          tmem_st16(lane_addr + kColS + (uint32_t)cc, v);
          put_sb8<kRaw>(sSb, sSbLo, r, cc, f + h16);
          put_sb8<kRaw>(sSb, sSbLo, r, cc + 8, f + h16 + 8);
        }
      }
      if constexpr (kZ) {
        tmem_st1(lane_addr + kColZ, __float_as_uint(z0));
        put_zk(sM0, r, z0);
      }
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kSReady]);
    }
    // With temp, these warps also turn the K tile of chunk j into k~ = k temp
    // (row r each) before MMA1 reads it: between two state refreshes, while
    // the P warps split the previous chunk, so it stays off the chunk's
    // critical path.
    auto scale_k = [&](int j) {
      const int st = j & 1;
      if (!warp_wait(&bars[kFull0 + st], (uint32_t)(j >> 1) & 1u)) return false;
      scale_k_row(sK + st * kTile, r, temp_at(args.temp, b, args.T, args.H, h, chunk_t0(j) + r));
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kKReady]);
      return true;
    };
    const bool write_state = last_seg && (args.flags & FAKLA_STATE_OUT) && args.S != nullptr;
    bool ok = true;
    if (has_temp && nch > 0) ok = scale_k(0);
    for (int i = 0; ok && i < nch && !warp_aborted(abort_flag); ++i) {
      ok = warp_wait(&bars[kBarS], (uint32_t)i & 1u);
      if (!ok) break;
      tc_fence_after();
      const bool sout = write_state && i == nch - 1;
#pragma unroll 1
      for (int cc = 0; cc < D; cc += 32) {
        uint32_t v[32];
        tmem_ld32(lane_addr + kColS + (uint32_t)cc, v);
        tmem_ld_wait();
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float f8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f8[e] = __uint_as_float(v[8 * g + e]);
          put_sb8<kRaw>(sSb, sSbLo, r, cc + 8 * g, f8);
        }
        if (sout && r < args.hd && cc < args.hd) {
          float4* dst = reinterpret_cast<float4*>(args.S + (bh * args.hd + r) * args.hd + cc);
#pragma unroll
          for (int g = 0; g < 8; ++g)
            dst[g] = make_float4(__uint_as_float(v[4 * g]), __uint_as_float(v[4 * g + 1]),
                                 __uint_as_float(v[4 * g + 2]), __uint_as_float(v[4 * g + 3]));
        }
      }
      if constexpr (kZ) {
        uint32_t zraw;
        tmem_ld1(lane_addr + kColZ, zraw);
        tmem_ld_wait();
        const float zf = __uint_as_float(zraw);
        put_zk(sM0, r, zf);
        if (!kRaw && sout && r < args.hd) args.z[bh * args.hd + r] = zf;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kSReady]);
      if (has_temp && i + 1 < nch) ok = scale_k(i + 1);
      if (split_o && ok) {
        // columns 64-127 of chunk i's output rows 32 q4 + lane (TMEM lane r)
        const uint32_t par = (uint32_t)i & 1u;
        ok = warp_wait(&bars[kBarO], par);
        if (!ok) break;
        tc_fence_after();
        uint32_t dz0, dz1, rsr;
        tmem_ld2(lane_addr + kColDz, dz0, dz1);
        tmem_ld1(lane_addr + kColRs + par, rsr);
        uint32_t va[32], vb[32];
        tmem_ld32(lane_addr + kColO + 64u, va);
        tmem_ld32(lane_addr + kColO + 96u, vb);
        tmem_ld_wait();
        const float inv =
            1.f / (__uint_as_float(rsr) + (__uint_as_float(dz0) + __uint_as_float(dz1)) + kEps);
        uint8_t* stg = sV + (i & 1) * kTile;  // the chunk's V tile, read by MMA4 and MMA3 before barO
        stage_scaled_32(va, inv, stg, r, 64);
        stage_scaled_32(vb, inv, stg, r, 96);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kOFree]);  // O may be overwritten now
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const int t0 = chunk_t0(i) + 32 * q4;
          if (t0 < args.T) {
            tma_store_4d(&tmO, stg + kAtom + q4 * (32 * 128), 64, h, t0, b);
            bulk_commit_group();
            bulk_wait_group_read<0>();
          }
          mbar_arrive(&bars[kEmpty0 + (i & 1)]);  // the V tile may be refilled
        }
        __syncwarp();
      }
    }
    if (split_o && lane == 0) bulk_wait_group<0>();  // output stores complete before the CTA exits
    if (!ok) {
      report_status(args.status, FAKLA_ERR_TIMEOUT);
      *abort_flag = 1;
    }
  } else {
    // ---------------------------------------------------------------- O: normalise + store
    const int q4 = warp & 3;
    const int r = 32 * q4 + lane;  // token r of the chunk
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q4) << 16);
    // The affine modes' four output warps share the chunk's vector (and the
    // centring vector) through shared memory and stop together (a named
    // barrier that ORs their wait results; every wait before it is bounded).
    const bool centre = MODE == kScanRowAdd && args.mvec != nullptr;
    // running chunk vector of the affine modes (feature r)
    float run = (kAffine && r < args.hd && args.vec_init != nullptr)
                    ? args.vec_init[(int64_t)bh_idx * args.hd + r] : 0.f;
    bool ok = true;
    int done = 0;
    for (int i = 0; i < nch && (kAffine || !warp_aborted(abort_flag)); ++i) {
      const uint32_t par = (uint32_t)i & 1u;
      const int t_tok = chunk_t0(i) + r;
      const int st = i & 1;
      const bool live = t_tok < args.T;
      const int64_t row = ((int64_t)b * args.T + (live ? t_tok : 0)) * args.H + h;
      const bool row_tile = kGrad || (MODE == kScanRevCol && args.dot_out != nullptr);
      bool wok = true;  // this warp's waits of the chunk
      if (kRowTile && row_tile) {
        // this warp's 32 rows of the row tensor into the Q tile, whose MMA
        // readers (MMA1, MMA2, MMA2b) completed with barS
        wok = warp_wait(&bars[kBarS], par);
        if (wok && lane == 0) {
          uint64_t* rb = &bars[kRow0 + q4];
          mbar_arrive_expect_tx(rb, na * 32 * 64 * 2);
          for (int a = 0; a < na; ++a)
            tma_load_4d(sQ + st * kTile + a * kAtom + q4 * (32 * 128), &tmR, rb, a * 64, h,
                        chunk_t0(i) + 32 * q4, b);
        }
      }
      // the chunk's vector and per-row scalars of the affine epilogues, loaded
      // before the wait so that their latency overlaps MMA3
      float vval = 0.f, coef = 0.f, scale = 1.f;
      if (kAffine) {
        vval = run;
        if (!args.vec_mma && r < args.hd)
          run += args.vec[((int64_t)bh_idx * nchunks_total + chunk_t0(i) / C) * args.hd + r];
        coef = MODE == kScanRowAdd ? (live ? args.add[row] : 0.f) : 1.f;
        if (args.row_scale != nullptr && live) scale = __bfloat162float(args.row_scale[row]);
      }
      if (wok) wok = warp_wait(&bars[kBarO], par);
      if (wok && kRowTile && row_tile) wok = warp_wait(&bars[kRow0 + q4], par);
      if constexpr (kAffine) {
        if (named_barrier_or(1, 128, !wok || *abort_flag != 0)) {
          ok = wok;
          break;
        }
        if (MODE == kScanRevCol && args.vec_mma) {
          // this chunk's sum (MMA-W, complete with barO) joins the running
          // vector after this chunk's own value was taken
          tc_fence_after();
          uint32_t w0, w1;
          tmem_ld2(lane_addr + kColZ + 16u * ((uint32_t)i & 1u), w0, w1);
          tmem_ld_wait();
          run += __uint_as_float(w0) + __uint_as_float(w1);
        }
        vec_sm[r] = vval;  // the previous chunk's readers passed the barrier above
        named_barrier_sync(1, 128);
      } else if (!wok) {
        ok = false;
        break;
      }
      tc_fence_after();
      float inv = 1.f;
      if constexpr (!kRaw) {
        uint32_t dz0, dz1, rsr;
        tmem_ld2(lane_addr + kColDz, dz0, dz1);
        tmem_ld1(lane_addr + kColRs + par, rsr);
        tmem_ld_wait();
        const float den = __uint_as_float(rsr) + (__uint_as_float(dz0) + __uint_as_float(dz1)) + kEps;
        inv = 1.f / den;
        if (args.den_out != nullptr && live)
          args.den_out[((int64_t)b * args.T + t_tok) * args.H + h] = den;
      }
      // Stage the normalised rows in this chunk's Q tile (its last readers,
      // MMA1/MMA2/MMA2b, completed before barO), or in its V tile (MMA4 and
      // MMA3, the last readers, completed with barO) ...
      uint8_t* stg = (kStageInV || kSplitV ? sV : sQ) + st * kTile;
      const uint8_t* rtile = sQ + st * kTile;
      if constexpr (kGrad) {
        // backward's forward pass: dden = -(bf16(g / den) . out), out in fp32;
        // the output rows are dnum = bf16(g / den) (stored when asked for),
        // written over g in the row tile that the store below reads
        float acc = 0.f;
#pragma unroll 1
        for (int cc = 0; cc < args.hd; cc += 64) {
          uint4 rh[8];
          load_row_smem(rtile, r, cc, rh);
          uint32_t va[32], vb[32];
          tmem_ld32(lane_addr + kColO + (uint32_t)cc, va);
          tmem_ld32(lane_addr + kColO + (uint32_t)(cc + 32), vb);
          tmem_ld_wait();
          acc += dden_dot_32(va, inv, rh);
          acc += dden_dot_32(vb, inv, rh + 4);
          if (args.dnum_store) store_row_smem(stg, r, cc, rh);
        }
        if (live) args.dden_out[row] = -acc;
      } else if (!kAffine) {
#pragma unroll 1
        for (int cc = 0; cc < (split_o ? 64 : args.hd); cc += 64) {
          uint32_t va[32], vb[32];
          tmem_ld32(lane_addr + kColO + (uint32_t)cc, va);
          tmem_ld32(lane_addr + kColO + (uint32_t)(cc + 32), vb);
          tmem_ld_wait();
          stage_scaled_32(va, inv, stg, r, cc);
          stage_scaled_32(vb, inv, stg, r, cc + 32);
        }
      } else if constexpr (kAffine) {
        // centring (kScanRowAdd): sigma = sum of this row's kept q'.k' + term
        // over every chunk so far = rs (this chunk) + q'.z (earlier chunks)
        float sig = 0.f;
        if constexpr (kZ) {
          uint32_t dz0, dz1, rsr;
          tmem_ld2(lane_addr + kColDz, dz0, dz1);
          tmem_ld1(lane_addr + kColRs + par, rsr);
          tmem_ld_wait();
          sig = __uint_as_float(rsr) + (__uint_as_float(dz0) + __uint_as_float(dz1));
        }
        if (!centre) sig = 0.f;
        constexpr bool kDot = MODE == kScanRevCol;
        float acc = 0.f;
#pragma unroll 1
        for (int cc = 0; cc < args.hd; cc += 64) {
          uint4 rh[8];
          if (kDot && row_tile) load_row_smem(rtile, r, cc, rh);
          uint32_t va[32], vb[32];
          tmem_ld32(lane_addr + kColO + (uint32_t)cc, va);
          tmem_ld32(lane_addr + kColO + (uint32_t)(cc + 32), vb);
          tmem_ld_wait();
          const float* mv = cc < 64 ? mlo_sm + cc : mhi_sm + (cc - 64);
          if (kDot && row_tile) {
            acc += stage_affine_32<true, kZ>(va, coef, vec_sm + cc, sig, mv, scale, rh, stg, r, cc);
            acc += stage_affine_32<true, kZ>(vb, coef, vec_sm + cc + 32, sig, mv + 32, scale, rh + 4, stg, r, cc + 32);
          } else {
            stage_affine_32<false, kZ>(va, coef, vec_sm + cc, sig, mv, scale, rh, stg, r, cc);
            stage_affine_32<false, kZ>(vb, coef, vec_sm + cc + 32, sig, mv + 32, scale, rh + 4, stg, r, cc + 32);
          }
        }
        if (kDot && row_tile && live) args.dot_out[row] = __float2bfloat16_rn(acc);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kOFree]);  // O may be overwritten now
      // ... and store this warp's 32 rows with TMA (rows past T are clipped).
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int t0 = chunk_t0(i) + 32 * q4;
        if (t0 < args.T && (!kGrad || args.dnum_store)) {
          for (int a = 0; a < (split_o ? 1 : na); ++a)
            tma_store_4d(&tmO, stg + a * kAtom + q4 * (32 * 128), a * 64, h, t0, b);
          bulk_commit_group();
          bulk_wait_group_read<0>();
        }
        if (!kSplitV) mbar_arrive(&bars[kEmptyQ0 + st]);  // the Q tile may be refilled
        if (kStageInV || kSplitV) mbar_arrive(&bars[kEmpty0 + st]);  // ... the V tile
      }
      __syncwarp();
      ++done;
    }
    // every chunk walked: the vector's total
    if (kAffine && done == nch && args.vec_total != nullptr && r < args.hd)
      args.vec_total[(int64_t)bh_idx * args.hd + r] = run;
    if (lane == 0) bulk_wait_group<0>();  // output stores complete before the CTA exits
    if (!ok) {
      report_status(args.status, FAKLA_ERR_TIMEOUT);
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Segment sums: for segment g < G-1 of sequence (b, h), dS = sum K~^T V and
// dz = sum K~ over its chunks, written to record g+1 of the sequence.
// ---------------------------------------------------------------------------
constexpr int kDStages = 3;
constexpr int kDThreads = 192;
constexpr int kDTile = 2 * kTile;  // K and V of one chunk: 64 KB
constexpr size_t kDOffOnes = 0;    // 1 KB block, rows 0-1 all 1.0
constexpr size_t kDOffStages = 1024;
constexpr size_t kDOperandBytes = kDOffStages + kDStages * kDTile;
constexpr size_t kDSmemBytes = kHeadBytes + 1024 + kDOperandBytes;

// One k*temp barrier per stage: the scaling warps may run up to three chunks
// ahead of the MMA warp, more than one barrier's two-phase parity can tell.
enum DBar {
  kDFull0 = 0,
  kDEmpty0 = kDFull0 + kDStages,
  kDKReady0 = kDEmpty0 + kDStages,
  kDDone = kDKReady0 + kDStages,
  kDNumBars
};
static_assert(kDNumBars * 8 + 8 <= kHeadBytes, "barrier area");

struct DeltaArgs {
  const __nv_bfloat16* temp;
  float* seg_init;  // (B*H, G) records
  int T, H, G, seg_chunks;
  int* status;
  int hd;  // 128, or 64 (second atom of each tile held at zero)
};

__global__ void __launch_bounds__(kDThreads, 1) scan_delta_sm100_kernel(
    const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
    const DeltaArgs args) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kDNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* smem = operand_base(smem_raw);
  if (smem + kDOperandBytes > smem_raw + kDSmemBytes) {
    if (threadIdx.x == 0) report_status(args.status, FAKLA_ERR_ALIGNMENT);
    return;
  }
  uint8_t* sOnes = smem + kDOffOnes;
  uint8_t* sSt = smem + kDOffStages;  // stage s: K at s*kDTile, V at s*kDTile + kTile

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int per = args.G - 1;
  const int bh_idx = blockIdx.x / per;
  const int seg = blockIdx.x % per;
  const int b = bh_idx / args.H;
  const int h = bh_idx % args.H;
  const int c0 = seg * args.seg_chunks;
  const int nch = args.seg_chunks;  // segments before the last are full
  const bool has_temp = args.temp != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDStages; ++s) {
      mbar_init(&bars[kDFull0 + s], 1);
      mbar_init(&bars[kDEmpty0 + s], 1);
      mbar_init(&bars[kDKReady0 + s], 4);
    }
    mbar_init(&bars[kDDone], 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (threadIdx.x < 64) reinterpret_cast<uint32_t*>(sOnes)[threadIdx.x] = 0x3F803F80u;
  const int na = args.hd == 64 ? 1 : 2;  // 64-column atoms loaded per tile
  if (na == 1) {
    constexpr int kPer = kAtom / 16;
    for (int o = threadIdx.x; o < 2 * kDStages * kPer; o += kDThreads) {
      const int t = o / kPer;  // K and V tile of each stage
      uint8_t* base = sSt + (t >> 1) * kDTile + (t & 1) * kTile + kAtom;
      reinterpret_cast<uint4*>(base)[o % kPer] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t kDColS = 0, kDColZ = 128;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nch && !*abort_flag; ++i) {
        const int st = i % kDStages;
        const uint32_t ph = (uint32_t)(i / kDStages) & 1u;
        if (!bar_wait(&bars[kDEmpty0 + st], ph ^ 1u, kWaitNs)) {
          report_status(args.status, FAKLA_ERR_TIMEOUT);
          *abort_flag = 1;
          break;
        }
        uint64_t* fb = &bars[kDFull0 + st];
        mbar_arrive_expect_tx(fb, 2 * na * kAtom);
        const int t0 = (c0 + i) * C;
        uint8_t* tk = sSt + st * kDTile;
        for (int a = 0; a < na; ++a) {
          tma_load_4d(tk + a * kAtom, &tmK, fb, a * 64, h, t0, b);
          tma_load_4d(tk + kTile + a * kAtom, &tmV, fb, a * 64, h, t0, b);
        }
        ++issued;
      }
      if (*abort_flag) {
        for (int i = issued - kDStages; i < issued; ++i)
          if (i >= 0)
            (void)bar_wait(&bars[kDFull0 + i % kDStages], (uint32_t)(i / kDStages) & 1u, kWaitNs);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idKV = idesc_bf16_f32(128, 128, true, true);
      constexpr uint32_t idK1 = idesc_bf16_f32(128, 16, true, false);
      const uint32_t aOnes = smem_u32(sOnes);
      bool ok = true;
      bool issued_any = false;
      for (int i = 0; i < nch && ok && !*abort_flag; ++i) {
        const int st = i % kDStages;
        const uint32_t ph = (uint32_t)(i / kDStages) & 1u;
        ok = bar_wait(&bars[kDFull0 + st], ph, kWaitNs);
        if (ok && has_temp) ok = bar_wait(&bars[kDKReady0 + st], ph, kWaitNs);
        if (!ok) break;
        tc_fence_after();
        issued_any = true;
        const uint32_t aK = smem_u32(sSt + st * kDTile);
        const uint32_t aV = aK + kTile;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          mma_ss(tmem + kDColS, mndesc(aK, j), mndesc(aV, j), idKV, (i > 0 || j > 0) ? 1u : 0u);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          // ONES: rows 0 and 1 of the block are row 0 of atoms 0 and 1.
          const uint64_t ones = smem_desc_sw128(aOnes + (uint32_t)((j >> 2) * 128 + (j & 3) * 32), 16, 1024);
          mma_ss(tmem + kDColZ, mndesc(aK, j), ones, idK1, (i > 0 || j > 0) ? 1u : 0u);
        }
        mma_commit(&bars[kDEmpty0 + st]);
      }
      if (!ok) {
        report_status(args.status, FAKLA_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      // Completion of everything issued (also the drain on the error path).
      if (issued_any) mma_commit(&bars[kDDone]);
      else mbar_arrive(&bars[kDDone]);
    }
  } else {
    const int q4 = warp & 3;
    const int r = 32 * q4 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q4) << 16);
    bool ok = true;
    if (has_temp) {
      for (int i = 0; i < nch && !warp_aborted(abort_flag); ++i) {
        const int st = i % kDStages;
        ok = warp_wait(&bars[kDFull0 + st], (uint32_t)(i / kDStages) & 1u);
        if (!ok) break;
        scale_k_row(sSt + st * kDTile, r, temp_at(args.temp, b, args.T, args.H, h, (c0 + i) * C + r));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kDKReady0 + st]);
      }
    }
    if (ok) ok = warp_wait(&bars[kDDone], 0);
    if (ok && !warp_aborted(abort_flag)) {
      tc_fence_after();
      const int64_t bh = (int64_t)b * args.H + h;
      float* rec = args.seg_init + (bh * args.G + seg + 1) * kStateFloats;
      float* srow = rec + (int64_t)r * D;
#pragma unroll 1
      for (int cc = 0; cc < D; cc += 32) {
        uint32_t v[32];
        tmem_ld32(lane_addr + kDColS + (uint32_t)cc, v);
        tmem_ld_wait();
        float4* dst = reinterpret_cast<float4*>(srow + cc);
#pragma unroll
        for (int g = 0; g < 8; ++g)
          dst[g] = make_float4(__uint_as_float(v[4 * g]), __uint_as_float(v[4 * g + 1]),
                               __uint_as_float(v[4 * g + 2]), __uint_as_float(v[4 * g + 3]));
      }
      uint32_t zraw;
      tmem_ld1(lane_addr + kDColZ, zraw);
      tmem_ld_wait();
      rec[(int64_t)D * D + r] = __uint_as_float(zraw);
    }
    if (!ok) {
      report_status(args.status, FAKLA_ERR_TIMEOUT);
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// Record 0 of each sequence <- the caller's initial state (or 0); record g <-
// record g-1 + the segment sum stored in record g. One thread per float4 of
// a record (coalesced across threads), running over the G records with the
// loads of 8 records in flight at once: the kernel is latency-bound, and one
// dependent load per record cost a round trip each.
__global__ void scan_prefix_kernel(float* seg_init, const float* S_in, const float* z_in, int G,
                                   int state_in, int hd) {
  constexpr int kS4 = D * D / 4;
  constexpr int kRec4 = (int)(kStateFloats / 4);
  griddep_wait();
  griddep_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= kRec4) return;
  const int64_t bh = blockIdx.y;
  float4* rec = reinterpret_cast<float4*>(seg_init + bh * G * kStateFloats);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (state_in) {
    // the caller's state is hd x hd (+ hd); records are D x D (+ D), zero-padded
    if (i < kS4) {
      const int f = (4 * i) / D, d = (4 * i) % D;
      if (f < hd && d < hd)
        acc = *reinterpret_cast<const float4*>(S_in + (bh * hd + f) * hd + d);
    } else {
      const int f = 4 * (i - kS4);
      if (f < hd) {
        const float* zp = z_in + bh * hd + f;
        acc = make_float4(zp[0], zp[1], zp[2], zp[3]);
      }
    }
  }
  rec[i] = acc;
  constexpr int kBatch = 8;
  for (int g0 = 1; g0 < G; g0 += kBatch) {
    float4 d[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
      if (g0 + j < G) d[j] = rec[(int64_t)(g0 + j) * kRec4 + i];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (g0 + j < G) {
        acc.x += d[j].x;
        acc.y += d[j].y;
        acc.z += d[j].z;
        acc.w += d[j].w;
        rec[(int64_t)(g0 + j) * kRec4 + i] = acc;
      }
    }
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static bool make_map_bthd(CUtensorMap* map, const void* base, int64_t B, int64_t T, int64_t H,
                          int box_t = C, int64_t row_elems = 0, int64_t hd = D) {
  // (B, T, H, hd) bf16 viewed as 4-D {d, h, t, b}; box = 64 d x 1 h x box_t t x 1 b.
  // row_elems: elements from one token's row to the next (H * hd when dense;
  // larger for a column block of a wider row, e.g. the q/k/v GEMM output).
  const int64_t re = row_elems > 0 ? row_elems : H * hd;
  const cuuint64_t dims[4] = {(cuuint64_t)hd, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)hd * 2, (cuuint64_t)re * 2, (cuuint64_t)T * re * 2};
  const cuuint32_t box[4] = {64, 1, (cuuint32_t)box_t, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return encode_tensor_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base),
                           dims, strides, box, estr, CU_TENSOR_MAP_SWIZZLE_128B);
}

bool scan_sm100_supported(int64_t B, int64_t T, int64_t H, int64_t Df, int64_t Dv) {
  return Df == Dv && (Df == D || Df == 64) && B >= 1 && T >= 1 && H >= 1 &&
         B * H <= (int64_t)(INT32_MAX / 256) && T <= (int64_t)INT32_MAX - C;
}

int scan_sm100_segments(int64_t B, int64_t T, int64_t H, int sms) {
  const int64_t bh = B * H;
  const int64_t nchunks = (T + C - 1) / C;
  if (bh * 4 >= (int64_t)sms * 3) return 1;  // three quarters of the SMs busy already
  int64_t G = sms / bh;
  if (G > nchunks / 2) G = nchunks / 2;  // segments of at least two chunks
  if (G < 2) return 1;
  const int64_t seg = (nchunks + G - 1) / G;
  return (int)((nchunks + seg - 1) / seg);
}

size_t scan_sm100_workspace_bytes(int64_t B, int64_t T, int64_t H, int sms) {
  const int G = scan_sm100_segments(B, T, H, sms);
  if (G <= 1) return 0;
  return (size_t)(B * H) * (size_t)G * (size_t)kStateFloats * sizeof(float);
}

template <int MODE>
static cudaError_t launch_main(const CUtensorMap& mQ, const CUtensorMap& mK, const CUtensorMap& mV,
                               const CUtensorMap& mO, const CUtensorMap& mR, const ScanArgs& a,
                               int64_t ctas, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(scan_sm100_kernel<MODE>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  return launch_chained(scan_sm100_kernel<MODE>, dim3((unsigned)ctas), dim3(kThreads), kSmemBytes, stream, 1u,
                        mQ, mK, mV, mO, mR, a);
}

static cudaError_t launch_scan_impl(const void* q, const void* k, const void* v, const void* temp,
                                    void* out, float* S, float* z, int64_t B, int64_t T, int64_t H,
                                    unsigned flags, const ScanBackwardArgs* m, void* workspace,
                                    size_t workspace_bytes, int sms, cudaStream_t stream, int* status,
                                    bool* encoded, int64_t in_row_elems, int64_t hd) {
  int mode = m != nullptr ? m->mode : kScanNormal;
  if (mode < kScanNormal || mode > kScanRevCol || (mode != kScanNormal && temp != nullptr) ||
      (hd != D && hd != 64) ||
      (mode == kScanNormal && m != nullptr && m->grad_rows != nullptr && m->dden_out == nullptr) ||
      ((mode == kScanRowAdd || mode == kScanRevCol) && m->add == nullptr) ||
      ((mode == kScanRowAdd || mode == kScanRevCol) && m->vec == nullptr && !(mode == kScanRevCol && m->vec_mma))) {
    *encoded = true;
    return cudaErrorInvalidValue;
  }
  if (mode == kScanNormal && m != nullptr && m->grad_rows != nullptr) mode = kScanNormalGrad;
  // The epilogue's row tensor: the output gradient (no output rows are
  // stored then) or the dot rows of mode 3.
  const void* rows = mode == kScanNormalGrad ? m->grad_rows
                     : (mode == kScanRevCol && m->dot_out != nullptr ? m->dot_rows : nullptr);
  if (mode == kScanNormalGrad && m->dnum_out == nullptr) out = const_cast<void*>(rows);
  if (mode == kScanNormalGrad && m->dnum_out != nullptr) out = m->dnum_out;
  CUtensorMap mQ, mK, mV, mO, mR;
  const bool ok = make_map_bthd(&mQ, q, B, T, H, C, in_row_elems, hd) &&
                  make_map_bthd(&mK, k, B, T, H, C, in_row_elems, hd) &&
                  make_map_bthd(&mV, v, B, T, H, C, in_row_elems, hd) &&
                  make_map_bthd(&mO, out, B, T, H, 32, 0, hd) &&
                  make_map_bthd(&mR, rows != nullptr ? rows : out, B, T, H, 32, 0, hd);
  *encoded = ok;
  if (!ok) return cudaErrorInvalidValue;
  const int64_t nchunks = (T + C - 1) / C;
  int G = (mode == kScanNormal || mode == kScanNormalGrad) ? scan_sm100_segments(B, T, H, sms) : 1;
  const size_t need = scan_sm100_workspace_bytes(B, T, H, sms);
  // Without room for the segment records the scan runs one CTA per sequence.
  if (G > 1 && (workspace == nullptr || workspace_bytes < need ||
                (reinterpret_cast<uintptr_t>(workspace) & 15u) != 0))
    G = 1;
  const int seg_chunks = (int)((nchunks + G - 1) / G);
  float* seg_init = G > 1 ? static_cast<float*>(workspace) : nullptr;
  const bool state_in = (flags & FAKLA_STATE_IN) && S != nullptr;

  if (G > 1) {
    DeltaArgs d;
    d.temp = (const __nv_bfloat16*)temp;
    d.seg_init = seg_init;
    d.T = (int)T;
    d.H = (int)H;
    d.G = G;
    d.seg_chunks = seg_chunks;
    d.hd = (int)hd;
    d.status = status;
    cudaError_t e = cudaFuncSetAttribute(scan_delta_sm100_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kDSmemBytes);
    if (e != cudaSuccess) return e;
    e = launch_chained(scan_delta_sm100_kernel, dim3((unsigned)(B * H * (G - 1))), dim3(kDThreads), kDSmemBytes,
                       stream, 1u, mK, mV, d);
    if (e != cudaSuccess) return e;
    const dim3 pgrid((unsigned)((kStateFloats / 4 + 255) / 256), (unsigned)(B * H));
    e = launch_chained(scan_prefix_kernel, pgrid, dim3(256), 0, stream, 1u, seg_init, (const float*)S,
                       (const float*)z, G, state_in ? 1 : 0, (int)hd);
    if (e != cudaSuccess) return e;
  }

  ScanArgs a;
  a.temp = (const __nv_bfloat16*)temp;
  a.S = S;
  a.z = z;
  a.seg_init = seg_init;
  a.T = (int)T;
  a.H = (int)H;
  a.G = G;
  a.seg_chunks = seg_chunks;
  a.flags = flags;
  a.status = status;
  a.hd = (int)hd;
  a.add = m ? m->add : nullptr;
  a.den_out = m ? m->den_out : nullptr;
  a.state_in_T = m ? m->state_in_T : 0;
  a.vec = m ? m->vec : nullptr;
  a.row_scale = m ? static_cast<const __nv_bfloat16*>(m->row_scale) : nullptr;
  a.dot_rows = m ? static_cast<const __nv_bfloat16*>(m->dot_rows) : nullptr;
  a.dot_out = m ? static_cast<__nv_bfloat16*>(m->dot_out) : nullptr;
  a.grad_rows = m ? static_cast<const __nv_bfloat16*>(m->grad_rows) : nullptr;
  a.dnum_store = (m != nullptr && m->dnum_out != nullptr) ? 1 : 0;
  a.mvec = m ? m->mvec : nullptr;
  a.vec_init = m ? m->vec_init : nullptr;
  a.vec_total = m ? m->vec_total : nullptr;
  a.vec_mma = (m != nullptr && m->vec_mma) ? 1 : 0;
  a.dden_out = m ? m->dden_out : nullptr;
  const int64_t ctas = B * H * G;
  switch (mode) {
    case kScanRowAdd: return launch_main<kScanRowAdd>(mQ, mK, mV, mO, mR, a, ctas, stream);
    case kScanRevRaw: return launch_main<kScanRevRaw>(mQ, mK, mV, mO, mR, a, ctas, stream);
    case kScanRevCol: return launch_main<kScanRevCol>(mQ, mK, mV, mO, mR, a, ctas, stream);
    case kScanNormalGrad: return launch_main<kScanNormalGrad>(mQ, mK, mV, mO, mR, a, ctas, stream);
    default: return launch_main<kScanNormal>(mQ, mK, mV, mO, mR, a, ctas, stream);
  }
}

cudaError_t launch_scan_sm100(const void* q, const void* k, const void* v, const void* temp,
                              void* out, float* S, float* z, int64_t B, int64_t T, int64_t H,
                              unsigned flags, void* workspace, size_t workspace_bytes, int sms,
                              cudaStream_t stream, int* status, bool* encoded, int64_t in_row_elems,
                              int64_t hd) {
  return launch_scan_impl(q, k, v, temp, out, S, z, B, T, H, flags, nullptr, workspace,
                          workspace_bytes, sms, stream, status, encoded, in_row_elems, hd);
}

cudaError_t launch_scan_sm100_mode(const void* q, const void* k, const void* v, const void* temp,
                                   void* out, float* S, float* z, int64_t B, int64_t T, int64_t H,
                                   unsigned flags, const ScanBackwardArgs& m, void* workspace,
                                   size_t workspace_bytes, int sms, cudaStream_t stream, int* status,
                                   bool* encoded, int64_t head_dim) {
  return launch_scan_impl(q, k, v, temp, out, S, z, B, T, H, flags, &m, workspace, workspace_bytes,
                          sms, stream, status, encoded, 0, head_dim);
}

}  // namespace fakla
