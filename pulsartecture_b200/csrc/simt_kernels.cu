// General-shape FA-KLA kernels on the CUDA cores (fp32 arithmetic).
//
// These serve (a) the fp32 precision mode, whose 1e-5 relative-L2 bar rules
// out bf16/tf32 tensor-core operands, and (b) bf16 shapes outside the tile set
// of the tensor-core kernels (head dims other than 128, unaligned pointers).
// The decode kernel here is the production decode path for every dtype: one
// decode step is a read-modify-write stream over the fp32 state, bound by HBM.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fakla_common.cuh"
#include "fakla_kernels.h"

namespace fakla {

// ---------------------------------------------------------------------------
// phi(x) = elu(x W^T + b) + 1, optionally times temp[row, head]: tiled fp32
// GEMM (64x64 output tile, 256 threads, 4x4 outputs per thread, K step 16).
// x: (rows, K) row-major, W: (N, K) row-major (nn.Linear weight).
// ---------------------------------------------------------------------------
namespace {
constexpr int kPhiTile = 64;
constexpr int kPhiK = 16;

template <typename T, int ACT>
__global__ void __launch_bounds__(256) phi_simt_kernel(
    const T* __restrict__ x, const T* __restrict__ W, const T* __restrict__ bias,
    const T* __restrict__ temp, T* __restrict__ out, int64_t rows, int64_t K,
    int64_t N, int64_t heads, float scale) {
  __shared__ float xs[kPhiK][kPhiTile + 4];
  __shared__ float ws[kPhiK][kPhiTile + 4];
  const int tid = threadIdx.x;
  const int64_t row0 = (int64_t)blockIdx.y * kPhiTile;
  const int64_t col0 = (int64_t)blockIdx.x * kPhiTile;
  const int tr = tid / 16, tc = tid % 16;  // 16x16 threads, 4x4 outputs each
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += kPhiK) {
    // 64 rows x 16 k per operand = 1024 elements, 4 per thread.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * 256;
      const int r = e / kPhiK, kk = e % kPhiK;
      const int64_t gk = k0 + kk;
      const int64_t gr = row0 + r, gc = col0 + r;
      xs[kk][r] = (gr < rows && gk < K) ? to_f32(x[gr * K + gk]) : 0.f;
      ws[kk][r] = (gc < N && gk < K) ? to_f32(W[gc * K + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kPhiK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = xs[kk][tr * 4 + i];
        b[i] = ws[kk][tc * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  const int64_t m = N / heads;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gr = row0 + tr * 4 + i;
    if (gr >= rows) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gc = col0 + tc * 4 + j;
      if (gc >= N) continue;
      const float pre = acc[i][j] + (bias ? to_f32(bias[gc]) : 0.f);
      const float tv = temp ? to_f32(temp[gr * heads + gc / m]) : 1.f;
      if constexpr (ACT == FAKLA_ACT_COSSIN) {
        float sn, cs;
        sincosf(pre, &sn, &cs);
        out[gr * 2 * N + gc] = from_f32<T>(cs * scale * tv);
        out[gr * 2 * N + N + gc] = from_f32<T>(sn * scale * tv);
      } else {
        out[gr * N + gc] = from_f32<T>(activate<ACT, false>(pre) * tv);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// The same map for narrow outputs (N <= kSkinnyN, e.g. a mixer's gate logits
// over a few base maps): one warp per row, which streams the row once with
// 16-byte loads (8 elements per lane and step) and keeps the N dot products in
// registers; W (N x K) stays in L1. A 64x64 tile would leave all but N of its
// 64 columns idle and read x with short accesses.
// ---------------------------------------------------------------------------
constexpr int kSkinnyN = 16;

template <typename T>
__device__ __forceinline__ void load8_f32(const T* p, float (&f)[8]) {
  if constexpr (sizeof(T) == 2) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
}

template <typename T, int ACT, int NM>
__global__ void __launch_bounds__(256) phi_skinny_kernel(
    const T* __restrict__ x, const T* __restrict__ W, const T* __restrict__ bias,
    const T* __restrict__ temp, T* __restrict__ out, int64_t rows, int64_t K,
    int64_t N, int64_t heads, float scale) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * K;
  float acc[NM];
#pragma unroll
  for (int n = 0; n < NM; ++n) acc[n] = 0.f;
  // K % 8 == 0 and 16-byte aligned rows (checked by the launcher); two
  // 8-element pieces of the row per step, both loaded before either is used
  for (int64_t k = (int64_t)lane * 8; k < K; k += 512) {
    const bool two = k + 256 < K;
    float xv[2][8];
    load8_f32(xr + k, xv[0]);
    if (two) load8_f32(xr + k + 256, xv[1]);
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      if (h2 == 1 && !two) break;
#pragma unroll
      for (int n = 0; n < NM; ++n) {
        if (n < N) {
          float wv[8];
          load8_f32(W + n * K + k + h2 * 256, wv);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[n] = fmaf(xv[h2][e], wv[e], acc[n]);
        }
      }
    }
  }
#pragma unroll
  for (int n = 0; n < NM; ++n) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[n] += __shfl_xor_sync(0xffffffffu, acc[n], o);
  }
  // lane n writes output column n
  float pre = 0.f;
#pragma unroll
  for (int n = 0; n < NM; ++n)
    if (lane == n) pre = acc[n];
  if (lane < N) {
    const int64_t m = N / heads;
    pre += bias ? to_f32(bias[lane]) : 0.f;
    const float tv = temp ? to_f32(temp[row * heads + lane / m]) : 1.f;
    if constexpr (ACT == FAKLA_ACT_COSSIN) {
      float sn, cs;
      sincosf(pre, &sn, &cs);
      out[row * 2 * N + lane] = from_f32<T>(cs * scale * tv);
      out[row * 2 * N + N + lane] = from_f32<T>(sn * scale * tv);
    } else {
      out[row * N + lane] = from_f32<T>(activate<ACT, false>(pre) * tv);
    }
  }
}

// ---------------------------------------------------------------------------
// Causal FA-KLA scan, one CTA per (b,h) sequence, token-sequential.
// Thread (g, dv) keeps S[f][dv] for f = g, g+G, g+2G, ... in registers
// (G = 256 / Dv feature groups) and its slice of z; per token it updates its
// state and produces partial numerator/denominator sums that are reduced
// across the G groups in shared memory, kTok tokens at a time.
// Follows the recurrence of cpu_kernels.cpp:107-164 with fp32 state.
// ---------------------------------------------------------------------------
constexpr int kTok = 16;
constexpr int kScanMaxF = 64;  // features per thread (register array bound)

template <typename T>
__global__ void __launch_bounds__(256) scan_simt_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const T* __restrict__ temp, T* __restrict__ out, float* __restrict__ S,
    float* __restrict__ z, int64_t T_len, int64_t H, int Df, int Dv, unsigned flags) {
  extern __shared__ float smem[];
  float* qs = smem;                  // [kTok][Df]
  float* ks = qs + kTok * Df;        // [kTok][Df]  (k * temp)
  float* vs = ks + kTok * Df;        // [kTok][Dv]
  const int G = 256 / Dv;            // >= 1 (Dv <= 256)
  float* pn = vs + kTok * Dv;        // [kTok][G][Dv]
  float* pd = pn + kTok * G * Dv;    // [kTok][G]

  const int64_t bh = blockIdx.x;
  const int64_t b = bh / H, h = bh % H;
  const int tid = threadIdx.x;
  const int g = tid / Dv, dv = tid % Dv;
  const bool active = g < G;
  const int nf = (Df + G - 1) / G;

  float s[kScanMaxF];
  float zr[kScanMaxF];
#pragma unroll
  for (int i = 0; i < kScanMaxF; ++i) {
    s[i] = 0.f;
    zr[i] = 0.f;
    const int f = g + i * G;
    if (active && i < nf && f < Df && (flags & FAKLA_STATE_IN)) {
      s[i] = S[(bh * Df + f) * Dv + dv];
      zr[i] = z[bh * Df + f];
    }
  }

  for (int64_t t0 = 0; t0 < T_len; t0 += kTok) {
    const int nt = (int)(T_len - t0 < kTok ? T_len - t0 : kTok);
    for (int e = tid; e < nt * Df; e += blockDim.x) {
      const int tt = e / Df, f = e % Df;
      const int64_t row = (b * T_len + t0 + tt) * H + h;
      const float tp = temp ? to_f32(temp[row]) : 1.f;
      qs[tt * Df + f] = to_f32(q[row * Df + f]);
      ks[tt * Df + f] = to_f32(k[row * Df + f]) * tp;
    }
    for (int e = tid; e < nt * Dv; e += blockDim.x) {
      const int tt = e / Dv, d = e % Dv;
      const int64_t row = (b * T_len + t0 + tt) * H + h;
      vs[tt * Dv + d] = to_f32(v[row * Dv + d]);
    }
    __syncthreads();
    if (active) {
      for (int tt = 0; tt < nt; ++tt) {
        const float vv = vs[tt * Dv + dv];
        float an = 0.f, ad = 0.f;
#pragma unroll
        for (int i = 0; i < kScanMaxF; ++i) {
          const int f = g + i * G;
          if (i < nf && f < Df) {
            const float kt = ks[tt * Df + f];
            const float qq = qs[tt * Df + f];
            zr[i] += kt;
            s[i] = fmaf(kt, vv, s[i]);
            an = fmaf(qq, s[i], an);
            ad = fmaf(qq, zr[i], ad);
          }
        }
        pn[(tt * G + g) * Dv + dv] = an;
        if (dv == 0) pd[tt * G + g] = ad;
      }
    }
    __syncthreads();
    for (int e = tid; e < nt * Dv; e += blockDim.x) {
      const int tt = e / Dv, d = e % Dv;
      float num = 0.f, den = 0.f;
      for (int gg = 0; gg < G; ++gg) {
        num += pn[(tt * G + gg) * Dv + d];
        den += pd[tt * G + gg];
      }
      const int64_t row = (b * T_len + t0 + tt) * H + h;
      out[row * Dv + d] = from_f32<T>(num * (1.f / (den + kEps)));
    }
    __syncthreads();
  }

  if (flags & FAKLA_STATE_OUT) {
#pragma unroll
    for (int i = 0; i < kScanMaxF; ++i) {
      const int f = g + i * G;
      if (active && i < nf && f < Df) {
        S[(bh * Df + f) * Dv + dv] = s[i];
        if (dv == 0) z[bh * Df + f] = zr[i];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Decode: one token for each of N*H sequences, state updated in place.
// One CTA per (n,h). Each row f of S (Dv floats) is handled by TPR = Dv/VEC
// threads with VEC-wide loads; the CTA covers RPP = 256/TPR rows per pass.
// S is read once and written once with streaming (evict-first) accesses:
//   S' = S + k~ (outer) v ;  z' = z + k~ ;  out = (phi_q^T S') / (phi_q . z' + eps)
// ---------------------------------------------------------------------------
template <int VEC>
struct VecF;
template <>
struct VecF<4> {
  using type = float4;
};
template <>
struct VecF<1> {
  using type = float;
};

__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ float ld_stream(const float* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float4* p, float4 v) { __stcs(p, v); }
__device__ __forceinline__ void st_stream(float* p, float v) { __stcs(p, v); }

__device__ __forceinline__ float4 upd(float4 s, float kt, float4 v) {
  return make_float4(fmaf(kt, v.x, s.x), fmaf(kt, v.y, s.y), fmaf(kt, v.z, s.z),
                     fmaf(kt, v.w, s.w));
}
__device__ __forceinline__ float upd(float s, float kt, float v) { return fmaf(kt, v, s); }
__device__ __forceinline__ void acc_add(float4& a, float q, float4 s) {
  a.x = fmaf(q, s.x, a.x);
  a.y = fmaf(q, s.y, a.y);
  a.z = fmaf(q, s.z, a.z);
  a.w = fmaf(q, s.w, a.w);
}
__device__ __forceinline__ void acc_add(float& a, float q, float s) { a = fmaf(q, s, a); }
__device__ __forceinline__ void zero(float4& a) { a = make_float4(0.f, 0.f, 0.f, 0.f); }
__device__ __forceinline__ void zero(float& a) { a = 0.f; }

template <typename T, int VEC>
__global__ void __launch_bounds__(256) decode_kernel(
    const T* __restrict__ qm, const T* __restrict__ km, const T* __restrict__ v,
    const T* __restrict__ temp, T* __restrict__ out, float* __restrict__ S,
    float* __restrict__ z, int Df, int Dv) {
  using V = typename VecF<VEC>::type;
  extern __shared__ float smem[];
  const int df4 = (Df + 3) & ~3, dv4 = (Dv + 3) & ~3;  // keep float4 views 16B-aligned
  float* phq = smem;        // [Df]
  float* kt = phq + df4;    // [Df]
  float* vv = kt + df4;     // [Dv]
  float* part = vv + dv4;   // [RPP][Dv]
  __shared__ float den_part[8];

  griddep_wait();  // phi(q), phi(k) come from the feature-map launch before this one
  griddep_launch_dependents();
  const int64_t bh = blockIdx.x;
  const int tid = threadIdx.x;
  const int TPR = Dv / VEC;
  const int RPP = 256 / TPR;
  const int lane = tid % TPR, rg = tid / TPR;
  const float tp = temp ? to_f32(temp[bh]) : 1.f;
  for (int f = tid; f < Df; f += 256) {
    phq[f] = to_f32(qm[bh * Df + f]);
    kt[f] = to_f32(km[bh * Df + f]) * tp;
  }
  for (int d = tid; d < Dv; d += 256) vv[d] = to_f32(v[bh * Dv + d]);
  __syncthreads();

  // Normaliser: z' = z + k~, den = phi_q . z'.
  float dpart = 0.f;
  for (int f = tid; f < Df; f += 256) {
    const float zn = z[bh * Df + f] + kt[f];
    z[bh * Df + f] = zn;
    dpart = fmaf(phq[f], zn, dpart);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dpart += __shfl_xor_sync(0xffffffffu, dpart, o);
  if ((tid & 31) == 0) den_part[tid >> 5] = dpart;

  V acc;
  zero(acc);
  if (rg < RPP) {
    const V vr = *reinterpret_cast<const V*>(vv + lane * VEC);
    V* base = reinterpret_cast<V*>(S + bh * (int64_t)Df * Dv) + lane;
    const int vstride = Dv / VEC;
    int f = rg;
    // 8 rows in flight per thread: issue the loads, then update/store.
    for (; f + 7 * RPP < Df; f += 8 * RPP) {
      V sv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sv[i] = ld_stream(base + (int64_t)(f + i * RPP) * vstride);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int ff = f + i * RPP;
        sv[i] = upd(sv[i], kt[ff], vr);
        st_stream(base + (int64_t)ff * vstride, sv[i]);
        acc_add(acc, phq[ff], sv[i]);
      }
    }
    for (; f < Df; f += RPP) {
      V sv = ld_stream(base + (int64_t)f * vstride);
      sv = upd(sv, kt[f], vr);
      st_stream(base + (int64_t)f * vstride, sv);
      acc_add(acc, phq[f], sv);
    }
    *reinterpret_cast<V*>(part + rg * Dv + lane * VEC) = acc;
  }
  __syncthreads();
  float den = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) den += den_part[w];
  const float inv = 1.f / (den + kEps);
  for (int d = tid; d < Dv; d += 256) {
    float num = 0.f;
    for (int r = 0; r < RPP; ++r) num += part[r * Dv + d];
    out[bh * Dv + d] = from_f32<T>(num * inv);
  }
}
}  // namespace

// ---------------------------------------------------------------------------
// Launchers (host). Shapes were validated by the caller (fakla_api.cu).
// ---------------------------------------------------------------------------
template <typename T, int ACT>
static cudaError_t launch_phi_simt_t(const void* x, const void* W, const void* bias,
                                     const void* temp, void* out, int64_t rows,
                                     int64_t K, int64_t N, int64_t heads, float scale,
                                     cudaStream_t stream) {
  const bool aligned16 = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(W)) & 15u) == 0;
  if (N <= kSkinnyN && K % 8 == 0 && aligned16) {
    const int64_t blocks = (rows + 7) / 8;
    if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
    if (N <= 4)
      phi_skinny_kernel<T, ACT, 4><<<(unsigned)blocks, 256, 0, stream>>>(
          (const T*)x, (const T*)W, (const T*)bias, (const T*)temp, (T*)out, rows, K, N, heads, scale);
    else
      phi_skinny_kernel<T, ACT, kSkinnyN><<<(unsigned)blocks, 256, 0, stream>>>(
          (const T*)x, (const T*)W, (const T*)bias, (const T*)temp, (T*)out, rows, K, N, heads, scale);
    return cudaGetLastError();
  }
  dim3 grid((unsigned)((N + kPhiTile - 1) / kPhiTile), (unsigned)((rows + kPhiTile - 1) / kPhiTile));
  phi_simt_kernel<T, ACT><<<grid, 256, 0, stream>>>(
      (const T*)x, (const T*)W, (const T*)bias, (const T*)temp, (T*)out, rows, K, N, heads, scale);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_phi_simt_dt(int act, const void* x, const void* W, const void* bias,
                                      const void* temp, void* out, int64_t rows, int64_t K,
                                      int64_t N, int64_t heads, float scale, cudaStream_t stream) {
#define FAKLA_PHI_CASE(A) \
  case A: return launch_phi_simt_t<T, A>(x, W, bias, temp, out, rows, K, N, heads, scale, stream);
  switch (act) {
    FAKLA_PHI_CASE(FAKLA_ACT_ELU1)
    FAKLA_PHI_CASE(FAKLA_ACT_RELU)
    FAKLA_PHI_CASE(FAKLA_ACT_SOFTPLUS)
    FAKLA_PHI_CASE(FAKLA_ACT_GELU)
    FAKLA_PHI_CASE(FAKLA_ACT_IDENTITY)
    FAKLA_PHI_CASE(FAKLA_ACT_SIGMOID)
    FAKLA_PHI_CASE(FAKLA_ACT_ABS)
    FAKLA_PHI_CASE(FAKLA_ACT_COSSIN)
    default: return cudaErrorInvalidValue;
  }
#undef FAKLA_PHI_CASE
}

cudaError_t launch_phi_simt(int dtype, const void* x, const void* W, const void* bias,
                            const void* temp, void* out, int64_t rows, int64_t K,
                            int64_t N, int64_t heads, int act, float scale, cudaStream_t stream) {
  if (dtype == FAKLA_BF16)
    return launch_phi_simt_dt<__nv_bfloat16>(act, x, W, bias, temp, out, rows, K, N, heads, scale, stream);
  return launch_phi_simt_dt<float>(act, x, W, bias, temp, out, rows, K, N, heads, scale, stream);
}

// ---------------------------------------------------------------------------
// KernelFeatureMixer combination: out[r, f] = sum_i w_i(r) feats[i, r, f] with
// w(r) = softmax(logits[r, :]) in fp32, rounded to T (as the reference's
// softmax(logits.float()).to(logits.dtype), mixer.py:134-135), and the sum
// accumulated in fp32. One thread per (row, VEC consecutive features); the
// weights of a row are recomputed per thread (n_maps is a handful).
// ---------------------------------------------------------------------------
constexpr int kMaxMaps = 32;

template <typename T, int VEC>
__global__ void __launch_bounds__(256) mix_features_kernel(const T* __restrict__ feats,
                                                           const T* __restrict__ logits,
                                                           T* __restrict__ out, int64_t rows,
                                                           int n_maps, int64_t F) {
  const int64_t per_row = F / VEC;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * per_row) return;
  const int64_t r = idx / per_row;
  const int64_t f0 = (idx % per_row) * VEC;
  float w[kMaxMaps];
  float mx = -INFINITY;
  for (int i = 0; i < n_maps; ++i) {
    w[i] = to_f32(logits[r * n_maps + i]);
    mx = fmaxf(mx, w[i]);
  }
  float den = 0.f;
  for (int i = 0; i < n_maps; ++i) {
    w[i] = expf(w[i] - mx);
    den += w[i];
  }
  const float inv = 1.f / den;
  float acc[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) acc[v] = 0.f;
  for (int i = 0; i < n_maps; ++i) {
    const float wi = to_f32(from_f32<T>(w[i] * inv));
    const T* src = feats + ((int64_t)i * rows + r) * F + f0;
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[v] = fmaf(wi, to_f32(src[v]), acc[v]);
  }
  T* dst = out + r * F + f0;
#pragma unroll
  for (int v = 0; v < VEC; ++v) dst[v] = from_f32<T>(acc[v]);
}

// The same combination for bf16 and up to kMixFast maps with 8 features per
// thread (16-byte loads and stores): the gate weights and every map's 8
// features are held in registers, all the map loads issued before any is
// used. The arithmetic and its order are those of mix_features_kernel.
constexpr int kMixFast = 8;

template <typename T>
__device__ __forceinline__ void store8_from_f32(T* p, const float (&f)[8]) {
  if constexpr (sizeof(T) == 2) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(p) = u;
  } else {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
}

template <typename T, int NMAX, int CH>
__global__ void __launch_bounds__(256) mix_features_fast_kernel(const T* __restrict__ feats,
                                                                const T* __restrict__ logits,
                                                                T* __restrict__ out, int64_t rows,
                                                                int n_maps, int64_t F) {
  // CH consecutive 8-feature pieces per thread (F % (8 CH) == 0)
  const int64_t per_row = F / (8 * CH);
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * per_row) return;
  const int64_t r = idx / per_row;
  const int64_t f0 = (idx % per_row) * 8 * CH;
  // the maps' features as raw bf16 (16 bytes per piece), converted when used
  uint4 x[NMAX][CH];
#pragma unroll
  for (int i = 0; i < NMAX; ++i)
    if (i < n_maps) {
#pragma unroll
      for (int c = 0; c < CH; ++c)
        x[i][c] = __ldg(reinterpret_cast<const uint4*>(feats + ((int64_t)i * rows + r) * F + f0) + c);
    }
  float w[NMAX];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < NMAX; ++i) {
    w[i] = i < n_maps ? to_f32(logits[r * n_maps + i]) : -INFINITY;
    mx = fmaxf(mx, w[i]);
  }
  float den = 0.f;
#pragma unroll
  for (int i = 0; i < NMAX; ++i) {
    if (i < n_maps) {
      w[i] = expf(w[i] - mx);
      den += w[i];
    }
  }
  const float inv = 1.f / den;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    float acc[8];
#pragma unroll
    for (int v = 0; v < 8; ++v) acc[v] = 0.f;
#pragma unroll
    for (int i = 0; i < NMAX; ++i) {
      if (i < n_maps) {
        const float wi = to_f32(from_f32<T>(w[i] * inv));
        const uint32_t u[4] = {x[i][c].x, x[i][c].y, x[i][c].z, x[i][c].w};
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          acc[2 * v] = fmaf(wi, __uint_as_float(u[v] << 16), acc[2 * v]);
          acc[2 * v + 1] = fmaf(wi, __uint_as_float(u[v] & 0xffff0000u), acc[2 * v + 1]);
        }
      }
    }
    store8_from_f32(out + r * F + f0 + 8 * c, acc);
  }
}

template <typename T>
static cudaError_t launch_mix_t(const void* feats, const void* logits, void* out, int64_t rows,
                                int64_t n_maps, int64_t F, cudaStream_t stream) {
  const bool vec = F % 8 == 0 && ((uintptr_t)feats & 15u) == 0 && ((uintptr_t)out & 15u) == 0;
  const int64_t threads = rows * (vec ? F / 8 : F);
  const unsigned grid = (unsigned)((threads + 255) / 256);
  if (vec && n_maps <= 4 && sizeof(T) == 2 && F % 16 == 0)
    mix_features_fast_kernel<T, 4, 2><<<(unsigned)((rows * (F / 16) + 255) / 256), 256, 0, stream>>>(
        (const T*)feats, (const T*)logits, (T*)out, rows, (int)n_maps, F);
  else if (vec && n_maps <= kMixFast && sizeof(T) == 2)
    mix_features_fast_kernel<T, kMixFast, 1><<<grid, 256, 0, stream>>>((const T*)feats, (const T*)logits,
                                                                     (T*)out, rows, (int)n_maps, F);
  else if (vec)
    mix_features_kernel<T, 8><<<grid, 256, 0, stream>>>((const T*)feats, (const T*)logits, (T*)out,
                                                       rows, (int)n_maps, F);
  else
    mix_features_kernel<T, 1><<<grid, 256, 0, stream>>>((const T*)feats, (const T*)logits, (T*)out,
                                                       rows, (int)n_maps, F);
  return cudaGetLastError();
}

bool mix_supported(int64_t n_maps) { return n_maps >= 1 && n_maps <= kMaxMaps; }

// d(elu(x) + 1)/dx from the output phi: 1 where phi > 1 (x > 0), phi otherwise.
template <typename T>
__global__ void phi_backward_kernel(const T* __restrict__ phi, const T* __restrict__ dphi,
                                    T* __restrict__ dpre, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float p = to_f32(phi[i]);
    dpre[i] = from_f32<T>(to_f32(dphi[i]) * (p > 1.f ? 1.f : p));
  }
}

// Derivatives of the fakla_feature_map activations at the pre-activation x.
template <int ACT>
__device__ __forceinline__ float activation_grad(float x) {
  if constexpr (ACT == FAKLA_ACT_ELU1) {
    return x > 0.f ? 1.f : expf(x);
  } else if constexpr (ACT == FAKLA_ACT_RELU) {
    return x > 0.f ? 1.f : 0.f;
  } else if constexpr (ACT == FAKLA_ACT_SOFTPLUS) {
    return x > 20.f ? 1.f : 1.f / (1.f + expf(-x));
  } else if constexpr (ACT == FAKLA_ACT_GELU) {
    return 0.5f * (1.f + erff(x * 0.70710678118654752f)) + x * 0.3989422804014327f * expf(-0.5f * x * x);
  } else if constexpr (ACT == FAKLA_ACT_SIGMOID) {
    const float sg = 1.f / (1.f + expf(-x));
    return sg * (1.f - sg);
  } else if constexpr (ACT == FAKLA_ACT_ABS) {
    return x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
  } else {
    return 1.f;  // FAKLA_ACT_IDENTITY
  }
}

template <typename T, int ACT>
__global__ void activation_backward_kernel(const T* __restrict__ pre, const T* __restrict__ dy,
                                           T* __restrict__ dpre, int64_t rows, int64_t n,
                                           float scale) {
  const int64_t total = rows * n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float x = to_f32(pre[i]);
    if constexpr (ACT == FAKLA_ACT_COSSIN) {
      const int64_t r = i / n, c = i % n;
      float sn, cs;
      sincosf(x, &sn, &cs);
      dpre[i] = from_f32<T>(scale * (cs * to_f32(dy[r * 2 * n + n + c]) - sn * to_f32(dy[r * 2 * n + c])));
    } else {
      dpre[i] = from_f32<T>(to_f32(dy[i]) * activation_grad<ACT>(x));
    }
  }
}

template <typename T>
static cudaError_t launch_act_bwd_t(int act, const void* pre, const void* dy, void* dpre,
                                    int64_t rows, int64_t n, float scale, cudaStream_t stream) {
  const int64_t want = (rows * n + 255) / 256;
  const unsigned grid = (unsigned)(want < 148 * 16 ? want : 148 * 16);
#define FAKLA_ACTB_CASE(A)                                                                 \
  case A:                                                                                  \
    activation_backward_kernel<T, A><<<grid, 256, 0, stream>>>((const T*)pre, (const T*)dy, \
                                                               (T*)dpre, rows, n, scale); \
    break;
  switch (act) {
    FAKLA_ACTB_CASE(FAKLA_ACT_ELU1)
    FAKLA_ACTB_CASE(FAKLA_ACT_RELU)
    FAKLA_ACTB_CASE(FAKLA_ACT_SOFTPLUS)
    FAKLA_ACTB_CASE(FAKLA_ACT_GELU)
    FAKLA_ACTB_CASE(FAKLA_ACT_IDENTITY)
    FAKLA_ACTB_CASE(FAKLA_ACT_SIGMOID)
    FAKLA_ACTB_CASE(FAKLA_ACT_ABS)
    FAKLA_ACTB_CASE(FAKLA_ACT_COSSIN)
    default: return cudaErrorInvalidValue;
  }
#undef FAKLA_ACTB_CASE
  return cudaGetLastError();
}

cudaError_t launch_activation_backward(int dtype, int act, const void* pre, const void* dy,
                                       void* dpre, int64_t rows, int64_t n, float scale,
                                       cudaStream_t stream) {
  if (dtype == FAKLA_BF16)
    return launch_act_bwd_t<__nv_bfloat16>(act, pre, dy, dpre, rows, n, scale, stream);
  return launch_act_bwd_t<float>(act, pre, dy, dpre, rows, n, scale, stream);
}

// Mixer backward: one warp per row. w = softmax(logits) rounded to T as in
// the forward; dw_i = dout . feats[i]; dlogits_i = w_i (dw_i - sum_j w_j dw_j);
// dfeats[i] = w_i dout.
template <typename T>
__global__ void mix_backward_kernel(const T* __restrict__ feats, const T* __restrict__ logits,
                                    const T* __restrict__ dout, T* __restrict__ dfeats,
                                    T* __restrict__ dlogits, int64_t rows, int n_maps, int64_t F) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float w[kMaxMaps], dw[kMaxMaps];
  float mx = -INFINITY;
  for (int i = 0; i < n_maps; ++i) {
    w[i] = to_f32(logits[r * n_maps + i]);
    mx = fmaxf(mx, w[i]);
  }
  float den = 0.f;
  for (int i = 0; i < n_maps; ++i) {
    w[i] = expf(w[i] - mx);
    den += w[i];
  }
  for (int i = 0; i < n_maps; ++i) {
    w[i] = to_f32(from_f32<T>(w[i] / den));
    dw[i] = 0.f;
  }
  for (int64_t c = lane; c < F; c += 32) {
    const float g = to_f32(dout[r * F + c]);
    for (int i = 0; i < n_maps; ++i) {
      const int64_t idx = ((int64_t)i * rows + r) * F + c;
      dw[i] = fmaf(g, to_f32(feats[idx]), dw[i]);
      if (dfeats) dfeats[idx] = from_f32<T>(w[i] * g);
    }
  }
  for (int i = 0; i < n_maps; ++i)
    for (int o = 16; o > 0; o >>= 1) dw[i] += __shfl_xor_sync(0xffffffffu, dw[i], o);
  if (dlogits && lane == 0) {
    float s = 0.f;
    for (int i = 0; i < n_maps; ++i) s += w[i] * dw[i];
    for (int i = 0; i < n_maps; ++i) dlogits[r * n_maps + i] = from_f32<T>(w[i] * (dw[i] - s));
  }
}

cudaError_t launch_mix_backward(int dtype, const void* feats, const void* logits, const void* dout,
                                void* dfeats, void* dlogits, int64_t rows, int64_t n_maps,
                                int64_t F, cudaStream_t stream) {
  const unsigned grid = (unsigned)((rows + 7) / 8);
  if (dtype == FAKLA_BF16)
    mix_backward_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        (const __nv_bfloat16*)feats, (const __nv_bfloat16*)logits, (const __nv_bfloat16*)dout,
        (__nv_bfloat16*)dfeats, (__nv_bfloat16*)dlogits, rows, (int)n_maps, F);
  else
    mix_backward_kernel<float><<<grid, 256, 0, stream>>>((const float*)feats, (const float*)logits,
                                                         (const float*)dout, (float*)dfeats,
                                                         (float*)dlogits, rows, (int)n_maps, F);
  return cudaGetLastError();
}

cudaError_t launch_phi_backward(int dtype, const void* phi, const void* dphi, void* dpre,
                                int64_t n, cudaStream_t stream) {
  const int64_t want = (n + 255) / 256;
  const unsigned grid = (unsigned)(want < 148 * 16 ? want : 148 * 16);
  if (dtype == FAKLA_BF16)
    phi_backward_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        (const __nv_bfloat16*)phi, (const __nv_bfloat16*)dphi, (__nv_bfloat16*)dpre, n);
  else
    phi_backward_kernel<float><<<grid, 256, 0, stream>>>((const float*)phi, (const float*)dphi,
                                                         (float*)dpre, n);
  return cudaGetLastError();
}

cudaError_t launch_mix_features(int dtype, const void* feats, const void* logits, void* out,
                                int64_t rows, int64_t n_maps, int64_t F, cudaStream_t stream) {
  if (dtype == FAKLA_BF16) return launch_mix_t<__nv_bfloat16>(feats, logits, out, rows, n_maps, F, stream);
  return launch_mix_t<float>(feats, logits, out, rows, n_maps, F, stream);
}

bool scan_simt_supported(int64_t Df, int64_t Dv) {
  if (Df < 1 || Dv < 1 || Dv > 256 || Df > 256) return false;
  const int64_t G = 256 / Dv;
  return (Df + G - 1) / G <= kScanMaxF;
}

size_t scan_simt_smem_bytes(int64_t Df, int64_t Dv) {
  const int64_t G = 256 / Dv;
  return sizeof(float) * (size_t)(2 * kTok * Df + kTok * Dv + kTok * G * Dv + kTok * G);
}

template <typename T>
static cudaError_t launch_scan_simt_t(const void* q, const void* k, const void* v,
                                      const void* temp, void* out, float* S, float* z,
                                      int64_t B, int64_t T_len, int64_t H, int64_t Df,
                                      int64_t Dv, unsigned flags, cudaStream_t stream) {
  const size_t smem = scan_simt_smem_bytes(Df, Dv);
  cudaError_t e = cudaFuncSetAttribute(scan_simt_kernel<T>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  scan_simt_kernel<T><<<(unsigned)(B * H), 256, smem, stream>>>(
      (const T*)q, (const T*)k, (const T*)v, (const T*)temp, (T*)out, S, z, T_len, H,
      (int)Df, (int)Dv, flags);
  return cudaGetLastError();
}

cudaError_t launch_scan_simt(int dtype, const void* q, const void* k, const void* v,
                             const void* temp, void* out, float* S, float* z, int64_t B,
                             int64_t T_len, int64_t H, int64_t Df, int64_t Dv,
                             unsigned flags, cudaStream_t stream) {
  if (dtype == FAKLA_BF16)
    return launch_scan_simt_t<__nv_bfloat16>(q, k, v, temp, out, S, z, B, T_len, H, Df, Dv,
                                             flags, stream);
  return launch_scan_simt_t<float>(q, k, v, temp, out, S, z, B, T_len, H, Df, Dv, flags,
                                   stream);
}

template <typename T>
static cudaError_t launch_decode_t(const void* q, const void* k, const void* v,
                                   const void* temp, void* out, float* S, float* z,
                                   int64_t NH, int64_t Df, int64_t Dv, cudaStream_t stream) {
  // float4 path needs Dv % 4 == 0 and Dv/4 threads per row (<= 256); the state
  // pointer is 16-byte aligned for every row when S is (checked by the caller).
  const bool vec4 = (Dv % 4 == 0) && (Dv / 4 <= 256) && (((uintptr_t)S & 15u) == 0);
  const int tpr = vec4 ? (int)(Dv / 4) : (int)Dv;
  const int rpp = 256 / tpr;
  const size_t smem = sizeof(float) * (size_t)(2 * ((Df + 3) & ~3) + ((Dv + 3) & ~3) + rpp * Dv);
  if (vec4) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel<T, 4>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_chained(decode_kernel<T, 4>, dim3((unsigned)NH), dim3(256), smem, stream, 1u, (const T*)q,
                          (const T*)k, (const T*)v, (const T*)temp, (T*)out, S, z, (int)Df, (int)Dv);
  } else {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel<T, 1>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_chained(decode_kernel<T, 1>, dim3((unsigned)NH), dim3(256), smem, stream, 1u, (const T*)q,
                          (const T*)k, (const T*)v, (const T*)temp, (T*)out, S, z, (int)Df, (int)Dv);
  }
}

// ---------------------------------------------------------------------------
// Linear-layer gradients on the CUDA cores (fp32, and bf16 shapes outside the
// tensor-core set): a tiled GEMM over strided operands,
//   C[m, n] = sum_k A[m sam + k sak] B[n sbn + k sbk]   (C row-major, fp32 accumulation)
// which covers dx = dpre W and dW = dpre^T x, and a column sum for the bias.
// ---------------------------------------------------------------------------
namespace {
template <typename T>
__global__ void __launch_bounds__(256) gemm_strided_simt_kernel(
    const T* __restrict__ A, int64_t sam, int64_t sak, const T* __restrict__ Bm, int64_t sbn,
    int64_t sbk, T* __restrict__ C, int64_t M, int64_t N, int64_t K) {
  __shared__ float as[kPhiK][kPhiTile + 4];
  __shared__ float bs[kPhiK][kPhiTile + 4];
  const int tid = threadIdx.x;
  const int64_t m0 = (int64_t)blockIdx.y * kPhiTile;
  const int64_t n0 = (int64_t)blockIdx.x * kPhiTile;
  const int tr = tid / 16, tc = tid % 16;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += kPhiK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * 256;
      // consecutive threads walk k when the operand is k-contiguous, else the
      // row index, so that either layout reads whole sectors
      const bool ak = sak == 1, bk = sbk == 1;
      const int ra = ak ? e / kPhiK : e % kPhiTile, ka = ak ? e % kPhiK : e / kPhiTile;
      const int rb = bk ? e / kPhiK : e % kPhiTile, kb = bk ? e % kPhiK : e / kPhiTile;
      const int64_t gm = m0 + ra, gka = k0 + ka, gn = n0 + rb, gkb = k0 + kb;
      as[ka][ra] = (gm < M && gka < K) ? to_f32(A[gm * sam + gka * sak]) : 0.f;
      bs[kb][rb] = (gn < N && gkb < K) ? to_f32(Bm[gn * sbn + gkb * sbk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kPhiK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = as[kk][tr * 4 + i];
        b[i] = bs[kk][tc * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gm = m0 + tr * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gn = n0 + tc * 4 + j;
      if (gn < N) C[gm * N + gn] = from_f32<T>(acc[i][j]);
    }
  }
}

constexpr int kColSumRows = 256;  // rows per partial sum of the column reduction

// partial[c, n] = sum of rows [c * kColSumRows, (c + 1) * kColSumRows) of column n
template <typename T>
__global__ void __launch_bounds__(256) colsum_partial_kernel(const T* __restrict__ x, float* __restrict__ partial,
                                                             int64_t rows, int64_t n) {
  const int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= n) return;
  const int64_t r0 = (int64_t)blockIdx.y * kColSumRows;
  const int64_t r1 = min(rows, r0 + kColSumRows);
  float acc = 0.f;
  for (int64_t r = r0; r < r1; ++r) acc += to_f32(x[r * n + col]);
  partial[(int64_t)blockIdx.y * n + col] = acc;
}

// out[n] = sum over the partial rows, in order (deterministic)
template <typename T>
__global__ void __launch_bounds__(256) colsum_final_kernel(const float* __restrict__ partial, T* __restrict__ out,
                                                           int64_t chunks, int64_t n) {
  const int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= n) return;
  float acc = 0.f;
  for (int64_t c = 0; c < chunks; ++c) acc += partial[c * n + col];
  out[col] = from_f32<T>(acc);
}

template <typename T>
cudaError_t launch_gemm_strided_t(const void* A, int64_t sam, int64_t sak, const void* Bm, int64_t sbn, int64_t sbk,
                                  void* C, int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  const dim3 grid((unsigned)((N + kPhiTile - 1) / kPhiTile), (unsigned)((M + kPhiTile - 1) / kPhiTile));
  gemm_strided_simt_kernel<T><<<grid, 256, 0, stream>>>((const T*)A, sam, sak, (const T*)Bm, sbn, sbk, (T*)C, M, N,
                                                        K);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_colsum_t(const void* x, void* out, float* partial, int64_t rows, int64_t n, cudaStream_t stream) {
  const int64_t chunks = (rows + kColSumRows - 1) / kColSumRows;
  const unsigned gx = (unsigned)((n + 255) / 256);
  colsum_partial_kernel<T><<<dim3(gx, (unsigned)chunks), 256, 0, stream>>>((const T*)x, partial, rows, n);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  colsum_final_kernel<T><<<gx, 256, 0, stream>>>(partial, (T*)out, chunks, n);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_gemm_strided(int dtype, const void* A, int64_t sam, int64_t sak, const void* Bm, int64_t sbn,
                                int64_t sbk, void* C, int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  if (dtype == FAKLA_BF16)
    return launch_gemm_strided_t<__nv_bfloat16>(A, sam, sak, Bm, sbn, sbk, C, M, N, K, stream);
  return launch_gemm_strided_t<float>(A, sam, sak, Bm, sbn, sbk, C, M, N, K, stream);
}

size_t colsum_workspace_bytes(int64_t rows, int64_t n) {
  return (size_t)((rows + kColSumRows - 1) / kColSumRows) * (size_t)n * sizeof(float);
}

cudaError_t launch_colsum(int dtype, const void* x, void* out, float* partial, int64_t rows, int64_t n,
                          cudaStream_t stream) {
  if (dtype == FAKLA_BF16) return launch_colsum_t<__nv_bfloat16>(x, out, partial, rows, n, stream);
  return launch_colsum_t<float>(x, out, partial, rows, n, stream);
}

cudaError_t launch_decode(int dtype, const void* q, const void* k, const void* v,
                          const void* temp, void* out, float* S, float* z, int64_t NH,
                          int64_t Df, int64_t Dv, cudaStream_t stream) {
  if (dtype == FAKLA_BF16)
    return launch_decode_t<__nv_bfloat16>(q, k, v, temp, out, S, z, NH, Df, Dv, stream);
  return launch_decode_t<float>(q, k, v, temp, out, S, z, NH, Df, Dv, stream);
}

}  // namespace fakla
