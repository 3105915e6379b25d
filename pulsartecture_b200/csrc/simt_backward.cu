// FA-KLA backward on CUDA cores (any dtype, head dims within the register
// budget below). For one (b, h) sequence the forward recurrence of the
// reference (ultra_rwka/backend/cpp/cpu/cpu_kernels.cpp:107-164) is
//
//   k~_t = k_t temp_t,  z_t = z_{t-1} + k~_t,  S_t = S_{t-1} + k~_t v_t^T,
//   den_t = q_t . z_t + eps,  out_t = S_t^T q_t / den_t.
//
// Given dout, with dnum_t = dout_t / den_t and dden_t = -(q_t^T S_t dout_t) / den_t^2:
//
//   dq_t  = S_t dnum_t + z_t dden_t = u_t / den_t + z_t dden_t,  u_t = S_t dout_t
//   G_s   = dS_T + sum_{t >= s} q_t dnum_t^T,  g_s = dz_T + sum_{t >= s} q_t dden_t
//   dk~_s = G_s v_s + g_s,  dv_s = G_s^T k~_s,  dk_s = dk~_s temp_s,  dtemp_s = dk~_s . k_s
//   dS_0  = G_0,  dz_0 = g_0
//
// Two token-sequential sweeps, one CTA per (b, h), fp32 state in registers:
//  * bwd_forward_kernel walks t upwards rebuilding S_t, z_t (thread (f, j)
//    holds the dv = j, j+J, ... entries of row f) and writes dq, 1/den_t and
//    dden_t (workspace);
//  * bwd_reverse_kernel walks t downwards accumulating G, g. G is kept twice,
//    by rows (thread (f, j), for dk~ = G v: a sum over dv) and by columns
//    (thread (gc, dv) holds f = gc, gc+Gc, ..., for dv = G^T k~: a sum over
//    f); both copies receive the same FMAs in the same order, so they hold
//    the same values.
// Tokens are staged kTok at a time in shared memory; per-token scalars
// (den, q.u, dtemp) are reduced per batch.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fakla_common.cuh"
#include "fakla_kernels.h"

namespace fakla {
namespace {

// 1024 threads with at most 16 state values each (per layout): short FMA
// chains per token and 8 warps per scheduler to hide their latency; with 256
// threads and 64 values the sweeps were latency-bound and the reverse one
// spilled.
constexpr int kThreads = 1024;
constexpr int kTok = 16;
constexpr int kMaxVals = 16;  // state values per thread per layout

struct BwdShape {
  int Df, Dv;
  int J;   // threads per row f (power of two); row layout uses Df * J threads
  int nr;  // values per thread in the row layout: ceil(Dv / J)
  int Gc;  // column groups: kThreads / Dv
  int nc;  // values per thread in the column layout: ceil(Df / Gc)
};

__host__ __device__ inline BwdShape bwd_shape(int Df, int Dv) {
  BwdShape s;
  s.Df = Df;
  s.Dv = Dv;
  int J = 1;
  while (Df * J * 2 <= kThreads && J < 32) J *= 2;
  s.J = J;
  s.nr = (Dv + J - 1) / J;
  s.Gc = kThreads / Dv;
  s.nc = s.Gc > 0 ? (Df + s.Gc - 1) / s.Gc : kMaxVals + 1;
  return s;
}

// Sum over the J lanes that share a row (J is a power of two <= 32: those
// lanes are adjacent in one warp).
__device__ __forceinline__ float row_sum(float v, int J) {
  for (int o = 1; o < J; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ void stage_tokens(const T* __restrict__ src, float* dst, int64_t b, int64_t t0,
                                             int nt, int64_t T_len, int64_t H, int64_t h, int D,
                                             const T* __restrict__ scale_by) {
  for (int e = threadIdx.x; e < nt * D; e += blockDim.x) {
    const int tt = e / D, f = e % D;
    const int64_t row = (b * T_len + t0 + tt) * H + h;
    float x = to_f32(src[row * D + f]);
    if (scale_by) x *= to_f32(scale_by[row]);
    dst[tt * D + f] = x;
  }
}

// ---------------------------------------------------------------------------
// Sweep 1 (t ascending): dq, and 1/den_t, dden_t into the workspace.
// smem: qs, ks (k~), zt [kTok][Df]; vs, ds [kTok][Dv]; us, zq, uq [kTok][Df];
//       den, dd [kTok]
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads) bwd_forward_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const T* __restrict__ temp, const T* __restrict__ dout, const float* __restrict__ S0,
    const float* __restrict__ z0, T* __restrict__ dq, float* __restrict__ rden_ws,
    float* __restrict__ dden_ws, int64_t T_len, int64_t H, int Df, int Dv) {
  extern __shared__ float smem[];
  const BwdShape sh = bwd_shape(Df, Dv);
  float* qs = smem;
  float* ks = qs + kTok * Df;
  float* vs = ks + kTok * Df;
  float* ds = vs + kTok * Dv;
  float* us = ds + kTok * Dv;
  float* zt = us + kTok * Df;
  float* zq = zt + kTok * Df;
  float* uq = zq + kTok * Df;
  float* den = uq + kTok * Df;
  float* dd = den + kTok;

  const int64_t bh = blockIdx.x;
  const int64_t b = bh / H, h = bh % H;
  const int tid = threadIdx.x;
  const int f = tid / sh.J, j = tid % sh.J;
  const bool active = f < Df;

  float s[kMaxVals];
  float zr = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVals; ++i) {
    s[i] = 0.f;
    const int d = j + i * sh.J;
    if (active && i < sh.nr && d < Dv && S0) s[i] = S0[(bh * Df + f) * Dv + d];
  }
  if (active && z0) zr = z0[bh * Df + f];

  for (int64_t t0 = 0; t0 < T_len; t0 += kTok) {
    const int nt = (int)(T_len - t0 < kTok ? T_len - t0 : kTok);
    stage_tokens(q, qs, b, t0, nt, T_len, H, h, Df, (const T*)nullptr);
    stage_tokens(k, ks, b, t0, nt, T_len, H, h, Df, temp);
    stage_tokens(v, vs, b, t0, nt, T_len, H, h, Dv, (const T*)nullptr);
    stage_tokens(dout, ds, b, t0, nt, T_len, H, h, Dv, (const T*)nullptr);
    __syncthreads();
    for (int tt = 0; tt < nt; ++tt) {
      float u = 0.f;
      const float kt = active ? ks[tt * Df + f] : 0.f;
#pragma unroll
      for (int i = 0; i < kMaxVals; ++i) {
        const int d = j + i * sh.J;
        if (i < sh.nr && d < Dv) {
          s[i] = fmaf(kt, vs[tt * Dv + d], s[i]);
          u = fmaf(s[i], ds[tt * Dv + d], u);
        }
      }
      zr += kt;
      u = row_sum(u, sh.J);
      if (active && j == 0) {
        const float qf = qs[tt * Df + f];
        us[tt * Df + f] = u;
        zt[tt * Df + f] = zr;
        zq[tt * Df + f] = qf * zr;
        uq[tt * Df + f] = qf * u;
      }
    }
    __syncthreads();
    // per token: den = sum_f q z + eps, dden = -(sum_f q u) / den^2 (one warp per token)
    const int warp = tid >> 5, lane = tid & 31;
    for (int tt = warp; tt < nt; tt += kThreads / 32) {
      float a = 0.f, c = 0.f;
      for (int ff = lane; ff < Df; ff += 32) {
        a += zq[tt * Df + ff];
        c += uq[tt * Df + ff];
      }
      for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        c += __shfl_xor_sync(0xffffffffu, c, o);
      }
      if (lane == 0) {
        const float dn = a + kEps;
        den[tt] = dn;
        dd[tt] = -c / (dn * dn);
        const int64_t row = (b * T_len + t0 + tt) * H + h;
        rden_ws[row] = 1.f / dn;
        dden_ws[row] = dd[tt];
      }
    }
    __syncthreads();
    for (int e = tid; e < nt * Df; e += blockDim.x) {
      const int tt = e / Df, ff = e % Df;
      const int64_t row = (b * T_len + t0 + tt) * H + h;
      dq[row * Df + ff] = from_f32<T>(us[tt * Df + ff] / den[tt] + zt[tt * Df + ff] * dd[tt]);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Sweep 2 (t descending): dk, dv, dtemp, dS_0, dz_0.
// smem: qs, ks (k~), kr (k) [kTok][Df]; vs, dn (dout / den) [kTok][Dv];
//       dkt, dkk [kTok][Df]; pv [kTok][Gc][Dv]; ddn [kTok]; tp [kTok]
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads) bwd_reverse_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const T* __restrict__ temp, const T* __restrict__ dout, const float* __restrict__ rden_ws,
    const float* __restrict__ dden_ws, const float* __restrict__ dS_final,
    const float* __restrict__ dz_final, T* __restrict__ dk, T* __restrict__ dv,
    T* __restrict__ dtemp, float* __restrict__ dS0, float* __restrict__ dz0, int64_t T_len,
    int64_t H, int Df, int Dv) {
  extern __shared__ float smem[];
  const BwdShape sh = bwd_shape(Df, Dv);
  float* qs = smem;
  float* ks = qs + kTok * Df;
  float* kr = ks + kTok * Df;
  float* dkt = kr + kTok * Df;
  float* dkk = dkt + kTok * Df;
  float* vs = dkk + kTok * Df;
  float* dn = vs + kTok * Dv;
  float* pv = dn + kTok * Dv;
  float* ddn = pv + kTok * sh.Gc * Dv;
  float* tp = ddn + kTok;

  const int64_t bh = blockIdx.x;
  const int64_t b = bh / H, h = bh % H;
  const int tid = threadIdx.x;
  const int f = tid / sh.J, j = tid % sh.J;       // row layout
  const bool ra = f < Df;
  const int gc = tid / Dv, dvc = tid % Dv;        // column layout
  const bool ca = gc < sh.Gc;

  float gr[kMaxVals], gcv[kMaxVals];
  float gz = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVals; ++i) {
    gr[i] = 0.f;
    gcv[i] = 0.f;
    const int d = j + i * sh.J;
    if (ra && i < sh.nr && d < Dv && dS_final) gr[i] = dS_final[(bh * Df + f) * Dv + d];
    const int fc = gc + i * sh.Gc;
    if (ca && i < sh.nc && fc < Df && dS_final) gcv[i] = dS_final[(bh * Df + fc) * Dv + dvc];
  }
  if (ra && dz_final) gz = dz_final[bh * Df + f];

  const int64_t nbatch = (T_len + kTok - 1) / kTok;
  for (int64_t bi = nbatch - 1; bi >= 0; --bi) {
    const int64_t t0 = bi * kTok;
    const int nt = (int)(T_len - t0 < kTok ? T_len - t0 : kTok);
    stage_tokens(q, qs, b, t0, nt, T_len, H, h, Df, (const T*)nullptr);
    stage_tokens(k, ks, b, t0, nt, T_len, H, h, Df, temp);
    stage_tokens(k, kr, b, t0, nt, T_len, H, h, Df, (const T*)nullptr);
    stage_tokens(v, vs, b, t0, nt, T_len, H, h, Dv, (const T*)nullptr);
    for (int e = threadIdx.x; e < nt * Dv; e += blockDim.x) {
      const int tt = e / Dv, d = e % Dv;
      const int64_t row = (b * T_len + t0 + tt) * H + h;
      dn[tt * Dv + d] = to_f32(dout[row * Dv + d]) * rden_ws[row];
    }
    for (int tt = threadIdx.x; tt < nt; tt += blockDim.x) {
      const int64_t row = (b * T_len + t0 + tt) * H + h;
      ddn[tt] = dden_ws[row];
      tp[tt] = temp ? to_f32(temp[row]) : 1.f;
    }
    __syncthreads();
    for (int tt = nt - 1; tt >= 0; --tt) {
      const float dden = ddn[tt];
      // row layout: G += q dnum^T (row f), g += q dden; dk~_f = G v + g
      float pk = 0.f;
      const float qf = ra ? qs[tt * Df + f] : 0.f;
#pragma unroll
      for (int i = 0; i < kMaxVals; ++i) {
        const int d = j + i * sh.J;
        if (i < sh.nr && d < Dv) {
          gr[i] = fmaf(qf, dn[tt * Dv + d], gr[i]);
          pk = fmaf(gr[i], vs[tt * Dv + d], pk);
        }
      }
      gz = fmaf(qf, dden, gz);
      pk = row_sum(pk, sh.J);
      if (ra && j == 0) {
        const float dkf = pk + gz;
        dkt[tt * Df + f] = dkf;
        dkk[tt * Df + f] = dkf * kr[tt * Df + f];
      }
      // column layout: the same G by columns; dv partial = sum over my f of G k~
      if (ca) {
        const float dnv = dn[tt * Dv + dvc];
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxVals; ++i) {
          const int fc = gc + i * sh.Gc;
          if (i < sh.nc && fc < Df) {
            gcv[i] = fmaf(qs[tt * Df + fc], dnv, gcv[i]);
            a = fmaf(gcv[i], ks[tt * Df + fc], a);
          }
        }
        pv[(tt * sh.Gc + gc) * Dv + dvc] = a;
      }
    }
    __syncthreads();
    for (int e = tid; e < nt * Df; e += blockDim.x) {
      const int tt = e / Df, ff = e % Df;
      const int64_t row = (b * T_len + t0 + tt) * H + h;
      dk[row * Df + ff] = from_f32<T>(dkt[tt * Df + ff] * tp[tt]);
    }
    for (int e = tid; e < nt * Dv; e += blockDim.x) {
      const int tt = e / Dv, d = e % Dv;
      float a = 0.f;
      for (int g2 = 0; g2 < sh.Gc; ++g2) a += pv[(tt * sh.Gc + g2) * Dv + d];
      const int64_t row = (b * T_len + t0 + tt) * H + h;
      dv[row * Dv + d] = from_f32<T>(a);
    }
    if (dtemp) {
      const int warp = tid >> 5, lane = tid & 31;
      for (int tt = warp; tt < nt; tt += kThreads / 32) {
        float a = 0.f;
        for (int ff = lane; ff < Df; ff += 32) a += dkk[tt * Df + ff];
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) dtemp[(b * T_len + t0 + tt) * H + h] = from_f32<T>(a);
      }
    }
    __syncthreads();
  }
  if (dS0) {
#pragma unroll
    for (int i = 0; i < kMaxVals; ++i) {
      const int d = j + i * sh.J;
      if (ra && i < sh.nr && d < Dv) dS0[(bh * Df + f) * Dv + d] = gr[i];
    }
  }
  if (dz0 && ra && j == 0) dz0[bh * Df + f] = gz;
}

}  // namespace

bool backward_simt_supported(int64_t Df, int64_t Dv) {
  if (Df < 1 || Dv < 1 || Df > kThreads || Dv > kThreads) return false;
  const BwdShape s = bwd_shape((int)Df, (int)Dv);
  return s.J <= 32 && s.nr <= kMaxVals && s.Gc >= 1 && s.nc <= kMaxVals;
}

size_t backward_workspace_bytes(int64_t B, int64_t T, int64_t H) {
  return 2 * (size_t)B * (size_t)T * (size_t)H * sizeof(float);
}

template <typename T>
static cudaError_t launch_backward_t(const void* q, const void* k, const void* v, const void* temp,
                                     const void* dout, const float* S0, const float* z0,
                                     const float* dS_final, const float* dz_final, void* dq,
                                     void* dk, void* dv, void* dtemp, float* dS0, float* dz0,
                                     int64_t B, int64_t T_len, int64_t H, int64_t Df, int64_t Dv,
                                     void* workspace, cudaStream_t stream) {
  const BwdShape sh = bwd_shape((int)Df, (int)Dv);
  float* rden = static_cast<float*>(workspace);
  float* dden = rden + B * T_len * H;
  const size_t smem1 = sizeof(float) * (size_t)(kTok * (6 * Df + 2 * Dv) + 2 * kTok);
  const size_t smem2 = sizeof(float) * (size_t)(kTok * (5 * Df + 2 * Dv + sh.Gc * Dv) + 2 * kTok);
  cudaError_t e = cudaFuncSetAttribute(bwd_forward_kernel<T>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(bwd_reverse_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem2);
  if (e != cudaSuccess) return e;
  bwd_forward_kernel<T><<<(unsigned)(B * H), kThreads, smem1, stream>>>(
      (const T*)q, (const T*)k, (const T*)v, (const T*)temp, (const T*)dout, S0, z0, (T*)dq,
      rden, dden, T_len, H, (int)Df, (int)Dv);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  bwd_reverse_kernel<T><<<(unsigned)(B * H), kThreads, smem2, stream>>>(
      (const T*)q, (const T*)k, (const T*)v, (const T*)temp, (const T*)dout, rden, dden, dS_final,
      dz_final, (T*)dk, (T*)dv, (T*)dtemp, dS0, dz0, T_len, H, (int)Df, (int)Dv);
  return cudaGetLastError();
}

cudaError_t launch_backward_simt(int dtype, const void* q, const void* k, const void* v,
                                 const void* temp, const void* dout, const float* S0,
                                 const float* z0, const float* dS_final, const float* dz_final,
                                 void* dq, void* dk, void* dv, void* dtemp, float* dS0, float* dz0,
                                 int64_t B, int64_t T, int64_t H, int64_t Df, int64_t Dv,
                                 void* workspace, cudaStream_t stream) {
  if (dtype == FAKLA_BF16)
    return launch_backward_t<__nv_bfloat16>(q, k, v, temp, dout, S0, z0, dS_final, dz_final, dq,
                                            dk, dv, dtemp, dS0, dz0, B, T, H, Df, Dv, workspace,
                                            stream);
  return launch_backward_t<float>(q, k, v, temp, dout, S0, z0, dS_final, dz_final, dq, dk, dv,
                                  dtemp, dS0, dz0, B, T, H, Df, Dv, workspace, stream);
}

}  // namespace fakla
