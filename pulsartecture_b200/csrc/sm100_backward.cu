// FA-KLA backward on tensor cores (bf16, Df = Dv = 128 or 64): the gradients of
// the recurrence of cpu_kernels.cpp:107-164 (simt_backward.cu states them)
// as four chunked scans of sm100_scan.cu plus small fp32 passes.
//
// With dnum_t = dout_t / den_t, dden_t = -(dout_t . out_t) / den_t, k~ = k temp,
// zb_c = z_0 + sum of k~ over the tokens before chunk c and
// W_c = dz_T + sum of dden_t q_t over the tokens after chunk c:
//
//   1. m = mean of k~ over the first chunk; sums of k~ per chunk (zb is their
//      prefix from z_0, formed by dq's scan), and with temp k~ and k~ - m in bf16
//   2. forward scan (mode 0) of (q, k~, v) -> den_t, dnum_t = bf16(dout_t / den_t),
//      and dden_t from its fp32 output
//   3. (none: dk~'s scan forms W, the suffix of the per-chunk sums of dden q
//      from dz_T, with one extra MMA per chunk, and writes dz_0)
//   4. dq  = causal scan of (q' = dnum, k' = v, v' = k~ - m) with dden_t added
//            to row t of q'k'^T, initial state S_0^T; epilogue + dden_t zb_c
//            + sigma_t m, sigma_t = the sum of row t of (q'k'^T + dden) over
//            every key so far (the chunk's row sum + q'.z', z' = sum of v)
//   5. dk~ = reversed scan of (q' = v, k' = dnum, v' = q) with dden_t added
//            to column t, initial state dS_T^T; epilogue + W_c, times temp_s
//            -> dk; dtemp_s = dk~_s . k_s
//   6. dv  = reversed scan of (q' = k~, k' = q, v' = dnum), initial state
//            dS_T; its final state is dS_0
//
// Precision: for positive feature maps the products behind dq and dk~ cancel
// along the features' common direction (sum_s c_ts k~_s with sum_s w_s c_ts
// = 0), so rounding the operands there would be amplified. Hence dden is
// formed from the same bf16 dnum the scans multiply with (dden_t =
// -bf16(dnum_t) . out_t, out_t in fp32); the unnormalised scans carry their
// state as bf16 hi + lo; and where an operand is not an exact bf16 input
// (k~ = k temp in dq) it enters centred, so that only the small deviations
// k~ - m are rounded while the common part m is added in fp32 (sigma, zb).
// Without temp, v' = k is exact and is not centred; dk~ multiplies the exact
// q and needs no centring.
//
// Every intermediate is (B, T, H, .) like the inputs, so the scans take
// them through the same tensor maps as the forward.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fakla.h"
#include "fakla_common.cuh"
#include "fakla_kernels.h"

namespace fakla {
namespace {

constexpr int D = 128;  // the widest head; heads of 64 use the same kernels
constexpr int C = 128;  // scan chunk (tokens)

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = u;
}

// s[bh][c][f] = scale * the sum over the tokens t of chunk c of w_t x_t[f],
// w = wf (fp32), else wh (bf16), else 1; with wx, also wx_t = bf16(w_t x_t),
// and with wxc, wxc_t = bf16(w_t x_t - mc[bh]) (w_t x_t in fp32). Grid (nchunks,
// B*H), 256 threads: hd/8 per token row (8 features each, 16-byte loads) over
// 256/(hd/8) tokens at a time, then a shared memory reduction over the token
// slots.
__global__ void bwd_chunk_sums_kernel(const __nv_bfloat16* __restrict__ x,
                                      const float* __restrict__ wf,
                                      const __nv_bfloat16* __restrict__ wh, float* __restrict__ s,
                                      __nv_bfloat16* __restrict__ wx, const float* __restrict__ mc,
                                      __nv_bfloat16* __restrict__ wxc, int T, int H, int hd,
                                      float scale) {
  __shared__ float red[32][D + 4];
  const int parts = hd / 8;
  const int nslots = 256 / parts;
  const int c = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int part = threadIdx.x % parts;  // features 8 part .. 8 part + 7
  const int slot = threadIdx.x / parts;  // token slot
  const int t1 = min(T, c * C + C);
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  float mv[8];  // the centring vector's 8 features (with wxc)
#pragma unroll
  for (int e = 0; e < 8; ++e) mv[e] = wxc != nullptr ? mc[(int64_t)bh * hd + part * 8 + e] : 0.f;
  // two tokens per step, both loads issued before either is used
  for (int t = c * C + slot; t < t1; t += 2 * nslots) {
    const bool two = t + nslots < t1;
    const int64_t r0 = ((int64_t)b * T + t) * H + h;
    const int64_t r1 = two ? r0 + (int64_t)nslots * H : r0;
    const float w0 = wf != nullptr ? wf[r0] : (wh != nullptr ? __bfloat162float(wh[r0]) : 1.f);
    const float w1 = !two ? 0.f : (wf != nullptr ? wf[r1] : (wh != nullptr ? __bfloat162float(wh[r1]) : 1.f));
    float x0[8], x1[8];
    load8(x + r0 * hd + part * 8, x0);
    load8(x + r1 * hd + part * 8, x1);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = fmaf(w1, x1[e], fmaf(w0, x0[e], acc[e]));
    if (wx != nullptr) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        x0[e] *= w0;
        x1[e] *= w1;
      }
      store8(wx + r0 * hd + part * 8, x0);
      if (two) store8(wx + r1 * hd + part * 8, x1);
      if (wxc != nullptr) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          x0[e] -= mv[e];
          x1[e] -= mv[e];
        }
        store8(wxc + r0 * hd + part * 8, x0);
        if (two) store8(wxc + r1 * hd + part * 8, x1);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) red[slot][part * 8 + e] = acc[e];
  __syncthreads();
  if (threadIdx.x < hd) {
    float v = 0.f;
    for (int i = 0; i < nslots; ++i) v += red[i][threadIdx.x];
    s[((int64_t)bh * gridDim.x + c) * hd + threadIdx.x] = v * scale;
  }
}

struct BwdLayout {
  size_t dden, dnum, kt, kc, zb, mk, scan, total;
};

BwdLayout bwd_layout(int64_t B, int64_t T, int64_t H, bool temp, int sms) {
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t rows = (size_t)(B * T * H);
  const size_t nch = (size_t)((T + C - 1) / C);
  const size_t chunk_vecs = up((size_t)(B * H) * nch * D * 4);
  BwdLayout l;
  size_t o = 0;
  l.dden = o; o += up(rows * 4);
  l.dnum = o; o += up(rows * D * 2);
  l.kt = o;   o += temp ? up(rows * D * 2) : 0;
  l.kc = o;   o += temp ? up(rows * D * 2) : 0;
  l.zb = o;   o += chunk_vecs;
  l.mk = o;   o += up((size_t)(B * H) * D * 4);
  l.scan = o; o += up(scan_sm100_workspace_bytes(B, T, H, sms));
  l.total = o;
  return l;
}

}  // namespace

bool backward_sm100_supported(int dtype, int64_t B, int64_t T, int64_t H, int64_t Df, int64_t Dv) {
  return dtype == FAKLA_BF16 && Df == Dv && (Df == D || Df == 64) && scan_sm100_supported(B, T, H, Df, Dv) &&
         B * T * H <= (int64_t)INT32_MAX;
}

size_t backward_sm100_workspace_bytes(int64_t B, int64_t T, int64_t H, int sms) {
  // sized for the temp case (the k~ buffers) and heads of 128; smaller heads
  // and calls without temp use a part of it
  return bwd_layout(B, T, H, true, sms).total;
}

cudaError_t launch_backward_sm100(const void* q, const void* k, const void* v, const void* temp,
                                  const void* dout, const float* S0, const float* z0,
                                  const float* dS_final, const float* dz_final, void* dq, void* dk,
                                  void* dv, void* dtemp, float* dS0, float* dz0, int64_t B,
                                  int64_t T, int64_t H, int64_t hd, void* workspace, int sms,
                                  cudaStream_t stream, int* status, bool* encoded) {
  const BwdLayout l = bwd_layout(B, T, H, temp != nullptr, sms);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto* dden = reinterpret_cast<float*>(ws + l.dden);
  auto* dnum = reinterpret_cast<__nv_bfloat16*>(ws + l.dnum);
  auto* kt = temp != nullptr ? reinterpret_cast<__nv_bfloat16*>(ws + l.kt) : nullptr;
  auto* kc = temp != nullptr ? reinterpret_cast<__nv_bfloat16*>(ws + l.kc) : nullptr;
  auto* zb = reinterpret_cast<float*>(ws + l.zb);
  auto* mk = reinterpret_cast<float*>(ws + l.mk);
  void* scan_ws = ws + l.scan;
  const size_t scan_bytes = l.total - l.scan;
  const int nch = (int)((T + C - 1) / C);
  const dim3 cgrid((unsigned)nch, (unsigned)(B * H));
  const auto* kh = static_cast<const __nv_bfloat16*>(k);
  const auto* th = static_cast<const __nv_bfloat16*>(temp);
  cudaError_t e;

  // 1. with temp the centring vector m (the first chunk's mean of k~), then
  // the sums of k~ per chunk (dq's scan turns them into zb as it walks the
  // chunks), and with temp k~ and k~ - m in bf16
  if (temp != nullptr) {
    bwd_chunk_sums_kernel<<<dim3(1u, (unsigned)(B * H)), 256, 0, stream>>>(
        kh, nullptr, th, mk, nullptr, nullptr, nullptr, (int)T, (int)H, (int)hd,
        1.f / (float)(T < C ? T : C));
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  bwd_chunk_sums_kernel<<<cgrid, 256, 0, stream>>>(kh, nullptr, th, zb, kt, mk, kc, (int)T, (int)H,
                                                   (int)hd, 1.f);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;

  // 2. forward: dden and dnum (no output rows)
  ScanBackwardArgs m{};
  m.mode = 0;
  m.grad_rows = dout;
  m.dden_out = dden;
  m.dnum_out = dnum;
  const unsigned in0 = S0 != nullptr ? FAKLA_STATE_IN : 0u;
  // k~ is precomputed: the scan then skips its in-tile temp scaling, which
  // the P warps would otherwise do on the critical path of every chunk
  const void* ktil = temp != nullptr ? (const void*)kt : k;
  e = launch_scan_sm100_mode(q, ktil, v, nullptr, nullptr, const_cast<float*>(S0),
                             const_cast<float*>(z0), B, T, H, in0, m, scan_ws, scan_bytes, sms,
                             stream, status, encoded, hd);
  if (e != cudaSuccess) return e;


  // 4. dq
  m = ScanBackwardArgs{};
  m.mode = 1;
  m.add = dden;
  m.vec = zb;
  m.vec_init = z0;
  m.mvec = temp != nullptr ? mk : nullptr;
  m.state_in_T = 1;
  e = launch_scan_sm100_mode(dnum, v, temp != nullptr ? (const void*)kc : k, nullptr, dq,
                             const_cast<float*>(S0), nullptr, B, T, H, in0, m, nullptr, 0, sms,
                             stream, status, encoded, hd);
  if (e != cudaSuccess) return e;

  // 5. dk (and dtemp); before dv, whose final state may overwrite dS_T in place
  m = ScanBackwardArgs{};
  m.mode = 3;
  m.add = dden;
  m.vec_mma = 1;  // W: the chunk sums of dden q come from the scan's own MMAs
  m.vec_init = dz_final;
  m.vec_total = dz0;
  m.state_in_T = 1;
  m.row_scale = temp;
  if (temp != nullptr && dtemp != nullptr) {
    m.dot_rows = k;
    m.dot_out = dtemp;
  }
  const unsigned fk = dS_final != nullptr ? FAKLA_STATE_IN : 0u;
  e = launch_scan_sm100_mode(v, dnum, q, nullptr, dk, const_cast<float*>(dS_final), nullptr, B, T,
                             H, fk, m, nullptr, 0, sms, stream, status, encoded, hd);
  if (e != cudaSuccess) return e;

  // 6. dv (and dS_0 as the reversed scan's final state)
  float* Sv = nullptr;
  unsigned fv = 0;
  if (dS0 != nullptr) {
    Sv = dS0;
    fv |= FAKLA_STATE_OUT;
    if (dS_final != nullptr) {
      if (dS_final != dS0 &&
          (e = cudaMemcpyAsync(dS0, dS_final, (size_t)(B * H) * hd * hd * sizeof(float),
                               cudaMemcpyDeviceToDevice, stream)) != cudaSuccess)
        return e;
      fv |= FAKLA_STATE_IN;
    }
  } else if (dS_final != nullptr) {
    Sv = const_cast<float*>(dS_final);
    fv |= FAKLA_STATE_IN;
  }
  m = ScanBackwardArgs{};
  m.mode = 2;
  return launch_scan_sm100_mode(ktil, q, dnum, nullptr, dv, Sv, nullptr, B, T, H, fv, m, nullptr, 0,
                                sms, stream, status, encoded, hd);
}

}  // namespace fakla
