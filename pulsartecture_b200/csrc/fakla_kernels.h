// Internal launcher declarations shared by the kernel files and the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fakla {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
bool encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank,
                       void* base, const cuuint64_t* dims, const cuuint64_t* strides,
                       const cuuint32_t* box, const cuuint32_t* elem_strides,
                       CUtensorMapSwizzle swizzle);

// CUDA-core kernels (simt_kernels.cu)
// act: FAKLA_ACT_*; for FAKLA_ACT_COSSIN, out has 2N columns (cos, then sin)
// scaled by `scale`.
cudaError_t launch_phi_simt(int dtype, const void* x, const void* W, const void* bias,
                            const void* temp, void* out, int64_t rows, int64_t K, int64_t N,
                            int64_t heads, int act, float scale, cudaStream_t stream);
bool mix_supported(int64_t n_maps);
cudaError_t launch_mix_features(int dtype, const void* feats, const void* logits, void* out,
                                int64_t rows, int64_t n_maps, int64_t F, cudaStream_t stream);
bool scan_simt_supported(int64_t Df, int64_t Dv);
size_t scan_simt_smem_bytes(int64_t Df, int64_t Dv);
cudaError_t launch_scan_simt(int dtype, const void* q, const void* k, const void* v,
                             const void* temp, void* out, float* S, float* z, int64_t B,
                             int64_t T, int64_t H, int64_t Df, int64_t Dv, unsigned flags,
                             cudaStream_t stream);
cudaError_t launch_decode(int dtype, const void* q, const void* k, const void* v,
                          const void* temp, void* out, float* S, float* z, int64_t NH,
                          int64_t Df, int64_t Dv, cudaStream_t stream);

// Backward on CUDA cores (simt_backward.cu).
bool backward_simt_supported(int64_t Df, int64_t Dv);
size_t backward_workspace_bytes(int64_t B, int64_t T, int64_t H);
cudaError_t launch_backward_simt(int dtype, const void* q, const void* k, const void* v,
                                 const void* temp, const void* dout, const float* S0,
                                 const float* z0, const float* dS_final, const float* dz_final,
                                 void* dq, void* dk, void* dv, void* dtemp, float* dS0, float* dz0,
                                 int64_t B, int64_t T, int64_t H, int64_t Df, int64_t Dv,
                                 void* workspace, cudaStream_t stream);
cudaError_t launch_phi_backward(int dtype, const void* phi, const void* dphi, void* dpre,
                                int64_t n, cudaStream_t stream);
cudaError_t launch_activation_backward(int dtype, int act, const void* pre, const void* dy,
                                       void* dpre, int64_t rows, int64_t n, float scale,
                                       cudaStream_t stream);
cudaError_t launch_mix_backward(int dtype, const void* feats, const void* logits, const void* dout,
                                void* dfeats, void* dlogits, int64_t rows, int64_t n_maps,
                                int64_t F, cudaStream_t stream);

// Linear-layer gradients on the CUDA cores: C (M, N) row-major =
// sum_k A[m*sam + k*sak] B[n*sbn + k*sbk]; column sums of x (rows, n) through
// colsum_workspace_bytes() of fp32 partial sums (deterministic order).
cudaError_t launch_gemm_strided(int dtype, const void* A, int64_t sam, int64_t sak, const void* Bm, int64_t sbn,
                                int64_t sbk, void* C, int64_t M, int64_t N, int64_t K, cudaStream_t stream);
size_t colsum_workspace_bytes(int64_t rows, int64_t n);
cudaError_t launch_colsum(int dtype, const void* x, void* out, float* partial, int64_t rows, int64_t n,
                          cudaStream_t stream);

// Tensor-core kernels (sm100_phi.cu, sm100_scan.cu); bf16 only.
bool phi_sm100_supported(int64_t rows, int64_t K, int64_t N, int64_t heads);
cudaError_t launch_phi_sm100(const void* x0, const void* x1, const void* W, const void* bias,
                             const void* temp0, const void* temp1, void* out0, void* out1,
                             int64_t rows, int64_t K, int64_t N, int64_t heads, int act,
                             float scale, cudaStream_t stream, int* status, bool* encoded);
// D (M, N) row-major bf16 = A B^T with fp32 accumulation on the tensor cores:
// A is (M, K) row-major, or (K, M) row-major when a_mn; B is (N, K) row-major,
// or (K, N) row-major when b_mn. N % 128 == 0; M and K are free (a ragged K
// reads zeros past its end).
bool gemm_sm100_supported(int64_t M, int64_t N, int64_t K, bool a_mn, bool b_mn);
cudaError_t launch_gemm_sm100(const void* A, bool a_mn, const void* B, bool b_mn, void* D, int64_t M,
                              int64_t N, int64_t K, cudaStream_t stream, int* status, bool* encoded);
// Df = Dv = 128, or 64 (the forward only: run in the 128-wide tiles with the
// second half held at zero).
bool scan_sm100_supported(int64_t B, int64_t T, int64_t H, int64_t Df, int64_t Dv);
// Segments per sequence the scan uses on a device with `sms` SMs (1 = one CTA
// per sequence), and the workspace that takes (0 when G = 1).
int scan_sm100_segments(int64_t B, int64_t T, int64_t H, int sms);
size_t scan_sm100_workspace_bytes(int64_t B, int64_t T, int64_t H, int sms);
// Falls back to one CTA per sequence when `workspace` is smaller than
// scan_sm100_workspace_bytes() (or NULL).
cudaError_t launch_scan_sm100(const void* q, const void* k, const void* v, const void* temp,
                              void* out, float* S, float* z, int64_t B, int64_t T, int64_t H,
                              unsigned flags, void* workspace, size_t workspace_bytes, int sms,
                              cudaStream_t stream, int* status, bool* encoded,
                              int64_t in_row_elems = 0, int64_t head_dim = 128);

// Tensor-core backward (sm100_backward.cu): bf16, Df = Dv = 128 or 64.
bool backward_sm100_supported(int dtype, int64_t B, int64_t T, int64_t H, int64_t Df, int64_t Dv);
size_t backward_sm100_workspace_bytes(int64_t B, int64_t T, int64_t H, int sms);
cudaError_t launch_backward_sm100(const void* q, const void* k, const void* v, const void* temp,
                                  const void* dout, const float* S0, const float* z0,
                                  const float* dS_final, const float* dz_final, void* dq, void* dk,
                                  void* dv, void* dtemp, float* dS0, float* dz0, int64_t B,
                                  int64_t T, int64_t H, int64_t hd, void* workspace, int sms,
                                  cudaStream_t stream, int* status, bool* encoded);
// The backward scans (sm100_scan.cu, run by sm100_backward.cu). mode: 0 the
// normalised forward (optionally writing den (B,T,H) and dden), 1 unnormalised causal with a per-row term `add` added to the kept q.k
// products, 2 unnormalised reversed (suffix state; s >= t kept), 3 as 2 with
// a per-column term. Epilogue of modes 1 and 3: out = (o + coef * vec[chunk]
// + sigma_t mvec) * row_scale, coef = add[t] (mode 1) or 1 (mode 3), sigma_t
// (mode 1 with mvec) = the sum of row t's kept q'.k' + term over all chunks so
// far; dot_out[t] = sum over d of the unscaled row times dot_rows[t]. state_in_T: S (with
// FAKLA_STATE_IN) holds the initial state transposed. Modes 1-3 run one CTA
// per sequence, without temp.
struct ScanBackwardArgs {
  int mode;
  const float* add;
  float* den_out;
  int state_in_T;
  const float* vec;   // modes 1, 3: required; per-chunk sums, accumulated by the scan in
                      // its walking order from vec_init (or 0) before each chunk
  const float* vec_init;  // (B*H, D) or null
  float* vec_total;       // (B*H, D): vec_init + all chunk sums, or null
  int vec_mma;            // mode 3: the chunk sums are v'^T add, formed on the tensor cores
                          // (vec is then not read)
  const float* mvec;  // mode 1: v' was centred by this (B*H, D) vector, or null
  const void* row_scale;
  const void* dot_rows;
  void* dot_out;  // bf16
  // mode 0 with grad_rows: dden_out[t] = -(bf16(grad_rows[t] / den_t) . out_t);
  // the output rows are not stored (out is not used), but dnum_out, if given,
  // receives bf16(grad_rows[t] / den_t)
  const void* grad_rows;
  float* dden_out;
  void* dnum_out;
};
cudaError_t launch_scan_sm100_mode(const void* q, const void* k, const void* v, const void* temp,
                                   void* out, float* S, float* z, int64_t B, int64_t T, int64_t H,
                                   unsigned flags, const ScanBackwardArgs& m, void* workspace,
                                   size_t workspace_bytes, int sms, cudaStream_t stream, int* status,
                                   bool* encoded, int64_t head_dim = 128);
// q/k/v GEMM: out (rows, 2*feat + vdim) = [phi(q) | phi(k) * temp | v] from
// x (rows, K) and W (2*feat + vdim, K).
bool qkv_sm100_supported(int64_t rows, int64_t K, int64_t feat, int64_t vdim, int64_t heads);
cudaError_t launch_qkv_sm100(const void* x, const void* W, const void* bias, const void* temp,
                             void* out, int64_t rows, int64_t K, int64_t feat, int64_t vdim,
                             int64_t heads, cudaStream_t stream, int* status, bool* encoded);

}  // namespace fakla
