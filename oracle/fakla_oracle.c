/*
 * FA-KLA oracle: a plain-C restatement of the reference's CPU algorithm.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA library in
 * pulsartecture_b200/csrc; the product never links, loads or calls it. Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use it.
 *
 * Parity pin: the restatement is checked against the reference's own
 * fa_kla_attention_cpu (ultra_rwka/backend/cpp/cpu/cpu_kernels.cpp:36-170),
 * compiled in place by oracle/build_ref.py, and against the golden fixtures in
 * tests/golden/ that were generated from that compiled reference plus the
 * reference's Python LearnablePositiveMap (tests/golden/make_golden.py).
 *
 * Layouts (row-major, contiguous), as in the reference (cpu_kernels.cpp:88-99):
 *   q, k : (B, T, H, Df)     v, out : (B, T, H, Dv)     temp : (B, T, H)
 * State (an extension; the reference keeps it in locals, cpu_kernels.cpp:78-79):
 *   S : (B, H, Df, Dv)       z : (B, H, Df)
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define FAKLA_ORACLE_EPS 1e-12 /* K_EPSILON, cpu_kernels.cpp:22 */

/* phi(x) = elu(x W^T + b) + 1 over `rows` rows, double accumulation.
 * Follows LearnablePositiveMap.forward (ultra_rwka/kernels/feature_maps.py:
 * 259-268) with num_layers=1 (one nn.Linear, feature_maps.py:224) and the
 * 'elu+1' activation (feature_maps.py:247-248). W is nn.Linear's weight,
 * shape (feat_dim, in_dim). bias may be NULL (use_bias=False).
 * If temp is non-NULL (shape (rows, heads)), output column n of row r is
 * additionally multiplied by temp[r, n / (feat_dim/heads)] -- the k-side
 * temperature scaling k~ = k*temp of cpu_kernels.cpp:121-123 applied per head. */
void fakla_oracle_phi_f64(const double* x, const double* W, const double* bias,
                          const double* temp, double* out, int64_t rows,
                          int64_t in_dim, int64_t feat_dim, int64_t heads) {
  const int64_t m = heads > 0 ? feat_dim / heads : feat_dim;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const double* xr = x + r * in_dim;
    for (int64_t n = 0; n < feat_dim; ++n) {
      const double* wn = W + n * in_dim;
      double acc = bias ? bias[n] : 0.0;
      for (int64_t i = 0; i < in_dim; ++i) acc += xr[i] * wn[i];
      double phi = (acc > 0.0 ? acc : expm1(acc)) + 1.0; /* F.elu(alpha=1) + 1 */
      if (temp) phi *= temp[r * heads + n / m];
      out[r * feat_dim + n] = phi;
    }
  }
}

/* The FA-KLA causal recurrence in double precision, with injected state.
 * Per (b,h), for t = 0..T-1 (cpu_kernels.cpp:107-164):
 *   k~ = k_t * temp_t            (121-123)
 *   z += k~                      (128-130)
 *   S += k~ (outer) v_t          (135-138)
 *   num = q_t^T S                (152)
 *   den = q_t . z                (156)
 *   out_t = num * 1/(den + eps)  (159-162)
 * The output at t includes token t (inclusive causal).
 * S0/z0: initial state or NULL for zeros (the reference always starts at zero,
 * cpu_kernels.cpp:78-79). S1/z1: final state or NULL. temp NULL = all ones.
 * Returns 0, or -1 (nothing written) for head dims outside [1, 256]. */
int fakla_oracle_attention_f64(const double* q, const double* k, const double* v,
                               const double* temp, double* out, const double* S0,
                               const double* z0, double* S1, double* z1, int64_t B,
                               int64_t T, int64_t H, int64_t Df, int64_t Dv) {
  if (Df < 1 || Dv < 1 || Df > 256 || Dv > 256) return -1;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t bh = 0; bh < B * H; ++bh) {
    const int64_t b = bh / H, h = bh % H;
    double* S = (double*)malloc(sizeof(double) * (size_t)(Df * Dv + 2 * Df + Dv));
    double* z = S + Df * Dv;
    double* kt = z + Df;
    double* num = kt + Df;
    if (S0) memcpy(S, S0 + bh * Df * Dv, sizeof(double) * Df * Dv);
    else memset(S, 0, sizeof(double) * Df * Dv);
    if (z0) memcpy(z, z0 + bh * Df, sizeof(double) * Df);
    else memset(z, 0, sizeof(double) * Df);
    for (int64_t t = 0; t < T; ++t) {
      const int64_t row = (b * T + t) * H + h;
      const double* qt = q + row * Df;
      const double* kk = k + row * Df;
      const double* vt = v + row * Dv;
      const double tp = temp ? temp[row] : 1.0;
      for (int64_t f = 0; f < Df; ++f) kt[f] = kk[f] * tp;
      for (int64_t f = 0; f < Df; ++f) z[f] += kt[f];
      for (int64_t f = 0; f < Df; ++f)
        for (int64_t d = 0; d < Dv; ++d) S[f * Dv + d] += kt[f] * vt[d];
      for (int64_t d = 0; d < Dv; ++d) num[d] = 0.0;
      for (int64_t f = 0; f < Df; ++f)
        for (int64_t d = 0; d < Dv; ++d) num[d] += qt[f] * S[f * Dv + d];
      double den = 0.0;
      for (int64_t f = 0; f < Df; ++f) den += qt[f] * z[f];
      const double inv = 1.0 / (den + FAKLA_ORACLE_EPS);
      for (int64_t d = 0; d < Dv; ++d) out[row * Dv + d] = num[d] * inv;
    }
    if (S1) memcpy(S1 + bh * Df * Dv, S, sizeof(double) * Df * Dv);
    if (z1) memcpy(z1 + bh * Df, z, sizeof(double) * Df);
    free(S);
  }
  return 0;
}

/* Same recurrence in float arithmetic, statement for statement as the
 * reference's fp32 instantiation (scalar_t = float, cpu_kernels.cpp:82-162):
 * float k~ buffer, float S/z, float reciprocal of (den + 1e-12f). Only the
 * summation order of the BLAS calls (matmul/dot) may differ.
 * Returns 0, or -1 (nothing written) for head dims outside [1, 256]. */
int fakla_oracle_attention_f32(const float* q, const float* k, const float* v,
                               const float* temp, float* out, const float* S0,
                               const float* z0, float* S1, float* z1, int64_t B,
                               int64_t T, int64_t H, int64_t Df, int64_t Dv) {
  if (Df < 1 || Dv < 1 || Df > 256 || Dv > 256) return -1;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t bh = 0; bh < B * H; ++bh) {
    const int64_t b = bh / H, h = bh % H;
    float* S = (float*)malloc(sizeof(float) * (size_t)(Df * Dv + 2 * Df + Dv));
    float* z = S + Df * Dv;
    float* kt = z + Df;
    float* num = kt + Df;
    if (S0) memcpy(S, S0 + bh * Df * Dv, sizeof(float) * Df * Dv);
    else memset(S, 0, sizeof(float) * Df * Dv);
    if (z0) memcpy(z, z0 + bh * Df, sizeof(float) * Df);
    else memset(z, 0, sizeof(float) * Df);
    for (int64_t t = 0; t < T; ++t) {
      const int64_t row = (b * T + t) * H + h;
      const float* qt = q + row * Df;
      const float* kk = k + row * Df;
      const float* vt = v + row * Dv;
      const float tp = temp ? temp[row] : 1.0f;
      for (int64_t f = 0; f < Df; ++f) kt[f] = kk[f] * tp;
      for (int64_t f = 0; f < Df; ++f) z[f] += kt[f];
      for (int64_t f = 0; f < Df; ++f)
        for (int64_t d = 0; d < Dv; ++d) S[f * Dv + d] += kt[f] * vt[d];
      for (int64_t d = 0; d < Dv; ++d) num[d] = 0.0f;
      for (int64_t f = 0; f < Df; ++f)
        for (int64_t d = 0; d < Dv; ++d) num[d] += qt[f] * S[f * Dv + d];
      float den = 0.0f;
      for (int64_t f = 0; f < Df; ++f) den += qt[f] * z[f];
      const float inv = 1.0f / (den + 1e-12f);
      for (int64_t d = 0; d < Dv; ++d) out[row * Dv + d] = num[d] * inv;
    }
    if (S1) memcpy(S1 + bh * Df * Dv, S, sizeof(float) * Df * Dv);
    if (z1) memcpy(z1 + bh * Df, z, sizeof(float) * Df);
    free(S);
  }
  return 0;
}

/* Round-to-nearest-even float -> bfloat16 -> float, as the device's
 * __float2bfloat16_rn does for finite values. Used to emulate the bf16 input
 * contract (inputs are bf16; the oracle computes on their exact values). */
void fakla_oracle_round_bf16(float* x, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    uint32_t u;
    memcpy(&u, &x[i], 4);
    if ((u & 0x7f800000u) == 0x7f800000u) continue; /* inf/nan unchanged */
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    memcpy(&x[i], &u, 4);
  }
}
