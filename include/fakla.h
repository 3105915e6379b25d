/*
 * fakla.h -- C ABI of the B200 (sm_100a) FA-KLA library, libfakla.so.
 *
 * FA-KLA is Ultra-RWKA's causal, temperature-modulated kernelized linear
 * attention. For every (batch b, head h) sequence and token t:
 *
 *   k~_t  = phi(k_t) * temp_t
 *   z_t   = z_{t-1} + k~_t                        (normaliser, fp32)
 *   S_t   = S_{t-1} + k~_t (outer) v_t            (state, fp32, Df x Dv)
 *   out_t = (phi(q_t)^T S_t) / (phi(q_t) . z_t + 1e-12)
 *
 * with phi(x) = elu(x W^T + b) + 1 (LearnablePositiveMap, one linear layer).
 *
 * Conventions shared by every entry point:
 *  - All pointers are device pointers unless stated otherwise. Tensors are
 *    dense row-major (C-contiguous) in the layouts given per function. The
 *    activations use the reference's (B, T, H, D) layout.
 *  - `dtype` selects the element type of the activations (q, k, v, temp, out,
 *    W, bias): FAKLA_F32 or FAKLA_BF16. The state S, z is always fp32, and all
 *    accumulation is fp32.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream). Every call is
 *    asynchronous and stream-ordered; the library keeps no per-call host state,
 *    so calls on different streams may run concurrently when their buffers are
 *    disjoint.
 *  - The caller owns every buffer. Functions that need temporary device memory
 *    take a caller-provided `workspace` of at least the size reported by the
 *    matching *_workspace_bytes() query.
 *  - Return value: FAKLA_OK or a fakla_status error code; nothing is launched
 *    on error. fakla_last_error() gives a message for the calling thread.
 *  - There is no CPU path: the library requires an sm_100 device.
 *
 * Each declaration names the reference interface it replaces
 * (0xAEC/Pulsartecture, paths relative to the repository root).
 */
#ifndef FAKLA_H_
#define FAKLA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FAKLA_VERSION 1

typedef enum fakla_dtype {
  FAKLA_F32 = 0,
  FAKLA_BF16 = 1
} fakla_dtype;

typedef enum fakla_status {
  FAKLA_OK = 0,
  FAKLA_ERR_INVALID_ARG = 1, /* null pointer, non-positive size, bad flag */
  FAKLA_ERR_UNSUPPORTED = 2, /* well-formed but outside the implemented set */
  FAKLA_ERR_ALIGNMENT = 3,   /* a pointer lacks the 16-byte alignment needed */
  FAKLA_ERR_CUDA = 4,        /* CUDA runtime error while launching */
  FAKLA_ERR_TIMEOUT = 5,     /* a bounded device-side wait expired */
  FAKLA_ERR_WORKSPACE = 6,   /* workspace missing or smaller than required */
  FAKLA_ERR_NO_DEVICE = 7    /* current device is not an sm_100 GPU */
} fakla_status;

/* Flags for the stateful entry points. */
#define FAKLA_STATE_IN 1u  /* read the initial (S, z) from the S/z buffers   */
#define FAKLA_STATE_OUT 2u /* write the final (S, z) to the S/z buffers      */

/* Human-readable name of a status code (static storage). */
const char* fakla_strerror(int status);

/* Detail message of the last failing call on this host thread ("" if none). */
const char* fakla_last_error(void);

/* Library ABI version (FAKLA_VERSION). */
int fakla_version(void);

/*
 * fakla_attention -- FA-KLA on already feature-mapped q and k.
 *
 * Replaces: ultra_rwka.backend.interface.fa_kla_attention(q_mapped, k_mapped,
 *   v_reshaped, temp), called at ultra_rwka/attention/tm_kla.py:319; its
 *   native kernels fa_kla_attention_cpu (ultra_rwka/backend/cpp/cpu/
 *   cpu_kernels.cpp:36) and fa_kla_attention_cuda (ultra_rwka/backend/cuda/
 *   fa_kla/kernel.cu:627).
 *
 *   q_mapped, k_mapped : (B, T, H, Df)   v : (B, T, H, Dv)
 *   temp               : (B, T, H), or NULL for all ones (tm_kla.py:303-306)
 *   out                : (B, T, H, Dv), written
 *   S : (B, H, Df, Dv) fp32, z : (B, H, Df) fp32 -- optional state (NULL with
 *       flags 0 reproduces the reference exactly: zero initial state, no
 *       state returned). FAKLA_STATE_IN reads the initial state from S/z;
 *       FAKLA_STATE_OUT overwrites S/z with the final state. S and z must be
 *       both NULL or both non-NULL.
 * Implemented: Df, Dv in [1, 256] on the general path; the tensor-core path
 * serves dtype BF16 with Df == Dv == 128 and all pointers 16-byte aligned.
 */
int fakla_attention(const void* q_mapped, const void* k_mapped, const void* v,
                    const void* temp, void* out, float* S, float* z, int64_t B,
                    int64_t T, int64_t H, int64_t Df, int64_t Dv, int dtype,
                    unsigned flags, void* workspace, size_t workspace_bytes,
                    void* stream);

/*
 * Workspace that lets fakla_attention split long sequences into segments run
 * by separate CTAs (when B*H alone would leave SMs idle): one fp32 (S, z)
 * record per segment. 0 when the call would not be split on the current
 * device. The workspace is optional: with less (or NULL) the scan runs one
 * CTA per (b, h) sequence, with the same result up to fp32 rounding.
 */
size_t fakla_attention_workspace_bytes(int64_t B, int64_t T, int64_t H,
                                       int64_t Df, int64_t Dv, int dtype);

/*
 * fakla_phi -- the positive feature map phi(x) = elu(x W^T + bias) + 1.
 *
 * Replaces: LearnablePositiveMap.forward (ultra_rwka/kernels/feature_maps.py:
 *   259-268) for num_layers=1, activation='elu+1' (feature_maps.py:224,248).
 *
 *   x    : (rows, in_dim)          W : (feat_dim, in_dim) (nn.Linear weight)
 *   bias : (feat_dim) or NULL      out : (rows, feat_dim), written
 *   temp : (rows, heads) or NULL; when given, output column n of row r is
 *          multiplied by temp[r, n / (feat_dim / heads)] (the k-side k*temp
 *          of cpu_kernels.cpp:121-123 folded into the map).
 */
int fakla_phi(const void* x, const void* W, const void* bias, const void* temp,
              void* out, int64_t rows, int64_t in_dim, int64_t feat_dim,
              int64_t heads, int dtype, void* stream);

/*
 * fakla_attention_backward -- gradients of fakla_attention.
 *
 * Reference: none -- the reference's FA-KLA has no backward (its gradient
 * test, tests/backend/test_fa_kla_gradients.py, is empty). This is the
 * derivative of the recurrence of cpu_kernels.cpp:107-164 (see fakla.h top):
 * with dnum_t = dout_t / den_t, dden_t = -(q_t^T S_t dout_t) / den_t^2 and
 * G_s = dS_final + sum_{t>=s} q_t dnum_t^T, g_s = dz_final + sum_{t>=s} q_t dden_t:
 *   dq_t = S_t dnum_t + z_t dden_t,  dk~_s = G_s v_s + g_s,  dv_s = G_s^T k~_s,
 *   dk_s = dk~_s temp_s,  dtemp_s = dk~_s . k_s,  dS0 = G_0,  dz0 = g_0.
 *
 *   q_mapped, k_mapped, v, temp : the forward's inputs (temp may be NULL)
 *   dout     : (B, T, H, Dv) gradient of the output
 *   S0, z0   : the forward's initial state, or NULL for zero
 *   dS_final, dz_final : gradient of the forward's final state, or NULL
 *   dq, dk   : (B, T, H, Df) written   dv : (B, T, H, Dv) written
 *   dtemp    : (B, T, H) written, or NULL     dS0, dz0 : written, or NULL
 * Gradients have the activation dtype; all accumulation is fp32. Needs a
 * workspace of fakla_attention_backward_workspace_bytes() (16-byte aligned for
 * the bf16 Df = Dv = 128 tensor-core path; with less, or unaligned tensors, the
 * call takes the CUDA-core path).
 */
int fakla_attention_backward(const void* q_mapped, const void* k_mapped, const void* v,
                             const void* temp, const void* dout, const float* S0,
                             const float* z0, const float* dS_final, const float* dz_final,
                             void* dq, void* dk, void* dv, void* dtemp, float* dS0, float* dz0,
                             int64_t B, int64_t T, int64_t H, int64_t Df, int64_t Dv,
                             int dtype, void* workspace, size_t workspace_bytes, void* stream);

size_t fakla_attention_backward_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t Df,
                                                int64_t Dv, int dtype);

/*
 * fakla_phi_backward -- gradient of the elu+1 activation from its output:
 * dpre = dphi * min(phi, 1)  (elu'(x) = 1 for x > 0, e^x = phi for x <= 0).
 *
 * Reference: none (no backward in the reference); the derivative of
 * F.elu(x) + 1 at feature_maps.py:248.
 *   phi, dphi, dpre : n elements each (dpre may alias dphi)
 */
int fakla_phi_backward(const void* phi, const void* dphi, void* dpre, int64_t n, int dtype,
                       void* stream);

/*
 * fakla_activation_backward -- gradient of a fakla_feature_map activation
 * from its pre-activation p = x W^T + bias: dpre = dy * act'(p); for
 * FAKLA_ACT_COSSIN, dy is (rows, 2 * n) and
 * dpre = scale * (cos p * dy[:, n + j] - sin p * dy[:, j]).
 *
 * Reference: none (no backward in the reference); derivatives of the
 * activations listed at fakla_activation.
 *   pre : (rows, n)   dy : (rows, n), or (rows, 2n) for COSSIN   dpre : (rows, n)
 */
int fakla_activation_backward(const void* pre, const void* dy, void* dpre, int64_t rows,
                              int64_t n, int act, float scale, int dtype, void* stream);

/*
 * fakla_linear_backward -- gradients of one linear layer y = x W^T + b from
 * dpre = dL/dy (for a feature map: the output of fakla_phi_backward or
 * fakla_activation_backward):
 *   dx = dpre W  (rows, in_dim)    dW = dpre^T x  (n_out, in_dim)    db = sum over rows of dpre  (n_out)
 *
 * Reference: none (no backward in the reference); the input, weight and bias
 * gradients of the nn.Linear inside LearnablePositiveMap (ultra_rwka/kernels/
 * feature_maps.py:224-232), GateNet and TemperatureFunction, and of the
 * projection of RandomFourierFeatures / OrthogonalRandomFeatures.
 *   x : (rows, in_dim)   W : (n_out, in_dim)   dpre : (rows, n_out)
 *   dx, dW, db : written when non-NULL (x may be NULL without dW, W without dx)
 * db needs a workspace of fakla_linear_backward_workspace_bytes() (fp32
 * partial sums, added in a fixed order); dx and dW need none. bf16 with
 * in_dim % 128 == 0, n_out % 8 == 0 and 16-byte aligned pointers runs both
 * products on the tensor cores (fp32 accumulation); other shapes and fp32 run
 * on the CUDA cores.
 */
int fakla_linear_backward(const void* x, const void* W, const void* dpre, void* dx, void* dW,
                          void* db, int64_t rows, int64_t in_dim, int64_t n_out, int dtype,
                          void* workspace, size_t workspace_bytes, void* stream);

size_t fakla_linear_backward_workspace_bytes(int64_t rows, int64_t in_dim, int64_t n_out,
                                             int dtype);

/*
 * fakla_mix_features_backward -- gradients of fakla_mix_features.
 * With w = softmax(logits) (rounded to dtype as in the forward):
 *   dfeats[i] = w_i dout,  dlogits_i = w_i (dw_i - sum_j w_j dw_j),  dw_i = dout . feats[i]
 *
 * Reference: none (no backward in the reference); the derivative of
 * KernelFeatureMixer's combination (mixer.py:134-150).
 *   feats : (n_maps, rows, feat_dim)  logits : (rows, n_maps)  dout : (rows, feat_dim)
 *   dfeats : like feats, or NULL      dlogits : like logits, or NULL
 */
int fakla_mix_features_backward(const void* feats, const void* logits, const void* dout,
                                void* dfeats, void* dlogits, int64_t rows, int64_t n_maps,
                                int64_t feat_dim, int dtype, void* stream);

/* Output activation of fakla_feature_map. */
typedef enum {
  FAKLA_ACT_ELU1 = 0,     /* elu(x) + 1                        (feature_maps.py:248) */
  FAKLA_ACT_RELU = 1,     /* max(x, 0)                         (feature_maps.py:250) */
  FAKLA_ACT_SOFTPLUS = 2, /* log(1 + e^x), x for x > 20        (feature_maps.py:252) */
  FAKLA_ACT_GELU = 3,     /* x/2 (1 + erf(x/sqrt 2))           (feature_maps.py:254, 239) */
  FAKLA_ACT_IDENTITY = 4, /* x                                 (gate logits, mixer.py:60-66) */
  FAKLA_ACT_SIGMOID = 5,  /* 1 / (1 + e^-x)                    (tm_kla.py:89) */
  FAKLA_ACT_ABS = 6,      /* |x|                               (tm_kla.py:89) */
  FAKLA_ACT_COSSIN = 7    /* [cos x, sin x] * scale            (feature_maps.py:30-37) */
} fakla_activation;

/*
 * fakla_feature_map -- one linear layer with its output activation,
 * out = act(x W^T + bias).
 *
 * Replaces: one layer of LearnablePositiveMap's MLP and its final activation
 *   (ultra_rwka/kernels/feature_maps.py:234-268, all four activations; hidden
 *   layers use FAKLA_ACT_GELU, feature_maps.py:239); the projection of
 *   RandomFourierFeatures / OrthogonalRandomFeatures (_rff_forward_script,
 *   feature_maps.py:30-37, with W given transposed); the layers of GateNet
 *   (kernels/mixer.py:11-66) and of TemperatureFunction (attention/
 *   tm_kla.py:17-107).
 *
 *   x    : (rows, in_dim)    W : (n_out, in_dim) (nn.Linear weight layout)
 *   bias : (n_out) or NULL
 *   out  : (rows, n_out), or (rows, 2 * n_out) for FAKLA_ACT_COSSIN: column n
 *          holds scale * cos(p_n) and column n_out + n holds scale * sin(p_n),
 *          p = x W^T + bias. `scale` is ignored by the other activations.
 * The tensor-core path serves BF16 with in_dim % 64 == 0, n_out % 128 == 0
 * and 16-byte aligned pointers; other shapes and F32 run on CUDA cores
 * (n_out <= 16 with in_dim % 8 == 0, e.g. gate logits, one warp per row).
 */
int fakla_feature_map(const void* x, const void* W, const void* bias, void* out,
                      int64_t rows, int64_t in_dim, int64_t n_out, int act,
                      float scale, int dtype, void* stream);

/*
 * fakla_mix_features -- the KernelFeatureMixer combination
 * out = sum_i softmax(logits)_i * feats_i.
 *
 * Replaces: the softmax gate and the weighted sum of KernelFeatureMixer
 *   (ultra_rwka/kernels/mixer.py:118-150 / 236-248): the softmax runs in fp32
 *   and its weights are rounded to `dtype` before the sum, as the reference's
 *   softmax(logits.float()).to(logits.dtype) does.
 *
 *   feats  : (n_maps, rows, feat_dim), map i's features in slice i
 *   logits : (rows, n_maps) gate logits     out : (rows, feat_dim)
 */
int fakla_mix_features(const void* feats, const void* logits, void* out, int64_t rows,
                       int64_t n_maps, int64_t feat_dim, int dtype, void* stream);

/*
 * fakla_prefill -- feature map and FA-KLA in one call (the phi GEMM, then
 * the chunked scan as its programmatic dependent launch): the hot path of
 * TMLinKernelAttn.forward from the projected q/k/v onward (ultra_rwka/
 * attention/tm_kla.py:268-332: feature_mapper on q and k, head split,
 * temperature, fa_kla_attention).
 *
 *   q, k : (B, T, in_dim)  projected queries/keys, in_dim = H_total * Dk; the
 *          feature map mixes all heads of a row, so every row is read whole.
 *   W    : (H * M, in_dim), bias : (H * M) or NULL -- the rows of the map that
 *          produce the H heads computed by this call (all heads, or a
 *          contiguous shard of heads on a multi-GPU run).
 *   v    : (B, T, H, Dv)   temp : (B, T, H) or NULL   out : (B, T, H, Dv)
 *   S, z, flags : as fakla_attention, with Df = M.
 * Workspace: fakla_prefill_workspace_bytes() = phi(q) and phi(k) buffers
 * (required) followed by the scan's segment records (optional, as in
 * fakla_attention_workspace_bytes).
 */
int fakla_prefill(const void* q, const void* k, const void* v, const void* temp,
                  const void* W, const void* bias, void* out, float* S, float* z,
                  int64_t B, int64_t T, int64_t in_dim, int64_t H, int64_t M,
                  int64_t Dv, int dtype, unsigned flags, void* workspace,
                  size_t workspace_bytes, void* stream);

size_t fakla_prefill_workspace_bytes(int64_t B, int64_t T, int64_t in_dim,
                                     int64_t H, int64_t M, int64_t Dv, int dtype);

/*
 * fakla_qkv_prefill -- the projections, the feature map and FA-KLA from the
 * layer input: TMLinKernelAttn.forward (ultra_rwka/attention/tm_kla.py:
 * 255-332) with q = x Wq^T + bq, k = x Wk^T + bk, v = x Wv^T + bv and
 * phi(y) = elu(y Wphi^T + bphi) + 1, the projections folded into the map:
 *   phi(q) = elu(x (Wphi Wq)^T + (Wphi bq + bphi)) + 1   (same for k).
 * One GEMM computes [phi(q) | phi(k) * temp | v] for every row of x, and the
 * scan reads those column blocks in place.
 *
 *   x    : (B, T, embed)
 *   W    : (2*H*M + H*Dv, embed) = [Wphi Wq ; Wphi Wk ; Wv]   (row blocks)
 *   bias : (2*H*M + H*Dv) = [Wphi bq + bphi ; Wphi bk + bphi ; bv], or NULL
 *   temp : (B, T, H) or NULL     out : (B, T, H, Dv)
 *   S, z, flags : as fakla_attention, with Df = M.
 * Implemented for BF16 with M = Dv = 128 or 64, embed % 64 == 0, (2*H*M + H*Dv) %
 * 128 == 0, 16-byte aligned pointers; other cases return FAKLA_ERR_UNSUPPORTED.
 * Workspace: fakla_qkv_prefill_workspace_bytes() (the GEMM output, then the
 * scan's optional segment records).
 */
int fakla_qkv_prefill(const void* x, const void* W, const void* bias, const void* temp,
                      void* out, float* S, float* z, int64_t B, int64_t T, int64_t embed,
                      int64_t H, int64_t M, int64_t Dv, int dtype, unsigned flags,
                      void* workspace, size_t workspace_bytes, void* stream);

size_t fakla_qkv_prefill_workspace_bytes(int64_t B, int64_t T, int64_t embed, int64_t H,
                                         int64_t M, int64_t Dv, int dtype);

/*
 * fakla_decode_mapped -- one recurrent step for N independent sequences on
 * already feature-mapped q, k. Reference: none (the reference is stateless,
 * tm_kla.py:229-337); this is the loop body of cpu_kernels.cpp:121-162 run on
 * one token with the state injected.
 *
 *   q_mapped, k_mapped : (N, H, Df)   v : (N, H, Dv)   temp : (N, H) or NULL
 *   S : (N, H, Df, Dv) fp32, z : (N, H, Df) fp32 -- read and updated in place
 *   out : (N, H, Dv), written (uses the updated state, as the reference does)
 */
int fakla_decode_mapped(const void* q_mapped, const void* k_mapped, const void* v,
                        const void* temp, void* out, float* S, float* z, int64_t N,
                        int64_t H, int64_t Df, int64_t Dv, int dtype, void* stream);

/*
 * fakla_decode -- feature map and one recurrent step in one call: phi(q), phi(k)
 * from projected rows q, k : (N, in_dim), then fakla_decode_mapped.
 * W : (H * M, in_dim), bias : (H * M) or NULL; v : (N, H, Dv);
 * temp : (N, H) or NULL; S : (N, H, M, Dv), z : (N, H, M) updated in place;
 * out : (N, H, Dv). Needs workspace >= fakla_decode_workspace_bytes().
 */
int fakla_decode(const void* q, const void* k, const void* v, const void* temp,
                 const void* W, const void* bias, void* out, float* S, float* z,
                 int64_t N, int64_t in_dim, int64_t H, int64_t M, int64_t Dv,
                 int dtype, void* workspace, size_t workspace_bytes, void* stream);

size_t fakla_decode_workspace_bytes(int64_t N, int64_t in_dim, int64_t H,
                                    int64_t M, int64_t Dv, int dtype);

/*
 * fakla_decode_noalloc -- fakla_decode for callers that cannot allocate
 * device memory. No counterpart in the reference (it has no decode step and
 * no C ABI); this is an addition of this library.
 *
 * Who needs it: hosts that bind the library through a bare C FFI and have no
 * device allocator to hand it a workspace, and per-token decode loops where a
 * cudaMalloc (which synchronises the device and can fail under memory
 * pressure) is not allowed. Same arguments and results as fakla_decode minus
 * the workspace: the phi(q), phi(k) scratch lives in a static device array of
 * FAKLA_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until
 * process exit; nothing is allocated per call.
 * Limit: 2 * N * H * M * sizeof(element) <= FAKLA_NOALLOC_SCRATCH_BYTES
 * (e.g. N=256, H=32, M=128 in bf16 uses 4 MiB); larger steps are rejected with
 * FAKLA_ERR_UNSUPPORTED (argument errors are reported first, as fakla_decode
 * reports them). The first call on a device looks up the array's device
 * address; make it before any stream capture. The address is kept for that
 * device's current CUDA context and looked up again once that context has
 * been destroyed and recreated (cudaDeviceReset). All calls share the one
 * array: calls whose GPU work overlaps race on it and must be serialised by
 * the caller. Nothing in it needs to start at zero (each call writes all the
 * scratch it reads).
 */
#define FAKLA_NOALLOC_SCRATCH_BYTES (8u << 20)

int fakla_decode_noalloc(const void* q, const void* k, const void* v,
                         const void* temp, const void* W, const void* bias,
                         void* out, float* S, float* z, int64_t N,
                         int64_t in_dim, int64_t H, int64_t M, int64_t Dv,
                         int dtype, void* stream);

/*
 * fakla_device_status -- synchronise `stream` and return (then clear) the
 * device-side status word that kernels set when a bounded wait expires
 * (FAKLA_ERR_TIMEOUT) or a device-side check fails. FAKLA_OK if clean.
 */
int fakla_device_status(void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FAKLA_H_ */
