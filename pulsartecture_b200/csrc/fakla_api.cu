// C ABI of libfakla.so (declared in include/fakla.h): argument validation,
// dispatch between the tensor-core (sm_100a tcgen05) and CUDA-core kernels,
// workspace carving, and error reporting. No allocation happens here: the
// caller passes every buffer, including the workspace.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "fakla_common.cuh"
#include "fakla_kernels.h"

// ---------------------------------------------------------------------------
// Errors
// ---------------------------------------------------------------------------
static thread_local char g_last_error[512];

int fakla_set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

static int cuda_fail(cudaError_t e, const char* what) {
  return fakla_set_error(FAKLA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

extern "C" const char* fakla_strerror(int status) {
  switch (status) {
    case FAKLA_OK: return "ok";
    case FAKLA_ERR_INVALID_ARG: return "invalid argument";
    case FAKLA_ERR_UNSUPPORTED: return "unsupported configuration";
    case FAKLA_ERR_ALIGNMENT: return "misaligned pointer";
    case FAKLA_ERR_CUDA: return "CUDA error";
    case FAKLA_ERR_TIMEOUT: return "device-side wait timed out";
    case FAKLA_ERR_WORKSPACE: return "workspace too small";
    case FAKLA_ERR_NO_DEVICE: return "no sm_100 device";
    default: return "unknown status";
  }
}

extern "C" const char* fakla_last_error(void) { return g_last_error; }

extern "C" int fakla_version(void) { return FAKLA_VERSION; }

// ---------------------------------------------------------------------------
// Per-device state: status word address, SM count, sm_100 check.
// ---------------------------------------------------------------------------
__device__ int g_device_status_word;

namespace {
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

template <typename Fn>
Fn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(p);
}
}  // namespace

unsigned long long fakla_context_id() {
  static const CtxGetCurrentFn get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  static const CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  if (get_current == nullptr || get_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id + 1;  // 0 stays "no context"
}

namespace {
constexpr int kMaxDevices = 64;
// Cached per device for the context they were queried in: a context that is
// destroyed (cudaDeviceReset) and recreated gets a new id, and the cache is
// refreshed on the next call instead of handing out a stale status address.
struct DeviceInfo {
  std::atomic<unsigned long long> ctx{0};
  std::atomic<int*> status{nullptr};
  int sms = 0;
  int major = 0;
  int* st() const { return status.load(std::memory_order_relaxed); }
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

DeviceInfo* device_info(int* err) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = cuda_fail(e == cudaSuccess ? cudaErrorInvalidDevice : e, "cudaGetDevice");
    return nullptr;
  }
  DeviceInfo* d = &g_dev[dev];
  const unsigned long long cur = fakla_context_id();
  if (cur != 0 && d->ctx.load(std::memory_order_acquire) == cur) return d;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (cur != 0 && d->ctx.load(std::memory_order_relaxed) == cur) return d;
  // These runtime calls also make the device's primary context current when
  // the calling thread has none yet.
  int major = 0, sms = 0;
  int* status = nullptr;
  e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaGetSymbolAddress((void**)&status, g_device_status_word);
  if (e != cudaSuccess) {
    *err = cuda_fail(e, "device query");
    return nullptr;
  }
  d->major = major;
  d->sms = sms;
  d->status.store(status, std::memory_order_relaxed);
  // 0 (context id unavailable) keeps the entry uncached: queried again next call
  d->ctx.store(fakla_context_id(), std::memory_order_release);
  return d;
}

int require_device(DeviceInfo** out) {
  int err = FAKLA_OK;
  DeviceInfo* d = device_info(&err);
  if (!d) return err;
  if (d->major != 10)
    return fakla_set_error(FAKLA_ERR_NO_DEVICE,
                           "current device has compute capability %d.x; libfakla is built for sm_100a",
                           d->major);
  *out = d;
  return FAKLA_OK;
}
}  // namespace

int* fakla_status_word() {
  int err;
  DeviceInfo* d = device_info(&err);
  return d ? d->st() : nullptr;
}

int fakla_sm_count() {
  int err;
  DeviceInfo* d = device_info(&err);
  return d && d->sms > 0 ? d->sms : 148;
}

extern "C" int fakla_device_status(void* stream) {
  DeviceInfo* d = nullptr;
  int rc = require_device(&d);
  if (rc != FAKLA_OK) return rc;
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  int value = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&value, g_device_status_word, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_status_word, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "status word");
  if (value != FAKLA_OK)
    return fakla_set_error(value, "device kernel reported: %s", fakla_strerror(value));
  return FAKLA_OK;
}

// ---------------------------------------------------------------------------
// cuTensorMapEncodeTiled via the runtime's driver entry point
// ---------------------------------------------------------------------------
namespace fakla {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

bool encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, void* base,
                       const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                       const cuuint32_t* elem_strides, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  return fn(map, dtype, rank, base, dims, strides, box, elem_strides,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace fakla

// ---------------------------------------------------------------------------
// Validation helpers
// ---------------------------------------------------------------------------
namespace {
constexpr int64_t kMaxHeadDim = 256;

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }
inline size_t esize(int dtype) { return dtype == FAKLA_BF16 ? 2 : 4; }
inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
// One of the two phi(q) / phi(k) buffers of the prefill workspace.
inline size_t phi_buffer_bytes(int64_t B, int64_t T, int64_t H, int64_t M, int dtype) {
  return round_up((size_t)B * (size_t)T * (size_t)H * (size_t)M * esize(dtype), 256);
}

int check_dtype(int dtype) {
  if (dtype != FAKLA_F32 && dtype != FAKLA_BF16)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "dtype %d is not FAKLA_F32 or FAKLA_BF16", dtype);
  return FAKLA_OK;
}

int check_state(const float* S, const float* z, unsigned flags) {
  if (flags & ~(FAKLA_STATE_IN | FAKLA_STATE_OUT))
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "unknown flag bits 0x%x", flags);
  if ((S == nullptr) != (z == nullptr))
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "S and z must be both NULL or both non-NULL");
  if (flags && S == nullptr)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "state flags given without S/z buffers");
  return FAKLA_OK;
}

// The tensor-core scan needs bf16, 128x128 heads and 16-byte aligned tensors
// (TMA base addresses; every (b,t,h) row is 256 bytes, so rows stay aligned).
bool use_sm100_scan(int dtype, const void* q, const void* k, const void* v, const void* out,
                    const float* S, int64_t B, int64_t T, int64_t H, int64_t Df, int64_t Dv) {
  return dtype == FAKLA_BF16 && fakla::scan_sm100_supported(B, T, H, Df, Dv) && aligned16(q) &&
         aligned16(k) && aligned16(v) && aligned16(out) && (S == nullptr || aligned16(S));
}

bool use_sm100_phi(int dtype, const void* x0, const void* x1, const void* W, const void* out0,
                   const void* out1, const void* bias, int64_t rows, int64_t K, int64_t N,
                   int64_t heads) {
  return dtype == FAKLA_BF16 && fakla::phi_sm100_supported(rows, K, N, heads) && aligned16(x0) &&
         (x1 == nullptr || aligned16(x1)) && aligned16(W) && aligned16(out0) &&
         (out1 == nullptr || aligned16(out1)) && (bias == nullptr || aligned16(bias));
}

int run_attention(const void* q, const void* k, const void* v, const void* temp, void* out,
                  float* S, float* z, int64_t B, int64_t T, int64_t H, int64_t Df, int64_t Dv,
                  int dtype, unsigned flags, void* workspace, size_t workspace_bytes,
                  cudaStream_t stream, DeviceInfo* d) {
  if (use_sm100_scan(dtype, q, k, v, out, S, B, T, H, Df, Dv)) {
    bool enc = false;
    cudaError_t e = fakla::launch_scan_sm100(q, k, v, temp, out, S, z, B, T, H, flags, workspace,
                                             workspace_bytes, d->sms, stream, d->st(), &enc, 0, Df);
    if (!enc) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "TMA descriptor encoding failed");
    if (e != cudaSuccess) return cuda_fail(e, "scan_sm100 launch");
    return FAKLA_OK;
  }
  if (!fakla::scan_simt_supported(Df, Dv))
    return fakla_set_error(FAKLA_ERR_UNSUPPORTED, "head dims Df=%lld Dv=%lld unsupported",
                           (long long)Df, (long long)Dv);
  cudaError_t e = fakla::launch_scan_simt(dtype, q, k, v, temp, out, S, z, B, T, H, Df, Dv,
                                          flags, stream);
  if (e != cudaSuccess) return cuda_fail(e, "scan_simt launch");
  return FAKLA_OK;
}

// phi for one or two row sets sharing W (q rows -> out0, k rows -> out1 with
// temp1); act is a FAKLA_ACT_* code (FAKLA_ACT_ELU1 for FA-KLA).
int run_phi(const void* x0, const void* x1, const void* W, const void* bias, const void* temp0,
            const void* temp1, void* out0, void* out1, int64_t rows, int64_t K, int64_t N,
            int64_t heads, int dtype, cudaStream_t stream, DeviceInfo* d,
            int act = FAKLA_ACT_ELU1, float scale = 1.f) {
  if (use_sm100_phi(dtype, x0, x1, W, out0, out1, bias, rows, K, N, heads)) {
    bool enc = false;
    cudaError_t e = fakla::launch_phi_sm100(x0, x1, W, bias, temp0, temp1, out0, out1, rows, K,
                                            N, heads, act, scale, stream, d->st(), &enc);
    if (!enc) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "TMA descriptor encoding failed");
    if (e != cudaSuccess) return cuda_fail(e, "phi_sm100 launch");
    return FAKLA_OK;
  }
  cudaError_t e =
      fakla::launch_phi_simt(dtype, x0, W, bias, temp0, out0, rows, K, N, heads, act, scale, stream);
  if (e == cudaSuccess && x1 != nullptr)
    e = fakla::launch_phi_simt(dtype, x1, W, bias, temp1, out1, rows, K, N, heads, act, scale, stream);
  if (e != cudaSuccess) return cuda_fail(e, "phi_simt launch");
  return FAKLA_OK;
}
}  // namespace

// ---------------------------------------------------------------------------
// Entry points
// ---------------------------------------------------------------------------
// Workspace of the segmented tensor-core scan (long sequences, few (b, h)
// pairs): one (S, z) fp32 record per segment. Zero when the call would not be
// segmented on the current device.
static size_t scan_workspace(int64_t B, int64_t T, int64_t H, int64_t Df, int64_t Dv, int dtype) {
  if (dtype != FAKLA_BF16 || !fakla::scan_sm100_supported(B, T, H, Df, Dv)) return 0;
  return round_up(fakla::scan_sm100_workspace_bytes(B, T, H, fakla_sm_count()), 256);
}

extern "C" size_t fakla_attention_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t Df,
                                                  int64_t Dv, int dtype) {
  if (B < 1 || T < 1 || H < 1 || Df < 1 || Dv < 1) return 0;
  return scan_workspace(B, T, H, Df, Dv, dtype);
}

extern "C" int fakla_attention(const void* q, const void* k, const void* v, const void* temp,
                               void* out, float* S, float* z, int64_t B, int64_t T, int64_t H,
                               int64_t Df, int64_t Dv, int dtype, unsigned flags, void* workspace,
                               size_t workspace_bytes, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!q || !k || !v || !out)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "q_mapped, k_mapped, v and out must be non-NULL");
  if (B < 1 || T < 1 || H < 1 || Df < 1 || Dv < 1)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "sizes must be positive (B=%lld T=%lld H=%lld Df=%lld Dv=%lld)",
                           (long long)B, (long long)T, (long long)H, (long long)Df, (long long)Dv);
  if (Df > kMaxHeadDim || Dv > kMaxHeadDim)
    return fakla_set_error(FAKLA_ERR_UNSUPPORTED, "head dims above %lld", (long long)kMaxHeadDim);
  if ((rc = check_state(S, z, flags))) return rc;
  DeviceInfo* d = nullptr;
  if ((rc = require_device(&d))) return rc;
  return run_attention(q, k, v, temp, out, S, z, B, T, H, Df, Dv, dtype, flags, workspace,
                       workspace_bytes, (cudaStream_t)stream, d);
}

extern "C" int fakla_phi(const void* x, const void* W, const void* bias, const void* temp,
                         void* out, int64_t rows, int64_t in_dim, int64_t feat_dim,
                         int64_t heads, int dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!x || !W || !out)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "x, W and out must be non-NULL");
  if (rows < 1 || in_dim < 1 || feat_dim < 1 || heads < 1 || feat_dim % heads != 0)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG,
                           "bad sizes rows=%lld in_dim=%lld feat_dim=%lld heads=%lld",
                           (long long)rows, (long long)in_dim, (long long)feat_dim, (long long)heads);
  DeviceInfo* d = nullptr;
  if ((rc = require_device(&d))) return rc;
  return run_phi(x, nullptr, W, bias, temp, nullptr, out, nullptr, rows, in_dim, feat_dim, heads,
                 dtype, (cudaStream_t)stream, d);
}

extern "C" size_t fakla_attention_backward_workspace_bytes(int64_t B, int64_t T, int64_t H,
                                                           int64_t Df, int64_t Dv, int dtype) {
  if (B < 1 || T < 1 || H < 1) return 0;
  size_t need = fakla::backward_workspace_bytes(B, T, H);
  if (fakla::backward_sm100_supported(dtype, B, T, H, Df, Dv)) {
    const size_t tc = fakla::backward_sm100_workspace_bytes(B, T, H, fakla_sm_count());
    if (tc > need) need = tc;
  }
  return round_up(need, 256);
}

extern "C" int fakla_attention_backward(const void* q, const void* k, const void* v,
                                        const void* temp, const void* dout, const float* S0,
                                        const float* z0, const float* dS_final,
                                        const float* dz_final, void* dq, void* dk, void* dv,
                                        void* dtemp, float* dS0, float* dz0, int64_t B, int64_t T,
                                        int64_t H, int64_t Df, int64_t Dv, int dtype,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!q || !k || !v || !dout || !dq || !dk || !dv)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "q, k, v, dout, dq, dk and dv must be non-NULL");
  if (B < 1 || T < 1 || H < 1 || Df < 1 || Dv < 1)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "sizes must be positive");
  if ((S0 == nullptr) != (z0 == nullptr) || (dS_final == nullptr) != (dz_final == nullptr) ||
      (dS0 == nullptr) != (dz0 == nullptr))
    return fakla_set_error(FAKLA_ERR_INVALID_ARG,
                           "S0/z0, dS_final/dz_final and dS0/dz0 must each be both NULL or both non-NULL");
  if (!fakla::backward_simt_supported(Df, Dv))
    return fakla_set_error(FAKLA_ERR_UNSUPPORTED, "backward head dims Df=%lld Dv=%lld unsupported",
                           (long long)Df, (long long)Dv);
  const size_t need = fakla_attention_backward_workspace_bytes(B, T, H, Df, Dv, dtype);
  if (workspace == nullptr || workspace_bytes < need)
    return fakla_set_error(FAKLA_ERR_WORKSPACE, "backward needs %zu workspace bytes, got %zu", need,
                           workspace == nullptr ? (size_t)0 : workspace_bytes);
  if (((uintptr_t)workspace & 3u) != 0)
    return fakla_set_error(FAKLA_ERR_ALIGNMENT, "workspace must be 4-byte aligned");
  DeviceInfo* d = nullptr;
  if ((rc = require_device(&d))) return rc;
  // Tensor cores: bf16 128x128 heads, 16-byte aligned tensors (TMA bases and
  // float4 state rows) and a workspace sized on this device.
  if (fakla::backward_sm100_supported(dtype, B, T, H, Df, Dv) && aligned16(q) && aligned16(k) &&
      aligned16(v) && aligned16(dout) && aligned16(dq) && aligned16(dk) && aligned16(dv) &&
      aligned16(workspace) && (S0 == nullptr || aligned16(S0)) &&
      (dS_final == nullptr || aligned16(dS_final)) && (dS0 == nullptr || aligned16(dS0)) &&
      workspace_bytes >= fakla::backward_sm100_workspace_bytes(B, T, H, d->sms)) {
    bool enc = false;
    cudaError_t e = fakla::launch_backward_sm100(q, k, v, temp, dout, S0, z0, dS_final, dz_final,
                                                 dq, dk, dv, dtemp, dS0, dz0, B, T, H, Df, workspace,
                                                 d->sms, (cudaStream_t)stream, d->st(), &enc);
    if (!enc) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "TMA descriptor encoding failed");
    if (e != cudaSuccess) return cuda_fail(e, "attention backward (sm100) launch");
    return FAKLA_OK;
  }
  cudaError_t e = fakla::launch_backward_simt(dtype, q, k, v, temp, dout, S0, z0, dS_final,
                                              dz_final, dq, dk, dv, dtemp, dS0, dz0, B, T, H, Df,
                                              Dv, workspace, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "attention backward launch");
  return FAKLA_OK;
}

extern "C" int fakla_phi_backward(const void* phi, const void* dphi, void* dpre, int64_t n,
                                  int dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!phi || !dphi || !dpre) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "NULL pointer");
  if (n < 1) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "n must be positive");
  DeviceInfo* d = nullptr;
  if ((rc = require_device(&d))) return rc;
  cudaError_t e = fakla::launch_phi_backward(dtype, phi, dphi, dpre, n, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "phi backward launch");
  return FAKLA_OK;
}

extern "C" int fakla_activation_backward(const void* pre, const void* dy, void* dpre, int64_t rows,
                                         int64_t n, int act, float scale, int dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!pre || !dy || !dpre) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "NULL pointer");
  if (act < FAKLA_ACT_ELU1 || act > FAKLA_ACT_COSSIN)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "unknown activation %d", act);
  if (rows < 1 || n < 1) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "sizes must be positive");
  DeviceInfo* d = nullptr;
  if ((rc = require_device(&d))) return rc;
  cudaError_t e = fakla::launch_activation_backward(dtype, act, pre, dy, dpre, rows, n, scale,
                                                    (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "activation backward launch");
  return FAKLA_OK;
}

extern "C" size_t fakla_linear_backward_workspace_bytes(int64_t rows, int64_t in_dim, int64_t n_out,
                                                        int dtype) {
  (void)in_dim;
  (void)dtype;
  if (rows < 1 || n_out < 1) return 0;
  return round_up(fakla::colsum_workspace_bytes(rows, n_out), 256);
}

extern "C" int fakla_linear_backward(const void* x, const void* W, const void* dpre, void* dx, void* dW,
                                     void* db, int64_t rows, int64_t in_dim, int64_t n_out, int dtype,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!dpre) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "dpre must be non-NULL");
  if ((dx && !W) || (dW && !x))
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "dx needs W and dW needs x");
  if (rows < 1 || in_dim < 1 || n_out < 1)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "sizes must be positive");
  if (db) {
    const size_t need = fakla_linear_backward_workspace_bytes(rows, in_dim, n_out, dtype);
    if (workspace == nullptr || workspace_bytes < need)
      return fakla_set_error(FAKLA_ERR_WORKSPACE, "the bias gradient needs %zu workspace bytes, got %zu", need,
                             workspace == nullptr ? (size_t)0 : workspace_bytes);
    if (((uintptr_t)workspace & 3u) != 0)
      return fakla_set_error(FAKLA_ERR_ALIGNMENT, "workspace must be 4-byte aligned");
  }
  DeviceInfo* d = nullptr;
  if ((rc = require_device(&d))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  // dx (rows, in_dim) = dpre (rows, n_out; K-major) W (n_out, in_dim; MN-major)
  if (dx) {
    cudaError_t e;
    if (dtype == FAKLA_BF16 && fakla::gemm_sm100_supported(rows, in_dim, n_out, false, true) && aligned16(dpre) &&
        aligned16(W) && aligned16(dx)) {
      bool enc = false;
      e = fakla::launch_gemm_sm100(dpre, false, W, true, dx, rows, in_dim, n_out, st, d->st(), &enc);
      if (!enc) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "TMA descriptor encoding failed");
    } else {
      e = fakla::launch_gemm_strided(dtype, dpre, n_out, 1, W, 1, in_dim, dx, rows, in_dim, n_out, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "input gradient launch");
  }
  // dW (n_out, in_dim) = dpre^T (dpre stored (rows, n_out): MN-major) x (rows, in_dim: MN-major)
  if (dW) {
    cudaError_t e;
    if (dtype == FAKLA_BF16 && fakla::gemm_sm100_supported(n_out, in_dim, rows, true, true) && aligned16(dpre) &&
        aligned16(x) && aligned16(dW)) {
      bool enc = false;
      e = fakla::launch_gemm_sm100(dpre, true, x, true, dW, n_out, in_dim, rows, st, d->st(), &enc);
      if (!enc) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "TMA descriptor encoding failed");
    } else {
      e = fakla::launch_gemm_strided(dtype, dpre, 1, n_out, x, 1, in_dim, dW, n_out, in_dim, rows, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "weight gradient launch");
  }
  if (db) {
    cudaError_t e = fakla::launch_colsum(dtype, dpre, db, (float*)workspace, rows, n_out, st);
    if (e != cudaSuccess) return cuda_fail(e, "bias gradient launch");
  }
  return FAKLA_OK;
}

extern "C" int fakla_mix_features_backward(const void* feats, const void* logits, const void* dout,
                                           void* dfeats, void* dlogits, int64_t rows,
                                           int64_t n_maps, int64_t feat_dim, int dtype,
                                           void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!feats || !logits || !dout) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "NULL pointer");
  if (rows < 1 || n_maps < 1 || feat_dim < 1)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "sizes must be positive");
  if (!fakla::mix_supported(n_maps))
    return fakla_set_error(FAKLA_ERR_UNSUPPORTED, "at most 32 feature maps can be mixed, got %lld",
                           (long long)n_maps);
  DeviceInfo* d = nullptr;
  if ((rc = require_device(&d))) return rc;
  cudaError_t e = fakla::launch_mix_backward(dtype, feats, logits, dout, dfeats, dlogits, rows,
                                             n_maps, feat_dim, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "mix backward launch");
  return FAKLA_OK;
}

extern "C" int fakla_feature_map(const void* x, const void* W, const void* bias, void* out,
                                 int64_t rows, int64_t in_dim, int64_t n_out, int act, float scale,
                                 int dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!x || !W || !out)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "x, W and out must be non-NULL");
  if (act < FAKLA_ACT_ELU1 || act > FAKLA_ACT_COSSIN)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "unknown activation %d", act);
  if (rows < 1 || in_dim < 1 || n_out < 1)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "bad sizes rows=%lld in_dim=%lld n_out=%lld",
                           (long long)rows, (long long)in_dim, (long long)n_out);
  DeviceInfo* d = nullptr;
  if ((rc = require_device(&d))) return rc;
  return run_phi(x, nullptr, W, bias, nullptr, nullptr, out, nullptr, rows, in_dim, n_out, 1,
                 dtype, (cudaStream_t)stream, d, act, scale);
}

extern "C" int fakla_mix_features(const void* feats, const void* logits, void* out, int64_t rows,
                                  int64_t n_maps, int64_t feat_dim, int dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!feats || !logits || !out)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "feats, logits and out must be non-NULL");
  if (rows < 1 || feat_dim < 1 || n_maps < 1)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "bad sizes rows=%lld n_maps=%lld feat_dim=%lld",
                           (long long)rows, (long long)n_maps, (long long)feat_dim);
  if (!fakla::mix_supported(n_maps))
    return fakla_set_error(FAKLA_ERR_UNSUPPORTED, "at most 32 feature maps can be mixed, got %lld",
                           (long long)n_maps);
  DeviceInfo* d = nullptr;
  if ((rc = require_device(&d))) return rc;
  cudaError_t e = fakla::launch_mix_features(dtype, feats, logits, out, rows, n_maps, feat_dim,
                                             (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "mix_features launch");
  return FAKLA_OK;
}

extern "C" size_t fakla_prefill_workspace_bytes(int64_t B, int64_t T, int64_t in_dim, int64_t H,
                                                int64_t M, int64_t Dv, int dtype) {
  (void)in_dim;
  if (B < 1 || T < 1 || H < 1 || M < 1 || Dv < 1) return 0;
  return 2 * phi_buffer_bytes(B, T, H, M, dtype) + scan_workspace(B, T, H, M, Dv, dtype);
}

extern "C" int fakla_prefill(const void* q, const void* k, const void* v, const void* temp,
                             const void* W, const void* bias, void* out, float* S, float* z,
                             int64_t B, int64_t T, int64_t in_dim, int64_t H, int64_t M,
                             int64_t Dv, int dtype, unsigned flags, void* workspace,
                             size_t workspace_bytes, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!q || !k || !v || !W || !out)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "q, k, v, W and out must be non-NULL");
  if (B < 1 || T < 1 || in_dim < 1 || H < 1 || M < 1 || Dv < 1)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "sizes must be positive");
  if (M > kMaxHeadDim || Dv > kMaxHeadDim)
    return fakla_set_error(FAKLA_ERR_UNSUPPORTED, "head dims above %lld", (long long)kMaxHeadDim);
  if ((rc = check_state(S, z, flags))) return rc;
  // phi(q), phi(k) buffers are required; the scan's segment records (the
  // rest of fakla_prefill_workspace_bytes) are used when they fit.
  const size_t need = 2 * phi_buffer_bytes(B, T, H, M, dtype);
  if (workspace == nullptr || workspace_bytes < need)
    return fakla_set_error(FAKLA_ERR_WORKSPACE, "prefill needs at least %zu workspace bytes, got %zu",
                           need, workspace == nullptr ? (size_t)0 : workspace_bytes);
  if (!aligned16(workspace))
    return fakla_set_error(FAKLA_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  if ((rc = require_device(&d))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t rows = B * T;
  uint8_t* ws = (uint8_t*)workspace;
  const size_t one = phi_buffer_bytes(B, T, H, M, dtype);
  void* phq = ws;
  void* phk = ws + one;
  // phi(q) and phi(k)*temp in one launch (k-side temperature fused, so the
  // scan below runs with temp = NULL); the rest of the workspace holds the
  // scan's segment records.
  rc = run_phi(q, k, W, bias, nullptr, temp, phq, phk, rows, in_dim, H * M, H, dtype, st, d);
  if (rc) return rc;
  return run_attention(phq, phk, v, nullptr, out, S, z, B, T, H, M, Dv, dtype, flags,
                       ws + 2 * one, workspace_bytes - 2 * one, st, d);
}

static size_t qkv_buffer_bytes(int64_t B, int64_t T, int64_t H, int64_t M, int64_t Dv) {
  return round_up((size_t)B * (size_t)T * (size_t)(2 * H * M + H * Dv) * 2, 256);
}

extern "C" size_t fakla_qkv_prefill_workspace_bytes(int64_t B, int64_t T, int64_t embed, int64_t H,
                                                    int64_t M, int64_t Dv, int dtype) {
  (void)embed;
  if (B < 1 || T < 1 || H < 1 || M < 1 || Dv < 1 || dtype != FAKLA_BF16) return 0;
  return qkv_buffer_bytes(B, T, H, M, Dv) + scan_workspace(B, T, H, M, Dv, dtype);
}

extern "C" int fakla_qkv_prefill(const void* x, const void* W, const void* bias, const void* temp,
                                 void* out, float* S, float* z, int64_t B, int64_t T,
                                 int64_t embed, int64_t H, int64_t M, int64_t Dv, int dtype,
                                 unsigned flags, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!x || !W || !out) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "x, W and out must be non-NULL");
  if (B < 1 || T < 1 || embed < 1 || H < 1 || M < 1 || Dv < 1)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "sizes must be positive");
  if ((rc = check_state(S, z, flags))) return rc;
  const int64_t rows = B * T;
  if (dtype != FAKLA_BF16 || M != Dv || (M != 128 && M != 64) ||
      !fakla::qkv_sm100_supported(rows, embed, H * M, H * Dv, H) ||
      !fakla::scan_sm100_supported(B, T, H, M, Dv))
    return fakla_set_error(FAKLA_ERR_UNSUPPORTED,
                           "fakla_qkv_prefill serves bf16, M = Dv = 128 or 64, embed %% 64 == 0 (got dtype=%d "
                           "M=%lld Dv=%lld embed=%lld)", dtype, (long long)M, (long long)Dv, (long long)embed);
  if (!aligned16(x) || !aligned16(W) || !aligned16(out) || (bias && !aligned16(bias)) ||
      (S && !aligned16(S)))
    return fakla_set_error(FAKLA_ERR_ALIGNMENT, "x, W, bias, out and S must be 16-byte aligned");
  const size_t need = qkv_buffer_bytes(B, T, H, M, Dv);
  if (workspace == nullptr || workspace_bytes < need)
    return fakla_set_error(FAKLA_ERR_WORKSPACE, "qkv prefill needs at least %zu workspace bytes, got %zu",
                           need, workspace == nullptr ? (size_t)0 : workspace_bytes);
  if (!aligned16(workspace))
    return fakla_set_error(FAKLA_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  if ((rc = require_device(&d))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* buf = (uint8_t*)workspace;
  bool enc = false;
  cudaError_t e = fakla::launch_qkv_sm100(x, W, bias, temp, buf, rows, embed, H * M, H * Dv, H, st,
                                          d->st(), &enc);
  if (!enc) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "TMA descriptor encoding failed");
  if (e != cudaSuccess) return cuda_fail(e, "qkv GEMM launch");
  const int64_t row_elems = 2 * H * M + H * Dv;
  const void* phq = buf;
  const void* phk = buf + (size_t)H * M * 2;
  const void* vv = buf + (size_t)2 * H * M * 2;
  e = fakla::launch_scan_sm100(phq, phk, vv, nullptr, out, S, z, B, T, H, flags, buf + need,
                               workspace_bytes - need, d->sms, st, d->st(), &enc, row_elems, M);
  if (!enc) return fakla_set_error(FAKLA_ERR_INVALID_ARG, "TMA descriptor encoding failed");
  if (e != cudaSuccess) return cuda_fail(e, "scan_sm100 launch");
  return FAKLA_OK;
}

extern "C" int fakla_decode_mapped(const void* q, const void* k, const void* v, const void* temp,
                                   void* out, float* S, float* z, int64_t N, int64_t H,
                                   int64_t Df, int64_t Dv, int dtype, void* stream) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!q || !k || !v || !out || !S || !z)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "q, k, v, out, S and z must be non-NULL");
  if (N < 1 || H < 1 || Df < 1 || Dv < 1)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "sizes must be positive");
  if (Df > kMaxHeadDim || Dv > kMaxHeadDim)
    return fakla_set_error(FAKLA_ERR_UNSUPPORTED, "head dims above %lld", (long long)kMaxHeadDim);
  DeviceInfo* d = nullptr;
  if ((rc = require_device(&d))) return rc;
  cudaError_t e = fakla::launch_decode(dtype, q, k, v, temp, out, S, z, N * H, Df, Dv,
                                       (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return FAKLA_OK;
}

extern "C" size_t fakla_decode_workspace_bytes(int64_t N, int64_t in_dim, int64_t H, int64_t M,
                                               int64_t Dv, int dtype) {
  (void)in_dim;
  (void)Dv;
  if (N < 1 || H < 1 || M < 1) return 0;
  return 2 * round_up((size_t)N * (size_t)H * (size_t)M * esize(dtype), 256);
}

int fakla_decode_check(const void* q, const void* k, const void* v, const void* W, const void* out,
                       const float* S, const float* z, int64_t N, int64_t in_dim, int64_t H,
                       int64_t M, int64_t Dv, int dtype) {
  int rc = check_dtype(dtype);
  if (rc) return rc;
  if (!q || !k || !v || !W || !out || !S || !z)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "q, k, v, W, out, S and z must be non-NULL");
  if (N < 1 || in_dim < 1 || H < 1 || M < 1 || Dv < 1)
    return fakla_set_error(FAKLA_ERR_INVALID_ARG, "sizes must be positive");
  if (M > kMaxHeadDim || Dv > kMaxHeadDim)
    return fakla_set_error(FAKLA_ERR_UNSUPPORTED, "head dims above %lld", (long long)kMaxHeadDim);
  return FAKLA_OK;
}

extern "C" int fakla_decode(const void* q, const void* k, const void* v, const void* temp,
                            const void* W, const void* bias, void* out, float* S, float* z,
                            int64_t N, int64_t in_dim, int64_t H, int64_t M, int64_t Dv, int dtype,
                            void* workspace, size_t workspace_bytes, void* stream) {
  int rc = fakla_decode_check(q, k, v, W, out, S, z, N, in_dim, H, M, Dv, dtype);
  if (rc) return rc;
  const size_t need = fakla_decode_workspace_bytes(N, in_dim, H, M, Dv, dtype);
  if (workspace == nullptr || workspace_bytes < need)
    return fakla_set_error(FAKLA_ERR_WORKSPACE, "decode needs %zu workspace bytes, got %zu", need,
                           workspace == nullptr ? (size_t)0 : workspace_bytes);
  if (!aligned16(workspace))
    return fakla_set_error(FAKLA_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  if ((rc = require_device(&d))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* ws = (uint8_t*)workspace;
  void* phq = ws;
  void* phk = ws + need / 2;
  rc = run_phi(q, k, W, bias, nullptr, temp, phq, phk, N, in_dim, H * M, H, dtype, st, d);
  if (rc) return rc;
  cudaError_t e = fakla::launch_decode(dtype, phq, phk, v, nullptr, out, S, z, N * H, M, Dv, st);
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return FAKLA_OK;
}
