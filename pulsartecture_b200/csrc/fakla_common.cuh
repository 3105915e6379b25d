// Shared device/host helpers for the FA-KLA kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fakla.h"

namespace fakla {

// Stability constant of the denominator: K_EPSILON in the reference's CPU
// kernel (ultra_rwka/backend/cpp/cpu/cpu_kernels.cpp:22), used for fp32 and
// bf16 activations alike (accumulation is fp32 in both).
constexpr float kEps = 1e-12f;

// Kernels that wait (bounded) receive a pointer to the device-side status word
// (defined in fakla_api.cu, one per device) and record the first failure in it
// with atomicCAS(0 -> code); fakla_device_status() reads and clears it.
__device__ __forceinline__ void report_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// Programmatic dependent launch (PDL). A kernel launched by launch_chained()
// may begin while the kernel before it on the stream is still running (on SMs
// that kernel has left): it sets up its shared memory, barriers and tensor
// memory, then griddep_wait() blocks until that kernel has completed and its
// memory is visible. Every thread calls it before its first global-memory
// access. griddep_launch_dependents() (after the wait) lets the next chained
// kernel be scheduled. For a kernel launched without the attribute both
// return at once.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// cudaLaunchKernelEx with programmatic dependent launch allowed and, when
// cluster_x > 1, clusters of cluster_x CTAs. Kernels launched this way call
// griddep_wait() before touching global memory.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_chained(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                  cudaStream_t stream, unsigned cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
#ifndef FAKLA_NO_PDL
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
#endif
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// phi activation: elu(x) + 1 = x + 1 for x > 0, exp(x) for x <= 0.
// (F.elu(x) + 1.0 with alpha = 1, ultra_rwka/kernels/feature_maps.py:248.)
__device__ __forceinline__ float elu_plus_one(float x) {
  return x > 0.f ? x + 1.f : expf(x);
}

// Same map with the hardware exp approximation (__expf): used where the
// result is rounded to bf16 (relative step 2^-8), far above its error.
__device__ __forceinline__ float elu_plus_one_fast(float x) {
  return x > 0.f ? x + 1.f : __expf(x);
}

// Output activations of the feature-map GEMMs (FAKLA_ACT_* in fakla.h),
// written from their definitions: torch's elu(alpha=1)+1, relu,
// softplus(beta=1, threshold=20), exact (erf) gelu, sigmoid and abs. kFast
// uses the hardware exp approximation where the result is rounded to bf16.
template <int ACT, bool kFast>
__device__ __forceinline__ float activate(float x) {
  if constexpr (ACT == FAKLA_ACT_ELU1) {
    return kFast ? elu_plus_one_fast(x) : elu_plus_one(x);
  } else if constexpr (ACT == FAKLA_ACT_RELU) {
    return x > 0.f ? x : 0.f;
  } else if constexpr (ACT == FAKLA_ACT_SOFTPLUS) {
    return x > 20.f ? x : log1pf(expf(x));
  } else if constexpr (ACT == FAKLA_ACT_GELU) {
    return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
  } else if constexpr (ACT == FAKLA_ACT_SIGMOID) {
    return 1.f / (1.f + expf(-x));
  } else if constexpr (ACT == FAKLA_ACT_ABS) {
    return fabsf(x);
  } else {
    return x;  // FAKLA_ACT_IDENTITY (COSSIN is handled by the callers)
  }
}

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

}  // namespace fakla

// Host-side helpers defined in fakla_api.cu.
int fakla_set_error(int status, const char* fmt, ...);
int* fakla_status_word();  // device address of the current device's status word
int fakla_sm_count();      // SM count of the current device (cached)
// Unique id (+1) of the calling thread's current CUDA context; 0 when there is
// none yet or the driver cannot say. Caches of device addresses key on it.
unsigned long long fakla_context_id();
// fakla_decode's argument checks (dtype, pointers, sizes, head dims), all
// but the workspace; FAKLA_OK or the error code with its message set.
int fakla_decode_check(const void* q, const void* k, const void* v, const void* W, const void* out,
                       const float* S, const float* z, int64_t N, int64_t in_dim, int64_t H,
                       int64_t M, int64_t Dv, int dtype);
