// Test-only kernels (built into tests/_build/libfakla_selftest.so, never part
// of the product library):
//  * umma_form_kernel: one 128x128x64 tcgen05 MMA in each operand form the
//    FA-KLA kernels use, with operands staged by plain loads into the same
//    128B-swizzled shared-memory layouts, so a layout mistake shows up as a
//    mismatch against a host matmul rather than deep inside a kernel.
//  * wait_timeout_kernel: waits on an mbarrier that nothing arrives on, with a
//    short bound, and must come back with FAKLA_ERR_TIMEOUT (no hang, no trap).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../pulsartecture_b200/csrc/sm100_umma.cuh"

using namespace fakla::sm100;

namespace {
constexpr int kAtom = 128 * 128;  // 128 rows x 128 bytes

// Stage a (rows x 128) bf16 row-major matrix from global into two 128B-swizzled
// atoms (columns 0-63, 64-127): the layout TMA writes for (64 x rows) boxes.
__device__ void stage_rows(uint8_t* dst, const __nv_bfloat16* src, int rows) {
  for (int e = threadIdx.x; e < rows * 128; e += blockDim.x) {
    const int r = e / 128, c = e % 128;
    uint8_t* atom = dst + (c >= 64 ? kAtom : 0);
    *reinterpret_cast<__nv_bfloat16*>(atom + sw128_offset(r, c & 63)) = src[e];
  }
}

// form 0: D = A B^T, A (128 x K=128) K-major, B (N=128 x K=128) K-major
// form 1: D = A^T B, A given as (K=128 x M=128) MN-major, B (K=128 x N=128) MN-major
// form 2: D = A B,   A (128 x K=128) K-major, B (K=128 x N=128) MN-major
// form 3: D = A B,   A (128 x K=128) in TMEM (bf16 pairs), B (K=128 x N=128) MN-major
__global__ void __launch_bounds__(128, 1) umma_form_kernel(int form, const __nv_bfloat16* A,
                                                           const __nv_bfloat16* B, float* D) {
  extern __shared__ uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = sm;
  uint8_t* sB = sm + 2 * kAtom;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + 4 * kAtom);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  stage_rows(sA, A, 128);
  stage_rows(sB, B, 128);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(slot, 256);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  const uint32_t dcol = 0, acol = 128;
  const uint32_t lane_addr = tmem + ((uint32_t)(32 * warp) << 16);
  if (form == 3) {
    // thread r writes row r of A as bf16 pairs into TMEM columns acol..acol+63
    for (int cc = 0; cc < 128; cc += 32) {
      uint32_t v[16];
      for (int i = 0; i < 16; ++i) {
        const int row = 32 * warp + lane;
        const uint32_t lo = __bfloat16_as_ushort(A[row * 128 + cc + 2 * i]);
        const uint32_t hi = __bfloat16_as_ushort(A[row * 128 + cc + 2 * i + 1]);
        v[i] = lo | (hi << 16);
      }
      tmem_st16(lane_addr + acol + (uint32_t)(cc / 2), v);
    }
    tmem_st_wait();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (threadIdx.x == 0) {
    const uint32_t a = smem_u32(sA), b = smem_u32(sB);
    for (int j = 0; j < 8; ++j) {
      const uint64_t ak = smem_desc_sw128(a + (uint32_t)((j >> 2) * kAtom + (j & 3) * 32), 16, 1024);
      const uint64_t bk = smem_desc_sw128(b + (uint32_t)((j >> 2) * kAtom + (j & 3) * 32), 16, 1024);
      const uint64_t amn = smem_desc_sw128(a + (uint32_t)(j * 2048), kAtom, 1024);
      const uint64_t bmn = smem_desc_sw128(b + (uint32_t)(j * 2048), kAtom, 1024);
      if (form == 0) mma_ss(tmem + dcol, ak, bk, idesc_bf16_f32(128, 128, false, false), j > 0);
      if (form == 1) mma_ss(tmem + dcol, amn, bmn, idesc_bf16_f32(128, 128, true, true), j > 0);
      if (form == 2) mma_ss(tmem + dcol, ak, bmn, idesc_bf16_f32(128, 128, false, true), j > 0);
      if (form == 3)
        mma_ts(tmem + dcol, tmem + acol + (uint32_t)(8 * j), bmn, idesc_bf16_f32(128, 128, false, true), j > 0);
    }
    mma_commit(bar);
  }
  const bool ok = mbar_wait(bar, 0, 1000000000ull);
  tc_fence_after();
  const int row = 32 * warp + lane;
  for (int cc = 0; cc < 128; cc += 32) {
    uint32_t v[32];
    tmem_ld32(lane_addr + dcol + (uint32_t)cc, v);
    tmem_ld_wait();
    for (int i = 0; i < 32; ++i) D[row * 128 + cc + i] = ok ? __uint_as_float(v[i]) : -1e30f;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

__global__ void wait_timeout_kernel(uint64_t limit_ns, int* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Nothing ever arrives on `bar`: the bounded wait must give up.
  const bool ok = mbar_wait(&bar, 0, limit_ns);
  if (threadIdx.x == 0) *status = ok ? 0 : 5 /* FAKLA_ERR_TIMEOUT */;
}
}  // namespace

extern "C" int selftest_umma_form(int form, const void* A, const void* B, void* D, void* stream) {
  const size_t smem = 1024 + 4 * kAtom + 64;
  cudaError_t e = cudaFuncSetAttribute(umma_form_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  umma_form_kernel<<<1, 128, smem, (cudaStream_t)stream>>>(form, (const __nv_bfloat16*)A,
                                                           (const __nv_bfloat16*)B, (float*)D);
  return (int)cudaGetLastError();
}

extern "C" int selftest_wait_timeout(uint64_t limit_ns, void* status, void* stream) {
  wait_timeout_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(limit_ns, (int*)status);
  return (int)cudaGetLastError();
}
