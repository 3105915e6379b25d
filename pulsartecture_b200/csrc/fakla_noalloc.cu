// fakla_decode_noalloc: the decode step for callers that cannot allocate.
//
// fakla_decode needs a small device workspace for phi(q) and phi(k) of the
// step. Some callers have no way to provide one: a host that binds this
// library through a bare C FFI (Go, Java, a serving runtime's plugin slot)
// often has no device allocator of its own, and calling cudaMalloc inside a
// per-token decode loop is not an option either -- it synchronises the device,
// can fail under memory pressure mid-generation, and some runtimes forbid it
// on the latency path outright. This entry point takes the same inputs and
// outputs as fakla_decode but keeps the workspace in a fixed-size array that
// lives in the library's own device memory image, so it allocates nothing.
//
// Properties a caller must know:
//  * The array holds FAKLA_NOALLOC_SCRATCH_BYTES (8 MiB) on every GPU that
//    loads the library, from module load until process exit.
//  * A step needs 2 * N * H * M * sizeof(element) scratch bytes (phi(q) and
//    phi(k)); larger requests are rejected with FAKLA_ERR_UNSUPPORTED and
//    nothing is launched.
//  * The first call on a device looks up the array's device address (with
//    that device current) and caches it for that device's current CUDA
//    context; make that first call before any stream capture. A call made
//    after the context was destroyed and recreated (cudaDeviceReset) looks
//    the address up again.
//  * Every call uses the same array. Each call overwrites all of the scratch
//    it reads (the phi kernel writes every phi(q)/phi(k) element before the
//    state kernel reads it), so nothing has to start at zero; but calls whose
//    work overlaps on the GPU (different streams, or different host threads
//    without ordering) race on the array and must be serialised by the caller.
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "fakla_common.cuh"

namespace {
constexpr size_t kScratchBytes = FAKLA_NOALLOC_SCRATCH_BYTES;
static_assert(kScratchBytes % 256 == 0, "scratch size");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
// Device address of the array per device, for the context it was looked up in.
struct ScratchSlot {
  std::atomic<unsigned long long> ctx{0};
  std::atomic<void*> addr{nullptr};
};
ScratchSlot g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

// Device address of g_noalloc_scratch on the current device (the host-side
// symbol is only a stand-in and must never be passed to a kernel).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fakla_set_error(FAKLA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return fakla_set_error(FAKLA_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  ScratchSlot& slot = g_scratch[dev];
  const unsigned long long cur = fakla_context_id();
  if (cur != 0 && slot.ctx.load(std::memory_order_acquire) == cur) {
    *out = slot.addr.load(std::memory_order_relaxed);
    return FAKLA_OK;
  }
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  void* p = nullptr;
  // with the device current; creates its primary context if the thread has none
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr)
    return fakla_set_error(FAKLA_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s",
                           cudaGetErrorString(e));
  slot.addr.store(p, std::memory_order_relaxed);
  slot.ctx.store(fakla_context_id(), std::memory_order_release);
  *out = p;
  return FAKLA_OK;
}
}  // namespace

extern "C" int fakla_decode_noalloc(const void* q, const void* k, const void* v, const void* temp,
                                    const void* W, const void* bias, void* out, float* S, float* z,
                                    int64_t N, int64_t in_dim, int64_t H, int64_t M, int64_t Dv,
                                    int dtype, void* stream) {
  // the argument checks of fakla_decode first, so a bad call reports its
  // real error rather than a scratch-size one
  int rc = fakla_decode_check(q, k, v, W, out, S, z, N, in_dim, H, M, Dv, dtype);
  if (rc != FAKLA_OK) return rc;
  const size_t need = fakla_decode_workspace_bytes(N, in_dim, H, M, Dv, dtype);
  if (need > kScratchBytes)
    return fakla_set_error(FAKLA_ERR_UNSUPPORTED,
                           "decode step needs %zu scratch bytes (2*N*H*M*elem), the static scratch "
                           "holds %zu; use fakla_decode with a caller workspace",
                           need, kScratchBytes);
  void* scratch = nullptr;
  rc = scratch_address(&scratch);
  if (rc != FAKLA_OK) return rc;
  return fakla_decode(q, k, v, temp, W, bias, out, S, z, N, in_dim, H, M, Dv, dtype, scratch,
                      kScratchBytes, stream);
}
