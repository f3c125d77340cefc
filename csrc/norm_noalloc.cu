// RMSNorm backward that allocates nothing: rlb_rmsnorm_bwd_noalloc.
//
// The regular entry point (rlb_rmsnorm_bwd) needs a [parts, dim] fp32 buffer
// for the per-block dw partial sums, which its callers allocate (the Python
// binding takes it from torch's caching allocator).  Some callers cannot
// allocate device memory at the point where they run the backward:
//   * a plain C / C++ host program that links only this shared library and has
//     no device allocator of its own to hand out a scratch buffer;
//   * code that runs inside an allocator's own out-of-memory or memory-release
//     path (for example a hook that recomputes activations to make room),
//     where calling back into the allocator would re-enter it or fail for lack
//     of the very memory it is trying to free.
// For them this variant keeps the partials in a file-scope __device__ array of
// fixed size, so the call performs no cudaMalloc / cudaFree and calls no
// allocating library routine (torch included).
//
// Scratch: kScratchFloats fp32 values = 4 MiB per device.  A call uses
// parts x dim of it, parts = min(ceil(rows / 2), 8 x SMs, kScratchFloats / dim),
// so any row count fits; only dim is limited (see below).  Nothing in the
// scratch needs to start at zero: every block of the backward kernel writes its
// whole partial row before the column-sum kernel reads it, so stale values from
// an earlier call are always overwritten.
//
// Setup: the first call on each device (with that device current) looks up the
// array's device address with cudaGetSymbolAddress, which may load this
// library's device code onto the device, and reads the SM count; both are
// cached per device.  Make that first call before any stream capture that will
// contain later calls.  Under lazy module loading (the CUDA default) that
// lookup is also the moment the 4 MiB array gets its device memory, so it can
// fail with cudaErrorMemoryAllocation when the device is full.  A caller that
// will run the backward from an out-of-memory path must therefore do the setup
// beforehand, while memory is still free: call rlb_rmsnorm_bwd_noalloc_init()
// once per device (with that device current), or make one ordinary call.
//
// Concurrency: every call on a device shares that device's single scratch
// array.  Calls issued on one stream run in order and are safe; calls that
// overlap in time (different streams, or different host threads on different
// streams) race on the scratch and give wrong dw.  Serialise them.
//
// Supported shapes: dim a multiple of 256 and at most 8192 (the block-per-row
// kernel of the regular entry point).  Other dims return cudaErrorInvalidValue
// without launching anything.  All tensor pointers must be 16-byte aligned.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "launchers.h"

namespace rlb {
// Defined in norm.cu: the wide backward's launcher, and the column-sum kernel (launched through its host stub).
void launch_rmsnorm_bwd_wide(int grid, const __nv_bfloat16* h, const __nv_bfloat16* w, const float* rstd,
                             const __nv_bfloat16* dy, const __nv_bfloat16* dres, __nv_bfloat16* dx, float* dw_part,
                             long long rows, int dim, cudaStream_t s);
__global__ void colsum_kernel(const float* __restrict__ part, int parts, int dim, float* __restrict__ out_f32,
                              __nv_bfloat16* __restrict__ out_bf16);
}  // namespace rlb

namespace {

constexpr long long kScratchFloats = 1LL << 20;  // 4 MiB of fp32 partial sums per device
constexpr int kMaxDim = 8192;
constexpr int kRowsPerBlock = 2;  // rows one backward block handles per iteration (norm.cu)
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_dw_scratch[kScratchFloats];

std::atomic<float*> g_scratch_ptr[kMaxDevices];
std::atomic<int> g_sm_count[kMaxDevices];
std::mutex g_setup_mu;

// Per-device lookup of the scratch address and SM count (first call only).
cudaError_t device_scratch(int dev, float** ptr, int* sms) {
  float* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p != nullptr) {
    *ptr = p;
    *sms = g_sm_count[dev].load(std::memory_order_relaxed);
    return cudaSuccess;
  }
  std::lock_guard<std::mutex> lock(g_setup_mu);
  p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    void* addr = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&addr, g_dw_scratch);
    if (err != cudaSuccess) return err;
    int count = 0;
    err = cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess) return err;
    g_sm_count[dev].store(count, std::memory_order_relaxed);
    p = static_cast<float*>(addr);
    g_scratch_ptr[dev].store(p, std::memory_order_release);
  }
  *ptr = p;
  *sms = g_sm_count[dev].load(std::memory_order_relaxed);
  return cudaSuccess;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" long long rlb_rmsnorm_bwd_noalloc_scratch_bytes() { return kScratchFloats * (long long)sizeof(float); }

// Runs the per-device setup for the current device now (address lookup, which
// brings the scratch array into device memory, and the SM count) and returns
// its cudaError_t value.  Idempotent; later calls on the device return at once.
extern "C" int rlb_rmsnorm_bwd_noalloc_init() {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  float* scratch = nullptr;
  int sms = 0;
  return device_scratch(dev, &scratch, &sms);
}

extern "C" int rlb_rmsnorm_bwd_noalloc(const void* h, const void* w, const float* rstd, const void* dy,
                                       const void* dres, void* dx, void* dw_out, int dw_is_f32, long long rows,
                                       int dim, cudaStream_t stream) {
  if (dim <= 0 || dim % 256 != 0 || dim > kMaxDim || rows < 0) return cudaErrorInvalidValue;
  if (!aligned16(h) || !aligned16(w) || !aligned16(dy) || !aligned16(dx) || (dres && !aligned16(dres)))
    return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  float* scratch = nullptr;
  int sms = 0;
  err = device_scratch(dev, &scratch, &sms);
  if (err != cudaSuccess) return err;

  long long parts = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  if (parts < 1) parts = 1;
  if (parts > (long long)sms * 8) parts = (long long)sms * 8;
  if (parts > kScratchFloats / dim) parts = kScratchFloats / dim;

  rlb::launch_rmsnorm_bwd_wide((int)parts, (const __nv_bfloat16*)h, (const __nv_bfloat16*)w, rstd,
                               (const __nv_bfloat16*)dy, (const __nv_bfloat16*)dres, (__nv_bfloat16*)dx, scratch, rows,
                               dim, stream);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  rlb::colsum_kernel<<<(dim + 31) / 32, 256, 0, stream>>>(scratch, (int)parts, dim,
                                                          dw_is_f32 ? (float*)dw_out : nullptr,
                                                          dw_is_f32 ? nullptr : (__nv_bfloat16*)dw_out);
  return cudaGetLastError();
}
