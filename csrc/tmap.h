// Host-side access to the driver's tensor-map encoder, shared by every TMA kernel's launcher.
//
// cuTensorMapEncodeTiled is a driver-API call: it needs a context current on the calling thread, and a
// thread that has made no CUDA runtime call yet has none (autograd's backward worker threads start that
// way; when the device they run for is already the runtime's default device, nothing before the first
// launcher binds a context, and the encoder returns CUDA_ERROR_INVALID_CONTEXT).  encode_fn() therefore
// binds the current device's primary context once per thread (cudaSetDevice) before returning the entry
// point, which is looked up once per process.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace rlb_tmap {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn lookup_encoder() {
  void* ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    return (EncodeTiledFn)ptr;
  return nullptr;
}

inline bool bind_thread_context() {
  thread_local bool bound = false;
  if (!bound) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess) return false;
    bound = true;
  }
  return true;
}

// The encoder, with a context current on this thread; nullptr if either is unavailable.
inline EncodeTiledFn encode_fn() {
  static const EncodeTiledFn fn = lookup_encoder();
  return (fn && bind_thread_context()) ? fn : nullptr;
}

}  // namespace rlb_tmap
