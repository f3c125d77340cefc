// Shared device helpers for the sm_100a kernels of rl_project_b200.
//
// Everything here is plain CUDA C++: no torch headers, so each kernel file
// compiles in seconds and can also be linked into non-torch callers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define RLB_DEVICE __device__ __forceinline__

namespace rlb {

// Error codes written to a device status word instead of trapping.  The host
// reads the word after the stream synchronises and raises a typed error.
enum StatusCode : int {
  kOk = 0,
  kTimeout = 1,      // a bounded wait ran out (code | (where << 8))
  kBadIndex = 2,     // an index (token id, block id, expert id) was out of range
  kBadShape = 3,
};

RLB_DEVICE void report(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

RLB_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

RLB_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `scratch` needs blockDim.x/32 floats.  Result broadcast to all threads.
RLB_DEVICE float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = (lane < nw) ? scratch[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

RLB_DEVICE float block_max(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = (lane < nw) ? scratch[lane] : -INFINITY;
  t = warp_max(t);
  return t;
}

// 16-byte vector of 8 bf16 values.
struct alignas(16) bf16x8 {
  __nv_bfloat162 h[4];
};

RLB_DEVICE void unpack8(const bf16x8& v, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

RLB_DEVICE bf16x8 pack8(const float* f) {
  bf16x8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

RLB_DEVICE bf16x8 ldg8(const __nv_bfloat16* p) { return *reinterpret_cast<const bf16x8*>(p); }
RLB_DEVICE void stg8(__nv_bfloat16* p, const bf16x8& v) { *reinterpret_cast<bf16x8*>(p) = v; }

RLB_DEVICE float silu(float x) { return x / (1.f + __expf(-x)); }

inline int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

}  // namespace rlb
