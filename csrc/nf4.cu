// NF4 dequantisation (src/forgeline/models/quantization/nf4.py:41-51 semantics):
// byte b holds index (b >> 4) for element 2i and (b & 15) for element 2i+1;
// value = table[index] * absmax[element / block].  One thread per byte, the
// 16-entry table in shared memory, bf16 or fp32 output.
#include "common.cuh"

namespace rlb {

__global__ void nf4_dequant_kernel(const uint8_t* __restrict__ packed, const float* __restrict__ absmax,
                                   const float* __restrict__ table, long long n, int block, void* out, int out_bf16) {
  __shared__ float lut[16];
  if (threadIdx.x < 16) lut[threadIdx.x] = table[threadIdx.x];
  __syncthreads();
  const long long nbytes = (n + 1) / 2;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nbytes;
       i += (long long)gridDim.x * blockDim.x) {
    const uint8_t b = packed[i];
    const long long e0 = 2 * i;
    const float s = absmax[e0 / block];  // block is even, so both elements share it
    const float v0 = lut[b >> 4] * s, v1 = lut[b & 15] * s;
    if (out_bf16) {
      __nv_bfloat16* o = (__nv_bfloat16*)out;
      o[e0] = __float2bfloat16(v0);
      if (e0 + 1 < n) o[e0 + 1] = __float2bfloat16(v1);
    } else {
      float* o = (float*)out;
      o[e0] = v0;
      if (e0 + 1 < n) o[e0 + 1] = v1;
    }
  }
}

}  // namespace rlb

cudaError_t rlb_nf4_dequant(const void* packed, const float* absmax, const float* table, long long n, int block,
                            void* out, int out_bf16, int sms, cudaStream_t s) {
  if (block % 2) return cudaErrorInvalidValue;
  long long work = (n + 1) / 2, g = (work + 255) / 256, cap = (long long)sms * 16;
  rlb::nf4_dequant_kernel<<<(int)(g < cap ? (g < 1 ? 1 : g) : cap), 256, 0, s>>>(
      (const uint8_t*)packed, absmax, table, n, block, out, out_bf16);
  return cudaGetLastError();
}
