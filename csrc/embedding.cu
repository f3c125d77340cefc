// Token embedding gather and its deterministic backward
// (src/forgeline/models/transformer/model.py:120-125: wte(idx)).
//   fwd: out[n, :] = W[idx[n], :]
//   bwd: dW[v, :] = sum_{n : idx[n] == v} dy[n, :]
// The backward consumes ids sorted on the device (with the permutation), so
// every vocabulary row is summed by ONE warp in a fixed order: no atomics,
// bitwise reproducible, fp32 accumulation.
#include "common.cuh"

namespace rlb {

__global__ void embed_fwd_kernel(const long long* __restrict__ idx, const __nv_bfloat16* __restrict__ W,
                                 __nv_bfloat16* __restrict__ out, long long n, int dim, long long vocab,
                                 int* status) {
  const int chunks = dim / 8;
  const long long total = n * chunks;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / chunks;
    const int c = (int)(i % chunks) * 8;
    const long long tok = idx[r];
    if (tok < 0 || tok >= vocab) {
      report(status, kBadIndex);
      stg8(out + r * dim + c, bf16x8{});
      continue;
    }
    stg8(out + r * dim + c, ldg8(W + tok * dim + c));
  }
}

// One warp per sorted position; only segment heads do work.
__global__ void embed_bwd_kernel(const long long* __restrict__ sorted_ids, const long long* __restrict__ perm,
                                 const __nv_bfloat16* __restrict__ dy, __nv_bfloat16* __restrict__ dW, long long n,
                                 int dim, long long vocab) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long i = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
    const long long id = sorted_ids[i];
    if (i > 0 && sorted_ids[i - 1] == id) continue;
    if (id < 0 || id >= vocab) continue;
    long long end = i + 1;
    while (end < n && sorted_ids[end] == id) ++end;
    for (int c = lane * 8; c < dim; c += 256) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (long long j = i; j < end; ++j) {
        float f[8];
        unpack8(ldg8(dy + perm[j] * dim + c), f);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] += f[k];
      }
      stg8(dW + id * dim + c, pack8(acc));
    }
  }
}

}  // namespace rlb

using namespace rlb;

cudaError_t rlb_embed_fwd(const long long* idx, const void* W, void* out, long long n, int dim, long long vocab,
                          int* status, int sms, cudaStream_t s) {
  if (dim % 8) return cudaErrorInvalidValue;
  long long work = n * (dim / 8);
  long long g = (work + 255) / 256, cap = (long long)sms * 16;
  embed_fwd_kernel<<<(int)(g < cap ? (g < 1 ? 1 : g) : cap), 256, 0, s>>>(idx, (const __nv_bfloat16*)W,
                                                                       (__nv_bfloat16*)out, n, dim, vocab, status);
  return cudaGetLastError();
}

// dW must be zero-filled by the caller (rows that no token hits stay zero).
cudaError_t rlb_embed_bwd(const long long* sorted_ids, const long long* perm, const void* dy, void* dW, long long n,
                          int dim, long long vocab, int sms, cudaStream_t s) {
  if (dim % 8) return cudaErrorInvalidValue;
  long long g = (n + 7) / 8, cap = (long long)sms * 32;
  embed_bwd_kernel<<<(int)(g < cap ? (g < 1 ? 1 : g) : cap), 256, 0, s>>>(
      sorted_ids, perm, (const __nv_bfloat16*)dy, (__nv_bfloat16*)dW, n, dim, vocab);
  return cudaGetLastError();
}
