// SwiGLU activation on the fused [gate | up] projection output
// (src/forgeline/models/transformer/feedforward.py:26: w2(silu(w1 x) * w3 x)).
//   fwd: a = silu(g) * u                     h13 [N, 2F] -> a [N, F]
//   bwd: dg = da * u * s * (1 + g (1 - s)),  du = da * silu(g)   (s = sigmoid(g))
// Also the GELU-tanh activation of the non-SwiGLU FFN variant.
#include "common.cuh"

namespace rlb {

__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ h13, __nv_bfloat16* __restrict__ out,
                                  long long rows, int F) {
  const int chunks = F / 8;
  const long long total = rows * chunks;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / chunks;
    const int c = (int)(i % chunks) * 8;
    float g[8], u[8], o[8];
    unpack8(ldg8(h13 + r * 2 * F + c), g);
    unpack8(ldg8(h13 + r * 2 * F + F + c), u);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = silu(g[k]) * u[k];
    stg8(out + r * F + c, pack8(o));
  }
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ h13, const __nv_bfloat16* __restrict__ da,
                                  __nv_bfloat16* __restrict__ dh13, long long rows, int F) {
  const int chunks = F / 8;
  const long long total = rows * chunks;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / chunks;
    const int c = (int)(i % chunks) * 8;
    float g[8], u[8], d[8], dg[8], du[8];
    unpack8(ldg8(h13 + r * 2 * F + c), g);
    unpack8(ldg8(h13 + r * 2 * F + F + c), u);
    unpack8(ldg8(da + r * F + c), d);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float s = 1.f / (1.f + __expf(-g[k]));
      du[k] = d[k] * g[k] * s;
      dg[k] = d[k] * u[k] * s * (1.f + g[k] * (1.f - s));
    }
    stg8(dh13 + r * 2 * F + c, pack8(dg));
    stg8(dh13 + r * 2 * F + F + c, pack8(du));
  }
}

RLB_DEVICE float gelu_tanh(float x, float* dgelu) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  const float inner = k0 * (x + k1 * x * x * x);
  const float th = tanhf(inner);
  if (dgelu) *dgelu = 0.5f * (1.f + th) + 0.5f * x * (1.f - th * th) * k0 * (1.f + 3.f * k1 * x * x);
  return 0.5f * x * (1.f + th);
}

__global__ void gelu_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ dy,
                            __nv_bfloat16* __restrict__ out, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n / 8;
       i += (long long)gridDim.x * blockDim.x) {
    float v[8], o[8], g[8];
    unpack8(ldg8(x + i * 8), v);
    if (dy) unpack8(ldg8(dy + i * 8), g);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float d;
      const float y = gelu_tanh(v[k], &d);
      o[k] = dy ? g[k] * d : y;
    }
    stg8(out + i * 8, pack8(o));
  }
}

}  // namespace rlb

using namespace rlb;

static int ew_grid(long long work, int sms) {
  long long g = (work + 255) / 256;
  long long cap = (long long)sms * 16;
  return (int)(g < 1 ? 1 : (g < cap ? g : cap));
}

cudaError_t rlb_swiglu_fwd(const void* h13, void* out, long long rows, int F, int sms, cudaStream_t s) {
  if (F % 8) return cudaErrorInvalidValue;
  swiglu_fwd_kernel<<<ew_grid(rows * (F / 8), sms), 256, 0, s>>>((const __nv_bfloat16*)h13, (__nv_bfloat16*)out,
                                                                  rows, F);
  return cudaGetLastError();
}

cudaError_t rlb_swiglu_bwd(const void* h13, const void* da, void* dh13, long long rows, int F, int sms,
                           cudaStream_t s) {
  if (F % 8) return cudaErrorInvalidValue;
  swiglu_bwd_kernel<<<ew_grid(rows * (F / 8), sms), 256, 0, s>>>(
      (const __nv_bfloat16*)h13, (const __nv_bfloat16*)da, (__nv_bfloat16*)dh13, rows, F);
  return cudaGetLastError();
}

// dy == nullptr: out = gelu(x); otherwise out = dy * gelu'(x).
cudaError_t rlb_gelu(const void* x, const void* dy, void* out, long long n, int sms, cudaStream_t s) {
  if (n % 8) return cudaErrorInvalidValue;
  gelu_kernel<<<ew_grid(n / 8, sms), 256, 0, s>>>((const __nv_bfloat16*)x, (const __nv_bfloat16*)dy,
                                                  (__nv_bfloat16*)out, n);
  return cudaGetLastError();
}
