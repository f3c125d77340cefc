// Multi-tensor AdamW / Adam over every trainable tensor in ONE launch, with the
// gradient-norm clip folded in on the device (no host synchronisation).
//
// Per element (torch.optim.AdamW semantics, the optimizer the reference builds
// in src/forgeline/training/common/optim.py:24-30):
//   g  = grad * clip_coef                         (clip_coef read from device memory)
//   adamw: p -= lr * wd * p        adam: g += wd * p
//   m = b1 m + (1-b1) g;  v = b2 v + (1-b2) g^2
//   p -= lr * (m / (1-b1^t)) / (sqrt(v / (1-b2^t)) + eps)
// The fp32 master weight is updated and the bf16 compute copy is rewritten.
//
// The squared-norm reduction writes one partial per block and a single block
// folds them in a fixed order, so the norm (and the clip) is bitwise
// reproducible run to run.
#include "common.cuh"

namespace rlb {

struct AdamTensor {
  float* master;           // fp32 master weights (updated in place)
  __nv_bfloat16* param16;  // bf16 compute copy, may be null
  const void* grad;        // bf16 or fp32
  float* m;
  float* v;
  long long n;
  float wd;
  int grad_bf16;
};

struct ChunkRef {
  int tensor;
  int chunk;
};

constexpr int kChunk = 16384;

RLB_DEVICE float load_grad(const AdamTensor& t, long long i) {
  return t.grad_bf16 ? __bfloat162float(((const __nv_bfloat16*)t.grad)[i]) : ((const float*)t.grad)[i];
}

RLB_DEVICE bool aligned(const void* p, int bytes) { return (((uintptr_t)p) & (bytes - 1)) == 0; }

// 4 consecutive gradient values (vector load when aligned)
RLB_DEVICE void load_grad4(const AdamTensor& t, long long i, float* g) {
  if (t.grad_bf16) {
    const uint2 u = *(const uint2*)((const __nv_bfloat16*)t.grad + i);
    const float2 a = __bfloat1622float2(*(const __nv_bfloat162*)&u.x);
    const float2 b = __bfloat1622float2(*(const __nv_bfloat162*)&u.y);
    g[0] = a.x; g[1] = a.y; g[2] = b.x; g[3] = b.y;
  } else {
    const float4 f = *(const float4*)((const float*)t.grad + i);
    g[0] = f.x; g[1] = f.y; g[2] = f.z; g[3] = f.w;
  }
}

RLB_DEVICE bool vec_ok(const AdamTensor& t) {
  return aligned(t.master, 16) && aligned(t.m, 16) && aligned(t.v, 16) && aligned(t.grad, t.grad_bf16 ? 8 : 16) &&
         (t.param16 == nullptr || aligned(t.param16, 8));
}

__global__ void __launch_bounds__(256) sumsq_kernel(const AdamTensor* __restrict__ ts, const ChunkRef* __restrict__ chunks,
                                                    int nchunks, float* __restrict__ partial) {
  __shared__ float scratch[8];
  float acc = 0.f;
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const AdamTensor t = ts[chunks[c].tensor];
    const long long base = (long long)chunks[c].chunk * kChunk;
    const long long end = min(base + kChunk, t.n);
    long long i0 = base;
    if (vec_ok(t)) {
      const long long vend = base + ((end - base) & ~3LL);
      for (long long i = base + 4 * threadIdx.x; i < vend; i += 4 * blockDim.x) {
        float g[4];
        load_grad4(t, i, g);
        acc += g[0] * g[0] + g[1] * g[1] + g[2] * g[2] + g[3] * g[3];
      }
      i0 = vend;
    }
    for (long long i = i0 + threadIdx.x; i < end; i += blockDim.x) {
      const float g = load_grad(t, i);
      acc += g * g;
    }
  }
  acc = block_sum(acc, scratch);
  if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

// clip_coef = min(1, max_norm / (norm + 1e-6)) (torch.nn.utils.clip_grad_norm_), also
// records the norm.  max_norm <= 0 disables clipping (coef 1).
// (no __restrict__: the distributed finish reads and writes norm_coef in place)
__global__ void finish_norm_kernel(const float* partial, int parts, float max_norm, float inv_scale, float* norm_out,
                                   float* coef_out, int squared_only) {
  __shared__ float scratch[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < parts; i += blockDim.x) acc += partial[i];
  acc = block_sum(acc, scratch);
  if (threadIdx.x == 0 && squared_only) {
    norm_out[0] = acc;  // sum of squares of this rank's shards; the host all-reduces it, then finishes
    return;
  }
  if (threadIdx.x == 0) {
    const float norm = sqrtf(acc) * inv_scale;
    norm_out[0] = norm;
    float coef = inv_scale;
    if (max_norm > 0.f && norm > max_norm) coef = inv_scale * max_norm / (norm + 1e-6f);
    // non-finite gradients: skip the update entirely (coef = 0 marks it)
    if (!(norm == norm) || norm == INFINITY) coef = 0.f;
    coef_out[0] = coef;
  }
}

__global__ void __launch_bounds__(256) adam_kernel(const AdamTensor* __restrict__ ts, const ChunkRef* __restrict__ chunks,
                                                   int nchunks, const float* __restrict__ coef_ptr, float lr, float b1,
                                                   float b2, float eps, float bc1, float bc2, int decoupled) {
  const float coef = coef_ptr ? coef_ptr[0] : 1.f;
  if (coef == 0.f) return;  // non-finite step skipped
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const AdamTensor t = ts[chunks[c].tensor];
    const long long base = (long long)chunks[c].chunk * kChunk;
    const long long end = min(base + kChunk, t.n);
    long long i0 = base;
    if (vec_ok(t)) {
      const long long vend = base + ((end - base) & ~3LL);
      for (long long i = base + 4 * threadIdx.x; i < vend; i += 4 * blockDim.x) {
        float g[4];
        load_grad4(t, i, g);
        float4 p4 = *(float4*)(t.master + i), m4 = *(float4*)(t.m + i), v4 = *(float4*)(t.v + i);
        float* p = (float*)&p4;
        float* m = (float*)&m4;
        float* v = (float*)&v4;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float gk = g[k] * coef;
          if (decoupled) p[k] -= lr * t.wd * p[k];
          else gk += t.wd * p[k];
          m[k] = b1 * m[k] + (1.f - b1) * gk;
          v[k] = b2 * v[k] + (1.f - b2) * gk * gk;
          p[k] -= lr * (m[k] / bc1) / (sqrtf(v[k] / bc2) + eps);
        }
        *(float4*)(t.master + i) = p4;
        *(float4*)(t.m + i) = m4;
        *(float4*)(t.v + i) = v4;
        if (t.param16) {
          __nv_bfloat162 lo = __floats2bfloat162_rn(p[0], p[1]), hi = __floats2bfloat162_rn(p[2], p[3]);
          uint2 u;
          u.x = *(uint32_t*)&lo;
          u.y = *(uint32_t*)&hi;
          *(uint2*)(t.param16 + i) = u;
        }
      }
      i0 = vend;
    }
    for (long long i = i0 + threadIdx.x; i < end; i += blockDim.x) {
      float p = t.master[i];
      float g = load_grad(t, i) * coef;
      if (decoupled) p -= lr * t.wd * p;
      else g += t.wd * p;
      const float m = b1 * t.m[i] + (1.f - b1) * g;
      const float v = b2 * t.v[i] + (1.f - b2) * g * g;
      t.m[i] = m;
      t.v[i] = v;
      p -= lr * (m / bc1) / (sqrtf(v / bc2) + eps);
      t.master[i] = p;
      if (t.param16) t.param16[i] = __float2bfloat16(p);
    }
  }
}

}  // namespace rlb

using namespace rlb;

int rlb_adam_chunk_size() { return kChunk; }

// `tensors`/`chunks` are device arrays (built once by the host).  `partial`
// holds >= grid floats; `norm_coef` 2 floats: [norm, coef].
cudaError_t rlb_grad_norm(const void* tensors, const void* chunks, int nchunks, float* partial, int grid,
                          float max_norm, float inv_scale, float* norm_coef, int squared_only, cudaStream_t s) {
  sumsq_kernel<<<grid, 256, 0, s>>>((const AdamTensor*)tensors, (const ChunkRef*)chunks, nchunks, partial);
  finish_norm_kernel<<<1, 1024, 0, s>>>(partial, grid, max_norm, inv_scale, norm_coef, norm_coef + 1, squared_only);
  return cudaGetLastError();
}

// Second half of a distributed norm: norm_coef[0] holds the all-reduced sum of squares.
cudaError_t rlb_grad_norm_finish(float* norm_coef, float max_norm, float inv_scale, cudaStream_t s) {
  finish_norm_kernel<<<1, 32, 0, s>>>(norm_coef, 1, max_norm, inv_scale, norm_coef, norm_coef + 1, 0);
  return cudaGetLastError();
}

cudaError_t rlb_adam_step(const void* tensors, const void* chunks, int nchunks, const float* coef, float lr, float b1,
                          float b2, float eps, int step, int decoupled, int grid, cudaStream_t s) {
  const float bc1 = 1.f - powf(b1, (float)step);
  const float bc2 = 1.f - powf(b2, (float)step);
  adam_kernel<<<grid, 256, 0, s>>>((const AdamTensor*)tensors, (const ChunkRef*)chunks, nchunks, coef, lr, b1, b2, eps,
                                   bc1, bc2, decoupled);
  return cudaGetLastError();
}

int rlb_adam_tensor_desc_bytes() { return (int)sizeof(AdamTensor); }
