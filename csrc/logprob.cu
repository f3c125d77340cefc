// Fused log-softmax over the vocabulary, gathered at a target id.
//
// Forward (one pass over each bf16 logits row, online max / sum-exp):
//   lse[r] = log sum_j exp(x_rj);  lp[r] = x_r,tgt - lse[r]  (0 when tgt < 0)
//   ent[r] = lse[r] - sum_j p_rj x_rj        (optional; entropy of the row)
// Backward, written IN PLACE over the logits row:
//   dx_rj = g_lp[r] * (1[j == tgt] - p_rj)  -  g_ent[r] * p_rj * (log p_rj + ent[r])
//
// This replaces F.cross_entropy (src/forgeline/models/transformer/model.py:154)
// and token_logprobs_from_logits (src/forgeline/models/policy.py:47-50):
// the [N, V] logits exist only in bf16 and never as an fp32 tensor.
#include "common.cuh"

namespace rlb {

struct OnlineStats {
  float m, s, t;  // running max, sum exp(x - m), sum exp(x - m) * x
};

RLB_DEVICE void online_add(OnlineStats& a, float x, bool with_t) {
  if (x > a.m) {
    const float f = __expf(a.m - x);
    a.s = a.s * f + 1.f;
    if (with_t) a.t = a.t * f + x;
    a.m = x;
  } else {
    const float e = __expf(x - a.m);
    a.s += e;
    if (with_t) a.t += e * x;
  }
}

RLB_DEVICE OnlineStats online_merge(OnlineStats a, OnlineStats b) {
  if (b.m == -INFINITY) return a;
  if (a.m == -INFINITY) return b;
  const float m = fmaxf(a.m, b.m);
  const float fa = __expf(a.m - m), fb = __expf(b.m - m);
  return OnlineStats{m, a.s * fa + b.s * fb, a.t * fa + b.t * fb};
}

template <int THREADS>
__global__ void __launch_bounds__(THREADS) logprob_fwd_kernel(
    const __nv_bfloat16* __restrict__ logits, long long ld, int V, const long long* __restrict__ tgt,
    float* __restrict__ lse_out, float* __restrict__ lp_out, float* __restrict__ ent_out, int* status) {
  __shared__ OnlineStats red[THREADS / 32];
  const long long r = blockIdx.x;
  const __nv_bfloat16* row = logits + r * ld;
  const bool with_t = ent_out != nullptr;
  OnlineStats st{-INFINITY, 0.f, 0.f};
  const bool vec = (ld % 8 == 0);
  int tail_start = 0;
  if (vec) {
    const int nv = V / 8;
    for (int i = threadIdx.x; i < nv; i += THREADS) {
      float f[8];
      unpack8(ldg8(row + (long long)i * 8), f);
      float bm = f[0];
#pragma unroll
      for (int k = 1; k < 8; ++k) bm = fmaxf(bm, f[k]);
      // fold 8 values with one rescale
      const float m = fmaxf(st.m, bm);
      float s = st.s * __expf(st.m - m), t = with_t ? st.t * __expf(st.m - m) : 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float e = __expf(f[k] - m);
        s += e;
        if (with_t) t += e * f[k];
      }
      st = OnlineStats{m, s, t};
    }
    tail_start = nv * 8;
  }
  for (int j = tail_start + threadIdx.x; j < V; j += THREADS) online_add(st, __bfloat162float(row[j]), with_t);
  // warp merge
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    OnlineStats other{__shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.s, o),
                      __shfl_xor_sync(0xffffffffu, st.t, o)};
    st = online_merge(st, other);
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = st;
  __syncthreads();
  if (threadIdx.x == 0) {
    OnlineStats a = red[0];
    for (int w = 1; w < THREADS / 32; ++w) a = online_merge(a, red[w]);
    const float lse = a.m + logf(a.s);
    lse_out[r] = lse;
    const long long tg = tgt ? tgt[r] : -1;
    float lp = 0.f;
    if (tg >= 0) {
      if (tg < V) lp = __bfloat162float(row[tg]) - lse;
      else report(status, kBadIndex);
    }
    if (lp_out) lp_out[r] = lp;
    if (ent_out) ent_out[r] = lse - a.t / a.s;
  }
}

// Log-sum-exp, target log-prob and entropy of each row from per-chunk statistics {max, sum exp(x - max),
// sum exp(x - max) * x} that the LM-head GEMM's epilogue wrote ([rows][chunks] float4): one warp per row
// merges its chunks (the online merge above), then reads the target's bf16 logit.  Same outputs as
// logprob_fwd_kernel, without a pass over the logits.
__global__ void logprob_combine_kernel(const float4* __restrict__ stats, int chunks, const __nv_bfloat16* __restrict__ logits,
                                       long long ld, int V, long long rows, const long long* __restrict__ tgt,
                                       float* __restrict__ lse_out, float* __restrict__ lp_out,
                                       float* __restrict__ ent_out, int* status) {
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  OnlineStats st{-INFINITY, 0.f, 0.f};
  const float4* row = stats + r * chunks;
  for (int i = lane; i < chunks; i += 32) {
    const float4 c = row[i];
    st = online_merge(st, OnlineStats{c.x, c.y, c.z});
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    OnlineStats other{__shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.s, o),
                      __shfl_xor_sync(0xffffffffu, st.t, o)};
    st = online_merge(st, other);
  }
  if (lane == 0) {
    const float lse = st.m + logf(st.s);
    lse_out[r] = lse;
    const long long tg = tgt ? tgt[r] : -1;
    float lp = 0.f;
    if (tg >= 0) {
      if (tg < V) lp = __bfloat162float(logits[r * ld + tg]) - lse;
      else report(status, kBadIndex);
    }
    if (lp_out) lp_out[r] = lp;
    if (ent_out) ent_out[r] = lse - st.t / st.s;
  }
}

template <int THREADS>
__global__ void __launch_bounds__(THREADS) logprob_bwd_kernel(
    __nv_bfloat16* __restrict__ logits, long long ld, int V, const long long* __restrict__ tgt,
    const float* __restrict__ lse, const float* __restrict__ g_lp, const float* __restrict__ ent,
    const float* __restrict__ g_ent, float scale) {
  const long long r = blockIdx.x;
  __nv_bfloat16* row = logits + r * ld;
  const float L = lse[r];
  const long long tg = tgt ? tgt[r] : -1;
  // rows with an ignored target output lp = 0 (a constant): no gradient through that term
  const float a = (g_lp && tg >= 0) ? g_lp[r] * scale : 0.f;
  const float b = g_ent ? g_ent[r] * scale : 0.f;
  const float H = (g_ent && ent) ? ent[r] : 0.f;
  const bool vec = (ld % 8 == 0);
  int tail_start = 0;
  if (vec) {
    const int nv = V / 8;
    for (int i = threadIdx.x; i < nv; i += THREADS) {
      float f[8], o[8];
      unpack8(ldg8(row + (long long)i * 8), f);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float logp = f[k] - L;
        const float p = __expf(logp);
        float d = -a * p;
        if (b != 0.f) d -= b * p * (logp + H);
        if ((long long)(i * 8 + k) == tg) d += a;
        o[k] = d;
      }
      stg8(row + (long long)i * 8, pack8(o));
    }
    tail_start = nv * 8;
  }
  for (int j = tail_start + threadIdx.x; j < V; j += THREADS) {
    const float logp = __bfloat162float(row[j]) - L;
    const float p = __expf(logp);
    float d = -a * p;
    if (b != 0.f) d -= b * p * (logp + H);
    if ((long long)j == tg) d += a;
    row[j] = __float2bfloat16(d);
  }
}

}  // namespace rlb

using namespace rlb;

cudaError_t rlb_logprob_fwd(const void* logits, long long ld, long long rows, int V, const long long* tgt,
                            float* lse, float* lp, float* ent, int* status, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  logprob_fwd_kernel<512><<<(unsigned)rows, 512, 0, s>>>((const __nv_bfloat16*)logits, ld, V, tgt, lse, lp, ent,
                                                         status);
  return cudaGetLastError();
}

cudaError_t rlb_logprob_combine(const void* stats, int chunks, const void* logits, long long ld, long long rows, int V,
                                const long long* tgt, float* lse, float* lp, float* ent, int* status, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  const int warps = 8;
  logprob_combine_kernel<<<(unsigned)((rows + warps - 1) / warps), 32 * warps, 0, s>>>(
      (const float4*)stats, chunks, (const __nv_bfloat16*)logits, ld, V, rows, tgt, lse, lp, ent, status);
  return cudaGetLastError();
}

cudaError_t rlb_logprob_bwd(void* logits, long long ld, long long rows, int V, const long long* tgt,
                            const float* lse, const float* g_lp, const float* ent, const float* g_ent, float scale,
                            cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  logprob_bwd_kernel<512><<<(unsigned)rows, 512, 0, s>>>((__nv_bfloat16*)logits, ld, V, tgt, lse, g_lp, ent, g_ent,
                                                         scale);
  return cudaGetLastError();
}
