// Fused MoE router (src/forgeline/models/moe/gate.py:39-79 semantics) after the router GEMM:
// one warp per token computes the scores (softmax or sigmoid of the fp32 logits), adds the
// aux-loss-free bias for selection only, keeps the top `limited` of `groups` expert groups by their
// best biased score, picks the top-k experts in descending order, gathers their unbiased scores
// (renormalised for sigmoid), scales them, and counts tokens per expert -- one launch instead of the
// ~12 PyTorch ops of the reference composition.
#include "common.cuh"

namespace rlb {

constexpr int kRouterWarps = 8;
constexpr int kRouterMaxE = 256;
constexpr int kRouterMaxK = 16;

__global__ void __launch_bounds__(kRouterWarps * 32) moe_route_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias, long long N, int E, int k, int groups,
    int limited, int sigmoid, float route_scale, float* __restrict__ scores, float* __restrict__ w_out,
    long long* __restrict__ idx_out, int* __restrict__ counts) {
  __shared__ float s_sel[kRouterWarps][kRouterMaxE];
  __shared__ int s_gkeep[kRouterWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kRouterWarps + warp;
  if (row >= N) return;
  const float* lg = logits + row * E;
  constexpr int PER = kRouterMaxE / 32;
  float s[PER], sel[PER];
  // scores
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    s[j] = e < E ? lg[e] : -INFINITY;
    m = fmaxf(m, s[j]);
  }
  if (!sigmoid) {
    m = warp_max(m);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      s[j] = e < E ? expf(s[j] - m) : 0.f;
      sum += s[j];
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int j = 0; j < PER; ++j) s[j] *= inv;
  } else {
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      s[j] = e < E ? 1.f / (1.f + expf(-s[j])) : 0.f;
    }
  }
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    if (e < E) {
      scores[row * E + e] = s[j];
      sel[j] = s[j] + (bias ? bias[e] : 0.f);
      s_sel[warp][e] = sel[j];
    } else {
      sel[j] = -INFINITY;
    }
  }
  __syncwarp();
  // group-limited routing: keep the `limited` groups with the largest best score
  if (groups > 1 && limited < groups) {
    const int gs = E / groups;
    float gmax = -INFINITY;
    if (lane < groups)
      for (int e = lane * gs; e < (lane + 1) * gs; ++e) gmax = fmaxf(gmax, s_sel[warp][e]);
    int keep = 0;
    for (int it = 0; it < limited; ++it) {  // iterative argmax over the groups (ties: lower group)
      float best = gmax;
      int bi = lane < groups ? lane : 0x7fffffff;
      if (lane >= groups || keep) best = -INFINITY;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) {
          best = ob;
          bi = oi;
        }
      }
      if (lane == bi) keep = 1;
    }
    s_gkeep[warp][lane] = keep;
    __syncwarp();
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !s_gkeep[warp][e / gs]) sel[j] = -INFINITY;
    }
  }
  // top-k, descending (ties: lower expert index)
  float wsum = 0.f, wk[kRouterMaxK];
  int ik[kRouterMaxK];
  for (int it = 0; it < k; ++it) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      if (e < E && (sel[j] > best || (sel[j] == best && e < bi))) {
        best = sel[j];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    // the owner lane removes the winner and supplies its unbiased score
    float sv = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      if (lane + 32 * j == bi) {
        sv = s[j];
        sel[j] = -INFINITY;
      }
    }
    sv = __shfl_sync(0xffffffffu, sv, bi & 31);
    wk[it] = sv;
    ik[it] = bi;
    wsum += sv;
  }
  if (lane == 0) {
    const float norm = sigmoid ? 1.f / (wsum + 1e-8f) : 1.f;
    for (int it = 0; it < k; ++it) {
      w_out[row * k + it] = wk[it] * norm * route_scale;
      idx_out[row * k + it] = ik[it];
      if (counts) atomicAdd(counts + ik[it], 1);
    }
  }
}

}  // namespace rlb

using namespace rlb;

cudaError_t rlb_moe_route(const float* logits, const float* bias, long long N, int E, int k, int groups,
                          int limited, int sigmoid, float route_scale, float* scores, float* w, long long* idx,
                          int* counts, cudaStream_t s) {
  if (N <= 0) return cudaSuccess;
  if (E < 1 || E > kRouterMaxE || k < 1 || k > kRouterMaxK || k > E || groups < 1 || groups > 32 || E % groups ||
      limited < 1 || limited > groups)
    return cudaErrorInvalidValue;
  const long long blocks = (N + kRouterWarps - 1) / kRouterWarps;
  moe_route_kernel<<<(unsigned)blocks, kRouterWarps * 32, 0, s>>>(logits, bias, N, E, k, groups, limited, sigmoid,
                                                                  route_scale, scores, w, idx, counts);
  return cudaGetLastError();
}
