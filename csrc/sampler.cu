// Fused temperature sampler: one pass over each logits row draws a token and
// returns its log-probability (the inference engine's sampling step).
//
// Sampling uses the Gumbel-max identity: argmax_i(l_i / T + G_i) with G_i
// i.i.d. standard Gumbel is an exact sample from softmax(l / T).  The Gumbel
// noise comes from a counter-based hash of (seed, row, column), so no RNG
// state is stored and a (seed, step) pair reproduces the draw.  The same pass
// keeps an online log-sum-exp of l / T, so the sampled token's log-probability
// costs nothing extra.  T = 0 gives the argmax (greedy) and the log-probability
// under T = 1.  One CTA per row; bf16 rows are read as 16-byte vectors.
#include "common.cuh"

namespace rlb {

// 64-bit finaliser of SplitMix64 (S. Vigna, public domain): a bijective mix
// whose output bits are close to independent for consecutive inputs.
RLB_DEVICE uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

// Standard Gumbel noise for (key, column): -log(-log(u)), u uniform in (0, 1).
RLB_DEVICE float gumbel(uint64_t key, uint32_t col) {
  const uint64_t h = mix64(key + 0x9e3779b97f4a7c15ULL * (uint64_t)(col + 1));
  const float u = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
  return -__logf(-__logf(u));
}

struct ArgState {
  float best;  // best perturbed score
  int idx;
  float m;     // running max of l / T
  float s;     // running sum of exp(l / T - m)
};

RLB_DEVICE void absorb(ArgState& st, float z, float score, int i) {
  if (score > st.best) {
    st.best = score;
    st.idx = i;
  }
  if (z == -INFINITY) return;  // masked entry: no probability mass
  if (z > st.m) {
    st.s = st.s * __expf(st.m - z) + 1.f;
    st.m = z;
  } else {
    st.s += __expf(z - st.m);
  }
}

RLB_DEVICE void merge(ArgState& a, const ArgState& b) {
  if (b.best > a.best || (b.best == a.best && b.idx < a.idx)) {
    a.best = b.best;
    a.idx = b.idx;
  }
  if (b.m == -INFINITY) return;
  if (a.m == -INFINITY) {
    a.m = b.m;
    a.s = b.s;
    return;
  }
  const float m = fmaxf(a.m, b.m);
  a.s = a.s * __expf(a.m - m) + b.s * __expf(b.m - m);
  a.m = m;
}

RLB_DEVICE ArgState shfl_state(const ArgState& st, int o) {
  return ArgState{__shfl_xor_sync(0xffffffffu, st.best, o), __shfl_xor_sync(0xffffffffu, st.idx, o),
                  __shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.s, o)};
}

template <int THREADS, typename T>
__global__ void __launch_bounds__(THREADS) sample_kernel(const T* __restrict__ logits, long long ld, int V,
                                                         const float* __restrict__ temperature,
                                                         unsigned long long seed, long long* __restrict__ tokens,
                                                         float* __restrict__ logprobs) {
  const int row = blockIdx.x;
  const T* x = logits + (long long)row * ld;
  const float temp = temperature[row];
  const bool greedy = !(temp > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / temp;
  const uint64_t key = mix64(seed ^ (0xd1b54a32d192ed03ULL * (uint64_t)(row + 1)));
  ArgState st{-INFINITY, 0x7fffffff, -INFINITY, 0.f};
  auto visit = [&](float l, int i) {
    const float z = l * inv_t;
    const float score = greedy ? l : z + gumbel(key, (uint32_t)i);
    absorb(st, z, score, i);
  };
  if constexpr (sizeof(T) == 2) {
    const bool vec = (V % 8 == 0) && (ld % 8 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    if (vec) {
      for (int base = threadIdx.x * 8; base < V; base += THREADS * 8) {
        float f[8];
        unpack8(ldg8(reinterpret_cast<const __nv_bfloat16*>(x) + base), f);
#pragma unroll
        for (int k = 0; k < 8; ++k) visit(f[k], base + k);
      }
    } else {
      for (int i = threadIdx.x; i < V; i += THREADS) visit(__bfloat162float(x[i]), i);
    }
  } else {
    for (int i = threadIdx.x; i < V; i += THREADS) visit((float)x[i], i);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) merge(st, shfl_state(st, o));
  __shared__ ArgState red[THREADS / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = st;
  __syncthreads();
  if (warp == 0) {
    st = lane < THREADS / 32 ? red[lane] : ArgState{-INFINITY, 0x7fffffff, -INFINITY, 0.f};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) merge(st, shfl_state(st, o));
    if (lane == 0) {
      const int tok = st.idx < V ? st.idx : 0;
      tokens[row] = tok;
      float l;
      if constexpr (sizeof(T) == 2) l = __bfloat162float(x[tok]);
      else l = (float)x[tok];
      logprobs[row] = l * inv_t - (st.m + __logf(st.s));
    }
  }
}

}  // namespace rlb

using namespace rlb;

cudaError_t rlb_sample(const void* logits, int is_bf16, long long ld, int rows, int V, const float* temperature,
                       unsigned long long seed, long long* tokens, float* logprobs, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  if (is_bf16)
    sample_kernel<1024, __nv_bfloat16><<<rows, 1024, 0, s>>>((const __nv_bfloat16*)logits, ld, V, temperature, seed,
                                                             tokens, logprobs);
  else
    sample_kernel<1024, float><<<rows, 1024, 0, s>>>((const float*)logits, ld, V, temperature, seed, tokens,
                                                     logprobs);
  return cudaGetLastError();
}
