// Paged-KV decode attention (one new query token per sequence) for the
// continuous-batching inference engine.
//
// KV pool layout: k_pool / v_pool [num_blocks][Hkv][BLOCK=16][D] bf16, one
// block table row per sequence ([B][max_blocks] int32) and a context length
// per sequence.  One CTA handles (kv head h, sequence b, split s): it loads each
// K/V row ONCE and scores it against all G = Hq/Hkv query heads that share the
// KV head (GQA packing), with an online softmax per query head.  4 warps take
// tokens round-robin; their partial (max, sum, acc) are merged in shared
// memory.  With several splits per sequence (long contexts, few sequences)
// each split writes unnormalised partials and a second kernel merges them
// (flash-decoding).  Optional sliding window (last `window` positions) and
// tanh soft-cap, as in src/forgeline/models/attention/causal.py:106-130.
// Block ids are bounds-checked: an out-of-range id is reported in `status`
// and the token is skipped (no out-of-bounds read).
#include "common.cuh"

namespace rlb {

constexpr int kBlock = 16;
constexpr int kWarps = 4;

template <int D, int G>
__global__ void __launch_bounds__(kWarps * 32) paged_decode_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_pool,
    const __nv_bfloat16* __restrict__ v_pool, const int* __restrict__ block_tables, const int* __restrict__ ctx_lens,
    __nv_bfloat16* __restrict__ out, float* __restrict__ part_acc, float* __restrict__ part_ml, int Hkv,
    int max_blocks, int num_blocks, int split_tokens, int n_splits, float scale, float softcap, int window,
    int* status) {
  constexpr int EPL = D / 32;  // elements per lane
  const int h = blockIdx.x, b = blockIdx.y, sp = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Hq = Hkv * G;
  const int len = ctx_lens[b];
  int t_begin = (window > 0 && len > window) ? len - window : 0;
  const int t0 = t_begin + sp * split_tokens;
  const int t1 = min(len, t0 + split_tokens);

  float qf[G][EPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const __nv_bfloat16* qp = q + ((long long)b * Hq + h * G + g) * D + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) qf[g][e] = __bfloat162float(qp[e]) * scale;
  }
  float m[G], l[G], acc[G][EPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[g][e] = 0.f;
  }
  const int* bt = block_tables + (long long)b * max_blocks;
  for (int t = t0 + warp; t < t1; t += kWarps) {
    const int blk = bt[t / kBlock];
    if (blk < 0 || blk >= num_blocks) {
      if (lane == 0) report(status, kBadIndex);
      continue;
    }
    const long long row = (((long long)blk * Hkv + h) * kBlock + (t % kBlock)) * D + lane * EPL;
    float kf[EPL], vf[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      kf[e] = __bfloat162float(k_pool[row + e]);
      vf[e] = __bfloat162float(v_pool[row + e]);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) s += qf[g][e] * kf[e];
      s = warp_sum(s);
      if (softcap > 0.f) s = tanhf(s / softcap) * softcap;
      const float mn = fmaxf(m[g], s);
      const float corr = __expf(m[g] - mn);
      const float p = __expf(s - mn);
      l[g] = l[g] * corr + p;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[g][e] = acc[g][e] * corr + p * vf[e];
      m[g] = mn;
    }
  }
  // merge the warps
  __shared__ float sm_m[kWarps][G], sm_l[kWarps][G];
  __shared__ float sm_acc[kWarps][G][D];
  if (lane == 0)
#pragma unroll
    for (int g = 0; g < G; ++g) {
      sm_m[warp][g] = m[g];
      sm_l[warp][g] = l[g];
    }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < EPL; ++e) sm_acc[warp][g][lane * EPL + e] = acc[g][e];
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm_m[w][g]);
    float L = 0.f, A = 0.f;
    if (M > -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float f = __expf(sm_m[w][g] - M);
        L += sm_l[w][g] * f;
        A += sm_acc[w][g][d] * f;
      }
    }
    const int hq = h * G + g;
    if (n_splits == 1) {
      out[((long long)b * Hq + hq) * D + d] = __float2bfloat16(L > 0.f ? A / L : 0.f);
    } else {
      const long long pi = ((long long)b * Hq + hq) * n_splits + sp;
      part_acc[pi * D + d] = A;
      if (d == 0) {
        part_ml[pi * 2] = M;
        part_ml[pi * 2 + 1] = L;
      }
    }
  }
}

// Merge split partials: out = sum_s acc_s e^{m_s - M} / sum_s l_s e^{m_s - M}.
template <int D>
__global__ void paged_combine_kernel(const float* __restrict__ part_acc, const float* __restrict__ part_ml,
                                     __nv_bfloat16* __restrict__ out, int n_splits) {
  const long long bh = blockIdx.x;  // b * Hq + hq
  float M = -INFINITY;
  for (int s = 0; s < n_splits; ++s) M = fmaxf(M, part_ml[(bh * n_splits + s) * 2]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.f, A = 0.f;
    if (M > -INFINITY)
      for (int s = 0; s < n_splits; ++s) {
        const long long pi = bh * n_splits + s;
        const float f = __expf(part_ml[pi * 2] - M);
        L += part_ml[pi * 2 + 1] * f;
        A += part_acc[pi * D + d] * f;
      }
    out[bh * D + d] = __float2bfloat16(L > 0.f ? A / L : 0.f);
  }
}

// Scatter the new token's K/V (one per sequence) into its slot of the pool.
__global__ void paged_write_kernel(const __nv_bfloat16* __restrict__ k_new, const __nv_bfloat16* __restrict__ v_new,
                                   __nv_bfloat16* __restrict__ k_pool, __nv_bfloat16* __restrict__ v_pool,
                                   const int* __restrict__ slot_block, const int* __restrict__ slot_off, int B, int Hkv,
                                   int D, int num_blocks, int* status) {
  const long long total = (long long)B * Hkv * D;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(i % D);
    const int hh = (int)((i / D) % Hkv);
    const int b = (int)(i / ((long long)D * Hkv));
    const int blk = slot_block[b];
    if (blk < 0 || blk >= num_blocks) {
      report(status, kBadIndex);
      continue;
    }
    const long long dst = (((long long)blk * Hkv + hh) * kBlock + slot_off[b]) * D + d;
    k_pool[dst] = k_new[i];
    v_pool[dst] = v_new[i];
  }
}

}  // namespace rlb

using namespace rlb;

#define RLB_PAGED_CASE(DD, GG)                                                                               \
  if (D == DD && G == GG) {                                                                                  \
    paged_decode_kernel<DD, GG><<<grid, kWarps * 32, 0, s>>>(                                                \
        (const __nv_bfloat16*)q, (const __nv_bfloat16*)k_pool, (const __nv_bfloat16*)v_pool, block_tables,    \
        ctx_lens, (__nv_bfloat16*)out, part_acc, part_ml, Hkv, max_blocks, num_blocks, split_tokens, n_splits, \
        scale, softcap, window, status);                                                                     \
    launched = true;                                                                                         \
  }

// q [B, Hq, D], out [B, Hq, D].  n_splits > 1 needs part_acc [B*Hq*n_splits*D] and
// part_ml [B*Hq*n_splits*2] fp32 scratch; split_tokens = tokens per split.
cudaError_t rlb_paged_decode(const void* q, const void* k_pool, const void* v_pool, const int* block_tables,
                             const int* ctx_lens, void* out, float* part_acc, float* part_ml, int B, int Hq, int Hkv,
                             int D, int max_blocks, int num_blocks, int split_tokens, int n_splits, float scale,
                             float softcap, int window, int* status, cudaStream_t s) {
  if (Hq % Hkv) return cudaErrorInvalidValue;
  const int G = Hq / Hkv;
  dim3 grid(Hkv, B, n_splits);
  bool launched = false;
  RLB_PAGED_CASE(64, 1) RLB_PAGED_CASE(64, 2) RLB_PAGED_CASE(64, 4) RLB_PAGED_CASE(64, 8)
  RLB_PAGED_CASE(128, 1) RLB_PAGED_CASE(128, 2) RLB_PAGED_CASE(128, 4) RLB_PAGED_CASE(128, 8)
  RLB_PAGED_CASE(32, 1) RLB_PAGED_CASE(32, 2) RLB_PAGED_CASE(32, 4)
  if (!launched) return cudaErrorNotSupported;
  if (n_splits > 1) {
    if (D == 64) paged_combine_kernel<64><<<B * Hq, 64, 0, s>>>(part_acc, part_ml, (__nv_bfloat16*)out, n_splits);
    else if (D == 128) paged_combine_kernel<128><<<B * Hq, 128, 0, s>>>(part_acc, part_ml, (__nv_bfloat16*)out, n_splits);
    else paged_combine_kernel<32><<<B * Hq, 32, 0, s>>>(part_acc, part_ml, (__nv_bfloat16*)out, n_splits);
  }
  return cudaGetLastError();
}

cudaError_t rlb_paged_write(const void* k_new, const void* v_new, void* k_pool, void* v_pool, const int* slot_block,
                            const int* slot_off, int B, int Hkv, int D, int num_blocks, int* status, int sms,
                            cudaStream_t s) {
  const long long total = (long long)B * Hkv * D;
  long long g = (total + 255) / 256, cap = (long long)sms * 8;
  paged_write_kernel<<<(int)(g < cap ? (g < 1 ? 1 : g) : cap), 256, 0, s>>>(
      (const __nv_bfloat16*)k_new, (const __nv_bfloat16*)v_new, (__nv_bfloat16*)k_pool, (__nv_bfloat16*)v_pool,
      slot_block, slot_off, B, Hkv, D, num_blocks, status);
  return cudaGetLastError();
}
