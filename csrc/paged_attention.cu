// Paged-KV decode attention (one new query token per sequence) for the
// continuous-batching inference engine.
//
// KV pool layout: k_pool / v_pool [num_blocks][Hkv][BLOCK=16][D] bf16, one
// block table row per sequence ([B][max_blocks] int32) and a context length
// per sequence.  One CTA handles (kv head h, sequence b, split s): it loads each
// K/V row ONCE and scores it against all G = Hq/Hkv query heads that share the
// KV head (GQA packing), with an online softmax per query head.  4 warps take
// whole 16-token blocks round-robin; their partial (max, sum, acc) are merged
// in shared memory.  With several splits per sequence (long contexts, few sequences)
// each split writes unnormalised partials and a second kernel merges them
// (flash-decoding).  Optional sliding window (last `window` positions) and
// tanh soft-cap, as in src/forgeline/models/attention/causal.py:106-130.
// Block ids are bounds-checked: an out-of-range id is reported in `status`
// and the token is skipped (no out-of-bounds read).
#include "common.cuh"

namespace rlb {

constexpr int kBlock = 16;
constexpr int kWarps = 4;

// Lane layout: a K/V row of D bf16 is D/8 16-byte vectors, so LPT = D/8 lanes
// cover one token row and a warp covers TPP = 32/LPT tokens per pass; a
// 16-token block takes PASSES = 16/TPP passes.  Lane (tok_in_pass, slice)
// holds dims [8 slice, 8 slice + 8) of its tokens.  Scores reduce over the LPT
// lanes of a token (log2 LPT shuffles); the softmax statistics (max, sum) are
// kept per lane over that lane's own tokens and merged once at the end, as are
// the P.V partial sums -- the only per-block cross-lane traffic is the score
// reduction.  Each warp takes whole blocks round-robin, so every load is a
// 16-byte vector and a warp has 2 x min(PASSES, 4) of them in flight at a time.
template <int D, int G>
__global__ void __launch_bounds__(kWarps * 32, (G <= 4 ? 4 : 2)) paged_decode_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_pool,
    const __nv_bfloat16* __restrict__ v_pool, const int* __restrict__ block_tables, const int* __restrict__ ctx_lens,
    __nv_bfloat16* __restrict__ out, float* __restrict__ part_acc, float* __restrict__ part_ml, int Hkv,
    int max_blocks, int num_blocks, int split_tokens, int n_splits, float scale, float softcap, int window,
    int* status) {
  constexpr int LPT = D / 8;          // lanes per token row
  constexpr int TPP = 32 / LPT;       // tokens per pass
  constexpr int PASSES = kBlock / TPP;
  const int h = blockIdx.x, b = blockIdx.y, sp = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slice = lane % LPT, tip = lane / LPT;
  const int Hq = Hkv * G;
  const int len = ctx_lens[b];
  const int t_begin = (window > 0 && len > window) ? len - window : 0;
  const int t0 = t_begin + sp * split_tokens;
  const int t1 = min(len, t0 + split_tokens);

  float qf[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    unpack8(ldg8(q + ((long long)b * Hq + h * G + g) * D + slice * 8), qf[g]);
#pragma unroll
    for (int e = 0; e < 8; ++e) qf[g][e] *= scale;
  }
  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
  }
  const int* bt = block_tables + (long long)b * max_blocks;
  if (t1 > t0) {
    const int jb0 = t0 / kBlock, jb1 = (t1 - 1) / kBlock;
    for (int jb = jb0 + warp; jb <= jb1; jb += kWarps) {
      const int blk = bt[jb];
      if (blk < 0 || blk >= num_blocks) {
        if (lane == 0) report(status, kBadIndex);
        continue;
      }
      const long long base = (((long long)blk * Hkv + h) * kBlock) * D + slice * 8;
      // loads go out CH passes at a time (all K and V vectors of a chunk before any use): enough
      // bytes in flight per warp while the register count stays low enough for 4 CTAs per SM
      constexpr int CH = PASSES < 4 ? PASSES : 4;
#pragma unroll
      for (int c0 = 0; c0 < PASSES; c0 += CH) {
        bf16x8 kv[CH], vv[CH];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const long long off = base + (long long)((c0 + c) * TPP + tip) * D;
          kv[c] = ldg8(k_pool + off);
          vv[c] = ldg8(v_pool + off);
        }
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int t = jb * kBlock + (c0 + c) * TPP + tip;
          const bool valid = t >= t0 && t < t1;
          float kf[8], vf[8];
          unpack8(kv[c], kf);
          unpack8(vv[c], vf);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            float s = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) s += qf[g][e] * kf[e];
#pragma unroll
            for (int o = 1; o < LPT; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (softcap > 0.f) s = tanhf(s / softcap) * softcap;
            if (!valid) continue;
            const float mn = fmaxf(m[g], s);
            const float corr = __expf(m[g] - mn);
            const float pr = __expf(s - mn);
            l[g] = l[g] * corr + pr;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[g][e] = acc[g][e] * corr + pr * vf[e];
            m[g] = mn;
          }
        }
      }
    }
  }
  // merge the TPP token lanes of each slice inside the warp, then the warps in shared memory
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int o = LPT; o < 32; o <<= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[g], o);
      const float lo = __shfl_xor_sync(0xffffffffu, l[g], o);
      const float mn = fmaxf(m[g], mo);
      const float ca = mn == -INFINITY ? 0.f : __expf(m[g] - mn);
      const float cb = mn == -INFINITY ? 0.f : __expf(mo - mn);
      l[g] = l[g] * ca + lo * cb;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float ao = __shfl_xor_sync(0xffffffffu, acc[g][e], o);
        acc[g][e] = acc[g][e] * ca + ao * cb;
      }
      m[g] = mn;
    }
  }
  __shared__ float sm_m[kWarps][G], sm_l[kWarps][G];
  __shared__ float sm_acc[kWarps][G][D];
  if (tip == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (slice == 0) {
        sm_m[warp][g] = m[g];
        sm_l[warp][g] = l[g];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) sm_acc[warp][g][slice * 8 + e] = acc[g][e];
    }
  }
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
