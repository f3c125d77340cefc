// Fused clipped-surrogate + KL loss of GRPO / PPO over per-token log-probs
// (src/forgeline/training/grpo.py:187-209 and training/common/logprobs.py:32-56 compute it
// with ~20 separate elementwise and reduction ops).
//
// One CTA per sequence g reads new / old / ref / mask once to form the masked sums, then
// once more to write the gradient of its two terms with respect to `new`:
//   ratio   sequence level: r = exp(sum((new - old) m) / M), M = max(sum(m), 1)
//           token level:    r_t = exp(new_t - old_t)
//   pl      -min(r A, clip(r, 1 - eps, 1 + eps) A)   (token level: masked mean over t)
//   kl      logprob-diff: sum((ref - new) m) / M
//           k3:           sum((exp(d) - d - 1) m) / M, d = ref - new
// d pl / d r is -A where r A <= clip(r) A and 0 elsewhere (the subgradient PyTorch's min / clamp
// give, ties included).  The batch combination (mean over sequences, the optional clamp of the
// KL at 0) is a handful of scalars and stays on the host side of the op.
#include "common.cuh"

namespace rlb {

constexpr int kLossThreads = 256;

RLB_DEVICE float surrogate_grad(float r, float A, float eps) {
  const float c = fminf(fmaxf(r, 1.f - eps), 1.f + eps);
  return (r * A <= c * A) ? -A : 0.f;
}

RLB_DEVICE float surrogate(float r, float A, float eps) {
  const float c = fminf(fmaxf(r, 1.f - eps), 1.f + eps);
  return -fminf(r * A, c * A);
}

__global__ void __launch_bounds__(kLossThreads) rl_loss_kernel(
    const float* __restrict__ lp_new, const float* __restrict__ lp_old, const float* __restrict__ lp_ref,
    const float* __restrict__ mask, const float* __restrict__ adv, int R, float eps, int token_level, int k3,
    float* __restrict__ pl_row, float* __restrict__ kl_row, float* __restrict__ dpl, float* __restrict__ dkl) {
  __shared__ float red[kLossThreads / 32];
  const int g = blockIdx.x;
  const long long base = (long long)g * R;
  const float A = adv[g];
  float m = 0.f, s_ratio = 0.f, s_kl = 0.f, s_tok = 0.f;
  for (int t = threadIdx.x; t < R; t += kLossThreads) {
    const float mk = mask[base + t];
    const float nw = lp_new[base + t], od = lp_old[base + t];
    const float d = lp_ref[base + t] - nw;
    m += mk;
    s_ratio += (nw - od) * mk;
    s_kl += (k3 ? (__expf(d) - d - 1.f) : d) * mk;
    if (token_level) s_tok += surrogate(__expf(nw - od), A, eps) * mk;
  }
  m = block_sum(m, red);
  s_ratio = block_sum(s_ratio, red);
  s_kl = block_sum(s_kl, red);
  s_tok = block_sum(s_tok, red);
  const float M = fmaxf(m, 1.f);
  const float r_seq = __expf(s_ratio / M);
  if (threadIdx.x == 0) {
    pl_row[g] = token_level ? s_tok / M : surrogate(r_seq, A, eps);
    kl_row[g] = s_kl / M;
  }
  const float g_seq = surrogate_grad(r_seq, A, eps) * r_seq / M;
  for (int t = threadIdx.x; t < R; t += kLossThreads) {
    const float mk = mask[base + t];
    const float nw = lp_new[base + t];
    float gp;
    if (token_level) {
      const float r = __expf(nw - lp_old[base + t]);
      gp = surrogate_grad(r, A, eps) * r * mk / M;
    } else {
      gp = g_seq * mk;
    }
    const float d = lp_ref[base + t] - nw;
    dpl[base + t] = gp;
    dkl[base + t] = (k3 ? (1.f - __expf(d)) : -1.f) * mk / M;
  }
}

}  // namespace rlb

using namespace rlb;

cudaError_t rlb_rl_loss(const float* lp_new, const float* lp_old, const float* lp_ref, const float* mask,
                        const float* adv, int G, int R, float eps, int token_level, int k3, float* pl_row,
                        float* kl_row, float* dpl, float* dkl, cudaStream_t s) {
  if (G <= 0 || R <= 0) return cudaSuccess;
  rl_loss_kernel<<<G, kLossThreads, 0, s>>>(lp_new, lp_old, lp_ref, mask, adv, R, eps, token_level, k3, pl_row,
                                            kl_row, dpl, dkl);
  return cudaGetLastError();
}
