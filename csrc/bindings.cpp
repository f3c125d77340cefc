// Torch bindings for the sm_100a kernels (module rl_project_b200._C).
// Every kernel file is plain CUDA with a C-style launcher; this file owns the
// tensor checks, the current-stream lookup and the error translation.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <mutex>
#include <unordered_map>
#include <cuda.h>
#include <cuda_runtime.h>

#include "launchers.h"
#include "tmap.h"

namespace {

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

inline int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = n;
  return n;
}

#define CHECK_OK(expr, what)                                                                 \
  do {                                                                                       \
    cudaError_t _e = (expr);                                                                 \
    TORCH_CHECK(_e == cudaSuccess, "rl_project_b200 kernel ", what, " failed: ",            \
                cudaGetErrorString(_e));                                                     \
  } while (0)

inline void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
inline void check_bf16(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
}
inline void check_contig(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}
// Every tensor a kernel dereferences must live on the device of the tensor that picks the launch device; a
// host tensor handed to a kernel is an illegal address on the GPU.
inline void check_dev(const at::Tensor& t, const at::Tensor& ref, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.device() == ref.device(), name, " must be a CUDA tensor on ", ref.device(),
              ", got ", t.device());
}
inline void check_dev(const c10::optional<at::Tensor>& t, const at::Tensor& ref, const char* name) {
  if (t.has_value()) check_dev(*t, ref, name);
}
inline long long* lptr(const at::Tensor& t) { return reinterpret_cast<long long*>(t.data_ptr<int64_t>()); }
inline const void* opt_ptr(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }

// ---------------------------------------------------------------- RMSNorm
std::vector<at::Tensor> rmsnorm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& delta, const at::Tensor& w,
                                    double eps) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_dev(w, x, "w");
  check_dev(delta, x, "delta");
  check_contig(x, "x");
  const c10::cuda::CUDAGuard g(x.device());
  const int dim = (int)x.size(-1);
  const long long rows = x.numel() / dim;
  auto y = at::empty_like(x);
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  at::Tensor h;
  if (delta.has_value()) {
    check_bf16(*delta, "delta");
    check_contig(*delta, "delta");
    h = at::empty_like(x);
  }
  CHECK_OK(rlb_rmsnorm_fwd(x.data_ptr(), opt_ptr(delta), w.data_ptr(), h.defined() ? h.data_ptr() : nullptr,
                           y.data_ptr(), rstd.data_ptr<float>(), rows, dim, (float)eps, sm_count(), cur_stream()),
           "rmsnorm_fwd");
  if (h.defined()) return {y, rstd, h};
  return {y, rstd};
}

std::vector<at::Tensor> rmsnorm_bwd(const at::Tensor& h, const at::Tensor& w, const at::Tensor& rstd,
                                    const at::Tensor& dy, const c10::optional<at::Tensor>& dres) {
  check_bf16(h, "h");
  check_bf16(dy, "dy");
  check_dev(w, h, "w");
  check_dev(rstd, h, "rstd");
  check_dev(dy, h, "dy");
  check_contig(h, "h");
  check_contig(dy, "dy");
  const c10::cuda::CUDAGuard g(h.device());
  const int dim = (int)h.size(-1);
  const long long rows = h.numel() / dim;
  auto dx = at::empty_like(h);
  const int grid = rlb_rmsnorm_bwd_parts(rows, dim, sm_count());
  auto part = at::empty({grid, dim}, h.options().dtype(at::kFloat));
  auto dw = at::empty_like(w);
  CHECK_OK(rlb_rmsnorm_bwd(h.data_ptr(), w.data_ptr(), rstd.data_ptr<float>(), dy.data_ptr(), opt_ptr(dres),
                           dx.data_ptr(), part.data_ptr<float>(), dw.data_ptr(), w.scalar_type() == at::kFloat, rows,
                           dim, sm_count(), cur_stream()),
           "rmsnorm_bwd");
  return {dx, dw};
}

// ---------------------------------------------------------------- index-error word
// One int32 per device that kernels without a caller-supplied status word report index errors into
// (first error kept).  bounds_status() reads it (synchronising) and optionally clears it.  The word is a
// plain cudaMalloc kept until the process exits (no tensor with static lifetime, which would be freed
// after the caching allocator during interpreter shutdown).
static int* bounds_word(const at::Device& d) {
  static std::mutex mu;
  static std::unordered_map<int, int*> words;
  std::lock_guard<std::mutex> lock(mu);
  auto it = words.find(d.index());
  if (it == words.end()) {
    const c10::cuda::CUDAGuard g(d);
    // allocated outside any stream capture: the first RoPE call on a device must come before capture
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    C10_CUDA_CHECK(cudaStreamIsCapturing(c10::cuda::getCurrentCUDAStream(d.index()).stream(), &cap));
    TORCH_CHECK(cap == cudaStreamCaptureStatusNone,
                "the first RoPE call on a device allocates its index-error word: make it before stream capture");
    int* w = nullptr;
    C10_CUDA_CHECK(cudaMalloc(&w, sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(w, 0, sizeof(int)));
    it = words.emplace(d.index(), w).first;
  }
  return it->second;
}

int64_t bounds_status(int64_t device, bool clear) {
  const at::Device d(at::kCUDA, (c10::DeviceIndex)device);
  const c10::cuda::CUDAGuard g(d);
  int* w = bounds_word(d);
  int v = 0;
  C10_CUDA_CHECK(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear && v) C10_CUDA_CHECK(cudaMemset(w, 0, sizeof(int)));
  return v;
}

// ---------------------------------------------------------------- NF4 GEMM
// mode 0: x [M, K] -> x W^T [M, N];  mode 1: dy [M, N] -> dy W [M, K].  W [N, K] given as NF4 packed bytes +
// absmax; K % 64 == 0.
at::Tensor nf4_gemm(const at::Tensor& A, const at::Tensor& packed, const at::Tensor& absmax, const at::Tensor& table,
                    int64_t mode, int64_t N, int64_t K, const at::Tensor& status) {
  check_bf16(A, "A");
  check_contig(A, "A");
  check_dev(packed, A, "packed");
  check_dev(absmax, A, "absmax");
  check_dev(table, A, "table");
  check_dev(status, A, "status");
  TORCH_CHECK(A.dim() == 2 && A.size(1) == (mode == 0 ? K : N), "A: [M, K] (mode 0) or [M, N] (mode 1)");
  TORCH_CHECK(packed.scalar_type() == at::kByte && packed.numel() * 2 >= N * K, "packed: uint8, N*K/2 bytes");
  TORCH_CHECK(absmax.scalar_type() == at::kFloat && absmax.numel() * 64 >= N * K, "absmax: fp32 per 64 elements");
  TORCH_CHECK(table.scalar_type() == at::kFloat && table.numel() == 16, "table: 16 fp32 levels");
  TORCH_CHECK(status.scalar_type() == at::kInt, "status: int32");
  const c10::cuda::CUDAGuard g(A.device());
  auto out = at::empty({A.size(0), mode == 0 ? N : K}, A.options());
  CHECK_OK(rlb_nf4_gemm((int)mode, (int)A.size(0), (int)N, (int)K, A.data_ptr(), packed.data_ptr(),
                        absmax.data_ptr<float>(), table.data_ptr<float>(), out.data_ptr(), status.data_ptr<int>(),
                        cur_stream()),
           "nf4_gemm");
  return out;
}

// ---------------------------------------------------------------- RoPE
std::vector<at::Tensor> rope_qkv_fwd(const at::Tensor& qkv, const at::Tensor& cos_t, const at::Tensor& sin_t,
                                     const c10::optional<at::Tensor>& positions, int64_t B, int64_t T, int64_t Hq,
                                     int64_t Hkv, int64_t D, int64_t pos_offset, bool heads_major) {
  check_bf16(qkv, "qkv");
  TORCH_CHECK(qkv.stride(-1) == 1, "qkv inner stride must be 1");
  check_dev(cos_t, qkv, "cos");
  check_dev(sin_t, qkv, "sin");
  check_dev(positions, qkv, "positions");
  const c10::cuda::CUDAGuard g(qkv.device());
  auto opts = qkv.options();
  at::Tensor q, k, v;
  if (heads_major) {
    q = at::empty({B, Hq, T, D}, opts);
    k = at::empty({B, Hkv, T, D}, opts);
    v = at::empty({B, Hkv, T, D}, opts);
  } else {
    q = at::empty({B, T, Hq, D}, opts);
    k = at::empty({B, T, Hkv, D}, opts);
    v = at::empty({B, T, Hkv, D}, opts);
  }
  const long long row_stride = qkv.stride(-2);
  CHECK_OK(rlb_rope_qkv_fwd(qkv.data_ptr(), row_stride, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                            cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
                            positions.has_value() ? positions->data_ptr<int>() : nullptr, (int)B, (int)T, (int)Hq,
                            (int)Hkv, (int)D, (int)pos_offset, heads_major ? 1 : 0, (int)cos_t.size(0),
                            bounds_word(qkv.device()), sm_count(), cur_stream()),
           "rope_qkv_fwd");
  return {q, k, v};
}

at::Tensor rope_qkv_bwd(const at::Tensor& dq, const at::Tensor& dk, const at::Tensor& dv, const at::Tensor& cos_t,
                        const at::Tensor& sin_t, const c10::optional<at::Tensor>& positions, int64_t B, int64_t T,
                        int64_t Hq, int64_t Hkv, int64_t D, int64_t pos_offset, bool heads_major) {
  check_bf16(dq, "dq");
  check_contig(dq, "dq");
  check_dev(dk, dq, "dk");
  check_dev(dv, dq, "dv");
  check_dev(cos_t, dq, "cos");
  check_dev(sin_t, dq, "sin");
  check_dev(positions, dq, "positions");
  check_contig(dk, "dk");
  check_contig(dv, "dv");
  const c10::cuda::CUDAGuard g(dq.device());
  auto dqkv = at::empty({B, T, (Hq + 2 * Hkv) * D}, dq.options());
  CHECK_OK(rlb_rope_qkv_bwd(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dqkv.data_ptr(), (Hq + 2 * Hkv) * D,
                            cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
                            positions.has_value() ? positions->data_ptr<int>() : nullptr, (int)B, (int)T, (int)Hq,
                            (int)Hkv, (int)D, (int)pos_offset, heads_major ? 1 : 0, (int)cos_t.size(0),
                            bounds_word(dq.device()), sm_count(), cur_stream()),
           "rope_qkv_bwd");
  return dqkv;
}

void rope_inplace(at::Tensor& x, const at::Tensor& cos_t, const at::Tensor& sin_t,
                  const c10::optional<at::Tensor>& positions, int64_t pos_offset, bool inverse) {
  // x viewed as [B, T, H, D] with arbitrary outer strides, inner stride 1
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() == 4 && x.stride(3) == 1, "rope_inplace expects [B,T,H,D] with unit inner stride");
  check_dev(cos_t, x, "cos");
  check_dev(sin_t, x, "sin");
  check_dev(positions, x, "positions");
  const c10::cuda::CUDAGuard g(x.device());
  CHECK_OK(rlb_rope_inplace(x.data_ptr(), (int)x.size(0), (int)x.size(1), (int)x.size(2), (int)x.size(3),
                            x.stride(0), x.stride(1), x.stride(2), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
                            positions.has_value() ? positions->data_ptr<int>() : nullptr, (int)pos_offset,
                            inverse ? 1 : 0, (int)cos_t.size(0), bounds_word(x.device()), sm_count(), cur_stream()),
           "rope_inplace");
}

// ---------------------------------------------------------------- SwiGLU / GELU
at::Tensor swiglu_fwd(const at::Tensor& h13) {
  check_bf16(h13, "h13");
  check_contig(h13, "h13");
  const c10::cuda::CUDAGuard g(h13.device());
  const int F = (int)(h13.size(-1) / 2);
  auto sizes = h13.sizes().vec();
  sizes.back() = F;
  auto out = at::empty(sizes, h13.options());
  CHECK_OK(rlb_swiglu_fwd(h13.data_ptr(), out.data_ptr(), h13.numel() / (2 * F), F, sm_count(), cur_stream()),
           "swiglu_fwd");
  return out;
}

at::Tensor swiglu_bwd(const at::Tensor& h13, const at::Tensor& da) {
  check_bf16(h13, "h13");
  check_contig(da, "da");
  const c10::cuda::CUDAGuard g(h13.device());
  const int F = (int)(h13.size(-1) / 2);
  auto dh = at::empty_like(h13);
  CHECK_OK(rlb_swiglu_bwd(h13.data_ptr(), da.data_ptr(), dh.data_ptr(), h13.numel() / (2 * F), F, sm_count(),
                          cur_stream()),
           "swiglu_bwd");
  return dh;
}

at::Tensor gelu(const at::Tensor& x, const c10::optional<at::Tensor>& dy) {
  check_bf16(x, "x");
  check_contig(x, "x");
  const c10::cuda::CUDAGuard g(x.device());
  auto out = at::empty_like(x);
  CHECK_OK(rlb_gelu(x.data_ptr(), opt_ptr(dy), out.data_ptr(), x.numel(), sm_count(), cur_stream()), "gelu");
  return out;
}

// ---------------------------------------------------------------- log-softmax gather
std::vector<at::Tensor> logprob_fwd(const at::Tensor& logits, const c10::optional<at::Tensor>& targets,
                                    bool with_entropy, const c10::optional<at::Tensor>& status) {
  check_bf16(logits, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be [N, V] with unit inner stride");
  check_dev(targets, logits, "targets");
  check_dev(status, logits, "status");
  const c10::cuda::CUDAGuard g(logits.device());
  const long long rows = logits.size(0);
  const int V = (int)logits.size(1);
  auto fopt = logits.options().dtype(at::kFloat);
  auto lse = at::empty({rows}, fopt);
  auto lp = at::empty({rows}, fopt);
  at::Tensor ent = with_entropy ? at::empty({rows}, fopt) : at::Tensor();
  const long long* tg = nullptr;
  if (targets.has_value()) {
    TORCH_CHECK(targets->scalar_type() == at::kLong && targets->is_contiguous(), "targets must be contiguous int64");
    tg = lptr(*targets);
  }
  CHECK_OK(rlb_logprob_fwd(logits.data_ptr(), logits.stride(0), rows, V, tg, lse.data_ptr<float>(),
                           lp.data_ptr<float>(), with_entropy ? ent.data_ptr<float>() : nullptr,
                           status.has_value() ? status->data_ptr<int>() : nullptr, cur_stream()),
           "logprob_fwd");
  if (with_entropy) return {lse, lp, ent};
  return {lse, lp};
}

// lse / lp (/ entropy) of each row from the LM-head GEMM's per-chunk statistics (gemm2_lse).
std::vector<at::Tensor> logprob_combine(const at::Tensor& stats, const at::Tensor& logits,
                                        const c10::optional<at::Tensor>& targets, bool with_entropy,
                                        const c10::optional<at::Tensor>& status) {
  check_bf16(logits, "logits");
  check_dev(stats, logits, "stats");
  check_dev(targets, logits, "targets");
  check_dev(status, logits, "status");
  TORCH_CHECK(stats.scalar_type() == at::kFloat && stats.dim() == 3 && stats.size(2) == 4 && stats.is_contiguous() &&
              stats.size(0) == logits.size(0), "stats must be fp32 [rows, chunks, 4]");
  const c10::cuda::CUDAGuard g(logits.device());
  const long long rows = logits.size(0);
  auto fopt = logits.options().dtype(at::kFloat);
  auto lse = at::empty({rows}, fopt);
  auto lp = at::empty({rows}, fopt);
  at::Tensor ent = with_entropy ? at::empty({rows}, fopt) : at::Tensor();
  const long long* tg = nullptr;
  if (targets.has_value()) {
    TORCH_CHECK(targets->scalar_type() == at::kLong && targets->is_contiguous(), "targets must be contiguous int64");
    tg = lptr(*targets);
  }
  CHECK_OK(rlb_logprob_combine(stats.data_ptr(), (int)stats.size(1), logits.data_ptr(), logits.stride(0), rows,
                               (int)logits.size(1), tg, lse.data_ptr<float>(), lp.data_ptr<float>(),
                               with_entropy ? ent.data_ptr<float>() : nullptr,
                               status.has_value() ? status->data_ptr<int>() : nullptr, cur_stream()),
           "logprob_combine");
  if (with_entropy) return {lse, lp, ent};
  return {lse, lp};
}

void logprob_bwd_(at::Tensor& logits, const c10::optional<at::Tensor>& targets, const at::Tensor& lse,
                  const c10::optional<at::Tensor>& g_lp, const c10::optional<at::Tensor>& ent,
                  const c10::optional<at::Tensor>& g_ent, double scale) {
  check_bf16(logits, "logits");
  check_dev(targets, logits, "targets");
  check_dev(lse, logits, "lse");
  check_dev(g_lp, logits, "g_lp");
  check_dev(ent, logits, "ent");
  check_dev(g_ent, logits, "g_ent");
  const c10::cuda::CUDAGuard g(logits.device());
  CHECK_OK(rlb_logprob_bwd(logits.data_ptr(), logits.stride(0), logits.size(0), (int)logits.size(1),
                           targets.has_value() ? lptr(*targets) : nullptr, lse.data_ptr<float>(),
                           g_lp.has_value() ? g_lp->data_ptr<float>() : nullptr,
                           ent.has_value() ? ent->data_ptr<float>() : nullptr,
                           g_ent.has_value() ? g_ent->data_ptr<float>() : nullptr, (float)scale, cur_stream()),
           "logprob_bwd");
}

// ---------------------------------------------------------------- AdamW
void grad_norm(const at::Tensor& tensors, const at::Tensor& chunks, int64_t nchunks, at::Tensor& partial,
               double max_norm, double inv_scale, at::Tensor& norm_coef, bool squared_only) {
  check_cuda(partial, "partial");
  check_dev(tensors, partial, "tensors");
  check_dev(chunks, partial, "chunks");
  check_dev(norm_coef, partial, "norm_coef");
  const c10::cuda::CUDAGuard g(partial.device());
  CHECK_OK(rlb_grad_norm(tensors.data_ptr(), chunks.data_ptr(), (int)nchunks, partial.data_ptr<float>(),
                         (int)partial.numel(), (float)max_norm, (float)inv_scale, norm_coef.data_ptr<float>(),
                         squared_only ? 1 : 0, cur_stream()),
           "grad_norm");
}

void grad_norm_finish(at::Tensor& norm_coef, double max_norm, double inv_scale) {
  check_cuda(norm_coef, "norm_coef");
  const c10::cuda::CUDAGuard g(norm_coef.device());
  CHECK_OK(rlb_grad_norm_finish(norm_coef.data_ptr<float>(), (float)max_norm, (float)inv_scale, cur_stream()),
           "grad_norm_finish");
}

void adam_step(const at::Tensor& tensors, const at::Tensor& chunks, int64_t nchunks,
               const c10::optional<at::Tensor>& coef, double lr, double b1, double b2, double eps, int64_t step,
               bool decoupled) {
  check_cuda(tensors, "tensors");
  check_dev(chunks, tensors, "chunks");
  check_dev(coef, tensors, "coef");
  const c10::cuda::CUDAGuard g(tensors.device());
  const int grid = std::min<int64_t>(nchunks, (int64_t)sm_count() * 8);
  CHECK_OK(rlb_adam_step(tensors.data_ptr(), chunks.data_ptr(), (int)nchunks,
                         coef.has_value() ? coef->data_ptr<float>() + 1 : nullptr, (float)lr, (float)b1, (float)b2,
                         (float)eps, (int)step, decoupled ? 1 : 0, grid < 1 ? 1 : grid, cur_stream()),
           "adam_step");
}

// ---------------------------------------------------------------- embedding
at::Tensor embed_fwd(const at::Tensor& idx, const at::Tensor& W, const c10::optional<at::Tensor>& status) {
  check_bf16(W, "W");
  TORCH_CHECK(idx.scalar_type() == at::kLong && idx.is_contiguous(), "idx must be contiguous int64");
  check_dev(idx, W, "idx");
  check_dev(status, W, "status");
  const c10::cuda::CUDAGuard g(W.device());
  auto sizes = idx.sizes().vec();
  sizes.push_back(W.size(1));
  auto out = at::empty(sizes, W.options());
  CHECK_OK(rlb_embed_fwd(lptr(idx), W.data_ptr(), out.data_ptr(), idx.numel(), (int)W.size(1),
                         W.size(0), status.has_value() ? status->data_ptr<int>() : nullptr, sm_count(), cur_stream()),
           "embed_fwd");
  return out;
}

at::Tensor embed_bwd(const at::Tensor& idx, const at::Tensor& dy, int64_t vocab) {
  check_bf16(dy, "dy");
  const c10::cuda::CUDAGuard g(dy.device());
  auto flat = idx.reshape({-1});
  check_dev(idx, dy, "idx");
  auto sorted = at::sort(flat);
  auto ids = std::get<0>(sorted).contiguous();
  auto perm = std::get<1>(sorted).contiguous();
  const int dim = (int)dy.size(-1);
  auto dW = at::zeros({vocab, dim}, dy.options());
  CHECK_OK(rlb_embed_bwd(lptr(ids), lptr(perm), dy.contiguous().data_ptr(),
                         dW.data_ptr(), flat.numel(), dim, vocab, sm_count(), cur_stream()),
           "embed_bwd");
  return dW;
}

// ---------------------------------------------------------------- NF4
at::Tensor nf4_dequant(const at::Tensor& packed, const at::Tensor& absmax, const at::Tensor& table, int64_t n,
                       int64_t block, bool bf16) {
  check_cuda(packed, "packed");
  check_dev(absmax, packed, "absmax");
  check_dev(table, packed, "table");
  const c10::cuda::CUDAGuard g(packed.device());
  auto out = at::empty({n}, packed.options().dtype(bf16 ? at::kBFloat16 : at::kFloat));
  CHECK_OK(rlb_nf4_dequant(packed.data_ptr(), absmax.data_ptr<float>(), table.data_ptr<float>(), n, (int)block,
                           out.data_ptr(), bf16 ? 1 : 0, sm_count(), cur_stream()),
           "nf4_dequant");
  return out;
}

// ---------------------------------------------------------------- tcgen05 GEMM
// out[M, N] (bf16 or fp32) = alpha * A B^T with A / B in K-major or MN-major storage.
void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, int64_t a_mn, int64_t b_mn, int64_t epi, int64_t M,
          int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, double alpha,
          const c10::optional<at::Tensor>& status) {
  check_bf16(A, "A");
  check_bf16(B, "B");
  check_dev(B, A, "B");
  check_dev(out, A, "out");
  check_dev(status, A, "status");
  check_cuda(out, "out");
  TORCH_CHECK((epi == 0 && out.scalar_type() == at::kBFloat16) || (epi != 0 && out.scalar_type() == at::kFloat),
              "gemm output dtype does not match the epilogue");
  const c10::cuda::CUDAGuard g(A.device());
  CHECK_OK(rlb_gemm((int)a_mn, (int)b_mn, (int)epi, (int)M, (int)N, (int)K, A.data_ptr(), lda, B.data_ptr(), ldb,
                    out.data_ptr(), ldc, (float)alpha, status.has_value() ? status->data_ptr<int>() : nullptr,
                    sm_count(), cur_stream()),
           "gemm");
}

// The same product on the 2-SM kernel (256 x 256 nsub tiles per CTA pair, TMA-store epilogue); max_ctas > 0
// caps its persistent grid (0: as many CTA pairs as fit on the device).  gemm2x adds the K-split count (> 1
// only into an fp32 output it reduce-adds to, epi 2) and the raster group height (0: default).
void gemm2x(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, int64_t a_mn, int64_t b_mn, int64_t epi,
            int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, double alpha,
            const c10::optional<at::Tensor>& status, int64_t max_ctas, int64_t nsub, int64_t splits, int64_t group_m) {
  check_bf16(A, "A");
  check_bf16(B, "B");
  check_dev(B, A, "B");
  check_dev(out, A, "out");
  check_dev(status, A, "status");
  check_cuda(out, "out");
  TORCH_CHECK((epi == 0 && out.scalar_type() == at::kBFloat16) || (epi != 0 && out.scalar_type() == at::kFloat),
              "gemm2 output dtype does not match the epilogue");
  const c10::cuda::CUDAGuard g(A.device());
  CHECK_OK(rlb_gemm2sm((int)a_mn, (int)b_mn, (int)epi, (int)nsub, (int)M, (int)N, (int)K, A.data_ptr(), lda, B.data_ptr(), ldb,
                       out.data_ptr(), ldc, (float)alpha, status.has_value() ? status->data_ptr<int>() : nullptr,
                       (int)max_ctas, cur_stream(), (int)splits, (int)group_m),
           "gemm2");
}

void gemm2(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, int64_t a_mn, int64_t b_mn, int64_t epi,
           int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, double alpha,
           const c10::optional<at::Tensor>& status, int64_t max_ctas, int64_t nsub) {
  gemm2x(A, B, out, a_mn, b_mn, epi, M, N, K, lda, ldb, ldc, alpha, status, max_ctas, nsub, 1, 0);
}

// x [M][K] times w13 = [W1; W3] ([2H][K]) with the SwiGLU activation fused into the epilogue: writes the
// projection h13 [M][2H] and the activation act [M][H].
void gemm2_swiglu(const at::Tensor& X, const at::Tensor& W13, at::Tensor& h13, at::Tensor& act, int64_t group_m,
                  int64_t max_ctas) {
  check_bf16(X, "x");
  check_bf16(W13, "w13");
  check_bf16(h13, "h13");
  check_bf16(act, "act");
  check_dev(W13, X, "w13");
  check_dev(h13, X, "h13");
  check_dev(act, X, "act");
  TORCH_CHECK(X.dim() == 2 && W13.dim() == 2 && X.size(1) == W13.size(1) && W13.size(0) % 2 == 0,
              "gemm2_swiglu: x [M, K] and w13 [2H, K] expected");
  const int64_t M = X.size(0), K = X.size(1), H = W13.size(0) / 2;
  TORCH_CHECK(X.stride(1) == 1 && W13.stride(1) == 1 && h13.stride(1) == 1 && act.is_contiguous(),
              "gemm2_swiglu: rows must be contiguous");
  TORCH_CHECK(h13.size(0) == M && h13.size(1) == 2 * H && act.size(0) == M && act.size(1) == H,
              "gemm2_swiglu: output shapes");
  const c10::cuda::CUDAGuard g(X.device());
  CHECK_OK(rlb_gemm2sm_swiglu((int)M, (int)H, (int)K, X.data_ptr(), X.stride(0), W13.data_ptr(), W13.stride(0),
                              h13.data_ptr(), h13.stride(0), act.data_ptr(), nullptr, (int)max_ctas, cur_stream(),
                              (int)group_m),
           "gemm2_swiglu");
}

// LM-head forward with the row statistics in the epilogue: logits [M][N] bf16 and stats [M][2 * ceil(N / 512)][4]
// fp32 (max, sum exp, sum exp * x, unused).
void gemm2_lse(const at::Tensor& A, const at::Tensor& B, at::Tensor& logits, at::Tensor& stats, int64_t group_m,
               int64_t max_ctas) {
  check_bf16(A, "h");
  check_bf16(B, "W");
  check_bf16(logits, "logits");
  check_dev(B, A, "W");
  check_dev(logits, A, "logits");
  check_dev(stats, A, "stats");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1) && A.stride(1) == 1 && B.stride(1) == 1,
              "gemm2_lse: h [M, K] and W [N, K] with contiguous rows expected");
  const int64_t M = A.size(0), N = B.size(0), K = A.size(1);
  TORCH_CHECK(logits.size(0) == M && logits.size(1) == N && logits.stride(1) == 1, "gemm2_lse: logits shape");
  TORCH_CHECK(stats.scalar_type() == at::kFloat && stats.is_contiguous() && stats.numel() == M * 2 * ((N + 511) / 512) * 4,
              "gemm2_lse: stats must be fp32 [M, 2 * ceil(N / 512), 4]");
  const c10::cuda::CUDAGuard g(A.device());
  CHECK_OK(rlb_gemm2sm_lse((int)M, (int)N, (int)K, A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0),
                           logits.data_ptr(), logits.stride(0), stats.data_ptr(), nullptr, (int)max_ctas, cur_stream(),
                           (int)group_m),
           "gemm2_lse");
}

// q, k, v ([B, T, H, D], token-major) = rope(split(x w^T)) for x [B*T, K] and w = [W_q; W_k; W_v] from one GEMM
// whose epilogue rotates q and k; positions [B*T] int32 (optional; else t + pos_offset).
std::vector<at::Tensor> gemm2_rope_qkv(const at::Tensor& X, const at::Tensor& W, const at::Tensor& cos_t,
                                       const at::Tensor& sin_t, const c10::optional<at::Tensor>& positions, int64_t B,
                                       int64_t T, int64_t Hq, int64_t Hkv, int64_t D, int64_t pos_offset,
                                       int64_t group_m, int64_t max_ctas) {
  check_bf16(X, "x");
  check_bf16(W, "w");
  check_dev(W, X, "w");
  check_dev(cos_t, X, "cos");
  check_dev(sin_t, X, "sin");
  check_dev(positions, X, "positions");
  TORCH_CHECK(X.dim() == 2 && W.dim() == 2 && X.size(1) == W.size(1) && X.stride(1) == 1 && W.stride(1) == 1 &&
              X.size(0) == B * T && W.size(0) == (Hq + 2 * Hkv) * D, "gemm2_rope_qkv: operand shapes");
  TORCH_CHECK(cos_t.scalar_type() == at::kFloat && sin_t.scalar_type() == at::kFloat && cos_t.is_contiguous() &&
              sin_t.is_contiguous() && cos_t.size(1) == D / 2, "gemm2_rope_qkv: cos / sin tables [rows, D/2] fp32");
  if (positions.has_value())
    TORCH_CHECK(positions->scalar_type() == at::kInt && positions->is_contiguous() && positions->numel() == B * T,
                "gemm2_rope_qkv: positions int32 [B*T]");
  const c10::cuda::CUDAGuard g(X.device());
  auto opts = X.options();
  auto q = at::empty({B, T, Hq, D}, opts), k = at::empty({B, T, Hkv, D}, opts), v = at::empty({B, T, Hkv, D}, opts);
  CHECK_OK(rlb_gemm2sm_rope_qkv((int)(B * T), (int)Hq, (int)Hkv, (int)D, (int)X.size(1), X.data_ptr(), X.stride(0),
                                W.data_ptr(), W.stride(0), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
                                positions.has_value() ? positions->data_ptr<int>() : nullptr, (int)T, (int)pos_offset,
                                (int)cos_t.size(0), bounds_word(X.device()), (int)max_ctas, cur_stream(), (int)group_m),
           "gemm2_rope_qkv");
  return {q, k, v};
}

// dh13 [M][2H] = SwiGLU backward of (dy [M][K] W2) against h13 [M][2H], W2 = the down projection's weight
// [K][H]: one GEMM whose epilogue applies the activation's backward (dh itself is never stored).
void gemm2_dgrad_swiglu(const at::Tensor& dY, const at::Tensor& W2, const at::Tensor& h13, at::Tensor& dh13,
                        int64_t group_m, int64_t max_ctas) {
  check_bf16(dY, "dy");
  check_bf16(W2, "w2");
  check_bf16(h13, "h13");
  check_bf16(dh13, "dh13");
  check_dev(W2, dY, "w2");
  check_dev(h13, dY, "h13");
  check_dev(dh13, dY, "dh13");
  TORCH_CHECK(dY.dim() == 2 && W2.dim() == 2 && dY.size(1) == W2.size(0) && dY.stride(1) == 1 && W2.stride(1) == 1,
              "gemm2_dgrad_swiglu: dy [M, K] and w2 [K, H] with contiguous rows expected");
  const int64_t M = dY.size(0), K = dY.size(1), H = W2.size(1);
  TORCH_CHECK(h13.size(0) == M && h13.size(1) == 2 * H && h13.stride(1) == 1 && dh13.size(0) == M &&
              dh13.size(1) == 2 * H && dh13.stride(1) == 1, "gemm2_dgrad_swiglu: h13 / dh13 must be [M, 2H]");
  const c10::cuda::CUDAGuard g(dY.device());
  CHECK_OK(rlb_gemm2sm_dgrad_swiglu((int)M, (int)H, (int)K, dY.data_ptr(), dY.stride(0), W2.data_ptr(), W2.stride(0),
                                    h13.data_ptr(), h13.stride(0), dh13.data_ptr(), dh13.stride(0), (int)max_ctas,
                                    cur_stream(), (int)group_m),
           "gemm2_dgrad_swiglu");
}

// Grouped GEMM (mixture-of-experts): see rlb_gemm_grouped for the two modes.
void gemm_grouped(int64_t mode, int64_t b_mn, int64_t epi, const at::Tensor& A, const at::Tensor& B, at::Tensor& out,
                  int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, double alpha,
                  int64_t groups, const c10::optional<at::Tensor>& tile_group,
                  const c10::optional<at::Tensor>& k_begin, const c10::optional<at::Tensor>& k_len, int64_t k_total,
                  const c10::optional<at::Tensor>& status) {
  check_bf16(A, "A");
  check_bf16(B, "B");
  check_dev(B, A, "B");
  check_dev(out, A, "out");
  check_dev(tile_group, A, "tile_group");
  check_dev(k_begin, A, "k_begin");
  check_dev(k_len, A, "k_len");
  check_dev(status, A, "status");
  for (const auto* t : {&tile_group, &k_begin, &k_len})
    if (t->has_value()) TORCH_CHECK((*t)->scalar_type() == at::kInt && (*t)->is_contiguous(), "int32 tables");
  TORCH_CHECK((epi == 0 && out.scalar_type() == at::kBFloat16) || (epi != 0 && out.scalar_type() == at::kFloat),
              "gemm_grouped output dtype does not match the epilogue");
  const c10::cuda::CUDAGuard g(A.device());
  CHECK_OK(rlb_gemm_grouped((int)mode, (int)b_mn, (int)epi, (int)M, (int)N, (int)K, A.data_ptr(), lda, B.data_ptr(),
                            ldb, out.data_ptr(), ldc, (float)alpha, (int)groups,
                            tile_group.has_value() ? tile_group->data_ptr<int>() : nullptr,
                            k_begin.has_value() ? k_begin->data_ptr<int>() : nullptr,
                            k_len.has_value() ? k_len->data_ptr<int>() : nullptr, k_total,
                            status.has_value() ? status->data_ptr<int>() : nullptr, sm_count(), cur_stream()),
           "gemm_grouped");
}

// Attention forward: q [B, T, Hq, D], k [B, T, Hkv, D], v [B, T, Hkv, DV] (token-major, contiguous bf16) -> out
// [B, T, Hq, DV]; lse [B, Hq, T] fp32 when defined (numel > 0).
void fmha_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& out, at::Tensor& lse,
              bool causal, double scale, int64_t window, double softcap, const at::Tensor& status) {
  check_bf16(q, "q");
  check_bf16(k, "k");
  check_bf16(v, "v");
  check_dev(k, q, "k");
  check_dev(v, q, "v");
  check_dev(out, q, "out");
  check_dev(status, q, "status");
  check_contig(q, "q");
  check_contig(k, "k");
  check_contig(v, "v");
  check_contig(out, "out");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "q, k, v: [B, T, H, D]");
  TORCH_CHECK(k.size(0) == q.size(0) && k.size(1) == q.size(1) && k.size(3) == q.size(3) && v.size(0) == k.size(0) &&
              v.size(1) == k.size(1) && v.size(2) == k.size(2), "k / v shapes do not match q");
  TORCH_CHECK(out.size(0) == q.size(0) && out.size(1) == q.size(1) && out.size(2) == q.size(2) &&
              out.size(3) == v.size(3) && out.scalar_type() == at::kBFloat16, "out: bf16 [B, T, Hq, d_v]");
  TORCH_CHECK(status.scalar_type() == at::kInt, "status: int32");
  float* lse_p = nullptr;
  if (lse.numel() > 0) {
    check_dev(lse, q, "lse");
    TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() == q.size(0) * q.size(2) * q.size(1),
                "lse: fp32 [B, Hq, T]");
    lse_p = lse.data_ptr<float>();
  }
  const c10::cuda::CUDAGuard g(q.device());
  CHECK_OK(rlb_fmha_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse_p, (int)q.size(0),
                        (int)q.size(1), (int)q.size(2), (int)k.size(2), (int)q.size(3), (int)v.size(3), causal ? 1 : 0,
                        (float)scale, (int)window, (float)softcap, status.data_ptr<int>(), cur_stream()),
           "fmha_fwd");
}

// Attention backward (same layouts as fmha_fwd): dq fp32 like q (zeroed here, accumulated by the kernel), dk / dv
// bf16 like k; lse / delta fp32 [B, Hq, T].
void fmha_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& dout,
              const at::Tensor& lse, const at::Tensor& delta, at::Tensor& dq, at::Tensor& dk, at::Tensor& dv,
              bool causal, double scale, int64_t window, double softcap, const at::Tensor& status) {
  using Ts = std::initializer_list<const at::Tensor*>;
  for (const at::Tensor* t : Ts{&q, &k, &v, &dout}) check_bf16(*t, "q/k/v/dout");
  for (const at::Tensor* t : Ts{&k, &v, &dout, &lse, &delta, &dq, &dk, &dv, &status}) check_dev(*t, q, "fmha_bwd operand");
  for (const at::Tensor* t : Ts{&q, &k, &v, &dout, &lse, &delta, &dq, &dk, &dv}) check_contig(*t, "fmha_bwd operand");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && k.sizes() == v.sizes() && dout.sizes() == q.sizes(), "[B, T, H, D] operands");
  TORCH_CHECK(dq.sizes() == q.sizes() && dq.scalar_type() == at::kFloat, "dq: fp32 like q");
  TORCH_CHECK(dk.sizes() == k.sizes() && dv.sizes() == k.sizes() && dk.scalar_type() == at::kBFloat16 &&
              dv.scalar_type() == at::kBFloat16, "dk / dv: bf16 like k");
  const int64_t rows = q.size(0) * q.size(2) * q.size(1);
  TORCH_CHECK(lse.scalar_type() == at::kFloat && delta.scalar_type() == at::kFloat && lse.numel() == rows &&
              delta.numel() == rows, "lse / delta: fp32 [B, Hq, T]");
  TORCH_CHECK(status.scalar_type() == at::kInt, "status: int32");
  const c10::cuda::CUDAGuard g(q.device());
  dq.zero_();
  CHECK_OK(rlb_fmha_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), dout.data_ptr(), lse.data_ptr<float>(),
                        delta.data_ptr<float>(), dq.data_ptr<float>(), dk.data_ptr(), dv.data_ptr(), (int)q.size(0),
                        (int)q.size(1), (int)q.size(2), (int)k.size(2), (int)q.size(3), causal ? 1 : 0, (float)scale,
                        (int)window, (float)softcap, status.data_ptr<int>(), cur_stream()),
           "fmha_bwd");
}

// out [M, N] = sum over the TP ranks of A_r [M, K] @ op(B_r), reduced in the GEMM epilogue over peer memory:
// b_mn = 0: B [N, K] (op = transpose, row-parallel output);  b_mn = 1: B [K, N] (column-parallel input gradient).
void gemm_allreduce(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, const std::vector<int64_t>& part,
                    const std::vector<int64_t>& flag, int64_t rank, int64_t epoch, double alpha,
                    const at::Tensor& status, int64_t grid, int64_t b_mn) {
  check_bf16(A, "A");
  check_bf16(B, "B");
  check_dev(B, A, "B");
  check_dev(out, A, "out");
  check_dev(status, A, "status");
  check_contig(A, "A");
  check_contig(B, "B");
  check_contig(out, "out");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && A.dim() == 2 && B.dim() == 2 && out.dim() == 2, "2-D bf16");
  const int64_t n = b_mn ? B.size(1) : B.size(0), kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(A.size(1) == kb && out.size(0) == A.size(0) && out.size(1) == n, "shape mismatch");
  TORCH_CHECK(part.size() == flag.size() && !part.empty() && part.size() <= 8, "one partial / flag slot per rank");
  TORCH_CHECK(status.scalar_type() == at::kInt, "status: int32");
  std::vector<unsigned long long> pp(part.begin(), part.end()), ff(flag.begin(), flag.end());
  const c10::cuda::CUDAGuard g(A.device());
  CHECK_OK(rlb_gemm_allreduce((int)b_mn, (int)A.size(0), (int)n, (int)A.size(1), A.data_ptr(), A.size(1),
                              B.data_ptr(), B.size(1), out.data_ptr(), out.size(1), (float)alpha, pp.data(), ff.data(),
                              (int)part.size(), (int)rank, (int)epoch, status.data_ptr<int>(), (int)grid,
                              cur_stream()),
           "gemm_allreduce");
}

// ---------------------------------------------------------------- paged KV decode
// q [B, Hq, D]; pools [num_blocks, Hkv, 16, D]; block_tables [B, max_blocks] int32; ctx_lens [B] int32
at::Tensor paged_decode(const at::Tensor& q, const at::Tensor& k_pool, const at::Tensor& v_pool,
                        const at::Tensor& block_tables, const at::Tensor& ctx_lens, int64_t split_tokens,
                        double scale, double softcap, int64_t window, const c10::optional<at::Tensor>& status) {
  check_bf16(q, "q");
  check_bf16(k_pool, "k_pool");
  check_dev(k_pool, q, "k_pool");
  check_dev(v_pool, q, "v_pool");
  check_dev(block_tables, q, "block_tables");
  check_dev(ctx_lens, q, "ctx_lens");
  check_dev(status, q, "status");
  check_contig(q, "q");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && ctx_lens.scalar_type() == at::kInt, "int32 tables");
  const c10::cuda::CUDAGuard g(q.device());
  const int B = (int)q.size(0), Hq = (int)q.size(1), D = (int)q.size(2);
  const int num_blocks = (int)k_pool.size(0), Hkv = (int)k_pool.size(1);
  const int max_blocks = (int)block_tables.size(1);
  const int max_ctx = max_blocks * 16;
  int n_splits = 1;
  if (split_tokens > 0) n_splits = (int)((max_ctx + split_tokens - 1) / split_tokens);
  if (n_splits < 1) n_splits = 1;
  auto out = at::empty_like(q);
  at::Tensor pa, pm;
  if (n_splits > 1) {
    pa = at::empty({(int64_t)B * Hq * n_splits * D}, q.options().dtype(at::kFloat));
    pm = at::empty({(int64_t)B * Hq * n_splits * 2}, q.options().dtype(at::kFloat));
  }
  CHECK_OK(rlb_paged_decode(q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), block_tables.data_ptr<int>(),
                            ctx_lens.data_ptr<int>(), out.data_ptr(), n_splits > 1 ? pa.data_ptr<float>() : nullptr,
                            n_splits > 1 ? pm.data_ptr<float>() : nullptr, B, Hq, Hkv, D, max_blocks, num_blocks,
                            n_splits > 1 ? (int)split_tokens : max_ctx, n_splits, (float)scale, (float)softcap,
                            (int)window, status.has_value() ? status->data_ptr<int>() : nullptr, cur_stream()),
           "paged_decode");
  return out;
}

void paged_write(const at::Tensor& k_new, const at::Tensor& v_new, at::Tensor& k_pool, at::Tensor& v_pool,
                 const at::Tensor& slot_block, const at::Tensor& slot_off, const c10::optional<at::Tensor>& status) {
  check_bf16(k_new, "k_new");
  check_contig(k_new, "k_new");
  check_dev(v_new, k_new, "v_new");
  check_dev(k_pool, k_new, "k_pool");
  check_dev(v_pool, k_new, "v_pool");
  check_dev(slot_block, k_new, "slot_block");
  check_dev(slot_off, k_new, "slot_off");
  check_dev(status, k_new, "status");
  check_contig(v_new, "v_new");
  const c10::cuda::CUDAGuard g(k_new.device());
  CHECK_OK(rlb_paged_write(k_new.data_ptr(), v_new.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(),
                           slot_block.data_ptr<int>(), slot_off.data_ptr<int>(), (int)k_new.size(0),
                           (int)k_pool.size(1), (int)k_pool.size(3), (int)k_pool.size(0),
                           status.has_value() ? status->data_ptr<int>() : nullptr, sm_count(), cur_stream()),
           "paged_write");
}

// ---------------------------------------------------------------- sampler
std::vector<at::Tensor> sample(const at::Tensor& logits, const at::Tensor& temperature, int64_t seed) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(-1) == 1, "logits must be [rows, V] with unit inner stride");
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 || logits.scalar_type() == at::kFloat, "bf16 or fp32 logits");
  TORCH_CHECK(temperature.scalar_type() == at::kFloat && temperature.numel() == logits.size(0),
              "one fp32 temperature per row");
  TORCH_CHECK(temperature.device() == logits.device(), "temperature must be on the logits' device");
  const c10::cuda::CUDAGuard g(logits.device());
  auto tokens = at::empty({logits.size(0)}, logits.options().dtype(at::kLong));
  auto lp = at::empty({logits.size(0)}, logits.options().dtype(at::kFloat));
  auto temp = temperature.contiguous();
  CHECK_OK(rlb_sample(logits.data_ptr(), logits.scalar_type() == at::kBFloat16, logits.stride(0),
                      (int)logits.size(0), (int)logits.size(1), temp.data_ptr<float>(),
                      (unsigned long long)seed, lptr(tokens), lp.data_ptr<float>(), cur_stream()),
           "sample");
  return {tokens, lp};
}

void wait_peers(const at::Tensor& my_flags, int64_t world, int64_t slot, int64_t epoch, int64_t limit_ns,
                const at::Tensor& status) {
  check_cuda(my_flags, "my_flags");
  check_dev(status, my_flags, "status");
  TORCH_CHECK(my_flags.scalar_type() == at::kInt && status.scalar_type() == at::kInt, "int32 flags / status");
  TORCH_CHECK(my_flags.numel() >= (slot + 1) * world, "flags too small for the slot");
  const c10::cuda::CUDAGuard g(my_flags.device());
  CHECK_OK(rlb_wait_peers(my_flags.data_ptr<int>(), (int)world, (int)slot, (int)epoch, (unsigned long long)limit_ns,
                          status.data_ptr<int>(), cur_stream()),
           "wait_peers");
}

// dst [rows, C] bf16: row i = row src_row[i] of rank src_rank[i]'s buffer (zeros where src_rank < 0)
void gather_rows(const at::Tensor& src_base, const at::Tensor& src_rank, const at::Tensor& src_row,
                 at::Tensor& dst, int64_t cap_rows, const at::Tensor& status) {
  check_bf16(dst, "dst");
  check_contig(dst, "dst");
  for (const at::Tensor* t : {&src_base, &src_rank, &src_row, &status}) check_dev(*t, dst, "gather table");
  TORCH_CHECK(src_base.scalar_type() == at::kLong && src_rank.scalar_type() == at::kInt &&
                  src_row.scalar_type() == at::kInt && status.scalar_type() == at::kInt,
              "gather tables: int64 bases, int32 ranks / rows / status");
  TORCH_CHECK(src_rank.numel() == dst.size(0) && src_row.numel() == dst.size(0), "one source per row");
  const c10::cuda::CUDAGuard g(dst.device());
  CHECK_OK(rlb_gather_rows(reinterpret_cast<const unsigned long long*>(src_base.data_ptr<int64_t>()),
                           src_rank.data_ptr<int>(), src_row.data_ptr<int>(), dst.size(0), (int)dst.size(1),
                           cap_rows, (int)src_base.numel(), dst.data_ptr(), status.data_ptr<int>(), sm_count(),
                           cur_stream()),
           "gather_rows");
}

void allgather_pull(const at::Tensor& src_base, int64_t S, at::Tensor& dst) {
  check_bf16(dst, "dst");
  check_contig(dst, "dst");
  check_dev(src_base, dst, "src_base");
  TORCH_CHECK(src_base.scalar_type() == at::kLong && dst.numel() == S * src_base.numel(), "dst: [world * S] bf16");
  const c10::cuda::CUDAGuard g(dst.device());
  CHECK_OK(rlb_allgather_pull(reinterpret_cast<const unsigned long long*>(src_base.data_ptr<int64_t>()), S,
                              (int)src_base.numel(), dst.data_ptr(), sm_count(), cur_stream()),
           "allgather_pull");
}

void multimem_bcast(const at::Tensor& src, int64_t mc_dst, int64_t nbytes) {
  check_cuda(src, "src");
  TORCH_CHECK(src.is_contiguous() && (int64_t)src.nbytes() >= nbytes, "src: contiguous, at least nbytes");
  const c10::cuda::CUDAGuard g(src.device());
  CHECK_OK(rlb_multimem_bcast(src.data_ptr(), (unsigned long long)mc_dst, nbytes, sm_count(), cur_stream()),
           "multimem_bcast");
}

// ---------------------------------------------------------------- MoE router
// -> {scores [N, E] fp32, w [N, k] fp32, idx [N, k] int64, counts [E] int32}
std::vector<at::Tensor> moe_route(const at::Tensor& logits, const c10::optional<at::Tensor>& bias, int64_t k,
                                  int64_t groups, int64_t limited, bool sigmoid, double route_scale) {
  check_cuda(logits, "logits");
  check_dev(bias, logits, "bias");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.is_contiguous(), "logits: fp32 [N, E]");
  if (bias.has_value()) TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == logits.size(1), "bias: fp32 [E]");
  const c10::cuda::CUDAGuard g(logits.device());
  const long long N = logits.size(0);
  const int E = (int)logits.size(1);
  auto scores = at::empty_like(logits);
  auto w = at::empty({N, k}, logits.options());
  auto idx = at::empty({N, k}, logits.options().dtype(at::kLong));
  auto counts = at::zeros({E}, logits.options().dtype(at::kInt));
  CHECK_OK(rlb_moe_route(logits.data_ptr<float>(), bias.has_value() ? bias->data_ptr<float>() : nullptr, N, E,
                         (int)k, (int)groups, (int)limited, sigmoid ? 1 : 0, (float)route_scale,
                         scores.data_ptr<float>(), w.data_ptr<float>(), lptr(idx), counts.data_ptr<int>(),
                         cur_stream()),
           "moe_route");
  return {scores, w, idx, counts};
}

// ---------------------------------------------------------------- fused RL loss
// -> {pl_row [G], kl_row [G], dpl [G, R], dkl [G, R]}; all inputs fp32 [G, R] (adv [G]).
std::vector<at::Tensor> rl_loss(const at::Tensor& lp_new, const at::Tensor& lp_old, const at::Tensor& lp_ref,
                                const at::Tensor& mask, const at::Tensor& adv, double eps, bool token_level,
                                bool k3) {
  check_cuda(lp_new, "lp_new");
  for (const at::Tensor* t : {&lp_old, &lp_ref, &mask}) {
    check_dev(*t, lp_new, "log-prob / mask");
    TORCH_CHECK(t->sizes() == lp_new.sizes() && t->scalar_type() == at::kFloat && t->is_contiguous(),
                "log-probs and mask: fp32 contiguous [G, R]");
  }
  check_dev(adv, lp_new, "adv");
  TORCH_CHECK(lp_new.dim() == 2 && lp_new.scalar_type() == at::kFloat && lp_new.is_contiguous(), "lp_new: fp32 [G, R]");
  TORCH_CHECK(adv.scalar_type() == at::kFloat && adv.numel() == lp_new.size(0) && adv.is_contiguous(), "adv: fp32 [G]");
  const c10::cuda::CUDAGuard g(lp_new.device());
  const int G = (int)lp_new.size(0), R = (int)lp_new.size(1);
  auto pl = at::empty({G}, lp_new.options());
  auto kl = at::empty({G}, lp_new.options());
  auto dpl = at::empty_like(lp_new);
  auto dkl = at::empty_like(lp_new);
  CHECK_OK(rlb_rl_loss(lp_new.data_ptr<float>(), lp_old.data_ptr<float>(), lp_ref.data_ptr<float>(),
                       mask.data_ptr<float>(), adv.data_ptr<float>(), G, R, (float)eps, token_level ? 1 : 0, k3 ? 1 : 0,
                       pl.data_ptr<float>(), kl.data_ptr<float>(), dpl.data_ptr<float>(), dkl.data_ptr<float>(),
                       cur_stream()),
           "rl_loss");
  return {pl, kl, dpl, dkl};
}

// ---------------------------------------------------------------- peer memory (CUDA IPC, no multicast object)
// A buffer allocated with cudaMalloc outside torch's caching allocator and rounded up to whole 2 MiB pages, so
// that the driver gives it pages of its own.  An IPC handle always names a whole allocation, so peer_handle
// exports the allocation's base (cuMemGetAddressRange) together with the buffer's offset from it, and peer_open
// adds the offset back: a pointer that is not an allocation base would otherwise map the wrong memory.
constexpr int64_t kPeerPage = 2 << 20;

at::Tensor peer_alloc(int64_t nbytes, int64_t device) {
  TORCH_CHECK(nbytes > 0, "peer_alloc: nbytes must be positive");
  const c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  const int64_t rounded = (nbytes + kPeerPage - 1) / kPeerPage * kPeerPage;
  void* p = nullptr;
  CHECK_OK(cudaMalloc(&p, (size_t)rounded), "peer_alloc");
  CHECK_OK(cudaMemset(p, 0, (size_t)rounded), "peer_alloc memset");
  CHECK_OK(cudaDeviceSynchronize(), "peer_alloc sync");
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, (c10::DeviceIndex)device);
  return torch::from_blob(p, {nbytes}, [device](void* q) {
    const c10::cuda::CUDAGuard gg((c10::DeviceIndex)device);
    cudaFree(q);
  }, opts);
}

// -> (64-byte handle of the allocation that contains buf, byte offset of buf in it)
std::tuple<py::bytes, int64_t> peer_handle(const at::Tensor& buf) {
  check_cuda(buf, "buf");
  const c10::cuda::CUDAGuard g(buf.device());
  // the driver entry point is looked up at run time (no link-time dependency on the driver library, so
  // the extension also imports on machines without a GPU driver)
  typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
  static AddressRangeFn address_range = nullptr;
  if (!address_range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    TORCH_CHECK(cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
                    q == cudaDriverEntryPointSuccess && fn != nullptr,
                "peer_handle: cuMemGetAddressRange is not available from the driver");
    address_range = (AddressRangeFn)fn;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  TORCH_CHECK(rlb_tmap::bind_thread_context(), "peer_handle: no CUDA context for this thread");
  TORCH_CHECK(address_range(&base, &size, (CUdeviceptr)buf.data_ptr()) == CUDA_SUCCESS,
              "peer_handle: cuMemGetAddressRange failed");
  const int64_t offset = (int64_t)((CUdeviceptr)buf.data_ptr() - base);
  TORCH_CHECK(offset >= 0 && (size_t)(offset + buf.nbytes()) <= size, "peer_handle: buffer outside its allocation");
  cudaIpcMemHandle_t h;
  CHECK_OK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "peer_handle");
  return {py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)), offset};
}

// -> base of the mapping (what peer_close takes); the buffer itself is at base + offset
int64_t peer_open(const py::bytes& handle, int64_t device) {
  std::string raw = handle;
  TORCH_CHECK(raw.size() == sizeof(cudaIpcMemHandle_t), "peer_open: bad handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, raw.data(), sizeof(h));
  const c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  CHECK_OK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "peer_open");
  return (int64_t)(uintptr_t)p;
}

void peer_close(int64_t base, int64_t device) {
  const c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  CHECK_OK(cudaIpcCloseMemHandle(reinterpret_cast<void*>((uintptr_t)base)), "peer_close");
}

// ---------------------------------------------------------------- fused reduce-scatter over peer memory
void signal_peers(const at::Tensor& flag_ptrs, int64_t rank, int64_t slot, int64_t epoch) {
  check_cuda(flag_ptrs, "flag_ptrs");
  TORCH_CHECK(flag_ptrs.scalar_type() == at::kLong && flag_ptrs.dim() == 1, "flag_ptrs: int64 [world]");
  const c10::cuda::CUDAGuard g(flag_ptrs.device());
  CHECK_OK(rlb_signal_peers(reinterpret_cast<const unsigned long long*>(flag_ptrs.data_ptr<int64_t>()),
                            (int)flag_ptrs.numel(), (int)rank, (int)slot, (int)epoch, cur_stream()),
           "signal_peers");
}

void fused_reduce_scatter(const at::Tensor& buf_ptrs, int64_t mc_base, const at::Tensor& my_flags, int64_t rank,
                          int64_t slot, int64_t epoch, int64_t shard, double scale, const at::Tensor& out,
                          bool accumulate, const c10::optional<at::Tensor>& sumsq, const at::Tensor& status,
                          int64_t limit_ns, int64_t ctas) {
  check_cuda(buf_ptrs, "buf_ptrs");
  TORCH_CHECK(buf_ptrs.scalar_type() == at::kLong && buf_ptrs.dim() == 1, "buf_ptrs: int64 [world]");
  TORCH_CHECK(my_flags.scalar_type() == at::kInt && my_flags.is_cuda(), "my_flags: int32 CUDA tensor");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == shard, "out: fp32 [shard]");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "out must be 16-byte aligned");
  TORCH_CHECK(shard % 8 == 0, "shard must be a multiple of 8 elements");
  TORCH_CHECK(status.scalar_type() == at::kInt && status.is_cuda(), "status: int32 CUDA tensor");
  if (sumsq.has_value()) TORCH_CHECK(sumsq->scalar_type() == at::kFloat && sumsq->is_cuda(), "sumsq: fp32 CUDA");
  const c10::cuda::CUDAGuard g(out.device());
  CHECK_OK(rlb_fused_reduce_scatter(reinterpret_cast<const unsigned long long*>(buf_ptrs.data_ptr<int64_t>()),
                                    (unsigned long long)mc_base, my_flags.data_ptr<int>(), (int)buf_ptrs.numel(),
                                    (int)rank, (int)slot, (int)epoch, shard, (float)scale, out.data_ptr<float>(),
                                    accumulate ? 1 : 0, sumsq.has_value() ? sumsq->data_ptr<float>() : nullptr,
                                    status.data_ptr<int>(), (unsigned long long)limit_ns, (int)ctas, cur_stream()),
           "fused_reduce_scatter");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "rl_project_b200 sm_100a kernels";
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("rope_qkv_fwd", &rope_qkv_fwd);
  m.def("rope_qkv_bwd", &rope_qkv_bwd);
  m.def("rope_inplace", &rope_inplace);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("gelu", &gelu);
  m.def("logprob_fwd", &logprob_fwd);
  m.def("logprob_bwd_", &logprob_bwd_);
  m.def("grad_norm", &grad_norm);
  m.def("grad_norm_finish", &grad_norm_finish);
  m.def("adam_step", &adam_step);
  m.def("adam_chunk_size", &rlb_adam_chunk_size);
  m.def("adam_tensor_desc_bytes", &rlb_adam_tensor_desc_bytes);
  m.def("embed_fwd", &embed_fwd);
  m.def("embed_bwd", &embed_bwd);
  m.def("nf4_dequant", &nf4_dequant);
  m.def("nf4_gemm", &nf4_gemm);
  m.def("gemm", &gemm);
  m.def("gemm2", &gemm2);
  m.def("gemm2x", &gemm2x);
  m.def("gemm2_swiglu", &gemm2_swiglu);
  m.def("gemm2_lse", &gemm2_lse);
  m.def("gemm2_rope_qkv", &gemm2_rope_qkv);
  m.def("gemm2_dgrad_swiglu", &gemm2_dgrad_swiglu);
  m.def("logprob_combine", &logprob_combine);
  m.def("gemm_grouped", &gemm_grouped);
  m.def("gemm_allreduce", &gemm_allreduce);
  m.def("fmha_fwd", &fmha_fwd);
  m.def("bounds_status", &bounds_status);
  m.def("fmha_bwd", &fmha_bwd);
  m.def("paged_decode", &paged_decode);
  m.def("paged_write", &paged_write);
  m.def("sample", &sample);
  m.def("rl_loss", &rl_loss);
  m.def("moe_route", &moe_route);
  m.def("peer_alloc", &peer_alloc);
  m.def("peer_handle", &peer_handle);
  m.def("peer_open", &peer_open);
  m.def("peer_close", &peer_close);
  m.def("signal_peers", &signal_peers);
  m.def("multimem_bcast", &multimem_bcast);
  m.def("allgather_pull", &allgather_pull);
  m.def("wait_peers", &wait_peers);
  m.def("gather_rows", &gather_rows);
  m.def("fused_reduce_scatter", &fused_reduce_scatter);
}
