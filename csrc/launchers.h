// C-style launchers exported by the kernel translation units.
#pragma once
#include <cuda_runtime.h>

cudaError_t rlb_rmsnorm_fwd(const void* x, const void* delta, const void* w, void* h_out, void* y, float* rstd,
                            long long rows, int dim, float eps, int sms, cudaStream_t s);
int rlb_rmsnorm_bwd_grid(long long rows, int sms);
int rlb_rmsnorm_bwd_parts(long long rows, int dim, int sms);
cudaError_t rlb_rmsnorm_bwd(const void* h, const void* w, const float* rstd, const void* dy, const void* dres,
                            void* dx, float* dw_part, void* dw_out, int dw_is_f32, long long rows, int dim, int sms,
                            cudaStream_t s);

// table_rows: rows of the cos / sin tables; a position outside them is reported in `status` (kBadIndex).
cudaError_t rlb_rope_qkv_fwd(const void* qkv, long long row_stride, void* q, void* k, void* v, const float* cos_t,
                             const float* sin_t, const int* positions, int B, int T, int Hq, int Hkv, int D,
                             int pos_offset, int heads_major, int table_rows, int* status, int sms, cudaStream_t s);
cudaError_t rlb_rope_qkv_bwd(const void* dq, const void* dk, const void* dv, void* dqkv, long long row_stride,
                             const float* cos_t, const float* sin_t, const int* positions, int B, int T, int Hq,
                             int Hkv, int D, int pos_offset, int heads_major, int table_rows, int* status, int sms,
                             cudaStream_t s);
cudaError_t rlb_rope_inplace(void* x, int B, int T, int H, int D, long long sb, long long st, long long sh,
                             const float* cos_t, const float* sin_t, const int* positions, int pos_offset,
                             int inverse, int table_rows, int* status, int sms, cudaStream_t s);

cudaError_t rlb_swiglu_fwd(const void* h13, void* out, long long rows, int F, int sms, cudaStream_t s);
cudaError_t rlb_swiglu_bwd(const void* h13, const void* da, void* dh13, long long rows, int F, int sms,
                           cudaStream_t s);
cudaError_t rlb_gelu(const void* x, const void* dy, void* out, long long n, int sms, cudaStream_t s);

cudaError_t rlb_logprob_fwd(const void* logits, long long ld, long long rows, int V, const long long* tgt,
                            float* lse, float* lp, float* ent, int* status, cudaStream_t s);
cudaError_t rlb_logprob_bwd(void* logits, long long ld, long long rows, int V, const long long* tgt,
                            const float* lse, const float* g_lp, const float* ent, const float* g_ent, float scale,
                            cudaStream_t s);

int rlb_adam_chunk_size();
int rlb_adam_tensor_desc_bytes();
cudaError_t rlb_grad_norm(const void* tensors, const void* chunks, int nchunks, float* partial, int grid,
                          float max_norm, float inv_scale, float* norm_coef, int squared_only, cudaStream_t s);
cudaError_t rlb_grad_norm_finish(float* norm_coef, float max_norm, float inv_scale, cudaStream_t s);
cudaError_t rlb_adam_step(const void* tensors, const void* chunks, int nchunks, const float* coef, float lr, float b1,
                          float b2, float eps, int step, int decoupled, int grid, cudaStream_t s);

cudaError_t rlb_embed_fwd(const long long* idx, const void* W, void* out, long long n, int dim, long long vocab,
                          int* status, int sms, cudaStream_t s);
cudaError_t rlb_embed_bwd(const long long* sorted_ids, const long long* perm, const void* dy, void* dW, long long n,
                          int dim, long long vocab, int sms, cudaStream_t s);

cudaError_t rlb_nf4_dequant(const void* packed, const float* absmax, const float* table, long long n, int block,
                            void* out, int out_bf16, int sms, cudaStream_t s);

cudaError_t rlb_gemm(int a_mn, int b_mn, int epi, int M, int N, int K, const void* A, long long lda, const void* B,
                     long long ldb, void* C, long long ldc, float alpha, int* status, int sms, cudaStream_t s);

// 2-SM variant (CTA pairs, 256 x 256 nsub tiles, nsub 1 or 2): same operands and epilogues; max_ctas > 0
// caps the grid; splits > 1 (epi 2 only) splits each tile's K into ranges that reduce-add into C; group_m is
// the raster group height in M tiles (0: default).
cudaError_t rlb_gemm2sm(int a_mn, int b_mn, int epi, int nsub, int M, int N, int K, const void* A, long long lda,
                        const void* B, long long ldb, void* C, long long ldc, float alpha, int* status, int max_ctas,
                        cudaStream_t s, int splits = 1, int group_m = 0);

// Gated-FFN forward on the 2-SM kernel: h13 = x w13^T ([M][2H], pitch ldh) and act = silu(gate) * up ([M][H])
// from one GEMM whose epilogue applies the activation.
cudaError_t rlb_gemm2sm_swiglu(int M, int H, int K, const void* X, long long ldx, const void* W13, long long ldw,
                               void* H13, long long ldh, void* act, int* status, int max_ctas, cudaStream_t s,
                               int group_m);

// LM-head forward with per-row statistics of each 256-column half tile in the epilogue (see gemm_2sm.cu).
cudaError_t rlb_gemm2sm_lse(int M, int N, int K, const void* A, long long lda, const void* B, long long ldb,
                            void* C, long long ldc, void* stats, int* status, int max_ctas, cudaStream_t s,
                            int group_m);
// Row log-sum-exp / target log-prob / entropy from those statistics (logprob.cu).
cudaError_t rlb_logprob_combine(const void* stats, int chunks, const void* logits, long long ld, long long rows, int V,
                                const long long* tgt, float* lse, float* lp, float* ent, int* status, cudaStream_t s);

// Attention input projection with RoPE and the q / k / v split in the epilogue (see gemm_2sm.cu).
cudaError_t rlb_gemm2sm_rope_qkv(int M, int Hq, int Hkv, int D, int K, const void* X, long long ldx, const void* W,
                                 long long ldw, void* q, void* k, void* v, const float* cos_t, const float* sin_t,
                                 const int* positions, int seq_T, int pos_offset, int table_rows, int* err,
                                 int max_ctas, cudaStream_t s, int group_m);

// Gated-FFN down projection's input gradient with the SwiGLU backward in the epilogue (see gemm_2sm.cu).
cudaError_t rlb_gemm2sm_dgrad_swiglu(int M, int H, int K, const void* dY, long long ldy, const void* W2, long long ldw,
                                     const void* h13, long long ldh, void* dh13, long long ldd, int max_ctas,
                                     cudaStream_t s, int group_m);

cudaError_t rlb_gemm_grouped(int mode, int b_mn, int epi, int M, int N, int K, const void* A, long long lda,
                             const void* B, long long ldb, void* C, long long ldc, float alpha, int groups,
                             const int* tile_group, const int* k_begin, const int* k_len, long long k_total,
                             int* status, int sms, cudaStream_t s);

// Row-parallel linear with the tensor-parallel all-reduce fused into the GEMM epilogue.
cudaError_t rlb_gemm_allreduce(int b_mn, int M, int N, int K, const void* A, long long lda, const void* B,
                               long long ldb, void* C, long long ldc, float alpha, const unsigned long long* part,
                               const unsigned long long* flag, int world, int rank, int epoch, int* status,
                               int grid, cudaStream_t s);

// NF4-weight GEMM with dequantisation in the tcgen05 main loop: mode 0 C[M][N] = A[M][K] W^T, mode 1
// C[M][K] = A[M][N] W; W [N][K] as NF4 (packed bytes, fp32 absmax per 64 elements, 16-level table).
cudaError_t rlb_nf4_gemm(int mode, int M, int N, int K, const void* A, const void* packed, const float* absmax,
                         const float* table, void* C, int* status, cudaStream_t s);

// Fused attention forward (tcgen05): q [B][T][Hq][D], k [B][T][Hkv][D], v [B][T][Hkv][DV], out [B][T][Hq][DV]
// bf16; lse [B][Hq][T] fp32 (natural log) or null.  (D, DV) = (64, 64), (128, 128) or (192, 128).
// window > 0: sliding window (t - s < window); softcap > 0: logits cap * tanh(logit / cap).
cudaError_t rlb_fmha_fwd(const void* q, const void* k, const void* v, void* out, float* lse, int B, int T, int Hq,
                         int Hkv, int D, int DV, int causal, float scale, int window, float softcap, int* status,
                         cudaStream_t s);
// Fused attention backward: dq fp32 [B][T][Hq][D] (zeroed by the caller, accumulated), dk / dv bf16
// [B][T][Hkv][D]; lse / delta fp32 [B][Hq][T] (delta = rowsum(dout * out)).
cudaError_t rlb_fmha_bwd(const void* q, const void* k, const void* v, const void* dout, const float* lse,
                         const float* delta, float* dq, void* dk, void* dv, int B, int T, int Hq, int Hkv, int D,
                         int causal, float scale, int window, float softcap, int* status, cudaStream_t s);

cudaError_t rlb_paged_decode(const void* q, const void* k_pool, const void* v_pool, const int* block_tables,
                             const int* ctx_lens, void* out, float* part_acc, float* part_ml, int B, int Hq, int Hkv,
                             int D, int max_blocks, int num_blocks, int split_tokens, int n_splits, float scale,
                             float softcap, int window, int* status, cudaStream_t s);
cudaError_t rlb_paged_write(const void* k_new, const void* v_new, void* k_pool, void* v_pool, const int* slot_block,
                            const int* slot_off, int B, int Hkv, int D, int num_blocks, int* status, int sms,
                            cudaStream_t s);

// Fused temperature sampler (Gumbel-max) with the sampled token's log-probability.
cudaError_t rlb_sample(const void* logits, int is_bf16, long long ld, int rows, int V, const float* temperature,
                       unsigned long long seed, long long* tokens, float* logprobs, cudaStream_t s);

// Reduce-scatter over peer memory fused with cast, scale, accumulation and the squared-norm partial.
cudaError_t rlb_signal_peers(const unsigned long long* flag_ptrs, int world, int rank, int slot, int epoch,
                             cudaStream_t s);
cudaError_t rlb_fused_reduce_scatter(const unsigned long long* buf_ptrs, unsigned long long mc_base,
                                     const int* my_flags, int world, int rank, int slot, int epoch, long long shard,
                                     float scale, float* out, int accumulate, float* sumsq, int* status,
                                     unsigned long long limit_ns, int ctas, cudaStream_t s);

// Fused clipped-surrogate + KL loss over per-token log-probs (GRPO / PPO), with the gradient wrt lp_new.
cudaError_t rlb_rl_loss(const float* lp_new, const float* lp_old, const float* lp_ref, const float* mask,
                        const float* adv, int G, int R, float eps, int token_level, int k3, float* pl_row,
                        float* kl_row, float* dpl, float* dkl, cudaStream_t s);

// Bounded wait for every peer's flag of `slot`; row gather from peer buffers (expert-parallel exchange).
cudaError_t rlb_wait_peers(const int* my_flags, int world, int slot, int epoch, unsigned long long limit_ns,
                           int* status, cudaStream_t s);
cudaError_t rlb_gather_rows(const unsigned long long* src_base, const int* src_rank, const int* src_row,
                            long long rows, int C, long long cap_rows, int world, void* dst, int* status, int sms,
                            cudaStream_t s);

// All-gather of equal bf16 shards from every rank's peer-visible buffer into dst [world * S].
cudaError_t rlb_allgather_pull(const unsigned long long* src_base, long long S, int world, void* dst, int sms,
                               cudaStream_t s);

// NVLS broadcast: store `nbytes` (multiple of 16) from local `src` through the multicast address `mc_dst`.
cudaError_t rlb_multimem_bcast(const void* src, unsigned long long mc_dst, long long nbytes, int sms,
                               cudaStream_t s);

// Fused MoE router after the router GEMM: scores, group-limited top-k, weights, per-expert counts.
cudaError_t rlb_moe_route(const float* logits, const float* bias, long long N, int E, int k, int groups,
                          int limited, int sigmoid, float route_scale, float* scores, float* w, long long* idx,
                          int* counts, cudaStream_t s);

// RMSNorm backward that allocates nothing (no counterpart in the reference):
// the dw partial sums live in a fixed 4 MiB file-scope __device__ array per
// device instead of a caller-allocated buffer.  Returns a cudaError_t value;
// dims that are not a multiple of 256 or exceed 8192 give cudaErrorInvalidValue.
// Overlapping calls on one device race on the shared scratch.
extern "C" int rlb_rmsnorm_bwd_noalloc(const void* h, const void* w, const float* rstd, const void* dy,
                                       const void* dres, void* dx, void* dw_out, int dw_is_f32, long long rows,
                                       int dim, cudaStream_t stream);
extern "C" long long rlb_rmsnorm_bwd_noalloc_scratch_bytes();
// Per-device setup of the above for the current device, done ahead of time (a caller that will run the
// backward from an out-of-memory path calls it while memory is still free).  Returns a cudaError_t value.
extern "C" int rlb_rmsnorm_bwd_noalloc_init();
