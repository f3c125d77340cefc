// Persistent 2-SM tcgen05 GEMM for sm_100a:  C[M, N] = alpha * op(A) op(B)^T  (bf16 in, fp32 accumulate).
//
// This is the GEMM behind every dense linear layer of the models (the reference runs them through
// F.linear: src/forgeline/models/transformer/feedforward.py:26, src/forgeline/models/attention/causal.py:81-83).
//
// Operand layouts (template flags, as in gemm_tcgen05.cu):
//   A_MN = 0: A stored [M][K] (K contiguous)      A_MN = 1: A stored [K][M] (M contiguous)
//   B_MN = 0: B stored [N][K] (K contiguous)      B_MN = 1: B stored [K][N] (N contiguous)
// covering a linear layer's forward (x W^T: 0/0), input gradient (dy W: 0/1) and weight gradient
// (dy^T x: 1/1) without transposes.
//
// Work unit: one 256 x (256 NSUB) tile of C per CTA pair (a 2-CTA cluster on one TPC).  Each CTA loads its
// own 128 rows of A and, for each of the NSUB 256-column sub-tiles, its own 128 rows of B (N) for a 64-deep
// K slice into its shared memory with plain TMA loads (no cluster-wide delivery).  The even CTA's elected
// thread issues tcgen05.mma.cta_group::2 with M = 256, N = 256, K = 16, which reads both CTAs' halves and
// writes 128 accumulator rows into each CTA's TMEM.  With NSUB = 2 one A slice feeds two MMAs (a 256 x 512
// tile), which cuts the operand bytes per FLOP by a quarter against 256 x 256 tiles; the accumulator then
// fills all 512 TMEM columns, so instead of double-buffering it the epilogue reads it out into registers
// and hands it back before converting and storing.
//
// Roles (one CTA per SM, persistent over tiles):
//   warp 0        TMA producer (both CTAs): a ring of 32 / 48 KB stages.  Completion of a stage is
//                 counted on the even CTA's `full` barrier (the even CTA arms it with both CTAs' bytes).
//   warp 1        TMEM owner (512 columns, allocated as a pair); in the even CTA one elected thread issues
//                 the MMAs and commits stage releases and finished accumulators to the barriers of both CTAs.
//   warps 2..     epilogue (both CTAs), 4 NSUB warps: warp w reads TMEM lane quarter w % 4 of one 256-column
//                 sub-tile.  bf16 output: tcgen05.ld all 256 columns, scale by alpha, pack to bf16 in
//                 registers, hand the accumulator back (to the even CTA's `tempty` barrier), then write
//                 128-B swizzled 32-row staging tiles and TMA-store them.  fp32 output: chunk by chunk
//                 through the staging tile, stored or accumulated into C with a TMA reduce-add.
// Every mbarrier wait is bounded; on timeout the kernel records an error in `status`, tells the peer
// CTA to stop, drains its own MMAs and stores, frees TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#include "sm100.cuh"
#include "tmap.h"

namespace gemm2 {

constexpr int BM = 256, SUBN = 256;  // C rows per CTA pair; columns per MMA / per accumulator sub-tile
constexpr int HM = 128, HN = 128;    // rows of A / of B (per sub-tile) each CTA holds
constexpr int BK = 64, UMMA_K = 16;
constexpr int A_BYTES = HM * BK * 2, B_SUB_BYTES = HN * BK * 2;
constexpr int EPI_TILE = 32 * 128;  // one warp's staging tile: 32 rows x 128 B
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 8;
constexpr uint32_t WAIT_LIMIT = 1u << 26;  // polls before a wait is declared dead (seconds)
constexpr int BAR_BYTES = 256;

// Per-NSUB configuration: tile width, ring depth, accumulator buffers, epilogue warps, shared memory.
template <int NSUB>
struct Cfg {
  static constexpr int BN = SUBN * NSUB;
  static constexpr int B_BYTES = B_SUB_BYTES * NSUB;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = NSUB == 1 ? 6 : 4;
  static constexpr int ACCS = NSUB == 1 ? 2 : 1;  // accumulator buffers (each BN TMEM columns)
  static constexpr int EPI_WARPS = 4 * NSUB;
  static constexpr int EPI_BUFS = NSUB == 1 ? 2 : 1;  // staging tiles per epilogue warp
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BUFS * EPI_TILE;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES + 1024;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget of one sm_100a CTA");
  static_assert(ACCS * BN <= TMEM_COLS, "accumulators fit in TMEM");
};

// kSwiGLU: forward of a gated FFN's fused [gate | up] projection (B = [W1; W3], N = the hidden width H).  A
// tile holds the gate and up columns of the same 256 hidden units (its two 256-column sub-tiles read W1 rows
// h.. and W3 rows H + h..); the epilogue stores both into h13 (kept for the backward) and silu(gate) * up,
// computed from their bf16 values as the standalone activation kernel does, into the activation output.
// kLogitsLSE: LM-head forward.  Stores the bf16 logits as kStoreBF16 does and, per row and per 256-column
// half tile, the running statistics of its bf16 values -- max m, sum exp(x - m) and sum exp(x - m) * x -- into
// `lse_stats` ([M][2 * tiles_n] float4), from which one small pass gets each row's log-sum-exp, target
// log-prob and entropy without reading the logits again.
// kRope64 / kRope128: attention input projection x [W_q; W_k; W_v]^T with rotary embedding applied in the
// epilogue (head dim 64 / 128, rotate-half pairs (i, i + D/2) of each q and k head by pos * inv_freq[i], from the
// bf16 values as the standalone RoPE kernel does) and the q / k / v column ranges stored into three token-major
// tensors (maps c, c2, c3).  A position outside the cos / sin table is reported in `rope_err` and that row
// is left unrotated.
// kSwiGLUBwd: input gradient of a gated FFN's down projection, dh = dy W2 (A = dy K-major, B = W2 [K][H] read
// MN-major), rounded to bf16 as a stored dh would be, and in the epilogue the SwiGLU backward against the
// forward's h13 [M][2H]: d gate = dh * up * s * (1 + gate * (1 - s)), d up = dh * gate * s (s = sigmoid(gate)),
// stored into dh13's two halves (maps c, c2).  dh itself is never written.
enum Epi : int { kStoreBF16 = 0, kStoreF32 = 1, kAccumF32 = 2, kSwiGLU = 3, kLogitsLSE = 4, kRope64 = 5, kRope128 = 6,
                 kSwiGLUBwd = 7 };

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

struct Params {
  int M, N, K;
  int splits;   // K ranges per tile (> 1 only with kAccumF32: each range reduce-adds its partial product)
  int group_m;  // M tiles per raster group (consecutive work units walk M inside a group, then N)
  float alpha;
  int* status;
  float* c32;     // kAccumF32: C itself, for the ragged edge chunks the threads accumulate directly
  long long ldc;
  float4* lse_stats;  // kLogitsLSE: [M][2 * ceil(N / 512)] per-half-tile row statistics
  // kRope64 / kRope128
  const float* rope_cos;  // [table_rows][D / 2]
  const float* rope_sin;
  const int* rope_pos;    // [M] positions, or null: (row % seq_T) + pos_offset
  int seq_T, pos_offset, table_rows, q_cols, kv_cols;
  int* rope_err;
  const __nv_bfloat16* h13;  // kSwiGLUBwd: the forward's [gate | up] projection, row pitch ldh
  long long ldh;
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int group_m, int& m, int& n) {
  const int per_group = group_m * num_n;
  const int g = t / per_group;
  const int first_m = g * group_m;
  const int gsize = min(num_m - first_m, group_m);
  const int r = t % per_group;
  m = first_m + r % gsize;
  n = r / gsize;
}

struct Ctl {
  volatile int* abort_flag;  // this CTA's stop flag
  uint32_t peer_abort;       // the peer CTA's stop flag (shared::cluster address)
  int* status;
};

__device__ __forceinline__ void fail(const Ctl& c, int where) {
  *c.abort_flag = 1;
  sm100::st_cluster_u32(c.peer_abort, 1u);
  if (c.status) atomicCAS(c.status, 0, 1 | (where << 8));
}

__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity) {
  return sm100::mbar_wait_bounded(bar, parity, WAIT_LIMIT);
}

// fp32 pair -> packed bf16x2
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int A_MN, int B_MN, int EPI, int NSUB>
__global__ void __launch_bounds__(Cfg<NSUB>::THREADS, 1) gemm2sm_kernel(const __grid_constant__ CUtensorMap tma_a,
                                                                        const __grid_constant__ CUtensorMap tma_b,
                                                                        const __grid_constant__ CUtensorMap tma_c,
                                                                        const __grid_constant__ CUtensorMap tma_c2,
                                                                        const __grid_constant__ CUtensorMap tma_c3,
                                                                        Params p) {
  using C = Cfg<NSUB>;
  constexpr int BN = C::BN, STAGES = C::STAGES, ACCS = C::ACCS;
  extern __shared__ uint8_t smem_raw[];
  // identical offsets in both CTAs: the pair MMA addresses the peer's operands at this CTA's offsets
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sE = smem + STAGES * C::STAGE_BYTES;
  uint64_t* full = (uint64_t*)(sE + C::EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = (uint32_t*)(drain + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const uint32_t rank = sm100::cluster_ctarank();  // 0: the CTA that issues the pair MMAs
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  static_assert(EPI != kSwiGLU || (NSUB == 2 && A_MN == 0 && B_MN == 0), "SwiGLU epilogue: forward, 256 x 512");
  static_assert(EPI != kLogitsLSE || (NSUB == 2 && A_MN == 0 && B_MN == 0), "LSE epilogue: forward, 256 x 512");
  constexpr bool ROPE = EPI == kRope64 || EPI == kRope128;
  static_assert(!ROPE || (NSUB == 2 && A_MN == 0 && B_MN == 0), "RoPE epilogue: forward, 256 x 512");
  static_assert(EPI != kSwiGLUBwd || (NSUB == 2 && A_MN == 0 && B_MN == 1), "SwiGLU backward: dy W, 256 x 512");
  constexpr int TN = EPI == kSwiGLU ? SUBN : BN;  // output columns (hidden units for kSwiGLU) per tile
  const int num_m = (p.M + BM - 1) / BM, num_n = (p.N + TN - 1) / TN;
  const int num_tiles = num_m * num_n;
  const int nk = (p.K + BK - 1) / BK;
  // work unit u: tile u % num_tiles, K blocks [kb_lo, kb_hi) of split u / num_tiles (split-major, so the
  // units in flight together share their K range and its operand slices in L2)
  const int num_units = num_tiles * p.splits;
  auto k_range = [&](int u, int& lo, int& hi) {
    const int sp = u / num_tiles;
    lo = (int)((long long)sp * nk / p.splits);
    hi = (int)((long long)(sp + 1) * nk / p.splits);
  };
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const Ctl ctl{abort_flag, sm100::mapa(sm100::smem_u32((const void*)abort_flag), rank ^ 1u), p.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&tfull[b], 1);
      sm100::mbar_init(&tempty[b], 2 * C::EPI_WARPS);  // every epilogue warp of both CTAs
    }
    sm100::mbar_init(drain, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tensormap(&tma_a);
    sm100::prefetch_tensormap(&tma_b);
    sm100::prefetch_tensormap(&tma_c);
    if (EPI == kSwiGLU || EPI == kRope64 || EPI == kRope128 || EPI == kSwiGLUBwd) {
      sm100::prefetch_tensormap(&tma_c2);
      sm100::prefetch_tensormap(&tma_c3);
    }
  }
  if (warp == 1) {
    sm100::tmem_alloc_pair(tmem_slot, TMEM_COLS);
    sm100::tmem_relinquish_pair();
  }
  sm100::tc_fence_before();
  sm100::cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA traffic
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint32_t full0 = sm100::mapa(sm100::smem_u32(full), 0);
      for (int u = cluster; u < num_units && !*abort_flag; u += nclusters) {
        int tm, tn, kb_lo, kb_hi;
        tile_coords(u % num_tiles, num_m, num_n, p.group_m, tm, tn);
        k_range(u, kb_lo, kb_hi);
        const int m0 = tm * BM + (int)rank * HM;  // this CTA's rows of A
        const int nb = tn * TN + (int)rank * HN;  // ... and of B in the first sub-tile
        bool dead = false;
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!wait(&empty[stage], phase ^ 1)) {
            fail(ctl, 1);
            dead = true;
            break;
          }
          const int k0 = kb * BK;
          if (!RLB_TMA_X_OK(A_MN ? m0 : k0) || !RLB_TMA_X_OK(B_MN ? nb : k0)) {
            fail(ctl, 7);
            dead = true;
            break;
          }
          if (rank == 0) sm100::mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
          const uint32_t fb = full0 + (uint32_t)stage * 8u;
          uint8_t* a = sA + stage * A_BYTES;
          uint8_t* b = sB + stage * C::B_BYTES;
          if (A_MN) {
#pragma unroll
            for (int h = 0; h < HM / 64; ++h) sm100::tma_load_2d_pair(a + h * (BK * 128), &tma_a, fb, m0 + 64 * h, k0);
          } else {
            sm100::tma_load_2d_pair(a, &tma_a, fb, k0, m0);
          }
#pragma unroll
          for (int j = 0; j < NSUB; ++j) {
            uint8_t* bj = b + j * B_SUB_BYTES;
            const int n0 = nb + j * (EPI == kSwiGLU ? p.N : SUBN);  // kSwiGLU: sub-tile 1 reads W3's rows
            if (B_MN) {
#pragma unroll
              for (int h = 0; h < HN / 64; ++h) sm100::tma_load_2d_pair(bj + h * (BK * 128), &tma_b, fb, n0 + 64 * h, k0);
            } else {
              sm100::tma_load_2d_pair(bj, &tma_b, fb, k0, n0);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (dead) break;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (even CTA)
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = sm100::idesc_bf16_f32(BM, SUBN, A_MN, B_MN);
      const uint32_t empty0 = sm100::mapa(sm100::smem_u32(empty), 0), empty1 = sm100::mapa(sm100::smem_u32(empty), 1);
      const uint32_t tfull0 = sm100::mapa(sm100::smem_u32(tfull), 0), tfull1 = sm100::mapa(sm100::smem_u32(tfull), 1);
      // MMAs of one 64-deep K slice (stage `st`, K block `kb` counted from the unit's first) into sub-tile j
      auto issue = [&](uint32_t d, int st, int kb, int j) {
        const uint32_t a = sm100::smem_u32(sA + st * A_BYTES);
        const uint32_t bj = sm100::smem_u32(sB + st * C::B_BYTES) + j * B_SUB_BYTES;
#pragma unroll
        for (int k = 0; k < BK / UMMA_K; ++k) {
          // K-major: +32 B per 16-element K step inside the 128-B swizzle row.
          // MN-major: a 16-element K step spans two 8-row (1024-B) atoms; 64-wide M / N blocks 8 KB apart.
          const uint64_t ad = A_MN ? sm100::desc_mnmajor_sw128(a + k * 2048, BK * 128)
                                   : sm100::desc_kmajor_sw128(a + k * 32);
          const uint64_t bd = B_MN ? sm100::desc_mnmajor_sw128(bj + k * 2048, BK * 128)
                                   : sm100::desc_kmajor_sw128(bj + k * 32);
          sm100::mma_f16_pair(d + j * SUBN, ad, bd, idesc, (kb | k) != 0);
        }
      };
      // the stage may be refilled in both CTAs once the MMAs issued so far have read it
      auto release = [&](int st) {
        sm100::mma_commit_pair(empty0 + (uint32_t)st * 8u);
        sm100::mma_commit_pair(empty1 + (uint32_t)st * 8u);
      };
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int u = cluster; u < num_units && !*abort_flag; u += nclusters) {
        int kb_lo, kb_hi;
        k_range(u, kb_lo, kb_hi);
        // NSUB == 2: one accumulator of two sub-tiles whose columns the epilogue hands back one after the
        // other (tempty[0], tempty[1]).  The sub-tile 0 MMAs of this tile start as soon as sub-tile 0 is
        // free; K slices whose sub-tile 1 MMAs must wait stay pending (their stages unreleased), at most a
        // ring's worth, and are caught up in order once sub-tile 1 is free.
        if (!wait(&tempty[acc], acc_phase ^ 1)) {
          fail(ctl, 2);
          break;
        }
        sm100::tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        bool sub1_free = NSUB == 1;
        int pend = 0, pend_kb = 0, pend_st = 0;  // pending K slices: count, first K block, its stage
        bool dead = false;
        auto catch_up = [&]() {
          for (int i = 0; i < pend; ++i) {
            const int st = (pend_st + i) % STAGES;
            issue(d, st, pend_kb + i - kb_lo, 1);
            release(st);
          }
          pend = 0;
        };
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!wait(&full[stage], phase)) {
            fail(ctl, 3);
            dead = true;
            break;
          }
          sm100::tc_fence_after();
          issue(d, stage, kb - kb_lo, 0);
          if constexpr (NSUB == 2) {
            if (!sub1_free) {
              bool now_free = sm100::mbar_test_wait(&tempty[1], acc_phase ^ 1);
              if (!now_free && pend + 1 == STAGES) {  // every stage is held: sub-tile 1 must be free first
                if (!wait(&tempty[1], acc_phase ^ 1)) {
                  fail(ctl, 5);
                  dead = true;
                  break;
                }
                now_free = true;
              }
              if (now_free) {
                sm100::tc_fence_after();  // sub-tile 1's MMAs after the epilogue's reads of its columns
                sub1_free = true;
              }
            }
            if (!sub1_free) {
              if (pend == 0) {
                pend_kb = kb;
                pend_st = stage;
              }
              ++pend;
            } else {
              catch_up();
              issue(d, stage, kb - kb_lo, 1);
              release(stage);
            }
          } else {
            release(stage);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!dead && pend) {  // fewer K slices than stages: finish sub-tile 1 once it is free
          if (!wait(&tempty[1], acc_phase ^ 1)) {
            fail(ctl, 5);
            dead = true;
          } else {
            sm100::tc_fence_after();
            catch_up();
          }
        }
        if (dead) break;
        sm100::mma_commit_pair(tfull0 + (uint32_t)acc * 8u);
        sm100::mma_commit_pair(tfull1 + (uint32_t)acc * 8u);
        if (++acc == ACCS) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // every MMA issued here completes before either CTA frees TMEM or shared memory
      sm100::mma_commit_pair(sm100::mapa(sm100::smem_u32(drain), 0));
      wait(drain, 0);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2.., both CTAs)
    const int ew = warp - 2;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    // NSUB == 1: warp ew converts the accumulator's 256 columns of its lane quarter.  NSUB == 2: the two warps
    // of a lane quarter split each sub-tile's columns in halves (`half`), both draining sub-tile 0 first.
    const int half = ew >> 2;
    uint8_t* stage_tiles = sE + ew * C::EPI_BUFS * EPI_TILE;
    const uint32_t tempty0 = sm100::mapa(sm100::smem_u32(tempty), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    int ebuf = 0;
    for (int u = cluster; u < num_units; u += nclusters) {
      if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
      int tm, tn;
      tile_coords(u % num_tiles, num_m, num_n, p.group_m, tm, tn);
      const int row0 = tm * BM + (int)rank * HM + q * 32;  // first C row of this warp's 32 rows
      if (!__all_sync(0xffffffffu, wait(&tfull[acc], acc_phase))) {
        if (lane == 0) fail(ctl, 4);
        break;
      }
      sm100::tc_fence_after();
      const uint32_t lanes = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      if constexpr ((EPI == kStoreBF16 || EPI == kSwiGLU || EPI == kLogitsLSE || ROPE || EPI == kSwiGLUBwd) &&
                    NSUB == 2) {
        // read this warp's 128 columns of sub-tile 0, hand sub-tile 0 back (the next tile's first MMAs may
        // start), then its 128 columns of sub-tile 1 and hand those back; all kept as packed bf16 in registers
        uint32_t pk[2][64];
#pragma unroll
        for (int sb = 0; sb < 2; ++sb) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t r[16];
            sm100::tmem_ld16(lanes + sb * SUBN + half * 128 + c * 16, r);
            sm100::tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 8; ++e)
              pk[sb][c * 8 + e] =
                  pack_bf16(__uint_as_float(r[2 * e]) * p.alpha, __uint_as_float(r[2 * e + 1]) * p.alpha);
          }
          sm100::tc_fence_before();
          __syncwarp();
          if (lane == 0) sm100::mbar_arrive_cluster(tempty0 + (uint32_t)sb * 8u);
        }
        if constexpr (EPI == kLogitsLSE) {
          // statistics of this row's 256 columns of the tile (128 per sub-tile), from the stored bf16 values:
          // one pass, folding 16 values at a time into the running max / sums with one rescale per group
          float m = -INFINITY, se = 0.f, te = 0.f;
#pragma unroll
          for (int sb = 0; sb < 2; ++sb) {
#pragma unroll
            for (int g8 = 0; g8 < 8; ++g8) {
              const int col = tn * BN + sb * SUBN + half * 128 + g8 * 16;  // first column of the group
              float x[16];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const uint32_t w = pk[sb][g8 * 8 + e];
                x[2 * e] = col + 2 * e < p.N ? __uint_as_float(w << 16) : -INFINITY;
                x[2 * e + 1] = col + 2 * e + 1 < p.N ? __uint_as_float(w & 0xffff0000u) : -INFINITY;
              }
              float gm = x[0];
#pragma unroll
              for (int e = 1; e < 16; ++e) gm = fmaxf(gm, x[e]);
              if (gm != -INFINITY) {
                const float mn = fmaxf(m, gm);
                const float f = __expf(m - mn);  // 0 while m is -inf
                se *= f;
                te *= f;
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                  const float ex = __expf(x[e] - mn);  // 0 for masked columns
                  se += ex;
                  te += x[e] == -INFINITY ? 0.f : ex * x[e];
                }
                m = mn;
              }
            }
          }
          const int row = row0 + lane;
          if (row < p.M) p.lse_stats[(long long)row * (2 * num_n) + 2 * tn + half] = make_float4(m, se, te, 0.f);
        }
        if constexpr (ROPE) {
          constexpr int D = EPI == kRope64 ? 64 : 128;
          constexpr int QW = D / 4;  // packed words (column pairs) in half a head
          const int row = row0 + lane;
          int pos = -1;
          if (row < p.M) {
            pos = p.rope_pos ? p.rope_pos[row] : row % p.seq_T + p.pos_offset;
            if (pos < 0 || pos >= p.table_rows) {
              if (p.rope_err) atomicCAS(p.rope_err, 0, 2);  // index error word: bad index
              pos = -1;
            }
          }
#pragma unroll
          for (int sb = 0; sb < 2; ++sb) {
            const int cb = tn * BN + sb * SUBN + half * 128;  // first column of this thread's 128 (whole heads)
            if (pos >= 0 && cb < p.q_cols + p.kv_cols) {    // q and k heads rotate, v passes through
              const float2* cs = reinterpret_cast<const float2*>(p.rope_cos + (long long)pos * (D / 2));
              const float2* sn = reinterpret_cast<const float2*>(p.rope_sin + (long long)pos * (D / 2));
#pragma unroll
              for (int hh = 0; hh < 128 / D; ++hh) {
#pragma unroll
                for (int i = 0; i < QW; ++i) {
                  const int w1 = hh * (D / 2) + i, w2 = w1 + QW;  // columns (2i, 2i+1) and their partners + D/2
                  const float2 c2 = __ldg(cs + i), s2 = __ldg(sn + i);
                  const float a0 = __uint_as_float(pk[sb][w1] << 16), a1 = __uint_as_float(pk[sb][w1] & 0xffff0000u);
                  const float b0 = __uint_as_float(pk[sb][w2] << 16), b1 = __uint_as_float(pk[sb][w2] & 0xffff0000u);
                  pk[sb][w1] = pack_bf16(a0 * c2.x - b0 * s2.x, a1 * c2.y - b1 * s2.y);
                  pk[sb][w2] = pack_bf16(b0 * c2.x + a0 * s2.x, b1 * c2.y + a1 * s2.y);
                }
              }
            }
          }
        }
        if constexpr (EPI == kSwiGLUBwd) {
          // pk holds dh; gate and up of this thread's row come from h13, 8 columns (16 B) at a time
          const int row = row0 + lane;
          const bool row_ok = row < p.M;
          const __nv_bfloat16* hrow = p.h13 + (long long)(row_ok ? row : 0) * p.ldh;
          // (sub-tile, chunk) outermost so each chunk's dh registers die after its two stores
#pragma unroll
          for (int sb = 0; sb < 2; ++sb) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const int col0 = tn * BN + sb * SUBN + half * 128 + c * 64;
#pragma unroll
              for (int o = 0; o < 2; ++o) {  // 0: d gate -> dh13[:, :H] (map c); 1: d up -> dh13[:, H:] (map c2)
                uint8_t* tile = stage_tiles;
                if (lane == 0) sm100::bulk_wait_read<0>();  // the staging tile's previous store has read it
                __syncwarp();
                uint8_t* rowp = tile + lane * 128;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  uint4 gv = make_uint4(0u, 0u, 0u, 0u), uv = make_uint4(0u, 0u, 0u, 0u);
                  if (row_ok && col0 + 8 * j < p.N) {
                    gv = __ldg(reinterpret_cast<const uint4*>(hrow + col0 + 8 * j));
                    if (o == 0) uv = __ldg(reinterpret_cast<const uint4*>(hrow + p.N + col0 + 8 * j));
                  }
                  uint32_t w[4];
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const uint32_t gw = e == 0 ? gv.x : (e == 1 ? gv.y : (e == 2 ? gv.z : gv.w));
                    const uint32_t uw = e == 0 ? uv.x : (e == 1 ? uv.y : (e == 2 ? uv.z : uv.w));
                    const uint32_t dw = pk[sb][c * 32 + 4 * j + e];
                    float r2[2];
#pragma unroll
                    for (int l = 0; l < 2; ++l) {
                      const float g = __uint_as_float(l ? (gw & 0xffff0000u) : (gw << 16));
                      const float u = __uint_as_float(l ? (uw & 0xffff0000u) : (uw << 16));
                      const float d = __uint_as_float(l ? (dw & 0xffff0000u) : (dw << 16));
                      const float sg = 1.f / (1.f + __expf(-g));
                      r2[l] = o == 0 ? d * u * sg * (1.f + g * (1.f - sg)) : d * g * sg;
                    }
                    w[e] = pack_bf16(r2[0], r2[1]);
                  }
                  *reinterpret_cast<uint4*>(rowp + ((j ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
                }
                sm100::fence_async_shared();
                __syncwarp();
                if (lane == 0 && row0 < p.M && col0 < p.N) {
                  sm100::tma_store_2d(o == 0 ? &tma_c : &tma_c2, tile, col0, row0);  // clipped at M and H
                  sm100::bulk_commit();
                }
              }
            }
          }
        } else {
        // kSwiGLU: out 0 / 1 are the gate / up halves of h13 (maps c, c2), out 2 the activation (map c3)
        constexpr int NOUT = EPI == kSwiGLU ? 3 : 2;
#pragma unroll
        for (int o = 0; o < NOUT; ++o) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int col0 = (EPI == kSwiGLU ? tn * SUBN : tn * BN + o * SUBN) + half * 128 + c * 64;
            uint8_t* tile = stage_tiles;
            if (lane == 0) sm100::bulk_wait_read<0>();  // the staging tile's previous store has read it
            __syncwarp();
            // row `lane`: 8 chunks of 16 B; chunk j stored at j ^ (row % 8) (the TMA 128-B swizzle)
            uint8_t* rowp = tile + lane * 128;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int i = c * 32 + 4 * j + e;
                if (o < 2) {
                  w[e] = pk[o][i];
                } else {  // silu(gate) * up from the bf16 pair values (bf16 -> fp32 is a 16-bit shift), rounded once
                  const uint32_t g2 = pk[0][i], u2 = pk[1][i];
                  w[e] = pack_bf16(silu(__uint_as_float(g2 << 16)) * __uint_as_float(u2 << 16),
                                   silu(__uint_as_float(g2 & 0xffff0000u)) * __uint_as_float(u2 & 0xffff0000u));
                }
              }
              *reinterpret_cast<uint4*>(rowp + ((j ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
            sm100::fence_async_shared();  // generic-proxy writes visible to the TMA engine
            __syncwarp();
            if (lane == 0 && row0 < p.M && col0 < p.N) {
              const CUtensorMap* map = o == 0 ? &tma_c : (o == 1 ? &tma_c2 : &tma_c3);
              int col = col0;
              if (ROPE) {  // q | k | v column ranges go to their own tensors
                map = &tma_c;
                if (col0 >= p.q_cols + p.kv_cols) {
                  map = &tma_c3;
                  col = col0 - p.q_cols - p.kv_cols;
                } else if (col0 >= p.q_cols) {
                  map = &tma_c2;
                  col = col0 - p.q_cols;
                }
              }
              sm100::tma_store_2d((EPI == kSwiGLU || ROPE) ? map : &tma_c, tile, col, row0);  // clipped at M and N
              sm100::bulk_commit();
            }
          }
        }
        }  // kSwiGLUBwd / other stores
      } else {
        // chunk by chunk through the staging tile (64 bf16 or 32 fp32 columns per 128-B row), the accumulator
        // released after the last read (double-buffered accumulators hide this, or fp32 output).  Warp ew
        // converts sub-tile `half` (NSUB == 2) and hands back both barriers' worth at its last read.
        constexpr int COLS = EPI == kStoreBF16 ? 64 : 32;
        const int n0 = tn * BN + half * SUBN;
        const uint32_t tbase = lanes + half * SUBN;
#pragma unroll 1
        for (int c = 0; c < SUBN / COLS; ++c) {
          uint32_t r[COLS];
          sm100::tmem_ld32(tbase + c * COLS, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
          if constexpr (COLS == 64) sm100::tmem_ld32(tbase + c * COLS + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
          sm100::tmem_ld_wait();
          if (c == SUBN / COLS - 1) {
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if (NSUB == 2) {  // both sub-tile barriers count every epilogue warp
                sm100::mbar_arrive_cluster(tempty0);
                sm100::mbar_arrive_cluster(tempty0 + 8u);
              } else {
                sm100::mbar_arrive_cluster(tempty0 + (uint32_t)acc * 8u);
              }
            }
          }
          const int col0 = n0 + c * COLS;
          if (EPI == kAccumF32 && (row0 + 32 > p.M || col0 + 32 > p.N)) {
            // A reduce-add box that runs past C's edge lost updates on B200 (tested: columns past the inner
            // extent), so a clipped chunk is accumulated by the threads: row `lane`, its columns below N.
            // Atomically: with split K, other units add their partial sums to the same elements.
            const int row = row0 + lane;
            if (row < p.M) {
              float* dst = p.c32 + (long long)row * p.ldc + col0;
#pragma unroll
              for (int e = 0; e < 32; ++e)
                if (col0 + e < p.N) atomicAdd(dst + e, __uint_as_float(r[e]) * p.alpha);
            }
            continue;
          }
          uint8_t* tile = stage_tiles + ebuf * EPI_TILE;
          if (lane == 0) {
            if (C::EPI_BUFS == 2) sm100::bulk_wait_read<1>();
            else sm100::bulk_wait_read<0>();
          }
          __syncwarp();
          uint8_t* rowp = tile + lane * 128;  // chunk j of row `lane` stored at j ^ (row % 8)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 v;
            if constexpr (COLS == 64) {
              v = make_uint4(pack_bf16(__uint_as_float(r[8 * j + 0]) * p.alpha, __uint_as_float(r[8 * j + 1]) * p.alpha),
                             pack_bf16(__uint_as_float(r[8 * j + 2]) * p.alpha, __uint_as_float(r[8 * j + 3]) * p.alpha),
                             pack_bf16(__uint_as_float(r[8 * j + 4]) * p.alpha, __uint_as_float(r[8 * j + 5]) * p.alpha),
                             pack_bf16(__uint_as_float(r[8 * j + 6]) * p.alpha, __uint_as_float(r[8 * j + 7]) * p.alpha));
            } else {
              v = make_uint4(__float_as_uint(__uint_as_float(r[4 * j]) * p.alpha),
                             __float_as_uint(__uint_as_float(r[4 * j + 1]) * p.alpha),
                             __float_as_uint(__uint_as_float(r[4 * j + 2]) * p.alpha),
                             __float_as_uint(__uint_as_float(r[4 * j + 3]) * p.alpha));
            }
            *reinterpret_cast<uint4*>(rowp + ((j ^ (lane & 7)) << 4)) = v;
          }
          sm100::fence_async_shared();
          __syncwarp();
          if (lane == 0 && row0 < p.M && col0 < p.N) {
            if (EPI == kAccumF32) sm100::tma_reduce_add_2d(&tma_c, tile, col0, row0);
            else sm100::tma_store_2d(&tma_c, tile, col0, row0);
            sm100::bulk_commit();
          }
          if (C::EPI_BUFS == 2) ebuf ^= 1;
        }
      }
      if (++acc == ACCS) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) sm100::bulk_wait_all();  // stores complete before the staging memory goes away
  }

  __syncwarp();  // reconverge the single-lane roles before the warp-aligned cluster barrier
  sm100::tc_fence_before();
  sm100::cluster_sync();  // the peer's MMAs into this CTA's TMEM and reads of its shared memory are done
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host
using rlb_tmap::EncodeTiledFn;
using rlb_tmap::encode_fn;

// 2-D tensor map over a row-major matrix [rows][cols] (cols contiguous, leading dimension `ld` elements),
// box {box_cols, box_rows}, 128-B swizzle (box_cols * element size == 128 B).
static bool make_map(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* ptr, long long rows,
                     long long cols, long long ld, int box_cols, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * esize)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    fprintf(stderr, "gemm2: tensor map rejected (CUresult %d): ptr %p rows %lld cols %lld ld %lld esize %d box %dx%d\n",
            (int)r, ptr, rows, cols, ld, esize, box_cols, box_rows);
  return r == CUDA_SUCCESS;
}

// Clusters of this kernel that can be resident at once on device `dev` (cached per instantiation and
// device): the persistent grid must not exceed it, or late clusters would run their tiles after the others.
template <int A_MN, int B_MN, int EPI, int NSUB>
static int max_clusters(int dev) {
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return 0;
  if (cache[dev] > 0) return cache[dev];
  auto kern = gemm2sm_kernel<A_MN, B_MN, EPI, NSUB>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(Cfg<NSUB>::THREADS, 1, 1);
  cfg.dynamicSmemBytes = Cfg<NSUB>::SMEM_BYTES;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, (void*)kern, &cfg) != cudaSuccess || n <= 0) {
    (void)cudaGetLastError();
    return 0;
  }
  cache[dev] = n;
  return n;
}

template <int A_MN, int B_MN, int EPI, int NSUB>
static cudaError_t launch(const void* A, long long lda, const void* B, long long ldb, void* Cp, long long ldc,
                          const Params& p, int max_ctas, cudaStream_t s, void* act = nullptr) {
  using C = Cfg<NSUB>;
  CUtensorMap ma, mb, mc;
  const CUtensorMapDataType bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  // K-major operand: [rows][K], box 64 k x 128 rows.  MN-major: [K][rows], box 64 rows x 64 k.
  const bool ok_a = A_MN ? make_map(&ma, bf, 2, A, p.K, p.M, lda, 64, BK) : make_map(&ma, bf, 2, A, p.M, p.K, lda, 64, HM);
  const long long b_rows = EPI == kSwiGLU ? 2LL * p.N : p.N;  // kSwiGLU: B = [W1; W3]
  const bool ok_b = B_MN ? make_map(&mb, bf, 2, B, p.K, p.N, ldb, 64, BK) : make_map(&mb, bf, 2, B, b_rows, p.K, ldb, 64, HN);
  CUtensorMap mc2, mc3;
  bool ok_c;
  if (EPI == kSwiGLUBwd) {  // the two halves of dh13 [M][2H] (row pitch ldc)
    ok_c = make_map(&mc, bf, 2, Cp, p.M, p.N, ldc, 64, 32) &&
           make_map(&mc2, bf, 2, (const __nv_bfloat16*)Cp + p.N, p.M, p.N, ldc, 64, 32);
    mc3 = mc;
  } else if (EPI == kRope64 || EPI == kRope128) {  // q [M][q_cols], k and v [M][kv_cols]; `act` holds {k, v}
    void* const* kv = static_cast<void* const*>(act);
    ok_c = make_map(&mc, bf, 2, Cp, p.M, p.q_cols, p.q_cols, 64, 32) &&
           make_map(&mc2, bf, 2, kv[0], p.M, p.kv_cols, p.kv_cols, 64, 32) &&
           make_map(&mc3, bf, 2, kv[1], p.M, p.kv_cols, p.kv_cols, 64, 32);
  } else if (EPI == kSwiGLU) {  // gate / up halves of h13 [M][2H] (row pitch ldc) and the activation [M][H]
    ok_c = make_map(&mc, bf, 2, Cp, p.M, p.N, ldc, 64, 32) &&
           make_map(&mc2, bf, 2, (const __nv_bfloat16*)Cp + p.N, p.M, p.N, ldc, 64, 32) &&
           make_map(&mc3, bf, 2, act, p.M, p.N, p.N, 64, 32);
  } else {
    ok_c = (EPI == kStoreBF16 || EPI == kLogitsLSE) ? make_map(&mc, bf, 2, Cp, p.M, p.N, ldc, 64, 32)
                             : make_map(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, Cp, p.M, p.N, ldc, 32, 32);
    mc2 = mc;
    mc3 = mc;
  }
  if (!ok_a || !ok_b || !ok_c) return cudaErrorInvalidResourceHandle;  // tensor-map encoding rejected an operand
  auto kern = gemm2sm_kernel<A_MN, B_MN, EPI, NSUB>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int clusters = max_clusters<A_MN, B_MN, EPI, NSUB>(dev);
  if (clusters <= 0) return cudaErrorNotSupported;
  if (max_ctas > 0 && clusters > max_ctas / 2) clusters = max_ctas / 2 > 0 ? max_ctas / 2 : 1;
  const int tile_n = EPI == kSwiGLU ? SUBN : C::BN;
  const int units = ((p.M + BM - 1) / BM) * ((p.N + tile_n - 1) / tile_n) * p.splits;
  if (clusters > units) clusters = units;
  (void)cudaGetLastError();  // drop a stale, non-sticky error left by unrelated calls on this thread
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  cfg.blockDim = dim3(C::THREADS, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, mc2, mc3, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace gemm2

// C = alpha * op(A) op(B)^T on the 2-SM kernel.  a_mn / b_mn select the operand storage (see top of file);
// epi: 0 = store bf16, 1 = store fp32, 2 = accumulate into fp32.  nsub: 1 = 256 x 256 tiles (double-buffered
// accumulators), 2 = 256 x 512 tiles (one A slice per two MMAs).  Leading dimensions must be multiples of 8
// elements (C: 16 bytes), base pointers 16-byte aligned.  max_ctas > 0 caps the grid (CTAs, even).
// splits > 1 divides each tile's K blocks into that many ranges, each its own work unit that reduce-adds its
// partial product into C (epi 2 only; C must hold the starting value, e.g. zeros): for products with few
// output tiles and a long K (weight gradients of narrow layers), where whole tiles would leave most of the
// last wave of CTA pairs idle.  group_m: M tiles per raster group (0: the default of 8).
cudaError_t rlb_gemm2sm(int a_mn, int b_mn, int epi, int nsub, int M, int N, int K, const void* A, long long lda,
                        const void* B, long long ldb, void* C, long long ldc, float alpha, int* status, int max_ctas,
                        cudaStream_t s, int splits, int group_m) {
  using namespace gemm2;
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  const int nk = (K + BK - 1) / BK;
  if (splits < 1 || splits > nk || (splits > 1 && epi != kAccumF32)) return cudaErrorInvalidValue;
  if (group_m < 1) group_m = GROUP_M;
  if ((lda % 8) || (ldb % 8) || ((ldc * (epi == kStoreBF16 ? 2 : 4)) % 16)) return cudaErrorInvalidPitchValue;
  if ((((uintptr_t)A) | ((uintptr_t)B) | ((uintptr_t)C)) & 15) return cudaErrorInvalidDevicePointer;
  if (nsub != 1 && nsub != 2) return cudaErrorInvalidValue;
  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.splits = splits;
  p.group_m = group_m;
  p.alpha = alpha;
  p.status = status;
  p.c32 = (float*)C;
  p.ldc = ldc;
#define RLB_GEMM2_CASE(AM, BMN, E)                                                                         \
  if (a_mn == AM && b_mn == BMN && epi == E)                                                               \
    return nsub == 1 ? launch<AM, BMN, E, 1>(A, lda, B, ldb, C, ldc, p, max_ctas, s)                       \
                     : launch<AM, BMN, E, 2>(A, lda, B, ldb, C, ldc, p, max_ctas, s);
  RLB_GEMM2_CASE(0, 0, 0)
  RLB_GEMM2_CASE(0, 1, 0)
  RLB_GEMM2_CASE(1, 1, 0)
  RLB_GEMM2_CASE(1, 1, 1)
  RLB_GEMM2_CASE(1, 1, 2)
  RLB_GEMM2_CASE(0, 0, 1)
  RLB_GEMM2_CASE(0, 0, 2)
#undef RLB_GEMM2_CASE
  return cudaErrorNotSupported;
}

// Forward of a gated FFN's fused projection on the 2-SM kernel with the SwiGLU activation in the epilogue:
// h13 = x [M][K] * w13^T (w13 = [W1; W3], [2H][K], K contiguous) stored [M][2H] (row pitch ldh), and
// act = silu(h13[:, :H]) * h13[:, H:] stored [M][H].  H, K, ldx, ldw and ldh multiples of 8; pointers
// 16-byte aligned.  group_m as for rlb_gemm2sm.
cudaError_t rlb_gemm2sm_swiglu(int M, int H, int K, const void* X, long long ldx, const void* W13, long long ldw,
                               void* H13, long long ldh, void* act, int* status, int max_ctas, cudaStream_t s,
                               int group_m) {
  using namespace gemm2;
  if (M <= 0 || H <= 0 || K <= 0) return cudaSuccess;
  if ((H % 8) || (ldx % 8) || (ldw % 8) || (ldh % 8) || ldh < 2LL * H) return cudaErrorInvalidPitchValue;
  if ((((uintptr_t)X) | ((uintptr_t)W13) | ((uintptr_t)H13) | ((uintptr_t)act)) & 15) return cudaErrorInvalidDevicePointer;
  Params p{};
  p.M = M;
  p.N = H;
  p.K = K;
  p.splits = 1;
  p.group_m = group_m < 1 ? GROUP_M : group_m;
  p.alpha = 1.f;
  p.status = status;
  p.c32 = nullptr;
  p.ldc = ldh;
  return launch<0, 0, kSwiGLU, 2>(X, ldx, W13, ldw, H13, ldh, p, max_ctas, s, act);
}

// LM-head forward on the 2-SM kernel: logits = h [M][K] * W^T (W [N][K]) stored bf16 (row pitch ldc), plus
// per row and per 256-column half tile the statistics (max, sum exp(x - max), sum exp(x - max) * x) of the
// stored bf16 values in stats [M][2 * ceil(N / 512)] (float4, fourth lane unused).
cudaError_t rlb_gemm2sm_lse(int M, int N, int K, const void* A, long long lda, const void* B, long long ldb,
                            void* C, long long ldc, void* stats, int* status, int max_ctas, cudaStream_t s,
                            int group_m) {
  using namespace gemm2;
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  if ((lda % 8) || (ldb % 8) || (ldc % 8)) return cudaErrorInvalidPitchValue;
  if ((((uintptr_t)A) | ((uintptr_t)B) | ((uintptr_t)C) | ((uintptr_t)stats)) & 15) return cudaErrorInvalidDevicePointer;
  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.splits = 1;
  p.group_m = group_m < 1 ? GROUP_M : group_m;
  p.alpha = 1.f;
  p.status = status;
  p.c32 = nullptr;
  p.ldc = ldc;
  p.lse_stats = (float4*)stats;
  return launch<0, 0, kLogitsLSE, 2>(A, lda, B, ldb, C, ldc, p, max_ctas, s);
}

// Attention input projection with rotary embedding in the epilogue: x [M][K] times w = [W_q; W_k; W_v]
// ([(Hq + 2 Hkv) D][K]); q [M][Hq D], k and v [M][Hkv D] (token-major, i.e. [B, T, H, D]) with q and k rotated by
// the cos / sin tables [table_rows][D / 2] at position positions[row] (or row % seq_T + pos_offset).  D is 64 or
// 128; Hq D and Hkv D multiples of 128.
cudaError_t rlb_gemm2sm_rope_qkv(int M, int Hq, int Hkv, int D, int K, const void* X, long long ldx, const void* W,
                                 long long ldw, void* q, void* k, void* v, const float* cos_t, const float* sin_t,
                                 const int* positions, int seq_T, int pos_offset, int table_rows, int* err,
                                 int max_ctas, cudaStream_t s, int group_m) {
  using namespace gemm2;
  if (M <= 0 || K <= 0) return cudaSuccess;
  if ((D != 64 && D != 128) || ((Hq * D) % 128) || ((Hkv * D) % 128) || seq_T <= 0) return cudaErrorInvalidValue;
  if ((ldx % 8) || (ldw % 8)) return cudaErrorInvalidPitchValue;
  if ((((uintptr_t)X) | ((uintptr_t)W) | ((uintptr_t)q) | ((uintptr_t)k) | ((uintptr_t)v)) & 15)
    return cudaErrorInvalidDevicePointer;
  Params p{};
  p.M = M;
  p.N = (Hq + 2 * Hkv) * D;
  p.K = K;
  p.splits = 1;
  p.group_m = group_m < 1 ? GROUP_M : group_m;
  p.alpha = 1.f;
  p.rope_cos = cos_t;
  p.rope_sin = sin_t;
  p.rope_pos = positions;
  p.seq_T = seq_T;
  p.pos_offset = pos_offset;
  p.table_rows = table_rows;
  p.q_cols = Hq * D;
  p.kv_cols = Hkv * D;
  p.rope_err = err;
  void* kv[2] = {k, v};
  return D == 64 ? launch<0, 0, kRope64, 2>(X, ldx, W, ldw, q, p.q_cols, p, max_ctas, s, kv)
                 : launch<0, 0, kRope128, 2>(X, ldx, W, ldw, q, p.q_cols, p, max_ctas, s, kv);
}

// Gated-FFN down projection's input gradient with the SwiGLU backward in the epilogue: dh = dy [M][K] W2 (W2
// stored [K][H], H contiguous), then dh13 [M][2H] = (d gate, d up) against h13 [M][2H] (row pitches ldh, ldd).
cudaError_t rlb_gemm2sm_dgrad_swiglu(int M, int H, int K, const void* dY, long long ldy, const void* W2, long long ldw,
                                     const void* h13, long long ldh, void* dh13, long long ldd, int max_ctas,
                                     cudaStream_t s, int group_m) {
  using namespace gemm2;
  if (M <= 0 || H <= 0 || K <= 0) return cudaSuccess;
  if ((H % 8) || (ldy % 8) || (ldw % 8) || (ldh % 8) || (ldd % 8) || ldh < 2LL * H || ldd < 2LL * H)
    return cudaErrorInvalidPitchValue;
  if ((((uintptr_t)dY) | ((uintptr_t)W2) | ((uintptr_t)h13) | ((uintptr_t)dh13)) & 15) return cudaErrorInvalidDevicePointer;
  Params p{};
  p.M = M;
  p.N = H;
  p.K = K;
  p.splits = 1;
  p.group_m = group_m < 1 ? GROUP_M : group_m;
  p.alpha = 1.f;
  p.ldc = ldd;
  p.h13 = (const __nv_bfloat16*)h13;
  p.ldh = ldh;
  return launch<0, 1, kSwiGLUBwd, 2>(dY, ldy, W2, ldw, dh13, ldd, p, max_ctas, s);
}
