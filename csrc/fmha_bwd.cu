// Fused multi-head attention, backward, for sm_100a (tcgen05 MMAs, TMEM accumulators, TMA loads).
//
// With X = Q K^T, S = f(scale X) (f(x) = x, or cap tanh(x / cap) for a logit soft-cap), P = softmax(S)
// (recomputed from the forward's log-sum-exp), O = P V:
//   dV = P^T dO,   dP = dO V^T,   dS = P * (dP - Delta),   Delta = rowsum(dO * O),
//   dX = scale f'(scale X) dS  (f' = 1 - tanh^2 with the cap, else 1),   dQ = dX K,   dK = dX^T Q.
// Masks as in the forward: causal and a sliding window; query tiles a key tile cannot reach are skipped.
// Same token-major [B, T, H, D] layouts, D = 64 or 128, grouped-query heads and causal mask as the forward
// (csrc/fmha_fwd.cu).  The reference differentiates attention through PyTorch autograd
// (``src/forgeline/models/attention/causal.py:79-134``).
//
// One CTA per (128-key tile, KV head, batch).  K_j and V_j stay in shared memory; the CTA walks every
// query tile that attends to them, for every query head of the KV group, so dK and dV accumulate in
// TMEM over the whole walk and are stored once (no atomics); dQ partials go to an fp32 buffer with
// atomic adds.  Per query tile i (192 threads):
//   warp 0      TMA producer: K_j, V_j once; Q_i and dO_i per step (one stage).
//   warp 1      TMEM owner and MMA issuer:
//                 S^T = K Q_i^T,  dP^T = V dO_i^T          (M = keys, N = queries, K = D; both operands
//                                                          K-major as loaded)
//                 dV += P^T dO_i,  dK += dS^T Q_i          (M = keys, N = D, K = queries; B operand read
//                                                          MN-major from the same Q / dO tiles)
//                 dQ_i = dS K                              (M = queries: the dS^T tile read MN-major)
//   warps 2-5   thread r owns key row r: P^T and dS^T rows from S^T and dP^T (log-sum-exp and Delta of
//               each query read from global memory, the same address for the whole warp), written as
//               bf16 into 128-B-swizzled shared tiles; then the dQ_i rows are added into dq; at the end
//               dK and dV rows are stored as bf16.
// TMEM columns: S^T 0..127, dP^T (then dQ_i) 128..255, dV 256.., dK 256 + D...
// Every mbarrier wait is bounded (timeout -> status word, every role stops, own loads and MMAs are
// waited for, TMEM freed).  No load uses cluster delivery.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include "sm100.cuh"
#include "tmap.h"

namespace fmha_bwd {

constexpr int BQ = 128, BKV = 128;
constexpr int SUB_BYTES = 128 * 64 * 2;
constexpr int TMEM_COLS = 512;
constexpr uint32_t WAIT_LIMIT = 1u << 26;
constexpr float LOG2E = 1.4426950408889634f;

template <int D>
struct Layout {
  static constexpr int DSUB = D / 64;
  // d 64: dQ has its own TMEM columns, Q / dO and P^T / dS^T are double-buffered, and dQ of a step is drained
  // while the next step computes.  d 128: TMEM holds S^T, dP^T, dV, dK only (512 columns), so dQ is computed
  // into S^T's columns and drained within its step, and shared memory takes one stage of each.
  static constexpr bool DQ_SEP = D == 64;
  static constexpr int QST = DQ_SEP ? 2 : 1;
  static constexpr int PST = DQ_SEP ? 2 : 1;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = K_OFF + DSUB * SUB_BYTES;
  static constexpr int Q_OFF = V_OFF + DSUB * SUB_BYTES;       // [QST][DSUB] boxes
  static constexpr int DO_OFF = Q_OFF + QST * DSUB * SUB_BYTES;  // [QST][DSUB]
  static constexpr int PT_OFF = DO_OFF + QST * DSUB * SUB_BYTES;  // P^T  [PST][2]: [128 keys][128 queries] bf16
  static constexpr int DS_OFF = PT_OFF + PST * 2 * SUB_BYTES;    // dS^T [PST][2]
  static constexpr int BAR_OFF = DS_OFF + PST * 2 * SUB_BYTES;
  static constexpr int BYTES = BAR_OFF + 256;
  static constexpr int TDQ = DQ_SEP ? 256 + 2 * D : 0;  // first TMEM column of dQ
  static_assert(BYTES + 1024 <= 232448, "shared memory budget of one sm_100a CTA");
  static_assert(!DQ_SEP || TDQ + D <= TMEM_COLS, "TMEM budget");
};
constexpr int THREADS = 320;  // warps 0-7 compute, 8 TMA producer, 9 TMEM owner + MMA issuer

struct Params {
  const float* lse;    // [B][Hq][T], natural log
  const float* delta;  // [B][Hq][T]
  float* dq;           // [B][T][Hq][D] fp32, accumulated (the caller zeroes it)
  __nv_bfloat16* dk;   // [B][T][Hkv][D]
  __nv_bfloat16* dv;   // [B][T][Hkv][D]
  int B, T, Hq, Hkv;
  float scale, scale_log2;
  int causal;
  int window;      // 0: none; else key s is visible to query t only if t - s < window
  float cap_in;    // soft-cap: scale / cap
  float cap_log2;  // soft-cap: cap * log2(e)
  int* status;
};

__device__ __forceinline__ void fail(int* status, volatile int* abort_flag, int where) {
  *abort_flag = 1;
  if (status) atomicCAS(status, 0, 1 | ((32 + where) << 8));
}

__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity) {
  return sm100::mbar_wait_bounded(bar, parity, WAIT_LIMIT);
}

// The same wait with one answer for the whole warp (the compute warps' TMEM loads are warp-collective,
// so a warp must never split on a wait that ran out for some lanes only).
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, wait(bar, parity));
}

// 4 fp32 values added into global memory with one vector reduction (no return value).
__device__ __forceinline__ void red_add_v4(float* dst, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// One CTA per (128-key tile j, KV head, batch); it walks every (query head of the group, query tile) pair that
// sees the tile ("steps", head-major), accumulating dK and dV in TMEM over the walk.  Per step t:
//   MMA     S^T = K Q_t^T, dP^T = V dO_t^T (keys x queries, K = D); then dV += P^T dO_t, dK += dS^T Q_t
//           (keys x D, K = queries) and dQ_t = dS K (queries x D, K = keys, dS^T read MN-major).
//   compute warps 0-7: warp w owns TMEM lane quarter w % 4 (32 keys) and query columns 64 (w / 4) .. + 64, in
//           32-column chunks: P^T and dS^T from S^T, dP^T, the forward's log-sum-exp and Delta, written bf16 into
//           128-B-swizzled shared tiles; then the rows of dQ (TMEM lane = query) are added into dq.
// With d 64 the next step's S^T / dP^T MMAs are issued as soon as the compute warps have read this step's, and
// dQ of step t is drained during step t + 1.
template <int D, bool CAP>
__global__ void __launch_bounds__(THREADS, 1) fmha_bwd_kernel(const __grid_constant__ CUtensorMap mq,
                                                              const __grid_constant__ CUtensorMap mk,
                                                              const __grid_constant__ CUtensorMap mv,
                                                              const __grid_constant__ CUtensorMap mdo, Params p) {
  using L = Layout<D>;
  constexpr int DSUB = L::DSUB, QST = L::QST, PST = L::PST;
  constexpr bool DQ_SEP = L::DQ_SEP;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sK = smem + L::K_OFF;
  uint8_t* sV = smem + L::V_OFF;
  uint8_t* sQ = smem + L::Q_OFF;
  uint8_t* sDO = smem + L::DO_OFF;
  uint8_t* sPT = smem + L::PT_OFF;
  uint8_t* sDS = smem + L::DS_OFF;
  uint64_t* bars = (uint64_t*)(smem + L::BAR_OFF);
  uint64_t* kvfull = bars;
  uint64_t* qfull = bars + 1;        // [QST]
  uint64_t* qempty = qfull + QST;    // [QST]
  uint64_t* sfull = qempty + QST;    // S^T, dP^T of the step computed
  uint64_t* sfree = sfull + 1;       // ... read by the compute warps (count 8)
  uint64_t* pfull = sfree + 1;       // [PST] P^T, dS^T of the step written (count 8)
  uint64_t* mdone = pfull + PST;     // the step's dV / dK / dQ MMAs done
  uint64_t* dqfree = mdone + 1;      // the step's dQ drained (count 8)
  uint64_t* done = dqfree + 1;       // every MMA done
  uint32_t* tmem_slot = (uint32_t*)(done + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = p.Hq / p.Hkv;
  const int kv0 = j * BKV;
  const int num_qt = (p.T + BQ - 1) / BQ;
  const int first_i = p.causal ? j : 0;  // causal: query tiles at or after the key tile
  // window: the last query that sees any key of this tile is kv0 + BKV - 1 + window - 1
  const int end_i = p.window > 0 ? min(num_qt, (kv0 + BKV + p.window - 2) / BQ + 1) : num_qt;
  const int nq = end_i - first_i;  // at least 1: the key tile's own diagonal query tile
  const int steps = G * nq;        // (query head, query tile) pairs, head-major

  if (threadIdx.x == 0) {
    sm100::mbar_init(kvfull, 1);
    for (int i = 0; i < QST; ++i) {
      sm100::mbar_init(&qfull[i], 1);
      sm100::mbar_init(&qempty[i], 1);
    }
    sm100::mbar_init(sfull, 1);
    sm100::mbar_init(sfree, 8);
    for (int i = 0; i < PST; ++i) sm100::mbar_init(&pfull[i], 8);
    sm100::mbar_init(mdone, 1);
    sm100::mbar_init(dqfree, 8);
    sm100::mbar_init(done, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tensormap(&mq);
    sm100::prefetch_tensormap(&mk);
    sm100::prefetch_tensormap(&mv);
    sm100::prefetch_tensormap(&mdo);
  }
  if (warp == 9) {
    sm100::tmem_alloc(tmem_slot, TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 256 + D, tDQ = tmem + L::TDQ;

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      if (!RLB_TMA_X_OK(hk * D) || !RLB_TMA_X_OK(hk * G * D)) fail(p.status, abort_flag, 8);
      sm100::mbar_arrive_expect_tx(kvfull, 2 * DSUB * SUB_BYTES);
#pragma unroll
      for (int s = 0; s < DSUB; ++s) {
        sm100::tma_load_3d(sK + s * SUB_BYTES, &mk, kvfull, hk * D + 64 * s, kv0, b);
        sm100::tma_load_3d(sV + s * SUB_BYTES, &mv, kvfull, hk * D + 64 * s, kv0, b);
      }
      int issued = 0;
      for (int t = 0; t < steps && !*abort_flag; ++t) {
        const int h = hk * G + t / nq, q0 = (first_i + t % nq) * BQ, st = t % QST;
        if (!wait(&qempty[st], ((t / QST) & 1) ^ 1)) {
          fail(p.status, abort_flag, 1);
          break;
        }
        sm100::mbar_arrive_expect_tx(&qfull[st], 2 * DSUB * SUB_BYTES);
#pragma unroll
        for (int s = 0; s < DSUB; ++s) {
          sm100::tma_load_3d(sQ + (st * DSUB + s) * SUB_BYTES, &mq, &qfull[st], h * D + 64 * s, q0, b);
          sm100::tma_load_3d(sDO + (st * DSUB + s) * SUB_BYTES, &mdo, &qfull[st], h * D + 64 * s, q0, b);
        }
        issued = t + 1;
      }
      wait(kvfull, 0);  // own loads land before exit: the last load of each stage
      for (int u = 0; u < QST; ++u) {
        const int t = issued - 1 - u;
        if (t >= 0) wait(&qfull[t % QST], (t / QST) & 1);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = sm100::idesc_bf16_f32(BKV, BQ, 0, 0);  // keys x queries, K = D
      constexpr uint32_t id_kv = sm100::idesc_bf16_f32(BKV, D, 0, 1);  // keys x D, K = queries
      constexpr uint32_t id_q = sm100::idesc_bf16_f32(BQ, D, 1, 1);    // queries x D, K = keys
      const uint32_t ka = sm100::smem_u32(sK), va = sm100::smem_u32(sV);
      bool ok = wait(kvfull, 0);
      if (!ok) fail(p.status, abort_flag, 2);
      // S^T(t), dP^T(t): the columns must have been read by the compute warps (step t - 1); with dQ in S^T's
      // columns, S^T(t) also waits for dQ(t - 1) to be drained
      auto first_half = [&](int t) -> bool {
        const int st = t % QST;
        if (!wait(&qfull[st], (t / QST) & 1)) return false;
        if (t >= 1 && !wait(sfree, (t - 1) & 1)) return false;
        sm100::tc_fence_after();
        const uint32_t qa = sm100::smem_u32(sQ + st * DSUB * SUB_BYTES), da = sm100::smem_u32(sDO + st * DSUB * SUB_BYTES);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (uint32_t)(k >> 2) * SUB_BYTES + (uint32_t)(k & 3) * 32;
          sm100::mma_f16(tDP, sm100::desc_kmajor_sw128(va + off), sm100::desc_kmajor_sw128(da + off), id_s, k > 0);
        }
        if (!DQ_SEP && t >= 1) {
          if (!wait(dqfree, (t - 1) & 1)) return false;
          sm100::tc_fence_after();
        }
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (uint32_t)(k >> 2) * SUB_BYTES + (uint32_t)(k & 3) * 32;
          sm100::mma_f16(tS, sm100::desc_kmajor_sw128(ka + off), sm100::desc_kmajor_sw128(qa + off), id_s, k > 0);
        }
        sm100::mma_commit(sfull);
        return true;
      };
      // dV, dK += ...(i), then dQ(i) once the previous dQ has been drained
      auto second_half = [&](int i) -> bool {
        const int st = i % QST, ps = i % PST;
        if (!wait(&pfull[ps], (i / PST) & 1)) return false;
        sm100::tc_fence_after();
        const uint32_t qa = sm100::smem_u32(sQ + st * DSUB * SUB_BYTES), da = sm100::smem_u32(sDO + st * DSUB * SUB_BYTES);
        const uint32_t pa = sm100::smem_u32(sPT + ps * 2 * SUB_BYTES), sa = sm100::smem_u32(sDS + ps * 2 * SUB_BYTES);
#pragma unroll
        for (int k = 0; k < BQ / 16; ++k) {
          // reduction over 16 queries: K-major A rows (P^T, dS^T) step 32 B in a swizzle row; the MN-major B
          // tiles (dO, Q) step 16 rows = 2048 B, their 64-column boxes SUB_BYTES apart
          const uint32_t off = (uint32_t)(k >> 2) * SUB_BYTES + (uint32_t)(k & 3) * 32;
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          sm100::mma_f16(tDV, sm100::desc_kmajor_sw128(pa + off), sm100::desc_mnmajor_sw128(da + k * 2048, SUB_BYTES),
                         id_kv, acc);
          sm100::mma_f16(tDK, sm100::desc_kmajor_sw128(sa + off), sm100::desc_mnmajor_sw128(qa + k * 2048, SUB_BYTES),
                         id_kv, acc);
        }
        sm100::mma_commit(&qempty[st]);
        if (DQ_SEP && i >= 1) {
          if (!wait(dqfree, (i - 1) & 1)) return false;
          sm100::tc_fence_after();
        }
#pragma unroll
        for (int k = 0; k < BKV / 16; ++k)  // reduction over 16 keys: dS read MN-major from dS^T, K read MN-major
          sm100::mma_f16(tDQ, sm100::desc_mnmajor_sw128(sa + k * 2048, SUB_BYTES),
                         sm100::desc_mnmajor_sw128(ka + k * 2048, SUB_BYTES), id_q, k > 0);
        sm100::mma_commit(mdone);
        return true;
      };
      for (int t = 0; ok && t <= steps && !*abort_flag; ++t) {
        if (DQ_SEP) {
          if (t < steps && !first_half(t)) ok = false;
          if (ok && t >= 1 && !second_half(t - 1)) ok = false;
        } else {
          if (t >= 1 && !second_half(t - 1)) ok = false;
          if (ok && t < steps && !first_half(t)) ok = false;
        }
        if (!ok) fail(p.status, abort_flag, 3);
      }
      sm100::mma_commit(done);  // also the drain: every MMA issued here has completed when it fires
      wait(done, 0);
    }
  } else {
    // ------------------------------------------------------------------ compute warps 0..7
    const int qq = warp & 3, hf = warp >> 2;
    const int row = qq * 32 + lane;  // key row (S^T, dP^T, dV, dK) or query row (dQ) of the tile
    const int key = kv0 + row;
    const uint32_t lanes = (uint32_t)(qq * 32) << 16;
    bool ok = true;
    // dQ of step i (TMEM lane = query of its tile) added into the fp32 accumulator: this warp's D / 2 columns
    auto drain = [&](int i) -> bool {
      if (!wait_warp(mdone, i & 1)) return false;
      sm100::tc_fence_after();
      const int h = hk * G + i / nq, q = (first_i + i % nq) * BQ + row;
      float* dq = p.dq + (((long long)b * p.T + q) * p.Hq + h) * D + hf * (D / 2);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        uint32_t r[32];
        sm100::tmem_ld32(tDQ + lanes + hf * (D / 2) + c * 32, r);
        sm100::tmem_ld_wait();
        if (q < p.T) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            red_add_v4(dq + c * 32 + e, __uint_as_float(r[e]), __uint_as_float(r[e + 1]), __uint_as_float(r[e + 2]),
                       __uint_as_float(r[e + 3]));
        }
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(dqfree);
      return true;
    };
    for (int t = 0; t < steps; ++t) {
      if (__any_sync(0xffffffffu, *abort_flag != 0)) {
        ok = false;
        break;
      }
      const int h = hk * G + t / nq, qi = first_i + t % nq, q0 = qi * BQ, ps = t % PST;
      if (!wait_warp(sfull, t & 1)) {
        fail(p.status, abort_flag, 5);
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const float* lse = p.lse + ((long long)b * p.Hq + h) * p.T;
      const float* delta = p.delta + ((long long)b * p.Hq + h) * p.T;
      const bool masked = (p.causal && qi == j) || (q0 + BQ > p.T) || (kv0 + BKV > p.T) ||
                          (p.window > 0 && q0 + BQ - 1 - kv0 >= p.window);
      uint8_t* pbox = sPT + (ps * 2 + hf) * SUB_BYTES;
      uint8_t* dbox = sDS + (ps * 2 + hf) * SUB_BYTES;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        const int col0 = hf * 64 + c * 32;  // first query column (within the tile) of this chunk
        uint32_t rs[32], rd[32];
        sm100::tmem_ld32(tS + lanes + col0, rs);
        sm100::tmem_ld32(tDP + lanes + col0, rd);
        sm100::tmem_ld_wait();
        if (c == 1) {  // S^T / dP^T fully read: the next step's MMAs may overwrite them
          sm100::tc_fence_before();
          __syncwarp();
          if (lane == 0) sm100::mbar_arrive(sfree);
        }
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const int qc = q0 + col0 + v * 8;  // first query of these 8 columns (same for the whole warp)
          float l2[8], dl[8];
          // vector loads only from 16-byte aligned rows (T a multiple of 4); scalar otherwise
          const bool vec = qc + 8 <= p.T && ((reinterpret_cast<uintptr_t>(lse + qc) |
                                               reinterpret_cast<uintptr_t>(delta + qc)) & 15) == 0;
          if (vec) {
            const float4 a0 = __ldg((const float4*)(lse + qc)), a1 = __ldg((const float4*)(lse + qc + 4));
            const float4 d0 = __ldg((const float4*)(delta + qc)), d1 = __ldg((const float4*)(delta + qc + 4));
            l2[0] = a0.x; l2[1] = a0.y; l2[2] = a0.z; l2[3] = a0.w; l2[4] = a1.x; l2[5] = a1.y; l2[6] = a1.z; l2[7] = a1.w;
            dl[0] = d0.x; dl[1] = d0.y; dl[2] = d0.z; dl[3] = d0.w; dl[4] = d1.x; dl[5] = d1.y; dl[6] = d1.z; dl[7] = d1.w;
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              l2[e] = qc + e < p.T ? __ldg(lse + qc + e) : 0.f;
              dl[e] = qc + e < p.T ? __ldg(delta + qc + e) : 0.f;
            }
          }
          float pf[8], df[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int q = qc + e;
            const bool valid = !masked || (q < p.T && key < p.T && (!p.causal || q >= key) &&
                                           (p.window <= 0 || q - key < p.window));
            const float x = __uint_as_float(rs[v * 8 + e]);
            float pv, dsc;
            if constexpr (CAP) {
              const float th = tanhf(x * p.cap_in);
              pv = sm100::ex2_approx(fmaf(p.cap_log2, th, -l2[e] * LOG2E));
              dsc = p.scale * (1.f - th * th);
            } else {
              pv = sm100::ex2_approx(fmaf(x, p.scale_log2, -l2[e] * LOG2E));
              dsc = p.scale;
            }
            pv = valid ? pv : 0.f;
            pf[e] = pv;
            df[e] = pv * (__uint_as_float(rd[v * 8 + e]) - dl[e]) * dsc;
          }
          const int chunk = c * 4 + v;  // 16-B chunk of this row within the 64-column box
          const int so = (row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4);
          *(uint4*)(pbox + so) = make_uint4(pack_bf16(pf[0], pf[1]), pack_bf16(pf[2], pf[3]), pack_bf16(pf[4], pf[5]),
                                            pack_bf16(pf[6], pf[7]));
          *(uint4*)(dbox + so) = make_uint4(pack_bf16(df[0], df[1]), pack_bf16(df[2], df[3]), pack_bf16(df[4], df[5]),
                                            pack_bf16(df[6], df[7]));
        }
      }
      sm100::fence_async_shared();  // P^T, dS^T visible to the tensor core
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&pfull[ps]);
      // dQ of the previous step (d 64) or of this one (d 128)
      const int di = DQ_SEP ? t - 1 : t;
      if (di >= 0 && !drain(di)) {
        fail(p.status, abort_flag, 6);
        ok = false;
        break;
      }
    }
    if (ok && DQ_SEP && !drain(steps - 1)) {
      fail(p.status, abort_flag, 6);
      ok = false;
    }
    if (ok) {
      if (wait_warp(done, 0)) {
        sm100::tc_fence_after();
        // every lane runs the (warp-collective) TMEM loads; only rows of real keys are stored
        const long long o = (((long long)b * p.T + key) * p.Hkv + hk) * D + hf * (D / 2);
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          uint32_t rv[32], rk[32];
          sm100::tmem_ld32(tDV + lanes + hf * (D / 2) + c * 32, rv);
          sm100::tmem_ld32(tDK + lanes + hf * (D / 2) + c * 32, rk);
          sm100::tmem_ld_wait();
          if (key >= p.T) continue;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const uint32_t* a = rv + v * 8;
            const uint32_t* k = rk + v * 8;
            *(uint4*)(p.dv + o + c * 32 + v * 8) =
                make_uint4(pack_bf16(__uint_as_float(a[0]), __uint_as_float(a[1])),
                           pack_bf16(__uint_as_float(a[2]), __uint_as_float(a[3])),
                           pack_bf16(__uint_as_float(a[4]), __uint_as_float(a[5])),
                           pack_bf16(__uint_as_float(a[6]), __uint_as_float(a[7])));
            *(uint4*)(p.dk + o + c * 32 + v * 8) =
                make_uint4(pack_bf16(__uint_as_float(k[0]), __uint_as_float(k[1])),
                           pack_bf16(__uint_as_float(k[2]), __uint_as_float(k[3])),
                           pack_bf16(__uint_as_float(k[4]), __uint_as_float(k[5])),
                           pack_bf16(__uint_as_float(k[6]), __uint_as_float(k[7])));
          }
        }
        sm100::tc_fence_before();
      } else {
        fail(p.status, abort_flag, 7);
      }
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host
using rlb_tmap::EncodeTiledFn;
using rlb_tmap::encode_fn;

static bool make_map(CUtensorMap* m, const void* ptr, int B, int T, int HD) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)T * HD * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)BQ, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D>
static cudaError_t launch(const void* q, const void* k, const void* v, const void* dout, const Params& p,
                          cudaStream_t s) {
  CUtensorMap mq, mk, mv, mdo;
  if (!make_map(&mq, q, p.B, p.T, p.Hq * D) || !make_map(&mk, k, p.B, p.T, p.Hkv * D) ||
      !make_map(&mv, v, p.B, p.T, p.Hkv * D) || !make_map(&mdo, dout, p.B, p.T, p.Hq * D))
    return cudaErrorInvalidResourceHandle;
  auto kern = p.cap_log2 > 0.f ? fmha_bwd_kernel<D, true> : fmha_bwd_kernel<D, false>;
  constexpr int smem = Layout<D>::BYTES + 1024;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  (void)cudaGetLastError();
  const dim3 grid((p.T + BKV - 1) / BKV, p.Hkv, p.B);
  kern<<<grid, THREADS, smem, s>>>(mq, mk, mv, mdo, p);
  return cudaGetLastError();
}

}  // namespace fmha_bwd

// q, dout [B][T][Hq][D], k, v [B][T][Hkv][D] bf16; lse, delta [B][Hq][T] fp32; dq [B][T][Hq][D] fp32 (zeroed by
// the caller, accumulated); dk, dv [B][T][Hkv][D] bf16 (written).
cudaError_t rlb_fmha_bwd(const void* q, const void* k, const void* v, const void* dout, const float* lse,
                         const float* delta, float* dq, void* dk, void* dv, int B, int T, int Hq, int Hkv, int D,
                         int causal, float scale, int window, float softcap, int* status, cudaStream_t s) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  if (window < 0 || softcap < 0.f) return cudaErrorInvalidValue;
  if ((D != 64 && D != 128) || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Hkv > 65535 || B > 65535)
    return cudaErrorInvalidValue;
  if ((((uintptr_t)q) | ((uintptr_t)k) | ((uintptr_t)v) | ((uintptr_t)dout) | ((uintptr_t)dk) | ((uintptr_t)dv)) & 15)
    return cudaErrorInvalidDevicePointer;
  fmha_bwd::Params p{};
  p.lse = lse;
  p.delta = delta;
  p.dq = dq;
  p.dk = (__nv_bfloat16*)dk;
  p.dv = (__nv_bfloat16*)dv;
  p.B = B;
  p.T = T;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  p.window = window;
  p.cap_in = softcap > 0.f ? scale / softcap : 0.f;
  p.cap_log2 = softcap > 0.f ? softcap * 1.4426950408889634f : 0.f;
  p.status = status;
  return D == 128 ? fmha_bwd::launch<128>(q, k, v, dout, p, s) : fmha_bwd::launch<64>(q, k, v, dout, p, s);
}
