// Fused multi-head attention, forward, for sm_100a: tcgen05 MMAs with TMEM accumulators, TMA tile loads.
//
//   out[b, t, h, :] = softmax(f(scale * q[b, t, h, :] . k[b, s, h / G, :]^T)  (+ masks)) v[b, s, h / G, :]
//
// with f(x) = x, or f(x) = cap * tanh(x / cap) for a logit soft-cap; masks: causal (s <= t) and a sliding
// window (t - s < window).  Key tiles that a query tile's rows cannot see at all are skipped.
//
// q, k, v and out are token-major [B, T, H, D] bf16 (the layout the fused RoPE kernel writes).  Head
// dims: D = 64 or 128 for q, k, v alike, or d_qk = 192 with d_v = 128 (multi-head latent attention with
// its decoupled RoPE part, prefill / training shape); grouped-query heads G = Hq / Hkv.  Optionally also writes lse[b, h, t] = log sum_s exp(scale q.k)
// (natural log) for a backward pass.  The reference runs attention through PyTorch
// (``src/forgeline/models/attention/causal.py:79-134``); this is the B200 kernel behind the same op.
//
// One CTA (192 threads) per (128-query tile, head, batch); causal CTAs start with the longest rows.
//   warp 0      TMA producer: the Q tile once, then K and V tiles (128 keys) through two-stage rings.
//   warp 1      TMEM owner (all 512 columns) and MMA issuer (one elected thread):
//                 S_j = Q K_j^T      M=128, N=128, K=D    -> TMEM S[j % 2]   (columns 0..255)
//                 O_j = P_j V_j      M=128, N=D,   K=128  -> TMEM O[j % 2]   (columns 256..511)
//               S_{j+1} is issued before O_j, so the tensor core computes the next scores while the
//               softmax warps work on the current ones.
//   warps 2-5   softmax: thread r owns query row r of the tile (warp w reads TMEM lanes 32 (w % 4)..).
//               Per key tile: row max of S_j (first read of the row), fold the previous tile's O_{j-1}
//               into the register accumulator with the online-softmax rescale, then exponentiate
//               (second read of the row), write P_j as bf16 into shared memory in the 128-byte-swizzled
//               K-major layout the MMA reads, and hand S[j % 2] back.  The final O is divided by the
//               softmax denominator and stored.
// P V accumulates per tile in TMEM and is folded into registers, so no TMEM accumulator is ever
// rescaled in place.  Every mbarrier wait is bounded: on timeout the kernel records an error in
// `status`, stops every role, waits (bounded) for its own TMA loads and MMAs, frees TMEM and returns.
// No load uses cluster delivery.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>
#include <climits>
#include <cstdlib>
#include <stdint.h>

#include "sm100.cuh"
#include "tmap.h"

namespace fmha {

constexpr int BQ = 128, BKV = 128;
constexpr int SUB_BYTES = 128 * 64 * 2;  // one [128 rows][64 columns] bf16 box, 128-B swizzled: 16 KB
constexpr int TMEM_COLS = 512;
constexpr uint32_t WAIT_LIMIT = 1u << 26;  // polls before a wait is declared dead (seconds)
constexpr float LN2 = 0.6931471805599453f;

template <int D, int DV>
struct Layout {
  static constexpr int DSUB = D / 64;   // 64-column boxes per row of Q / K
  static constexpr int VSUB = DV / 64;  // ... of V
  // V stages: two when they fit in shared memory, one for the 192-wide Q / K tiles
  static constexpr int VST = (3 * DSUB + 2 * VSUB + 2) * SUB_BYTES + 256 + 1024 <= 232448 ? 2 : 1;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + DSUB * SUB_BYTES;
  static constexpr int V_OFF = K_OFF + 2 * DSUB * SUB_BYTES;
  static constexpr int P_OFF = V_OFF + VST * VSUB * SUB_BYTES;
  static constexpr int BAR_OFF = P_OFF + 2 * SUB_BYTES;  // P: [128 queries][128 keys] as two boxes
  static constexpr int BYTES = BAR_OFF + 256;
};
// Every launch asks for at least the D = 128 footprint, so at most one CTA is resident per SM (a CTA
// allocates all 512 TMEM columns).
template <int D, int DV>
constexpr int smem_request() {
  return (Layout<D, DV>::BYTES > Layout<128, 128>::BYTES ? Layout<D, DV>::BYTES : Layout<128, 128>::BYTES) + 1024;
}

struct Params {
  __nv_bfloat16* out;  // [B][T][Hq][D]
  float* lse;          // [B][Hq][T] or nullptr
  int B, T, Hq, Hkv;
  float scale_log2;  // softmax scale * log2(e)
  int causal;
  int window;        // 0: none; else key s is visible to query t only if t - s < window
  float cap_in;      // soft-cap: scale / cap (the tanh argument per raw score)
  float cap_log2;    // soft-cap: cap * log2(e)
  int* status;
};

// Score of one raw accumulator value in log2 units: scale * x * log2(e), or cap * tanh(scale * x / cap) * log2(e).
template <bool CAP>
__device__ __forceinline__ float score_log2(float x, const Params& p) {
  if constexpr (CAP) return p.cap_log2 * tanhf(x * p.cap_in);
  else return x * p.scale_log2;
}

__device__ __forceinline__ void fail(int* status, volatile int* abort_flag, int where) {
  *abort_flag = 1;
  if (status) atomicCAS(status, 0, 1 | (where << 8));
}

__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity) {
  return sm100::mbar_wait_bounded(bar, parity, WAIT_LIMIT);
}

// fp32 pair -> packed bf16x2
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// The same wait with one answer for the whole warp (the compute warps' TMEM loads are warp-collective,
// so a warp must never split on a wait that ran out for some lanes only).
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, wait(bar, parity));
}

template <int D, int DV, bool CAP>
__global__ void __launch_bounds__(192, 1) fmha_fwd_kernel(const __grid_constant__ CUtensorMap mq,
                                                          const __grid_constant__ CUtensorMap mk,
                                                          const __grid_constant__ CUtensorMap mv, Params p) {
  using L = Layout<D, DV>;
  constexpr int DSUB = L::DSUB, VSUB = L::VSUB, VST = L::VST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem + L::Q_OFF;
  uint8_t* sK = smem + L::K_OFF;
  uint8_t* sV = smem + L::V_OFF;
  uint8_t* sP = smem + L::P_OFF;
  uint64_t* bars = (uint64_t*)(smem + L::BAR_OFF);
  uint64_t* qfull = bars;
  uint64_t* kfull = bars + 1;
  uint64_t* kempty = bars + 3;
  uint64_t* vfull = bars + 5;
  uint64_t* vempty = bars + 7;
  uint64_t* sfull = bars + 9;
  uint64_t* sempty = bars + 11;
  uint64_t* pfull = bars + 13;
  uint64_t* ofull = bars + 14;
  uint64_t* oempty = bars + 16;
  uint64_t* drain = bars + 18;
  uint32_t* tmem_slot = (uint32_t*)(bars + 20);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_qt = (p.T + BQ - 1) / BQ;
  const int qt = num_qt - 1 - (int)blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int q0 = qt * BQ;
  const int nkv_all = (p.T + BKV - 1) / BKV;
  const int j_end = p.causal ? min(qt + 1, nkv_all) : nkv_all;                   // one past the last key tile
  const int j0 = p.window > 0 ? min(max(q0 - p.window + 1, 0) / BKV, j_end) : 0;  // first key tile any row sees
  // key tiles this query tile reads (at least the diagonal one); loop step j reads key tile j0 + j
  const int n = j_end - j0;
  // a tile needs per-element masks if it runs past T, crosses the causal diagonal, or reaches below the
  // window of the tile's last row
  const int win_lo = p.window > 0 ? q0 + BQ - p.window : INT_MIN;

  if (threadIdx.x == 0) {
    sm100::mbar_init(qfull, 1);
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&kfull[i], 1);
      sm100::mbar_init(&kempty[i], 1);
      sm100::mbar_init(&vfull[i], 1);
      sm100::mbar_init(&vempty[i], 1);
      sm100::mbar_init(&sfull[i], 1);
      sm100::mbar_init(&sempty[i], 4);
      sm100::mbar_init(&ofull[i], 1);
      sm100::mbar_init(&oempty[i], 4);
    }
    sm100::mbar_init(pfull, 4);
    sm100::mbar_init(drain, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tensormap(&mq);
    sm100::prefetch_tensormap(&mk);
    sm100::prefetch_tensormap(&mv);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int k_issued = 0, v_issued = 0;  // key tiles whose K / V loads were issued
      if (!RLB_TMA_X_OK(h * D) || !RLB_TMA_X_OK(hk * D) || !RLB_TMA_X_OK(hk * DV)) fail(p.status, abort_flag, 12);
      sm100::mbar_arrive_expect_tx(qfull, DSUB * SUB_BYTES);
#pragma unroll
      for (int s = 0; s < DSUB; ++s) sm100::tma_load_3d(sQ + s * SUB_BYTES, &mq, qfull, h * D + 64 * s, q0, b);
      for (int j = 0; j < n && !*abort_flag; ++j) {
        const int buf = j & 1;
        const uint32_t par = (j >> 1) & 1;
        if (!wait(&kempty[buf], par ^ 1)) {
          fail(p.status, abort_flag, 1);
          break;
        }
        sm100::mbar_arrive_expect_tx(&kfull[buf], DSUB * SUB_BYTES);
#pragma unroll
        for (int s = 0; s < DSUB; ++s)
          sm100::tma_load_3d(sK + (buf * DSUB + s) * SUB_BYTES, &mk, &kfull[buf], hk * D + 64 * s, (j0 + j) * BKV, b);
        k_issued = j + 1;
        const int vb = j % VST;
        if (!wait(&vempty[vb], ((j / VST) & 1) ^ 1)) {
          fail(p.status, abort_flag, 2);
          break;
        }
        sm100::mbar_arrive_expect_tx(&vfull[vb], VSUB * SUB_BYTES);
#pragma unroll
        for (int s = 0; s < VSUB; ++s)
          sm100::tma_load_3d(sV + (vb * VSUB + s) * SUB_BYTES, &mv, &vfull[vb], hk * DV + 64 * s, (j0 + j) * BKV, b);
        v_issued = j + 1;
      }
      // every load issued here lands before the CTA exits (a buffer's earlier loads were consumed
      // before its next one was issued, so waiting for the last load of each buffer is enough)
      wait(qfull, 0);
      for (int t = 0; t < 2; ++t) {
        const int jk = k_issued - 1 - t, jv = v_issued - 1 - t;
        if (jk >= 0) wait(&kfull[jk & 1], (jk >> 1) & 1);
        if (jv >= 0 && t < VST) wait(&vfull[jv % VST], (jv / VST) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = sm100::idesc_bf16_f32(BQ, BKV, 0, 0);  // Q, K both K-major
      constexpr uint32_t id_o = sm100::idesc_bf16_f32(BQ, DV, 0, 1);   // P K-major, V [keys][DV]: MN-major
      bool ok = wait(qfull, 0);
      if (!ok) fail(p.status, abort_flag, 3);
      const uint32_t qa = sm100::smem_u32(sQ), pa = sm100::smem_u32(sP);
      for (int j = 0; ok && j <= n && !*abort_flag; ++j) {
        if (j < n) {
          const int buf = j & 1;
          const uint32_t par = (j >> 1) & 1;
          if (!wait(&kfull[buf], par)) {
            fail(p.status, abort_flag, 4);
            break;
          }
          if (!wait(&sempty[buf], par ^ 1)) {
            fail(p.status, abort_flag, 5);
            break;
          }
          sm100::tc_fence_after();
          const uint32_t ka = sm100::smem_u32(sK + buf * DSUB * SUB_BYTES);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            // 16 columns of D per MMA: box k / 4, +32 B per step inside the 128-B swizzle row
            const uint32_t off = (uint32_t)(k >> 2) * SUB_BYTES + (uint32_t)(k & 3) * 32;
            sm100::mma_f16(tmem + buf * BKV, sm100::desc_kmajor_sw128(qa + off), sm100::desc_kmajor_sw128(ka + off),
                           id_s, k > 0);
          }
          sm100::mma_commit(&kempty[buf]);
          sm100::mma_commit(&sfull[buf]);
        }
        if (j >= 1) {
          const int i = j - 1, ib = i & 1;
          const uint32_t ipar = (i >> 1) & 1;
          if (!wait(pfull, i & 1)) {
            fail(p.status, abort_flag, 6);
            break;
          }
          if (!wait(&vfull[i % VST], (i / VST) & 1)) {
            fail(p.status, abort_flag, 7);
            break;
          }
          if (!wait(&oempty[ib], ipar ^ 1)) {
            fail(p.status, abort_flag, 8);
            break;
          }
          sm100::tc_fence_after();
          const uint32_t va = sm100::smem_u32(sV + (i % VST) * VSUB * SUB_BYTES);
#pragma unroll
          for (int k = 0; k < BKV / 16; ++k) {
            // P: 16 keys per MMA (K-major, like Q);  V: 16 key rows = two 8-row 1024-B atoms, the
            // 64-column boxes along D one SUB_BYTES apart
            const uint32_t poff = (uint32_t)(k >> 2) * SUB_BYTES + (uint32_t)(k & 3) * 32;
            sm100::mma_f16(tmem + 2 * BKV + ib * DV, sm100::desc_kmajor_sw128(pa + poff),
                           sm100::desc_mnmajor_sw128(va + k * 2048, SUB_BYTES), id_o, k > 0);
          }
          sm100::mma_commit(&vempty[i % VST]);
          sm100::mma_commit(&ofull[ib]);
        }
      }
      // every MMA issued here completes before TMEM is released
      sm100::mma_commit(drain);
      wait(drain, 0);
    }
  } else {
    // ------------------------------------------------------------------ softmax (warps 2..5)
    const int qq = warp & 3;
    const int row = qq * 32 + lane;
    const int rq = q0 + row;
    const uint32_t lanes = tmem + ((uint32_t)(qq * 32) << 16);
    float O[DV];
#pragma unroll
    for (int d = 0; d < DV; ++d) O[d] = 0.f;
    float m = -INFINITY, l = 0.f;  // running row max (log2 units) and denominator
    float m_o = -INFINITY;         // max the register accumulator O is scaled to
    float m_p = -INFINITY;         // max the last P written was scaled to
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (__any_sync(0xffffffffu, *abort_flag != 0)) {
        ok = false;
        break;
      }
      const int buf = j & 1;
      const uint32_t par = (j >> 1) & 1;
      if (!wait_warp(&sfull[buf], par)) {
        fail(p.status, abort_flag, 9);
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const uint32_t ts = lanes + buf * BKV;
      const int kv0 = (j0 + j) * BKV;
      const bool masked = (kv0 + BKV > p.T) || (p.causal && kv0 + BKV - 1 > q0) || (kv0 < win_lo);
      // pass 1: row max over this key tile
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < BKV / 32; ++c) {
        uint32_t r[32];
        sm100::tmem_ld32(ts + c * 32, r);
        sm100::tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int col = kv0 + c * 32 + e;
          const bool valid =
              !masked || (col < p.T && (!p.causal || col <= rq) && (p.window <= 0 || rq - col < p.window));
          mx = valid ? fmaxf(mx, score_log2<CAP>(__uint_as_float(r[e]), p)) : mx;
        }
      }
      const float m_new = fmaxf(m, mx);
      // fold the previous tile's P V into the accumulator (both brought to the max P_{j-1} used)
      if (j >= 1) {
        const int i = j - 1, ib = i & 1;
        if (!wait_warp(&ofull[ib], (i >> 1) & 1)) {
          fail(p.status, abort_flag, 10);
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const float a = (m_o == -INFINITY) ? 0.f : exp2f(m_o - m_p);
#pragma unroll
        for (int c = 0; c < DV / 32; ++c) {
          uint32_t r[32];
          sm100::tmem_ld32(lanes + 2 * BKV + ib * DV + c * 32, r);
          sm100::tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) O[c * 32 + e] = fmaf(O[c * 32 + e], a, __uint_as_float(r[e]));
        }
        m_o = m_p;
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&oempty[ib]);
      }
      // pass 2: probabilities, row sum, bf16 P into shared memory (the previous P V has finished reading it)
      const float moff = (m_new == -INFINITY) ? 0.f : m_new;
      float rs = 0.f;
#pragma unroll 1
      for (int c = 0; c < BKV / 32; ++c) {
        uint32_t r[32];
        sm100::tmem_ld32(ts + c * 32, r);
        sm100::tmem_ld_wait();
        // row `row` of the box holding keys [64 (c / 2), 64 (c / 2) + 64): 8-row atoms of 1024 B, 16-B
        // chunk k of a 128-B row stored at chunk k ^ (row % 8) (the TMA / UMMA 128-B swizzle)
        uint8_t* prow = sP + (c >> 1) * SUB_BYTES + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int col = kv0 + c * 32 + v * 8 + e;
            const bool valid =
                !masked || (col < p.T && (!p.causal || col <= rq) && (p.window <= 0 || rq - col < p.window));
            f[e] = valid ? exp2f(score_log2<CAP>(__uint_as_float(r[v * 8 + e]), p) - moff) : 0.f;
            rs += f[e];
          }
          uint4 pk;
          uint32_t* w = (uint32_t*)&pk;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 hh = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
            w[e] = *(uint32_t*)&hh;
          }
          const int chunk = (c & 1) * 4 + v;
          *(uint4*)(prow + ((chunk ^ (row & 7)) << 4)) = pk;
        }
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&sempty[buf]);
      sm100::fence_async_shared();  // P (generic-proxy stores) visible to the tensor core
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(pfull);
      l = (m == -INFINITY ? 0.f : l * exp2f(m - m_new)) + rs;
      m = m_new;
      m_p = m_new;
    }
    if (ok && n > 0) {
      const int i = n - 1, ib = i & 1;
      if (wait_warp(&ofull[ib], (i >> 1) & 1)) {
        sm100::tc_fence_after();
        const float a = (m_o == -INFINITY) ? 0.f : exp2f(m_o - m_p);
#pragma unroll
        for (int c = 0; c < DV / 32; ++c) {
          uint32_t r[32];
          sm100::tmem_ld32(lanes + 2 * BKV + ib * DV + c * 32, r);
          sm100::tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) O[c * 32 + e] = fmaf(O[c * 32 + e], a, __uint_as_float(r[e]));
        }
        sm100::tc_fence_before();
        if (rq < p.T) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
          __nv_bfloat16* dst = p.out + (((long long)b * p.T + rq) * p.Hq + h) * DV;
#pragma unroll
          for (int v = 0; v < DV / 8; ++v) {
            uint4 pk;
            uint32_t* w = (uint32_t*)&pk;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __nv_bfloat162 hh = __floats2bfloat162_rn(O[v * 8 + 2 * e] * inv, O[v * 8 + 2 * e + 1] * inv);
              w[e] = *(uint32_t*)&hh;
            }
            *(uint4*)(dst + v * 8) = pk;
          }
          if (p.lse) p.lse[((long long)b * p.Hq + h) * p.T + rq] = l > 0.f ? (m + log2f(l)) * LN2 : -INFINITY;
        }
      } else {
        fail(p.status, abort_flag, 11);
      }
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ two heads per CTA
// For grouped-query attention with an even group size and d_qk == d_v in {64, 128}: one CTA takes the same
// 128-query tile of two heads h0, h0 + 1 of one KV group, so every K / V tile is loaded once for both and the
// tensor core alternates between the heads' MMAs.  384 threads (three warpgroups; the launch gives each thread
// 168 registers, then `setmaxnreg` moves them: 224 to each softmax thread, 56 to the third warpgroup --
// 256 x 224 + 128 x 56 = 64512 = 384 x 168):
//   warps 0-3 / 4-7   softmax of head 0 / head 1: thread r owns query row r of its head.  Per key tile the S row
//                     is read from TMEM once (128 registers), the row max updated, the exponentials written as
//                     bf16 P into shared memory; O stays in TMEM and is rescaled there only when the running
//                     max grows by more than RESCALE (log2 units) -- P entries are otherwise exponentials
//                     against a stale max, at most 2^RESCALE, which bf16 and the fp32 accumulator hold exactly
//                     enough.  The final O is read once, divided by the softmax denominator and stored.
//   warp 8            TMA producer: both Q tiles once, then K / V tiles through rings.  (Warps 10, 11 idle.)
//   warp 9            TMEM owner (512 columns: S0 0..127, S1 128..255, O0 256.., O1 256 + D..) and MMA issuer:
//                     S_h(j) = Q_h K_j^T for both heads, then O_h += P_h(j - 1) V_{j - 1}.
constexpr float RESCALE = 8.0f;
constexpr int PAIR_THREADS = 384;

template <int N>
__device__ __forceinline__ void reg_alloc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
__device__ __forceinline__ void reg_dealloc() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }

template <int D>
struct PairLayout {
  static constexpr int DSUB = D / 64;
  static constexpr int KST = 2;
  static constexpr int VST = D == 64 ? 2 : 1;  // D = 128: one V stage keeps the CTA within shared memory
  static constexpr int PST = D == 64 ? 2 : 1;  // P buffers per head (D = 64: P(j) written while P(j - 1) V runs)
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + 2 * DSUB * SUB_BYTES;
  static constexpr int V_OFF = K_OFF + KST * DSUB * SUB_BYTES;
  static constexpr int P_OFF = V_OFF + VST * DSUB * SUB_BYTES;  // [PST][head][2 boxes]
  static constexpr int BAR_OFF = P_OFF + PST * 2 * 2 * SUB_BYTES;
  static constexpr int BYTES = BAR_OFF + 512;
  static_assert(BYTES + 1024 <= 232448, "shared memory budget of one sm_100a CTA");
};

template <int D, bool CAP>
__global__ void __launch_bounds__(PAIR_THREADS, 1) fmha_fwd_pair_kernel(const __grid_constant__ CUtensorMap mq,
                                                               const __grid_constant__ CUtensorMap mk,
                                                               const __grid_constant__ CUtensorMap mv, Params p) {
  using L = PairLayout<D>;
  constexpr int DSUB = L::DSUB, KST = L::KST, VST = L::VST, PST = L::PST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem + L::Q_OFF;
  uint8_t* sK = smem + L::K_OFF;
  uint8_t* sV = smem + L::V_OFF;
  uint8_t* sP = smem + L::P_OFF;
  uint64_t* bars = (uint64_t*)(smem + L::BAR_OFF);
  uint64_t* qfull = bars;
  uint64_t* kfull = bars + 1;
  uint64_t* kempty = kfull + KST;
  uint64_t* vfull = kempty + KST;
  uint64_t* vempty = vfull + VST;
  uint64_t* sfull = vempty + VST;  // [head]
  uint64_t* sfree = sfull + 2;     // [head]
  // [head][tile parity]: a barrier per tile parity cannot run two phases ahead of a waiter (a head finishing
  // tiles j and j + 2 needs P(j) V in between)
  uint64_t* pfull = sfree + 2;
  uint64_t* odone = pfull + 4;
  uint64_t* drain = odone + 4;
  uint32_t* tmem_slot = (uint32_t*)(drain + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_qt = (p.T + BQ - 1) / BQ;
  const int qt = num_qt - 1 - (int)blockIdx.x;  // longest causal rows first
  const int h0 = 2 * blockIdx.y, b = blockIdx.z;
  const int hk = h0 / (p.Hq / p.Hkv);
  const int q0 = qt * BQ;
  const int nkv_all = (p.T + BKV - 1) / BKV;
  const int j_end = p.causal ? min(qt + 1, nkv_all) : nkv_all;
  const int j0 = p.window > 0 ? min(max(q0 - p.window + 1, 0) / BKV, j_end) : 0;
  const int n = j_end - j0;  // at least 1 (the diagonal tile); loop step j reads key tile j0 + j
  const int win_lo = p.window > 0 ? q0 + BQ - p.window : INT_MIN;

  if (threadIdx.x == 0) {
    sm100::mbar_init(qfull, 1);
    for (int i = 0; i < KST; ++i) {
      sm100::mbar_init(&kfull[i], 1);
      sm100::mbar_init(&kempty[i], 1);
    }
    for (int i = 0; i < VST; ++i) {
      sm100::mbar_init(&vfull[i], 1);
      sm100::mbar_init(&vempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&sfull[i], 1);
      sm100::mbar_init(&sfree[i], 4);
    }
    for (int i = 0; i < 4; ++i) {
      sm100::mbar_init(&pfull[i], 4);
      sm100::mbar_init(&odone[i], 1);
    }
    sm100::mbar_init(drain, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tensormap(&mq);
    sm100::prefetch_tensormap(&mk);
    sm100::prefetch_tensormap(&mv);
  }
  if (warp == 9) {
    sm100::tmem_alloc(tmem_slot, TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp >= 8) {
    reg_dealloc<56>();  // the whole third warpgroup, before its roles split
  if (warp == 8) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int k_issued = 0, v_issued = 0;
      if (!RLB_TMA_X_OK(h0 * D) || !RLB_TMA_X_OK(hk * D)) fail(p.status, abort_flag, 12);
      sm100::mbar_arrive_expect_tx(qfull, 2 * DSUB * SUB_BYTES);
#pragma unroll
      for (int w = 0; w < 2; ++w)
#pragma unroll
        for (int s = 0; s < DSUB; ++s)
          sm100::tma_load_3d(sQ + (w * DSUB + s) * SUB_BYTES, &mq, qfull, (h0 + w) * D + 64 * s, q0, b);
      for (int j = 0; j < n && !*abort_flag; ++j) {
        const int kb = j % KST, vb = j % VST;
        if (!wait(&kempty[kb], ((j / KST) & 1) ^ 1)) {
          fail(p.status, abort_flag, 1);
          break;
        }
        sm100::mbar_arrive_expect_tx(&kfull[kb], DSUB * SUB_BYTES);
#pragma unroll
        for (int s = 0; s < DSUB; ++s)
          sm100::tma_load_3d(sK + (kb * DSUB + s) * SUB_BYTES, &mk, &kfull[kb], hk * D + 64 * s, (j0 + j) * BKV, b);
        k_issued = j + 1;
        if (!wait(&vempty[vb], ((j / VST) & 1) ^ 1)) {
          fail(p.status, abort_flag, 2);
          break;
        }
        sm100::mbar_arrive_expect_tx(&vfull[vb], DSUB * SUB_BYTES);
#pragma unroll
        for (int s = 0; s < DSUB; ++s)
          sm100::tma_load_3d(sV + (vb * DSUB + s) * SUB_BYTES, &mv, &vfull[vb], hk * D + 64 * s, (j0 + j) * BKV, b);
        v_issued = j + 1;
      }
      // every load issued here lands before the CTA exits: the last load of each ring slot
      wait(qfull, 0);
      for (int t = 0; t < KST; ++t) {
        const int jk = k_issued - 1 - t;
        if (jk >= 0) wait(&kfull[jk % KST], (jk / KST) & 1);
      }
      for (int t = 0; t < VST; ++t) {
        const int jv = v_issued - 1 - t;
        if (jv >= 0) wait(&vfull[jv % VST], (jv / VST) & 1);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = sm100::idesc_bf16_f32(BQ, BKV, 0, 0);
      constexpr uint32_t id_o = sm100::idesc_bf16_f32(BQ, D, 0, 1);
      bool ok = wait(qfull, 0);
      if (!ok) fail(p.status, abort_flag, 3);
      for (int j = 0; ok && j <= n && !*abort_flag; ++j) {
        if (j < n) {
          const int kb = j % KST;
          if (!wait(&kfull[kb], (j / KST) & 1)) {
            fail(p.status, abort_flag, 4);
            break;
          }
          const uint32_t ka = sm100::smem_u32(sK + kb * DSUB * SUB_BYTES);
          for (int w = 0; w < 2 && ok; ++w) {
            if (!wait(&sfree[w], (j & 1) ^ 1)) {
              fail(p.status, abort_flag, 5);
              ok = false;
              break;
            }
            sm100::tc_fence_after();
            const uint32_t qa = sm100::smem_u32(sQ + w * DSUB * SUB_BYTES);
#pragma unroll
            for (int k = 0; k < D / 16; ++k) {
              const uint32_t off = (uint32_t)(k >> 2) * SUB_BYTES + (uint32_t)(k & 3) * 32;
              sm100::mma_f16(tmem + w * BKV, sm100::desc_kmajor_sw128(qa + off), sm100::desc_kmajor_sw128(ka + off),
                             id_s, k > 0);
            }
            sm100::mma_commit(&sfull[w]);
          }
          if (!ok) break;
          sm100::mma_commit(&kempty[kb]);
        }
        if (j >= 1) {
          const int i = j - 1, vb = i % VST;
          if (!wait(&vfull[vb], (i / VST) & 1)) {
            fail(p.status, abort_flag, 7);
            break;
          }
          const uint32_t va = sm100::smem_u32(sV + vb * DSUB * SUB_BYTES);
          for (int w = 0; w < 2 && ok; ++w) {
            if (!wait(&pfull[2 * w + (i & 1)], (i >> 1) & 1)) {
              fail(p.status, abort_flag, 6);
              ok = false;
              break;
            }
            sm100::tc_fence_after();
            const uint32_t pa = sm100::smem_u32(sP + ((i % PST) * 2 + w) * 2 * SUB_BYTES);
#pragma unroll
            for (int k = 0; k < BKV / 16; ++k) {
              const uint32_t poff = (uint32_t)(k >> 2) * SUB_BYTES + (uint32_t)(k & 3) * 32;
              sm100::mma_f16(tmem + 2 * BKV + w * D, sm100::desc_kmajor_sw128(pa + poff),
                             sm100::desc_mnmajor_sw128(va + k * 2048, SUB_BYTES), id_o, (i > 0 || k > 0) ? 1u : 0u);
            }
            sm100::mma_commit(&odone[2 * w + (i & 1)]);
          }
          if (!ok) break;
          sm100::mma_commit(&vempty[vb]);
        }
      }
      sm100::mma_commit(drain);  // every MMA issued here completes before TMEM is released
      wait(drain, 0);
    }
  }
  } else {
    // ------------------------------------------------------------------ softmax (warps 0..7)
    reg_alloc<224>();
    const int w = warp >> 2, qq = warp & 3;
    const int row = qq * 32 + lane;
    const int rq = q0 + row;
    const uint32_t lanes = tmem + ((uint32_t)(qq * 32) << 16);
    const uint32_t tS = lanes + w * BKV, tO = lanes + 2 * BKV + w * D;
    // P V of tile i has completed (odone of head w, tile parity i & 1, phase i / 2)
    auto pv_done = [&](int i) { return wait_warp(&odone[2 * w + (i & 1)], (i >> 1) & 1); };
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (__any_sync(0xffffffffu, *abort_flag != 0)) {
        ok = false;
        break;
      }
      if (!wait_warp(&sfull[w], j & 1)) {
        fail(p.status, abort_flag, 9);
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      uint32_t sv[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) sm100::tmem_ld32(tS + c * 32, sv[c]);
      sm100::tmem_ld_wait();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&sfree[w]);  // the next S of this head may overwrite the columns
      const int kv0 = (j0 + j) * BKV;
      const bool masked = (kv0 + BKV > p.T) || (p.causal && kv0 + BKV - 1 > q0) || (kv0 < win_lo);
      // masked entries become -inf once, before the max
      if (masked) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int col = kv0 + c * 32 + e;
            const bool valid =
                col < p.T && (!p.causal || col <= rq) && (p.window <= 0 || rq - col < p.window);
            if (!valid) sv[c][e] = __float_as_uint(-INFINITY);
          }
      }
      float mx8[8];  // independent chains: the max is 16 dependent steps, not 128
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int e = 0; e < 32; ++e) mx8[e & 7] = fmaxf(mx8[e & 7], __uint_as_float(sv[c][e]));
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      // the score transform is increasing, so the max of the scores is the transform of the raw max
      const float m_tile = mx == -INFINITY ? -INFINITY : score_log2<CAP>(mx, p);
      const float m_new = fmaxf(m_used, m_tile);
      const bool need = m_new > m_used + RESCALE;  // also the first finite max
      const float alpha = !need ? 1.f : (m_used == -INFINITY ? 0.f : sm100::ex2_approx(m_used - m_new));
      // this tile's P buffer was last read by P V of tile j - PST; an O rescale needs every earlier P V done
      const bool rescale = j >= 1 && __any_sync(0xffffffffu, need);
      const int wait_tile = rescale ? j - 1 : j - PST;
      if (wait_tile >= 0) {
        if (!pv_done(wait_tile)) {
          fail(p.status, abort_flag, 10);
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        if (rescale) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t r[32];
            sm100::tmem_ld32(tO + c * 32, r);
            sm100::tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            sm100::tmem_st32(tO + c * 32, r);
          }
          sm100::tmem_st_wait();
        }
      }
      if (need) {
        m_used = m_new;
        l *= alpha;
      }
      // P = 2^(score - m_used) as bf16, 128-byte-swizzled K-major rows (see the single-head kernel)
      uint8_t* myP = sP + ((j % PST) * 2 + w) * 2 * SUB_BYTES;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};  // one partial sum per 32-column chunk
      const float moff = m_used == -INFINITY ? 0.f : m_used;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint8_t* prow = myP + (c >> 1) * SUB_BYTES + (row >> 3) * 1024 + (row & 7) * 128;
        float& rs = rs4[c];
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float x0 = __uint_as_float(sv[c][v * 8 + 2 * e]), x1 = __uint_as_float(sv[c][v * 8 + 2 * e + 1]);
            const float p0 = x0 == -INFINITY ? 0.f : sm100::ex2_approx(score_log2<CAP>(x0, p) - moff);
            const float p1 = x1 == -INFINITY ? 0.f : sm100::ex2_approx(score_log2<CAP>(x1, p) - moff);
            rs += p0 + p1;
            pk[e] = pack_bf16(p0, p1);
          }
          const int chunk = (c & 1) * 4 + v;
          *(uint4*)(prow + ((chunk ^ (row & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
      l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      sm100::fence_async_shared();  // P (generic-proxy stores) visible to the tensor core
      sm100::tc_fence_before();     // and the O rescale ordered before the next P V
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&pfull[2 * w + (j & 1)]);
    }
    if (ok) {
      if (pv_done(n - 1)) {
        sm100::tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        __nv_bfloat16* dst = p.out + (((long long)b * p.T + rq) * p.Hq + h0 + w) * D;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          sm100::tmem_ld32(tO + c * 32, r);
          sm100::tmem_ld_wait();
          if (rq < p.T) {
#pragma unroll
            for (int v = 0; v < 4; ++v)
              *(uint4*)(dst + c * 32 + v * 8) =
                  make_uint4(pack_bf16(__uint_as_float(r[v * 8 + 0]) * inv, __uint_as_float(r[v * 8 + 1]) * inv),
                             pack_bf16(__uint_as_float(r[v * 8 + 2]) * inv, __uint_as_float(r[v * 8 + 3]) * inv),
                             pack_bf16(__uint_as_float(r[v * 8 + 4]) * inv, __uint_as_float(r[v * 8 + 5]) * inv),
                             pack_bf16(__uint_as_float(r[v * 8 + 6]) * inv, __uint_as_float(r[v * 8 + 7]) * inv));
          }
        }
        sm100::tc_fence_before();
        if (p.lse && rq < p.T)
          p.lse[((long long)b * p.Hq + h0 + w) * p.T + rq] = l > 0.f ? (m_used + log2f(l)) * LN2 : -INFINITY;
      } else {
        fail(p.status, abort_flag, 11);
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

// [B][T][H * D] bf16 viewed as a 3-D map (columns, tokens, batch); box = 64 columns x 128 tokens x 1.
// Rows past T read as zeros, so a tile never spills into the next sequence.
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

template <int D, int DV>
static cudaError_t launch(const void* q, const void* k, const void* v, const Params& p, cudaStream_t s) {
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, q, p.B, p.T, p.Hq * D) || !make_map(&mk, k, p.B, p.T, p.Hkv * D) ||
      !make_map(&mv, v, p.B, p.T, p.Hkv * DV))
    return cudaErrorInvalidResourceHandle;
  auto kern = p.cap_log2 > 0.f ? fmha_fwd_kernel<D, DV, true> : fmha_fwd_kernel<D, DV, false>;
  constexpr int smem = smem_request<D, DV>();
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  (void)cudaGetLastError();
  const dim3 grid((p.T + BQ - 1) / BQ, p.Hq, p.B);
  kern<<<grid, 192, smem, s>>>(mq, mk, mv, p);
  return cudaGetLastError();
}

template <int D>
static cudaError_t launch_pair(const void* q, const void* k, const void* v, const Params& p, cudaStream_t s) {
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, q, p.B, p.T, p.Hq * D) || !make_map(&mk, k, p.B, p.T, p.Hkv * D) ||
      !make_map(&mv, v, p.B, p.T, p.Hkv * D))
    return cudaErrorInvalidResourceHandle;
  auto kern = p.cap_log2 > 0.f ? fmha_fwd_pair_kernel<D, true> : fmha_fwd_pair_kernel<D, false>;
  constexpr int smem = PairLayout<D>::BYTES + 1024;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  (void)cudaGetLastError();
  const dim3 grid((p.T + BQ - 1) / BQ, p.Hq / 2, p.B);
  kern<<<grid, PAIR_THREADS, smem, s>>>(mq, mk, mv, p);
  return cudaGetLastError();
}

}  // namespace fmha

// RLB_FMHA_SINGLE=1 keeps every shape on the one-head-per-CTA kernel (A/B measurements).
static bool rlb_fmha_single_head_only() {
  static const int v = [] {
    const char* e = getenv("RLB_FMHA_SINGLE");
    return e != nullptr && e[0] == '1' ? 1 : 0;
  }();
  return v != 0;
}

// q [B][T][Hq][D], k [B][T][Hkv][D], v [B][T][Hkv][DV], out [B][T][Hq][DV] (bf16, contiguous); lse
// [B][Hq][T] fp32 or null.  (D, DV) = (64, 64), (128, 128) or (192, 128).  window > 0: sliding window;
// softcap > 0: tanh logit cap.
cudaError_t rlb_fmha_fwd(const void* q, const void* k, const void* v, void* out, float* lse, int B, int T, int Hq,
                         int Hkv, int D, int DV, int causal, float scale, int window, float softcap, int* status,
                         cudaStream_t s) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  if (window < 0 || softcap < 0.f) return cudaErrorInvalidValue;
  const bool shape_ok = (D == 64 && DV == 64) || (D == 128 && DV == 128) || (D == 192 && DV == 128);
  if (!shape_ok || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Hq > 65535 || B > 65535) return cudaErrorInvalidValue;
  if ((((uintptr_t)q) | ((uintptr_t)k) | ((uintptr_t)v) | ((uintptr_t)out)) & 15) return cudaErrorInvalidDevicePointer;
  fmha::Params p{};
  p.out = (__nv_bfloat16*)out;
  p.lse = lse;
  p.B = B;
  p.T = T;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  p.window = window;
  p.cap_in = softcap > 0.f ? scale / softcap : 0.f;
  p.cap_log2 = softcap > 0.f ? softcap * 1.4426950408889634f : 0.f;
  p.status = status;
  // grouped heads in pairs (even group size, d_qk == d_v): two heads per CTA share each K / V tile
  if (D == DV && D != 192 && (Hq / Hkv) % 2 == 0 && !rlb_fmha_single_head_only())
    return D == 128 ? fmha::launch_pair<128>(q, k, v, p, s) : fmha::launch_pair<64>(q, k, v, p, s);
  if (D == 192) return fmha::launch<192, 128>(q, k, v, p, s);
  return D == 128 ? fmha::launch<128, 128>(q, k, v, p, s) : fmha::launch<64, 64>(q, k, v, p, s);
}
