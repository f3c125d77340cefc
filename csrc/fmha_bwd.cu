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

namespace fmha_bwd {

constexpr int BQ = 128, BKV = 128;
constexpr int SUB_BYTES = 128 * 64 * 2;
constexpr int TMEM_COLS = 512;
constexpr uint32_t WAIT_LIMIT = 1u << 26;
constexpr float LOG2E = 1.4426950408889634f;

template <int D>
struct Layout {
  static constexpr int DSUB = D / 64;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = K_OFF + DSUB * SUB_BYTES;
  static constexpr int Q_OFF = V_OFF + DSUB * SUB_BYTES;
  static constexpr int DO_OFF = Q_OFF + DSUB * SUB_BYTES;
  static constexpr int PT_OFF = DO_OFF + DSUB * SUB_BYTES;  // P^T  [128 keys][128 queries] bf16
  static constexpr int DS_OFF = PT_OFF + 2 * SUB_BYTES;     // dS^T [128 keys][128 queries] bf16
  static constexpr int BAR_OFF = DS_OFF + 2 * SUB_BYTES;
  static constexpr int BYTES = BAR_OFF + 256;
};
constexpr int SMEM_REQUEST = Layout<128>::BYTES + 1024;  // one CTA per SM (it holds all TMEM columns)

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

// 8 fp32 values -> 8 bf16 in one 16-B chunk of row `row` of a 128-B-swizzled [128][64] box.
__device__ __forceinline__ void store_chunk(uint8_t* box, int row, int chunk, const float* f) {
  uint4 pk;
  uint32_t* w = (uint32_t*)&pk;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    __nv_bfloat162 hh = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
    w[e] = *(uint32_t*)&hh;
  }
  *(uint4*)(box + (row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4)) = pk;
}

// 4 fp32 values added into global memory with one vector reduction (no return value).
__device__ __forceinline__ void red_add_v4(float* dst, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

template <int D, bool CAP>
__global__ void __launch_bounds__(192, 1) fmha_bwd_kernel(const __grid_constant__ CUtensorMap mq,
                                                          const __grid_constant__ CUtensorMap mk,
                                                          const __grid_constant__ CUtensorMap mv,
                                                          const __grid_constant__ CUtensorMap mdo, Params p) {
  using L = Layout<D>;
  constexpr int DSUB = L::DSUB;
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
  uint64_t* qfull = bars + 1;
  uint64_t* qempty = bars + 2;
  uint64_t* sfull = bars + 3;
  uint64_t* sfree = bars + 4;
  uint64_t* pfull = bars + 5;
  uint64_t* dqfull = bars + 6;
  uint64_t* dqfree = bars + 7;
  uint64_t* done = bars + 8;
  uint32_t* tmem_slot = (uint32_t*)(bars + 10);
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
  const int steps = G * nq;  // (query head, query tile) pairs, head-major

  if (threadIdx.x == 0) {
    sm100::mbar_init(kvfull, 1);
    sm100::mbar_init(qfull, 1);
    sm100::mbar_init(qempty, 1);
    sm100::mbar_init(sfull, 1);
    sm100::mbar_init(sfree, 4);
    sm100::mbar_init(pfull, 4);
    sm100::mbar_init(dqfull, 1);
    sm100::mbar_init(dqfree, 4);
    sm100::mbar_init(done, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tensormap(&mq);
    sm100::prefetch_tensormap(&mk);
    sm100::prefetch_tensormap(&mv);
    sm100::prefetch_tensormap(&mdo);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 256 + D;

  if (warp == 0) {
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
        const int h = hk * G + t / nq, q0 = (first_i + t % nq) * BQ;
        if (!wait(qempty, (t & 1) ^ 1)) {
          fail(p.status, abort_flag, 1);
          break;
        }
        sm100::mbar_arrive_expect_tx(qfull, 2 * DSUB * SUB_BYTES);
#pragma unroll
        for (int s = 0; s < DSUB; ++s) {
          sm100::tma_load_3d(sQ + s * SUB_BYTES, &mq, qfull, h * D + 64 * s, q0, b);
          sm100::tma_load_3d(sDO + s * SUB_BYTES, &mdo, qfull, h * D + 64 * s, q0, b);
        }
        issued = t + 1;
      }
      wait(kvfull, 0);  // own loads land before exit
      if (issued > 0) wait(qfull, (issued - 1) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = sm100::idesc_bf16_f32(BKV, BQ, 0, 0);   // keys x queries, K = D
      constexpr uint32_t id_kv = sm100::idesc_bf16_f32(BKV, D, 0, 1);   // keys x D, K = queries
      constexpr uint32_t id_q = sm100::idesc_bf16_f32(BQ, D, 1, 1);     // queries x D, K = keys
      const uint32_t ka = sm100::smem_u32(sK), va = sm100::smem_u32(sV), qa = sm100::smem_u32(sQ),
                     da = sm100::smem_u32(sDO), pa = sm100::smem_u32(sPT), sa = sm100::smem_u32(sDS);
      bool ok = wait(kvfull, 0);
      if (!ok) fail(p.status, abort_flag, 2);
      for (int t = 0; ok && t < steps && !*abort_flag; ++t) {
        const uint32_t par = t & 1;
        if (!wait(qfull, par) || !wait(sfree, par ^ 1) || !wait(dqfree, par ^ 1)) {
          fail(p.status, abort_flag, 3);
          break;
        }
        sm100::tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (uint32_t)(k >> 2) * SUB_BYTES + (uint32_t)(k & 3) * 32;
          sm100::mma_f16(tS, sm100::desc_kmajor_sw128(ka + off), sm100::desc_kmajor_sw128(qa + off), id_s, k > 0);
          sm100::mma_f16(tDP, sm100::desc_kmajor_sw128(va + off), sm100::desc_kmajor_sw128(da + off), id_s, k > 0);
        }
        sm100::mma_commit(sfull);
        if (!wait(pfull, par)) {
          fail(p.status, abort_flag, 4);
          break;
        }
        sm100::tc_fence_after();
#pragma unroll
        for (int k = 0; k < BQ / 16; ++k) {
          // reduction over 16 queries: K-major A rows (P^T, dS^T) step 32 B in a swizzle row; the
          // MN-major B tiles (dO, Q) step 16 rows = 2048 B, their 64-column boxes SUB_BYTES apart
          const uint32_t off = (uint32_t)(k >> 2) * SUB_BYTES + (uint32_t)(k & 3) * 32;
          const uint32_t acc = (t > 0 || k > 0) ? 1u : 0u;
          sm100::mma_f16(tDV, sm100::desc_kmajor_sw128(pa + off), sm100::desc_mnmajor_sw128(da + k * 2048, SUB_BYTES),
                         id_kv, acc);
          sm100::mma_f16(tDK, sm100::desc_kmajor_sw128(sa + off), sm100::desc_mnmajor_sw128(qa + k * 2048, SUB_BYTES),
                         id_kv, acc);
        }
#pragma unroll
        for (int k = 0; k < BKV / 16; ++k) {
          // reduction over 16 keys: dS read MN-major from the dS^T tile, K read MN-major
          sm100::mma_f16(tDP, sm100::desc_mnmajor_sw128(sa + k * 2048, SUB_BYTES),
                         sm100::desc_mnmajor_sw128(ka + k * 2048, SUB_BYTES), id_q, k > 0);
        }
        sm100::mma_commit(qempty);
        sm100::mma_commit(dqfull);
      }
      sm100::mma_commit(done);  // also the drain: every MMA issued here has completed when it fires
      wait(done, 0);
    }
  } else {
    // ------------------------------------------------------------------ compute warps 2..5
    const int qq = warp & 3;
    const int row = qq * 32 + lane;  // key row (S^T, dP^T, dV, dK) or query row (dQ) of the tile
    const int key = kv0 + row;
    const uint32_t lanes = (uint32_t)(qq * 32) << 16;
    bool ok = true;
    for (int t = 0; t < steps; ++t) {
      if (__any_sync(0xffffffffu, *abort_flag != 0)) {
        ok = false;
        break;
      }
      const int h = hk * G + t / nq, qi = first_i + t % nq, q0 = qi * BQ;
      const uint32_t par = t & 1;
      if (!wait_warp(sfull, par)) {
        fail(p.status, abort_flag, 5);
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const float* lse = p.lse + ((long long)b * p.Hq + h) * p.T;
      const float* delta = p.delta + ((long long)b * p.Hq + h) * p.T;
      const bool masked = (p.causal && qi == j) || (q0 + BQ > p.T) || (kv0 + BKV > p.T) ||
                          (p.window > 0 && q0 + BQ - 1 - kv0 >= p.window);
#pragma unroll 1
      for (int c = 0; c < BQ / 32; ++c) {
        uint32_t rs[32], rd[32];
        sm100::tmem_ld32(tS + lanes + c * 32, rs);
        sm100::tmem_ld32(tDP + lanes + c * 32, rd);
        sm100::tmem_ld_wait();
        uint8_t* pbox = sPT + (c >> 1) * SUB_BYTES;
        uint8_t* dbox = sDS + (c >> 1) * SUB_BYTES;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          float pf[8], df[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int q = q0 + c * 32 + v * 8 + e;
            const bool valid = !masked || (q < p.T && key < p.T && (!p.causal || q >= key) &&
                                           (p.window <= 0 || q - key < p.window));
            const float l2 = valid ? __ldg(lse + q) * LOG2E : 0.f;
            const float dl = valid ? __ldg(delta + q) : 0.f;
            const float x = __uint_as_float(rs[v * 8 + e]);
            float pv, dsc;
            if constexpr (CAP) {
              const float th = tanhf(x * p.cap_in);
              pv = valid ? exp2f(fmaf(p.cap_log2, th, -l2)) : 0.f;
              dsc = p.scale * (1.f - th * th);
            } else {
              pv = valid ? exp2f(fmaf(x, p.scale_log2, -l2)) : 0.f;
              dsc = p.scale;
            }
            pf[e] = pv;
            df[e] = pv * (__uint_as_float(rd[v * 8 + e]) - dl) * dsc;
          }
          const int chunk = (c & 1) * 4 + v;
          store_chunk(pbox, row, chunk, pf);
          store_chunk(dbox, row, chunk, df);
        }
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(sfree);
      sm100::fence_async_shared();  // P^T, dS^T visible to the tensor core
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(pfull);
      // dQ_i rows (TMEM lane = query of the tile) into the fp32 accumulator
      if (!wait_warp(dqfull, par)) {
        fail(p.status, abort_flag, 6);
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const int q = q0 + row;
      float* dq = p.dq + (((long long)b * p.T + q) * p.Hq + h) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        sm100::tmem_ld32(tDP + lanes + c * 32, r);
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
    }
    if (ok && steps > 0) {
      if (wait_warp(done, 0)) {
        sm100::tc_fence_after();
        {
          // every lane runs the (warp-collective) TMEM loads; only rows of real keys are stored
          const long long o = (((long long)b * p.T + key) * p.Hkv + hk) * D;
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t rv[32], rk[32];
            sm100::tmem_ld32(tDV + lanes + c * 32, rv);
            sm100::tmem_ld32(tDK + lanes + c * 32, rk);
            sm100::tmem_ld_wait();
            if (key >= p.T) continue;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 pv, pk;
              uint32_t* wv = (uint32_t*)&pv;
              uint32_t* wk = (uint32_t*)&pk;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                __nv_bfloat162 a = __floats2bfloat162_rn(__uint_as_float(rv[v * 8 + 2 * e]),
                                                         __uint_as_float(rv[v * 8 + 2 * e + 1]));
                __nv_bfloat162 bb = __floats2bfloat162_rn(__uint_as_float(rk[v * 8 + 2 * e]),
                                                          __uint_as_float(rk[v * 8 + 2 * e + 1]));
                wv[e] = *(uint32_t*)&a;
                wk[e] = *(uint32_t*)&bb;
              }
              *(uint4*)(p.dv + o + c * 32 + v * 8) = pv;
              *(uint4*)(p.dk + o + c * 32 + v * 8) = pk;
            }
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
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)ptr;
  }
  return fn;
}

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
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_REQUEST);
  if (e != cudaSuccess) return e;
  (void)cudaGetLastError();
  const dim3 grid((p.T + BKV - 1) / BKV, p.Hkv, p.B);
  kern<<<grid, 192, SMEM_REQUEST, s>>>(mq, mk, mv, mdo, p);
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
