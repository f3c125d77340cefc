// Persistent tcgen05 GEMM for sm_100a:  C[M, N] = A[M, K] * B[N, K]^T  (bf16 in, fp32 accumulate).
//
// Operand layouts (template flags):
//   A_MN = 0: A stored [M][K] (K contiguous)      A_MN = 1: A stored [K][M] (M contiguous)
//   B_MN = 0: B stored [N][K] (K contiguous)      B_MN = 1: B stored [K][N] (N contiguous)
// which covers a linear layer's forward (x W^T: 0/0), input gradient
// (dy W: 0/1) and weight gradient (dy^T x: 1/1) without any transposes.
//
// Structure (one CTA per SM, 192 threads):
//   warp 0      TMA producer: fills a 4-stage shared-memory ring (A 128x64, B 256x64
//               bf16 tiles, 128-B swizzle), completion counted on mbarriers.
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators) and one
//               elected thread issues tcgen05.mma (M=128, N=256, K=16) per 16-wide
//               K step; tcgen05.commit releases smem stages and publishes finished
//               accumulators.
//   warps 2-5   epilogue: tcgen05.ld the accumulator (each warp owns its 32-lane
//               TMEM quarter), convert, store to global; then hand the TMEM buffer
//               back so the next tile's MMAs overlap this tile's epilogue.
// Tiles are visited in M-grouped order so a wave of CTAs shares B tiles in L2.
// Every mbarrier wait is bounded; on timeout the kernel records an error in
// `status`, stops all roles, frees its TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "sm100.cuh"
#include "tmap.h"

namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, UMMA_K = 16;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 16;
constexpr uint32_t WAIT_LIMIT = 1u << 26;  // polls before a wait is declared dead (seconds)
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;

enum Epi : int { kStoreBF16 = 0, kStoreF32 = 1, kAccumF32 = 2, kAllReduceBF16 = 3 };

__device__ __forceinline__ int ld_acquire_sys_i32(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys_i32(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint4 ld_volatile_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

constexpr unsigned long long AR_WAIT_NS = 20ull * 1000 * 1000 * 1000;  // a peer's tile may take this long

// Barrier over the four epilogue warps with a bounded wait (a hardware named barrier would wait forever
// if one warp had left the tile loop on an abort): every warp adds one to a shared counter and waits
// until it reaches the warp's running target.  Returns false (after recording the failure) on timeout.
__device__ __forceinline__ bool epilogue_sync(volatile int* ctr, int& target, int* status, volatile int* abort_flag,
                                              int lane) {
  target += 4;
  __syncwarp();
  int ok = 1;
  if (lane == 0) {
    __threadfence();
    atomicAdd((int*)ctr, 1);
    long long polls = 0;
    while (*ctr < target) {
      if (++polls > (long long)(AR_WAIT_NS / 32)) {
        ok = 0;
        *abort_flag = 1;
        if (status) atomicCAS(status, 0, 1 | (6 << 8));
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

struct Params {
  int M, N, K;
  void* C;
  long long ldc;
  float alpha;
  int* status;
  // grouped problems (one launch for every expert of an MoE layer)
  int mode;               // kPlain, kGroupM or kGroupK
  const int* tile_group;  // kGroupM: group of each BM-row tile of A and C (-1: tile unused, skipped)
  int b_group_rows;       // kGroupM: rows of B's tensor map per group (N if B is [N][K], K if [K][N])
  const int* k_begin;     // kGroupK: first reduction row of each group
  const int* k_len;       // kGroupK: reduction rows of each group (a multiple of BK; 0 gives a zero tile)
  int groups;             // kGroupK: number of groups; group g's C starts at C + g * M * ldc
  // kAllReduceBF16 epilogue (tensor-parallel row-parallel output): this launch's slot of every rank's
  // bf16 partial buffer ([M][N], ld N) and flag array (int32 [tiles][world]); all ranks run the same
  // launch sequence with the same shapes and grid.
  unsigned long long ar_part[8];
  unsigned long long ar_flag[8];
  int ar_world, ar_rank, ar_epoch;
};

// kGroupM: C rows are grouped in BM-row tiles, each tile multiplies with its group's B.
// kGroupK: each group reduces over its own range of rows of A and B (weight gradients per expert).
enum Mode : int { kPlain = 0, kGroupM = 1, kGroupK = 2 };

struct Tile {
  int m0, n0;
  int g;       // group (0 for plain)
  int kfirst;  // first reduction element
  int nk;      // BK steps (0: nothing to multiply)
  bool skip;   // kGroupM tile of unused rows
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& m, int& n);

__device__ __forceinline__ Tile tile_at(const Params& p, int t, int num_m, int num_n, int nk) {
  Tile r{0, 0, 0, 0, nk, false};
  int tm, tn;
  if (p.mode == kGroupK) {
    const int per = num_m * num_n;
    r.g = t / per;
    tile_coords(t % per, num_m, num_n, tm, tn);
    r.kfirst = p.k_begin[r.g];
    r.nk = p.k_len[r.g] / BK;
  } else {
    tile_coords(t, num_m, num_n, tm, tn);
    if (p.mode == kGroupM) {
      r.g = p.tile_group[tm];
      r.skip = r.g < 0;
    }
  }
  r.m0 = tm * BM;
  r.n0 = tn * BN;
  return r;
}

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& m, int& n) {
  const int per_group = GROUP_M * num_n;
  const int g = t / per_group;
  const int first_m = g * GROUP_M;
  const int gsize = min(num_m - first_m, GROUP_M);
  const int r = t % per_group;
  m = first_m + r % gsize;
  n = r / gsize;
}

__device__ __forceinline__ void fail(int* status, volatile int* abort_flag, int where) {
  *abort_flag = 1;
  if (status) atomicCAS(status, 0, 1 | (where << 8));
}

template <int A_MN, int B_MN, int EPI>
__global__ void __launch_bounds__(192, 1) gemm_kernel(const __grid_constant__ CUtensorMap tma_a,
                                                      const __grid_constant__ CUtensorMap tma_b, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = (uint64_t*)(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = (uint32_t*)(tempty + 2);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  volatile int* ep_ctr = abort_flag + 1;  // epilogue-warp barrier counter (all-reduce epilogue)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (p.M + BM - 1) / BM, num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n * (p.mode == kGroupK ? p.groups : 1);
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&tfull[b], 1);
      sm100::mbar_init(&tempty[b], 4);
    }
    *abort_flag = 0;
    *ep_ctr = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tensormap(&tma_a);
    sm100::prefetch_tensormap(&tma_b);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        const Tile tl = tile_at(p, t, num_m, num_n, nk);
        if (tl.skip) continue;
        const int m0 = tl.m0;
        // B rows of this tile's group: along N for [N][K] storage, along K for [K][N]
        const int n0 = tl.n0 + (p.mode == kGroupM && !B_MN ? tl.g * p.b_group_rows : 0);
        const int kb_off = (p.mode == kGroupM && B_MN) ? tl.g * p.b_group_rows : 0;
        for (int kb = 0; kb < tl.nk; ++kb) {
          if (!sm100::mbar_wait_bounded(&empty[stage], phase ^ 1, WAIT_LIMIT)) {
            fail(p.status, abort_flag, 1);
            break;
          }
          // innermost (x) coordinates of the loads below: K for K-major operands, M / N for MN-major ones
          if (!RLB_TMA_X_OK(A_MN ? m0 : tl.kfirst + kb * BK) || !RLB_TMA_X_OK(B_MN ? n0 : tl.kfirst + kb * BK)) {
            fail(p.status, abort_flag, 7);
            break;
          }
          sm100::mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          uint8_t* a = sA + stage * A_BYTES;
          uint8_t* b = sB + stage * B_BYTES;
          const int k0 = tl.kfirst + kb * BK;
          if (A_MN) {
#pragma unroll
            for (int h = 0; h < BM / 64; ++h) sm100::tma_load_2d(a + h * (BK * 128), &tma_a, &full[stage], m0 + 64 * h, k0);
          } else {
            sm100::tma_load_2d(a, &tma_a, &full[stage], k0, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int h = 0; h < BN / 64; ++h)
              sm100::tma_load_2d(b + h * (BK * 128), &tma_b, &full[stage], n0 + 64 * h, k0 + kb_off);
          } else {
            sm100::tma_load_2d(b, &tma_b, &full[stage], k0, n0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = sm100::idesc_bf16_f32(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        const Tile tl = tile_at(p, t, num_m, num_n, nk);
        if (tl.skip || tl.nk == 0) continue;  // no accumulator used (the epilogue skips or zero-fills)
        if (!sm100::mbar_wait_bounded(&tempty[acc], acc_phase ^ 1, WAIT_LIMIT)) {
          fail(p.status, abort_flag, 2);
          break;
        }
        sm100::tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        bool dead = false;
        for (int kb = 0; kb < tl.nk; ++kb) {
          if (!sm100::mbar_wait_bounded(&full[stage], phase, WAIT_LIMIT)) {
            fail(p.status, abort_flag, 3);
            dead = true;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t a = sm100::smem_u32(sA + stage * A_BYTES);
          const uint32_t b = sm100::smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            // K-major: +32 B per 16-element K step inside the 128-B swizzle row.
            // MN-major: a 16-element K step spans two 8-row (1024-B) atoms.
            const uint64_t ad = A_MN ? sm100::desc_mnmajor_sw128(a + k * 2048, BK * 128)
                                     : sm100::desc_kmajor_sw128(a + k * 32);
            const uint64_t bd = B_MN ? sm100::desc_mnmajor_sw128(b + k * 2048, BK * 128)
                                     : sm100::desc_kmajor_sw128(b + k * 32);
            sm100::mma_f16(d, ad, bd, idesc, (kb | k) != 0);
          }
          sm100::mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (dead) break;
        sm100::mma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    int ep_target = 0;
    for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
      const Tile tl = tile_at(p, t, num_m, num_n, nk);
      if (tl.skip) continue;
      const int m0 = tl.m0, n0 = tl.n0;
      const int row = m0 + q * 32 + lane;
      const long long c_off = p.mode == kGroupK ? (long long)tl.g * p.M * p.ldc : 0;
      if (tl.nk == 0) {
        // empty reduction (an expert without tokens): the product is zero
        if (EPI != kAccumF32 && row < p.M) {
          for (int col = n0; col < n0 + BN && col < p.N; ++col) {
            if (EPI == kStoreBF16) ((__nv_bfloat16*)p.C)[c_off + (long long)row * p.ldc + col] = __float2bfloat16(0.f);
            else ((float*)p.C)[c_off + (long long)row * p.ldc + col] = 0.f;
          }
        }
        continue;
      }
      if (!sm100::mbar_wait_bounded(&tfull[acc], acc_phase, WAIT_LIMIT)) {
        fail(p.status, abort_flag, 4);
        break;
      }
      sm100::tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      if constexpr (EPI == kAllReduceBF16) {
        // pass 1: this rank's bf16 partial of the tile into its own buffer, then the accumulator is free
        __nv_bfloat16* mine = (__nv_bfloat16*)p.ar_part[p.ar_rank];
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          sm100::tmem_ld32(tbase + c * 32, r);
          sm100::tmem_ld_wait();
          const int col0 = n0 + c * 32;
          if (row < p.M && col0 < p.N) {
            __nv_bfloat16* out = mine + (long long)row * p.N + col0;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 pk;
              uint32_t* w = (uint32_t*)&pk;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[v * 8 + 2 * e]) * p.alpha,
                                                         __uint_as_float(r[v * 8 + 2 * e + 1]) * p.alpha);
                w[e] = *(uint32_t*)&h;
              }
              *(uint4*)(out + v * 8) = pk;
            }
          }
        }
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&tempty[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
        // publish the tile to every rank, then wait (bounded) for every rank's partial of it
        if (!epilogue_sync(ep_ctr, ep_target, p.status, abort_flag, lane)) break;
        const int tile = t;
        if (warp == 2 && lane == 0) {
          __threadfence_system();
          for (int r2 = 0; r2 < p.ar_world; ++r2)
            st_release_sys_i32((int*)p.ar_flag[r2] + (long long)tile * p.ar_world + p.ar_rank, p.ar_epoch);
          const int* fl = (const int*)p.ar_flag[p.ar_rank] + (long long)tile * p.ar_world;
          const unsigned long long t0 = now_ns();
          long long polls = 0;
          for (int r2 = 0; r2 < p.ar_world && !*abort_flag; ++r2) {
            while (ld_acquire_sys_i32(fl + r2) < p.ar_epoch) {
              if (++polls > (long long)(AR_WAIT_NS / 32) || now_ns() - t0 > AR_WAIT_NS) {
                fail(p.status, abort_flag, 5);
                break;
              }
              __nanosleep(32);
            }
          }
        }
        if (!epilogue_sync(ep_ctr, ep_target, p.status, abort_flag, lane)) break;
        if (*abort_flag) break;
        // pass 2: sum every rank's bf16 partial in rank order (identical on all ranks), store bf16.  Two
        // 32-column chunks per round: 8 loads of 16 B in flight per rank before the adds (peer loads are
        // NVLink round trips).  Plain loads: the flag acquire and the barrier above order them after
        // the peers' stores, and no address of this tile was read earlier in this launch.
#pragma unroll 1
        for (int c = 0; c < BN / 32; c += 2) {
          const int col0 = n0 + c * 32;
          if (row >= p.M || col0 >= p.N) continue;
          const bool two = col0 + 32 < p.N;
          float sacc[2][32];
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int e = 0; e < 32; ++e) sacc[h][e] = 0.f;
          for (int r2 = 0; r2 < p.ar_world; ++r2) {
            const __nv_bfloat16* src = (const __nv_bfloat16*)p.ar_part[r2] + (long long)row * p.N + col0;
            uint4 raw[2][4];
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int v = 0; v < 4; ++v)
                raw[h][v] = (h == 0 || two) ? *(const uint4*)(src + h * 32 + v * 8) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                const __nv_bfloat162* hv = (const __nv_bfloat162*)&raw[h][v];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 f = __bfloat1622float2(hv[e]);
                  sacc[h][v * 8 + 2 * e] += f.x;
                  sacc[h][v * 8 + 2 * e + 1] += f.y;
                }
              }
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (h == 1 && !two) break;
            __nv_bfloat16* out = (__nv_bfloat16*)p.C + (long long)row * p.ldc + col0 + h * 32;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 pk;
              uint32_t* w = (uint32_t*)&pk;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                __nv_bfloat162 hh = __floats2bfloat162_rn(sacc[h][v * 8 + 2 * e], sacc[h][v * 8 + 2 * e + 1]);
                w[e] = *(uint32_t*)&hh;
              }
              *(uint4*)(out + v * 8) = pk;
            }
          }
        }
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        sm100::tmem_ld32(tbase + c * 32, r);
        sm100::tmem_ld_wait();
        const int col0 = n0 + c * 32;
        if (row < p.M && col0 < p.N) {
          if (EPI == kStoreBF16) {
            __nv_bfloat16* out = (__nv_bfloat16*)p.C + c_off + (long long)row * p.ldc + col0;
            if (col0 + 32 <= p.N) {
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                uint4 pk;
                uint32_t* w = (uint32_t*)&pk;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[v * 8 + 2 * e]) * p.alpha,
                                                           __uint_as_float(r[v * 8 + 2 * e + 1]) * p.alpha);
                  w[e] = *(uint32_t*)&h;
                }
                *(uint4*)(out + v * 8) = pk;
              }
            } else {
#pragma unroll
              for (int e = 0; e < 32; ++e)  // static indexing keeps r[] in registers
                if (col0 + e < p.N) out[e] = __float2bfloat16(__uint_as_float(r[e]) * p.alpha);
            }
          } else {
            float* out = (float*)p.C + c_off + (long long)row * p.ldc + col0;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              if (col0 + e < p.N) {
                const float v = __uint_as_float(r[e]) * p.alpha;
                if (EPI == kAccumF32) out[e] += v;
                else out[e] = v;
              }
            }
          }
        }
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host
using rlb_tmap::EncodeTiledFn;
using rlb_tmap::encode_fn;

// 2-D bf16 tensor map over a row-major matrix [rows][cols] (cols contiguous), box {64 cols, box_rows}.
static bool make_map(CUtensorMap* m, const void* ptr, long long rows, long long cols, long long ld, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int A_MN, int B_MN, int EPI>
static cudaError_t launch(const void* A, long long lda, const void* B, long long ldb, const Params& p, int sms,
                          cudaStream_t s, long long a_rows = 0, long long b_rows = 0) {
  CUtensorMap ma, mb;
  // A_MN: memory [K][M] (box 64 m x 64 k); else [M][K] (box 64 k x 128 m).  a_rows / b_rows override the
  // row extent of a map (grouped operands span every group's rows).
  const long long ar = a_rows ? a_rows : (A_MN ? p.K : p.M);
  const long long br = b_rows ? b_rows : (B_MN ? p.K : p.N);
  const bool ok_a = A_MN ? make_map(&ma, A, ar, p.M, lda, BK) : make_map(&ma, A, ar, p.K, lda, BM);
  const bool ok_b = B_MN ? make_map(&mb, B, br, p.N, ldb, BK) : make_map(&mb, B, br, p.K, ldb, BN);
  if (!ok_a || !ok_b) return cudaErrorInvalidResourceHandle;  // tensor-map encoding rejected the operand
  auto k = gemm_kernel<A_MN, B_MN, EPI>;
  // (per launch: the attribute is cheap to set and the caller may be any host thread)
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  (void)cudaGetLastError();  // drop a stale, non-sticky error left by unrelated calls on this thread
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN) * (p.mode == kGroupK ? p.groups : 1);
  const int grid = tiles < sms ? tiles : sms;
  k<<<grid, 192, SMEM_BYTES, s>>>(ma, mb, p);
  return cudaGetLastError();
}

}  // namespace gemm

// C = alpha * op(A) op(B)^T.  a_mn / b_mn select the operand storage (see top of file);
// epi: 0 = store bf16, 1 = store fp32, 2 = accumulate into fp32.
// Requirements: leading dimensions multiples of 8 elements, 16-B aligned base pointers.
cudaError_t rlb_gemm(int a_mn, int b_mn, int epi, int M, int N, int K, const void* A, long long lda, const void* B,
                     long long ldb, void* C, long long ldc, float alpha, int* status, int sms, cudaStream_t s) {
  using namespace gemm;
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  if ((lda % 8) || (ldb % 8)) return cudaErrorInvalidPitchValue;
  if ((((uintptr_t)A) & 15) || (((uintptr_t)B) & 15)) return cudaErrorInvalidDevicePointer;
  Params p{};
  p.M = M; p.N = N; p.K = K; p.C = C; p.ldc = ldc; p.alpha = alpha; p.status = status; p.mode = kPlain;
#define RLB_GEMM_CASE(AM, BMN, E) \
  if (a_mn == AM && b_mn == BMN && epi == E) return launch<AM, BMN, E>(A, lda, B, ldb, p, sms, s);
  RLB_GEMM_CASE(0, 0, 0)
  RLB_GEMM_CASE(0, 1, 0)
  RLB_GEMM_CASE(1, 1, 0)
  RLB_GEMM_CASE(1, 1, 1)
  RLB_GEMM_CASE(1, 1, 2)
  RLB_GEMM_CASE(0, 0, 1)
  RLB_GEMM_CASE(0, 0, 2)
#undef RLB_GEMM_CASE
  return cudaErrorNotSupported;
}

// Grouped GEMMs for mixture-of-experts layers (one launch per layer and pass).
//   mode 1 (M-grouped): rows of A / C are tokens sorted by expert with every expert's segment padded to a
//     multiple of 128 rows; tile_group[i] is the expert of rows [128 i, 128 i + 128) (-1: unused, skipped).
//     b_mn = 0: B holds groups x [N][K] (x W_e^T, forward);  b_mn = 1: B holds groups x [K][N] (dy W_e,
//     input gradient; K must then be a multiple of 64).  C is [M][N].
//   mode 2 (K-grouped): A [K_total][M] and B [K_total][N] (both MN-major); group g reduces rows
//     [k_begin[g], k_begin[g] + k_len[g]) (k_len a multiple of 64) into C_g = C + g M ldc (weight gradients).
cudaError_t rlb_gemm_grouped(int mode, int b_mn, int epi, int M, int N, int K, const void* A, long long lda,
                             const void* B, long long ldb, void* C, long long ldc, float alpha, int groups,
                             const int* tile_group, const int* k_begin, const int* k_len, long long k_total,
                             int* status, int sms, cudaStream_t s) {
  using namespace gemm;
  if (M <= 0 || N <= 0 || K <= 0 || groups <= 0) return cudaSuccess;
  if ((lda % 8) || (ldb % 8)) return cudaErrorInvalidPitchValue;
  if ((((uintptr_t)A) & 15) || (((uintptr_t)B) & 15)) return cudaErrorInvalidDevicePointer;
  if (mode == kGroupM) {
    if (!tile_group || (b_mn && K % BK)) return cudaErrorInvalidValue;
    Params p{};
    p.M = M; p.N = N; p.K = K; p.C = C; p.ldc = ldc; p.alpha = alpha; p.status = status;
    p.mode = kGroupM; p.tile_group = tile_group; p.b_group_rows = b_mn ? K : N;
    const long long brows = (long long)groups * (b_mn ? K : N);
    if (b_mn == 0 && epi == kStoreBF16) return launch<0, 0, kStoreBF16>(A, lda, B, ldb, p, sms, s, 0, brows);
    if (b_mn == 1 && epi == kStoreBF16) return launch<0, 1, kStoreBF16>(A, lda, B, ldb, p, sms, s, 0, brows);
    return cudaErrorNotSupported;
  }
  if (mode == kGroupK) {
    if (!k_begin || !k_len || k_total <= 0) return cudaErrorInvalidValue;
    Params p{};
    p.M = M; p.N = N; p.K = K; p.C = C; p.ldc = ldc; p.alpha = alpha; p.status = status;
    p.mode = kGroupK; p.k_begin = k_begin; p.k_len = k_len; p.groups = groups;
    if (epi == kStoreBF16) return launch<1, 1, kStoreBF16>(A, lda, B, ldb, p, sms, s, k_total, k_total);
    if (epi == kStoreF32) return launch<1, 1, kStoreF32>(A, lda, B, ldb, p, sms, s, k_total, k_total);
    if (epi == kAccumF32) return launch<1, 1, kAccumF32>(A, lda, B, ldb, p, sms, s, k_total, k_total);
    return cudaErrorNotSupported;
  }
  return cudaErrorInvalidValue;
}

// Tensor-parallel GEMM with the all-reduce in the epilogue: C = sum over ranks of alpha * A_r op(B_r)
// (A [M][K] K-major; C bf16 [M][ldc]).  b_mn = 0: B [N][K] (row-parallel output, x W^T);  b_mn = 1:
// B [K][N] (column-parallel input gradient, dy W).  part / flag: this launch's slot of every rank's
// partial buffer (bf16 [M][N]) and tile-flag array (int32 [tiles][world]); epoch grows by one per use
// of the slot.  N must be a multiple of 32 and every rank must make the same call (same shapes, same
// grid) in the same order.
cudaError_t rlb_gemm_allreduce(int b_mn, int M, int N, int K, const void* A, long long lda, const void* B,
                               long long ldb, void* C, long long ldc, float alpha, const unsigned long long* part,
                               const unsigned long long* flag, int world, int rank, int epoch, int* status,
                               int grid, cudaStream_t s) {
  using namespace gemm;
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  if ((lda % 8) || (ldb % 8) || (N % 32) || (ldc % 8)) return cudaErrorInvalidPitchValue;
  if ((((uintptr_t)A) & 15) || (((uintptr_t)B) & 15) || (((uintptr_t)C) & 15)) return cudaErrorInvalidDevicePointer;
  if (world < 1 || world > 8 || rank < 0 || rank >= world || grid < 1) return cudaErrorInvalidValue;
  Params p{};
  p.M = M; p.N = N; p.K = K; p.C = C; p.ldc = ldc; p.alpha = alpha; p.status = status; p.mode = kPlain;
  for (int r = 0; r < world; ++r) {
    if ((part[r] & 15) || (flag[r] & 3)) return cudaErrorInvalidDevicePointer;
    p.ar_part[r] = part[r];
    p.ar_flag[r] = flag[r];
  }
  p.ar_world = world;
  p.ar_rank = rank;
  p.ar_epoch = epoch;
  if (b_mn) return launch<0, 1, kAllReduceBF16>(A, lda, B, ldb, p, grid, s);
  return launch<0, 0, kAllReduceBF16>(A, lda, B, ldb, p, grid, s);
}
