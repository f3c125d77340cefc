// GEMM with an NF4-quantised weight, dequantised inside the tcgen05 main loop (the QLoRA base layer).
//
//   mode 0 (forward):         C[M][N] = A[M][K] W^T     A = x  bf16 [M][K]
//   mode 1 (input gradient):  C[M][K] = A[M][N] W       A = dy bf16 [M][N]
//
// W is the weight [N][K] stored as NF4 (csrc/nf4.cu, src/forgeline/models/quantization/nf4.py:41-51):
// row-major elements in blocks of 64 with one fp32 absmax each, two 4-bit level indices per byte (high
// nibble = even element).  K must be a multiple of 64, so no block straddles two rows.  The reference
// dequantises the whole weight to a dense tensor on every forward and then calls F.linear
// (src/forgeline/models/quantization/nf4.py:73-75); here the weight crosses HBM at 4.5 bits per element
// and is expanded tile by tile in shared memory.
//
// One CTA per 128 x 256 output tile, 320 threads:
//   warp 0      TMA producer for the A tiles (128 rows x 64 of the reduction dim, 128-B swizzle).
//   warp 1      TMEM owner (one 128 x 256 fp32 accumulator) and MMA issuer (tcgen05.mma, M=128, N=256).
//   warps 2-5   epilogue: tcgen05.ld, convert, store bf16.
//   warps 6-9   dequantisers: each thread expands rows of the stage's NF4 tile through a 16-entry shared
//               table into the 128-B-swizzled bf16 B tile the MMA reads (mode 0: K-major [256][64];
//               mode 1: four MN-major [64][64] boxes), then fence.proxy.async and arrive on the stage.
// A stage is full when the A tile's bytes landed (TMA) and the four dequantiser warps arrived.  Every
// mbarrier wait is bounded (timeout -> status word, every role stops, TMEM freed).  No load uses
// cluster delivery.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "sm100.cuh"
#include "tmap.h"

namespace nf4gemm {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, UMMA_K = 16;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr uint32_t WAIT_LIMIT = 1u << 26;
constexpr int THREADS = 320;

struct Params {
  int mode;       // 0: x W^T, 1: dy W
  int M, N, K;    // W is [N][K]
  const uint8_t* packed;
  const float* absmax;
  const float* table;
  __nv_bfloat16* C;
  int* status;
};

__device__ __forceinline__ void fail(int* status, volatile int* abort_flag, int where) {
  *abort_flag = 1;
  if (status) atomicCAS(status, 0, 1 | ((64 + where) << 8));
}

__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity) {
  return sm100::mbar_wait_bounded(bar, parity, WAIT_LIMIT);
}

// Expand 64 NF4 elements (32 bytes at `src`, one absmax) into row `row` of a 128-B-swizzled [rows][64] box.
__device__ __forceinline__ void expand_row(uint8_t* box, int row, const uint8_t* src, float scale, const float* lut,
                                           bool valid) {
  uint4 raw[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
  if (valid) {
    raw[0] = *reinterpret_cast<const uint4*>(src);
    raw[1] = *reinterpret_cast<const uint4*>(src + 16);
  }
  const uint8_t* bytes = reinterpret_cast<const uint8_t*>(raw);
  uint8_t* base = box + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
  for (int chunk = 0; chunk < 8; ++chunk) {  // 8 elements = 4 bytes per 16-B chunk
    uint4 pk;
    uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint8_t by = bytes[chunk * 4 + e];
      const float hi = valid ? lut[by >> 4] * scale : 0.f, lo = valid ? lut[by & 15] * scale : 0.f;
      __nv_bfloat162 h = __floats2bfloat162_rn(hi, lo);  // element 2i (high nibble) first
      w[e] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(base + ((chunk ^ (row & 7)) << 4)) = pk;
  }
}

__global__ void __launch_bounds__(THREADS, 1) nf4_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = (uint64_t*)(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint32_t* tmem_slot = (uint32_t*)(tfull + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  float* lut = (float*)(tmem_slot + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_out = p.mode == 0 ? p.N : p.K;  // output columns
  const int red = p.mode == 0 ? p.K : p.N;    // reduction length
  const int m0 = blockIdx.y * BM, c0 = blockIdx.x * BN;
  const int nk = (red + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full[s], 1 + 4);  // TMA arrival + four dequantiser warps
      sm100::mbar_init(&empty[s], 1);
    }
    sm100::mbar_init(tfull, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tensormap(&tma_a);
  }
  if (threadIdx.x < 16) lut[threadIdx.x] = p.table[threadIdx.x];
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, BN);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- A producer
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nk && !*abort_flag; ++kb) {
        const int s = kb % STAGES;
        const uint32_t par = (kb / STAGES) & 1;
        if (!wait(&empty[s], par ^ 1)) {
          fail(p.status, abort_flag, 1);
          break;
        }
        if (!RLB_TMA_X_OK(kb * BK)) {
          fail(p.status, abort_flag, 2);
          break;
        }
        sm100::mbar_arrive_expect_tx(&full[s], A_BYTES);
        sm100::tma_load_2d(sA + s * A_BYTES, &tma_a, &full[s], kb * BK, m0);
        issued = kb + 1;
      }
      // own loads land before exit: the last load of each stage (earlier ones were consumed)
      for (int t = 0; t < STAGES && t < issued; ++t) {
        const int kb = issued - 1 - t;
        wait(&full[kb % STAGES], (kb / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = sm100::idesc_bf16_f32(BM, BN, 0, p.mode == 1 ? 1 : 0);
      for (int kb = 0; kb < nk && !*abort_flag; ++kb) {
        const int s = kb % STAGES;
        if (!wait(&full[s], (kb / STAGES) & 1)) {
          fail(p.status, abort_flag, 3);
          break;
        }
        sm100::tc_fence_after();
        const uint32_t a = sm100::smem_u32(sA + s * A_BYTES), b = sm100::smem_u32(sB + s * B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / UMMA_K; ++k) {
          const uint64_t bd = p.mode == 1 ? sm100::desc_mnmajor_sw128(b + k * 2048, BK * 128)
                                          : sm100::desc_kmajor_sw128(b + k * 32);
          sm100::mma_f16(tmem, sm100::desc_kmajor_sw128(a + k * 32), bd, idesc, (kb | k) != 0);
        }
        sm100::mma_commit(&empty[s]);
      }
      sm100::mma_commit(tfull);  // also the drain: fires once every MMA issued here completed
      wait(tfull, 0);
    }
  } else if (warp >= 6) {
    // ---------------------------------------------------------------- dequantisers (128 threads)
    const int t = threadIdx.x - 6 * 32;
    for (int kb = 0; kb < nk; ++kb) {
      if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
      const int s = kb % STAGES;
      if (!__all_sync(0xffffffffu, wait(&empty[s], ((kb / STAGES) & 1) ^ 1))) {
        fail(p.status, abort_flag, 4);
        break;
      }
      uint8_t* bt = sB + s * B_BYTES;
      const int k0 = kb * BK;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int pr = t + 128 * i;
        int wrow, wcol, row;
        uint8_t* box;
        bool valid;
        if (p.mode == 0) {
          // K-major B [256 output columns = rows of W][64 reduction elements]
          row = pr;
          wrow = c0 + pr;
          wcol = k0;
          box = bt;
          valid = wrow < p.N;
        } else {
          // MN-major B: box h holds reduction rows (rows of W) x 64 output columns (columns of W)
          const int h = pr >> 6;
          row = pr & 63;
          wrow = k0 + row;
          wcol = c0 + 64 * h;
          box = bt + h * (BK * 128);
          valid = wrow < p.N && wcol < p.K;
        }
        const long long e = valid ? (long long)wrow * p.K + wcol : 0;
        expand_row(box, row, p.packed + e / 2, valid ? p.absmax[e / 64] : 0.f, lut, valid);
      }
      sm100::fence_async_shared();  // generic-proxy stores visible to the tensor core
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&full[s]);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int q = warp & 3;
    if (__all_sync(0xffffffffu, wait(tfull, 0)) && !*abort_flag) {
      sm100::tc_fence_after();
      const int row = m0 + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        sm100::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, r);
        sm100::tmem_ld_wait();
        const int col0 = c0 + c * 32;
        if (row >= p.M || col0 >= n_out) continue;
        __nv_bfloat16* out = p.C + (long long)row * n_out + col0;
        if (col0 + 32 <= n_out && (n_out & 7) == 0) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 pk;
            uint32_t* w = (uint32_t*)&pk;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[v * 8 + 2 * e]), __uint_as_float(r[v * 8 + 2 * e + 1]));
              w[e] = *(uint32_t*)&h;
            }
            *(uint4*)(out + v * 8) = pk;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (col0 + e < n_out) out[e] = __float2bfloat16(__uint_as_float(r[e]));
        }
      }
      sm100::tc_fence_before();
    } else {
      fail(p.status, abort_flag, 5);
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, BN);
  }
}

using rlb_tmap::EncodeTiledFn;
using rlb_tmap::encode_fn;

}  // namespace nf4gemm

// mode 0: C[M][N] = A[M][K] W^T;  mode 1: C[M][K] = A[M][N] W.  W [N][K] in NF4 (packed, absmax per 64,
// table of the 16 levels); A, C bf16 row-major and contiguous.  K % 64 == 0.
cudaError_t rlb_nf4_gemm(int mode, int M, int N, int K, const void* A, const void* packed, const float* absmax,
                         const float* table, void* C, int* status, cudaStream_t s) {
  using namespace nf4gemm;
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  if ((mode != 0 && mode != 1) || K % 64) return cudaErrorInvalidValue;
  const int red = mode == 0 ? K : N, n_out = mode == 0 ? N : K;
  if (red % 8) return cudaErrorInvalidPitchValue;  // A rows must be 16-byte aligned for TMA
  if ((((uintptr_t)A) & 15) || (((uintptr_t)packed) & 15)) return cudaErrorInvalidDevicePointer;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return cudaErrorInvalidResourceHandle;
  CUtensorMap ma;
  cuuint64_t dims[2] = {(cuuint64_t)red, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)red * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)BM};
  cuuint32_t estr[2] = {1, 1};
  if (enc(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(A), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidResourceHandle;
  Params p{};
  p.mode = mode;
  p.M = M;
  p.N = N;
  p.K = K;
  p.packed = (const uint8_t*)packed;
  p.absmax = absmax;
  p.table = table;
  p.C = (__nv_bfloat16*)C;
  p.status = status;
  cudaError_t e = cudaFuncSetAttribute(nf4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  (void)cudaGetLastError();
  const dim3 grid((n_out + BN - 1) / BN, (M + BM - 1) / BM);
  nf4_gemm_kernel<<<grid, THREADS, SMEM_BYTES, s>>>(ma, p);
  return cudaGetLastError();
}
