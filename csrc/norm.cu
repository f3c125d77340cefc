// RMSNorm forward / backward, optionally fused with the residual add that
// precedes it in a pre-norm block:
//   h = x (+ delta);  y = h * rsqrt(mean(h^2) + eps) * w
// Widths that are multiples of 256 (the model widths) use one block per row and
// one 16-byte vector per thread (few registers, full occupancy); other widths use
// one warp per row with NV vectors per lane.  Rows are read from HBM once per pass;
// the weight gradient is summed per block, then across blocks in a fixed order.
// Semantics follow src/forgeline/models/transformer/norm.py:9-17 (fp32 statistics).
#include "common.cuh"

namespace rlb {

template <int NV>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ delta,
    const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ h_out,
    __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out, long long rows, int dim, float eps) {
  const int lane = threadIdx.x & 31;
  const long long warps_total = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
       row += warps_total) {
    const __nv_bfloat16* xr = x + row * dim;
    float v[NV][8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j) * 8;
      if (c < dim) {
        unpack8(ldg8(xr + c), v[j]);
        if (delta != nullptr) {
          float d[8];
          unpack8(ldg8(delta + row * dim + c), d);
#pragma unroll
          for (int k = 0; k < 8; ++k) v[j][k] += d[k];
          // the residual stream is kept in bf16: round before the statistics so
          // that forward and backward see the same h
          bf16x8 hv = pack8(v[j]);
          stg8(h_out + row * dim + c, hv);
          unpack8(hv, v[j]);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) ss += v[j][k] * v[j][k];
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)dim + eps);
    if (lane == 0 && rstd_out != nullptr) rstd_out[row] = r;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j) * 8;
      if (c < dim) {
        float wf[8], o[8];
        unpack8(ldg8(w + c), wf);
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = v[j][k] * r * wf[k];
        stg8(y + row * dim + c, pack8(o));
      }
    }
  }
}

// dx = r * (dxh - xh * mean(dxh * xh)),  dxh = dy * w,  xh = h * r
// dx additionally gets `dres` (gradient arriving on the residual stream).
// Per-block partial sums of dw = sum_rows dy * xh go to dw_part[blockIdx.x].
template <int NV>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ w,
    const float* __restrict__ rstd, const __nv_bfloat16* __restrict__ dy,
    const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx,
    float* __restrict__ dw_part, long long rows, int dim) {
  extern __shared__ float smem[];  // [8 warps][dim]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float acc[NV][8];
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[j][k] = 0.f;
  float wf[NV][8];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = (lane + 32 * j) * 8;
    if (c < dim) unpack8(ldg8(w + c), wf[j]);
  }
  const long long warps_total = (long long)gridDim.x * 8;
  for (long long row = (long long)blockIdx.x * 8 + warp; row < rows; row += warps_total) {
    const float r = rstd[row];
    float xh[NV][8], g[NV][8];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j) * 8;
      if (c < dim) {
        unpack8(ldg8(h + row * dim + c), xh[j]);
        unpack8(ldg8(dy + row * dim + c), g[j]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          xh[j][k] *= r;
          acc[j][k] += g[j][k] * xh[j][k];
          g[j][k] *= wf[j][k];
          dot += g[j][k] * xh[j][k];
        }
      }
    }
    dot = warp_sum(dot) / (float)dim;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j) * 8;
      if (c < dim) {
        float o[8];
        float rr[8];
        if (dres != nullptr) unpack8(ldg8(dres + row * dim + c), rr);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          o[k] = r * (g[j][k] - xh[j][k] * dot);
          if (dres != nullptr) o[k] += rr[k];
        }
        stg8(dx + row * dim + c, pack8(o));
      }
    }
  }
  // reduce the 8 warps' dw partials through shared memory
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = (lane + 32 * j) * 8;
    if (c < dim)
#pragma unroll
      for (int k = 0; k < 8; ++k) smem[warp * dim + c + k] = acc[j][k];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) s += smem[q * dim + c];
    dw_part[(long long)blockIdx.x * dim + c] = s;
  }
}

// ---------------------------------------------------------------------------
// Wide rows (dim % 256 == 0, dim <= 8192): a block owns R rows at a time, one
// 16-byte vector per thread per row (blockDim = dim / 8).  All R rows' loads are
// issued before the single block reduction, so each warp keeps R x 2 x 16 B in
// flight instead of stalling on one row per barrier.
constexpr int kRows = 4;

template <int R>
RLB_DEVICE void rows_sum(float (&v)[R], float* red) {  // red: [R][32]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float t = warp_sum(v[r]);
    if (lane == 0) red[r * 32 + warp] = t;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float t = 0.f;
    for (int i = 0; i < nw; ++i) t += red[r * 32 + i];
    v[r] = t;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(1024) rmsnorm_fwd_wide(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ delta,
                                 const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ h_out,
                                 __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out, long long rows, int dim,
                                 float eps) {
  __shared__ float red[kRows * 32];
  const int c = threadIdx.x * 8;
  float wf[8];
  unpack8(ldg8(w + c), wf);
  for (long long row0 = (long long)blockIdx.x * kRows; row0 < rows; row0 += (long long)gridDim.x * kRows) {
    float v[kRows][8], ss[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const long long row = row0 + r;
      ss[r] = 0.f;
      if (row < rows) {
        unpack8(ldg8(x + row * dim + c), v[r]);
        if (delta != nullptr) {
          float d[8];
          unpack8(ldg8(delta + row * dim + c), d);
#pragma unroll
          for (int k = 0; k < 8; ++k) v[r][k] += d[k];
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const long long row = row0 + r;
      if (row < rows) {
        if (delta != nullptr) {
          bf16x8 hv = pack8(v[r]);
          stg8(h_out + row * dim + c, hv);
          unpack8(hv, v[r]);  // statistics of the rounded residual stream
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) ss[r] += v[r][k] * v[r][k];
      }
    }
    rows_sum<kRows>(ss, red);
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const long long row = row0 + r;
      if (row >= rows) continue;
      const float rs = rsqrtf(ss[r] / (float)dim + eps);
      if (threadIdx.x == 0 && rstd_out) rstd_out[row] = rs;
      float o[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = v[r][k] * rs * wf[k];
      stg8(y + row * dim + c, pack8(o));
    }
  }
}

constexpr int kRowsBwd = 2;  // the backward keeps 3 input vectors per row live

// MAXT: the largest block this instantiation is launched with (dim / 8 threads).  Up to dim 4096 the
// 512-thread bound leaves ptxas the registers it wants; dim 8192 needs 1024 threads, which caps them at 64.
template <int MAXT>
__global__ void __launch_bounds__(MAXT) rmsnorm_bwd_wide(const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ w,
                                 const float* __restrict__ rstd, const __nv_bfloat16* __restrict__ dy,
                                 const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx,
                                 float* __restrict__ dw_part, long long rows, int dim) {
  constexpr int kRows = kRowsBwd;
  __shared__ float red[kRows * 32];
  const int c = threadIdx.x * 8;
  float wf[8], acc[8];
  unpack8(ldg8(w + c), wf);
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = 0.f;
  const long long stride = (long long)gridDim.x * kRows;
  // raw operands of the rows in flight: the next rows' loads are issued before this iteration's reduction
  bf16x8 nh[kRows], ng[kRows], nr[kRows];
  float nrs[kRows];
  auto issue = [&](long long r0) {
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const long long row = r0 + r;
      if (row < rows) {
        nrs[r] = rstd[row];
        nh[r] = ldg8(h + row * dim + c);
        ng[r] = ldg8(dy + row * dim + c);
        if (dres != nullptr) nr[r] = ldg8(dres + row * dim + c);
      }
    }
  };
  long long row0 = (long long)blockIdx.x * kRows;
  issue(row0);
  for (; row0 < rows; row0 += stride) {
    float xh[kRows][8], g[kRows][8], dot[kRows], rs[kRows];
    bf16x8 rres[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      dot[r] = 0.f;
      rs[r] = 0.f;
      if (row0 + r < rows) {
        rs[r] = nrs[r];
        unpack8(nh[r], xh[r]);
        unpack8(ng[r], g[r]);
        rres[r] = nr[r];
      }
    }
    if (row0 + stride < rows) issue(row0 + stride);
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      if (row0 + r < rows) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          xh[r][k] *= rs[r];
          acc[k] += g[r][k] * xh[r][k];
          g[r][k] *= wf[k];
          dot[r] += g[r][k] * xh[r][k];
        }
      }
    }
    rows_sum<kRows>(dot, red);
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const long long row = row0 + r;
      if (row >= rows) continue;
      const float m = dot[r] / (float)dim;
      float o[8];
      if (dres != nullptr) {
        float rr[8];
        unpack8(rres[r], rr);
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = rs[r] * (g[r][k] - xh[r][k] * m) + rr[k];
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = rs[r] * (g[r][k] - xh[r][k] * m);
      }
      stg8(dx + row * dim + c, pack8(o));
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) dw_part[(long long)blockIdx.x * dim + c + k] = acc[k];
}

// Column sums of a [parts, dim] fp32 matrix -> dw (bf16 or fp32), fixed order:
// block = 32 columns x 8 row-slices, each slice strides over the parts, then the
// 8 slice sums are added in shared memory.

__global__ void colsum_kernel(const float* __restrict__ part, int parts, int dim, float* __restrict__ out_f32,
                              __nv_bfloat16* __restrict__ out_bf16) {
  __shared__ float tile[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + tx;
  float s = 0.f;
  if (c < dim)
    for (int p = ty; p < parts; p += 8) s += part[(long long)p * dim + c];
  tile[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && c < dim) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += tile[i][tx];
    if (out_f32) out_f32[c] = t;
    if (out_bf16) out_bf16[c] = __float2bfloat16(t);
  }
}

// one thread per 8 columns, up to 1024 threads (dim 8192): the wide kernels are bounded to 64 registers
static bool wide_ok(int dim) { return dim % 256 == 0 && dim <= 8192; }

static int wide_grid(long long rows, int sms) {
  const long long want = (rows + kRowsBwd - 1) / kRowsBwd;
  const long long cap = (long long)sms * 8;
  return (int)(want < cap ? (want < 1 ? 1 : want) : cap);
}

// The wide backward with `grid` blocks of dim / 8 threads (dim a multiple of 256, at most 8192), partial
// column sums of dw into dw_part[grid][dim].  Also used by the allocation-free entry point (norm_noalloc.cu).
void launch_rmsnorm_bwd_wide(int grid, const __nv_bfloat16* h, const __nv_bfloat16* w, const float* rstd,
                             const __nv_bfloat16* dy, const __nv_bfloat16* dres, __nv_bfloat16* dx, float* dw_part,
                             long long rows, int dim, cudaStream_t s) {
  auto k = dim / 8 > 512 ? rmsnorm_bwd_wide<1024> : rmsnorm_bwd_wide<512>;
  k<<<grid, dim / 8, 0, s>>>(h, w, rstd, dy, dres, dx, dw_part, rows, dim);
}

static int pick_grid(long long rows, int sms) {
  long long want = (rows + 7) / 8;
  long long cap = (long long)sms * 8;
  return (int)(want < cap ? want : cap);
}

#define RLB_NV_DISPATCH(dim, KERNEL_CALL)           \
  do {                                              \
    if ((dim) <= 256) { constexpr int NV = 1; KERNEL_CALL; }        \
    else if ((dim) <= 512) { constexpr int NV = 2; KERNEL_CALL; }   \
    else if ((dim) <= 1024) { constexpr int NV = 4; KERNEL_CALL; }  \
    else { return cudaErrorInvalidValue; }          \
  } while (0)

}  // namespace rlb

using namespace rlb;

// Launchers (return cudaError_t so bindings can raise).
cudaError_t rlb_rmsnorm_fwd(const void* x, const void* delta, const void* w, void* h_out, void* y, float* rstd,
                            long long rows, int dim, float eps, int sms, cudaStream_t s) {
  if (dim % 8 != 0) return cudaErrorInvalidValue;
  if (wide_ok(dim)) {
    rmsnorm_fwd_wide<<<wide_grid(rows, sms), dim / 8, 0, s>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)delta, (const __nv_bfloat16*)w, (__nv_bfloat16*)h_out,
        (__nv_bfloat16*)y, rstd, rows, dim, eps);
    return cudaGetLastError();
  }
  const int grid = pick_grid(rows, sms);
  RLB_NV_DISPATCH(dim, (rmsnorm_fwd_kernel<NV><<<grid, 256, 0, s>>>(
                           (const __nv_bfloat16*)x, (const __nv_bfloat16*)delta, (const __nv_bfloat16*)w,
                           (__nv_bfloat16*)h_out, (__nv_bfloat16*)y, rstd, rows, dim, eps)));
  return cudaGetLastError();
}

// dw_part must hold grid*dim floats where grid = rlb_rmsnorm_bwd_grid(rows, sms).
int rlb_rmsnorm_bwd_grid(long long rows, int sms) { return pick_grid(rows, sms) < 1 ? 1 : pick_grid(rows, sms); }
int rlb_rmsnorm_bwd_parts(long long rows, int dim, int sms) {
  return wide_ok(dim) ? wide_grid(rows, sms) : rlb_rmsnorm_bwd_grid(rows, sms);
}

cudaError_t rlb_rmsnorm_bwd(const void* h, const void* w, const float* rstd, const void* dy, const void* dres,
                            void* dx, float* dw_part, void* dw_out, int dw_is_f32, long long rows, int dim, int sms,
                            cudaStream_t s) {
  if (dim % 8 != 0) return cudaErrorInvalidValue;
  if (wide_ok(dim)) {
    const int g = wide_grid(rows, sms);
    launch_rmsnorm_bwd_wide(g, (const __nv_bfloat16*)h, (const __nv_bfloat16*)w, rstd, (const __nv_bfloat16*)dy,
                            (const __nv_bfloat16*)dres, (__nv_bfloat16*)dx, dw_part, rows, dim, s);
    colsum_kernel<<<ceil_div(dim, 32), 256, 0, s>>>(dw_part, g, dim, dw_is_f32 ? (float*)dw_out : nullptr,
                                                    dw_is_f32 ? nullptr : (__nv_bfloat16*)dw_out);
    return cudaGetLastError();
  }
  const int grid = rlb_rmsnorm_bwd_grid(rows, sms);
  const size_t smem = (size_t)8 * dim * sizeof(float);
  RLB_NV_DISPATCH(dim, ({
                    auto k = rmsnorm_bwd_kernel<NV>;
                    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
                    k<<<grid, 256, smem, s>>>((const __nv_bfloat16*)h, (const __nv_bfloat16*)w, rstd,
                                              (const __nv_bfloat16*)dy, (const __nv_bfloat16*)dres,
                                              (__nv_bfloat16*)dx, dw_part, rows, dim);
                  }));
  colsum_kernel<<<ceil_div(dim, 32), 256, 0, s>>>(dw_part, grid, dim, dw_is_f32 ? (float*)dw_out : nullptr,
                                                   dw_is_f32 ? nullptr : (__nv_bfloat16*)dw_out);
  return cudaGetLastError();
}
