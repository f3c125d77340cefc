// Rotary position embedding (rotate-half convention) fused with the head split
// of the fused QKV projection output.
//
//   qkv [B, T, (Hq + 2*Hkv) * D]  --fwd-->  q [B,Hq,T,D], k [B,Hkv,T,D], v [B,Hkv,T,D]
//   (or [B,T,H,D] when heads_major == 0)
//   backward applies the transposed rotation and re-interleaves into dqkv.
//
// Pair (i, i + D/2) is rotated by angle pos * inv_freq[i]:
//   o_i = x_i c - x_{i+h} s,   o_{i+h} = x_{i+h} c + x_i s
// which is x*cos + rotate_half(x)*sin of src/forgeline/models/attention/rotary.py:68-76.
// The cos/sin table is [table_rows, D/2] fp32 built on the host from inv_freq
// (base theta, linear or YaRN scaling already folded in).  A position outside
// the table is reported in `status` (kBadIndex) and that pair is passed through
// unrotated instead of reading past the table.
#include "common.cuh"

namespace rlb {

struct RopeArgs {
  const __nv_bfloat16* src;
  __nv_bfloat16* dst;
  const __nv_bfloat16* q_src;  // backward sources
  const __nv_bfloat16* k_src;
  const __nv_bfloat16* v_src;
  __nv_bfloat16* q_dst;        // forward destinations
  __nv_bfloat16* k_dst;
  __nv_bfloat16* v_dst;
  const float* cos_t;
  const float* sin_t;
  const int* positions;        // optional [B*T]
  int B, T, Hq, Hkv, D, pos_offset, heads_major, table_rows;
  long long row_stride;        // elements between consecutive tokens of qkv
  int* status;                 // index errors (first kept)
};

RLB_DEVICE long long head_offset(const RopeArgs& a, int b, int t, int head, int H) {
  // offset of the first element of (b, head, t) in a [B,H,T,D] or [B,T,H,D] tensor
  if (a.heads_major) return (((long long)b * H + head) * a.T + t) * a.D;
  return (((long long)b * a.T + t) * H + head) * a.D;
}

// One thread = 8 consecutive dims of the first half of one (token, head) and
// their 8 partners in the second half.  IT is the index type: 32-bit whenever the
// whole index space (plus one grid stride) fits, so the per-chunk div / mod that
// locate (token, head, chunk) are 32-bit operations; the cos / sin values of the 8
// dims are two 16-byte loads each (the table rows are 16-byte aligned: D/2 % 4 == 0).
template <bool INVERSE, typename IT>
__global__ void rope_qkv_kernel(RopeArgs a) {
  const int half = a.D >> 1;
  const int chunks = half >> 3;
  const int heads = a.Hq + 2 * a.Hkv;
  const IT total = (IT)a.B * a.T * heads * chunks;
  for (IT idx = (IT)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (IT)gridDim.x * blockDim.x) {
    const int c = (int)(idx % chunks);
    const IT r = idx / chunks;
    const int head = (int)(r % heads);
    const IT tok = r / heads;
    const int t = (int)(tok % a.T), b = (int)(tok / a.T);
    const int i0 = c * 8;
    // where this head lives on the split side
    __nv_bfloat16* dptr;
    const __nv_bfloat16* sptr;
    bool rotate = true;
    int H, hl;
    if (head < a.Hq) { H = a.Hq; hl = head; }
    else if (head < a.Hq + a.Hkv) { H = a.Hkv; hl = head - a.Hq; }
    else { H = a.Hkv; hl = head - a.Hq - a.Hkv; rotate = false; }
    const long long split_off = head_offset(a, b, t, hl, H);
    const long long fused_off = (long long)tok * a.row_stride + (long long)head * a.D;
    if (!INVERSE) {
      sptr = a.src + fused_off;
      dptr = (head < a.Hq ? a.q_dst : (head < a.Hq + a.Hkv ? a.k_dst : a.v_dst)) + split_off;
    } else {
      sptr = (head < a.Hq ? a.q_src : (head < a.Hq + a.Hkv ? a.k_src : a.v_src)) + split_off;
      dptr = a.dst + fused_off;
    }
    bf16x8 lo = ldg8(sptr + i0), hi = ldg8(sptr + i0 + half);
    const int pos = rotate ? (a.positions ? a.positions[tok] : t + a.pos_offset) : 0;
    if (rotate && (pos < 0 || pos >= a.table_rows)) {
      report(a.status, kBadIndex);
      rotate = false;
    }
    if (rotate) {
      const float4* ct = reinterpret_cast<const float4*>(a.cos_t + (long long)pos * half + i0);
      const float4* st = reinterpret_cast<const float4*>(a.sin_t + (long long)pos * half + i0);
      const float4 c4[2] = {__ldg(ct), __ldg(ct + 1)}, s4[2] = {__ldg(st), __ldg(st + 1)};
      const float* cs = reinterpret_cast<const float*>(c4);
      const float* sn = reinterpret_cast<const float*>(s4);
      float xl[8], xh[8], ol[8], oh[8];
      unpack8(lo, xl);
      unpack8(hi, xh);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float sk = INVERSE ? -sn[k] : sn[k];
        ol[k] = xl[k] * cs[k] - xh[k] * sk;
        oh[k] = xh[k] * cs[k] + xl[k] * sk;
      }
      lo = pack8(ol);
      hi = pack8(oh);
    }
    stg8(dptr + i0, lo);
    stg8(dptr + i0 + half, hi);
  }
}

static int grid_for(long long work, int sms) {
  long long g = (work + 255) / 256;
  long long cap = (long long)sms * 16;
  return (int)(g < 1 ? 1 : (g < cap ? g : cap));
}

// 32-bit indices when the index space and one grid stride fit in an int
template <bool INVERSE>
static void launch_rope_qkv(const RopeArgs& a, long long work, int sms, cudaStream_t s) {
  const int grid = grid_for(work, sms);
  if (work + (long long)grid * 256 < 2147483647LL)
    rope_qkv_kernel<INVERSE, int><<<grid, 256, 0, s>>>(a);
  else
    rope_qkv_kernel<INVERSE, long long><<<grid, 256, 0, s>>>(a);
}

// In-place rotation of x[b, t, h, 0:D] addressed with explicit strides.
__global__ void rope_inplace_kernel(__nv_bfloat16* x, int B, int T, int H, int D, long long sb, long long st,
                                    long long sh, const float* cos_t, const float* sin_t, const int* positions,
                                    int pos_offset, int inverse, int table_rows, int* status) {
  const int half = D >> 1;
  const long long total = (long long)B * T * H * half;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(idx % half);
    long long r = idx / half;
    const int h = (int)(r % H);
    r /= H;
    const int t = (int)(r % T), b = (int)(r / T);
    const int pos = positions ? positions[(long long)b * T + t] : t + pos_offset;
    if (pos < 0 || pos >= table_rows) {
      if (i == 0) report(status, kBadIndex);
      continue;  // left unrotated
    }
    __nv_bfloat16* p = x + b * sb + t * st + h * sh;
    const float xl = __bfloat162float(p[i]), xh = __bfloat162float(p[i + half]);
    const float cs = cos_t[(long long)pos * half + i];
    const float sn = inverse ? -sin_t[(long long)pos * half + i] : sin_t[(long long)pos * half + i];
    p[i] = __float2bfloat16(xl * cs - xh * sn);
    p[i + half] = __float2bfloat16(xh * cs + xl * sn);
  }
}

}  // namespace rlb

using namespace rlb;

cudaError_t rlb_rope_qkv_fwd(const void* qkv, long long row_stride, void* q, void* k, void* v, const float* cos_t,
                             const float* sin_t, const int* positions, int B, int T, int Hq, int Hkv, int D,
                             int pos_offset, int heads_major, int table_rows, int* status, int sms, cudaStream_t s) {
  if (D % 16 != 0) return cudaErrorInvalidValue;
  RopeArgs a{};
  a.src = (const __nv_bfloat16*)qkv;
  a.q_dst = (__nv_bfloat16*)q;
  a.k_dst = (__nv_bfloat16*)k;
  a.v_dst = (__nv_bfloat16*)v;
  a.cos_t = cos_t;
  a.sin_t = sin_t;
  a.positions = positions;
  a.B = B; a.T = T; a.Hq = Hq; a.Hkv = Hkv; a.D = D; a.pos_offset = pos_offset; a.heads_major = heads_major;
  a.row_stride = row_stride;
  a.table_rows = table_rows;
  a.status = status;
  const long long work = (long long)B * T * (Hq + 2 * Hkv) * (D / 16);
  launch_rope_qkv<false>(a, work, sms, s);
  return cudaGetLastError();
}

cudaError_t rlb_rope_qkv_bwd(const void* dq, const void* dk, const void* dv, void* dqkv, long long row_stride,
                             const float* cos_t, const float* sin_t, const int* positions, int B, int T, int Hq,
                             int Hkv, int D, int pos_offset, int heads_major, int table_rows, int* status, int sms,
                             cudaStream_t s) {
  if (D % 16 != 0) return cudaErrorInvalidValue;
  RopeArgs a{};
  a.q_src = (const __nv_bfloat16*)dq;
  a.k_src = (const __nv_bfloat16*)dk;
  a.v_src = (const __nv_bfloat16*)dv;
  a.dst = (__nv_bfloat16*)dqkv;
  a.cos_t = cos_t;
  a.sin_t = sin_t;
  a.positions = positions;
  a.B = B; a.T = T; a.Hq = Hq; a.Hkv = Hkv; a.D = D; a.pos_offset = pos_offset; a.heads_major = heads_major;
  a.row_stride = row_stride;
  a.table_rows = table_rows;
  a.status = status;
  const long long work = (long long)B * T * (Hq + 2 * Hkv) * (D / 16);
  launch_rope_qkv<true>(a, work, sms, s);
  return cudaGetLastError();
}

cudaError_t rlb_rope_inplace(void* x, int B, int T, int H, int D, long long sb, long long st, long long sh,
                             const float* cos_t, const float* sin_t, const int* positions, int pos_offset,
                             int inverse, int table_rows, int* status, int sms, cudaStream_t s) {
  if (D % 2 != 0) return cudaErrorInvalidValue;
  const long long work = (long long)B * T * H * (D / 2);
  rope_inplace_kernel<<<grid_for(work, sms), 256, 0, s>>>((__nv_bfloat16*)x, B, T, H, D, sb, st, sh, cos_t, sin_t,
                                                         positions, pos_offset, inverse, table_rows, status);
  return cudaGetLastError();
}
