// Communication kernels over NVLink peer memory (every buffer a peer reads is a CUDA-IPC mapping of
// the owner's allocation, or the NVLink multicast address of a torch symmetric buffer):
//
// * fused_rs_kernel: sharded-data-parallel gradient reduce-scatter fused with the fp32 cast, the
//   1/world scale, accumulation and the squared-norm partial.  The reference reduces through torch
//   FSDP's NCCL reduce-scatter (src/forgeline/distributed/strategies.py:100-122) and DDP's
//   per-parameter all-reduce (src/forgeline/training/common/trainer.py:122-139), then casts, averages
//   and clips in separate passes.  Rank r owns elements [r S, (r + 1) S) of every rank's slot; it sums
//   the world copies -- plain peer loads, or one `multimem.ld_reduce` through the multicast address
//   (fp32 accumulation in the switch) -- and writes or adds the fp32 shard gradient.
// * gather_rows_kernel: expert-parallel dispatch / combine, a row gather from the peers' slots
//   straight into the grouped expert GEMM's layout (the reference runs experts in a Python loop on
//   every rank: src/forgeline/models/moe/layer.py:32-38).
// * allgather_pull_kernel: FSDP parameter all-gather by pulls.
// * multimem_bcast_kernel: weight broadcast through NVSwitch multicast (the reference ships full
//   state_dicts through Ray's object store: src/forgeline/orchestration/ray_backend.py:408-417).
//
// Every exchange is "pack into my slot, raise my flag in every rank's flag array (system-scope
// release), one thread waits (bounded) for every peer's flag, then pull".  A wait that runs out sets
// `status` (kTimeout | slot << 8) and the data kernels that follow return without writing, as does
// every later one until the caller clears the status.  Slot reuse is made safe by the callers'
// ordering (rl_project_b200/parallel/fused_comm.py, expert_p2p.py).
#include "common.cuh"

namespace rlb {

RLB_DEVICE int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

RLB_DEVICE void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

RLB_DEVICE unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Thread p raises this rank's flag for `slot` on rank p: flags_p[slot * world + rank] = epoch.
__global__ void signal_peers_kernel(const unsigned long long* __restrict__ flag_ptrs, int world, int rank, int slot,
                                    int epoch) {
  const int p = threadIdx.x;
  if (p >= world) return;
  __threadfence_system();
  int* f = reinterpret_cast<int*>(flag_ptrs[p]) + (long long)slot * world + rank;
  st_release_sys(f, epoch);
}

// Bounded wait by one thread for every peer's flag of `slot` to reach `epoch`.
RLB_DEVICE bool wait_flags(const int* my_flags, int world, int slot, int epoch, unsigned long long limit_ns,
                           int* status) {
  const unsigned long long t0 = globaltimer_ns();
  const long long max_polls = (long long)(limit_ns / 32) + 1024;  // caps the loop even if the timer stalls
  for (int p = 0; p < world; ++p) {
    const int* f = my_flags + (long long)slot * world + p;
    long long polls = 0;
    while (ld_acquire_sys(f) < epoch) {
      if (++polls > max_polls || globaltimer_ns() - t0 > limit_ns) {
        report(status, kTimeout | (slot << 8));
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// 8 bf16 of every rank at one address through the multicast mapping, summed in fp32 by the switch.
RLB_DEVICE void multimem_sum8(const __nv_bfloat16* mc, float* out) {
  uint32_t r0, r1, r2, r3;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "l"(mc)
               : "memory");
  const uint32_t r[4] = {r0, r1, r2, r3};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(r[i] << 16);
    out[2 * i + 1] = __uint_as_float(r[i] & 0xffff0000u);
  }
}

// 16-byte load of a peer's (or this rank's) slot.  The data kernel starts after the wait kernel observed every
// peer's flag, and the slot does not change while the kernel runs, so ordinary loads that the compiler may
// batch freely are enough.
RLB_DEVICE uint4 ld16(const void* p) { return *reinterpret_cast<const uint4*>(p); }

RLB_DEVICE void add8(const uint4& raw, float* acc) {
  float f[8];
  unpack8(*reinterpret_cast<const bf16x8*>(&raw), f);
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] += f[k];
}

// One thread waits (bounded) for every peer's flag; the data kernel that follows in the stream starts only
// once the wait kernel has returned, so no SM is held by spinning CTAs while a peer is still computing.
__global__ void wait_peers_kernel(const int* __restrict__ my_flags, int world, int slot, int epoch,
                                  unsigned long long limit_ns, int* status) {
  if (threadIdx.x == 0) wait_flags(my_flags, world, slot, epoch, limit_ns, status);
}

constexpr int kRsThreads = 256;

// PB peers are loaded together, U vectors per peer: PB * U 16-byte loads in flight per thread before the
// adds (16 for every world size: PB = min(world, 8) rounded up to 2 / 4 / 8, U = 16 / PB).
template <int PB, int U, bool MULTIMEM>
__global__ void __launch_bounds__(kRsThreads) fused_rs_kernel(
    const unsigned long long* __restrict__ buf_ptrs, unsigned long long mc_base, int world, int rank,
    long long shard, float scale, float* __restrict__ out, int accumulate, float* __restrict__ sumsq,
    const int* status) {
  __shared__ int ok;
  __shared__ float red[kRsThreads / 32];
  // a failed wait (this launch's or an earlier one's) leaves every later reduce of the step undone
  if (threadIdx.x == 0) ok = *reinterpret_cast<const volatile int*>(status) == 0;
  __syncthreads();
  if (!ok) return;
  const long long lo = (long long)rank * shard;
  const long long nvec = shard / 8;
  const long long stride = (long long)gridDim.x * kRsThreads;
  float sq = 0.f;
  for (long long v0 = (long long)blockIdx.x * kRsThreads + threadIdx.x; v0 < nvec; v0 += stride * U) {
    float acc[U][8];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[u][k] = 0.f;
    if constexpr (MULTIMEM) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long v = v0 + u * stride;
        if (v < nvec) multimem_sum8(reinterpret_cast<const __nv_bfloat16*>(mc_base) + lo + v * 8, acc[u]);
      }
    } else {
      for (int p0 = 0; p0 < world; p0 += PB) {
        uint4 raw[PB][U];
#pragma unroll
        for (int j = 0; j < PB; ++j) {
          const int p = p0 + j;
          const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(buf_ptrs[p < world ? p : p0]) + lo;
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const long long v = v0 + u * stride;
            if (p < world && v < nvec) raw[j][u] = ld16(src + v * 8);
            else raw[j][u] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
#pragma unroll
        for (int j = 0; j < PB; ++j)
#pragma unroll
          for (int u = 0; u < U; ++u) add8(raw[j][u], acc[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long v = v0 + u * stride;
      if (v >= nvec) continue;
      float4* o = reinterpret_cast<float4*>(out + v * 8);
      float4 a = make_float4(acc[u][0] * scale, acc[u][1] * scale, acc[u][2] * scale, acc[u][3] * scale);
      float4 b = make_float4(acc[u][4] * scale, acc[u][5] * scale, acc[u][6] * scale, acc[u][7] * scale);
      if (accumulate) {
        const float4 pa = o[0], pb = o[1];
        a.x += pa.x; a.y += pa.y; a.z += pa.z; a.w += pa.w;
        b.x += pb.x; b.y += pb.y; b.z += pb.z; b.w += pb.w;
      }
      o[0] = a;
      o[1] = b;
      sq += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
    }
  }
  if (sumsq != nullptr) {
    sq = block_sum(sq, red);
    if (threadIdx.x == 0) atomicAdd(sumsq, sq);
  }
}

// Row gather over peer memory (expert-parallel dispatch / combine): dst row i = row src_row[i] of rank
// src_rank[i]'s buffer (C bf16 per row), or zeros where src_rank[i] < 0.  A row index outside the source's
// capacity is reported (kBadIndex) and its row left zero.
__global__ void __launch_bounds__(256) gather_rows_kernel(const unsigned long long* __restrict__ src_base,
                                                          const int* __restrict__ src_rank,
                                                          const int* __restrict__ src_row, long long rows, int C,
                                                          long long cap_rows, int world,
                                                          __nv_bfloat16* __restrict__ dst, int* status) {
  const int vec = C / 8;
  const long long total = rows * vec;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride * 4) {
    uint4 v[4];
    long long di[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long j = i + u * stride;
      di[u] = -1;
      v[u] = make_uint4(0u, 0u, 0u, 0u);
      if (j >= total) continue;
      const long long r = j / vec;
      const int c = (int)(j % vec);
      di[u] = r * C + c * 8;
      const int sr = src_rank[r];
      const int row = src_row[r];
      if (sr < 0) continue;
      if (sr >= world || row < 0 || row >= cap_rows) {
        report(status, kBadIndex);
        continue;
      }
      v[u] = ld16(reinterpret_cast<const __nv_bfloat16*>(src_base[sr]) + (long long)row * C + c * 8);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (di[u] >= 0) *reinterpret_cast<uint4*>(dst + di[u]) = v[u];
  }
}

// All-gather over peer memory: dst[r * S + i] = rank r's shard[i] (bf16, S a multiple of 8).
__global__ void __launch_bounds__(256) allgather_pull_kernel(const unsigned long long* __restrict__ src_base,
                                                             long long S, int world, __nv_bfloat16* __restrict__ dst) {
  const long long per = S / 8;
  const long long total = per * world;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride * 4) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long j = i + u * stride;
      if (j < total) v[u] = ld16(reinterpret_cast<const __nv_bfloat16*>(src_base[j / per]) + (j % per) * 8);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long j = i + u * stride;
      if (j < total) *reinterpret_cast<uint4*>(dst + j * 8) = v[u];
    }
  }
}

// Broadcast through NVSwitch: the source rank stores each 16-byte vector once to the multicast
// address and the switch writes it into every rank's copy of the buffer (source egress = one copy,
// whatever the world size).  Ends with a system-scope fence so the stores are ordered before the
// barrier the caller issues next.
__global__ void __launch_bounds__(256) multimem_bcast_kernel(const uint4* __restrict__ src,
                                                             unsigned long long mc_dst, long long n16) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) {
    const uint4 v = src[i];
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_dst + 16ull * i),
                 "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
  }
  __threadfence_system();
}

}  // namespace rlb

using namespace rlb;

cudaError_t rlb_multimem_bcast(const void* src, unsigned long long mc_dst, long long nbytes, int sms,
                               cudaStream_t s) {
  if (nbytes <= 0) return cudaSuccess;
  if (nbytes % 16 || (reinterpret_cast<uintptr_t>(src) & 15) || (mc_dst & 15)) return cudaErrorInvalidValue;
  const long long n16 = nbytes / 16;
  long long grid = (n16 + 255) / 256;
  if (grid > 2LL * sms) grid = 2LL * sms;
  multimem_bcast_kernel<<<(int)grid, 256, 0, s>>>(reinterpret_cast<const uint4*>(src), mc_dst, n16);
  return cudaGetLastError();
}

cudaError_t rlb_signal_peers(const unsigned long long* flag_ptrs, int world, int rank, int slot, int epoch,
                             cudaStream_t s) {
  if (world < 1 || world > 32) return cudaErrorInvalidValue;
  signal_peers_kernel<<<1, 32, 0, s>>>(flag_ptrs, world, rank, slot, epoch);
  return cudaGetLastError();
}

cudaError_t rlb_fused_reduce_scatter(const unsigned long long* buf_ptrs, unsigned long long mc_base,
                                     const int* my_flags, int world, int rank, int slot, int epoch, long long shard,
                                     float scale, float* out, int accumulate, float* sumsq, int* status,
                                     unsigned long long limit_ns, int ctas, cudaStream_t s) {
  if (shard % 8 != 0 || world < 1 || world > 32 || ctas < 1) return cudaErrorInvalidValue;
  wait_peers_kernel<<<1, 32, 0, s>>>(my_flags, world, slot, epoch, limit_ns, status);
  const long long nvec = shard / 8;
  const int U = mc_base ? 8 : (world <= 2 ? 8 : world <= 4 ? 4 : 2);
  const long long per_cta = (long long)kRsThreads * U;
  long long grid = (nvec + per_cta - 1) / per_cta;
  if (grid > ctas) grid = ctas;
  if (grid < 1) grid = 1;
  const dim3 g((unsigned)grid), b(kRsThreads);
#define RLB_RS_ARGS buf_ptrs, mc_base, world, rank, shard, scale, out, accumulate, sumsq, status
  if (mc_base) fused_rs_kernel<1, 8, true><<<g, b, 0, s>>>(RLB_RS_ARGS);
  else if (world <= 2) fused_rs_kernel<2, 8, false><<<g, b, 0, s>>>(RLB_RS_ARGS);
  else if (world <= 4) fused_rs_kernel<4, 4, false><<<g, b, 0, s>>>(RLB_RS_ARGS);
  else fused_rs_kernel<8, 2, false><<<g, b, 0, s>>>(RLB_RS_ARGS);
#undef RLB_RS_ARGS
  return cudaGetLastError();
}

cudaError_t rlb_wait_peers(const int* my_flags, int world, int slot, int epoch, unsigned long long limit_ns,
                           int* status, cudaStream_t s) {
  if (world < 1 || world > 32) return cudaErrorInvalidValue;
  wait_peers_kernel<<<1, 32, 0, s>>>(my_flags, world, slot, epoch, limit_ns, status);
  return cudaGetLastError();
}

cudaError_t rlb_gather_rows(const unsigned long long* src_base, const int* src_rank, const int* src_row,
                            long long rows, int C, long long cap_rows, int world, void* dst, int* status, int sms,
                            cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  if (C % 8 || (reinterpret_cast<uintptr_t>(dst) & 15)) return cudaErrorInvalidValue;
  const long long total = rows * (C / 8);
  long long grid = (total + 1023) / 1024;
  if (grid > 4LL * sms) grid = 4LL * sms;
  if (grid < 1) grid = 1;
  gather_rows_kernel<<<(int)grid, 256, 0, s>>>(src_base, src_rank, src_row, rows, C, cap_rows, world,
                                               reinterpret_cast<__nv_bfloat16*>(dst), status);
  return cudaGetLastError();
}

cudaError_t rlb_allgather_pull(const unsigned long long* src_base, long long S, int world, void* dst, int sms,
                               cudaStream_t s) {
  if (S <= 0) return cudaSuccess;
  if (S % 8 || world < 1 || world > 32 || (reinterpret_cast<uintptr_t>(dst) & 15)) return cudaErrorInvalidValue;
  const long long total = S / 8 * world;
  long long grid = (total + 1023) / 1024;
  if (grid > 2LL * sms) grid = 2LL * sms;
  if (grid < 1) grid = 1;
  allgather_pull_kernel<<<(int)grid, 256, 0, s>>>(src_base, S, world, reinterpret_cast<__nv_bfloat16*>(dst));
  return cudaGetLastError();
}
