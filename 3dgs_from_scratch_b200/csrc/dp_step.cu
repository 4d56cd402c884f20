// dp_step.cu -- the data-parallel optimizer step as one kernel over NVLink /
// NVSwitch: gradient reduce-scatter, Adam on this rank's shard, all-gather
// of the updated parameters.
//
// Data-parallel training over camera views (one process per GPU, a full
// replica of the Gaussians on each) ends every step with a sum of the flat
// gradient over the ranks and the same Adam update on every rank (the
// reference trains on one GPU, scripts/train.py:160-221). Instead of an
// all-reduce of the whole gradient followed by a full-size Adam on every
// rank, each rank owns 1/world of the flat buffer and, in one launch:
//   1. waits until every rank has reached this step (its gradient complete);
//   2. for each float4 of its shard, reads the sum of that float4 over all
//      ranks' gradient buffers -- one multimem.ld_reduce through the NVSwitch
//      (the switch fetches and adds) when a multicast mapping exists, else
//      peer loads of every rank's buffer added in rank order;
//   3. applies Adam with its shard of the optimizer state (so each rank keeps
//      only 1/world of the Adam moments);
//   4. writes the new parameters to every rank's parameter buffer -- one
//      multimem.st (the switch replicates) or a peer store per rank;
//   5. waits until every rank has written, so that when the kernel has
//      finished on a rank, its parameter buffer holds the whole update.
// Every rank also publishes, with its arrival at the first barrier, whether
// its device status word holds an error from earlier in the step (its
// gradient may then be incomplete); if any rank does, every rank skips
// steps 2-4 -- the update is dropped on all ranks alike, so the replicas
// stay identical -- and a rank without an error of its own records
// GS_ERR_PEER.
// The gradient crosses NVLink once per rank (in, reduced) and the parameters
// once per rank (out); no all-reduce and no full-size Adam pass remain.
//
// Synchronisation: block b of every rank signals block b of every other rank
// (a release store of the step's epoch into the peer's flag word, after a
// system-scope fence) and waits for the same from all of them (acquire
// loads). Every block of a rank thus waits for the same block of every other
// rank, so kernel completion on a rank implies every block of every rank
// has passed the barrier. The grid never exceeds one block per SM, so all
// blocks are resident together. Each wait is bounded by the global timer;
// on expiry the block records GS_ERR_DEVICE_TIMEOUT in the status word and
// returns (the other ranks then time out in turn), and the host reads the
// status with gs_check_status.
//
// No TMA or bulk copy is used: every access to another GPU's memory is a
// plain load, store or multimem operation.
#include "adam.cuh"

namespace gs {

#ifndef GS_DP_THREADS
#define GS_DP_THREADS 512
#endif
#ifndef GS_DP_UNROLL
#define GS_DP_UNROLL 4
#endif
constexpr int kDpThreads = GS_DP_THREADS;
constexpr int kDpMaxWorld = 8;
constexpr int kDpUnroll = GS_DP_UNROLL;                 // float4s in flight per thread
constexpr unsigned long long kDpTimeoutNs = 4000000000ull;  // 4 s per wait

struct DpPeers {
  float4 *grad[kDpMaxWorld];
  float4 *param[kDpMaxWorld];
  uint32_t *flags[kDpMaxWorld];
};

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float4 multimem_ld_reduce_add(const float4 *mc) {
  float4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}

__device__ __forceinline__ void multimem_st(float4 *mc, const float4 &v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

// Flag word of (phase, block, source rank) in a rank's flag buffer.
__device__ __forceinline__ size_t flag_index(int phase, int block, int nblocks, int src) {
  return ((size_t)phase * nblocks + block) * kDpMaxWorld + src;
}

// Barrier between block blockIdx.x of every rank. Returns false (and records
// a timeout) if some rank did not arrive within kDpTimeoutNs.
__device__ bool rank_barrier(const DpPeers &P, int world, int rank, int phase, uint32_t epoch,
                             uint32_t *status) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();  // this block's earlier accesses come before the signals below
  const int peer = threadIdx.x;
  if (peer < world) {
    __threadfence_system();
    st_release_sys(P.flags[peer] + flag_index(phase, blockIdx.x, gridDim.x, rank), epoch);
    const uint32_t *mine = P.flags[rank] + flag_index(phase, blockIdx.x, gridDim.x, peer);
    const unsigned long long t0 = global_timer_ns();
    while ((int32_t)(ld_acquire_sys(mine) - epoch) < 0) {
      if (global_timer_ns() - t0 > kDpTimeoutNs) {
        atomicExch(status, (uint32_t)GS_ERR_DEVICE_TIMEOUT);
        s_ok = 0;
        break;
      }
      __nanosleep(256);
    }
  }
  __syncthreads();
  return s_ok != 0;
}

template <bool MULTIMEM>
__global__ void __launch_bounds__(kDpThreads) dp_adam_kernel(
    DpPeers P, float4 *mc_grad, float4 *mc_param, int world, int rank, int64_t shard4,
    float4 *__restrict__ m, float4 *__restrict__ v, AdamGroups G, float b1, float b2,
    uint32_t epoch, float4 *__restrict__ grad_out, uint32_t *status) {
  // this rank's status for the step, to every rank (phase-2 words: 2 epoch +
  // error), ahead of the release store of the first barrier
  __shared__ int s_skip;
  const uint32_t err = ld_volatile_u32(status) != 0u ? 1u : 0u;
  if (threadIdx.x == 0) s_skip = 0;
  if (threadIdx.x < world)
    P.flags[threadIdx.x][flag_index(2, blockIdx.x, gridDim.x, rank)] = 2u * epoch + err;
  if (!rank_barrier(P, world, rank, 0, epoch, status)) return;
  if (threadIdx.x < world) {
    const uint32_t w = ld_acquire_sys(P.flags[rank] + flag_index(2, blockIdx.x, gridDim.x,
                                                                 threadIdx.x));
    if (w != 2u * epoch) atomicOr(&s_skip, 1);
  }
  __syncthreads();
  if (s_skip) {
    if (threadIdx.x == 0 && !err) atomicCAS(status, 0u, (uint32_t)GS_ERR_PEER);
    rank_barrier(P, world, rank, 1, epoch, status);
    return;
  }
  const int64_t off4 = (int64_t)rank * shard4;
  const float4 *own = P.param[rank];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < shard4;
       i0 += stride * kDpUnroll) {
    float4 g[kDpUnroll];
#pragma unroll
    for (int u = 0; u < kDpUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < shard4) {
        if (MULTIMEM) {
          g[u] = multimem_ld_reduce_add(mc_grad + off4 + i);
        } else {
          float4 s = P.grad[0][off4 + i];
          for (int r = 1; r < world; ++r) {
            const float4 x = P.grad[r][off4 + i];
            s.x += x.x;
            s.y += x.y;
            s.z += x.z;
            s.w += x.w;
          }
          g[u] = s;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kDpUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= shard4) break;
      float4 p = own[off4 + i], mm = m[i], vv = v[i];
      adam_float4(G, 4 * (off4 + i), p, g[u], mm, vv, b1, b2);
      m[i] = mm;
      v[i] = vv;
      if (grad_out) grad_out[i] = g[u];
      if (MULTIMEM) {
        multimem_st(mc_param + off4 + i, p);
      } else {
        for (int r = 0; r < world; ++r) P.param[r][off4 + i] = p;
      }
    }
  }
  rank_barrier(P, world, rank, 1, epoch, status);
}

}  // namespace gs

using namespace gs;

extern "C" size_t gs_dp_flag_words(int max_blocks) {
  if (max_blocks <= 0) return 0;
  return (size_t)3 * max_blocks * kDpMaxWorld;  // two barriers and the status exchange
}

extern "C" int gs_dp_max_blocks(void) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return sms;
}

extern "C" int gs_dp_adam_step(int world, int rank, void *const *grad_ptrs,
                               void *const *param_ptrs, void *const *flag_ptrs,
                               void *mc_grad, void *mc_param, int64_t n, float *exp_avg_shard,
                               float *exp_avg_sq_shard, int num_groups,
                               const int64_t *group_ends, const float *lrs, const float *eps,
                               float beta1, float beta2, int64_t step, uint32_t epoch,
                               int num_blocks, float *grad_shard_out, void *stream) {
  if (world < 1 || world > kDpMaxWorld || rank < 0 || rank >= world || n <= 0 ||
      n % (4 * world) != 0 || grad_ptrs == nullptr || param_ptrs == nullptr ||
      flag_ptrs == nullptr || exp_avg_shard == nullptr || exp_avg_sq_shard == nullptr)
    return GS_ERR_INVALID_ARGUMENT;
  if ((mc_grad == nullptr) != (mc_param == nullptr)) return GS_ERR_INVALID_ARGUMENT;
  const int max_blocks = gs_dp_max_blocks();
  if (num_blocks < 1 || num_blocks > max_blocks) return GS_ERR_INVALID_ARGUMENT;
  DpPeers P{};
  uintptr_t align = (uintptr_t)exp_avg_shard | (uintptr_t)exp_avg_sq_shard |
                    (uintptr_t)grad_shard_out | (uintptr_t)mc_grad | (uintptr_t)mc_param;
  for (int r = 0; r < world; ++r) {
    if (grad_ptrs[r] == nullptr || param_ptrs[r] == nullptr || flag_ptrs[r] == nullptr)
      return GS_ERR_INVALID_ARGUMENT;
    align |= (uintptr_t)grad_ptrs[r] | (uintptr_t)param_ptrs[r] | ((uintptr_t)flag_ptrs[r] & 3);
    P.grad[r] = reinterpret_cast<float4 *>(grad_ptrs[r]);
    P.param[r] = reinterpret_cast<float4 *>(param_ptrs[r]);
    P.flags[r] = reinterpret_cast<uint32_t *>(flag_ptrs[r]);
  }
  if (align & 15) return GS_ERR_INVALID_ARGUMENT;
  AdamGroups G;
  int rc = build_adam_groups(n, num_groups, group_ends, lrs, eps, beta1, beta2, step, &G);
  if (rc) return rc;
  const int64_t shard4 = n / world / 4;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint32_t *status = device_status_word();
  if (status == nullptr) return GS_ERR_CUDA;
  if (mc_grad) {
    dp_adam_kernel<true><<<num_blocks, kDpThreads, 0, st>>>(
        P, reinterpret_cast<float4 *>(mc_grad), reinterpret_cast<float4 *>(mc_param), world, rank,
        shard4, reinterpret_cast<float4 *>(exp_avg_shard),
        reinterpret_cast<float4 *>(exp_avg_sq_shard), G, beta1, beta2, epoch,
        reinterpret_cast<float4 *>(grad_shard_out), status);
  } else {
    dp_adam_kernel<false><<<num_blocks, kDpThreads, 0, st>>>(
        P, nullptr, nullptr, world, rank, shard4, reinterpret_cast<float4 *>(exp_avg_shard),
        reinterpret_cast<float4 *>(exp_avg_sq_shard), G, beta1, beta2, epoch,
        reinterpret_cast<float4 *>(grad_shard_out), status);
  }
  count_launch();
  return launch_status();
}
