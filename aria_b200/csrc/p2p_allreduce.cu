// p2p_allreduce.cu -- the reduction step of the column-split FFN of the
// scaled-up config over NVLink peer memory, and the IPC plumbing it needs.
//
// The split (BASELINE configs[4] decode at batch 64 on 2..8 GPUs): every rank
// computes ffn_up on its column range and multiplies the result by its rows
// of ffn_down, so the layer's output is the SUM over ranks of f32 partials
// [M][d_model], added into the f16 residual stream.  NCCL's all-reduce plus a
// separate residual add costs two launches and NCCL's protocol latency per
// layer; here one kernel per rank does both, one-shot:
//
//   * block 0 publishes "my partial of epoch e is complete" by a system-scope
//     release store of e into a flag word in every peer's memory (the
//     partial was written by the preceding kernel on this rank's stream);
//   * every block waits (bounded, %globaltimer) until each peer's flag word in
//     this rank's memory holds e, then adds all ranks' partials -- read
//     straight from the peers' memory over NVLink, in rank order, so every
//     rank computes identical bits -- to its share of h;
//   * the last block to finish advances the epoch kept in this rank's
//     memory, so a CUDA graph replaying the same launches stays in step.
//
// Partials are kept one buffer per layer: a rank rewrites layer l's buffer
// one step later, after it has seen every peer publish the epochs in between,
// i.e. after every peer's reduction of layer l (which reads that buffer) has
// completed on the peer's stream.  A peer that never publishes makes the
// wait run out: the kernel records ARIA_Q4_DEVERR_PEER_TIMEOUT, leaves h
// unchanged and returns.  No multicast and no NVLS: plain peer loads and
// stores through IPC mappings.
#include <cuda_runtime.h>

#include "q4_common.cuh"

namespace aria_q4 {

constexpr int kP2PMaxRanks = 8;
constexpr int kP2PErrPeerTimeout = 4;
constexpr int kP2PThreads = 256;

struct P2PArgs {
  const float* part[kP2PMaxRanks];  // this layer's partial on every rank (peers: IPC-mapped)
  unsigned* flag[kP2PMaxRanks];     // every rank's flag words: flag[p][r] = last epoch rank r published to p
  unsigned* state;                  // this rank's [epoch, blocks finished]
  int nranks, rank;
  __half* h;                        // residual stream, n f16 elements, h += sum of the partials
  int n;
  unsigned long long wait_ns;
};

static __device__ int g_p2p_error = 0;

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long p2p_globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(kP2PThreads) p2p_allreduce_kernel(const P2PArgs a) {
  __shared__ unsigned s_epoch;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    // the previous call's last block stored the epoch before that kernel ended
    const unsigned e = *reinterpret_cast<volatile unsigned*>(a.state) + 1u;
    s_epoch = e;
    if (blockIdx.x == 0) {
      __threadfence_system();
      for (int p = 0; p < a.nranks; p++)
        if (p != a.rank) st_release_sys(a.flag[p] + a.rank, e);
    }
    bool ok = true;
    const unsigned long long t0 = p2p_globaltimer();
    for (int p = 0; p < a.nranks && ok; p++) {
      if (p == a.rank) continue;
      while ((int)(ld_acquire_sys(a.flag[a.rank] + p) - e) < 0) {
        if (p2p_globaltimer() - t0 > a.wait_ns) {
          ok = false;
          atomicCAS(&g_p2p_error, 0, kP2PErrPeerTimeout);
          break;
        }
      }
    }
    s_ok = ok ? 1 : 0;
  }
  __syncthreads();
  if (s_ok) {
    // 8 elements per thread and step: two 16-byte loads per partial, one
    // 16-byte load and store of h
    const int n8 = a.n >> 3;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += gridDim.x * blockDim.x) {
      float acc[8];
      const uint4 hv = reinterpret_cast<const uint4*>(a.h)[i];
      const __half2* h2 = reinterpret_cast<const __half2*>(&hv);
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float2 f = __half22float2(h2[u]);
        acc[2 * u] = f.x;
        acc[2 * u + 1] = f.y;
      }
      float sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int p = 0; p < a.nranks; p++) {
        const float4* src = reinterpret_cast<const float4*>(a.part[p]) + 2 * (size_t)i;
        const float4 v0 = __ldcg(src), v1 = __ldcg(src + 1);
        sum[0] += v0.x; sum[1] += v0.y; sum[2] += v0.z; sum[3] += v0.w;
        sum[4] += v1.x; sum[5] += v1.y; sum[6] += v1.z; sum[7] += v1.w;
      }
      uint4 ov;
      __half2* o2 = reinterpret_cast<__half2*>(&ov);
#pragma unroll
      for (int u = 0; u < 4; u++) o2[u] = __floats2half2_rn(acc[2 * u] + sum[2 * u], acc[2 * u + 1] + sum[2 * u + 1]);
      reinterpret_cast<uint4*>(a.h)[i] = ov;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned done = atomicAdd(a.state + 1, 1u);
    if (done == gridDim.x - 1) {
      a.state[1] = 0u;
      __threadfence();
      *reinterpret_cast<volatile unsigned*>(a.state) = s_epoch;
    }
  }
}

// h[0..n) += sum over ranks of part[r][0..n) (f32), one-shot over peer memory.
// n a multiple of 8; h and every part 16-byte aligned.
cudaError_t launch_p2p_allreduce(const float* const* part, unsigned* const* flag, unsigned* state, int nranks,
                                 int rank, __half* h, int n, unsigned long long wait_ns, cudaStream_t st) {
  P2PArgs a;
  for (int p = 0; p < kP2PMaxRanks; p++) {
    a.part[p] = p < nranks ? part[p] : nullptr;
    a.flag[p] = p < nranks ? flag[p] : nullptr;
  }
  a.state = state;
  a.nranks = nranks;
  a.rank = rank;
  a.h = h;
  a.n = n;
  a.wait_ns = wait_ns;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int need = (n / 8 + kP2PThreads - 1) / kP2PThreads;
  const int grid = need < sms ? (need > 0 ? need : 1) : sms;
  p2p_allreduce_kernel<<<grid, kP2PThreads, 0, st>>>(a);
  return cudaGetLastError();
}

// Reads and clears this unit's device error flag (synchronous).
int p2p_take_device_error() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_p2p_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) cudaMemcpyToSymbol(g_p2p_error, &zero, sizeof(int));
  return v;
}

}  // namespace aria_q4
