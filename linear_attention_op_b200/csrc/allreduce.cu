// All-reduce (sum) of bf16 partials over NVLink peer memory, for the small per-layer outputs of
// tensor-parallel decode (512 KB .. 8 MB), where a ring collective is latency-bound.
//
// Every rank owns two slot buffers and a flag page mapped into all other ranks (CUDA IPC).  Call e (the
// device-side epoch + 1) uses slot e % 2: the out_proj GEMM writes the rank's partial into its own slot,
// then this kernel
//   1. announces "partial ready" for e by a release store into every rank's arrive[rank] flag and waits
//      (bounded) until every rank's announcement is visible in its own flag page;
//   2. two ranks: sums both partials in rank order straight from the peers' slots (one shot);
//      more ranks: reduce-scatter + all-gather -- rank r sums slice r of every partial (rank order) into
//      slice r of its own slot and of the output; each CTA then announces its share of the slice
//      (reduced[rank][cta]) and copies the same share of every other rank's reduced slice once that rank's
//      CTA of the same index has announced it;
//   3. advances the epoch once every CTA has read it.
// The kernel lets the next kernel in the stream launch as soon as it starts (programmatic dependent
// launch): the next step's in_proj streams its weights while this kernel waits on its peers.
// Every rank computes identical bits (rank-order sums).  No rank rewrites a slot a peer may still read: a
// rank writes slot e % 2 again only at call e + 2, after its call e + 1 saw every peer arrive at e + 1,
// which each peer does only after finishing its call e.  The epoch lives in device memory, so the kernel
// replays correctly inside a CUDA graph.  Every wait gives up after GDN_WAIT_TIMEOUT_NS, records
// kErrWaitPeer and skips the rest.
#include <cuda_bf16.h>

#include <algorithm>

#include "gemm.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace gdn {

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *p >= e.  False (and the error word set) after GDN_WAIT_TIMEOUT_NS.
__device__ __forceinline__ bool wait_flag(const unsigned long long* p, unsigned long long e) {
  if (ld_acquire_sys(p) >= e) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (ld_acquire_sys(p) >= e) return true;
    if (globaltimer_ns() - t0 > GDN_WAIT_TIMEOUT_NS) {
      record_error(kErrWaitPeer);
      return false;
    }
  }
}

// Lane p of warp 0 waits for flags[p * stride] >= e, p in [0, world), all flags polled at once (an acquire
// load at system scope costs an L2 round trip, so world sequential polls would cost world of them); the CTA
// learns the outcome.
__device__ __forceinline__ bool cta_wait_all_stride(const unsigned long long* flags, int stride, int world,
                                                    unsigned long long e, int* s_abort) {
  if (threadIdx.x < 32) {
    const bool ok = threadIdx.x >= world || wait_flag(flags + static_cast<int64_t>(threadIdx.x) * stride, e);
    if (!__all_sync(0xffffffffu, ok) && threadIdx.x == 0) *s_abort = 1;
  }
  __syncthreads();
  return *s_abort == 0;
}
__device__ __forceinline__ bool cta_wait_all(const unsigned long long* flags, int world, unsigned long long e,
                                             int* s_abort) {
  return cta_wait_all_stride(flags, 1, world, e, s_abort);
}

// Sum of the world partials of 8 bf16 (vector i of each slot), in rank order.
__device__ __forceinline__ uint4 sum8(const P2PAllReduceArgs& a, int64_t slot, int64_t i) {
  uint4 v[kP2PMaxRanks];
#pragma unroll
  for (int p = 0; p < kP2PMaxRanks; ++p)
    if (p < a.world) v[p] = __ldcg(reinterpret_cast<const uint4*>(static_cast<const char*>(a.src[p]) + slot) + i);
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
  for (int p = 0; p < kP2PMaxRanks; ++p) {
    if (p < a.world) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[p]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
  }
  uint4 o;
  __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
  return o;
}

__global__ void __launch_bounds__(256) allreduce_p2p_kernel(P2PAllReduceArgs a) {
  __shared__ int s_abort;
  // Launched with programmatic dependent launch: it starts once out_proj has finished and its partial is
  // in memory.
  griddep_wait();
  // The next kernel (the next step's in_proj) may start streaming its weights now; its own dependent
  // wait still orders every read of this kernel's output after this grid completes.
  griddep_launch_dependents();
  const unsigned long long e = *reinterpret_cast<volatile unsigned long long*>(a.epoch) + 1;
  if (threadIdx.x == 0) s_abort = 0;
  __syncthreads();
  const int64_t slot = static_cast<int64_t>(e & 1) * a.slot_bytes;
  const int64_t nv = a.n / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  uint4* out = reinterpret_cast<uint4*>(a.out);
  // 1. partial ready.  The grid is at most one CTA per SM and so fully resident: the other CTAs' waits can
  //    rely on CTA 0 running.
  if (blockIdx.x == 0 && threadIdx.x < a.world) st_release_sys(a.flags[threadIdx.x] + a.rank, e);
  bool ok = cta_wait_all(a.flags[a.rank], a.world, e, &s_abort);
  if (ok && a.world == 2) {
    for (int64_t i = tid0; i < nv; i += stride) out[i] = sum8(a, slot, i);
  } else if (ok) {
    // 2a. reduce-scatter: slice r of every partial, into slice r of this rank's slot and of the output
    const int64_t per = (nv + a.world - 1) / a.world;
    const int64_t lo = per * a.rank, hi = min(nv, lo + per);
    uint4* mine = reinterpret_cast<uint4*>(static_cast<char*>(const_cast<void*>(a.src[a.rank])) + slot);
    for (int64_t i = lo + tid0; i < hi; i += stride) {
      const uint4 o = sum8(a, slot, i);
      mine[i] = o;
      out[i] = o;
    }
    // CTA c of every rank covers the same offsets inside each slice, so CTA c of rank p copies exactly
    // what CTA c of rank r reduced: a per-CTA "reduced" flag replaces a grid-wide barrier.
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < a.world)
      st_release_sys(a.flags[threadIdx.x] + kP2PReducedOff + a.rank * kP2PMaxCtas + blockIdx.x, e);
    // 2b. all-gather of the other ranks' reduced slices, every peer's load in flight at once
    ok = cta_wait_all_stride(a.flags[a.rank] + kP2PReducedOff + blockIdx.x, kP2PMaxCtas, a.world, e, &s_abort);
    if (ok) {
      for (int64_t k = tid0; k < per; k += stride) {
        uint4 v[kP2PMaxRanks];
#pragma unroll
        for (int p = 0; p < kP2PMaxRanks; ++p)
          if (p < a.world && p != a.rank && per * p + k < nv)
            v[p] = __ldcg(reinterpret_cast<const uint4*>(static_cast<const char*>(a.src[p]) + slot) + per * p + k);
#pragma unroll
        for (int p = 0; p < kP2PMaxRanks; ++p)
          if (p < a.world && p != a.rank && per * p + k < nv) out[per * p + k] = v[p];
      }
    }
  }
  // 3. the last CTA to finish advances the epoch (every CTA has read it by then)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.cta_done, 1u) == gridDim.x - 1) {
      a.cta_done[0] = 0u;
      *reinterpret_cast<volatile unsigned long long*>(a.epoch) = e;
    }
  }
}

__global__ void peer_wait_selftest_kernel(const unsigned long long* flag, unsigned long long value) {
  wait_flag(flag, value);
}

cudaError_t peer_wait_selftest(const unsigned long long* flag, unsigned long long value, cudaStream_t stream) {
  if (!flag || (reinterpret_cast<uintptr_t>(flag) & 7)) return cudaErrorInvalidValue;
  count_launch();
  peer_wait_selftest_kernel<<<1, 1, 0, stream>>>(flag, value);
  return cudaGetLastError();
}

cudaError_t allreduce_p2p(const P2PAllReduceArgs& a, cudaStream_t stream) {
  if (a.world < 2 || a.world > kP2PMaxRanks || a.rank < 0 || a.rank >= a.world || a.n <= 0 || (a.n & 7) || !a.out)
    return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t nv = a.n / 8;
  const int grid = static_cast<int>(std::min<int64_t>(std::min(sms, kP2PMaxCtas), (nv + 255) / 256));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  return cudaLaunchKernelEx(&cfg, allreduce_p2p_kernel, a);
}

}  // namespace gdn
