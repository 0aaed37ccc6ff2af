// shard.cu -- device side of the row-sharded matmul (one process per GPU).
//
// Rank r of G owns output rows [r*R, (r+1)*R) of an M = G*R row matrix. Each
// rank computes y_r [B][R] for its rows into slot r of a gather buffer
// [G][B][R]; an in-place NCCL all-gather over NVLink fills the other slots;
// this kernel then interleaves the slots into the row-major output
// y [B][M] (y[b][r*R + i] = gather[r][b][i]). At B = 1 the slot order already
// is the output order and the host skips this kernel.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace ouroq {
namespace {

// grid: (ceil(R/4 / 256), B, G); each thread moves four consecutive floats
__global__ void __launch_bounds__(256) shard_interleave_kernel(const float* __restrict__ gather,
                                                               float* __restrict__ y, int B, int R,
                                                               int G) {
  const int r = blockIdx.z, b = blockIdx.y;
  const int i = (blockIdx.x * 256 + threadIdx.x) * 4;
  if (i >= R) return;
  const float* src = gather + ((size_t)r * B + b) * R;
  float* dst = y + (size_t)b * R * G + (size_t)r * R;
  if (i + 3 < R && (R & 3) == 0) {
    *reinterpret_cast<float4*>(dst + i) = *reinterpret_cast<const float4*>(src + i);
  } else {
    for (int k = i; k < i + 4 && k < R; ++k) dst[k] = src[k];
  }
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Peer-store all-gather of the sharded product. Every value travels with its
// step number in one aligned 64-bit word (step << 32 | fp32 bits): a single
// store is seen whole or not at all, so a reader needs no flag, fence or
// counter -- it waits until the word carries the step it expects. Every rank
// runs this kernel after its local rows are in `staging` [B][R]:
//   1. wait for the product (programmatic dependent launch: full completion)
//   2. e = this rank's step counter + 1; store staging into slot `rank` of
//      parity e&1 of every rank's landing buffer (peer stores over NVLink)
//   3. read this rank's landing buffer, waiting (bounded) for each word to
//      carry step e, and write the values interleaved into y [B][G*R]
//   4. the last CTA to finish advances the step counter
// Steps of one rank are stream-ordered and a rank cannot finish step e before
// every peer has stored its step-e rows, so a peer is at most one step ahead:
// two parities suffice. A wait past timeout_ns records kDevPeerTimeout in the
// status word and leaves the rest of y unwritten.
__global__ void __launch_bounds__(256) shard_gather_kernel(const __grid_constant__ ShardGather P) {
  pdl_wait();
  // The next product may start streaming its weights now: it writes `staging`
  // and reads nothing of ours before its own wait for this grid to finish.
  pdl_launch_dependents();
  __shared__ unsigned s_e;
  __shared__ int s_abort;
  if (threadIdx.x == 0) {
    s_e = *reinterpret_cast<volatile unsigned*>(P.step) + 1u;
    s_abort = 0;
  }
  __syncthreads();
  const unsigned e = s_e;
  const unsigned long long tag = (unsigned long long)e << 32;
  const size_t slot = (size_t)P.B * P.R;  // words per rank slot
  const size_t par_off = (size_t)(e & 1u) * P.G * slot;
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t nth = (size_t)gridDim.x * blockDim.x;
  // 2. push
  const unsigned* src = reinterpret_cast<const unsigned*>(P.staging);
  for (size_t i = tid; i < slot; i += nth) {
    const unsigned long long w = tag | src[i];
    for (int g = 0; g < P.G; ++g)
      st_volatile_u64(P.peers[g] + par_off + (size_t)P.rank * slot + i, w);
  }
  // 3. collect
  const unsigned long long* land = P.peers[P.rank] + par_off;
  const size_t total = (size_t)P.G * slot;
  const unsigned long long t0 = global_ns();
  for (size_t i = tid; i < total; i += nth) {
    unsigned long long w = ld_volatile_u64(land + i);
    unsigned spins = 0;
    while ((unsigned)(w >> 32) != e) {
      if ((++spins & 1023u) == 0) {
        if (*reinterpret_cast<volatile int*>(&s_abort)) break;
        if (global_ns() - t0 > P.timeout_ns) {
          atomicExch(P.status, kDevPeerTimeout);
          *reinterpret_cast<volatile int*>(&s_abort) = 1;
          break;
        }
      }
      w = ld_volatile_u64(land + i);
    }
    if ((unsigned)(w >> 32) != e) break;
    const size_t r = i % P.R;
    const size_t gb = i / P.R;
    const int b = (int)(gb % P.B);
    const int g = (int)(gb / P.B);
    P.y[(size_t)b * P.R * P.G + (size_t)g * P.R + r] = __uint_as_float((unsigned)w);
  }
  __syncthreads();
  // 4. advance the step counter once every CTA is done with step e
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(P.done, 1u);
    if (prev == gridDim.x - 1) {
      *P.done = 0u;
      *P.step = e;
    }
  }
}

}  // namespace

cudaError_t launch_shard_gather(const ShardGather& P, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  // about 2 words per thread of the collect phase, at most kShardGatherCtas CTAs
  const size_t words = (size_t)P.G * P.B * P.R;
  size_t ctas = (words + 511) / 512;
  ctas = ctas < 1 ? 1 : (ctas > (size_t)kShardGatherCtas ? (size_t)kShardGatherCtas : ctas);
  cfg.gridDim = dim3((unsigned)ctas, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, shard_gather_kernel, P);
}

cudaError_t launch_shard_interleave(const float* gather, float* y, int B, int R, int G,
                                    cudaStream_t s) {
  if (B <= 0 || R <= 0 || G <= 0) return cudaSuccess;
  const dim3 grid((unsigned)(((R + 3) / 4 + 255) / 256), (unsigned)B, (unsigned)G);
  shard_interleave_kernel<<<grid, 256, 0, s>>>(gather, y, B, R, G);
  return cudaGetLastError();
}

}  // namespace ouroq
