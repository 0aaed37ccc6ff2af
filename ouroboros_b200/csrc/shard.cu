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

}  // namespace

cudaError_t launch_shard_interleave(const float* gather, float* y, int B, int R, int G,
                                    cudaStream_t s) {
  if (B <= 0 || R <= 0 || G <= 0) return cudaSuccess;
  const dim3 grid((unsigned)(((R + 3) / 4 + 255) / 256), (unsigned)B, (unsigned)G);
  shard_interleave_kernel<<<grid, 256, 0, s>>>(gather, y, B, R, G);
  return cudaGetLastError();
}

}  // namespace ouroq
