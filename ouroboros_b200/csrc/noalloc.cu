// noalloc.cu -- the fixed scratch area behind ouroq_gemm_f32act_noalloc.
//
// ouroq_gemm_f32act quantises large batches into a per-context buffer that it
// grows with cudaMalloc (and cudaFree of the old one) when a bigger batch
// arrives. Some callers cannot let that happen while they run: a serving loop
// that reserved the GPU's memory up front for weights and caches (a late
// cudaMalloc can fail there), or one on a latency budget (cudaFree waits for
// the whole device). For them the scratch lives here instead, as storage
// compiled into the library: the CUDA runtime sets it up, one copy per device,
// when it loads this library's kernels on that device.
//
// Layout: int8 activation codes q [B][K] at offset 0 (B*K <= kNoAllocQBytes),
// then fp32 token scales s_x [B] at offset kNoAllocQBytes (B <= kNoAllocMaxTokens).
// Nothing here has to start at zero: the quantiser writes every code and scale
// that the matmul kernels later read, and rows past B are never read from
// memory (the tensor-core path's copy engine fills them with zeros).
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace ouroq {

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

cudaError_t noalloc_scratch_address(void** ptr) {
  return cudaGetSymbolAddress(ptr, g_noalloc_scratch);
}

}  // namespace ouroq
