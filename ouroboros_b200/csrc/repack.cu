// repack.cu -- upload-time conversion of the canonical host layouts of the
// C ABI into the device layouts documented in kernels.h.
//
// Canonical TERNARY2 (host): row-major [M][K/4], code c = w + 1 of element k
//   in byte k/4, bits 2*(k%4).
// Canonical SIGN1G128 (host): row-major [M][K/8], sign bit of element k in
//   byte k/8, bit k%8 (1 -> +1, 0 -> -1).
// Both conversions are pure bit permutations inside each 32-bit word, so one
// thread produces one output word from the matching input word.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace ouroq {
namespace {

// Output word t: byte b, bits (2j, 2j+1) <- code of k = 16t + 4j + b,
// i.e. input byte j (of the same word), bits 2b.
__global__ void repack_tern2_kernel(const uint32_t* __restrict__ in, uint32_t* __restrict__ out,
                                    size_t nwords) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nwords;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t w = in[i];
    uint32_t o = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t byte = (w >> (8 * j)) & 0xFFu;
#pragma unroll
      for (int b = 0; b < 4; ++b) o |= ((byte >> (2 * b)) & 3u) << (8 * b + 2 * j);
    }
    out[i] = o;
  }
}

// Output word t: byte b, bit j <- sign bit of k = 32t + 4j + b, which sits in
// input bit (4j + b) of the same word.
__global__ void repack_sign1_kernel(const uint32_t* __restrict__ in, uint32_t* __restrict__ out,
                                    size_t nwords) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nwords;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t w = in[i];
    uint32_t o = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int b = 0; b < 4; ++b) o |= ((w >> (4 * j + b)) & 1u) << (8 * b + j);
    out[i] = o;
  }
}

}  // namespace

cudaError_t launch_repack_tern2(const uint8_t* canon, uint8_t* dev, int M, int K, cudaStream_t s) {
  const size_t nwords = (size_t)M * (K / 16);
  if (nwords == 0) return cudaSuccess;
  const int threads = 256;
  const size_t blocks = (nwords + threads - 1) / threads;
  repack_tern2_kernel<<<(unsigned)(blocks < 65535 * 16 ? blocks : 65535 * 16), threads, 0, s>>>(
      reinterpret_cast<const uint32_t*>(canon), reinterpret_cast<uint32_t*>(dev), nwords);
  return cudaGetLastError();
}

cudaError_t launch_repack_sign1(const uint8_t* canon, uint8_t* dev, int M, int K, cudaStream_t s) {
  const size_t nwords = (size_t)M * (K / 32);
  if (nwords == 0) return cudaSuccess;
  const int threads = 256;
  const size_t blocks = (nwords + threads - 1) / threads;
  repack_sign1_kernel<<<(unsigned)(blocks < 65535 * 16 ? blocks : 65535 * 16), threads, 0, s>>>(
      reinterpret_cast<const uint32_t*>(canon), reinterpret_cast<uint32_t*>(dev), nwords);
  return cudaGetLastError();
}

}  // namespace ouroq
