// repack.cu -- upload-time conversion of the canonical host layouts of the
// C ABI into the tiled device layouts documented in kernels.h.
//
// Canonical TERNARY2 (host): row-major [M][K/4], code c = w + 1 of element k
//   in byte k/4, bits 2*(k%4).
// Canonical SIGN1G128 (host): row-major [M][K/8], sign bit of element k in
//   byte k/8, bit k%8 (1 -> +1, 0 -> -1); fp16 scales [M][K/128].
// One thread produces one 32-bit device word: it reads the matching canonical
// word, permutes its bits, and stores it at the tiled position. Rows past M in
// the last tile are written as zero.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace ouroq {
namespace {

__device__ __forceinline__ uint32_t perm_tern(uint32_t w) {
  // out byte b, bits (2j, 2j+1) <- code of k = 16t + 4j + b = in byte j, bits 2b
  uint32_t o = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t byte = (w >> (8 * j)) & 0xFFu;
#pragma unroll
    for (int b = 0; b < 4; ++b) o |= ((byte >> (2 * b)) & 3u) << (8 * b + 2 * j);
  }
  return o;
}

__device__ __forceinline__ uint32_t perm_sign(uint32_t w) {
  // out byte b, bit j <- sign bit of k = 32t + 4j + b = in bit (4j + b)
  uint32_t o = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int b = 0; b < 4; ++b) o |= ((w >> (4 * j + b)) & 1u) << (8 * b + j);
  return o;
}

// dev word index -> (tile, chunk, row, word-in-chunk); 4 words per 16-B chunk
template <int FMT>
__global__ void repack_kernel(const uint32_t* __restrict__ in, uint32_t* __restrict__ out, int M,
                              int rb_words, size_t ndev) {
  const int C = rb_words / 4;  // 16-byte chunks per row
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < ndev;
       i += (size_t)gridDim.x * blockDim.x) {
    const int wi = (int)(i & 3);
    const size_t rest = i >> 2;             // chunk-row index within the tiled array
    const int r = (int)(rest % kTileRows);
    const size_t tc = rest / kTileRows;     // tile * C + chunk
    const int c = (int)(tc % C);
    const size_t t = tc / C;
    const size_t row = t * kTileRows + r;
    uint32_t v = 0;
    if (row < (size_t)M) {
      const uint32_t w = in[row * rb_words + (size_t)c * 4 + wi];
      v = FMT == kTern2 ? perm_tern(w) : perm_sign(w);
    }
    out[i] = v;
  }
}

// scales: canonical [M][G] fp16 -> [ntiles][G][32]
__global__ void repack_scales_kernel(const uint16_t* __restrict__ in, uint16_t* __restrict__ out,
                                     int M, int G, size_t ndev) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < ndev;
       i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i % kTileRows);
    const size_t tg = i / kTileRows;
    const int g = (int)(tg % G);
    const size_t t = tg / G;
    const size_t row = t * kTileRows + r;
    out[i] = row < (size_t)M ? in[row * G + g] : (uint16_t)0;
  }
}

unsigned grid_for(size_t n) {
  const size_t blocks = (n + 255) / 256;
  return (unsigned)(blocks < 148 * 64 ? blocks : 148 * 64);
}

}  // namespace

size_t tiled_weight_bytes(int fmt, int M, int K) {
  const size_t rb = fmt == kTern2 ? (size_t)K / 4 : (size_t)K / 8;
  return (size_t)((M + kTileRows - 1) / kTileRows) * kTileRows * rb;
}

size_t tiled_scale_bytes(int M, int K) {
  return (size_t)((M + kTileRows - 1) / kTileRows) * kTileRows * (K / 128) * 2;
}

cudaError_t launch_repack(int fmt, const uint8_t* canon, uint8_t* dev, int M, int K, cudaStream_t s) {
  const int rb_words = fmt == kTern2 ? K / 16 : K / 32;
  const size_t ndev = tiled_weight_bytes(fmt, M, K) / 4;
  if (ndev == 0) return cudaSuccess;
  if (fmt == kTern2)
    repack_kernel<kTern2><<<grid_for(ndev), 256, 0, s>>>(reinterpret_cast<const uint32_t*>(canon),
                                                          reinterpret_cast<uint32_t*>(dev), M,
                                                          rb_words, ndev);
  else
    repack_kernel<kSign1><<<grid_for(ndev), 256, 0, s>>>(reinterpret_cast<const uint32_t*>(canon),
                                                          reinterpret_cast<uint32_t*>(dev), M,
                                                          rb_words, ndev);
  return cudaGetLastError();
}

cudaError_t launch_repack_scales(const uint16_t* canon, uint16_t* dev, int M, int K,
                                 cudaStream_t s) {
  const size_t ndev = tiled_scale_bytes(M, K) / 2;
  if (ndev == 0) return cudaSuccess;
  repack_scales_kernel<<<grid_for(ndev), 256, 0, s>>>(canon, dev, M, K / 128, ndev);
  return cudaGetLastError();
}

}  // namespace ouroq
