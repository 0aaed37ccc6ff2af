// quant.cu -- K1: fused blockwise Walsh-Hadamard rotation + per-token absmax
// int8 quantisation, and the fp32 rotate_fwd / rotate_inv operators.
//
// Reference semantics:
//   rotate_fwd  cluster/src/infer/hadamard.rs:41-53  (v *= s; WHT per block; v *= 1/sqrt(N))
//   rotate_inv  cluster/src/infer/hadamard.rs:57-66  (WHT per block; v *= s * (1/sqrt(N)))
//   butterfly   cluster/src/infer/hadamard.rs:15-31  (h = 1, 2, 4, ...; lo = a+b, hi = a-b)
// The rotation is bit-identical to the reference (see hadamard.cuh).
//
// Per-token absmax quantisation (kernel K1; not in the reference): s_x = absmax / 127,
// q = clamp(rint(v / s_x), -127, 127), s_x == 0 -> q = 0.
//
// One CTA per (token, job). The token row is staged in shared memory and
// rotated by the butterflies of hadamard.cuh.
#include <cuda_runtime.h>

#include "common.cuh"
#include "hadamard.cuh"
#include "kernels.h"

namespace ouroq {
namespace {

constexpr int kQuantThreads = 256;

__global__ void __launch_bounds__(kQuantThreads) quantize_kernel(const __grid_constant__ QuantLaunch L) {
  extern __shared__ __align__(16) float row[];
  __shared__ float red[kQuantThreads / 32];
  pdl_launch_dependents();
  pdl_wait();

  const QuantJob& J = L.jobs[blockIdx.y];
  const int b = blockIdx.x;
  const int K = J.K;
  const float* x = J.x + (size_t)b * K;

  // stage the token row (K % 4 == 0, 16-byte aligned rows checked on the host)
  for (int i = threadIdx.x * 4; i < K; i += blockDim.x * 4) {
    float4 t = *reinterpret_cast<const float4*>(x + i);
    *reinterpret_cast<float4*>(row + i) = t;
  }
  __syncthreads();
  if (J.had_block > 0) {
    rotate_dispatch(row, J.signs, K, J.had_block, J.had_scale, 0, threadIdx.x >> 5, blockDim.x >> 5);
    __syncthreads();
    if (J.x_rot) {
      float* xr = J.x_rot + (size_t)b * K;
      for (int i = threadIdx.x; i < K; i += blockDim.x) xr[i] = row[i];
    }
  }

  float amax = 0.0f;
  for (int i = threadIdx.x; i < K; i += blockDim.x) amax = fmaxf(amax, fabsf(row[i]));
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    t = warp_max(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float s = __fdiv_rn(red[0], 127.0f);
  const float rs = __frcp_rn(s);
  if (threadIdx.x == 0) J.s_x[b] = s;

  int8_t* q = J.q + (size_t)b * K;
  for (int i = threadIdx.x * 4; i < K; i += blockDim.x * 4) {
    char4 o;
    int v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = quant_code(row[i + e], s, rs);
    o.x = (signed char)v[0];
    o.y = (signed char)v[1];
    o.z = (signed char)v[2];
    o.w = (signed char)v[3];
    *reinterpret_cast<char4*>(q + i) = o;
  }
}

__global__ void __launch_bounds__(kQuantThreads)
    rotate_kernel(const float* __restrict__ x, float* __restrict__ out,
                  const float* __restrict__ signs, int K, int block, float scale, int inverse) {
  extern __shared__ __align__(16) float row[];
  const int b = blockIdx.x;
  const float* xr = x + (size_t)b * K;
  for (int i = threadIdx.x; i < K; i += blockDim.x) row[i] = xr[i];
  __syncthreads();
  rotate_dispatch(row, signs, K, block, scale, inverse ? 2 : 1, threadIdx.x >> 5, blockDim.x >> 5);
  __syncthreads();
  float* o = out + (size_t)b * K;
  for (int i = threadIdx.x; i < K; i += blockDim.x) o[i] = row[i];
}

}  // namespace

cudaError_t launch_quantize(const QuantLaunch& L, cudaStream_t s, bool pdl) {
  if (L.B <= 0 || L.njobs <= 0) return cudaSuccess;
  int maxK = 0;
  for (int j = 0; j < L.njobs; ++j) maxK = L.jobs[j].K > maxK ? L.jobs[j].K : maxK;
  size_t smem = (size_t)maxK * sizeof(float);
  cudaError_t e = ensure_max_smem<quantize_kernel>();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(L.B, L.njobs, 1);
  cfg.blockDim = dim3(kQuantThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, quantize_kernel, L);
}

cudaError_t launch_rotate(const float* x, float* out, const float* signs, int B, int K, int block,
                          float scale, int inverse, cudaStream_t s) {
  if (B <= 0) return cudaSuccess;
  size_t smem = (size_t)K * sizeof(float);
  cudaError_t e = ensure_max_smem<rotate_kernel>();
  if (e != cudaSuccess) return e;
  rotate_kernel<<<B, kQuantThreads, smem, s>>>(x, out, signs, K, block, scale, inverse);
  return cudaGetLastError();
}

}  // namespace ouroq
