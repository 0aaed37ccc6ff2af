// quant.cu -- K1: fused blockwise Walsh-Hadamard rotation + per-token absmax
// int8 quantisation, and the fp32 rotate_fwd / rotate_inv operators.
//
// Reference semantics:
//   rotate_fwd  cluster/src/infer/hadamard.rs:41-53  (v *= s; WHT per block; v *= 1/sqrt(N))
//   rotate_inv  cluster/src/infer/hadamard.rs:57-66  (WHT per block; v *= s * (1/sqrt(N)))
//   butterfly   cluster/src/infer/hadamard.rs:15-31  (h = 1, 2, 4, ...; lo = a+b, hi = a-b)
// The butterfly network here pairs the same elements in the same stage order,
// so every output is the same sequence of IEEE adds as the reference and the
// rotation is bit-identical to it. All float ops use explicit _rn intrinsics
// so the compiler cannot contract them into fused multiply-adds.
//
// Quantisation (north_star K1; not in the reference): s_x = absmax / 127,
// q = clamp(rint(v / s_x), -127, 127), s_x == 0 -> q = 0.
//
// One CTA per (token, job). The token row is staged in shared memory; each
// warp rotates spans of 32*E elements with E = max(1, block/32) elements per
// lane: butterfly stages h < E run in registers, stages h >= E exchange with
// lane ^ (h/E) through warp shuffles.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace ouroq {
namespace {

constexpr int kQuantThreads = 256;

template <int E>
__device__ __forceinline__ void wht_span(float* v, int lane, int block) {
  // in-register stages: h = 1 .. E/2 (element distance within the lane)
#pragma unroll
  for (int h = 1; h < E; h <<= 1) {
#pragma unroll
    for (int i = 0; i < E; ++i) {
      if ((i & h) == 0) {
        float a = v[i], b = v[i + h];
        v[i] = __fadd_rn(a, b);
        v[i + h] = __fsub_rn(a, b);
      }
    }
  }
  // cross-lane stages: element distance h = E*m for lane distance m
  for (int m = 1; m * E < block; m <<= 1) {
    const bool hi = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      float other = __shfl_xor_sync(0xffffffffu, v[i], m);
      // lower index keeps a+b, upper index gets a-b with a = lower element
      v[i] = hi ? __fsub_rn(other, v[i]) : __fadd_rn(v[i], other);
    }
  }
}

// mode 0: (optional rotate_fwd) + quantise; mode 1: rotate_fwd only; mode 2: rotate_inv only
template <int E>
__device__ void rotate_row(float* row, const float* signs, int K, int block, float scale,
                           int mode) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int span = 32 * E;
  for (int base = warp * span; base < K; base += nwarps * span) {
    float v[E];
    const int off = base + lane * E;
    // Only spans narrower than 32 elements (block < 32) can overhang K; the
    // overhanging lanes form whole blocks of their own, so their zeros never
    // mix with valid elements in the shuffles below.
    const bool valid = off < K;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      float t = valid ? row[off + i] : 0.0f;
      if (valid && mode != 2 && signs) t = __fmul_rn(t, signs[off + i]);
      v[i] = t;
    }
    wht_span<E>(v, lane, block);
    if (valid) {
#pragma unroll
      for (int i = 0; i < E; ++i) {
        float t = v[i];
        if (mode == 2)
          t = __fmul_rn(t, __fmul_rn(signs ? signs[off + i] : 1.0f, scale));
        else
          t = __fmul_rn(t, scale);
        row[off + i] = t;
      }
    }
  }
}

__device__ void rotate_dispatch(float* row, const float* signs, int K, int block, float scale,
                                int mode) {
  switch (block) {
    case 2: case 4: case 8: case 16: case 32: rotate_row<1>(row, signs, K, block, scale, mode); break;
    case 64: rotate_row<2>(row, signs, K, block, scale, mode); break;
    case 128: rotate_row<4>(row, signs, K, block, scale, mode); break;
    case 256: rotate_row<8>(row, signs, K, block, scale, mode); break;
    case 512: rotate_row<16>(row, signs, K, block, scale, mode); break;
    case 1024: rotate_row<32>(row, signs, K, block, scale, mode); break;
    default: break;  // rejected on the host
  }
}

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
    rotate_dispatch(row, J.signs, K, J.had_block, J.had_scale, 0);
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
  if (threadIdx.x == 0) J.s_x[b] = s;

  int8_t* q = J.q + (size_t)b * K;
  for (int i = threadIdx.x * 4; i < K; i += blockDim.x * 4) {
    char4 o;
    int v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int iv = 0;
      if (s != 0.0f) {
        float r = rintf(__fdiv_rn(row[i + e], s));
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        iv = (int)r;
      }
      v[e] = iv;
    }
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
  rotate_dispatch(row, signs, K, block, scale, inverse ? 2 : 1);
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
