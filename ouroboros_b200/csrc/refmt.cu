// refmt.cu -- GPU decode of the reference's own ternary shard formats behind
// matvec_q / matmul_q: fp32 activations in, fp32 outputs out, no activation
// quantisation. Both kernels reproduce the reference's floating-point
// operation order exactly, so their outputs are bit-identical to it.
//
// PTQ1_0 ("Tl1", cluster/src/infer/dequant.rs:123-171): groups of 128 weights
//   in 28 bytes: qs[24] | qh[2] | f16 d. Element order: n*16+m for qs[0..16],
//   80+n*8+m for qs[16..24], 120+n*2+m for qh[0..2]. Trit of byte b at digit n:
//   q = b*3^n mod 256, t = ((q*3) >> 8) - 1 (dequant.rs:134-138).
//   Order = tl1_rows_avx2 (ops.rs:499-584), the reference's x86 path: per
//   group four lane accumulators, lane j adding, for n = 0..4, the terms of
//   bytes qs[j], qs[4+j], qs[8+j], qs[12+j], qs[16+j], qs[20+j]; each term is
//   ((float)t * d) * x with separate multiplies and an add (no FMA). The row sum
//   then adds the eight qh terms in order (n, m) and the group's
//   hsum = (acc0 + acc2) + (acc1 + acc3), group after group.
// TQ1_0 (dequant.rs:50-105): blocks of 256 weights in 54 bytes:
//   qs[48] | qh[4] | f16 d; element order qs[0..32] x 5 digits, qs[32..48] x 5,
//   qh x 4. Order = matvec_qblock (ops.rs:101-128): dequantise the row,
//   w = ((float)digit - 1) * d, then dot (ops.rs:53-60): s += w * x in
//   element order, one running sum.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace ouroq {
namespace {

__device__ __forceinline__ int ptq1_digit(uint32_t byte, uint32_t pow3) {
  const uint32_t q = (byte * pow3) & 0xFFu;
  return (int)((q * 3u) >> 8);
}

// ((float)t * d) * x, t = digit - 1
__device__ __forceinline__ float term(uint32_t byte, uint32_t pow3, float d, float x) {
  const float t = (float)(ptq1_digit(byte, pow3) - 1);
  return __fmul_rn(__fmul_rn(t, d), x);
}

constexpr int kTl1Threads = 256;
constexpr int kTl1XStride = 129;  // padded group stride of x in shared memory (bank spread)

// grid (row blocks, tokens). R rows per CTA; work item = (row, group).
__global__ void __launch_bounds__(kTl1Threads) tl1_matvec_kernel(const __grid_constant__ RefLaunch P,
                                                                int R) {
  extern __shared__ float sm[];
  const int G = P.K / 128;
  float* xs = sm;                                  // [G][129]
  float* part = sm + (size_t)G * kTl1XStride;      // [R*G][9]: eight qh terms + hsum
  const int b = blockIdx.y;
  const int row0 = blockIdx.x * R;
  const float* x = P.x + (size_t)b * P.K;
  for (int i = threadIdx.x; i < P.K; i += blockDim.x) xs[(i >> 7) * kTl1XStride + (i & 127)] = x[i];
  __syncthreads();
  const uint32_t pw[5] = {1u, 3u, 9u, 27u, 81u};
  for (int p = threadIdx.x; p < R * G; p += blockDim.x) {
    const int r = p / G, g = p - (p / G) * G;
    const int row = row0 + r;
    if (row >= P.M) continue;
    const uint32_t* gw = reinterpret_cast<const uint32_t*>(P.w + ((size_t)row * G + g) * 28);
    uint32_t wd[7];
#pragma unroll
    for (int i = 0; i < 7; ++i) wd[i] = __ldg(gw + i);
    const float d = __half2float(__ushort_as_half((unsigned short)(wd[6] >> 16)));
    const float* xg = xs + g * kTl1XStride;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int n = 0; n < 5; ++n) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int sh = 8 * j;
        acc[j] = __fadd_rn(term((wd[0] >> sh) & 0xFFu, pw[n], d, xg[n * 16 + j]), acc[j]);
        acc[j] = __fadd_rn(term((wd[1] >> sh) & 0xFFu, pw[n], d, xg[n * 16 + 4 + j]), acc[j]);
        acc[j] = __fadd_rn(term((wd[2] >> sh) & 0xFFu, pw[n], d, xg[n * 16 + 8 + j]), acc[j]);
        acc[j] = __fadd_rn(term((wd[3] >> sh) & 0xFFu, pw[n], d, xg[n * 16 + 12 + j]), acc[j]);
        acc[j] = __fadd_rn(term((wd[4] >> sh) & 0xFFu, pw[n], d, xg[80 + n * 8 + j]), acc[j]);
        acc[j] = __fadd_rn(term((wd[5] >> sh) & 0xFFu, pw[n], d, xg[80 + n * 8 + 4 + j]), acc[j]);
      }
    }
    float* out = part + (size_t)p * 9;
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int m = 0; m < 2; ++m) out[n * 2 + m] = term((wd[6] >> (8 * m)) & 0xFFu, pw[n], d, xg[120 + n * 2 + m]);
    out[8] = __fadd_rn(__fadd_rn(acc[0], acc[2]), __fadd_rn(acc[1], acc[3]));
  }
  __syncthreads();
  // the row sum: group after group, eight tail terms then the group's hsum
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const int row = row0 + r;
    if (row >= P.M) continue;
    float sum = 0.0f;
    const float* pr = part + (size_t)r * G * 9;
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int k = 0; k < 9; ++k) sum = __fadd_rn(sum, pr[g * 9 + k]);
    }
    P.y[(size_t)b * P.ldy + row] = sum;
  }
}

// TQ1_0: a team of 8 lanes per row. Per 256-element block the team decodes
// the weights times x into shared memory (element order), then the team's
// first lane adds them up in order -- the running sum is the only serial part.
constexpr int kTq1Threads = 256;
constexpr int kTq1Rows = kTq1Threads / 8;   // 32 rows per CTA
constexpr int kTq1ProdStride = 257;         // padded row stride of the product buffer

__device__ __forceinline__ int tq1_byte_of(int e, int* n) {
  if (e < 160) {
    *n = e >> 5;
    return e & 31;
  }
  if (e < 240) {
    const int f = e - 160;
    *n = f >> 4;
    return 32 + (f & 15);
  }
  const int f = e - 240;
  *n = f >> 2;
  return 48 + (f & 3);
}

__global__ void __launch_bounds__(kTq1Threads) tq1_matvec_kernel(const __grid_constant__ RefLaunch P) {
  extern __shared__ float sm[];
  float* xs = sm;                                   // [K]
  float* prod = sm + P.K;                           // [32 rows][257]
  const int b = blockIdx.y;
  const float* x = P.x + (size_t)b * P.K;
  for (int i = threadIdx.x; i < P.K; i += blockDim.x) xs[i] = x[i];
  __syncthreads();
  const int team = threadIdx.x >> 3, k = threadIdx.x & 7;
  const int row = blockIdx.x * kTq1Rows + team;
  const bool live = row < P.M;
  const int nblk = P.K / 256;
  const size_t rb = (size_t)nblk * 54;
  const uint8_t* wr = P.w + (size_t)(live ? row : 0) * rb;
  float* pr = prod + team * kTq1ProdStride;
  const uint32_t pw[5] = {1u, 3u, 9u, 27u, 81u};
  // the 8 lanes of a team sit in one warp: team lanes = 8 consecutive lanes
  const unsigned team_mask = 0xFFu << ((threadIdx.x & 31) & ~7);
  float sum = 0.0f;
  for (int blk = 0; blk < nblk; ++blk) {
    const uint8_t* bb = wr + (size_t)blk * 54;
    if (live) {
      const float d =
          __half2float(__ushort_as_half((unsigned short)(bb[52] | ((unsigned)bb[53] << 8))));
      const float* xb = xs + blk * 256;
      for (int e = k; e < 256; e += 8) {
        int n;
        const int byte_idx = tq1_byte_of(e, &n);
        const float w = __fmul_rn(__fsub_rn((float)ptq1_digit(bb[byte_idx], pw[n]), 1.0f), d);
        pr[e] = __fmul_rn(w, xb[e]);
      }
    }
    __syncwarp(team_mask);
    if (k == 0 && live) {
      for (int e = 0; e < 256; ++e) sum = __fadd_rn(sum, pr[e]);
    }
    __syncwarp(team_mask);
  }
  if (k == 0 && live) P.y[(size_t)b * P.ldy + row] = sum;
}

}  // namespace

size_t tl1_smem_bytes(int K, int R) {
  const int G = K / 128;
  return ((size_t)G * kTl1XStride + (size_t)R * G * 9) * sizeof(float);
}

int tl1_rows_per_cta(int K) {
  const int G = K / 128;
  int R = 1024 / G;
  return R < 1 ? 1 : R;
}

size_t tq1_smem_bytes(int K) { return ((size_t)K + (size_t)kTq1Rows * kTq1ProdStride) * sizeof(float); }

cudaError_t launch_refmt_matvec(const RefLaunch& P, cudaStream_t s) {
  if (P.M <= 0 || P.B <= 0) return cudaSuccess;
  if (P.fmt == kPtq1) {
    const int R = tl1_rows_per_cta(P.K);
    const size_t smem = tl1_smem_bytes(P.K, R);
    cudaError_t e = ensure_max_smem<tl1_matvec_kernel>();
    if (e != cudaSuccess) return e;
    const dim3 grid((unsigned)((P.M + R - 1) / R), (unsigned)P.B, 1);
    tl1_matvec_kernel<<<grid, kTl1Threads, smem, s>>>(P, R);
    return cudaGetLastError();
  }
  if (P.fmt == kTq1) {
    const size_t smem = tq1_smem_bytes(P.K);
    cudaError_t e = ensure_max_smem<tq1_matvec_kernel>();
    if (e != cudaSuccess) return e;
    const dim3 grid((unsigned)((P.M + kTq1Rows - 1) / kTq1Rows), (unsigned)P.B, 1);
    tq1_matvec_kernel<<<grid, kTq1Threads, smem, s>>>(P);
    return cudaGetLastError();
  }
  return cudaErrorInvalidValue;
}

}  // namespace ouroq
