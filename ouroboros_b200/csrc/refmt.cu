// refmt.cu -- GPU decode of the reference's own ternary shard formats behind
// matvec_q / matmul_q: fp32 activations in, fp32 outputs out, no activation
// quantisation. Every kernel reproduces the reference's floating-point
// operation order exactly, so its outputs are bit-identical to it: PTQ1_0 in
// matvec_tl1's order for one token and in matmul_tl1's K-column order for a
// batch (tl1_columns_kernel, below), TQ1_0 in matvec_qblock's order.
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

// Next digit of a byte: with q = byte * 3^n mod 256 in *q, returns digit n
// ((q * 3) >> 8) and leaves byte * 3^(n+1) mod 256 in *q.
__device__ __forceinline__ uint32_t next_digit(uint32_t* q) {
  const uint32_t q3 = *q * 3u;
  *q = q3 & 0xFFu;
  return q3 >> 8;
}

// ((float)(digit - 1) * d) * x, exactly as the reference rounds it (the digit
// is 0, 1 or 2, so the trit is selected rather than converted).
__device__ __forceinline__ float term(uint32_t digit, float d, float x) {
  const float t = digit == 0u ? -1.0f : (digit == 1u ? 0.0f : 1.0f);
  return __fmul_rn(__fmul_rn(t, d), x);
}

constexpr int kTl1Threads = 256;
constexpr int kTl1XStride = 129;  // padded group stride of x in shared memory (bank spread)

// grid (row blocks, tokens). R rows per CTA; work item = (row, group).
__global__ void __launch_bounds__(kTl1Threads, 2) tl1_matvec_kernel(const __grid_constant__ RefLaunch P,
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
  // the next work item's 28 bytes are fetched while the current one is decoded
  uint32_t nwd[7];
  auto fetch = [&](int p, uint32_t* out) {
    const int r = p / G, g = p - (p / G) * G;
    const int row = row0 + r < P.M ? row0 + r : P.M - 1;
    const uint32_t* gw = reinterpret_cast<const uint32_t*>(P.w + ((size_t)row * G + g) * 28);
#pragma unroll
    for (int i = 0; i < 7; ++i) out[i] = __ldg(gw + i);
  };
  if (threadIdx.x < R * G) fetch(threadIdx.x, nwd);
  for (int p = threadIdx.x; p < R * G; p += blockDim.x) {
    const int r = p / G, g = p - (p / G) * G;
    const int row = row0 + r;
    uint32_t wd[7];
#pragma unroll
    for (int i = 0; i < 7; ++i) wd[i] = nwd[i];
    if (p + (int)blockDim.x < R * G) fetch(p + blockDim.x, nwd);
    if (row >= P.M) continue;
    const float d = __half2float(__ushort_as_half((unsigned short)(wd[6] >> 16)));
    const float* xg = xs + g * kTl1XStride;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    uint32_t q[24];  // byte * 3^n mod 256 of qs[0..24], advanced one digit per n
#pragma unroll
    for (int i = 0; i < 24; ++i) q[i] = (wd[i >> 2] >> (8 * (i & 3))) & 0xFFu;
#pragma unroll 1
    for (int n = 0; n < 5; ++n) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // lane j: bytes j, 4+j, 8+j, 12+j, 16+j, 20+j (three digits8 calls of ops.rs:553-557)
        acc[j] = __fadd_rn(term(next_digit(&q[j]), d, xg[n * 16 + j]), acc[j]);
        acc[j] = __fadd_rn(term(next_digit(&q[4 + j]), d, xg[n * 16 + 4 + j]), acc[j]);
        acc[j] = __fadd_rn(term(next_digit(&q[8 + j]), d, xg[n * 16 + 8 + j]), acc[j]);
        acc[j] = __fadd_rn(term(next_digit(&q[12 + j]), d, xg[n * 16 + 12 + j]), acc[j]);
        acc[j] = __fadd_rn(term(next_digit(&q[16 + j]), d, xg[80 + n * 8 + j]), acc[j]);
        acc[j] = __fadd_rn(term(next_digit(&q[20 + j]), d, xg[80 + n * 8 + 4 + j]), acc[j]);
      }
    }
    float* out = part + (size_t)p * 9;
    uint32_t qh[2] = {wd[6] & 0xFFu, (wd[6] >> 8) & 0xFFu};
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int m = 0; m < 2; ++m)
        out[n * 2 + m] = term(next_digit(&qh[m]), d, xg[120 + n * 2 + m]);
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

// PTQ1_0 times K columns in matmul_tl1's x86 order (tl1_rows_avx2_k,
// ops.rs:381-481; matmul_q takes it for every K, ops.rs:219-230): for each
// (row, column) two 4-lane accumulators a, b run over the whole row -- a lane
// j takes the terms of bytes j, 8+j, 16+j of each stage n (x at n*16+j,
// n*16+8+j, 80+n*8+j), b lane j those of bytes 4+j, 12+j, 20+j (x at
// n*16+4+j, n*16+12+j, 80+n*8+4+j) -- and one scalar tail sum takes the eight
// qh terms, group after group; y = tail + (hsum(a) + hsum(b)) with
// hsum(v) = (v0 + v2) + (v1 + v3). One thread per (row, column), 32 rows a
// CTA; the columns of a row read its weights through the read-only cache.
constexpr int kTl1ColThreads = 256;
constexpr int kTl1ColRows = 32;

__global__ void __launch_bounds__(kTl1ColThreads) tl1_columns_kernel(const __grid_constant__ RefLaunch P) {
  const int G = P.K / 128;
  const int k = P.B;
  const int row0 = blockIdx.x * kTl1ColRows;
  for (int p = threadIdx.x; p < kTl1ColRows * k; p += blockDim.x) {
    const int r = p / k, c = p - (p / k) * k;
    const int row = row0 + r;
    if (row >= P.M) continue;
    const float* x = P.x + (size_t)c * P.K;
    float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float bv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float tail = 0.0f;
#pragma unroll 1
    for (int g = 0; g < G; ++g) {
      const uint32_t* gw = reinterpret_cast<const uint32_t*>(P.w + ((size_t)row * G + g) * 28);
      uint32_t wd[7];
#pragma unroll
      for (int i = 0; i < 7; ++i) wd[i] = __ldg(gw + i);
      const float d = __half2float(__ushort_as_half((unsigned short)(wd[6] >> 16)));
      const float* xg = x + (size_t)g * 128;
      uint32_t q[24];  // byte * 3^n mod 256 of qs[0..24], advanced one digit per n
#pragma unroll
      for (int i = 0; i < 24; ++i) q[i] = (wd[i >> 2] >> (8 * (i & 3))) & 0xFFu;
#pragma unroll 1
      for (int n = 0; n < 5; ++n) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          a[j] = __fadd_rn(term(next_digit(&q[j]), d, __ldg(xg + n * 16 + j)), a[j]);
          bv[j] = __fadd_rn(term(next_digit(&q[4 + j]), d, __ldg(xg + n * 16 + 4 + j)), bv[j]);
          a[j] = __fadd_rn(term(next_digit(&q[8 + j]), d, __ldg(xg + n * 16 + 8 + j)), a[j]);
          bv[j] = __fadd_rn(term(next_digit(&q[12 + j]), d, __ldg(xg + n * 16 + 12 + j)), bv[j]);
          a[j] = __fadd_rn(term(next_digit(&q[16 + j]), d, __ldg(xg + 80 + n * 8 + j)), a[j]);
          bv[j] = __fadd_rn(term(next_digit(&q[20 + j]), d, __ldg(xg + 80 + n * 8 + 4 + j)), bv[j]);
        }
      }
      uint32_t qh[2] = {wd[6] & 0xFFu, (wd[6] >> 8) & 0xFFu};
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int m = 0; m < 2; ++m)
          tail = __fadd_rn(tail, term(next_digit(&qh[m]), d, __ldg(xg + 120 + n * 2 + m)));
    }
    const float ha = __fadd_rn(__fadd_rn(a[0], a[2]), __fadd_rn(a[1], a[3]));
    const float hb = __fadd_rn(__fadd_rn(bv[0], bv[2]), __fadd_rn(bv[1], bv[3]));
    P.y[(size_t)c * P.ldy + row] = __fadd_rn(tail, __fadd_rn(ha, hb));
  }
}

// TQ1_0: 32 rows per CTA, four warps. Warps 1-3 decode the weights of a
// 256-element block times x into a double-buffered product tile [32 rows][256];
// warp 0 (lane = row) adds each row's products in element order -- the one
// serial chain of the reference's dot. Named barriers hand the buffers over.
constexpr int kTq1Warps = 4;
constexpr int kTq1Threads = kTq1Warps * 32;
constexpr int kTq1Rows = 32;
constexpr int kTq1ProdStride = 257;  // padded row stride: lanes of a warp hit distinct banks

__device__ __forceinline__ void bar_sync(unsigned id, unsigned n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_arrive(unsigned id, unsigned n) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// element index of digit n of code byte m in a TQ1_0 block (dequant.rs:61-79)
__device__ __forceinline__ int tq1_elem(int m, int n) {
  return m < 32 ? n * 32 + m : (m < 48 ? 160 + n * 16 + (m - 32) : 240 + n * 4 + (m - 48));
}

__global__ void __launch_bounds__(kTq1Threads) tq1_matvec_kernel(const __grid_constant__ RefLaunch P) {
  extern __shared__ float sm[];
  float* xs = sm;                  // [K]
  float* prod = sm + P.K;          // [2][32][257]
  const int b = blockIdx.y;
  const float* x = P.x + (size_t)b * P.K;
  for (int i = threadIdx.x; i < P.K; i += blockDim.x) xs[i] = x[i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kTq1Rows + lane;
  const bool live = row < P.M;
  const int nblk = P.K / 256;
  const uint8_t* wr = P.w + (size_t)(live ? row : 0) * ((size_t)nblk * 54);
  // barrier ids: 1 + buf = "products of buf ready", 3 + buf = "buf free"
  if (warp == 0) {
    float sum = 0.0f;
    for (int blk = 0; blk < nblk; ++blk) {
      const int buf = blk & 1;
      bar_sync(1 + buf, kTq1Threads);
      const float* src = prod + (size_t)buf * kTq1Rows * kTq1ProdStride + lane * kTq1ProdStride;
      for (int e = 0; e < 256; e += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = src[e + j];
#pragma unroll
        for (int j = 0; j < 8; ++j) sum = __fadd_rn(sum, v[j]);
      }
      if (blk + 2 < nblk) bar_arrive(3 + buf, kTq1Threads);  // the decoders refill buf
    }
    if (live) P.y[(size_t)b * P.ldy + row] = sum;
  } else {
    const int dw = warp - 1;  // decode warp 0..2: code bytes m = dw, dw + 3, ...
    constexpr int kSlots = (52 + kTq1Warps - 2) / (kTq1Warps - 1);  // 18 bytes per lane per block
    // this lane's code bytes and scale of a block, all loads issued together;
    // the next block's are fetched while the current one is decoded
    auto fetch = [&](int blk, uint32_t* by, float* d) {
      const uint8_t* bb = wr + (size_t)blk * 54;
#pragma unroll
      for (int i = 0; i < kSlots; ++i) {
        const int m = dw + (kTq1Warps - 1) * i;
        by[i] = m < 52 ? (uint32_t)__ldg(bb + m) : 0u;
      }
      *d = __half2float(__ushort_as_half((unsigned short)(__ldg(bb + 52) | ((unsigned)__ldg(bb + 53) << 8))));
    };
    uint32_t cur[kSlots], nxt[kSlots];
    float dcur = 0.0f, dnxt = 0.0f;
    fetch(0, cur, &dcur);
    for (int blk = 0; blk < nblk; ++blk) {
      const int buf = blk & 1;
      if (blk + 1 < nblk) fetch(blk + 1, nxt, &dnxt);
      if (blk >= 2) bar_sync(3 + buf, kTq1Threads);
      float* dst = prod + (size_t)buf * kTq1Rows * kTq1ProdStride + lane * kTq1ProdStride;
      const float* xb = xs + blk * 256;
#pragma unroll
      for (int i = 0; i < kSlots; ++i) {
        const int m = dw + (kTq1Warps - 1) * i;
        if (m >= 52) continue;
        uint32_t q = cur[i];
        const int nd = m < 48 ? 5 : 4;
        for (int n = 0; n < nd; ++n) {
          const uint32_t q3 = q * 3u;
          q = q3 & 0xFFu;
          const int e = tq1_elem(m, n);
          // w = ((float)digit - 1) * d, then w * x (the dot's product)
          const float w = __fmul_rn((float)(q3 >> 8) - 1.0f, dcur);
          dst[e] = __fmul_rn(w, xb[e]);
        }
      }
#pragma unroll
      for (int i = 0; i < kSlots; ++i) cur[i] = nxt[i];
      dcur = dnxt;
      bar_arrive(1 + buf, kTq1Threads);
    }
  }
}

// The same K-column order with each group's trits decoded once per row for
// all the columns of a block (up to kTl1BlkCols at a time): thread = (row,
// lane j), lane j carrying a[j] and b[j] of every column of the block (lane 0
// also the tail), the four lanes of a row combined by shuffles at the end --
// the same additions in the same order as tl1_columns_kernel, per column.
// x of the block sits in shared memory column-interleaved, a chunk of groups
// at a time, so one 16-byte load gives four columns' x of one element.
constexpr int kTl1BlkCols = 8;
constexpr int kTl1BlkRows = 64;
constexpr int kTl1BlkThreads = kTl1BlkRows * 4;
constexpr int kTl1BlkChunk = 8;  // groups of x staged at a time (32 KB)

__global__ void __launch_bounds__(kTl1BlkThreads) tl1_colblock_kernel(const __grid_constant__ RefLaunch P) {
  __shared__ __align__(16) float xs[kTl1BlkChunk * 128 * kTl1BlkCols];
  const int G = P.K / 128;
  const int c0 = blockIdx.y * kTl1BlkCols;
  const int nc = P.B - c0 < kTl1BlkCols ? P.B - c0 : kTl1BlkCols;
  const int r = threadIdx.x >> 2, j = threadIdx.x & 3;
  const int row = blockIdx.x * kTl1BlkRows + r;
  const bool live = row < P.M;
  float a[kTl1BlkCols], bv[kTl1BlkCols], tail[kTl1BlkCols];
#pragma unroll
  for (int c = 0; c < kTl1BlkCols; ++c) a[c] = bv[c] = tail[c] = 0.0f;
  for (int g0 = 0; g0 < G; g0 += kTl1BlkChunk) {
    const int ng = G - g0 < kTl1BlkChunk ? G - g0 : kTl1BlkChunk;
    __syncthreads();  // the previous chunk's x is no longer read
    for (int i = threadIdx.x; i < ng * 128 * kTl1BlkCols; i += kTl1BlkThreads) {
      const int e = i / kTl1BlkCols, c = i - e * kTl1BlkCols;
      xs[i] = c < nc ? P.x[(size_t)(c0 + c) * P.K + (size_t)g0 * 128 + e] : 0.0f;
    }
    __syncthreads();
    if (!live) continue;
    for (int gi = 0; gi < ng; ++gi) {
      const uint32_t* gw = reinterpret_cast<const uint32_t*>(P.w + ((size_t)row * G + g0 + gi) * 28);
      uint32_t wd[7];
#pragma unroll
      for (int i = 0; i < 7; ++i) wd[i] = __ldg(gw + i);
      const float d = __half2float(__ushort_as_half((unsigned short)(wd[6] >> 16)));
      const float* xg = xs + gi * 128 * kTl1BlkCols;
      // lane j's bytes: qs[j + 4i] = byte j of word i, i = 0..5
      uint32_t q[6];
#pragma unroll
      for (int i = 0; i < 6; ++i) q[i] = (wd[i] >> (8 * j)) & 0xFFu;
      auto apply = [&](uint32_t digit, int e, float* acc) {
        const float t = digit == 0u ? -1.0f : (digit == 1u ? 0.0f : 1.0f);
        const float td = __fmul_rn(t, d);
        const float4* xp = reinterpret_cast<const float4*>(xg + e * kTl1BlkCols);
        const float4 x0 = xp[0], x1 = xp[1];
        const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int c = 0; c < kTl1BlkCols; ++c) acc[c] = __fadd_rn(__fmul_rn(td, xv[c]), acc[c]);
      };
#pragma unroll 1
      for (int n = 0; n < 5; ++n) {
        apply(next_digit(&q[0]), n * 16 + j, a);
        apply(next_digit(&q[1]), n * 16 + 4 + j, bv);
        apply(next_digit(&q[2]), n * 16 + 8 + j, a);
        apply(next_digit(&q[3]), n * 16 + 12 + j, bv);
        apply(next_digit(&q[4]), 80 + n * 8 + j, a);
        apply(next_digit(&q[5]), 80 + n * 8 + 4 + j, bv);
      }
      if (j == 0) {
        uint32_t qh[2] = {wd[6] & 0xFFu, (wd[6] >> 8) & 0xFFu};
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int m = 0; m < 2; ++m) apply(next_digit(&qh[m]), 120 + n * 2 + m, tail);
      }
    }
  }
  // hsum(a) = (a0 + a2) + (a1 + a3) over the lanes of the row, likewise b
  const unsigned lanes = 0xffffffffu;
  const int base = (threadIdx.x & 31) & ~3;
#pragma unroll
  for (int c = 0; c < kTl1BlkCols; ++c) {
    const float a1 = __shfl_sync(lanes, a[c], base + 1), a2 = __shfl_sync(lanes, a[c], base + 2),
                a3 = __shfl_sync(lanes, a[c], base + 3);
    const float b1 = __shfl_sync(lanes, bv[c], base + 1), b2 = __shfl_sync(lanes, bv[c], base + 2),
                b3 = __shfl_sync(lanes, bv[c], base + 3);
    if (j == 0 && live && c < nc) {
      const float ha = __fadd_rn(__fadd_rn(a[c], a2), __fadd_rn(a1, a3));
      const float hb = __fadd_rn(__fadd_rn(bv[c], b2), __fadd_rn(b1, b3));
      P.y[(size_t)(c0 + c) * P.ldy + row] = __fadd_rn(tail[c], __fadd_rn(ha, hb));
    }
  }
}

}  // namespace

size_t tl1_smem_bytes(int K, int R) {
  const int G = K / 128;
  return ((size_t)G * kTl1XStride + (size_t)R * G * 9) * sizeof(float);
}

int tl1_rows_per_cta(int K, int M, int num_sms) {
  // at most ~1024 (row, group) items per CTA, and at least two CTAs per SM
  const int G = K / 128;
  int cap = 1024 / G;
  if (cap < 1) cap = 1;
  int R = (M + 2 * num_sms - 1) / (2 * num_sms);
  if (R < 1) R = 1;
  return R < cap ? R : cap;
}

size_t tq1_smem_bytes(int K) {
  return ((size_t)K + 2 * (size_t)kTq1Rows * kTq1ProdStride) * sizeof(float);
}

cudaError_t launch_refmt_matvec(const RefLaunch& P, int num_sms, cudaStream_t s) {
  if (P.M <= 0 || P.B <= 0) return cudaSuccess;
  if (P.fmt == kPtq1) {
    const int R = tl1_rows_per_cta(P.K, P.M, num_sms);
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

cudaError_t launch_tl1_columns(const RefLaunch& P, cudaStream_t s) {
  if (P.M <= 0 || P.B <= 0) return cudaSuccess;
  if (P.fmt != kPtq1) return cudaErrorInvalidValue;
  // from two columns on, decode each group once for a block of up to eight
  if (P.B >= 2) {
    const dim3 grid((unsigned)((P.M + kTl1BlkRows - 1) / kTl1BlkRows),
                    (unsigned)((P.B + kTl1BlkCols - 1) / kTl1BlkCols), 1);
    tl1_colblock_kernel<<<grid, kTl1BlkThreads, 0, s>>>(P);
    return cudaGetLastError();
  }
  const dim3 grid((unsigned)((P.M + kTl1ColRows - 1) / kTl1ColRows), 1, 1);
  tl1_columns_kernel<<<grid, kTl1ColThreads, 0, s>>>(P);
  return cudaGetLastError();
}

}  // namespace ouroq
