// head.cu -- the reference's 16-bit weight formats behind matvec_q and the
// greedy tied lm_head.
//
//   F16  (QuantKind::F16,  ops.rs:131-153)  y[r] = sum_i f16_to_f32(w[r][i]) * x[i]
//   BF16 (QuantKind::Bf16, ops.rs:600-620)  the same with bf16 weights
//
// The reference sums each row as one fp32 chain in element order, rounding
// every product and every sum (no fused multiply-add); here lane = row and
// the chain is kept exactly so (__fmul_rn / __fadd_rn, never contracted), so
// results are bit-identical. Weights are
// stored as in the shard (row-major, 2 bytes per element) and read once,
// whole cache lines of one row at a time (head_tiled_kernel below).
//
// With kArgmax the launch also reduces finite_argmax (mod.rs:70-83, used by
// argmax_token mod.rs:191-194) of each sequence's logits: NaN is skipped and
// the first maximum wins. Each logit becomes a 64-bit key (order-preserving
// float bits above the complemented row), so one atomicMax per CTA and
// sequence finds the answer; the last CTA to finish (an atomic count) turns
// the keys into token ids and clears them and the count for the next launch.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace ouroq {
namespace {

constexpr int kHeadThreads = 256;  // rows per CTA (lane = row)
constexpr int kHeadKC = 512;       // elements of x staged per pass
constexpr int kHeadMaxNB = 8;      // sequences per CTA (grid.y covers more)

template <bool kBf16>
__device__ __forceinline__ float w2f(uint32_t bits16) {
  if (kBf16) return __uint_as_float(bits16 << 16);
  return __half2float(__ushort_as_half((unsigned short)bits16));
}

template <bool kBf16>
__device__ __forceinline__ void cvt8(const uint4 v, float (&f)[8]) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (kBf16) {
      f[2 * j] = __uint_as_float(u[j] << 16);
      f[2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
    } else {
      const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&u[j]));
      f[2 * j] = t.x;
      f[2 * j + 1] = t.y;
    }
  }
}

// acc[b] = acc[b] + w * x[b], each operation rounded to nearest. (The packed
// f32x2 forms, even written as mul.rn / add.rn, did not reproduce the
// separately rounded scalar chain on B200, so every sequence has its own.)
template <int NB>
__device__ __forceinline__ void chain_step(float (&acc)[NB], float w, const float* xk) {
  if constexpr (NB == 1) {
    acc[0] = __fadd_rn(acc[0], __fmul_rn(w, xk[0]));
  } else {
#pragma unroll
    for (int p = 0; p < NB / 4; ++p) {
      const float4 xx = reinterpret_cast<const float4*>(xk)[p];
      acc[4 * p] = __fadd_rn(acc[4 * p], __fmul_rn(w, xx.x));
      acc[4 * p + 1] = __fadd_rn(acc[4 * p + 1], __fmul_rn(w, xx.y));
      acc[4 * p + 2] = __fadd_rn(acc[4 * p + 2], __fmul_rn(w, xx.z));
      acc[4 * p + 3] = __fadd_rn(acc[4 * p + 3], __fmul_rn(w, xx.w));
    }
    if constexpr (NB % 4 == 2) {
      const float2 xx = reinterpret_cast<const float2*>(xk)[NB / 2 - 1];
      acc[NB - 2] = __fadd_rn(acc[NB - 2], __fmul_rn(w, xx.x));
      acc[NB - 1] = __fadd_rn(acc[NB - 1], __fmul_rn(w, xx.y));
    }
  }
}

// finite_argmax key: larger value first, then the smaller row; 0 = no value.
// +0 and -0 compare equal in the reference, so zero is made +0 first.
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
  const uint32_t bits = v == 0.0f ? 0u : __float_as_uint(v);
  const uint32_t ord = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
  return ((unsigned long long)ord << 32) | (0xffffffffu - (uint32_t)row);
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
    v = t > v ? t : v;
  }
  return v;
}

// The end of finite_argmax for one CTA: red[w][b] holds warp w's best key
// for sequence b; the CTA maximum goes to the global key with one atomicMax,
// and the last CTA to finish writes the tokens and clears keys and counter.
template <int NB, int kWarps>
__device__ __forceinline__ void argmax_finish(const HeadLaunch& L,
                                              unsigned long long (&red)[kWarps][NB], int b0,
                                              int nb) {
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x < nb) {
    unsigned long long key = 0;
    for (int w = 0; w < kWarps; ++w) key = red[w][threadIdx.x] > key ? red[w][threadIdx.x] : key;
    if (key) atomicMax(L.key + b0 + threadIdx.x, key);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // one fence: cumulative, it orders the CTA's atomicMax calls (ordered
    // before it by the barrier) before the count
    __threadfence();
    last = atomicAdd(L.counter, 1u) == gridDim.x * gridDim.y - 1;
    if (last) __threadfence();
  }
  __syncthreads();
  if (last) {
    for (int b = threadIdx.x; b < L.B; b += blockDim.x) {
      const unsigned long long key = atomicExch(L.key + b, 0ull);
      // every logit NaN: the reference's best stays 0
      L.tokens[b] = key ? (long long)(0xffffffffu - (uint32_t)key) : 0;
    }
    if (threadIdx.x == 0) *L.counter = 0u;
  }
}

// warp w folds its lanes' logits (lane = row) into red[w][b]
template <int NB, int kWarps>
__device__ __forceinline__ void argmax_fold(unsigned long long (&red)[kWarps][NB],
                                            const float (&acc)[NB], bool live, int row, int nb) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    unsigned long long key = 0;
    if (live && b < nb && !isnan(acc[b])) key = argmax_key(acc[b], row);
    key = warp_max_u64(key);
    if (lane == 0 && key > red[warp][b]) red[warp][b] = key;
  }
}

// ---- rows of any length or alignment: lane = row, element loads ----
// grid (ceil(M / 256), ceil(B / NB)), block 256; dynamic shared memory
// x chunk [kHeadKC][NB] (sequence index fastest).
template <int NB, bool kBf16, bool kArgmax>
__global__ void __launch_bounds__(kHeadThreads) head_rows_kernel(HeadLaunch L) {
  extern __shared__ __align__(16) float xs[];
  __shared__ unsigned long long red[kHeadThreads / 32][NB];
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x * kHeadThreads + threadIdx.x;
  const bool live = row < L.M;
  const int b0 = blockIdx.y * NB;
  const int nb = min(NB, L.B - b0);
  const uint16_t* wr = L.w + (size_t)(live ? row : 0) * L.K;
  float acc[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
  for (int k0 = 0; k0 < L.K; k0 += kHeadKC) {
    const int kc = min(kHeadKC, L.K - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < NB * kc; i += kHeadThreads) {
      const int b = i / kc, k = i - b * kc;
      xs[k * NB + b] = b < nb ? L.x[(size_t)(b0 + b) * L.K + k0 + k] : 0.0f;
    }
    __syncthreads();
    if (!live) continue;
    for (int k = 0; k < kc; ++k) chain_step<NB>(acc, w2f<kBf16>(__ldg(wr + k0 + k)), xs + k * NB);
  }
  if (L.y && live) {
#pragma unroll
    for (int b = 0; b < NB; ++b)
      if (b < nb) L.y[(size_t)(b0 + b) * L.ldy + row] = acc[b];
  }
  if constexpr (kArgmax) {
    if ((threadIdx.x & 31) == 0)
      for (int b = 0; b < NB; ++b) red[threadIdx.x >> 5][b] = 0;
    __syncwarp();
    argmax_fold<NB, kHeadThreads / 32>(red, acc, live, row, nb);
    argmax_finish<NB, kHeadThreads / 32>(L, red, b0, nb);
  }
}

// ---- K % 8 == 0, w and x 16-byte aligned: staged and coalesced ----
// Persistent CTAs of 256 threads walk row sets of 256 rows (lane = row), each
// as K / 64 tiles. A stage holds one tile -- 256 rows x 64 elements, rows
// padded to 144 B, so lane r reading 16 B of its own row meets no bank
// conflict -- and the same 64 elements of x for every sequence. All threads
// fill stages with cp.async (8 consecutive threads copy the 128 contiguous
// bytes of one row), kTileStages - 1 tiles ahead, the sequence of tiles
// running on across row sets. The CTA works in lockstep, one barrier a tile.
constexpr int kTileRows = 256;
constexpr int kTileK = 64;
constexpr int kTilePitch = kTileK + 8;  // halves: 144 bytes
constexpr int kTileStages = 3;
constexpr int kMaxNB = 32;

__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  // src_bytes 0: nothing is read and the 16 bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int NB>
__host__ __device__ constexpr size_t tile_stage_bytes() {
  return (size_t)kTileRows * kTilePitch * 2 + (size_t)NB * kTileK * 4;
}

template <int NB, bool kBf16, bool kArgmax>
__global__ void __launch_bounds__(kTileRows) head_tiled_kernel(HeadLaunch L) {
  extern __shared__ __align__(16) unsigned char tile_smem[];
  __shared__ unsigned long long red[kTileRows / 32][NB];
  constexpr size_t SB = tile_stage_bytes<NB>();
  constexpr size_t WB = (size_t)kTileRows * kTilePitch * 2;
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x;
  const int b0 = blockIdx.y * NB;
  const int nb = min(NB, L.B - b0);
  const int nsets = (L.M + kTileRows - 1) / kTileRows;
  const int nck = (L.K + kTileK - 1) / kTileK;
  const int my_sets = (int)blockIdx.x < nsets ? (nsets - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = my_sets * nck;
  if (kArgmax && (tid & 31) == 0)
    for (int b = 0; b < NB; ++b) red[tid >> 5][b] = 0;

  auto issue = [&](int g) {
    if (g < total) {
      const int i = g / nck, c = g - i * nck;
      const int r0 = ((int)blockIdx.x + i * (int)gridDim.x) * kTileRows;
      const int k0 = c * kTileK;
      const int units = min(kTileK, L.K - k0) / 8;
      unsigned char* st = tile_smem + (size_t)(g % kTileStages) * SB;
      uint16_t* ws = reinterpret_cast<uint16_t*>(st);
      float* xs = reinterpret_cast<float*>(st + WB);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int q = tid + j * kTileRows;
        const int rr = q >> 3, u = q & 7;
        if (u < units && r0 + rr < L.M)
          cp_async16(ws + rr * kTilePitch + u * 8, L.w + (size_t)(r0 + rr) * L.K + k0 + u * 8, 16);
      }
      for (int q = tid; q < NB * (kTileK / 4); q += kTileRows) {
        const int b = q / (kTileK / 4), v = q % (kTileK / 4);
        const bool ok = b < nb && v < units * 2;
        cp_async16(xs + b * kTileK + v * 4, ok ? L.x + (size_t)(b0 + b) * L.K + k0 + v * 4 : L.x,
                   ok ? 16u : 0u);
      }
    }
    cp_async_commit();  // possibly empty: one group per tile
  };

#pragma unroll
  for (int g = 0; g < kTileStages - 1; ++g) issue(g);
  float acc[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
  for (int g = 0; g < total; ++g) {
    cp_async_wait<kTileStages - 2>();
    __syncthreads();  // tile g landed for everyone; tile g - 1 fully consumed
    issue(g + kTileStages - 1);
    const int i = g / nck, c = g - i * nck;
    const int row = ((int)blockIdx.x + i * (int)gridDim.x) * kTileRows + tid;
    const bool live = row < L.M;
    const int units = min(kTileK, L.K - c * kTileK) / 8;
    const unsigned char* st = tile_smem + (size_t)(g % kTileStages) * SB;
    const uint16_t* wrow = reinterpret_cast<const uint16_t*>(st) + tid * kTilePitch;
    const float* xs = reinterpret_cast<const float*>(st + WB);
    if (live) {
      for (int u = 0; u < units; ++u) {
        float f[8];
        cvt8<kBf16>(*reinterpret_cast<const uint4*>(wrow + u * 8), f);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const float4 xa = *reinterpret_cast<const float4*>(xs + b * kTileK + u * 8);
          const float4 xb = *reinterpret_cast<const float4*>(xs + b * kTileK + u * 8 + 4);
          const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[b] = __fadd_rn(acc[b], __fmul_rn(f[e], xv[e]));
        }
      }
    }
    if (c == nck - 1) {  // this row set is complete
      if (L.y && live) {
#pragma unroll
        for (int b = 0; b < NB; ++b)
          if (b < nb) L.y[(size_t)(b0 + b) * L.ldy + row] = acc[b];
      }
      if constexpr (kArgmax) argmax_fold<NB, kTileRows / 32>(red, acc, live, row, nb);
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
    }
  }
  cp_async_wait<0>();
  if constexpr (kArgmax) argmax_finish<NB, kTileRows / 32>(L, red, b0, nb);
}

template <int NB, bool kBf16, bool kArgmax>
cudaError_t launch_nb(const HeadLaunch& L, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  const unsigned groups = (unsigned)((L.B + NB - 1) / NB);
  if (L.vec) {
    cudaError_t e = ensure_max_smem<head_tiled_kernel<NB, kBf16, kArgmax>>();
    if (e != cudaSuccess) return e;
    const size_t smem = kTileStages * tile_stage_bytes<NB>();
    // resident CTAs per SM by shared memory (228 KB per SM, 1 KB reserved per CTA)
    const int per_sm = smem + 1024 <= 114 * 1024 ? 2 : 1;
    const int nsets = (L.M + kTileRows - 1) / kTileRows;
    // the fewest row sets per CTA that fit one resident wave, and just enough
    // CTAs for them, so that every CTA has the same number of sets
    const int slots = L.num_sms * per_sm;
    const int per_cta = (nsets + slots - 1) / slots;
    const int grid = (nsets + per_cta - 1) / per_cta;
    cfg.gridDim = dim3((unsigned)grid, groups, 1);
    cfg.blockDim = dim3(kTileRows);
    cfg.dynamicSmemBytes = smem;
  } else {
    cfg.gridDim = dim3((unsigned)((L.M + kHeadThreads - 1) / kHeadThreads), groups, 1);
    cfg.blockDim = dim3(kHeadThreads);
    cfg.dynamicSmemBytes = (size_t)kHeadKC * NB * sizeof(float);
  }
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (L.vec) return cudaLaunchKernelEx(&cfg, head_tiled_kernel<NB, kBf16, kArgmax>, L);
  return cudaLaunchKernelEx(&cfg, head_rows_kernel<NB, kBf16, kArgmax>, L);
}

template <bool kBf16, bool kArgmax>
cudaError_t launch_fmt(const HeadLaunch& L, cudaStream_t s, bool pdl) {
  if (L.B <= 1) return launch_nb<1, kBf16, kArgmax>(L, s, pdl);
  if (L.B <= 2) return launch_nb<2, kBf16, kArgmax>(L, s, pdl);
  if (L.B <= 4) return launch_nb<4, kBf16, kArgmax>(L, s, pdl);
  if (L.B <= 8 || !L.vec) return launch_nb<kHeadMaxNB, kBf16, kArgmax>(L, s, pdl);
  if (L.B <= 16) return launch_nb<16, kBf16, kArgmax>(L, s, pdl);
  return launch_nb<kMaxNB, kBf16, kArgmax>(L, s, pdl);
}

}  // namespace

cudaError_t launch_head(const HeadLaunch& L, cudaStream_t s, bool pdl) {
  if (L.M <= 0 || L.B <= 0) return cudaSuccess;
  const bool argmax = L.tokens != nullptr;
  if (L.bf16) return argmax ? launch_fmt<true, true>(L, s, pdl) : launch_fmt<true, false>(L, s, pdl);
  return argmax ? launch_fmt<false, true>(L, s, pdl) : launch_fmt<false, false>(L, s, pdl);
}

}  // namespace ouroq
