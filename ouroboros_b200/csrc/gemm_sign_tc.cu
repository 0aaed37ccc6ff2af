// gemm_sign_tc.cu -- K4 for 1-bit sign weights: a batch of int8 tokens times
// a SIGN1G128 matrix (one sign bit per weight, an fp16 scale per 128 k) on the
// 5th-generation tensor cores.
//
// Reference operator: the batched matmul of a Qwen35 stage (wh_batched ->
// wmat_batched, cluster/src/infer/qwen35.rs:810-812, infer/mod.rs:152-167;
// ops::matmul_tl1, ops.rs:162-215): K activation columns share each weight
// row. Arithmetic: this library's sign form, bit-identical to the CPU oracle
// (oracle/oracle.h, the sign GEMM): per 128-k group g,
//   acc_g = sum_{k in g} (bit ? +1 : -1) * q_k           (exact int32)
//   y = (sum over g ascending of fp32(acc_g) * scale_g) * s_x   (fp32, in order)
//
// Tensor-core form. With bit codes c in {0, 1}, acc_g = 2 * D_g - Q_g where
// D_g = sum c * q (one tcgen05.mma kind::i8 chain of four K = 32 steps, u8 x
// s8 -> s32) and Q_g = sum q over the group. Each group gets its own int32
// accumulator in tensor memory, so the fp32 fold can run group by group in
// ascending order, exactly as the oracle's loop does.
//
// One CTA owns 128 weight rows (M of the MMA; the 1-bit codes expanded to
// bytes and written straight into tensor memory) and NT tokens (N: int8
// activations, TMA-loaded into shared memory with the 128-byte swizzle), and
// walks all of K in stages of four groups:
//   warp 0       producer: per stage, bulk copies of the packed bits and the
//                fp16 scales of the four 32-row tiles, TMA loads of the
//                activations
//   warp 1       allocates tensor memory; one lane issues the MMAs of group g
//                into accumulator D[g % ND], commits them to mbarriers
//   warps 2-9    expand each row's 128 bits of a group into 128 bytes (one
//                tcgen05.st of 32 columns; the two warps of a lane quarter take
//                alternate groups)
//   warps 10-13  fold: per stage, the token sums Q_g of its groups (from the
//                activation tile) and this row's scales; per group, D_g out of
//                tensor memory, acc_g, the term and the ordered fp32 sum of
//                each (row, token), one thread per row; finally y
// Tensor memory (512 columns x 128 lanes): accumulators D in columns [0, 256)
// (ND = min(8, 256 / NT) of NT columns each), expanded bit blocks A in eight
// 32-column buffers from column 256.
// Every wait is bounded and reports through the status word.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace ouroq {
namespace {

constexpr int kSgRows = 128;      // weight rows per CTA = MMA M
constexpr int kSgGroupK = 128;    // k per scale group = one A buffer = four MMAs
constexpr int kSgStageK = 512;    // k per pipeline stage (four groups)
constexpr int kSgGroupsPerStage = kSgStageK / kSgGroupK;
constexpr int kSgXWarps = 8;      // expansion warps, two per tensor-memory lane quarter
constexpr int kSgFWarps = 4;      // fold warps, one per lane quarter
constexpr int kSgThreads = 64 + (kSgXWarps + kSgFWarps) * 32;
constexpr int kSgMaxStages = 6;
constexpr uint32_t kSgA0 = 256;   // first column of the A buffers
constexpr int kSgABufs = 8;
constexpr int kSgMaxD = 8;
constexpr int kSgMaxTok = 32;     // largest token tile (the fold keeps one fp32 sum per token)

struct SgPlan {
  uint32_t bars, tmem, qs, stage0, w_off, sc_off, stage_bytes, total;
  int nd;  // accumulators (groups in flight between the MMAs and the fold)
};

// Stage: [activations: four boxes of NT rows x 128 B, 128-byte swizzle]
// [packed bits: four tiles x four chunks x 512 B][scales: four tiles x four
// groups x 64 B]. Token sums: [stage slot][group][kSgMaxTok tokens] int32.
__host__ __device__ inline SgPlan sg_plan(int NT, int stages) {
  SgPlan p;
  p.bars = 0;    // full[6], sfree[6], afull[8], afree[8], dfull[8], dfree[8]
  p.tmem = 384;  // allocated tensor-memory address
  p.qs = 512;
  p.stage0 = (p.qs + (uint32_t)stages * kSgGroupsPerStage * kSgMaxTok * 4 + 1023) & ~1023u;
  p.w_off = (uint32_t)NT * kSgStageK;
  p.sc_off = p.w_off + 4u * kSgGroupsPerStage * 512u;
  p.stage_bytes = (p.sc_off + 4u * kSgGroupsPerStage * 64u + 1023) & ~1023u;
  p.total = p.stage0 + (uint32_t)stages * p.stage_bytes + 1024;  // + alignment slack
  p.nd = 256 / NT < kSgMaxD ? 256 / NT : kSgMaxD;
  return p;
}

template <int NT>
__global__ void __launch_bounds__(kSgThreads, 1)
    gemm_sign_tc_kernel(const __grid_constant__ CUtensorMap act_map, const __grid_constant__ TcLaunch P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const SgPlan pl = sg_plan(NT, P.stages);
  const int S = P.stages, ND = pl.nd;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + pl.bars);
  uint64_t* sfree = full + kSgMaxStages;
  uint64_t* afull = sfree + kSgMaxStages;
  uint64_t* afree = afull + kSgABufs;
  uint64_t* dfull = afree + kSgABufs;
  uint64_t* dfree = dfull + kSgMaxD;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + pl.tmem);
  int* qsb = reinterpret_cast<int*>(smem + pl.qs);
  uint8_t* stages = smem + pl.stage0;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kSgRows;
  const int tok_base = P.tok0 + blockIdx.y * NT;
  const int nv = P.nvalid - (int)blockIdx.y * NT < NT ? P.nvalid - (int)blockIdx.y * NT : NT;
  const int G = P.K / kSgGroupK;
  const int C = P.K / 128;  // 16-byte chunks (128 sign bits) per packed row
  const int nstages = (P.K + kSgStageK - 1) / kSgStageK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&sfree[i], 1 + kSgFWarps);  // the MMAs' commit and every fold warp
    }
    for (int i = 0; i < kSgABufs; ++i) {
      mbar_init(&afull[i], 4);
      mbar_init(&afree[i], 1);
    }
    for (int i = 0; i < kSgMaxD; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dfree[i], kSgFWarps);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const int ntiles = (P.M + kTileRows - 1) / kTileRows - row0 / kTileRows;
      const int vt = ntiles < 4 ? ntiles : 4;
      bool waited = false;
      for (int i = 0; i < nstages; ++i) {
        const int slot = i % S;
        if (i >= S && !mbar_wait(&sfree[slot], ((i / S) - 1) & 1, P.status)) break;
        const int k0 = i * kSgStageK;
        const int SUB = (P.K - k0 < kSgStageK ? P.K - k0 : kSgStageK) / kSgGroupK;
        uint8_t* st = stages + (size_t)slot * pl.stage_bytes;
        mbar_arrive_expect_tx(&full[slot], (uint32_t)(vt * SUB * (512 + 64) + NT * SUB * 128));
        for (int t = 0; t < vt; ++t) {
          const size_t tile = (size_t)(row0 / kTileRows + t);
          bulk_g2s_stream(st + pl.w_off + t * (kSgGroupsPerStage * 512),
                          P.w + (tile * C + (size_t)(k0 / 128)) * 512, (uint32_t)SUB * 512u, &full[slot],
                          pol);
          bulk_g2s_stream(st + pl.sc_off + t * (kSgGroupsPerStage * 64),
                          reinterpret_cast<const uint8_t*>(P.scales) + (tile * G + (size_t)(k0 / 128)) * 64,
                          (uint32_t)SUB * 64u, &full[slot], pol);
        }
        if (!waited) {
          pdl_wait();  // activations may come from the previous grid
          waited = true;
        }
        for (int u = 0; u < SUB; ++u)
          tma_load_2d(st + (uint32_t)u * NT * 128u, &act_map, k0 + u * kSgGroupK, tok_base, &full[slot]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issue (one lane) ----------------
    if (lane == 0) {
      // instruction descriptor: D s32, A u8, B s8, both K-major, N = NT, M = 128
      const uint32_t idesc =
          (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(kSgRows >> 4) << 24);
      bool ok = true;
      int g = 0;
      for (int i = 0; i < nstages && ok; ++i) {
        const int slot = i % S;
        ok = mbar_wait(&full[slot], (i / S) & 1, P.status);
        const uint8_t* st = stages + (size_t)slot * pl.stage_bytes;
        const int k0 = i * kSgStageK;
        const int SUB = (P.K - k0 < kSgStageK ? P.K - k0 : kSgStageK) / kSgGroupK;
        for (int u = 0; u < SUB && ok; ++u, ++g) {
          const int b = g % kSgABufs, d = g % ND;
          ok = mbar_wait(&afull[b], (g / kSgABufs) & 1, P.status);
          if (ok && g >= ND) ok = mbar_wait(&dfree[d], ((g / ND) - 1) & 1, P.status);
          if (!ok) break;
          tc_fence_after();
          const uint8_t* act = st + (uint32_t)u * NT * 128u;
#pragma unroll
          for (int mb = 0; mb < 4; ++mb) {
            const uint64_t bd = smem_desc(act + mb * 32, 16, 1024, 2);
            mma_i8_ts(tmem + (uint32_t)(d * NT), tmem + kSgA0 + (uint32_t)b * 32u + (uint32_t)mb * 8u, bd,
                      idesc, mb > 0 ? 1u : 0u);
          }
          mma_commit(&afree[b]);  // the A buffer may be refilled
          mma_commit(&dfull[d]);  // the group's accumulator is complete
        }
        mma_commit(&sfree[slot]);
      }
    }
    __syncwarp();
  } else if (warp < 2 + kSgXWarps) {
    // ---------------- expansion ----------------
    // A sign word covers k = 32t .. 32t+31 with bit j of byte b holding k =
    // 32t + 4j + b, so (word >> j) & 0x01010101 is the byte codes of four
    // consecutive k: column 8t + j of the group's 32-column A block.
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    bool ok = true;
    int g = 0;
    for (int i = 0; i < nstages; ++i) {
      const int slot = i % S;
      const int k0 = i * kSgStageK;
      const int SUB = (P.K - k0 < kSgStageK ? P.K - k0 : kSgStageK) / kSgGroupK;
      if (SUB == 1 && ((g & 1) != h)) {
        ++g;
        continue;
      }
      if (ok) ok = mbar_wait(&full[slot], (i / S) & 1, P.status);
      const uint8_t* src = stages + (size_t)slot * pl.stage_bytes + pl.w_off +
                           (r >> 5) * (kSgGroupsPerStage * 512) + (r & 31) * 16;
      for (int u = 0; u < SUB; ++u, ++g) {
        if ((g & 1) != h) continue;
        const int b = g % kSgABufs;
        if (ok && g >= kSgABufs) ok = mbar_wait(&afree[b], ((g / kSgABufs) - 1) & 1, P.status);
        const uint4 wv = *reinterpret_cast<const uint4*>(src + u * 512);
        const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t a[32];
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
          for (int j = 0; j < 8; ++j) a[t * 8 + j] = (w4[t] >> j) & 0x01010101u;
        tmem_st32(tmem + lane_base + kSgA0 + (uint32_t)b * 32u, a);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[b]);
      }
    }
  } else {
    // ---------------- fold ----------------
    const int fw = warp - (2 + kSgXWarps);  // 0..3
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int row = row0 + r;
    float sum[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) sum[j] = 0.0f;
    bool ok = true;
    int g = 0;
    for (int i = 0; i < nstages; ++i) {
      const int slot = i % S;
      const int k0 = i * kSgStageK;
      const int SUB = (P.K - k0 < kSgStageK ? P.K - k0 : kSgStageK) / kSgGroupK;
      const uint8_t* st = stages + (size_t)slot * pl.stage_bytes;
      if (ok) ok = mbar_wait(&full[slot], (i / S) & 1, P.status);
      // token sums Q of the stage's groups: token t = 32 fw + lane, row t of
      // each swizzled activation box
      int* qs = qsb + slot * (kSgGroupsPerStage * kSgMaxTok);
      const int t = fw * 32 + lane;
      if (t < NT) {
        for (int u = 0; u < SUB; ++u) {
          const uint8_t* act = st + (uint32_t)u * NT * 128u + t * 128;
          int sq = 0;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 v = *reinterpret_cast<const uint4*>(act + ((c ^ (t & 7)) * 16));
            sq = __dp4a((int)v.x, 0x01010101, sq);
            sq = __dp4a((int)v.y, 0x01010101, sq);
            sq = __dp4a((int)v.z, 0x01010101, sq);
            sq = __dp4a((int)v.w, 0x01010101, sq);
          }
          qs[u * kSgMaxTok + t] = sq;
        }
      }
      // this row's fp16 scales of the stage's groups
      float sc[kSgGroupsPerStage];
#pragma unroll
      for (int u = 0; u < kSgGroupsPerStage; ++u)
        sc[u] = u < SUB ? __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(
                              st + pl.sc_off + (r >> 5) * (kSgGroupsPerStage * 64) + u * 64 + (r & 31) * 2)))
                        : 0.0f;
      named_bar_sync(2, kSgFWarps * 32);  // the stage's token sums are complete
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfree[slot]);  // this warp is done with the stage's data
#pragma unroll
      for (int u = 0; u < kSgGroupsPerStage; ++u, ++g) {
        if (u >= SUB) break;
        const int d = g % ND;
        if (ok) ok = mbar_wait(&dfull[d], (g / ND) & 1, P.status);
        tc_fence_after();
#pragma unroll
        for (int j0 = 0; j0 < NT; j0 += 32) {
          uint32_t dv[32];
          tmem_ld32(tmem + lane_base + (uint32_t)(d * NT + j0), dv);
          if (j0 + 32 >= NT) {
            // the accumulator has been read: the MMAs of group g + ND may reuse it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&dfree[d]);
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = j0 + j;
            if (n < NT) {
              const int acc = 2 * (int)dv[j] - qs[u * kSgMaxTok + n];
              sum[n] = __fadd_rn(sum[n], __fmul_rn(__int2float_rn(acc), sc[u]));
              if (P.acc && n < nv && row < P.M) P.acc[((size_t)(tok_base + n) * P.M + row) * G + g] = acc;
            }
          }
        }
      }
    }
#pragma unroll
    for (int n = 0; n < NT; ++n)
      if (n < nv && row < P.M)
        P.y[(size_t)(tok_base + n) * P.ldy + row] = __fmul_rn(sum[n], P.s_x[tok_base + n]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int NT>
cudaError_t launch_sign_t(const TcLaunch& L0, const int8_t* q, int Btot, int smem_optin, cudaStream_t s) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return cudaErrorNotSupported;
  cudaError_t e = ensure_max_smem<gemm_sign_tc_kernel<NT>>();
  if (e != cudaSuccess) return e;
  TcLaunch L = L0;
  L.N = NT;
  int stages = kSgMaxStages;
  while (stages > 2 && sg_plan(NT, stages).total > (uint32_t)smem_optin - 2048u) --stages;
  L.stages = stages;
  size_t smem = sg_plan(NT, stages).total;
  // One CTA per SM (each allocates all 512 tensor-memory columns): more than
  // half of the SM's shared memory per CTA.
  int dev = 0, per_sm = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  if (e != cudaSuccess) return e;
  if (smem <= (size_t)per_sm / 2) smem = (size_t)per_sm / 2 + 1024;
  if (smem > (size_t)smem_optin) return cudaErrorInvalidValue;
  // activations [Btot][K] int8, box 128 B x NT rows, 128-byte swizzle, zero fill
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)L.K, (cuuint64_t)Btot};
  const cuuint64_t strides[1] = {(cuuint64_t)L.K};
  const cuuint32_t box[2] = {128u, (cuuint32_t)NT};
  const cuuint32_t estr[2] = {1u, 1u};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(q), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  const dim3 grid((L.M + kSgRows - 1) / kSgRows, (L.nvalid + NT - 1) / NT, 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kSgThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  return cudaLaunchKernelEx(&cfg, gemm_sign_tc_kernel<NT>, map, L);
}

}  // namespace

bool gemm_sign_tc_supported(int M, int K, int B) { return M > 0 && K > 0 && K % kSgGroupK == 0 && B >= 1; }

cudaError_t launch_gemm_sign_tc(const TcLaunch& L, const int8_t* q, int Btot, int smem_optin,
                                cudaStream_t s) {
  if (L.nvalid <= 0) return cudaSuccess;
  if (!L.scales) return cudaErrorInvalidValue;
  // token tile: 32 (larger batches take several tiles), or 16
  if (L.nvalid > 16) return launch_sign_t<32>(L, q, Btot, smem_optin, s);
  return launch_sign_t<16>(L, q, Btot, smem_optin, s);
}

}  // namespace ouroq
