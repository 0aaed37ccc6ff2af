// gemm_tc.cu -- K4: batched packed-ternary x int8 GEMM on the 5th-generation
// tensor cores (tcgen05.mma kind::i8, accumulators in tensor memory).
//
// Reference operator: ops::matmul_q / matmul_tl1 (cluster/src/infer/ops.rs:
// 162-230): K activation columns share each weight row, the output is
// [k][out_len]. Here the arithmetic is the BitNet b1.58 form: int8 activations, exact
// int32 accumulation, y = ((float)acc * w_scale) * s_x, identical to the CPU
// oracle (oracle/oracle.h).
//
// Tiling ("swap AB"): the MMA's M = 128 weight rows (operand A: 2-bit codes
// expanded to u8 c = w + 1 and written straight into tensor memory), N = up
// to 256 tokens (operand B: the int8 activations, TMA-loaded into shared
// memory with the 128-byte swizzle), K = 32 per instruction. One CTA owns 128
// rows of W and one tile of N tokens (the grid covers row tiles x token tiles,
// N chosen on the host so that the grid fills the SMs) and walks all of K:
//   warp 0      producer: per stage, bulk copies of the packed weight slice
//               (four 32-row tiles of the tiled device layout) + TMA tensor
//               loads of the activation slice
//   warp 1      allocates tensor memory; one lane issues the MMAs (A from
//               tensor memory, B from shared memory) and commits them to
//               mbarriers
//   warps 2-9   expand 2-bit codes to bytes (tcgen05.st into 8 rotating A
//               buffers; two warps per tensor-memory lane quarter take
//               alternate 128-k sub-blocks), sum each token's activations (the
//               correction for c = w + 1), then run the epilogue out of tensor
//               memory
// Keeping A out of shared memory matters: expanding in shared memory would
// cost a 4x write plus a 4x MMA read per packed byte, more shared-memory
// bandwidth than the HBM stream feeds.
// The accumulator is D[row][token] = sum_k c * q; acc = D - sum_k q.
//
// Split K. A CTA's rate is set by the MMAs it issues: on B200 one
// tcgen05.mma of kind::i8 (M = 128, K = 32) takes 110-160 clocks alone at any
// N from 16 to 256 (one or several accumulators), about 210 (N = 16) to 390
// (N = 256) clocks inside this kernel. When the (row tile x token tile) grid
// leaves SMs idle, the launcher splits
// K over a cluster of 2 or 4 CTAs (grid z): each accumulates its K range,
// then CTAs z > 0 stage their int32 partials D and token sums in their own
// shared memory and send them to CTA 0's with one bulk shared-to-shared copy
// each (completion counted on an mbarrier of CTA 0), and CTA 0 adds them and
// writes the outputs. Integer sums: exact in any order.
// Every wait is bounded and reports through the status word.
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace ouroq {
namespace {

constexpr int kTcRows = 128;     // weight rows per CTA = MMA M
constexpr int kSliceK = 128;     // k per A buffer = 4 MMAs of K = 32
constexpr int kXWarps = 8;       // expansion warps: two per tensor-memory lane quarter
constexpr int kTcThreads = 64 + kXWarps * 32;  // producer, MMA issuer, expansion
constexpr int kMaxTcStages = 6;

// Tensor memory (512 columns x 128 lanes, 32 bit): accumulator D[row][token]
// in columns [0, 256); expanded weight blocks A (128 rows x 128 k = 32
// columns each, 4 int8 per column) in kTmemABufs buffers from column 256.
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemA0 = 256;
constexpr int kTmemABufs = 8;  // even buffers: sub-blocks of half 0, odd: half 1

struct TcPlan {
  uint32_t bars, tmem, qsum, stage0, stage_bytes, act_off, total;
  int ks;  // k per TMA stage (multiple of 128)
};

// Stage = the packed weights of 128 rows x ks k (four 32-row tiles, ks*8 B
// each) followed by the activations (ks/128 swizzled 128-byte column blocks
// of N rows). Larger k slices for small N keep enough weight bytes in flight.
__host__ __device__ inline TcPlan tc_plan(int N, int stages) {
  TcPlan p;
  p.ks = N <= 64 ? 512 : (N <= 128 ? 256 : 128);
  p.bars = 0;    // full[6], sfree[6], afull[8], afree[8], accfull, xfull
  p.tmem = 256;  // allocated tensor-memory address
  p.qsum = 512;  // int [256]
  p.stage0 = 2048;
  p.act_off = (uint32_t)p.ks * 32;  // 4 tiles x ks*8 B of packed weights
  p.stage_bytes = ((p.act_off + (uint32_t)N * (uint32_t)p.ks + 1023) / 1024) * 1024;
  p.total = p.stage0 + (uint32_t)stages * p.stage_bytes + 1024;  // + alignment slack
  return p;
}

__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ TcGroup Gp, const __grid_constant__ TcLaunch P0) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // this CTA's job of the group (parameter reads at fixed offsets only)
  int jj = 0;
#pragma unroll
  for (int q = 1; q < kMaxTcJobs; ++q)
    if (q < Gp.njobs && (int)blockIdx.x >= Gp.tile_begin[q]) jj = q;
  TcLaunch P = P0;
  const CUtensorMap* act_map = &Gp.maps[0];
  int tile0 = 0;
#pragma unroll
  for (int q = 0; q < kMaxTcJobs; ++q)
    if (q == jj) {
      P.w = Gp.jobs[q].w;
      P.y = Gp.jobs[q].y;
      P.acc = Gp.jobs[q].acc;
      P.s_x = Gp.jobs[q].s_x;
      P.w_scale = Gp.jobs[q].w_scale;
      P.M = Gp.jobs[q].M;
      P.K = Gp.jobs[q].K;
      P.ldy = Gp.jobs[q].ldy;
      act_map = &Gp.maps[q];
      tile0 = Gp.tile_begin[q];
    }
  // 1024-byte alignment for the swizzled activation tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const TcPlan pl = tc_plan(P.N, P.stages);
  const int S = P.stages;
  const int KS = pl.ks;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + pl.bars);
  uint64_t* sfree = full + kMaxTcStages;
  uint64_t* afull = sfree + kMaxTcStages;
  uint64_t* afree = afull + kTmemABufs;
  uint64_t* accfull = afree + kTmemABufs;
  uint64_t* xfull = accfull + 1;  // split K, CTA 0: the other CTAs' partials landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + pl.tmem);
  int* qsum = reinterpret_cast<int*>(smem + pl.qsum);
  uint8_t* stages = smem + pl.stage0;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = ((int)blockIdx.x - tile0) * kTcRows;
  // token tile of this CTA: [tok_base, tok_base + nv), at most P.N tokens
  const int tok_base = P.tok0 + blockIdx.y * P.N;
  const int nv = P.nvalid - blockIdx.y * P.N < P.N ? P.nvalid - blockIdx.y * P.N : P.N;
  // this CTA's K range [kb, ke) (split K: CTA z of the cluster takes the
  // z-th of Z even parts, in whole 128-k sub-blocks, never empty), walked in
  // stages of KS (the last one may be shorter)
  const int Z = P.ksplit > 1 ? P.ksplit : 1;
  const int z = Z > 1 ? (int)blockIdx.z : 0;
  const int nsb = P.K / kSliceK;
  const int kb = (int)((long long)nsb * z / Z) * kSliceK;
  const int ke = (int)((long long)nsb * (z + 1) / Z) * kSliceK;
  const int nstages = (ke - kb + KS - 1) / KS;
  const int C = P.K / 64;  // 16-byte chunks per packed row

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&sfree[i], 1);
    }
    for (int i = 0; i < kTmemABufs; ++i) {
      mbar_init(&afull[i], 4);
      mbar_init(&afree[i], 1);
    }
    mbar_init(accfull, 1);
    mbar_init(xfull, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  for (int i = threadIdx.x; i < 256; i += blockDim.x) qsum[i] = 0;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      // 32-row tiles of this CTA that exist (the last CTA may cover fewer)
      const int ntiles = (P.M + kTileRows - 1) / kTileRows - row0 / kTileRows;
      const int vt = ntiles < 4 ? ntiles : 4;
      bool waited = false;
      for (int i = 0; i < nstages; ++i) {
        const int k0 = kb + i * KS;
        const int slot = i % S;
        if (i >= S && !mbar_wait(&sfree[slot], ((i / S) - 1) & 1, P.status)) break;
        const int ks = ke - k0 < KS ? ke - k0 : KS;
        const int SUB = ks / kSliceK;
        const uint32_t wbytes = (uint32_t)ks * 8u;  // per 32-row tile
        uint8_t* st = stages + (size_t)slot * pl.stage_bytes;
        mbar_arrive_expect_tx(&full[slot], wbytes * (uint32_t)vt + (uint32_t)(P.N * ks));
        for (int t = 0; t < vt; ++t) {
          const size_t tile = (size_t)(row0 / kTileRows + t);
          bulk_g2s_stream(st + t * (KS * 8), P.w + (tile * C + (size_t)(k0 / 64)) * 512, wbytes,
                          &full[slot], pol);
        }
        if (!waited) {
          pdl_wait();  // activations may come from the previous grid
          waited = true;
        }
        for (int u = 0; u < SUB; ++u)
          tma_load_2d(st + pl.act_off + (uint32_t)u * (uint32_t)P.N * 128u, act_map,
                      k0 + u * kSliceK, tok_base, &full[slot]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issue (one lane) ----------------
    if (lane == 0) {
      // instruction descriptor: D s32, A u8, B s8, both K-major, N, M = 128
      const uint32_t idesc = (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(P.N >> 3) << 17) |
                             ((uint32_t)(kTcRows >> 4) << 24);
      bool ok = true;
      int g = 0;
      for (int i = 0; i < nstages && ok; ++i) {
        const int k0 = kb + i * KS;
        const int slot = i % S;
        ok = mbar_wait(&full[slot], (i / S) & 1, P.status);
        uint8_t* st = stages + (size_t)slot * pl.stage_bytes;
        const int SUB = (ke - k0 < KS ? ke - k0 : KS) / kSliceK;
        for (int u = 0; u < SUB && ok; ++u, ++g) {
          const int b = g % kTmemABufs;
          ok = mbar_wait(&afull[b], (g / kTmemABufs) & 1, P.status);
          if (!ok) break;
          tc_fence_after();
          const uint8_t* act = st + pl.act_off + (uint32_t)u * (uint32_t)P.N * 128u;
#pragma unroll
          for (int mb = 0; mb < 4; ++mb) {
            // B: activations, 128-byte swizzle: rows 128 B apart, 8-row groups
            //    1024 B apart (SBO); K block mb starts 32 B into the row
            const uint64_t bd = smem_desc(act + mb * 32, 16, 1024, 2);
            mma_i8_ts(tmem, tmem + kTmemA0 + (uint32_t)b * 32u + (uint32_t)mb * 8u, bd, idesc,
                      (i > 0 || u > 0 || mb > 0) ? 1u : 0u);
          }
          mma_commit(&afree[b]);  // the A buffer may be refilled once these MMAs finished
        }
        mma_commit(&sfree[slot]);  // and the stage (weights + activations)
      }
      mma_commit(accfull);
    }
    __syncwarp();
  } else {
    // ---------------- expansion + epilogue (warps 2..9) ----------------
    // Warp w may only touch tensor-memory lanes 32*(w%4) .. +31, so the lane
    // quarter is w%4; the two warps of a quarter take alternate 128-k
    // sub-blocks (half h takes g with g%2 == h) so that one expands while the
    // other waits on its tensor-memory store.
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    const int r = q * 32 + lane;      // weight row within the CTA tile (= TMEM lane)
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    int qs0 = 0, qs1 = 0;             // partial sum_k q for tokens e and e + 128
    const int e = ((warp - 2) & 3) * 32 + lane;
    bool ok = true;
    int g = 0;
    for (int i = 0; i < nstages; ++i) {
      const int k0 = kb + i * KS;
      const int slot = i % S;
      const int SUB = (ke - k0 < KS ? ke - k0 : KS) / kSliceK;
      // a stage holds a sub-block of this half unless it has one sub-block of the other
      if (SUB == 1 && ((g & 1) != h)) {
        ++g;
        continue;
      }
      if (ok) ok = mbar_wait(&full[slot], (i / S) & 1, P.status);
      const uint8_t* st = stages + (size_t)slot * pl.stage_bytes;
      const uint8_t* src = st + (r >> 5) * (KS * 8) + (r & 31) * 16;
      for (int u = 0; u < SUB; ++u, ++g) {
        if ((g & 1) != h) continue;
        const int b = g % kTmemABufs;
        if (ok && g >= kTmemABufs) ok = mbar_wait(&afree[b], ((g / kTmemABufs) - 1) & 1, P.status);
        // expand this row's two 64-k chunks of the sub-block into 32 columns
        uint32_t a[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint4 wv = *reinterpret_cast<const uint4*>(src + (2 * u + c) * 512);
          const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            a[c * 16 + t * 4 + 0] = w4[t] & 0x03030303u;
            a[c * 16 + t * 4 + 1] = (w4[t] >> 2) & 0x03030303u;
            a[c * 16 + t * 4 + 2] = (w4[t] >> 4) & 0x03030303u;
            a[c * 16 + t * 4 + 3] = (w4[t] >> 6) & 0x03030303u;
          }
        }
        tmem_st32(tmem + lane_base + kTmemA0 + (uint32_t)b * 32u, a);
        // activation sums of this sub-block: rows e and e + 128 of the swizzled tile
        const uint8_t* act = st + pl.act_off + (uint32_t)u * (uint32_t)P.N * 128u;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int n = e + half * 128;
          if (n < P.N) {
            int sum = 0;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const uint4 v = *reinterpret_cast<const uint4*>(act + n * 128 + ((c ^ (n & 7)) * 16));
              sum = __dp4a((int)v.x, 0x01010101, sum);
              sum = __dp4a((int)v.y, 0x01010101, sum);
              sum = __dp4a((int)v.z, 0x01010101, sum);
              sum = __dp4a((int)v.w, 0x01010101, sum);
            }
            if (half == 0) qs0 += sum; else qs1 += sum;
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[b]);
      }
    }
    if (e < P.N) atomicAdd(&qsum[e], qs0);
    if (e + 128 < P.N) atomicAdd(&qsum[e + 128], qs1);
    named_bar_sync(1, kXWarps * 32);
    if (ok) ok = mbar_wait(accfull, 0, P.status);
    tc_fence_after();
  }
  // ---- split K: the partials of CTA z > 0 go to slot z - 1 of CTA 0's stage
  // area. A slot: D as [row][NP] int32 (NP = N + 4: rows 16-byte aligned,
  // spread over the banks), then the token sums [N].
  const int NP = P.N + 4;
  const uint32_t slot_bytes = (uint32_t)(kTcRows * NP + P.N) * 4u;
  if (Z > 1) {
    if (z == 0 && threadIdx.x == 0) mbar_arrive_expect_tx(xfull, (uint32_t)(Z - 1) * slot_bytes);
    cluster_sync_all();  // every CTA's MMAs are done: the stage areas are free
    if (z > 0 && warp >= 2) {
      const int q = warp & 3, h = (warp - 2) >> 2, r = q * 32 + lane;
      const uint32_t lane_base = (uint32_t)(q * 32) << 16;
      int* stg = reinterpret_cast<int*>(stages);
      for (int j0 = h * 32; j0 < P.N; j0 += 64) {
        uint32_t d[32];
        tmem_ld32(tmem + lane_base + (uint32_t)j0, d);
        uint4* dst = reinterpret_cast<uint4*>(stg + r * NP + j0);
#pragma unroll
        for (int v = 0; v < 8; ++v)
          if (j0 + 4 * v < P.N) dst[v] = make_uint4(d[4 * v], d[4 * v + 1], d[4 * v + 2], d[4 * v + 3]);
      }
      const int e = ((warp - 2) & 3) * 32 + lane;
      if (h == 0)
        for (int t = e; t < P.N; t += 128) stg[kTcRows * NP + t] = qsum[t];
      fence_proxy_async_smem();  // visible to the bulk copy
      named_bar_sync(1, kXWarps * 32);
      if (warp == 2 && lane == 0)
        bulk_s2s_cluster(peer_smem(stages + (size_t)(z - 1) * slot_bytes, 0), stages, slot_bytes,
                         peer_smem(xfull, 0));
    }
  }
  if (z == 0 && warp >= 2) {
    // ---- epilogue: D[row][token] from tensor memory (plus the other CTAs'
    // partials), 32-column chunks split by half
    const int q = warp & 3, h = (warp - 2) >> 2, r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int* part = reinterpret_cast<const int*>(stages);
    if (Z > 1) {
      mbar_wait(xfull, 0, P.status);
      const int e = ((warp - 2) & 3) * 32 + lane;
      if (h == 0)
        for (int t = e; t < P.N; t += 128)
          for (int zz = 1; zz < Z; ++zz) qsum[t] += part[(size_t)(zz - 1) * (slot_bytes / 4) + kTcRows * NP + t];
      named_bar_sync(1, kXWarps * 32);
    }
    const int row = row0 + r;
    for (int j0 = h * 32; j0 < P.N; j0 += 64) {
      uint32_t d[32];
      tmem_ld32(tmem + lane_base + (uint32_t)j0, d);
      for (int zz = 1; zz < Z; ++zz) {
        const uint4* src =
            reinterpret_cast<const uint4*>(part + (size_t)(zz - 1) * (slot_bytes / 4) + r * NP + j0);
#pragma unroll
        for (int v = 0; v < 8; ++v)
          if (j0 + 4 * v < P.N) {
            const uint4 pv = src[v];
            d[4 * v] += pv.x;
            d[4 * v + 1] += pv.y;
            d[4 * v + 2] += pv.z;
            d[4 * v + 3] += pv.w;
          }
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = j0 + j;
        if (n < nv && row < P.M) {
          const int tok = tok_base + n;
          const int acc = (int)d[j] - qsum[n];
          P.y[(size_t)tok * P.ldy + row] =
              __fmul_rn(__fmul_rn(__int2float_rn(acc), P.w_scale), P.s_x[tok]);
          if (P.acc) P.acc[(size_t)tok * P.M + row] = acc;
        }
      }
    }
  }
  // CTA 0 has read every partial (its copies completed): the other CTAs'
  // shared memory may go
  if (Z > 1) cluster_sync_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

size_t gemm_tc_smem_bytes(int N, int stages) { return tc_plan(N, stages).total; }

bool gemm_tc_supported(int fmt, int M, int K, int B) {
  return fmt == kTern2 && M > 0 && K % kSliceK == 0 && B >= 1;
}

namespace {
// Clusters of `cs` CTAs of gemm_tc_kernel (one per SM) that fit at once; 0
// when clusters cannot be launched.
int tc_cluster_capacity(int cs, size_t smem) {
  static int cache[64][3] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const int k = cs == 2 ? 0 : (cs == 4 ? 1 : 2);
  if (dev < 64 && cache[dev][k]) return cache[dev][k] > 0 ? cache[dev][k] : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, (unsigned)cs);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)cs;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel, &cfg) != cudaSuccess) n = 0;
  cudaGetLastError();
  if (dev < 64) cache[dev][k] = n > 0 ? n : -1;
  return n;
}
}  // namespace

cudaError_t launch_gemm_tc_group(const TcLaunch& L0, const TcJob* jobs, const int8_t* const* q, int n,
                                 int Btot, int smem_optin, int num_sms, cudaStream_t s, bool pdl) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return cudaErrorNotSupported;
  if (n < 1 || n > kMaxTcJobs) return cudaErrorInvalidValue;
  cudaError_t e = ensure_max_smem<gemm_tc_kernel>();
  if (e != cudaSuccess) return e;
  if (L0.nvalid <= 0) return cudaSuccess;
  TcLaunch L = L0;
  int dev = 0, per_sm = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  if (e != cudaSuccess) return e;
  // One CTA per SM, always: every CTA allocates all 512 tensor-memory
  // columns, so a second CTA on the SM would wait in tcgen05.alloc until the
  // first one ends -- forever, if both belong to one cluster and the first
  // waits for it at a cluster barrier. More than half of the SM's shared
  // memory per CTA rules that out.
  const size_t smem_floor = (size_t)per_sm / 2 + 1024;
  if (smem_floor > (size_t)smem_optin) return cudaErrorInvalidValue;
  auto stages_for = [&](int N) {
    int st = kMaxTcStages;
    while (st > 2 && tc_plan(N, st).total > (uint32_t)smem_optin - 2048u) --st;
    return st;
  };
  TcGroup G{};
  G.njobs = n;
  int tiles = 0, min_nsb = 1 << 30;
  for (int j = 0; j < n; ++j) {
    G.jobs[j] = jobs[j];
    G.tile_begin[j] = tiles;
    tiles += (jobs[j].M + kTcRows - 1) / kTcRows;
    const int nsb = jobs[j].K / kSliceK;
    min_nsb = nsb < min_nsb ? nsb : min_nsb;
  }
  for (int j = n; j <= kMaxTcJobs; ++j) G.tile_begin[j] = tiles;
  // Token tile N (even tiles: N = ceil(B / nt) rounded up to 16) and K split
  // Z: the pair with the smallest modelled time. A CTA of job j costs (clocks,
  // from traces of this kernel on B200) K_j / 32 / Z MMAs x (200 + 0.75 N),
  // plus the split's exchange 1000 + 30 N (Z - 1). One job: waves x that
  // cost; a group: the larger of its longest CTA and all CTAs' work spread
  // over the SMs. A split needs a sub-block per part, room in CTA 0's stage
  // area for the partials, and its clusters resident at once.
  double best = -1.0;
  int bestN = 16, bestZ = 1;
  for (int nt = 1; nt <= (L.nvalid + 15) / 16; ++nt) {
    int N = (L.nvalid + nt - 1) / nt;
    N = (N + 15) / 16 * 16;
    if (N > 256) continue;
    if ((L.nvalid + N - 1) / N != nt) continue;  // the same tiling as a smaller nt
    const int st = stages_for(N);
    const TcPlan pl = tc_plan(N, st);
    for (int Z = 1; Z <= 4; Z *= 2) {
      if (Z > 1) {
        if (min_nsb < Z) break;
        if ((size_t)(Z - 1) * (kTcRows * (N + 4) + N) * 4 > (size_t)st * pl.stage_bytes) break;
        const long cap = tc_cluster_capacity(Z, smem_floor);
        if (cap <= 0) break;
      }
      const long slots = Z > 1 ? (long)tc_cluster_capacity(Z, smem_floor) * Z : num_sms;
      const double xchg = Z > 1 ? 1000.0 + 30.0 * N * (Z - 1) : 0.0;
      double t;
      if (n == 1) {
        const long ctas = (long)tiles * nt * Z;
        t = (double)((ctas + slots - 1) / slots) * ((double)jobs[0].K / 32.0 / Z * (200.0 + 0.75 * N) + xchg);
      } else {
        double longest = 0.0, work = 0.0;
        for (int j = 0; j < n; ++j) {
          const double c = (double)jobs[j].K / 32.0 / Z * (200.0 + 0.75 * N) + xchg;
          longest = c > longest ? c : longest;
          work += c * (double)((jobs[j].M + kTcRows - 1) / kTcRows) * nt * Z;
        }
        t = work / (double)slots > longest ? work / (double)slots : longest;
      }
      if (best < 0.0 || t < best) {
        best = t;
        bestN = N;
        bestZ = Z;
      }
    }
  }
  L.N = bestN;
  L.ksplit = bestZ;
  const int stages = stages_for(L.N);
  L.stages = stages;
  size_t smem = tc_plan(L.N, stages).total;
  if (smem < smem_floor) smem = smem_floor;
  if (smem > (size_t)smem_optin) return cudaErrorInvalidValue;
  const int nt = (L.nvalid + L.N - 1) / L.N;
  // activations [Btot][K_j] int8, box 128 B x N rows, 128-byte swizzle, zero fill
  for (int j = 0; j < n; ++j) {
    const cuuint64_t dims[2] = {(cuuint64_t)jobs[j].K, (cuuint64_t)Btot};
    const cuuint64_t strides[1] = {(cuuint64_t)jobs[j].K};
    const cuuint32_t box[2] = {128u, (cuuint32_t)L.N};
    const cuuint32_t estr[2] = {1u, 1u};
    if (enc(&G.maps[j], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(q[j]), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  // one CTA per (128-row tile of a job, token tile, part of K)
  const dim3 grid(tiles, nt, L.ksplit);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (L.ksplit > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = (unsigned)L.ksplit;
    ++na;
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = (unsigned)na;
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel, G, L);
}

cudaError_t launch_gemm_tc(const TcLaunch& L, const int8_t* q, int Btot, int smem_optin, int num_sms,
                           cudaStream_t s, bool pdl) {
  TcJob j{};
  j.w = L.w;
  j.y = L.y;
  j.acc = L.acc;
  j.s_x = L.s_x;
  j.w_scale = L.w_scale;
  j.M = L.M;
  j.K = L.K;
  j.ldy = L.ldy;
  return launch_gemm_tc_group(L, &j, &q, 1, Btot, smem_optin, num_sms, s, pdl);
}

}  // namespace ouroq
