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
// bytes and written straight into tensor memory), NT tokens (N: int8
// activations, TMA-loaded into shared memory with the 128-byte swizzle) and a
// contiguous range of groups, walked in stages of four groups:
//   warp 0       producer: per stage, bulk copies of the packed bits and the
//                fp16 scales of the four 32-row tiles, TMA loads of the
//                activations
//   warp 1       allocates tensor memory; one lane issues the MMAs of group g
//                into accumulator D[g % ND], commits them to mbarriers
//   warps 2-5    expand each row's 128 bits of a group into 128 bytes (one
//                tcgen05.st of 32 columns; one warp per lane quarter)
//   warps 6-13   fold: per stage, the token sums Q_g of its groups (from the
//                activation tile) and this row's scales; per group, D_g out of
//                tensor memory, acc_g, the term and the ordered fp32 sum of
//                each (row, token); two warps per lane quarter, one per half
//                of the tokens
//
// Splitting K. With few 128-row tiles (4096 rows: 32 tiles) one CTA per tile
// leaves most SMs idle and each CTA issues 4 MMAs per group for every group
// of K. So the launcher may split the groups over a cluster of Z CTAs (grid
// z): CTA z runs the MMAs of its own range of at most ND groups at once, all
// its accumulators resident in tensor memory. The fp32 fold must still run in
// ascending group order, so it is chained: CTA 0 folds its groups from zero
// and sends its 128 x NT partial sums to CTA 1 (each fold warp its slice, one
// bulk shared-to-shared copy, completion on an mbarrier of CTA 1); CTA 1, which
// has meanwhile parked its own groups' terms in tensor memory, continues the
// same sums with them, and so on; the last CTA writes y. The additions are the
// oracle's, in the oracle's order; only where they run changes.
//
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
constexpr int kSgXWarps = 4;      // expansion warps, one per tensor-memory lane quarter
constexpr int kSgFWarps = 8;      // fold warps, two per lane quarter (token halves)
constexpr int kSgXWarp0 = 2;      // first expansion warp
constexpr int kSgFWarp0 = kSgXWarp0 + kSgXWarps;  // first fold warp
constexpr int kSgThreads = 64 + (kSgXWarps + kSgFWarps) * 32;
constexpr int kSgMaxStages = 6;
constexpr uint32_t kSgA0 = 256;   // first column of the A buffers
constexpr int kSgABufs = 8;
constexpr int kSgMaxD = 8;
constexpr int kSgMaxTok = 32;     // largest token tile
constexpr int kSgMaxSplit = 4;    // CTAs of a cluster splitting the groups

struct SgPlan {
  uint32_t bars, tmem, sxs, qs, chain, chain_bytes, stage0, w_off, sc_off, stage_bytes, total;
  int nd;  // accumulators (groups in flight between the MMAs and the fold)
};

// Stage: [activations: four boxes of NT rows x 128 B, 128-byte swizzle]
// [packed bits: four tiles x four chunks x 512 B][scales: four tiles x four
// groups x 64 B]. Token sums: [stage slot][group][kSgMaxTok tokens] int32.
// Chain buffer: the partial sums passed between the CTAs of a split, [token
// half][row][NT / 2 + 4] fp32 (rows 16-byte aligned and spread over the
// banks; each fold warp's 32 rows contiguous).
__host__ __device__ inline SgPlan sg_plan(int NT, int stages) {
  SgPlan p;
  p.bars = 0;    // full[6], sfree[6], afull[8], afree[8], dfull[8], dfree[8], xfull
  p.tmem = 384;  // allocated tensor-memory address
  p.sxs = 512;   // the token tile's activation scales, fp32 [32]
  p.qs = 640;
  p.chain = p.qs + (uint32_t)stages * kSgGroupsPerStage * kSgMaxTok * 4;
  p.chain_bytes = 2u * kSgRows * (uint32_t)(NT / 2 + 4) * 4u;
  p.stage0 = (p.chain + p.chain_bytes + 1023) & ~1023u;
  p.w_off = (uint32_t)NT * kSgStageK;
  p.sc_off = p.w_off + 4u * kSgGroupsPerStage * 512u;
  p.stage_bytes = (p.sc_off + 4u * kSgGroupsPerStage * 64u + 1023) & ~1023u;
  p.total = p.stage0 + (uint32_t)stages * p.stage_bytes + 1024;  // + alignment slack
  p.nd = 256 / NT < kSgMaxD ? 256 / NT : kSgMaxD;
  return p;
}

// Bounded wait that backs off between polls: for warps that wait long (the
// expansion warps wait for the MMAs to free an A buffer) so that they leave
// the issue slots to the fold warps on the same SM sub-partitions.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity, unsigned* status) {
  for (unsigned i = 0; i < kSpinLimit / 64; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(64);
  }
  atomicExch(status, kDevWaitTimeout);
  return false;
}

// fp32 value of an integer |v| < 2^22, exactly: the 1.5 * 2^23 addend puts v
// in the low mantissa bits (full-rate integer add and float subtract instead
// of the conversion pipe).
__device__ __forceinline__ float small_int_to_float(int v) {
  return __fsub_rn(__int_as_float(v + 0x4B400000), 0x1.8p23f);
}

// The two halves of the cluster barrier (.aligned: the whole warp executes
// them together, hence the __syncwarp).
__device__ __forceinline__ void sg_cluster_arrive() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void sg_cluster_wait() {
  __syncwarp();
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Tensor-memory columns [c, c + W) of this warp's 32 lanes, W = 16 or 8.
template <int W>
__device__ __forceinline__ void tmem_ld_w(uint32_t taddr, uint32_t* r) {
  if constexpr (W == 16)
    tmem_ld16(taddr, r);
  else
    tmem_ld8(taddr, r);
}

// Group range [gb, ge) of CTA z of a split of G groups over Z CTAs.
__host__ __device__ inline int sg_group_begin(int G, int Z, int z) { return (int)((long)G * z / Z); }

// kAcc: also write the group accumulators to P.acc (a debug output; a
// separate instantiation keeps the fold's registers free of it).
template <int NT, bool kAcc>
__global__ void __launch_bounds__(kSgThreads, 1)
    gemm_sign_tc_kernel(const __grid_constant__ CUtensorMap act_map, const __grid_constant__ TcLaunch P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int TW = NT / 2;  // tokens of one fold warp
  const SgPlan pl = sg_plan(NT, P.stages);
  const int S = P.stages, ND = pl.nd;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + pl.bars);
  uint64_t* sfree = full + kSgMaxStages;
  uint64_t* afull = sfree + kSgMaxStages;
  uint64_t* afree = afull + kSgABufs;
  uint64_t* dfull = afree + kSgABufs;
  uint64_t* dfree = dfull + kSgMaxD;
  uint64_t* xfull = dfree + kSgMaxD;  // the previous CTA's partial sums have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + pl.tmem);
  float* sxs = reinterpret_cast<float*>(smem + pl.sxs);
  int* qsb = reinterpret_cast<int*>(smem + pl.qs);
  float* chain = reinterpret_cast<float*>(smem + pl.chain);
  uint8_t* stages = smem + pl.stage0;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kSgRows;
  const int tok_base = P.tok0 + blockIdx.y * NT;
  const int nv = P.nvalid - (int)blockIdx.y * NT < NT ? P.nvalid - (int)blockIdx.y * NT : NT;
  const int G = P.K / kSgGroupK;
  const int C = P.K / 128;  // 16-byte chunks (128 sign bits) per packed row
  // this CTA's groups [gb, gb + ng) (grid z = rank in the cluster)
  const int Z = P.ksplit > 1 ? P.ksplit : 1;
  const int z = Z > 1 ? (int)blockIdx.z : 0;
  const int gb = sg_group_begin(G, Z, z);
  const int ng = sg_group_begin(G, Z, z + 1) - gb;
  const int nstages = (ng + kSgGroupsPerStage - 1) / kSgGroupsPerStage;
  auto sub_of = [&](int i) {  // groups of stage i
    const int left = ng - i * kSgGroupsPerStage;
    return left < kSgGroupsPerStage ? left : kSgGroupsPerStage;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&sfree[i], 1 + kSgFWarps);  // the MMAs' commit and every fold warp
    }
    for (int i = 0; i < kSgABufs; ++i) {
      mbar_init(&afull[i], kSgXWarps);
      mbar_init(&afree[i], 1);
    }
    for (int i = 0; i < kSgMaxD; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dfree[i], kSgFWarps);
    }
    mbar_init(xfull, 1);
    if (z > 0) mbar_arrive_expect_tx(xfull, pl.chain_bytes);  // every fold warp's slice
    fence_mbar_init();
  }
  __syncthreads();  // barriers initialised
  // cluster phase A: every CTA's barriers are initialised (waited for before
  // the chain's sums are sent, or at the end)
  if (Z > 1) sg_cluster_arrive();
  bool waited_a = Z == 1;
  pdl_launch_dependents();
  // tensor memory for every warp but the producer, whose first copies do not
  // wait for it
  uint32_t tmem = 0;
  if (warp != 0) {
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    named_bar_sync(3, kSgThreads - 32);
    tc_fence_after();
    tmem = *tmem_slot;
  }

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
        const int g0 = gb + i * kSgGroupsPerStage;
        const int SUB = sub_of(i);
        uint8_t* st = stages + (size_t)slot * pl.stage_bytes;
        mbar_arrive_expect_tx(&full[slot], (uint32_t)(vt * SUB * (512 + 64) + NT * SUB * 128));
        for (int t = 0; t < vt; ++t) {
          const size_t tile = (size_t)(row0 / kTileRows + t);
          bulk_g2s_stream(st + pl.w_off + t * (kSgGroupsPerStage * 512), P.w + (tile * C + (size_t)g0) * 512,
                          (uint32_t)SUB * 512u, &full[slot], pol);
          bulk_g2s_stream(st + pl.sc_off + t * (kSgGroupsPerStage * 64),
                          reinterpret_cast<const uint8_t*>(P.scales) + (tile * G + (size_t)g0) * 64,
                          (uint32_t)SUB * 64u, &full[slot], pol);
        }
        if (!waited) {
          pdl_wait();  // activations may come from the previous grid
          waited = true;
        }
        for (int u = 0; u < SUB; ++u)
          tma_load_2d(st + (uint32_t)u * NT * 128u, &act_map, (g0 + u) * kSgGroupK, tok_base, &full[slot]);
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
        const int SUB = sub_of(i);
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
  } else if (warp < kSgFWarp0) {
    // ---------------- expansion ----------------
    // A sign word covers k = 32t .. 32t+31 with bit j of byte b holding k =
    // 32t + 4j + b, so (word >> j) & 0x01010101 is the byte codes of four
    // consecutive k: column 8t + j of the group's 32-column A block.
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    bool ok = true;
    int g = 0;
    for (int i = 0; i < nstages; ++i) {
      const int slot = i % S;
      const int SUB = sub_of(i);
      if (ok) ok = mbar_wait(&full[slot], (i / S) & 1, P.status);
      const uint8_t* src = stages + (size_t)slot * pl.stage_bytes + pl.w_off +
                           (r >> 5) * (kSgGroupsPerStage * 512) + (r & 31) * 16;
      for (int u = 0; u < SUB; ++u, ++g) {
        const int b = g % kSgABufs;
        if (ok && g >= kSgABufs) ok = mbar_wait_backoff(&afree[b], ((g / kSgABufs) - 1) & 1, P.status);
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
    // CTA 0 of a split (and every CTA without one) adds each group's term into
    // its sums as the group's MMAs complete. A later CTA of a split computes
    // its terms as its MMAs complete and parks them in tensor memory in place
    // of the accumulators (the launcher gives it at most ND groups, so no
    // accumulator is reused); once the previous CTA's sums arrive, only the
    // ordered additions remain on the chain.
    const int fw = warp - kSgFWarp0;  // 0..7
    const int q = warp & 3;
    const int j0 = (fw >> 2) * TW;    // this warp's tokens [j0, j0 + TW)
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int row = row0 + r;
    // the chain buffer: [token half][row][TW + 4], so a warp's 32 rows x TW
    // sums are one contiguous slice, sent by the warp itself
    constexpr uint32_t kSlice = 32u * (uint32_t)(TW + 4) * 4u;
    float* my_slice = chain + (size_t)((fw >> 2) * kSgRows + q * 32) * (TW + 4);
    float* mine = my_slice + (size_t)lane * (TW + 4);
    const bool chained = z > 0;
    float sum[TW];
#pragma unroll
    for (int j = 0; j < TW; ++j) sum[j] = 0.0f;
    bool ok = true;
    int g = 0;
    for (int i = 0; i < nstages; ++i) {
      const int slot = i % S;
      const int SUB = sub_of(i);
      const uint8_t* st = stages + (size_t)slot * pl.stage_bytes;
      if (ok) ok = mbar_wait(&full[slot], (i / S) & 1, P.status);
      // token sums Q of the stage's groups: fold warp fw < SUB takes group
      // fw, lane t token t (row t of the group's swizzled activation box)
      int* qs = qsb + slot * (kSgGroupsPerStage * kSgMaxTok);
      if (fw < SUB && lane < NT) {
        const int t = lane;
        const uint8_t* act = st + (uint32_t)fw * NT * 128u + t * 128;
        int sq = 0;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = *reinterpret_cast<const uint4*>(act + ((c ^ (t & 7)) * 16));
          sq = __dp4a((int)v.x, 0x01010101, sq);
          sq = __dp4a((int)v.y, 0x01010101, sq);
          sq = __dp4a((int)v.z, 0x01010101, sq);
          sq = __dp4a((int)v.w, 0x01010101, sq);
        }
        qs[fw * kSgMaxTok + t] = sq;
      }
      // the tile's activation scales, once (written by the previous grid,
      // which has completed: the stage's activations were loaded after it)
      if (i == 0 && fw == kSgFWarps - 1 && lane < nv) sxs[lane] = P.s_x[tok_base + lane];
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
        uint32_t dv[TW];
        tmem_ld_w<TW>(tmem + lane_base + (uint32_t)(d * NT + j0), dv);
        // the term of group g: fp32(acc_g) * scale_g, |acc_g| <= 127 * 128
        // (exact through small_int_to_float)
        const int4* q4 = reinterpret_cast<const int4*>(qs + u * kSgMaxTok + j0);
        uint32_t tv[TW];
#pragma unroll
        for (int j4 = 0; j4 < TW / 4; ++j4) {
          const int4 qv = q4[j4];
          const int qq[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = 4 * j4 + e;
            const float term = __fmul_rn(small_int_to_float(2 * (int)dv[j] - qq[e]), sc[u]);
            if (chained)
              tv[j] = __float_as_uint(term);
            else
              sum[j] = __fadd_rn(sum[j], term);
          }
        }
        if (kAcc && row < P.M) {
          // debug output: the group accumulators, [token][row][group]
          int32_t* ap = P.acc + ((size_t)(tok_base + j0) * P.M + row) * G + gb + g;
          const size_t ts = (size_t)P.M * G;
#pragma unroll
          for (int j = 0; j < TW; ++j)
            if (j0 + j < nv) ap[(size_t)j * ts] = 2 * (int)dv[j] - qs[u * kSgMaxTok + j0 + j];
        }
        if (chained) {
          if constexpr (TW == 16)
            tmem_st16(tmem + lane_base + (uint32_t)(d * NT + j0), tv);
          else
            tmem_st8(tmem + lane_base + (uint32_t)(d * NT + j0), tv);
        }
        // the accumulator has been read (a chained CTA's is not reused)
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dfree[d]);
      }
    }
    if (chained) {
      tmem_wait_st();
      // the sums so far, from the previous CTA of the split (waited for even
      // after a failed wait: the copy must not land in a CTA that has left)
      const bool got = mbar_wait(xfull, 0, P.status);
      ok = ok && got;
#pragma unroll
      for (int j = 0; j < TW; j += 4) {
        const float4 v = *reinterpret_cast<const float4*>(mine + j);
        sum[j] = v.x;
        sum[j + 1] = v.y;
        sum[j + 2] = v.z;
        sum[j + 3] = v.w;
      }
      // the ordered additions of this CTA's terms, two groups' loads in flight
      for (int g0 = 0; g0 < ng; g0 += 2) {
        uint32_t ta[TW], tb[TW];
        const uint32_t c0 = tmem + lane_base + (uint32_t)((g0 % ND) * NT + j0);
        const uint32_t c1 = tmem + lane_base + (uint32_t)(((g0 + 1) % ND) * NT + j0);
        if constexpr (TW == 16) {
          tmem_ld16_nw(c0, ta);
          tmem_ld16_nw(c1, tb);
        } else {
          tmem_ld8_nw(c0, ta);
          tmem_ld8_nw(c1, tb);
        }
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < TW; ++j) sum[j] = __fadd_rn(sum[j], __uint_as_float(ta[j]));
        if (g0 + 1 < ng) {
#pragma unroll
          for (int j = 0; j < TW; ++j) sum[j] = __fadd_rn(sum[j], __uint_as_float(tb[j]));
        }
      }
    }
    if (z < Z - 1) {
      // pass the sums on to the next CTA of the split: each warp its slice,
      // one bulk shared-to-shared copy (measured faster than remote stores
      // with a release arrive)
      sg_cluster_wait();  // phase A: its barriers are initialised
      waited_a = true;
#pragma unroll
      for (int j = 0; j < TW; j += 4)
        *reinterpret_cast<float4*>(mine + j) = make_float4(sum[j], sum[j + 1], sum[j + 2], sum[j + 3]);
      fence_proxy_async_smem();  // visible to the bulk copy
      __syncwarp();
      if (lane == 0)
        bulk_s2s_cluster(peer_smem(my_slice, (uint32_t)(z + 1)), my_slice, kSlice,
                         peer_smem(xfull, (uint32_t)(z + 1)));
    } else {
#pragma unroll
      for (int j = 0; j < TW; ++j) {
        const int n = j0 + j;
        if (n < nv && row < P.M) P.y[(size_t)(tok_base + n) * P.ldy + row] = __fmul_rn(sum[j], sxs[n]);
      }
    }
  }
  if (Z > 1) {
    if (!waited_a) sg_cluster_wait();
    // phase B: the next CTA has received this CTA's sums (it waited for them
    // before arriving), so this CTA's shared memory may go
    sg_cluster_arrive();
    sg_cluster_wait();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Clusters of Z CTAs of gemm_sign_tc_kernel<NT> (one per SM) that fit at
// once; 0 when clusters cannot be launched.
template <int NT, bool kAcc>
int sg_cluster_capacity(int Z, size_t smem) {
  static int cache[64][3] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const int k = Z == 2 ? 0 : (Z == 4 ? 1 : 2);
  if (dev < 64 && cache[dev][k]) return cache[dev][k] > 0 ? cache[dev][k] : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, (unsigned)Z);
  cfg.blockDim = dim3(kSgThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)Z;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_sign_tc_kernel<NT, kAcc>, &cfg) != cudaSuccess) n = 0;
  cudaGetLastError();
  if (dev < 64) cache[dev][k] = n > 0 ? n : -1;
  return n;
}

// Split of the groups over a cluster: OUROQ_SIGN_KSPLIT = 1, 2 or 4 forces it
// (where it is possible), otherwise the cost model below chooses.
int sg_forced_split() {
  const char* e = getenv("OUROQ_SIGN_KSPLIT");
  if (!e || !*e) return 0;
  const int v = atoi(e);
  return (v == 1 || v == 2 || v == 4) ? v : 0;
}

template <int NT, bool kAcc>
cudaError_t launch_sign_t(const TcLaunch& L0, const int8_t* q, int Btot, int smem_optin, int num_sms,
                          cudaStream_t s, bool pdl) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return cudaErrorNotSupported;
  cudaError_t e = ensure_max_smem<gemm_sign_tc_kernel<NT, kAcc>>();
  if (e != cudaSuccess) return e;
  TcLaunch L = L0;
  L.N = NT;
  int stages = kSgMaxStages;
  while (stages > 2 && sg_plan(NT, stages).total > (uint32_t)smem_optin - 2048u) --stages;
  L.stages = stages;
  size_t smem = sg_plan(NT, stages).total;
  // One CTA per SM (each allocates all 512 tensor-memory columns; two CTAs
  // of one cluster on an SM would wait for each other): more than half of the
  // SM's shared memory per CTA.
  int dev = 0, per_sm = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  if (e != cudaSuccess) return e;
  if (smem <= (size_t)per_sm / 2) smem = (size_t)per_sm / 2 + 1024;
  if (smem > (size_t)smem_optin) return cudaErrorInvalidValue;
  // The split Z with the smallest modelled time (clocks): waves x (the MMAs
  // of a CTA's groups + fixed cost + the chained fold of the other CTAs'
  // groups and their hand-overs). A split needs every CTA to hold all its
  // accumulators at once (at most ND groups) and its clusters resident.
  const int G = L.K / kSgGroupK;
  const int mt = (L.M + kSgRows - 1) / kSgRows, nt = (L.nvalid + NT - 1) / NT;
  const int nd = sg_plan(NT, stages).nd;
  constexpr double kMmaGroup = 880.0, kFoldGroup = 250.0, kFixed = 1500.0, kHop = 1000.0;
  const int forced = sg_forced_split();
  double best = -1.0;
  int bestZ = 1;
  for (int Z = 1; Z <= kSgMaxSplit; Z *= 2) {
    const int ngmax = (G + Z - 1) / Z;
    if (Z > 1 && (G < Z || ngmax > nd)) continue;
    const long cap = Z > 1 ? sg_cluster_capacity<NT, kAcc>(Z, smem) : num_sms;
    if (cap <= 0) continue;
    const long slots = Z > 1 ? cap * Z : num_sms;
    const long waves = ((long)mt * nt * Z + slots - 1) / slots;
    const double per = Z > 1 ? ngmax * kMmaGroup + kFixed + (Z - 1) * (ngmax * kFoldGroup + kHop)
                             : ngmax * (kMmaGroup > kFoldGroup ? kMmaGroup : kFoldGroup) + kFixed;
    const double t = (double)waves * per;
    if (forced ? Z == forced : (best < 0.0 || t < best)) {
      best = t;
      bestZ = Z;
    }
  }
  L.ksplit = bestZ;
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
  // one CTA per (128-row tile, token tile, part of the groups)
  const dim3 grid(mt, nt, L.ksplit);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kSgThreads, 1, 1);
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
  return cudaLaunchKernelEx(&cfg, gemm_sign_tc_kernel<NT, kAcc>, map, L);
}

}  // namespace

bool gemm_sign_tc_supported(int M, int K, int B) { return M > 0 && K > 0 && K % kSgGroupK == 0 && B >= 1; }

cudaError_t launch_gemm_sign_tc(const TcLaunch& L, const int8_t* q, int Btot, int smem_optin, int num_sms,
                                cudaStream_t s, bool pdl) {
  if (L.nvalid <= 0) return cudaSuccess;
  if (!L.scales) return cudaErrorInvalidValue;
  // token tile: 32 (larger batches take several tiles), or 16
  if (L.acc) {
    if (L.nvalid > 16) return launch_sign_t<32, true>(L, q, Btot, smem_optin, num_sms, s, pdl);
    return launch_sign_t<16, true>(L, q, Btot, smem_optin, num_sms, s, pdl);
  }
  if (L.nvalid > 16) return launch_sign_t<32, false>(L, q, Btot, smem_optin, num_sms, s, pdl);
  return launch_sign_t<16, false>(L, q, Btot, smem_optin, num_sms, s, pdl);
}

}  // namespace ouroq
