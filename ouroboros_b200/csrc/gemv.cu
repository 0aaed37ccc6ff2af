// gemv.cu -- K2 / K3: packed ternary (2-bit) and 1-bit-sign weight x int8
// activation GEMV for small token batches (B <= 8), grouped over up to eight
// matrices per launch.
//
// Reference operator: ops::matvec_q / matmul_q (cluster/src/infer/ops.rs:76-84,
// 219-230), called per named tensor by Stage::wm / wmat_batched
// (cluster/src/infer/mod.rs:138-167). The arithmetic follows north_star
// (int8 activations, int32 accumulation, fp32 epilogue) as fixed in
// oracle/oracle.h.
//
// Design (sm_100a):
//  * Work unit = tile of 32 weight rows x all of K. A CTA (one per SM) walks a
//    contiguous range of tiles across the job list, so a CTA changes job at
//    most a few times.
//  * Weights stream HBM -> shared memory with 1-D bulk copies (one per row
//    per K-slice) into an NS-stage ring tracked by mbarriers. A dedicated
//    producer warp issues them; rows are padded by 16 B so that consumer lanes
//    (one lane per row) read 16-byte chunks without bank conflicts.
//  * Programmatic dependent launch: the producer issues the first NS weight
//    stages BEFORE griddepcontrol.wait (weights never depend on the previous
//    kernel); only the activation copy waits. Successor kernels are released
//    at entry, so their weight prefetch overlaps this kernel's tail.
//  * Activations (int8 [B][K]) sit in shared memory (double-buffered per job
//    switch) and are read as warp-wide broadcasts.
//  * Math: with the device layout of kernels.h, masking a weight word with
//    0x03030303 << 2j (ternary) or 0x01010101 << j (sign) gives four byte
//    lanes = code * 2^(2j) (or bit * 2^j) for four consecutive k, and one
//    dp4a.u32.s32 against the matching int8 word accumulates them. Separate
//    accumulators per mask are shifted back exactly at the end:
//      ternary: acc = sum_j (A_j >> 2j) - sum(q)            (c = w + 1)
//      sign:    acc_g = 2 * sum_j (A_j >> j) - sum_{k in g}(q)
//  * Epilogues in fp32 with explicit _rn intrinsics (no contraction), in the
//    oracle's order, so y is bit-identical to the CPU oracle.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace ouroq {
namespace {

constexpr int kRows = 32;           // rows per tile (one per consumer lane)
constexpr int kCWarps = 8;          // consumer warps
constexpr int kThreads = (kCWarps + 1) * 32;
constexpr int kStages = 4;          // ring depth
constexpr int kTernSliceChunks = 32;  // 16-B chunks per row per stage (512 B)
constexpr int kSignSliceChunks = 16;  // 256 B per row per stage (16 groups)

// Stage row pitch: ternary rows are 512 B of weights + 16 B pad (132 words,
// = 4 mod 32 banks); sign rows are 256 B of weights + 32 B of fp16 group
// scales + 16 B pad (76 words, = 12 mod 32). Both make the eight lanes of a
// quarter-warp hit disjoint banks with 16-byte loads.
template <int FMT>
struct Fmt;
template <>
struct Fmt<kTern2> {
  static constexpr int kSliceChunks = kTernSliceChunks;
  static constexpr int kWeightsPerChunk = 64;
  static constexpr int kPitch = kTernSliceChunks * 16 + 16;
  __device__ static int row_bytes(int K) { return K / 4; }
};
template <>
struct Fmt<kSign1> {
  static constexpr int kSliceChunks = kSignSliceChunks;
  static constexpr int kWeightsPerChunk = 128;
  static constexpr int kPitch = kSignSliceChunks * 16 + 32 + 16;
  __device__ static int row_bytes(int K) { return K / 8; }
};

// Shared-memory plan (dynamic), all offsets 16-byte aligned:
//   [0, 64)                          mbarriers: full[kStages], empty[kStages], xfull[2], xempty[2]
//   stage ring                       kStages * kRows * pitch
//   x buffers                        2 * B * maxK bytes
//   qsum                             2 * B * maxG ints   (ternary: maxG = 1)
//   red / terms                      ternary: kCWarps*B*32 ints; sign: B*slice*32 floats
struct Plan {
  uint32_t ring, xbuf, qsum, red, total;
};

__host__ __device__ inline Plan make_plan(int fmt, int B, int maxK) {
  Plan p;
  const int slice = fmt == kTern2 ? kTernSliceChunks : kSignSliceChunks;
  const int pitch = fmt == kTern2 ? Fmt<kTern2>::kPitch : Fmt<kSign1>::kPitch;
  const int maxG = fmt == kTern2 ? 1 : maxK / 128;
  p.ring = 128;
  p.xbuf = p.ring + kStages * kRows * pitch;
  p.qsum = p.xbuf + 2 * B * maxK;
  p.red = p.qsum + ((2 * B * maxG * 4 + 15) / 16) * 16;
  const uint32_t red_bytes = fmt == kTern2 ? kCWarps * B * 32 * 4 : B * slice * 32 * 4;
  p.total = p.red + red_bytes;
  return p;
}

struct TileInfo {
  int job, row0, rows;
};

__device__ __forceinline__ TileInfo tile_info(const GemvLaunch& L, int t) {
  int j = 0;
#pragma unroll 1
  while (j + 1 < L.njobs && t >= L.jobs[j + 1].tile_begin) ++j;
  TileInfo ti;
  ti.job = j;
  ti.row0 = (t - L.jobs[j].tile_begin) * kRows;
  int r = L.jobs[j].M - ti.row0;
  ti.rows = r < kRows ? r : kRows;
  return ti;
}

template <int FMT>
__device__ __forceinline__ int nslices_of(int K) {
  const int C = K / Fmt<FMT>::kWeightsPerChunk;
  return (C + Fmt<FMT>::kSliceChunks - 1) / Fmt<FMT>::kSliceChunks;
}

// Slice s covers chunks [c0, c1) of the row. Ternary slices are balanced;
// sign slices start at multiples of 16 groups so that their fp16 scales
// (32 B per full slice) stay 16-byte aligned for the bulk copy.
template <int FMT>
__device__ __forceinline__ void slice_range(int K, int s, int ns, int& c0, int& c1) {
  const int C = K / Fmt<FMT>::kWeightsPerChunk;
  const int per = FMT == kTern2 ? (C + ns - 1) / ns : Fmt<FMT>::kSliceChunks;
  c0 = s * per;
  c1 = c0 + per < C ? c0 + per : C;
}

template <int FMT, int B>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ GemvLaunch L) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int SC = Fmt<FMT>::kSliceChunks;
  constexpr int PITCH = Fmt<FMT>::kPitch;

  int maxK = 0;
  for (int j = 0; j < L.njobs; ++j) maxK = L.jobs[j].K > maxK ? L.jobs[j].K : maxK;
  const Plan P = make_plan(FMT, B, maxK);
  const int maxG = FMT == kTern2 ? 1 : maxK / 128;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kStages;
  uint64_t* xfull = empty + kStages;
  uint64_t* xempty = xfull + 2;
  uint8_t* ring = smem + P.ring;
  int8_t* xbuf = reinterpret_cast<int8_t*>(smem + P.xbuf);
  int* qsum = reinterpret_cast<int*>(smem + P.qsum);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // contiguous tile range of this CTA
  const int t_begin = (int)(((long long)blockIdx.x * L.ntiles) / gridDim.x);
  const int t_end = (int)(((long long)(blockIdx.x + 1) * L.ntiles) / gridDim.x);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kCWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&xfull[i], 1);
      mbar_init(&xempty[i], kCWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kCWarps) {
    // ---------------- producer warp ----------------
    uint64_t pol = policy_evict_first();
    // total stage count of this CTA (needed to size the pre-wait prefetch)
    int total = 0;
    for (int t = t_begin; t < t_end; ++t) total += nslices_of<FMT>(L.jobs[tile_info(L, t).job].K);
    const int prefetch = total < kStages ? total : kStages;
    bool waited = false;
    int xi = 0;            // x copies issued
    int x_next_tile = t_begin;  // first tile whose job's x copy is still pending
    int last_job = -1;
    int st = 0;

    // issue the x copies for every job switch among tiles [x_next_tile, upto]
    auto issue_x_upto = [&](int upto) {
      for (; x_next_tile <= upto; ++x_next_tile) {
        const int j = tile_info(L, x_next_tile).job;
        if (j == last_job) continue;
        last_job = j;
        const int buf = xi & 1;
        if (xi >= 2) {
          if (!mbar_wait(&xempty[buf], ((xi >> 1) - 1) & 1, L.status)) return false;
        }
        const GemvJob& J = L.jobs[j];
        const uint32_t bytes = (uint32_t)(B * J.K);
        if (lane == 0) {
          mbar_arrive_expect_tx(&xfull[buf], bytes);
          bulk_g2s(xbuf + (size_t)buf * B * maxK, J.q, bytes, &xfull[buf]);
        }
        __syncwarp();
        ++xi;
      }
      return true;
    };

    bool ok = true;
    for (int t = t_begin; t < t_end && ok; ++t) {
      const TileInfo ti = tile_info(L, t);
      const GemvJob& J = L.jobs[ti.job];
      const int rb = Fmt<FMT>::row_bytes(J.K);
      const int ns = nslices_of<FMT>(J.K);
      for (int s = 0; s < ns; ++s, ++st) {
        if (st == prefetch && !waited) {
          pdl_wait();
          waited = true;
          ok = issue_x_upto(t);
          if (!ok) break;
        } else if (waited) {
          ok = issue_x_upto(t);
          if (!ok) break;
        }
        const int slot = st % kStages;
        if (st >= kStages) {
          if (!mbar_wait(&empty[slot], ((st / kStages) - 1) & 1, L.status)) {
            ok = false;
            break;
          }
        }
        int c0, c1;
        slice_range<FMT>(J.K, s, ns, c0, c1);
        const uint32_t sb = (uint32_t)(c1 - c0) * 16;
        // sign: fp16 scales of the slice, rounded up to 16 B (rows padded on upload)
        const uint32_t scb = FMT == kSign1 ? (uint32_t)(((c1 - c0) * 2 + 15) / 16) * 16 : 0u;
        if (lane == 0) mbar_arrive_expect_tx(&full[slot], (sb + scb) * ti.rows);
        __syncwarp();
        if (lane < ti.rows) {
          uint8_t* dst = ring + (size_t)slot * kRows * PITCH + lane * PITCH;
          const uint8_t* src = J.w + (size_t)(ti.row0 + lane) * rb + (size_t)c0 * 16;
          bulk_g2s_stream(dst, src, sb, &full[slot], pol);
          if (FMT == kSign1) {
            const uint16_t* ssrc = J.scales + (size_t)(ti.row0 + lane) * J.gpad + c0;
            bulk_g2s(dst + SC * 16, ssrc, scb, &full[slot]);
          }
        }
        __syncwarp();
      }
    }
    if (ok && !waited) {
      pdl_wait();
      ok = issue_x_upto(t_end - 1);
    }
    // Drain: every bulk copy issued into this CTA's shared memory must land
    // before the CTA exits (consumers normally wait for all of them already;
    // this matters only after a timed-out wait).
    for (int i = (st > kStages ? st - kStages : 0); i < st; ++i)
      mbar_wait(&full[i % kStages], (i / kStages) & 1, L.status);
    for (int i = (xi > 2 ? xi - 2 : 0); i < xi; ++i) mbar_wait(&xfull[i & 1], (i >> 1) & 1, L.status);
    return;
  }

  // ---------------- consumer warps ----------------
  pdl_wait();
  int* red = reinterpret_cast<int*>(smem + P.red);
  float* terms = reinterpret_cast<float*>(smem + P.red);
  const int nct = kCWarps * 32;
  const int ctid = threadIdx.x;
  int xc = 0;  // x buffers consumed
  int cur_job = -1;
  int st = 0;
  bool ok = true;

  // A failed (timed-out) wait clears `ok`: later waits are skipped but every
  // warp keeps walking the same sequence of named barriers, so the CTA always
  // terminates; the host sees the status word.
  for (int t = t_begin; t < t_end; ++t) {
    const TileInfo ti = tile_info(L, t);
    const GemvJob& J = L.jobs[ti.job];
    const int K = J.K;
    const int ns = nslices_of<FMT>(K);
    if (ti.job != cur_job) {
      if (cur_job >= 0) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&xempty[(xc - 1) & 1]);
      }
      if (ok) ok = mbar_wait(&xfull[xc & 1], (xc >> 1) & 1, L.status);
      cur_job = ti.job;
      ++xc;
      // per-token (ternary) or per-group (sign) activation sums
      const int8_t* xs = xbuf + (size_t)((xc - 1) & 1) * B * maxK;
      int* qs = qsum + ((xc - 1) & 1) * B * maxG;
      named_bar_sync(1, nct);  // previous users of this qsum buffer are done
      if (FMT == kTern2) {
        if (ctid < B) qs[ctid] = 0;
        named_bar_sync(1, nct);
        for (int b = 0; b < B; ++b) {
          int part = 0;
          for (int i = ctid * 16; i < K; i += nct * 16) {
            uint4 v = *reinterpret_cast<const uint4*>(xs + (size_t)b * K + i);
            part = __dp4a((int)v.x, 0x01010101, part);
            part = __dp4a((int)v.y, 0x01010101, part);
            part = __dp4a((int)v.z, 0x01010101, part);
            part = __dp4a((int)v.w, 0x01010101, part);
          }
          part = warp_sum(part);
          if (lane == 0) atomicAdd(&qs[b], part);
        }
      } else {
        const int G = K / 128;
        for (int p = ctid; p < B * G; p += nct) {
          const int b = p / G, g = p % G;
          const int8_t* src = xs + (size_t)b * K + g * 128;
          int part = 0;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            uint4 v = *reinterpret_cast<const uint4*>(src + i * 16);
            part = __dp4a((int)v.x, 0x01010101, part);
            part = __dp4a((int)v.y, 0x01010101, part);
            part = __dp4a((int)v.z, 0x01010101, part);
            part = __dp4a((int)v.w, 0x01010101, part);
          }
          qs[b * maxG + g] = part;
        }
      }
      named_bar_sync(1, nct);
    }
    const int8_t* xs = xbuf + (size_t)((xc - 1) & 1) * B * maxK;
    const int* qs = qsum + ((xc - 1) & 1) * B * maxG;
    const int row = ti.row0 + lane;
    const bool row_ok = lane < ti.rows;

    if (FMT == kTern2) {
      int A[B][4];
#pragma unroll
      for (int b = 0; b < B; ++b)
#pragma unroll
        for (int j = 0; j < 4; ++j) A[b][j] = 0;

      for (int s = 0; s < ns; ++s, ++st) {
        const int slot = st % kStages;
        if (ok) ok = mbar_wait(&full[slot], (st / kStages) & 1, L.status);
        int c0, c1;
        slice_range<FMT>(K, s, ns, c0, c1);
        const uint8_t* wrow = ring + (size_t)slot * kRows * PITCH + lane * PITCH;
        for (int kc = warp; kc < c1 - c0; kc += kCWarps) {
          const uint4 wv = *reinterpret_cast<const uint4*>(wrow + kc * 16);
          const uint32_t wl[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int b = 0; b < B; ++b) {
            const uint4* xp = reinterpret_cast<const uint4*>(xs + (size_t)b * K + (size_t)(c0 + kc) * 64);
#pragma unroll
            for (int t4 = 0; t4 < 4; ++t4) {
              const uint4 xv = xp[t4];
              A[b][0] = dp4a_us(wl[t4] & 0x03030303u, xv.x, A[b][0]);
              A[b][1] = dp4a_us(wl[t4] & 0x0C0C0C0Cu, xv.y, A[b][1]);
              A[b][2] = dp4a_us(wl[t4] & 0x30303030u, xv.z, A[b][2]);
              A[b][3] = dp4a_us(wl[t4] & 0xC0C0C0C0u, xv.w, A[b][3]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
      // cross-warp reduction of the exact per-warp partials
#pragma unroll
      for (int b = 0; b < B; ++b)
        red[(warp * B + b) * 32 + lane] = A[b][0] + (A[b][1] >> 2) + (A[b][2] >> 4) + (A[b][3] >> 6);
      named_bar_sync(2, nct);
      for (int b = warp; b < B; b += kCWarps) {
        int acc = -qs[b];
#pragma unroll
        for (int w = 0; w < kCWarps; ++w) acc += red[(w * B + b) * 32 + lane];
        if (row_ok) {
          const float y = __fmul_rn(__fmul_rn(__int2float_rn(acc), J.w_scale), J.s_x[b]);
          J.y[(size_t)b * J.ldy + row] = y;
          if (J.acc) J.acc[(size_t)b * J.M + row] = acc;
        }
      }
      named_bar_sync(2, nct);
    } else {
      const int G = K / 128;
      float sum[B];
#pragma unroll
      for (int b = 0; b < B; ++b) sum[b] = 0.0f;
      for (int s = 0; s < ns; ++s, ++st) {
        const int slot = st % kStages;
        if (ok) ok = mbar_wait(&full[slot], (st / kStages) & 1, L.status);
        int c0, c1;
        slice_range<FMT>(K, s, ns, c0, c1);
        const uint8_t* wrow = ring + (size_t)slot * kRows * PITCH + lane * PITCH;
        for (int kc = warp; kc < c1 - c0; kc += kCWarps) {
          const uint4 wv = *reinterpret_cast<const uint4*>(wrow + kc * 16);
          const uint32_t wl[4] = {wv.x, wv.y, wv.z, wv.w};
          const int g = c0 + kc;
          const float sc = __half2float(
              __ushort_as_half(*reinterpret_cast<const uint16_t*>(wrow + SC * 16 + kc * 2)));
#pragma unroll
          for (int b = 0; b < B; ++b) {
            const uint4* xp = reinterpret_cast<const uint4*>(xs + (size_t)b * K + (size_t)g * 128);
            int a[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) a[j] = 0;
#pragma unroll
            for (int t4 = 0; t4 < 4; ++t4) {
              const uint4 x0 = xp[2 * t4], x1 = xp[2 * t4 + 1];
              const uint32_t w = wl[t4];
              a[0] = dp4a_us(w & 0x01010101u, x0.x, a[0]);
              a[1] = dp4a_us(w & 0x02020202u, x0.y, a[1]);
              a[2] = dp4a_us(w & 0x04040404u, x0.z, a[2]);
              a[3] = dp4a_us(w & 0x08080808u, x0.w, a[3]);
              a[4] = dp4a_us(w & 0x10101010u, x1.x, a[4]);
              a[5] = dp4a_us(w & 0x20202020u, x1.y, a[5]);
              a[6] = dp4a_us(w & 0x40404040u, x1.z, a[6]);
              a[7] = dp4a_us(w & 0x80808080u, x1.w, a[7]);
            }
            const int sb = a[0] + (a[1] >> 1) + (a[2] >> 2) + (a[3] >> 3) + (a[4] >> 4) +
                           (a[5] >> 5) + (a[6] >> 6) + (a[7] >> 7);
            const int accg = 2 * sb - qs[b * maxG + g];
            terms[(b * SC + kc) * 32 + lane] = __fmul_rn(__int2float_rn(accg), sc);
            if (J.acc && row_ok) J.acc[((size_t)b * J.M + row) * G + g] = accg;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        named_bar_sync(2, nct);
        // ordered (ascending g) fp32 accumulation by the owner warp of each token
#pragma unroll
        for (int b = 0; b < B; ++b) {
          if (b % kCWarps != warp) continue;  // static index keeps sum[] in registers
          float v = sum[b];
          for (int kc = 0; kc < c1 - c0; ++kc) v = __fadd_rn(v, terms[(b * SC + kc) * 32 + lane]);
          sum[b] = v;
        }
        named_bar_sync(2, nct);
      }
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (b % kCWarps == warp && row_ok) J.y[(size_t)b * J.ldy + row] = __fmul_rn(sum[b], J.s_x[b]);
      }
    }
  }
}

template <int FMT, int B>
cudaError_t launch_t(const GemvLaunch& L, int grid, size_t smem, cudaStream_t s, bool pdl) {
  cudaError_t e = ensure_max_smem<gemv_kernel<FMT, B>>();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<FMT, B>, L);
}

template <int FMT>
cudaError_t launch_fmt(const GemvLaunch& L, int grid, size_t smem, cudaStream_t s, bool pdl) {
  switch (L.B) {
    case 1: return launch_t<FMT, 1>(L, grid, smem, s, pdl);
    case 2: return launch_t<FMT, 2>(L, grid, smem, s, pdl);
    case 3: return launch_t<FMT, 3>(L, grid, smem, s, pdl);
    case 4: return launch_t<FMT, 4>(L, grid, smem, s, pdl);
    case 5: return launch_t<FMT, 5>(L, grid, smem, s, pdl);
    case 6: return launch_t<FMT, 6>(L, grid, smem, s, pdl);
    case 7: return launch_t<FMT, 7>(L, grid, smem, s, pdl);
    case 8: return launch_t<FMT, 8>(L, grid, smem, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

size_t gemv_smem_bytes(int fmt, int B, int maxK) { return make_plan(fmt, B, maxK).total; }

cudaError_t launch_gemv(const GemvLaunch& L, int num_sms, cudaStream_t s, bool pdl) {
  if (L.ntiles <= 0) return cudaSuccess;
  int maxK = 0;
  for (int j = 0; j < L.njobs; ++j) maxK = L.jobs[j].K > maxK ? L.jobs[j].K : maxK;
  const size_t smem = gemv_smem_bytes(L.fmt, L.B, maxK);
  const int grid = L.ntiles < num_sms ? L.ntiles : num_sms;
  if (L.fmt == kTern2) return launch_fmt<kTern2>(L, grid, smem, s, pdl);
  if (L.fmt == kSign1) return launch_fmt<kSign1>(L, grid, smem, s, pdl);
  return cudaErrorInvalidValue;
}

}  // namespace ouroq
