// gemv.cu -- K2 / K3: packed ternary (2-bit) and 1-bit-sign weight x int8
// activation GEMV for small token batches (B <= 8), grouped over up to eight
// matrices per launch, optionally with the activation quantisation (and the
// blockwise Hadamard rotation) fused into the prologue.
//
// Reference operator: ops::matvec_q / matmul_q (cluster/src/infer/ops.rs:76-84,
// 219-230), called per named tensor by Stage::wm / wmat_batched
// (cluster/src/infer/mod.rs:138-167). The arithmetic is this library's BitNet
// b1.58 form (per-token int8 activations, int32 accumulation, fp32 epilogue) with the conventions
// fixed by the CPU oracle (oracle/oracle.h).
//
// Design (sm_100a):
//  * Work unit = tile of 32 weight rows x all of K. A CTA (one per SM) walks a
//    contiguous range of tiles; the host balances the ranges by weight bytes.
//  * Weights stream HBM -> shared memory through a ring of up to 13 stages
//    tracked by mbarriers, one 1-D bulk copy per stage (a K-slice of a 32-row
//    tile is contiguous in the tiled device layout: 8-32 KB per copy; small
//    copies are limited by the copy engine's op rate, large ones run at HBM
//    speed). A producer warp issues them and never waits for the previous
//    grid: weights do not depend on it.
//  * 15 consumer warps. Before touching weights they wait for the previous
//    grid (programmatic dependent launch), then load the activations of every
//    job of the CTA with ordinary loads (not through the copy queue, where
//    they would sit behind the weight prefetch), optionally rotate them
//    (blockwise Walsh-Hadamard), take the per-token absmax, quantise to int8
//    and keep them in shared memory with their per-group sums.
//  * Consumer lanes (one per row) read chunk c of rows 0..31 = 512 contiguous
//    bytes of a stage: no bank conflicts. Activations are read as broadcasts.
//  * The job table is copied from the kernel parameters into shared memory
//    once: dependent lookups into the parameter bank miss the constant cache
//    one after another.
//  * Math: with the device layout of kernels.h, masking a weight word with
//    0x03030303 << 2j (ternary) or 0x01010101 << j (sign) gives four byte
//    lanes = code * 4^j (or bit * 2^j) for four consecutive k, and one
//    dp4a.u32.s32 against the matching int8 word accumulates them. Separate
//    accumulators per mask are shifted back exactly at the end:
//      ternary: acc = sum_j (A_j >> 2j) - sum(q)            (c = w + 1)
//      sign:    acc_g = 2 * sum_j (A_j >> j) - sum_{k in g}(q)
//    The integer pipe (half the issue rate) bounds this loop at about 64
//    packed-ternary bytes per clock per SM, 1.4x the SM's share of HBM.
//  * Epilogues in fp32 with explicit _rn intrinsics (no contraction), in the
//    oracle's order, so y is bit-identical to the CPU oracle.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "hadamard.cuh"
#include "kernels.h"

namespace ouroq {
namespace {

constexpr int kRows = kTileRows;      // rows per tile (one per consumer lane)
// 15 consumer warps + 1 producer warp = 16 warps: four per SM sub-partition,
// which leaves each thread 128 registers (a 17th warp would cap them at 96).
constexpr int kCWarps = 15;
constexpr int kCThreads = kCWarps * 32;
constexpr int kThreads = kCThreads + 32;
constexpr int kMaxStages = kMaxGemvStages;
constexpr int kTernSliceChunks = 64;  // 16-B chunks per row per stage (32 KB stage)
constexpr int kSignSliceChunks = 32;  // 32 groups per row per stage (16 KB + 2 KB scales)

// Stage layout: weights [chunk][32 rows][16 B]; sign stages append the fp16
// group scales of the slice as [group][32 rows].
template <int FMT>
struct Fmt;
template <>
struct Fmt<kTern2> {
  static constexpr int kSliceChunks = kTernSliceChunks;
  static constexpr int kWeightsPerChunk = 64;
  static constexpr int kStageBytes = kTernSliceChunks * 512;
};
template <>
struct Fmt<kSign1> {
  static constexpr int kSliceChunks = kSignSliceChunks;
  static constexpr int kWeightsPerChunk = 128;
  static constexpr int kStageBytes = kSignSliceChunks * (512 + 64);
};

__host__ __device__ constexpr uint32_t align128(uint32_t v) { return (v + 127u) & ~127u; }

// Shared-memory plan (dynamic), every region 128-byte aligned:
//   job table   copy of the GemvLaunch parameters
//   barriers    full[13], empty[13]
//   ring        stages * stage bytes
//   xwork       xcap bytes: int8 activations [job][B][K] of the CTA's jobs
//   qg          gcap ints: per-(token, 128-group) activation sums
//   sx / qtot   [8 jobs][8 tokens] per-token scales / sums
//   red         ternary: max(2, defer) x kCWarps*B*32 ints; sign: 2 x B*slice*32 floats
struct Plan {
  uint32_t bars, ring, xwork, qg, sx, qtot, red, total;
};

// Deferred reduction (ternary): when the per-warp partials of all the CTA's
// tiles fit in this many bytes, every warp runs through its tiles without a
// CTA barrier and the tiles are reduced together at the end.
constexpr uint32_t kDeferBudget = 48u * 1024u;

__host__ __device__ inline Plan make_plan(int fmt, int B, int stages, int xcap, int gcap,
                                          int defer = 0) {
  Plan p;
  const uint32_t slice = fmt == kTern2 ? kTernSliceChunks : kSignSliceChunks;
  const uint32_t stage = fmt == kTern2 ? Fmt<kTern2>::kStageBytes : Fmt<kSign1>::kStageBytes;
  const uint32_t b = (uint32_t)B;
  p.bars = align128(sizeof(GemvLaunch));
  p.ring = p.bars + 256;
  p.xwork = p.ring + (uint32_t)stages * stage;
  p.qg = p.xwork + align128((uint32_t)xcap);
  p.sx = p.qg + align128((uint32_t)gcap * 4u);
  p.qtot = p.sx + 256;
  p.red = p.qtot + 256;
  // ternary: two buffers of per-warp partials (one barrier per tile), or one
  // slot per tile of the CTA (deferred reduction)
  const uint32_t nbuf = defer > 2 ? (uint32_t)defer : 2u;
  const uint32_t red_bytes = fmt == kTern2 ? nbuf * kCWarps * b * 32u * 4u : 2u * b * slice * 32u * 4u;
  p.total = p.red + align128(red_bytes);
  return p;
}

struct TileInfo {
  int job, row0, rows;
};

__host__ __device__ __forceinline__ TileInfo tile_info(const GemvLaunch& L, int t) {
  int j = 0;
  while (j + 1 < L.njobs && t >= L.jobs[j + 1].tile_begin) ++j;
  TileInfo ti;
  ti.job = j;
  ti.row0 = (t - L.jobs[j].tile_begin) * kRows;
  const int r = L.jobs[j].M - ti.row0;
  ti.rows = r < kRows ? r : kRows;
  return ti;
}

template <int FMT>
__device__ __forceinline__ int chunks_of(int K) {
  return K / Fmt<FMT>::kWeightsPerChunk;
}

template <int FMT>
__device__ __forceinline__ int nslices_of(int K) {
  return (chunks_of<FMT>(K) + Fmt<FMT>::kSliceChunks - 1) / Fmt<FMT>::kSliceChunks;
}

// Slice s covers chunks [c0, c1) of the row (balanced split).
template <int FMT>
__device__ __forceinline__ void slice_range(int K, int s, int ns, int& c0, int& c1) {
  const int C = chunks_of<FMT>(K);
  const int per = (C + ns - 1) / ns;
  c0 = s * per;
  c1 = c0 + per < C ? c0 + per : C;
}

// Position in the weight ring: slot index and how many times it wrapped.
struct RingPos {
  int slot = 0, round = 0;
  __device__ __forceinline__ void next(int ns) {
    if (++slot == ns) {
      slot = 0;
      ++round;
    }
  }
};

// ---------------------------------------------------------------- prologue
// The activations of a CTA's jobs are processed as "units" of 32*E = 128
// consecutive values of one token row, E = 4 per lane; a unit holds whole
// rotation blocks (block <= 128) and exactly one 128-group. Units of all (job, token) rows are numbered consecutively and
// dealt to warps round-robin; each warp loads NB = max(1, 16/E) units before
// using any of them, so a pass costs a few memory round trips, not one per
// unit (in-order issue stalls at the first use of a load).
struct Seg {
  const float* x;     // fp32 row (global)
  int8_t* q;          // int8 row (shared)
  int* qg;            // per-128-group sums (shared)
  int first_unit;     // global index of the row's first unit
  int sidx;           // index into the per-token scale table
};

template <int E>
__device__ __forceinline__ void load_unit(float* v, const float* src) {
#pragma unroll
  for (int i = 0; i < E; i += 4) {
    const float4 t = *reinterpret_cast<const float4*>(src + i);
    v[i] = t.x;
    v[i + 1] = t.y;
    v[i + 2] = t.z;
    v[i + 3] = t.w;
  }
}

// rotate_fwd of hadamard.rs:41-53 on one unit (block hb <= 32*E)
template <int E>
__device__ __forceinline__ void rotate_unit(float* v, const float* signs, int off, int hb,
                                            float hscale, int lane) {
  if (hb <= 0) return;
  if (signs) {
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = __fmul_rn(v[i], signs[off + i]);
  }
  wht_span<E>(v, lane, hb);
#pragma unroll
  for (int i = 0; i < E; ++i) v[i] = __fmul_rn(v[i], hscale);
}

// Four int8 codes packed into a word; their sum is returned through *sum.
// Kept out of line: the prologue runs once per CTA and the code every SM has to
// fetch cold stays small (inlining it measured no faster and cost 30 registers).
__device__ __noinline__ uint32_t quant4(float a, float b, float c, float d, float s, float rs,
                                        int* sum) {
  const int c0 = quant_code(a, s, rs), c1 = quant_code(b, s, rs), c2 = quant_code(c, s, rs),
            c3 = quant_code(d, s, rs);
  *sum += c0 + c1 + c2 + c3;
  return (uint32_t)(c0 & 0xFF) | ((uint32_t)(c1 & 0xFF) << 8) | ((uint32_t)(c2 & 0xFF) << 16) |
         ((uint32_t)c3 << 24);
}

__device__ __forceinline__ int seg_of(const Seg* segs, int nseg, int unit) {
  int s = 0;
  while (s + 1 < nseg && unit >= segs[s + 1].first_unit) ++s;
  return s;
}

// One warp's share of the prologue. Units u = warp, warp + kCWarps, ... of
// the CTA. The first R = max(1, 24/E) of them are loaded (all loads issued before any
// use), rotated and kept in registers across the absmax barrier, so a CTA
// whose rows fit pays a single memory round trip; further units are loaded
// again for the quantisation pass (shared memory leaves L1 too small to hold
// them).
template <int E>
__device__ void prologue_units(const Seg* segs, int nseg, int nunits, const float* signs, int hb,
                               float hscale, int* amax_bits, float* sx, int* qtot, int nscale,
                               int B, int warp, int lane) {
  constexpr int R = E >= 24 ? 1 : 24 / E;
  constexpr int kLanesPerGroup = 128 / E;
  float v[R][E];
  int sg[R], off[R];
  // ---- pass 1: load, rotate, absmax
#pragma unroll
  for (int k = 0; k < R; ++k) {
    const int u = warp + k * kCWarps;
    sg[k] = -1;
    if (u < nunits) {
      sg[k] = seg_of(segs, nseg, u);
      off[k] = (u - segs[sg[k]].first_unit) * 32 * E + lane * E;
      load_unit<E>(v[k], segs[sg[k]].x + off[k]);
    }
  }
  auto absmax_unit = [&](const float* w, int seg) {
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < E; ++i) m = fmaxf(m, fabsf(w[i]));
    m = warp_max(m);
    if (lane == 0) atomicMax(&amax_bits[segs[seg].sidx], __float_as_int(m));
  };
#pragma unroll
  for (int k = 0; k < R; ++k) {
    if (sg[k] < 0) continue;  // warp-uniform
    rotate_unit<E>(v[k], signs, off[k], hb, hscale, lane);
    absmax_unit(v[k], sg[k]);
  }
  // further units (large batches): R at a time, every load of a batch issued
  // before its first use, so a warp pays one memory round trip per R units
  for (int u0 = warp + R * kCWarps; u0 < nunits; u0 += R * kCWarps) {
    float w[R][E];
    int wsg[R], wo[R];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const int u = u0 + k * kCWarps;
      wsg[k] = -1;
      if (u < nunits) {
        wsg[k] = seg_of(segs, nseg, u);
        wo[k] = (u - segs[wsg[k]].first_unit) * 32 * E + lane * E;
        load_unit<E>(w[k], segs[wsg[k]].x + wo[k]);
      }
    }
#pragma unroll
    for (int k = 0; k < R; ++k) {
      if (wsg[k] < 0) continue;
      rotate_unit<E>(w[k], signs, wo[k], hb, hscale, lane);
      absmax_unit(w[k], wsg[k]);
    }
  }
  named_bar_sync(1, kCThreads);
  const int ctid = threadIdx.x;
  if (ctid < nscale && (ctid & 7) < B) sx[ctid] = __fdiv_rn(__int_as_float(amax_bits[ctid]), 127.0f);
  named_bar_sync(1, kCThreads);
  // ---- pass 2: quantise, store int8 codes and 128-group sums; each warp adds
  // the code sums of consecutive units of one row in a register and into the
  // token's total once per row it leaves (integer sums: the order is free)
  int run_seg = -1, run_sum = 0;
  auto flush = [&]() {
    if (run_seg >= 0 && lane % kLanesPerGroup == 0) atomicAdd(&qtot[segs[run_seg].sidx], run_sum);
    run_sum = 0;
  };
  auto quant_unit = [&](const float* w, int seg, int o) {
    if (seg != run_seg) {  // warp-uniform
      flush();
      run_seg = seg;
    }
    const Seg& S = segs[seg];
    const float sc = sx[S.sidx];
    const float rsc = __frcp_rn(sc);
    int sum = 0;
#pragma unroll
    for (int i = 0; i < E; i += 4)
      *reinterpret_cast<uint32_t*>(S.q + o + i) = quant4(w[i], w[i + 1], w[i + 2], w[i + 3], sc, rsc, &sum);
#pragma unroll
    for (int d = kLanesPerGroup / 2; d >= 1; d >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, d);
    if (lane % kLanesPerGroup == 0) {
      S.qg[o / 128] = sum;
      run_sum += sum;
    }
  };
#pragma unroll
  for (int k = 0; k < R; ++k) {
    if (sg[k] < 0) continue;
    quant_unit(v[k], sg[k], off[k]);
  }
  for (int u0 = warp + R * kCWarps; u0 < nunits; u0 += R * kCWarps) {
    float w[R][E];
    int wsg[R], wo[R];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const int u = u0 + k * kCWarps;
      wsg[k] = -1;
      if (u < nunits) {
        wsg[k] = seg_of(segs, nseg, u);
        wo[k] = (u - segs[wsg[k]].first_unit) * 32 * E + lane * E;
        load_unit<E>(w[k], segs[wsg[k]].x + wo[k]);
      }
    }
#pragma unroll
    for (int k = 0; k < R; ++k) {
      if (wsg[k] < 0) continue;
      rotate_unit<E>(w[k], signs, wo[k], hb, hscale, lane);
      quant_unit(w[k], wsg[k], wo[k]);
    }
  }
  flush();
}


// Fused RMSNorm prologue: every job of the launch reads one activation row
// per token. v = x + r (or silu(x) * r), h = v (CTA 0 only), a = v * inv * w
// with inv = 1 / sqrt(mean(v^2) + eps) (ops.rs:12-17, a = (v * inv) * w), then
// the per-token absmax quantisation of a, once for all the CTA's jobs: the
// codes and group sums go to the first job's slots and every job reads them.
// The whole row stays in registers (the host admits only rows of at most
// kNormFusedMaxUnits units), and the sum of squares is combined across warps
// in a fixed order, so every CTA computes the same codes.
template <int B>
__device__ void prologue_norm(const NormSpec& N, int8_t* xq, int* qg, float* sx, int* qtot,
                              int njs, int* amax_bits, float* ssq, float* inv_s, int warp,
                              int lane) {
  constexpr int E = 4, R = 6;
  static_assert(R * kCWarps == kNormFusedMaxUnits, "register budget of the fused norm");
  const int K = N.K;
  const int upt = K / (32 * E);  // units (128 values) per token
  const int nunits = B * upt;
  if (threadIdx.x < B) {
    amax_bits[threadIdx.x] = 0;
    qtot[threadIdx.x] = 0;  // token sums, in the first job's slots (read by every job)
  }
  float v[R][E];
  float ssl[B];
#pragma unroll
  for (int b = 0; b < B; ++b) ssl[b] = 0.0f;
#pragma unroll
  for (int k = 0; k < R; ++k) {
    const int u = warp + k * kCWarps;
    if (u < nunits) {
      const int b = u / upt;
      const size_t at = (size_t)b * K + (size_t)(u - b * upt) * 32 * E + lane * E;
      load_unit<E>(v[k], N.x + at);
      if (N.r) {
        float r[E];
        load_unit<E>(r, N.r + at);
#pragma unroll
        for (int i = 0; i < E; ++i)
          v[k][i] = N.mode == 1 ? v[k][i] / (1.0f + expf(-v[k][i])) * r[i] : v[k][i] + r[i];
      }
      if (N.h && blockIdx.x == 0)
        *reinterpret_cast<float4*>(N.h + at) = make_float4(v[k][0], v[k][1], v[k][2], v[k][3]);
      float s = 0.0f;
#pragma unroll
      for (int i = 0; i < E; ++i) s += v[k][i] * v[k][i];
#pragma unroll
      for (int b2 = 0; b2 < B; ++b2)
        if (b2 == b) ssl[b2] += s;
    }
  }
#pragma unroll
  for (int b = 0; b < B; ++b) {
    const float t = warp_sum_f(ssl[b]);
    if (lane == 0) ssq[b * kCWarps + warp] = t;
  }
  named_bar_sync(1, kCThreads);
  if (threadIdx.x < B) {
    float t = 0.0f;
    for (int w = 0; w < kCWarps; ++w) t += ssq[threadIdx.x * kCWarps + w];
    inv_s[threadIdx.x] = 1.0f / sqrtf(t / (float)K + N.eps);
  }
  named_bar_sync(1, kCThreads);
#pragma unroll
  for (int k = 0; k < R; ++k) {
    const int u = warp + k * kCWarps;
    if (u < nunits) {  // warp-uniform
      const int b = u / upt;
      const int o = (u - b * upt) * 32 * E + lane * E;
      float wv[E];
      load_unit<E>(wv, N.w + o);
      const float iv = inv_s[b];
      float m = 0.0f;
#pragma unroll
      for (int i = 0; i < E; ++i) {
        v[k][i] = v[k][i] * iv * wv[i];
        m = fmaxf(m, fabsf(v[k][i]));
      }
      m = warp_max(m);
      if (lane == 0) atomicMax(&amax_bits[b], __float_as_int(m));
    }
  }
  named_bar_sync(1, kCThreads);
  if (threadIdx.x < B) {
    const float sc = __fdiv_rn(__int_as_float(amax_bits[threadIdx.x]), 127.0f);
    for (int j = 0; j < njs; ++j) sx[j * 8 + threadIdx.x] = sc;
  }
  named_bar_sync(1, kCThreads);
  int tsum[B];
#pragma unroll
  for (int b = 0; b < B; ++b) tsum[b] = 0;
#pragma unroll
  for (int k = 0; k < R; ++k) {
    const int u = warp + k * kCWarps;
    if (u < nunits) {
      const int b = u / upt, ut = u - b * upt;
      const int o = ut * 32 * E + lane * E;
      const float sc = sx[b];
      const float rsc = __frcp_rn(sc);
      int sum = 0;
      *reinterpret_cast<uint32_t*>(xq + (size_t)b * K + o) =
          quant4(v[k][0], v[k][1], v[k][2], v[k][3], sc, rsc, &sum);
      sum = warp_sum(sum);
      if (lane == 0) qg[b * (K / 128) + ut] = sum;
#pragma unroll
      for (int b2 = 0; b2 < B; ++b2)
        if (b2 == b) tsum[b2] += sum;
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int b = 0; b < B; ++b)
      if (tsum[b]) atomicAdd(&qtot[b], tsum[b]);
  }
}

template <int FMT, int B>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ GemvLaunch Lp) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int SC = Fmt<FMT>::kSliceChunks;
  constexpr int STAGE = Fmt<FMT>::kStageBytes;

  // ---- job table -> shared memory (one parallel load instead of serial parameter reads)
  {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(&Lp);
    uint32_t* dst = reinterpret_cast<uint32_t*>(smem);
    for (int i = threadIdx.x; i < (int)(sizeof(GemvLaunch) / 4); i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  const GemvLaunch& L = *reinterpret_cast<const GemvLaunch*>(smem);
  const int NS = L.stages;
  const Plan P = make_plan(FMT, B, NS, L.xcap, L.gcap, L.defer);

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P.bars);
  uint64_t* empty = full + kMaxStages;
  uint8_t* ring = smem + P.ring;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kCWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  // this CTA's tile range (balanced by weight bytes on the host)
  const int t_begin = L.cta_tile[blockIdx.x];
  const int t_end = L.cta_tile[blockIdx.x + 1];
  if (t_begin >= t_end) return;

  if (warp == kCWarps) {
    // ---------------- producer warp: weights only ----------------
    const uint64_t pol = policy_evict_first();
    int st = 0;
    RingPos rp;
    bool ok = true;
    for (int t = t_begin; t < t_end && ok; ++t) {
      const TileInfo ti = tile_info(L, t);
      const GemvJob& J = L.jobs[ti.job];
      const int ns = nslices_of<FMT>(J.K);
      const int C = chunks_of<FMT>(J.K);
      const size_t tile = (size_t)(ti.row0 / kRows);
      for (int s = 0; s < ns; ++s, ++st) {
        const int slot = rp.slot;
        if (rp.round > 0 && !mbar_wait(&empty[slot], (rp.round - 1) & 1, L.status)) {
          ok = false;
          break;
        }
        rp.next(NS);
        int c0, c1;
        slice_range<FMT>(J.K, s, ns, c0, c1);
        const uint32_t wb = (uint32_t)(c1 - c0) * 512;
        const uint32_t sb = FMT == kSign1 ? (uint32_t)(c1 - c0) * 64 : 0u;
        if (lane == 0) {
          uint8_t* dst = ring + (size_t)slot * STAGE;
          mbar_arrive_expect_tx(&full[slot], wb + sb);
          bulk_g2s_stream(dst, J.w + (tile * C + c0) * 512, wb, &full[slot], pol);
          if (FMT == kSign1)
            bulk_g2s(dst + SC * 512, J.scales + (tile * C + c0) * kRows, sb, &full[slot]);
        }
        __syncwarp();
      }
    }
    // Drain: every bulk copy issued into this CTA's shared memory must land
    // before the CTA exits (consumers normally wait for all of them already;
    // this matters only after a timed-out wait).
    for (int i = (st > NS ? st - NS : 0); i < st; ++i)
      mbar_wait(&full[i % NS], (i / NS) & 1, L.status);
    return;
  }

  // ---------------- consumer warps ----------------
  const int ctid = threadIdx.x;
  const int j_lo = tile_info(L, t_begin).job;
  const int j_hi = tile_info(L, t_end - 1).job;
  int8_t* xwork = reinterpret_cast<int8_t*>(smem + P.xwork);
  int* qg_base = reinterpret_cast<int*>(smem + P.qg);
  float* sx_s = reinterpret_cast<float*>(smem + P.sx);    // [job - j_lo][b]
  int* qtot_s = reinterpret_cast<int*>(smem + P.qtot);    // [job - j_lo][b]

  // activations of this CTA's jobs may be produced by the previous grid
  pdl_wait();

  // ---- prologue: activations of jobs j_lo..j_hi -> int8 in shared memory
  const bool shared_x = L.norm.w != nullptr;  // every job reads the first job's codes
  if (shared_x) {
    __shared__ float ssq[2 * kCWarps];
    __shared__ float inv_s[2];
    __shared__ int amax_n[2];
    if constexpr (B <= 2)
      prologue_norm<B>(L.norm, xwork, qg_base, sx_s, qtot_s, j_hi - j_lo + 1, amax_n, ssq, inv_s,
                       warp, lane);
  } else if (L.fused) {
    // one segment per (job, token) row; all jobs of a fused launch share the
    // rotation block (checked on the host), hence one unit size E
    __shared__ Seg segs[kMaxGemvJobs * 8];
    __shared__ int amax_bits[kMaxGemvJobs * 8];
    // units of 128 values (the host routes rotation blocks above 128 through
    // the stand-alone quantiser)
    constexpr int e = 4;
    int nseg = 0, nunits = 0;
    {
      int xoff = 0, goff = 0;
      for (int jj = j_lo; jj <= j_hi; ++jj) {
        const GemvJob& J = L.jobs[jj];
        for (int b = 0; b < B; ++b, ++nseg) {
          if (ctid == 0) {
            segs[nseg].x = J.xf + (size_t)b * J.K;
            segs[nseg].q = xwork + xoff + b * J.K;
            segs[nseg].qg = qg_base + goff + b * (J.K / 128);
            segs[nseg].first_unit = nunits;
            segs[nseg].sidx = (jj - j_lo) * 8 + b;
            amax_bits[(jj - j_lo) * 8 + b] = 0;
            qtot_s[(jj - j_lo) * 8 + b] = 0;
          }
          nunits += J.K / (32 * e);
        }
        xoff += B * J.K;
        goff += B * (J.K / 128);
      }
    }
    named_bar_sync(1, kCThreads);
    const GemvJob& J0 = L.jobs[j_lo];
    prologue_units<e>(segs, nseg, nunits, J0.signs, J0.had_block, J0.had_scale, amax_bits, sx_s,
                      qtot_s, (j_hi - j_lo + 1) * 8, B, warp, lane);
  } else {
    // Pre-quantised codes: every (job, token, 128-group) unit of the CTA's jobs
    // is one 128-byte copy into shared memory plus its code sum. A job's units
    // are contiguous in the source ([B][K] int8), in xwork and in qg, so unit
    // u of job j is at offset (u - first unit of j) * 128 of each; a warp
    // issues kCopyBatch units' loads before it uses any of them.
    constexpr int kCopyBatch = 8;
    __shared__ int ufirst[kMaxGemvJobs + 1], uxoff[kMaxGemvJobs], ugoff[kMaxGemvJobs];
    const int njl = j_hi - j_lo + 1;
    if (ctid == 0) {
      int u = 0, xoff = 0, goff = 0;
      for (int jl = 0; jl < njl; ++jl) {
        const int K = L.jobs[j_lo + jl].K;
        ufirst[jl] = u;
        uxoff[jl] = xoff;
        ugoff[jl] = goff;
        u += B * (K / 128);
        xoff += B * K;
        goff += B * (K / 128);
      }
      ufirst[njl] = u;
    }
    if (ctid < njl * B) {
      const int jl = ctid / B, b = ctid - (ctid / B) * B;
      sx_s[jl * 8 + b] = L.jobs[j_lo + jl].s_x[b];
    }
    named_bar_sync(1, kCThreads);
    const int nunits = ufirst[njl];
    for (int u0 = warp; u0 < nunits; u0 += kCopyBatch * kCWarps) {
      uint32_t v[kCopyBatch];
      int jk[kCopyBatch];
#pragma unroll
      for (int k = 0; k < kCopyBatch; ++k) {
        const int u = u0 + k * kCWarps;
        jk[k] = -1;
        if (u < nunits) {
          int jl = 0;
          while (u >= ufirst[jl + 1]) ++jl;
          jk[k] = jl;
          v[k] = *reinterpret_cast<const uint32_t*>(L.jobs[j_lo + jl].q +
                                                    (size_t)(u - ufirst[jl]) * 128 + lane * 4);
        }
      }
#pragma unroll
      for (int k = 0; k < kCopyBatch; ++k) {
        if (jk[k] < 0) continue;  // warp-uniform
        const int jl = jk[k], ul = u0 + k * kCWarps - ufirst[jl];
        *reinterpret_cast<uint32_t*>(xwork + uxoff[jl] + ul * 128 + lane * 4) = v[k];
        const int sum = warp_sum(__dp4a((int)v[k], 0x01010101, 0));
        if (lane == 0) qg_base[ugoff[jl] + ul] = sum;
      }
    }
  }
  named_bar_sync(1, kCThreads);
  if (FMT == kTern2 && !L.fused) {
    // per-token sums of each job (the fused prologues add them up as they
    // quantise): one warp per (job, token), lanes over groups
    const int npairs = (j_hi - j_lo + 1) * B;
    for (int pr = warp; pr < npairs; pr += kCWarps) {
      const int jl = pr / B, b = pr - (pr / B) * B;
      int goff = 0;
      if (!shared_x)
        for (int jj = j_lo; jj < j_lo + jl; ++jj) goff += B * (L.jobs[jj].K / 128);
      const int G = L.jobs[j_lo + jl].K / 128;
      int s = 0;
      for (int g = lane; g < G; g += 32) s += qg_base[goff + b * G + g];
      s = warp_sum(s);
      if (lane == 0) qtot_s[jl * 8 + b] = s;
    }
    named_bar_sync(1, kCThreads);
  }

  int* red = reinterpret_cast<int*>(smem + P.red);
  float* terms = reinterpret_cast<float*>(smem + P.red);
  int st = 0;
  int first = warp;  // chunk rotation: chunk kc of stage st belongs to warp (kc + st) % kCWarps
  int tpar = 0;      // parity of the ternary partial-sum buffer
  RingPos rp;
  bool ok = true;
  int cur_job = -1, xoff = 0, goff = 0;
  // A failed (timed-out) wait clears `ok`: later waits are skipped but every
  // warp keeps walking the same sequence of named barriers, so the CTA always
  // terminates; the host sees the status word.
  for (int t = t_begin; t < t_end; ++t) {
    const TileInfo ti = tile_info(L, t);
    const GemvJob& J = L.jobs[ti.job];
    const int K = J.K;
    const int G = K / 128;
    const int ns = nslices_of<FMT>(K);
    if (ti.job != cur_job) {
      if (cur_job >= 0 && !shared_x) {
        xoff += B * L.jobs[cur_job].K;
        goff += B * (L.jobs[cur_job].K / 128);
      }
      cur_job = ti.job;
    }
    const int8_t* xs = xwork + xoff;
    const int* qg = qg_base + goff;
    const float* sx = sx_s + (ti.job - j_lo) * 8;
    const int* qtot = qtot_s + (shared_x ? 0 : (ti.job - j_lo) * 8);
    const int row = ti.row0 + lane;
    const bool row_ok = lane < ti.rows;

    if (FMT == kTern2) {
      int A[B][4];
#pragma unroll
      for (int b = 0; b < B; ++b)
#pragma unroll
        for (int j = 0; j < 4; ++j) A[b][j] = 0;

      const int C = chunks_of<FMT>(K);
      const int per = (C + ns - 1) / ns;  // slice_range's split, computed once per tile
      for (int s = 0; s < ns; ++s, ++st) {
        const int slot = rp.slot;
        if (ok) ok = mbar_wait(&full[slot], rp.round & 1, L.status);
        rp.next(NS);
        const int c0 = s * per;
        const int c1 = c0 + per < C ? c0 + per : C;
        const uint8_t* stg = ring + (size_t)slot * STAGE + lane * 16;
        const int nck = c1 - c0;
        // chunk kc belongs to warp (kc + st) % kCWarps: the remainder chunks of
        // a stage land on different warps from stage to stage
        const int8_t* xrow = xs + (size_t)c0 * 64;
        for (int kc = first; kc < nck; kc += 2 * kCWarps) {
          // two chunks per iteration: every shared load is issued before the math
          const bool two = kc + kCWarps < nck;
          const int kd = two ? kc + kCWarps : kc;
          const uint4 wa = *reinterpret_cast<const uint4*>(stg + kc * 512);
          const uint4 wb = *reinterpret_cast<const uint4*>(stg + kd * 512);
          const uint32_t wl[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
          for (int b = 0; b < B; ++b) {
            const uint4* xa = reinterpret_cast<const uint4*>(xrow + (size_t)b * K + kc * 64);
            const uint4* xb = reinterpret_cast<const uint4*>(xrow + (size_t)b * K + kd * 64);
            uint4 xv[8];
#pragma unroll
            for (int t4 = 0; t4 < 4; ++t4) {
              xv[t4] = xa[t4];
              xv[4 + t4] = xb[t4];
            }
#pragma unroll
            for (int t4 = 0; t4 < 8; ++t4) {
              if (t4 >= 4 && !two) break;  // odd chunk count: the second chunk is absent
              A[b][0] = dp4a_us(wl[t4] & 0x03030303u, xv[t4].x, A[b][0]);
              A[b][1] = dp4a_us(wl[t4] & 0x0C0C0C0Cu, xv[t4].y, A[b][1]);
              A[b][2] = dp4a_us(wl[t4] & 0x30303030u, xv[t4].z, A[b][2]);
              A[b][3] = dp4a_us(wl[t4] & 0xC0C0C0C0u, xv[t4].w, A[b][3]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        first = first == 0 ? kCWarps - 1 : first - 1;
      }
      if (L.defer) {
        // this warp's exact partials of the tile, reduced after the last tile
        int* rb = red + ((t - t_begin) * kCWarps + warp) * B * 32;
#pragma unroll
        for (int b = 0; b < B; ++b)
          rb[b * 32 + lane] = A[b][0] + (A[b][1] >> 2) + (A[b][2] >> 4) + (A[b][3] >> 6);
        continue;
      }
      // cross-warp reduction of the exact per-warp partials. Two buffers: a
      // buffer is rewritten two tiles later, after every warp has passed the
      // next tile's barrier, so its readers are done -- one barrier per tile.
      int* rb = red + tpar * (kCWarps * B * 32);
      tpar ^= 1;
#pragma unroll
      for (int b = 0; b < B; ++b)
        rb[(warp * B + b) * 32 + lane] = A[b][0] + (A[b][1] >> 2) + (A[b][2] >> 4) + (A[b][3] >> 6);
      named_bar_sync(2, kCThreads);
      for (int b = warp; b < B; b += kCWarps) {
        int acc = -qtot[b];
#pragma unroll
        for (int w = 0; w < kCWarps; ++w) acc += rb[(w * B + b) * 32 + lane];
        if (row_ok) {
          const float y = __fmul_rn(__fmul_rn(__int2float_rn(acc), J.w_scale), sx[b]);
          J.y[(size_t)b * J.ldy + row] = y;
          if (J.acc) J.acc[(size_t)b * J.M + row] = acc;
        }
      }
    } else {
      float sum[B];
#pragma unroll
      for (int b = 0; b < B; ++b) sum[b] = 0.0f;
      for (int s = 0; s < ns; ++s, ++st) {
        const int slot = rp.slot;
        if (ok) ok = mbar_wait(&full[slot], rp.round & 1, L.status);
        rp.next(NS);
        int c0, c1;
        slice_range<FMT>(K, s, ns, c0, c1);
        const uint8_t* stg = ring + (size_t)slot * STAGE;
        // the stage's terms, in one of two buffers: a buffer is rewritten two
        // stages later, after its reader (the token's owner warp) has passed
        // the next stage's barrier -- one CTA barrier per stage
        float* tb = terms + (st & 1) * (B * SC * 32);
        const int sfirst = ((warp - st) % kCWarps + kCWarps) % kCWarps;
        for (int kc = sfirst; kc < c1 - c0; kc += kCWarps) {
          const uint4 wv = *reinterpret_cast<const uint4*>(stg + kc * 512 + lane * 16);
          const uint32_t wl[4] = {wv.x, wv.y, wv.z, wv.w};
          const int g = c0 + kc;
          const float sc = __half2float(__ushort_as_half(
              *reinterpret_cast<const uint16_t*>(stg + SC * 512 + kc * 64 + lane * 2)));
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
            const int accg = 2 * sb - qg[b * G + g];
            tb[(b * SC + kc) * 32 + lane] = __fmul_rn(__int2float_rn(accg), sc);
            if (J.acc && row_ok) J.acc[((size_t)b * J.M + row) * G + g] = accg;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        named_bar_sync(2, kCThreads);
        // ordered (ascending g) fp32 accumulation by the owner warp of each token
#pragma unroll
        for (int b = 0; b < B; ++b) {
          if (b % kCWarps != warp) continue;  // static index keeps sum[] in registers
          float v = sum[b];
          for (int kc = 0; kc < c1 - c0; ++kc) v = __fadd_rn(v, tb[(b * SC + kc) * 32 + lane]);
          sum[b] = v;
        }
      }
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (b % kCWarps == warp && row_ok) J.y[(size_t)b * J.ldy + row] = __fmul_rn(sum[b], sx[b]);
      }
    }
  }
  if (FMT == kTern2 && L.defer) {
    // every tile's partials are in place: warp w reduces (tile, token) pairs
    // w, w + kCWarps, ... and writes the outputs
    named_bar_sync(2, kCThreads);
    const int ntl = t_end - t_begin;
    for (int i = warp; i < ntl * B; i += kCWarps) {
      const int tl = i / B, b = i - tl * B;
      const TileInfo ti = tile_info(L, t_begin + tl);
      const GemvJob& J = L.jobs[ti.job];
      const int* rb = red + (size_t)tl * kCWarps * B * 32 + b * 32 + lane;
      int acc = -qtot_s[(shared_x ? 0 : (ti.job - j_lo) * 8) + b];
#pragma unroll
      for (int w = 0; w < kCWarps; ++w) acc += rb[w * B * 32];
      if (lane < ti.rows) {
        const int row = ti.row0 + lane;
        const float y =
            __fmul_rn(__fmul_rn(__int2float_rn(acc), J.w_scale), sx_s[(ti.job - j_lo) * 8 + b]);
        J.y[(size_t)b * J.ldy + row] = y;
        if (J.acc) J.acc[(size_t)b * J.M + row] = acc;
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

void balance_tiles(GemvLaunch& L, int grid, int per_chunk, int unit_q) {
  // Tiles of job j weigh K_j / per_chunk (proportional to their bytes); with
  // unit_q > 0 a CTA also pays unit_q / 4 x B per 128-value unit of every
  // distinct input it quantises (its prologue); loads are kept in quarters. The contiguous split that minimises
  // the heaviest CTA: the smallest bound cap for which filling CTAs greedily
  // (a CTA takes the next tile while its load stays within cap) needs at most
  // `grid` CTAs, found by bisection. A launch ends with its heaviest CTA, so
  // this bound is what the split costs.
  const int tiles = L.ntiles;
  auto tile_w = [&](int j) { return 4LL * (L.jobs[j].K / per_chunk); };
  auto input_w = [&](int j) { return (long long)unit_q * L.B * (L.jobs[j].K / 128); };
  // does job j read an input that jobs jf .. j-1 (the CTA's earlier jobs) do not?
  auto new_input = [&](int jf, int j) {
    for (int i = jf; i < j; ++i)
      if (L.jobs[i].xf == L.jobs[j].xf && L.jobs[i].K == L.jobs[j].K) return false;
    return true;
  };
  // greedy fill under cap; returns the CTAs it needs (and writes the split)
  auto fill = [&](long long cap, bool write) {
    int n = 1, j = 0, jf = -1, jprev = -1;
    long long load = 0;
    if (write) L.cta_tile[0] = 0;
    for (int t = 0; t < tiles; ++t) {
      while (j + 1 < L.njobs && t >= L.jobs[j + 1].tile_begin) ++j;
      const long long w = tile_w(j);
      long long x = 0;
      if (jf < 0 || (j != jprev && new_input(jf, j))) x = input_w(j);
      if (jf >= 0 && load + w + x > cap) {
        if (write && n <= grid) L.cta_tile[n] = (uint16_t)t;
        ++n;
        load = 0;
        jf = -1;
        x = input_w(j);
      }
      if (jf < 0) jf = j;
      load += w + x;
      jprev = j;
    }
    if (write)
      for (int c = n; c <= grid; ++c) L.cta_tile[c] = (uint16_t)tiles;
    return n;
  };
  long long lo = 0, hi = 0;
  {
    int j = 0;
    for (int t = 0; t < tiles; ++t) {
      while (j + 1 < L.njobs && t >= L.jobs[j + 1].tile_begin) ++j;
      const long long one = tile_w(j) + input_w(j);
      lo = one > lo ? one : lo;
      hi += one;
    }
  }
  if (hi < lo) hi = lo;
  while (lo < hi) {
    const long long mid = (lo + hi) / 2;
    if (fill(mid, false) <= grid) hi = mid;
    else lo = mid + 1;
  }
  fill(lo, true);
}

bool gemv_prepare(GemvLaunch& L, int num_sms, int smem_optin, int* grid_out, size_t* smem_out) {
  const int wpc = L.fmt == kTern2 ? 64 : 128;
  int tiles = 0;
  long long total = 0;
  for (int j = 0; j < L.njobs; ++j) {
    L.jobs[j].tile_begin = tiles;
    const int nt = (L.jobs[j].M + kRows - 1) / kRows;
    tiles += nt;
    total += (long long)nt * (L.jobs[j].K / wpc);
  }
  L.ntiles = tiles;
  *grid_out = 0;
  *smem_out = 0;
  if (tiles <= 0) return true;
  if (tiles > 65535 || L.B < 1 || L.B > kGemvMaxB) return false;
  int grid = tiles < num_sms ? tiles : num_sms;
  if (grid > kMaxGemvCtas) grid = kMaxGemvCtas;
  (void)total;
  balance_tiles(L, grid, wpc, 0);
  // activations one CTA keeps resident: the jobs its tile range touches (one
  // row for all of them under a fused norm)
  int xcap = 0, gcap = 0;
  if (L.norm.w) {
    if (L.B > 2 || L.norm.K % 128 || L.B * L.norm.K / 128 > kNormFusedMaxUnits) return false;
    for (int j = 0; j < L.njobs; ++j)
      if (L.jobs[j].K != L.norm.K || L.jobs[j].had_block) return false;
    xcap = L.B * L.norm.K;
    gcap = L.B * (L.norm.K / 128);
  }
  for (int c = 0; c < grid && !L.norm.w; ++c) {
    if (L.cta_tile[c] >= L.cta_tile[c + 1]) continue;
    const int jlo = tile_info(L, L.cta_tile[c]).job;
    const int jhi = tile_info(L, L.cta_tile[c + 1] - 1).job;
    int x = 0, g = 0;
    for (int j = jlo; j <= jhi; ++j) {
      x += L.B * L.jobs[j].K;
      g += L.B * (L.jobs[j].K / 128);
    }
    xcap = x > xcap ? x : xcap;
    gcap = g > gcap ? g : gcap;
  }
  L.xcap = xcap;
  L.gcap = gcap;
  // most tiles one CTA owns: the deferred reduction keeps a slot per tile
  int maxt = 0;
  for (int c = 0; c < grid; ++c) {
    const int nt = L.cta_tile[c + 1] - L.cta_tile[c];
    maxt = nt > maxt ? nt : maxt;
  }
  L.defer = L.fmt == kTern2 && (uint32_t)maxt * kCWarps * L.B * 32u * 4u <= kDeferBudget ? maxt : 0;
  // deepest ring that fits next to the activations (4 KB are left for the
  // kernel's static shared memory); capping it at the slices a CTA streams
  // measured slower on the wide shapes and no faster in decode
  const uint32_t budget = (uint32_t)smem_optin - 4096u;
  // the deferred partials must leave room for a ring of at least four stages
  if (L.defer && make_plan(L.fmt, L.B, 4, xcap, gcap, L.defer).total > budget) L.defer = 0;
  int stages = kMaxStages;
  while (stages > 2 && make_plan(L.fmt, L.B, stages, xcap, gcap, L.defer).total > budget) --stages;
  L.stages = stages;
  const size_t smem = make_plan(L.fmt, L.B, stages, xcap, gcap, L.defer).total;
  if (smem > budget) return false;
  *grid_out = grid;
  *smem_out = smem;
  return true;
}

cudaError_t launch_gemv(GemvLaunch& L, int num_sms, int smem_optin, cudaStream_t s, bool pdl) {
  int grid = 0;
  size_t smem = 0;
  if (!gemv_prepare(L, num_sms, smem_optin, &grid, &smem)) return cudaErrorInvalidValue;
  if (grid == 0) return cudaSuccess;
  if (L.fmt == kTern2) return launch_fmt<kTern2>(L, grid, smem, s, pdl);
  if (L.fmt == kSign1) return launch_fmt<kSign1>(L, grid, smem, s, pdl);
  return cudaErrorInvalidValue;
}

}  // namespace ouroq
