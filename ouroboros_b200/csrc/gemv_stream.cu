// gemv_stream.cu -- the decode GEMV for one to eight tokens (K2 at B <= 8):
// packed ternary weights x fp32 activations, the per-token absmax int8
// quantisation fused in, grouped over up to eight matrices per launch.
//
// Reference operator: ops::matvec_q (cluster/src/infer/ops.rs:76-84), called
// once per named tensor by Stage::wm (cluster/src/infer/mod.rs:138-147), seven
// times per layer in run_layer (infer/mod.rs:305-335). Arithmetic: this
// library's BitNet b1.58 form with the conventions fixed by the CPU oracle
// (oracle/oracle.h): s_x = absmax / 127, q = clamp(rint(x / s_x)), int32
// accumulation, y = ((float)acc * w_scale) * s_x -- bit-identical to it.
//
// Why a second GEMV kernel. At one token a layer's five projections move
// 17.4 MB, 117 KB per SM: a few microseconds of HBM time, so what bounds a
// launch is its critical path, not bandwidth. This kernel shortens it:
//  * The weight stream starts at CTA entry: the producer warp copies the
//    launch parameters with one round of independent loads, initialises the
//    ring's mbarriers and issues its copies before anything else runs. With
//    one CTA per SM a CTA's whole share (up to 6 x 32 KB) is in flight at
//    once. Weights never depend on the previous kernel; only the activations
//    do, and only the consumers wait for it (griddepcontrol.wait), so the
//    copies overlap the previous launch's tail and this launch's prologue.
//    (Two CTAs per SM, so that the next launch streams beside this one,
//    measured slower: 8 consumer warps compute too slowly.)
//  * An optional L2 prefetch of the next call's weights (ouroq_set_prefetch),
//    issued once the CTA's own copies are out.
//  * Chunk-major stages. A stage is a K-slice of up to four 32-row tiles of
//    one matrix (one bulk copy per tile: in the tiled layout a K-slice of a
//    tile is contiguous). A consumer warp takes one 16-byte chunk position
//    of the stage, loads the int8 activations of that chunk into registers
//    once and applies them to the same chunk of every tile of the stage: one
//    shared-memory load and 16 mask + 16 dp4a per tile and lane, with 4 x T
//    independent accumulator chains per lane (measured on resident weights:
//    about 45 packed bytes per clock per SM; mma.sync m16n8k32 u8 x s8 with
//    the same masking reached 31). From three tokens on, a stage holds two
//    tiles (five tokens on: one), the masked weight words of a chunk stay in
//    registers and the activations are loaded token by token (broadcast
//    shared-memory loads), so a lane's accumulators still fit its registers;
//    the batched verify of K = 4-8 columns (qwen35.rs:1378-1409) runs here.
//  * A short prologue: the activations of the CTA's matrices are loaded with
//    every load issued before any use, each distinct input row once (gate
//    and up share theirs), reduced and quantised in registers, with the
//    rounding done in the full-rate pipes.
//
// Layout (kernels.h): tile t, chunk c, row r at (t * C + c) * 512 + r * 16.
// In a stage, tile i's chunks [c0, c1) sit at i * (c1 - c0) * 512, so lane r
// reading chunk k of tile i touches 512 contiguous bytes (no bank conflicts).
#include <cuda_runtime.h>

#include "common.cuh"
#include "hadamard.cuh"
#include "kernels.h"

namespace ouroq {
namespace {

constexpr int kRows = kTileRows;
constexpr int kCW = 15;                     // consumer warps (16 with the producer: 128 registers)
constexpr int kSThreads = (kCW + 1) * 32;   // + one producer warp
// Tiles per stage (one accumulator set each) at batch B: four up to two
// tokens, fewer beyond, so that a lane's accumulators stay in registers.
__host__ __device__ constexpr int tiles_for(int B) { return B <= 2 ? 4 : (B <= 4 ? 2 : 1); }
// A prologue row (input i, token b) is encoded as i << kSegShift | b.
constexpr int kSegShift = 3;
constexpr int kSegMask = (1 << kSegShift) - 1;
constexpr uint32_t kStage = 32u * 1024u;    // bytes per ring slot
constexpr int kMaxNS = 6;                   // ring depth limit
constexpr int kMaxIn = kMaxGemvJobs;        // distinct inputs of one CTA
constexpr int kRegUnits = 5;                // 128-value units a warp keeps in registers
constexpr int kMaxGroups = 16;              // tile groups of one CTA whose partials can wait
constexpr int kClusterCtas = 4;             // CTAs of a cluster that share the quantisation
#ifndef OUROQ_STREAM_CLUSTER_MIN_UNITS
// A CTA whose inputs hold more 128-value units than this quantises them
// together with the other CTAs of a cluster (below it the quantisation is one
// round of loads, shorter than the two cluster barriers sharing costs).
#define OUROQ_STREAM_CLUSTER_MIN_UNITS 80
#endif

__host__ __device__ constexpr uint32_t al128(uint32_t v) { return (v + 127u) & ~127u; }

// Shared-memory plan (dynamic part), every region 128-byte aligned.
struct SPlan {
  uint32_t bars, red, xq, ring, total;
};
// `groups`: tile groups whose partial sums are kept until the CTA's end (0:
// one buffer, reduced after every group).
__host__ __device__ inline SPlan splan(int B, int ns, int xcap, int groups) {
  SPlan p;
  p.bars = al128(sizeof(GemvLaunch));
  p.red = p.bars + 128;  // full[6] + empty[6] mbarriers
  p.xq = p.red + al128((uint32_t)(groups > 0 ? groups : 1) * kCW * tiles_for(B) * B * 32 * 4);
  p.ring = p.xq + al128((uint32_t)xcap);
  p.total = p.ring + (uint32_t)ns * kStage;
  return p;
}

// Per-CTA tables, filled by consumer thread 0 before the dependency wait.
struct STab {
  const float* x[kMaxIn];   // distinct fp32 inputs
  int K[kMaxIn];
  int xoff[kMaxIn];         // byte offset of input i's codes [B][K] in xq
  int ufirst[kMaxIn + 1];   // first 128-value unit of input i (all B rows)
  int in_of[kMaxGemvJobs];  // job (relative to the CTA's first job) -> input
  int nin;
  float sx[kMaxIn][kStreamMaxB];  // per-token scales
  int qtot[kMaxIn][kStreamMaxB];  // per-token code sums
  int amax[kMaxIn][kStreamMaxB];  // absmax bits
};

__device__ __forceinline__ int job_of(const GemvLaunch& L, int t) {
  int j = 0;
  while (j + 1 < L.njobs && t >= L.jobs[j + 1].tile_begin) ++j;
  return j;
}

// Stage geometry of a tile group of T tiles of a K-chunk row: slices of at
// most `sc` chunks (kStage / 512 / T, rounded down to a multiple of kCW), cut
// evenly into multiples of kCW where possible.
struct Geo {
  int C, ns, per;
};
__device__ __forceinline__ Geo geo(int K, int T) {
  Geo g;
  g.C = K / 64;
  int sc = (int)(kStage / 512u) / T;
  if (sc >= kCW) sc -= sc % kCW;
  g.ns = (g.C + sc - 1) / sc;
  int per = (g.C + g.ns - 1) / g.ns;
  if (per % kCW) {
    const int up = per + kCW - per % kCW;
    if (up <= sc) per = up;
  }
  g.per = per;
  g.ns = (g.C + per - 1) / per;
  return g;
}

// quant_code (hadamard.cuh) with the rounding done by the 1.5 * 2^23 addend
// instead of rint + float-to-int conversion (both on the quarter-rate
// conversion pipe): for |t| < 2^22, t + 1.5 * 2^23 rounds t to the nearest
// integer, ties to even, exactly as rint does, and that integer sits in the
// low mantissa bits. The tie guard and the division fallback are unchanged,
// so the code is still rint(__fdiv_rn(v, s)) clamped to +-127, bit for bit.
__device__ __forceinline__ int quant_code_fast(float v, float s, float rs) {
  if (s == 0.0f) return 0;
  const float t = __fmul_rn(v, rs);
  const float m = __fadd_rn(t, 0x1.8p23f);
  const float r = __fsub_rn(m, 0x1.8p23f);
  int q;
  if (fabsf(__fsub_rn(t, r)) < 0.5f - 0x1p-14f) {
    q = __float_as_int(m) - 0x4B400000;
  } else {
    q = (int)fminf(fmaxf(rintf(__fdiv_rn(v, s)), -127.0f), 127.0f);
  }
  return q < -127 ? -127 : (q > 127 ? 127 : q);
}

// Four int8 codes of a, b, c, d packed into a word; their sum added to *sum.
__device__ __forceinline__ uint32_t quant4s(float a, float b, float c, float d, float s, float rs,
                                            int* sum) {
  const int c0 = quant_code_fast(a, s, rs), c1 = quant_code_fast(b, s, rs),
            c2 = quant_code_fast(c, s, rs), c3 = quant_code_fast(d, s, rs);
  *sum += c0 + c1 + c2 + c3;
  return (uint32_t)(c0 & 0xFF) | ((uint32_t)(c1 & 0xFF) << 8) | ((uint32_t)(c2 & 0xFF) << 16) |
         ((uint32_t)c3 << 24);
}

// The same four codes without a branch: the rounding of quant_code_fast for
// each value, and `exact` cleared when any of them lies within 2^-14 of a
// tie (or rs overflowed). The caller redoes a unit with quant4s -- the
// division fallback -- when any lane of the warp reports that, so the codes
// are always rint(__fdiv_rn(v, s)) clamped, bit for bit.
__device__ __forceinline__ uint32_t quant4_nobranch(const float* v, float rs, int* sum, bool* exact) {
  uint32_t w = 0;
  int su = 0;
  bool ok = true;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float t = __fmul_rn(v[i], rs);
    const float m = __fadd_rn(t, 0x1.8p23f);
    ok &= fabsf(__fsub_rn(t, __fsub_rn(m, 0x1.8p23f))) < 0.5f - 0x1p-14f;
    int q = __float_as_int(m) - 0x4B400000;
    q = q < -127 ? -127 : (q > 127 ? 127 : q);
    su += q;
    w |= (uint32_t)(q & 0xFF) << (8 * i);
  }
  *sum += su;
  *exact = ok;
  return w;
}

// Relaxed reductions into (possibly another CTA's) shared memory of the
// cluster, and the two halves of the cluster barrier.
__device__ __forceinline__ void red_max_cluster(uint32_t addr, int v) {
  asm volatile("red.relaxed.cluster.shared::cluster.max.s32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void red_add_cluster(uint32_t addr, int v) {
  asm volatile("red.relaxed.cluster.shared::cluster.add.s32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
// (.aligned: the whole warp executes them together, hence the __syncwarp)
__device__ __forceinline__ void cluster_arrive() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  __syncwarp();
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Unit u (128 consecutive values of one token row) -> (input, token, offset
// of the unit in the input's [B][K] block). B <= 2: no division.
template <int B>
__device__ __forceinline__ void unit_at(const STab& S, int u, int& in, int& b, int& off) {
  in = 0;
  while (in + 1 < S.nin && u >= S.ufirst[in + 1]) ++in;
  const int r = u - S.ufirst[in];
  if constexpr (B <= 2)
    b = (B > 1 && r >= S.K[in] / 128) ? 1 : 0;
  else
    b = r / (S.K[in] / 128);
  off = r * 128;  // = b * K + (unit within the row) * 128
}

// The exact path for one unit (some value of the warp's unit lies next to a
// rounding tie, or the scale is 0): codes through quant4s, out of line so
// that the common path stays short. Returns (codes, their sum).
__device__ __noinline__ uint2 quant4_exact(float a, float b, float c, float d, float s, float rs) {
  int sum = 0;
  const uint32_t w = quant4s(a, b, c, d, s, rs, &sum);
  return make_uint2(w, (uint32_t)sum);
}

// Consumer prologue: quantise every distinct input row of the CTA into xq.
// A warp takes units u = warp, warp + kCW, ...; consecutive units of a warp
// almost always belong to one row, so a lane keeps a running max (then sum)
// per row and the warp reduces once per row it leaves, not once per unit.
template <int B>
__device__ void stream_prologue(STab& S, int8_t* xq, int warp, int lane) {
  const int nunits = S.ufirst[S.nin];
  float v[kRegUnits][4];
  int seg[kRegUnits], uoff[kRegUnits];  // row (input * 2 + token) and offset of each unit
  // pass 1: every load issued before any use
#pragma unroll
  for (int k = 0; k < kRegUnits; ++k) {
    const int u = warp + k * kCW;
    seg[k] = -1;
    if (u < nunits) {
      int in, b, off;
      unit_at<B>(S, u, in, b, off);
      seg[k] = (in << kSegShift | b);
      uoff[k] = off;
      const float4 t = *reinterpret_cast<const float4*>(S.x[in] + off + lane * 4);
      v[k][0] = t.x;
      v[k][1] = t.y;
      v[k][2] = t.z;
      v[k][3] = t.w;
    }
  }
  int cur = -1;
  float m = 0.0f;
  auto flush_max = [&]() {
    if (cur >= 0) {
      const float t = warp_max(m);
      if (lane == 0) atomicMax(&S.amax[cur >> kSegShift][cur & kSegMask], __float_as_int(t));
    }
    m = 0.0f;
  };
  auto absmax4 = [](float a, float b, float c, float d) {
    return fmaxf(fmaxf(fabsf(a), fabsf(b)), fmaxf(fabsf(c), fabsf(d)));
  };
#pragma unroll
  for (int k = 0; k < kRegUnits; ++k) {
    if (seg[k] < 0) continue;  // warp-uniform
    if (seg[k] != cur) {
      flush_max();
      cur = seg[k];
    }
    m = fmaxf(m, absmax4(v[k][0], v[k][1], v[k][2], v[k][3]));
  }
  for (int u0 = warp + kRegUnits * kCW; u0 < nunits; u0 += kCW) {  // units beyond the registers
    int in, b, off;
    unit_at<B>(S, u0, in, b, off);
    const float4 t = *reinterpret_cast<const float4*>(S.x[in] + off + lane * 4);
    if ((in << kSegShift | b) != cur) {
      flush_max();
      cur = (in << kSegShift | b);
    }
    m = fmaxf(m, absmax4(t.x, t.y, t.z, t.w));
  }
  flush_max();
  named_bar_sync(1, kCW * 32);
  // every thread derives the scales it needs from the maxima; threads 0..
  // also publish them for the epilogue
  if (threadIdx.x < S.nin * B) {
    const int in = threadIdx.x / B, b = threadIdx.x - in * B;
    S.sx[in][b] = __fdiv_rn(__int_as_float(S.amax[in][b]), 127.0f);
  }
  // pass 2: codes into xq, code sums per row (integer: the order is free).
  // Scales first (a warp's units span one or two rows), then the codes of all
  // register-held units in straight-line code; one warp vote sends the rare
  // unit with a value next to a rounding tie through the exact division.
  float scu[kRegUnits], rsu[kRegUnits];
  {
    int c = -1;
    float sc = 0.0f, rs = 0.0f;
#pragma unroll
    for (int k = 0; k < kRegUnits; ++k) {
      if (seg[k] >= 0 && seg[k] != c) {
        c = seg[k];
        sc = __fdiv_rn(__int_as_float(S.amax[c >> kSegShift][c & kSegMask]), 127.0f);
        rs = __frcp_rn(sc);
      }
      scu[k] = sc;
      rsu[k] = rs;
    }
  }
  uint32_t code[kRegUnits];
  int usum[kRegUnits];
#pragma unroll
  for (int k = 0; k < kRegUnits; ++k) {
    bool ok = true;
    usum[k] = 0;
    code[k] = quant4_nobranch(v[k], rsu[k], &usum[k], &ok);
    ok = (seg[k] < 0) || (ok && scu[k] != 0.0f);
    if (__any_sync(0xffffffffu, !ok)) {
      const uint2 e = quant4_exact(v[k][0], v[k][1], v[k][2], v[k][3], scu[k], rsu[k]);
      code[k] = e.x;
      usum[k] = (int)e.y;
    }
  }
  cur = -1;
  int sum = 0;
  auto flush_sum = [&]() {
    if (cur >= 0) {
      const int t = warp_sum(sum);
      if (lane == 0) atomicAdd(&S.qtot[cur >> kSegShift][cur & kSegMask], t);
    }
    sum = 0;
  };
#pragma unroll
  for (int k = 0; k < kRegUnits; ++k) {
    if (seg[k] < 0) continue;  // warp-uniform
    if (seg[k] != cur) {
      flush_sum();
      cur = seg[k];
    }
    sum += usum[k];
    *reinterpret_cast<uint32_t*>(xq + S.xoff[seg[k] >> kSegShift] + uoff[k] + lane * 4) = code[k];
  }
  for (int u0 = warp + kRegUnits * kCW; u0 < nunits; u0 += kCW) {  // units beyond the registers
    int in, b, off;
    unit_at<B>(S, u0, in, b, off);
    const float4 t = *reinterpret_cast<const float4*>(S.x[in] + off + lane * 4);
    if ((in << kSegShift | b) != cur) {
      flush_sum();
      cur = (in << kSegShift | b);
    }
    const float sc = __fdiv_rn(__int_as_float(S.amax[in][b]), 127.0f);
    *reinterpret_cast<uint32_t*>(xq + S.xoff[in] + off + lane * 4) =
        quant4s(t.x, t.y, t.z, t.w, sc, __frcp_rn(sc), &sum);
  }
  flush_sum();
  named_bar_sync(1, kCW * 32);
}

// The same quantisation shared by the `cs` CTAs of a cluster, which hold the
// same inputs (the union of the cluster's jobs, at the same offsets in every
// CTA's xq). CTA `rank` takes units u = rank + cs * (warp + kCW * k): its
// row maxima go to every CTA's S.amax by remote max-reductions, its codes to
// every CTA's xq by remote stores and its code sums to every S.qtot by remote
// adds. Three cluster barrier phases order it: phase 0 (arrived at by the
// caller once the tables are built, waited for here after the loads are
// issued) -- every CTA's S.amax / S.qtot are zeroed; phase 1 -- every maximum
// is in; phase 2 -- every code and sum is in. Nothing is read from another
// CTA, and nothing is written to one after phase 2, so no CTA can leave while
// a peer still addresses its memory. Results are those of stream_prologue:
// max and integer sums do not depend on the order.
template <int B>
__device__ void stream_prologue_cluster(STab& S, int8_t* xq, int warp, int lane, int cs, int rank) {
  const int nunits = S.ufirst[S.nin];
  const int u0 = rank + cs * warp, ustep = cs * kCW;
  float v[kRegUnits][4];
  int seg[kRegUnits], uoff[kRegUnits];
#pragma unroll
  for (int k = 0; k < kRegUnits; ++k) {
    const int u = u0 + k * ustep;
    seg[k] = -1;
    if (u < nunits) {
      int in, b, off;
      unit_at<B>(S, u, in, b, off);
      seg[k] = (in << kSegShift | b);
      uoff[k] = off;
      const float4 t = *reinterpret_cast<const float4*>(S.x[in] + off + lane * 4);
      v[k][0] = t.x;
      v[k][1] = t.y;
      v[k][2] = t.z;
      v[k][3] = t.w;
    }
  }
  cluster_wait();  // phase 0: the peers' tables are ready for remote updates
  int cur = -1;
  float m = 0.0f;
  auto flush_max = [&]() {
    if (cur >= 0) {
      const float t = warp_max(m);
      if (lane < cs) red_max_cluster(peer_smem(&S.amax[cur >> kSegShift][cur & kSegMask], lane), __float_as_int(t));
    }
    m = 0.0f;
  };
  auto absmax4 = [](float a, float b, float c, float d) {
    return fmaxf(fmaxf(fabsf(a), fabsf(b)), fmaxf(fabsf(c), fabsf(d)));
  };
#pragma unroll
  for (int k = 0; k < kRegUnits; ++k) {
    if (seg[k] < 0) continue;  // warp-uniform
    if (seg[k] != cur) {
      flush_max();
      cur = seg[k];
    }
    m = fmaxf(m, absmax4(v[k][0], v[k][1], v[k][2], v[k][3]));
  }
  for (int u = u0 + kRegUnits * ustep; u < nunits; u += ustep) {  // units beyond the registers
    int in, b, off;
    unit_at<B>(S, u, in, b, off);
    const float4 t = *reinterpret_cast<const float4*>(S.x[in] + off + lane * 4);
    if ((in << kSegShift | b) != cur) {
      flush_max();
      cur = (in << kSegShift | b);
    }
    m = fmaxf(m, absmax4(t.x, t.y, t.z, t.w));
  }
  flush_max();
  cluster_arrive();
  cluster_wait();  // phase 1: every CTA's S.amax holds the full row maxima
  if (threadIdx.x < S.nin * B) {
    const int in = threadIdx.x / B, b = threadIdx.x - in * B;
    S.sx[in][b] = __fdiv_rn(__int_as_float(S.amax[in][b]), 127.0f);
  }
  float scu[kRegUnits], rsu[kRegUnits];
  {
    int c = -1;
    float sc = 0.0f, rs = 0.0f;
#pragma unroll
    for (int k = 0; k < kRegUnits; ++k) {
      if (seg[k] >= 0 && seg[k] != c) {
        c = seg[k];
        sc = __fdiv_rn(__int_as_float(S.amax[c >> kSegShift][c & kSegMask]), 127.0f);
        rs = __frcp_rn(sc);
      }
      scu[k] = sc;
      rsu[k] = rs;
    }
  }
  uint32_t code[kRegUnits];
  int usum[kRegUnits];
#pragma unroll
  for (int k = 0; k < kRegUnits; ++k) {
    bool ok = true;
    usum[k] = 0;
    code[k] = quant4_nobranch(v[k], rsu[k], &usum[k], &ok);
    ok = (seg[k] < 0) || (ok && scu[k] != 0.0f);
    if (__any_sync(0xffffffffu, !ok)) {
      const uint2 e = quant4_exact(v[k][0], v[k][1], v[k][2], v[k][3], scu[k], rsu[k]);
      code[k] = e.x;
      usum[k] = (int)e.y;
    }
  }
  cur = -1;
  int sum = 0;
  auto flush_sum = [&]() {
    if (cur >= 0) {
      const int t = warp_sum(sum);
      if (lane < cs) red_add_cluster(peer_smem(&S.qtot[cur >> kSegShift][cur & kSegMask], lane), t);
    }
    sum = 0;
  };
  auto put = [&](const int8_t* dst, uint32_t w) {
    for (int q = 0; q < cs; ++q) st_cluster_u32(peer_smem(dst, q), w);
  };
#pragma unroll
  for (int k = 0; k < kRegUnits; ++k) {
    if (seg[k] < 0) continue;  // warp-uniform
    if (seg[k] != cur) {
      flush_sum();
      cur = seg[k];
    }
    sum += usum[k];
    put(xq + S.xoff[seg[k] >> kSegShift] + uoff[k] + lane * 4, code[k]);
  }
  for (int u = u0 + kRegUnits * ustep; u < nunits; u += ustep) {  // units beyond the registers
    int in, b, off;
    unit_at<B>(S, u, in, b, off);
    const float4 t = *reinterpret_cast<const float4*>(S.x[in] + off + lane * 4);
    if ((in << kSegShift | b) != cur) {
      flush_sum();
      cur = (in << kSegShift | b);
    }
    const float sc = __fdiv_rn(__int_as_float(S.amax[in][b]), 127.0f);
    put(xq + S.xoff[in] + off + lane * 4, quant4s(t.x, t.y, t.z, t.w, sc, __frcp_rn(sc), &sum));
  }
  flush_sum();
  cluster_arrive();
  cluster_wait();  // phase 2: codes and code sums complete in every CTA
}

// The consumer side of one tile group: TC tiles (1..tiles_for(B), a
// compile-time constant) of one matrix through its G.ns stages; each warp's
// exact partial sums end in red[warp][tile][token][lane].
template <int B, int TC>
__device__ __forceinline__ void consume_group(const Geo& G, const int8_t* xrow, int K,
                                              const uint8_t* ring, uint64_t* full, uint64_t* empty,
                                              int NS, int& st, int& cslot, int& cphase, bool& ok,
                                              unsigned* status, int* red, int warp, int lane) {
  constexpr int T = TC;
  constexpr int TM = tiles_for(B);
  static_assert(T >= 1 && T <= TM, "tile count");
  int A[T][B][4];
#pragma unroll
  for (int i = 0; i < T; ++i)
#pragma unroll
    for (int b = 0; b < B; ++b)
#pragma unroll
      for (int m = 0; m < 4; ++m) A[i][b][m] = 0;
  for (int s = 0; s < G.ns; ++s, ++st) {
    const int slot = cslot;
    if (ok) ok = mbar_wait(&full[slot], cphase, status);
    if (++cslot == NS) {
      cslot = 0;
      cphase ^= 1;
    }
    const int c0 = s * G.per;
    const int nck = (c0 + G.per < G.C ? c0 + G.per : G.C) - c0;
    const uint8_t* sb = ring + (size_t)slot * kStage + lane * 16;
    // chunk k of stage st belongs to warp (k + st) % kCW: leftover chunks of
    // short stages fall on different warps from stage to stage
    for (int k = ((warp - st) % kCW + kCW) % kCW; k < nck; k += kCW) {
      if constexpr (B <= 2) {
        // the activations of the chunk in registers, applied to every tile
        uint4 xv[B][4];
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const uint4* xp = reinterpret_cast<const uint4*>(xrow + (size_t)b * K + (size_t)(c0 + k) * 64);
#pragma unroll
          for (int q = 0; q < 4; ++q) xv[b][q] = xp[q];
        }
        uint4 wv[T];
#pragma unroll
        for (int i = 0; i < T; ++i) wv[i] = *reinterpret_cast<const uint4*>(sb + ((size_t)i * nck + k) * 512);
#pragma unroll
        for (int i = 0; i < T; ++i) {
          const uint32_t wl[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
          for (int b = 0; b < B; ++b) {
            const uint32_t xw[4][4] = {{xv[b][0].x, xv[b][0].y, xv[b][0].z, xv[b][0].w},
                                       {xv[b][1].x, xv[b][1].y, xv[b][1].z, xv[b][1].w},
                                       {xv[b][2].x, xv[b][2].y, xv[b][2].z, xv[b][2].w},
                                       {xv[b][3].x, xv[b][3].y, xv[b][3].z, xv[b][3].w}};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              A[i][b][0] = dp4a_us(wl[q] & 0x03030303u, xw[q][0], A[i][b][0]);
              A[i][b][1] = dp4a_us(wl[q] & 0x0C0C0C0Cu, xw[q][1], A[i][b][1]);
              A[i][b][2] = dp4a_us(wl[q] & 0x30303030u, xw[q][2], A[i][b][2]);
              A[i][b][3] = dp4a_us(wl[q] & 0xC0C0C0C0u, xw[q][3], A[i][b][3]);
            }
          }
        }
      } else {
        // more tokens: the masked weight words of the chunk in registers, the
        // activations loaded token by token (broadcast shared-memory loads)
        uint32_t wm[T][4][4];
#pragma unroll
        for (int i = 0; i < T; ++i) {
          const uint4 wv = *reinterpret_cast<const uint4*>(sb + ((size_t)i * nck + k) * 512);
          const uint32_t wl[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            wm[i][q][0] = wl[q] & 0x03030303u;
            wm[i][q][1] = wl[q] & 0x0C0C0C0Cu;
            wm[i][q][2] = wl[q] & 0x30303030u;
            wm[i][q][3] = wl[q] & 0xC0C0C0C0u;
          }
        }
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const uint4* xp = reinterpret_cast<const uint4*>(xrow + (size_t)b * K + (size_t)(c0 + k) * 64);
          const uint4 x0 = xp[0], x1 = xp[1], x2 = xp[2], x3 = xp[3];
          const uint32_t xw[4][4] = {{x0.x, x0.y, x0.z, x0.w},
                                     {x1.x, x1.y, x1.z, x1.w},
                                     {x2.x, x2.y, x2.z, x2.w},
                                     {x3.x, x3.y, x3.z, x3.w}};
#pragma unroll
          for (int i = 0; i < T; ++i)
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
              for (int m = 0; m < 4; ++m) A[i][b][m] = dp4a_us(wm[i][q][m], xw[q][m], A[i][b][m]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  // exact shift-back of the four masked accumulators
#pragma unroll
  for (int i = 0; i < T; ++i)
#pragma unroll
    for (int b = 0; b < B; ++b)
      red[((warp * TM + i) * B + b) * 32 + lane] =
          A[i][b][0] + (A[i][b][1] >> 2) + (A[i][b][2] >> 4) + (A[i][b][3] >> 6);
}

// This CTA's even share of the next launch's weight ranges, into L2 (the
// next launch then streams them from L2: measured 1.4 us instead of 3.3 us
// for a cold 117 KB per SM).
__device__ __noinline__ void prefetch_next(const GemvLaunch& L) {
  if (L.npf <= 0) return;
  uint64_t total = 0;
  for (int e = 0; e < L.npf; ++e) total += L.pf_bytes[e];
  const uint64_t share = ((total + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
  const uint64_t lo = (uint64_t)blockIdx.x * share;
  const uint64_t hi = lo + share < total ? lo + share : total;
  uint64_t base = 0;
  for (int e = 0; e < L.npf && lo < hi; ++e) {
    const uint64_t end = base + L.pf_bytes[e];
    const uint64_t b0 = lo > base ? lo : base, b1 = hi < end ? hi : end;
    for (uint64_t a = b0; a < b1; a += 32768) {
      const uint64_t n = b1 - a < 32768 ? b1 - a : 32768;
      prefetch_l2(L.pf_ptr[e] + (a - base), (uint32_t)n);
    }
    base = end;
  }
}

template <int B>
__global__ void __launch_bounds__(kSThreads, 1)
    gemv_stream_kernel(const __grid_constant__ GemvLaunch Lp) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ STab S;
  __shared__ int grp_job[kMaxGroups], grp_t0[kMaxGroups], grp_T[kMaxGroups];
  const int NS = Lp.stages;
  const SPlan P = splan(B, NS, Lp.xcap, Lp.defer);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P.bars);
  uint64_t* empty = full + kMaxNS;
  uint8_t* ring = smem + P.ring;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const GemvLaunch& L = *reinterpret_cast<const GemvLaunch*>(smem);

  if (warp == kCW) {
    // ---------------- producer: weights only, never waits for the previous
    // grid. Its 32 lanes copy the launch parameters into shared memory with
    // independent loads (one round trip, instead of the dependent chain of
    // parameter reads a walk over the job table would be), then it issues
    // the copies of every stage the ring can hold.
    {
      const uint32_t* src = reinterpret_cast<const uint32_t*>(&Lp);
      uint32_t* dst = reinterpret_cast<uint32_t*>(smem);
      constexpr int kWords = (int)(sizeof(GemvLaunch) / 4);
      uint32_t v[(kWords + 31) / 32];
#pragma unroll
      for (int r = 0; r < (kWords + 31) / 32; ++r)
        if (r * 32 + lane < kWords) v[r] = src[r * 32 + lane];
#pragma unroll
      for (int r = 0; r < (kWords + 31) / 32; ++r)
        if (r * 32 + lane < kWords) dst[r * 32 + lane] = v[r];
    }
    if (lane == 0) {
      for (int i = 0; i < NS; ++i) {
        mbar_init(&full[i], 1);
        mbar_init(&empty[i], kCW);
      }
      fence_mbar_init();
    }
    __threadfence_block();
    __syncwarp();
    named_bar_arrive(2, kSThreads);  // job table and ring barriers ready for the consumers
    pdl_launch_dependents();
    const int t_begin = L.cta_tile[blockIdx.x], t_end = L.cta_tile[blockIdx.x + 1];
    const uint64_t pol = policy_evict_first();
    int st = 0, pslot = 0, pphase = 0;  // stage count, ring slot, slot wrap parity
    bool ok = true;
    // In a cluster every thread takes part in the prologue's three barrier
    // phases. The producer passes them once the ring is full (before its first
    // wait for a free slot: the consumers free slots only after phase 2), or
    // after its last copy when the ring never fills.
    const bool clustered = Lp.cluster > 1;
    bool joined = !clustered;
    auto join_cluster = [&]() {
      cluster_wait();
      cluster_arrive();
      cluster_wait();
      cluster_arrive();
      cluster_wait();
      joined = true;
    };
    if (clustered) cluster_arrive();  // phase 0
    for (int t0 = t_begin; t0 < t_end && ok;) {
      const int j = job_of(L, t0);
      const GemvJob& J = L.jobs[j];
      const int seg_end =
          (j + 1 < L.njobs && L.jobs[j + 1].tile_begin < t_end) ? L.jobs[j + 1].tile_begin : t_end;
      const uint8_t* wbase = J.w;
      const int tb = J.tile_begin;
      constexpr int TM = tiles_for(B);
      const Geo G0 = geo(J.K, TM);
      for (int tg = t0; tg < seg_end && ok; tg += TM) {
        const int T = seg_end - tg < TM ? seg_end - tg : TM;
        const Geo G = T == TM ? G0 : geo(J.K, T);
        for (int s = 0; s < G.ns; ++s, ++st) {
          const int slot = pslot;
          if (st >= NS && !joined) join_cluster();
          if (st >= NS && !mbar_wait(&empty[slot], pphase ^ 1, L.status)) {
            ok = false;
            break;
          }
          if (++pslot == NS) {
            pslot = 0;
            pphase ^= 1;
          }
          const int c0 = s * G.per;
          const int c1 = c0 + G.per < G.C ? c0 + G.per : G.C;
          const uint32_t nb = (uint32_t)(c1 - c0) * 512u;
          if (lane == 0) {
            uint8_t* dst = ring + (size_t)slot * kStage;
            mbar_arrive_expect_tx(&full[slot], nb * (uint32_t)T);
            const size_t tile0 = (size_t)(tg - tb);
            for (int i = 0; i < T; ++i)
              bulk_g2s_stream(dst + (size_t)i * nb, wbase + ((tile0 + i) * G.C + c0) * 512, nb,
                              &full[slot], pol);
          }
          __syncwarp();
        }
      }
      t0 = seg_end;
    }
    if (!joined) join_cluster();
    if (lane == 0) prefetch_next(L);
    // every copy into this CTA's shared memory lands before the CTA exits
    for (int i = (st > NS ? st - NS : 0); i < st; ++i) mbar_wait(&full[i % NS], (i / NS) & 1, L.status);
    return;
  }

  // ---------------- consumers: distinct inputs and tile groups of the CTA
  named_bar_sync(2, kSThreads);  // the producer has copied the job table and set up the ring
  const int t_begin = L.cta_tile[blockIdx.x], t_end = L.cta_tile[blockIdx.x + 1];
  // the inputs quantised here: those of this CTA's tiles, or in a cluster
  // those of all its CTAs' tiles (the same table in every CTA of it)
  const int cs = L.cluster > 1 ? L.cluster : 1;
  const int rank = cs > 1 ? (int)cluster_rank() : 0;
  const int c0 = (int)blockIdx.x - rank;
  const int u_begin = L.cta_tile[c0], u_end = L.cta_tile[c0 + cs];
  const int j_lo = job_of(L, u_begin);
  if (threadIdx.x == 0) {
    const int j_hi = job_of(L, u_end - 1);
    int nin = 0, xo = 0, uo = 0;
    for (int j = j_lo; j <= j_hi; ++j) {
      const GemvJob& J = L.jobs[j];
      int i = 0;
      while (i < nin && !(S.x[i] == J.xf && S.K[i] == J.K)) ++i;
      if (i == nin) {
        S.x[i] = J.xf;
        S.K[i] = J.K;
        S.xoff[i] = xo;
        S.ufirst[i] = uo;
        for (int b = 0; b < kStreamMaxB; ++b) {
          S.amax[i][b] = 0;
          S.qtot[i][b] = 0;
        }
        xo += B * J.K;
        uo += B * (J.K / 128);
        ++nin;
      }
      S.in_of[j - j_lo] = i;
    }
    S.ufirst[nin] = uo;
    S.nin = nin;
  }
  named_bar_sync(1, kCW * 32);
  if (cs > 1) cluster_arrive();  // phase 0: this CTA's table is ready
  pdl_launch_dependents();

  int8_t* xq = reinterpret_cast<int8_t*>(smem + P.xq);
  int* red = reinterpret_cast<int*>(smem + P.red);
  pdl_wait();
  if (cs > 1)
    stream_prologue_cluster<B>(S, xq, warp, lane, cs, rank);
  else
    stream_prologue<B>(S, xq, warp, lane);

  // tile groups; with L.defer the partial sums of all of them stay in shared
  // memory and are reduced after the last one (one CTA barrier), otherwise
  // each group is reduced (two barriers) before the next reuses the buffer
  const bool defer = L.defer != 0;
  constexpr int TM = tiles_for(B);
  const int gstride = kCW * TM * B * 32;  // ints of one group's partials
  auto reduce_group = [&](int g, const int* rg) {
    const int j = grp_job[g], tg = grp_t0[g], T = grp_T[g];
    const GemvJob& J = L.jobs[j];
    const int in = S.in_of[j - j_lo];
    for (int p = warp; p < T * B; p += kCW) {
      const int i = p / B, b = p - (p / B) * B;
      int acc = -S.qtot[in][b];
#pragma unroll
      for (int w = 0; w < kCW; ++w) acc += rg[((w * TM + i) * B + b) * 32 + lane];
      const int row = (tg + i - J.tile_begin) * kRows + lane;
      if (row < J.M) {
        J.y[(size_t)b * J.ldy + row] = __fmul_rn(__fmul_rn(__int2float_rn(acc), J.w_scale), S.sx[in][b]);
        if (J.acc) J.acc[(size_t)b * J.M + row] = acc;
      }
    }
  };
  int st = 0, cslot = 0, cphase = 0;  // stage count, ring slot, slot wrap parity
  bool ok = true;
  int ngrp = 0;
  for (int t0 = t_begin; t0 < t_end;) {
    const int j = job_of(L, t0);
    const GemvJob& J = L.jobs[j];
    const int in = S.in_of[j - j_lo];
    const int8_t* xrow = xq + S.xoff[in];
    const int K = J.K;
    const int seg_end = (j + 1 < L.njobs && L.jobs[j + 1].tile_begin < t_end) ? L.jobs[j + 1].tile_begin : t_end;
    // groups of TM tiles, the remainder last
    for (int tg = t0; tg < seg_end; tg += TM, ++ngrp) {
      const int T = seg_end - tg < TM ? seg_end - tg : TM;
      const Geo G = geo(K, T);
      const int g = defer ? ngrp : 0;
      int* rg = red + (size_t)g * gstride;
      if (threadIdx.x == 0) {
        grp_job[g] = j;
        grp_t0[g] = tg;
        grp_T[g] = T;
      }
      // the tile count as a compile-time constant: straight-line loop bodies
#define OUROQ_CONSUME(TC) \
  consume_group<B, TC>(G, xrow, K, ring, full, empty, NS, st, cslot, cphase, ok, L.status, rg, warp, lane)
      if constexpr (TM == 4) {
        switch (T) {
          case 4: OUROQ_CONSUME(4); break;
          case 3: OUROQ_CONSUME(3); break;
          case 2: OUROQ_CONSUME(2); break;
          default: OUROQ_CONSUME(1); break;
        }
      } else if constexpr (TM == 2) {
        if (T == 2)
          OUROQ_CONSUME(2);
        else
          OUROQ_CONSUME(1);
      } else {
        OUROQ_CONSUME(1);
      }
#undef OUROQ_CONSUME
      if (!defer) {
        named_bar_sync(1, kCW * 32);
        reduce_group(0, red);
        named_bar_sync(1, kCW * 32);
      }
    }
    t0 = seg_end;
  }
  if (defer) {
    named_bar_sync(1, kCW * 32);
    for (int g = 0; g < ngrp; ++g) reduce_group(g, red + (size_t)g * gstride);
  }
}

// Shared memory one CTA may use (one CTA per SM).
int stream_smem_budget() {
  static int budget[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev < 64 && budget[dev]) return budget[dev];
  int per_sm = 0, reserved = 0, optin = 0;
  if (cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return 0;
  // static shared memory: the same tables at every batch size
  cudaFuncAttributes fa, fb;
  if (cudaFuncGetAttributes(&fa, gemv_stream_kernel<1>) != cudaSuccess ||
      cudaFuncGetAttributes(&fb, gemv_stream_kernel<kStreamMaxB>) != cudaSuccess)
    return 0;
  const int st = (int)(fa.sharedSizeBytes > fb.sharedSizeBytes ? fa.sharedSizeBytes : fb.sharedSizeBytes);
  int b = per_sm - reserved - st;
  if (b > optin - st) b = optin - st;
  if (dev < 64) budget[dev] = b;
  return b;
}

template <int B>
cudaError_t launch_stream_t(const GemvLaunch& L, int grid, size_t smem, cudaStream_t s, bool pdl) {
  static int done[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64 || !done[dev]) {
    e = cudaFuncSetAttribute(gemv_stream_kernel<B>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             stream_smem_budget());
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(gemv_stream_kernel<B>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             100);
    if (e != cudaSuccess) return e;
    if (dev < 64) done[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kSThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (L.cluster > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)L.cluster;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, gemv_stream_kernel<B>, L);
}

// CTAs of gemv_stream_kernel<B> that run at once in clusters of kClusterCtas
// (one CTA per SM; clusters do not span GPCs, so this can be below the SM
// count). 0 when clusters cannot be launched.
template <int B>
int cluster_ctas_t() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev < 64 && cache[dev]) return cache[dev] > 0 ? cache[dev] : 0;
  int n = -1;
  const int budget = stream_smem_budget();
  if (budget > 0 &&
      cudaFuncSetAttribute(gemv_stream_kernel<B>, cudaFuncAttributeMaxDynamicSharedMemorySize, budget) ==
          cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kClusterCtas, 1, 1);
    cfg.blockDim = dim3(kSThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)budget;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kClusterCtas;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemv_stream_kernel<B>, &cfg) == cudaSuccess &&
        clusters > 0)
      n = clusters * kClusterCtas;
  }
  cudaGetLastError();  // a refused query leaves no error behind
  if (dev < 64) cache[dev] = n;
  return n > 0 ? n : 0;
}

int cluster_ctas(int B) {
  switch (B) {
    case 1: return cluster_ctas_t<1>();
    case 2: return cluster_ctas_t<2>();
    case 3: return cluster_ctas_t<3>();
    case 4: return cluster_ctas_t<4>();
    case 5: return cluster_ctas_t<5>();
    case 6: return cluster_ctas_t<6>();
    case 7: return cluster_ctas_t<7>();
    case 8: return cluster_ctas_t<8>();
    default: return 0;
  }
}

}  // namespace

// The prologue's cost in the tile split: quarters of a weight chunk (512
// bytes) that quantising one 128-value input unit of a token is worth on a
// CTA's critical path. Measured on the BitNet-2B layer (B = 1, 5,000 steps):
// 0 (weights only) 8.31 us a step, 2 to 7 quarters 7.85 us, 8 and 12 quarters
// 8.54 us (B = 2: 11.71 us at 0, 11.73 us from 2 to 6). OUROQ_STREAM_UNIT_Q
// overrides it.
int stream_unit_weight() {
  const char* e = getenv("OUROQ_STREAM_UNIT_Q");
  if (e && *e) {
    const int v = atoi(e);
    if (v >= 0 && v <= 256) return v;
  }
  return 4;
}

bool gemv_stream_prepare(GemvLaunch& L, int num_sms, int* grid_out, size_t* smem_out) {
  *grid_out = 0;
  *smem_out = 0;
  if (L.fmt != kTern2 || !L.fused || L.norm.w || L.B < 1 || L.B > kStreamMaxB) return false;
  int tiles = 0;
  for (int j = 0; j < L.njobs; ++j) {
    const GemvJob& J = L.jobs[j];
    if (J.had_block || J.K % 128 || J.K <= 0) return false;
    L.jobs[j].tile_begin = tiles;
    tiles += (J.M + kRows - 1) / kRows;
  }
  L.ntiles = tiles;
  if (tiles <= 0) return true;
  if (tiles > 65535) return false;
  // int8 codes of the distinct inputs of the jobs that tiles [t0, t1) touch
  auto codes_of = [&](int t0, int t1) {
    int jlo = 0, jhi = 0;
    while (jlo + 1 < L.njobs && t0 >= L.jobs[jlo + 1].tile_begin) ++jlo;
    while (jhi + 1 < L.njobs && t1 - 1 >= L.jobs[jhi + 1].tile_begin) ++jhi;
    int x = 0;
    for (int j = jlo; j <= jhi; ++j) {
      bool seen = false;
      for (int i = jlo; i < j; ++i) seen |= L.jobs[i].xf == L.jobs[j].xf && L.jobs[i].K == L.jobs[j].K;
      if (!seen) x += L.B * L.jobs[j].K;
    }
    return x;
  };
  // the split over single CTAs; the largest share of codes a CTA quantises
  auto split = [&](int grid_max, int cs) {
    int grid = tiles < grid_max ? tiles : grid_max;
    balance_tiles(L, grid, 64, stream_unit_weight());
    // no empty CTA beyond the last cluster: the split fills CTAs from the first one on
    while (grid > 1 && L.cta_tile[grid - 1] >= L.cta_tile[grid]) --grid;
    const int used = grid;
    grid = (grid + cs - 1) / cs * cs;  // <= grid_max, a multiple of cs
    for (int c = used + 1; c <= grid; ++c) L.cta_tile[c] = L.cta_tile[used];  // empty CTAs
    return grid;
  };
  int cs = 1;
  int grid = split(num_sms < kMaxGemvCtas ? num_sms : kMaxGemvCtas, 1);
  int xcap = 0;
  for (int c = 0; c < grid; ++c) {
    const int x = codes_of(L.cta_tile[c], L.cta_tile[c + 1]);
    xcap = x > xcap ? x : xcap;
  }
  if (xcap / 128 > OUROQ_STREAM_CLUSTER_MIN_UNITS && grid >= kClusterCtas) {
    // large inputs: quantise each once per cluster instead of once per CTA
    int gmax = cluster_ctas(L.B);
    if (gmax > num_sms) gmax = num_sms;
    if (gmax > kMaxGemvCtas) gmax = kMaxGemvCtas;
    gmax -= gmax % kClusterCtas;
    if (gmax >= kClusterCtas) {
      cs = kClusterCtas;
      grid = split(gmax, cs);
      xcap = 0;
      for (int c = 0; c < grid; c += cs) {
        const int x = codes_of(L.cta_tile[c], L.cta_tile[c + cs]);
        xcap = x > xcap ? x : xcap;
      }
    }
  }
  L.cluster = cs;
  L.xcap = xcap;
  // tile groups of each CTA (runs of up to tiles_for(B) tiles of one matrix)
  const int TM = tiles_for(L.B);
  int maxg = 0;
  for (int c = 0; c < grid; ++c) {
    int n = 0;
    for (int t0 = L.cta_tile[c]; t0 < L.cta_tile[c + 1];) {
      int j = 0;
      while (j + 1 < L.njobs && t0 >= L.jobs[j + 1].tile_begin) ++j;
      const int seg_end = (j + 1 < L.njobs && L.jobs[j + 1].tile_begin < L.cta_tile[c + 1])
                              ? L.jobs[j + 1].tile_begin : L.cta_tile[c + 1];
      n += (seg_end - t0 + TM - 1) / TM;  // full groups of TM, the remainder last
      t0 = seg_end;
    }
    maxg = n > maxg ? n : maxg;
  }
  const int budget = stream_smem_budget();
  if (budget <= 0) return false;
  // keep every group's partials when that still leaves a ring of four stages
  L.defer = maxg <= kMaxGroups && (int)splan(L.B, 4, xcap, maxg).total <= budget ? maxg : 0;
  int ns = kMaxNS;
  while (ns > 2 && (int)splan(L.B, ns, xcap, L.defer).total > budget) --ns;
  if ((int)splan(L.B, ns, xcap, L.defer).total > budget) return false;
  L.stages = ns;
  *grid_out = grid;
  *smem_out = splan(L.B, ns, xcap, L.defer).total;
  return true;
}

cudaError_t launch_gemv_stream(GemvLaunch& L, int grid, size_t smem, cudaStream_t s, bool pdl) {
  if (grid == 0) return cudaSuccess;
  switch (L.B) {
    case 1: return launch_stream_t<1>(L, grid, smem, s, pdl);
    case 2: return launch_stream_t<2>(L, grid, smem, s, pdl);
    case 3: return launch_stream_t<3>(L, grid, smem, s, pdl);
    case 4: return launch_stream_t<4>(L, grid, smem, s, pdl);
    case 5: return launch_stream_t<5>(L, grid, smem, s, pdl);
    case 6: return launch_stream_t<6>(L, grid, smem, s, pdl);
    case 7: return launch_stream_t<7>(L, grid, smem, s, pdl);
    case 8: return launch_stream_t<8>(L, grid, smem, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ouroq
