// decode.cu -- the step either side of the ternary path in a decode layer
// (cluster/src/infer/mod.rs:298-336), fused into a few kernels:
//   rmsnorm_vec_kernel    y = rmsnorm(x + r) * w, optionally h = x + r (residual);
//                         rmsnorm_kernel for rows of any width or alignment
//   swiglu_norm_vec_kernel  y = rmsnorm(silu(gate) * up) * w (swiglu_norm_kernel
//                         for any width)
//   rope_append_kernel    NeoX RoPE of q and k at the current position, k and v
//                         appended to the layer's KV cache
//   attn_decode_kernel    causal GQA attention, split over cache slices with
//                         the slices merged by the last CTA; optionally with
//                         the RoPE and the append above fused in
// fp32 throughout, like the reference (ops.rs:11-40, mod.rs:337-365). The
// position lives in device memory so that a whole decode step can be
// replayed as a CUDA graph; a position outside the cache is refused in the
// kernels (status word) rather than written.
#include <cuda_runtime.h>

#include <cstdint>
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace ouroq {
namespace {

constexpr int kNormThreads = 256;
constexpr int kHeadDim = 128;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum_f(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.0f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    t = warp_sum_f(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

// Rows of up to kNormMaxVec float4 per thread are held in registers: every
// thread issues all its loads at once (one memory round trip), the block sums
// the squares, then scales and stores. Each thread reads and writes only its
// own elements, so y or h may alias x.
constexpr int kNormVecThreads = 512;
constexpr int kNormMaxVec = 4;  // rows of up to 512 * 4 * 4 = 8192 floats

__device__ __forceinline__ float block_sum_vec(float v, float* red) {
  v = warp_sum_f(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = l < (int)(blockDim.x >> 5) ? red[l] : 0.0f;
    t = warp_sum_f(t);
    if (l == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

// one CTA per row; v = x + r, h = v (if requested), y = v * inv * w with
// inv = 1 / sqrt(mean(v^2) + eps) (ops.rs:12-17)
template <int VPT>
__global__ void __launch_bounds__(kNormVecThreads) rmsnorm_vec_kernel(const float4* x,
                                                                     const float4* r, float4* h,
                                                                     const float4* __restrict__ w,
                                                                     float4* y, int n4, float eps) {
  __shared__ float red[33];
  pdl_launch_dependents();  // the next kernel may start its prologue
  pdl_wait();               // inputs come from the previous kernel
  const size_t base = (size_t)blockIdx.x * n4;
  float4 v[VPT];
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * kNormVecThreads;
    v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < n4) {
      v[j] = x[base + i];
      if (r) {
        const float4 rr = r[base + i];
        v[j].x += rr.x;
        v[j].y += rr.y;
        v[j].z += rr.z;
        v[j].w += rr.w;
      }
    }
    ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  }
  ss = block_sum_vec(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)(4 * n4) + eps);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * kNormVecThreads;
    if (i < n4) {
      if (h) h[base + i] = v[j];
      const float4 ww = w[i];
      y[base + i] = make_float4(v[j].x * inv * ww.x, v[j].y * inv * ww.y, v[j].z * inv * ww.z,
                                v[j].w * inv * ww.w);
    }
  }
}

// y = rmsnorm(silu(g) * u) * w, silu(x) = x / (1 + exp(-x)) (ops.rs:34-36)
__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

template <int VPT>
__global__ void __launch_bounds__(kNormVecThreads) swiglu_norm_vec_kernel(
    const float4* __restrict__ g, const float4* __restrict__ u, const float4* __restrict__ w,
    float4* y, int n4, float eps) {
  __shared__ float red[33];
  pdl_launch_dependents();  // the next kernel may start its prologue
  pdl_wait();               // inputs come from the previous kernel
  const size_t base = (size_t)blockIdx.x * n4;
  float4 a[VPT];
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * kNormVecThreads;
    a[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < n4) {
      const float4 gg = g[base + i], uu = u[base + i];
      a[j] = make_float4(silu_mul(gg.x, uu.x), silu_mul(gg.y, uu.y), silu_mul(gg.z, uu.z),
                         silu_mul(gg.w, uu.w));
    }
    ss += a[j].x * a[j].x + a[j].y * a[j].y + a[j].z * a[j].z + a[j].w * a[j].w;
  }
  ss = block_sum_vec(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)(4 * n4) + eps);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * kNormVecThreads;
    if (i < n4) {
      const float4 ww = w[i];
      y[base + i] = make_float4(a[j].x * inv * ww.x, a[j].y * inv * ww.y, a[j].z * inv * ww.z,
                                a[j].w * inv * ww.w);
    }
  }
}

// Rows of any length or alignment: a strided loop per CTA.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float* x, const float* r,
                                                               float* h,
                                                               const float* __restrict__ w,
                                                               float* y, int n, float eps) {
  __shared__ float red[32];
  pdl_launch_dependents();  // the next kernel may start its prologue
  pdl_wait();               // inputs come from the previous kernel
  const size_t row = blockIdx.x;
  const float* xr = x + row * n;
  const float* rr = r ? r + row * n : nullptr;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = rr ? xr[i] + rr[i] : xr[i];
    ss += v * v;
  }
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = rr ? xr[i] + rr[i] : xr[i];
    if (h) h[row * n + i] = v;
    y[row * n + i] = v * inv * w[i];
  }
}

__global__ void __launch_bounds__(kNormThreads) swiglu_norm_kernel(const float* __restrict__ g,
                                                                   const float* __restrict__ u,
                                                                   const float* __restrict__ w,
                                                                   float* __restrict__ y, int n,
                                                                   float eps) {
  __shared__ float red[32];
  pdl_launch_dependents();  // the next kernel may start its prologue
  pdl_wait();               // inputs come from the previous kernel
  const size_t row = blockIdx.x;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float a = silu_mul(g[row * n + i], u[row * n + i]);
    y[row * n + i] = a;
    ss += a * a;
  }
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) y[row * n + i] = y[row * n + i] * inv * w[i];
}

// cos and sin of pos * theta_i, theta_i = 1 / base^(2i/128) (ops.rs:24-26)
__device__ __forceinline__ void rope_cs(long long pos, int i, float base, float& c, float& s) {
  const float theta = 1.0f / powf(base, (float)(2 * i) / (float)kHeadDim);
  const float ang = (float)pos * theta;
  c = cosf(ang);
  s = sinf(ang);
}

// grid (B, n_head + n_kv), block 64: one head per CTA, lane i rotates the
// pair (i, i + 64) (NeoX, ops.rs:21-33). Query heads are rotated in place;
// key heads are rotated into the cache at pos, value heads copied there.
__global__ void rope_append_kernel(DecodeAttn P) {
  pdl_launch_dependents();  // the next kernel may start its prologue
  pdl_wait();               // inputs come from the previous kernel
  const int b = blockIdx.x, hd = blockIdx.y, i = threadIdx.x;
  const long long pos = *P.pos;
  if (pos < 0 || pos >= P.tmax) {
    if (hd == 0 && i == 0) atomicExch(P.status, kDevBadPosition);
    return;
  }
  float c, s;
  rope_cs(pos, i, P.rope_base, c, s);
  if (hd < P.n_head) {
    float* v = P.q + ((size_t)b * P.n_head + hd) * kHeadDim;
    const float x0 = v[i], x1 = v[i + 64];
    v[i] = x0 * c - x1 * s;
    v[i + 64] = x1 * c + x0 * s;
    return;
  }
  const int kv = hd - P.n_head;
  const float* k = P.k + ((size_t)b * P.n_kv + kv) * kHeadDim;
  const float* vv = P.v + ((size_t)b * P.n_kv + kv) * kHeadDim;
  const size_t at = (((size_t)b * P.n_kv + kv) * P.tmax + pos) * kHeadDim;
  const float x0 = k[i], x1 = k[i + 64];
  P.kcache[at + i] = x0 * c - x1 * s;
  P.kcache[at + i + 64] = x1 * c + x0 * s;
  P.vcache[at + i] = vv[i];
  P.vcache[at + i + 64] = vv[i + 64];
}

// ---- decode attention: one launch per layer ----
//
// grid (B, n_kv, S), block NW + 1 warps, where G = n_head / n_kv query heads
// share a KV head, kG is G rounded up to a power of two (lanes of heads >= G
// idle) and NW = 2 kG compute warps (kG for kG = 8). The CTA takes cache positions [t0, t1) of the causal range
// [0, pos], cut into S equal slices from the device-side position. The last
// warp (one lane) streams the slice in stages of 32 positions: K by a 2-D
// tensor copy in four 32 x 32 boxes with the 128-byte swizzle (16-byte unit
// u of row r lands at u ^ (r & 7)), V by a plain bulk copy.
//
// Compute warp w takes positions w*PW .. w*PW + PW - 1 of every stage for all
// heads at once: in the scores lane (g, p, h) forms half h of the 128-dim dot
// of head g's query with row p (the whole dot when kG = 8), the halves added
// with one shuffle. Lanes of one row read the same K address and lanes of one
// head the same query address (query rows padded to 528 bytes, K swizzled,
// the two halves a bank group apart), so each step reads one 128-byte
// wavefront of each. For G = 4 that is 8 compute warps of 4 positions. Each head keeps an online softmax (max m,
// sum l) over the warp's positions in its PW lanes; then every lane adds
// dims 4l..4l+3 of P.V for all heads, V read once per warp with the
// probabilities shuffled across. Each (warp, head) leaves one partial record
// (m, l, acc); the last CTA of the (sequence, KV head) to finish -- counted
// with an atomic -- merges the S * NW records of each head into the output
// and resets the counter for the next launch.
//
// kRope: q and k arrive un-rotated; the CTA rotates its queries, and the CTA
// whose slice holds pos rotates k and writes k and v to the cache at pos.
// Its staged copy of row pos may predate that write, so the new row's score
// and values are taken from registers instead.
constexpr int kAttnP = 32;       // cache positions per stage
constexpr int kAttnStages = 2;   // ~70 KB a CTA: three CTAs share an SM
constexpr int kAttnRec = 132;    // floats per partial record: m, l, 2 unused, acc[128]
constexpr int kAttnMaxRecs = 128;  // records per head: slices x compute warps
constexpr int kAttnMaxG = 8;
constexpr int kQPitch = kHeadDim + 4;  // floats: 528-byte query rows
constexpr size_t kAttnKStage = (size_t)kAttnP * kHeadDim * sizeof(float);  // 16 KB
constexpr size_t kAttnVStage = kAttnKStage;

struct AttnTail {
  float q[kAttnMaxG][kQPitch];
  uint64_t full[kAttnStages];
  uint64_t empty[kAttnStages];
  uint64_t qready;
  int issued;
  int last;
};
// the stages (1024-byte aligned for the swizzled copies), then the tail;
// +1024 for the alignment of the dynamic shared memory base
constexpr size_t kAttnSmem = kAttnStages * (kAttnKStage + kAttnVStage) + sizeof(AttnTail) + 1024;
// the merge weights reuse the V stages once every copy has landed
static_assert(kAttnMaxRecs * kAttnMaxG * sizeof(float) <= kAttnStages * kAttnVStage,
              "merge weights fit in the V stages");

__host__ __device__ constexpr int attn_kg(int G) { return G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8; }

// lanes per dot product
// (splitting a dot over two lanes doubles the warps but needs registers
// beyond the three-CTAs-per-SM budget; one lane per dot measured faster)
__host__ __device__ constexpr int attn_ds(int) { return 1; }
__host__ __device__ constexpr int attn_nw(int kG) { return kG * attn_ds(kG); }

template <bool kRope, int kG>
__global__ void __launch_bounds__((attn_nw(kG) + 1) * 32, 3)
    attn_decode_kernel(const __grid_constant__ CUtensorMap kmap, DecodeAttn P) {
  extern __shared__ __align__(16) unsigned char attn_smem[];
  constexpr int kDS = attn_ds(kG);         // lanes per dot product
  constexpr int NW = attn_nw(kG);          // compute warps
  constexpr int PW = kAttnP / NW;          // positions per compute warp per stage
  constexpr int kGL = PW * kDS;            // lanes per head in the score layout
  constexpr int kUnits = kHeadDim / 4 / kDS;  // float4 units per lane per dot
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(attn_smem) + 1023) & ~uintptr_t(1023));
  float* kst = reinterpret_cast<float*>(base);
  float* vst = reinterpret_cast<float*>(base + kAttnStages * kAttnKStage);
  AttnTail& S = *reinterpret_cast<AttnTail*>(base + kAttnStages * (kAttnKStage + kAttnVStage));
  const int b = blockIdx.x, kh = blockIdx.y, sidx = blockIdx.z;
  const int G = P.n_head / P.n_kv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();
  // The position and the cache rows before it were written by earlier decode
  // steps, which completed before this step's first kernel started (the step
  // begins with ordinary launches), so they are read before the wait for the
  // previous kernel; q, k, v, the row at pos and every write come after it.
  const long long pos = *P.pos;
  float* out = P.out + ((size_t)b * P.n_head + (size_t)kh * G) * kHeadDim;
  if (pos < 0 || pos >= P.tmax) {
    pdl_wait();
    if (threadIdx.x == 0 && kh == 0 && sidx == 0) atomicExch(P.status, kDevBadPosition);
    if (sidx == 0)
      for (int i = threadIdx.x; i < G * kHeadDim; i += blockDim.x) out[i] = 0.0f;
    return;
  }
  const int T = (int)pos + 1;
  const int cs = (T + P.splits - 1) / P.splits;
  const int t0 = min(sidx * cs, T);
  const int t1 = min(t0 + cs, T);
  const int n = t1 - t0;
  const int nchunks = (n + kAttnP - 1) / kAttnP;
  const int pos_chunk = (kRope && pos >= t0 && pos < t1) ? (int)(pos - t0) / kAttnP : -1;
  const size_t head_row = ((size_t)b * P.n_kv + kh) * P.tmax;  // first cache row of this head
  const float* vbase = P.vcache + head_row * kHeadDim;
  if (threadIdx.x == 0) {
    for (int st = 0; st < kAttnStages; ++st) {
      mbar_init(&S.full[st], 1);
      mbar_init(&S.empty[st], NW);
    }
    mbar_init(&S.qready, NW);
    S.issued = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == NW) {
    // Without kRope the row at pos was appended by the caller, possibly by the
    // launch just before this one: the slice holding it is fetched only after
    // the dependency wait. (With kRope this kernel writes that row itself and
    // takes it from registers, so every stage may be fetched early.)
    if (!kRope) pdl_wait();
    if (lane == 0) {
      int c = 0;
      for (; c < nchunks; ++c) {
        const int st = c % kAttnStages;
        if (c >= kAttnStages && !mbar_wait(&S.empty[st], ((c / kAttnStages) - 1) & 1, P.status))
          break;
        const int rows = min(kAttnP, n - c * kAttnP);
        const int r0 = t0 + c * kAttnP;
        mbar_arrive_expect_tx(&S.full[st], (uint32_t)kAttnKStage + (uint32_t)rows * kHeadDim * 4u);
#pragma unroll
        for (int db = 0; db < kHeadDim / 32; ++db)  // whole boxes; rows past the slice are unused
          tma_load_2d(kst + (size_t)st * kAttnP * kHeadDim + db * kAttnP * 32, &kmap, db * 32,
                      (int)(head_row + r0), &S.full[st]);
        bulk_g2s(vst + (size_t)st * kAttnP * kHeadDim, vbase + (size_t)r0 * kHeadDim,
                 (uint32_t)rows * kHeadDim * 4u, &S.full[st]);
      }
      S.issued = c;
    }
  } else {
    pdl_wait();  // q, k, v come from the previous kernel
    // this CTA's queries, rotated (warp w takes head w)
    if (warp < G) {
      const float* qg = P.q + ((size_t)b * P.n_head + (size_t)kh * G + warp) * kHeadDim;
      float* qw = S.q[warp];
      if (kRope) {
        for (int i = lane; i < 64; i += 32) {
          float c, s;
          rope_cs(pos, i, P.rope_base, c, s);
          const float x0 = qg[i], x1 = qg[i + 64];
          qw[i] = x0 * c - x1 * s;
          qw[i + 64] = x1 * c + x0 * s;
        }
      } else {
        reinterpret_cast<float4*>(qw)[lane] = reinterpret_cast<const float4*>(qg)[lane];
      }
    }
    // the new key and value rows, rotated, for the CTA that holds pos; lane l
    // keeps key dims l, l + 32, l + 64, l + 96 and value dims 4l..4l+3
    float kr0 = 0.f, kr1 = 0.f, kr2 = 0.f, kr3 = 0.f;
    float4 vnew = make_float4(0.f, 0.f, 0.f, 0.f);
    if (pos_chunk >= 0) {
      const float* kn = P.k + ((size_t)b * P.n_kv + kh) * kHeadDim;
      const float* vn = P.v + ((size_t)b * P.n_kv + kh) * kHeadDim;
      float c, s;
      rope_cs(pos, lane, P.rope_base, c, s);
      kr0 = kn[lane] * c - kn[lane + 64] * s;
      kr2 = kn[lane + 64] * c + kn[lane] * s;
      rope_cs(pos, lane + 32, P.rope_base, c, s);
      kr1 = kn[lane + 32] * c - kn[lane + 96] * s;
      kr3 = kn[lane + 96] * c + kn[lane + 32] * s;
      vnew = reinterpret_cast<const float4*>(vn)[lane];
      if (warp == 0) {
        float* kc = P.kcache + (head_row + pos) * kHeadDim;
        kc[lane] = kr0;
        kc[lane + 32] = kr1;
        kc[lane + 64] = kr2;
        kc[lane + 96] = kr3;
        reinterpret_cast<float4*>(P.vcache + (head_row + pos) * kHeadDim)[lane] = vnew;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.qready);
    mbar_wait(&S.qready, 0, P.status);
    const int my_g = lane / kGL;                 // score layout: lane = (g, p, dh)
    const int p = (lane % kGL) / kDS, dh = lane % kDS;
    const int row = warp * PW + p;               // this lane's row in every stage
    // the new key's score for this lane's head, taken from registers: the
    // staged copy of row pos predates the write above
    float s_new = 0.0f;
    if (pos_chunk >= 0) {
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        if (g < G) {
          const float* qg = S.q[g];
          const float d = warp_sum_f(qg[lane] * kr0 + qg[lane + 32] * kr1 + qg[lane + 64] * kr2 +
                                     qg[lane + 96] * kr3);
          if (g == my_g) s_new = d * P.scale;
        }
      }
    }
    // swizzled K addresses of this lane's row: unit u of a box at (u ^ (row & 7))
    const int rsw = row & 7;
    const float* qrow = S.q[my_g < G ? my_g : 0];
    float m = -INFINITY, l = 0.0f;
    float acc[kG][4];
#pragma unroll
    for (int g = 0; g < kG; ++g) acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.0f;
    for (int c = 0; c < nchunks; ++c) {
      const int st = c % kAttnStages;
      if (!mbar_wait(&S.full[st], (c / kAttnStages) & 1, P.status)) break;
      const int rows = min(kAttnP, n - c * kAttnP);
      const int rnew = c == pos_chunk ? (int)(pos - t0) - c * kAttnP : -1;
      const float* kb = kst + (size_t)st * kAttnP * kHeadDim + row * 32;
      float sc = -INFINITY;
      if (my_g < G && row < rows) {
        float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll 8
        for (int i = 0; i < kUnits; ++i) {
          // the second half-lane walks its units 4 ahead, so the two halves
          // of a row never read the same bank group
          const int unit = kDS == 2 ? dh * kUnits + ((i + dh * 4) & (kUnits - 1)) : i;
          const int db = unit >> 3, u = unit & 7;
          const float4 kk = *reinterpret_cast<const float4*>(kb + db * kAttnP * 32 + ((u ^ rsw) << 2));
          const float4 qq = *reinterpret_cast<const float4*>(qrow + unit * 4);
          d0 += qq.x * kk.x;
          d1 += qq.y * kk.y;
          d2 += qq.z * kk.z;
          d3 += qq.w * kk.w;
        }
        sc = (d0 + d1) + (d2 + d3);
      }
      if (kDS == 2) sc += __shfl_xor_sync(0xffffffffu, sc, 1);  // the other half of the dims
      sc *= P.scale;
      if (my_g < G && row < rows && row == rnew) sc = s_new;
      // online softmax of each head over this warp's PW positions (kGL lanes)
      float mx = sc;
#pragma unroll
      for (int o = 1; o < kGL; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mn = fmaxf(m, mx);
      const float corr = mn == -INFINITY ? 1.0f : expf(m - mn);
      const float pv = sc == -INFINITY ? 0.0f : expf(sc - mn);
      float ps = dh == 0 ? pv : 0.0f;
#pragma unroll
      for (int o = 1; o < kGL; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l = l * corr + ps;
      m = mn;
      // P.V: lane holds dims 4*lane..4*lane+3 of every head
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        const float cg = __shfl_sync(0xffffffffu, corr, g * kGL);
        acc[g][0] *= cg;
        acc[g][1] *= cg;
        acc[g][2] *= cg;
        acc[g][3] *= cg;
      }
      const float* vb = vst + (size_t)st * kAttnP * kHeadDim + lane * 4;
#pragma unroll
      for (int q = 0; q < PW; ++q) {
        const int r = warp * PW + q;
        if (r >= rows) break;  // the stage holds only `rows` value rows
        float4 vv;
        if (r == rnew)
          vv = vnew;
        else
          vv = *reinterpret_cast<const float4*>(vb + r * kHeadDim);
#pragma unroll
        for (int g = 0; g < kG; ++g) {
          const float pg = __shfl_sync(0xffffffffu, pv, (g * PW + q) * kDS);
          acc[g][0] += pg * vv.x;
          acc[g][1] += pg * vv.y;
          acc[g][2] += pg * vv.z;
          acc[g][3] += pg * vv.w;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[st]);
    }
    // records [S][NW][G][132]: (m, l) from the head's first lane, acc from all
    float* recs = P.part + (((size_t)b * P.n_kv + kh) * P.splits + sidx) * NW * G * (size_t)kAttnRec +
                  (size_t)warp * G * kAttnRec;
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      if (g < G) {
        float* rec = recs + (size_t)g * kAttnRec;
        if (lane == g * kGL) {
          rec[0] = m;
          rec[1] = l;
        }
        reinterpret_cast<float4*>(rec + 4)[lane] =
            make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // no copy may still be landing when the stages are reused or the CTA
    // exits: wait (bounded) for the last copy issued into each stage
    const int issued = S.issued;
    for (int st = 0; st < kAttnStages && st < issued; ++st) {
      const int c_last = st + ((issued - 1 - st) / kAttnStages) * kAttnStages;
      mbar_wait(&S.full[st], (c_last / kAttnStages) & 1, P.status);
    }
    // one fence: it is cumulative, so it orders every record write of the CTA
    // (ordered before it by the barrier) before the count
    __threadfence();
    const unsigned prev = atomicAdd(&P.counter[(size_t)b * P.n_kv + kh], 1u);
    S.last = prev == (unsigned)P.splits - 1;
    if (S.last) __threadfence();  // and the other CTAs' records before the reads below
  }
  __syncthreads();
  if (!S.last) return;
  // merge: out_g = sum_j acc_j e^(m_j - M) / sum_j l_j e^(m_j - M) over the
  // NR = S*NW records j of head g; warp g takes head g, lanes stride the records
  const int NR = P.splits * NW;
  float* sm_e = vst;  // [NR][G] merge weights
  const float* hrecs = P.part + (((size_t)b * P.n_kv + kh) * P.splits) * NW * G * (size_t)kAttnRec;
  if (warp < G) {
    const int g = warp;
    constexpr int kPer = kAttnMaxRecs / 32;
    float mj[kPer], lj[kPer];
    float M = -INFINITY;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int j = lane + 32 * q;
      const float* r = hrecs + ((size_t)j * G + g) * kAttnRec;
      mj[q] = j < NR ? __ldcg(r) : -INFINITY;
      lj[q] = j < NR ? __ldcg(r + 1) : 0.0f;
      M = fmaxf(M, mj[q]);
    }
    M = warp_max(M);  // finite: the first record holds position 0
    float L = 0.0f;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      mj[q] = mj[q] == -INFINITY ? 0.0f : expf(mj[q] - M);
      L += lj[q] * mj[q];
    }
    L = warp_sum_f(L);
    const float invL = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int j = lane + 32 * q;
      if (j < NR) sm_e[j * G + g] = mj[q] * invL;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * (kHeadDim / 4); i += blockDim.x) {
    const int g = i / (kHeadDim / 4), c4 = i % (kHeadDim / 4);
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 16
    for (int j = 0; j < NR; ++j) {
      const float e = sm_e[j * G + g];
      const float4 a =
          __ldcg(reinterpret_cast<const float4*>(hrecs + ((size_t)j * G + g) * kAttnRec + 4) + c4);
      o.x += a.x * e;
      o.y += a.y * e;
      o.z += a.z * e;
      o.w += a.w * e;
    }
    reinterpret_cast<float4*>(out + (size_t)g * kHeadDim)[c4] = o;
  }
  if (threadIdx.x == 0) P.counter[(size_t)b * P.n_kv + kh] = 0u;
}

}  // namespace

namespace {
bool vec_ok(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Launch with programmatic stream serialisation when pdl is set: every kernel
// here waits (griddepcontrol.wait) before touching global memory, and lets
// its successor start early, so launch latency overlaps the previous kernel.
template <typename... Params, typename... Args>
cudaError_t launch_k(void (*k)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}
}  // namespace

cudaError_t launch_rmsnorm(const float* x, const float* r, float* h, const float* w, float* y,
                           int B, int n, float eps, cudaStream_t s, bool pdl) {
  if (B <= 0) return cudaSuccess;
  const int n4 = n / 4;
  if (n % 4 == 0 && n4 <= kNormVecThreads * kNormMaxVec && vec_ok(x) && (!r || vec_ok(r)) &&
      (!h || vec_ok(h)) && vec_ok(w) && vec_ok(y)) {
    auto x4 = reinterpret_cast<const float4*>(x);
    auto r4 = reinterpret_cast<const float4*>(r);
    auto h4 = reinterpret_cast<float4*>(h);
    auto w4 = reinterpret_cast<const float4*>(w);
    auto y4 = reinterpret_cast<float4*>(y);
    auto k = n4 <= kNormVecThreads       ? rmsnorm_vec_kernel<1>
             : n4 <= 2 * kNormVecThreads ? rmsnorm_vec_kernel<2>
                                         : rmsnorm_vec_kernel<4>;
    return launch_k(k, dim3(B), dim3(kNormVecThreads), 0, s, pdl, x4, r4, h4, w4, y4, n4, eps);
  }
  return launch_k(rmsnorm_kernel, dim3(B), dim3(kNormThreads), 0, s, pdl, x, r, h, w, y, n, eps);
}

cudaError_t launch_swiglu_norm(const float* g, const float* u, const float* w, float* y, int B,
                               int n, float eps, cudaStream_t s, bool pdl) {
  if (B <= 0) return cudaSuccess;
  const int n4 = n / 4;
  if (n % 4 == 0 && n4 <= kNormVecThreads * kNormMaxVec && vec_ok(g) && vec_ok(u) && vec_ok(w) &&
      vec_ok(y)) {
    auto g4 = reinterpret_cast<const float4*>(g);
    auto u4 = reinterpret_cast<const float4*>(u);
    auto w4 = reinterpret_cast<const float4*>(w);
    auto y4 = reinterpret_cast<float4*>(y);
    auto k = n4 <= kNormVecThreads       ? swiglu_norm_vec_kernel<1>
             : n4 <= 2 * kNormVecThreads ? swiglu_norm_vec_kernel<2>
                                         : swiglu_norm_vec_kernel<4>;
    return launch_k(k, dim3(B), dim3(kNormVecThreads), 0, s, pdl, g4, u4, w4, y4, n4, eps);
  }
  return launch_k(swiglu_norm_kernel, dim3(B), dim3(kNormThreads), 0, s, pdl, g, u, w, y, n, eps);
}

cudaError_t launch_rope_append(const DecodeAttn& P, cudaStream_t s, bool pdl) {
  if (P.B <= 0) return cudaSuccess;
  return launch_k(rope_append_kernel, dim3(P.B, P.n_head + P.n_kv), dim3(kHeadDim / 2), 0, s, pdl,
                  P);
}

int attn_splits(int B, int n_head, int n_kv, int tmax, int num_sms) {
  // one resident wave (three CTAs per SM): longer slices stream better than
  // more, shorter ones, whose fixed cost (launch, query, record, count) would
  // be paid per wave; at least four stages of positions per slice (fewer
  // records for the merge; measured faster at B = 1 than two), and at most
  // kAttnMaxRecs records per head for the merge
  const int slots = 3 * num_sms;
  int S = slots / (B * n_kv);
  const int max_s = (tmax + 4 * kAttnP - 1) / (4 * kAttnP);
  if (S > max_s) S = max_s;
  const int max_rec = kAttnMaxRecs / attn_nw(attn_kg(n_head / n_kv));
  if (S > max_rec) S = max_rec;
  return S < 1 ? 1 : S;
}

size_t attn_part_floats(int B, int n_head, int n_kv, int splits) {
  return (size_t)B * n_kv * splits * attn_nw(attn_kg(n_head / n_kv)) * (n_head / n_kv) * kAttnRec;
}

namespace {
template <bool kRope, int kG>
cudaError_t launch_attn_t(const CUtensorMap& map, const DecodeAttn& P, cudaStream_t s, bool pdl) {
  cudaError_t e = ensure_max_smem<attn_decode_kernel<kRope, kG>>();
  if (e != cudaSuccess) return e;
  return launch_k(attn_decode_kernel<kRope, kG>, dim3(P.B, P.n_kv, P.splits),
                  dim3((attn_nw(kG) + 1) * 32), kAttnSmem, s, pdl, map, P);
}
template <int kG>
cudaError_t launch_attn_g(const CUtensorMap& map, const DecodeAttn& P, bool rope, cudaStream_t s,
                          bool pdl) {
  return rope ? launch_attn_t<true, kG>(map, P, s, pdl) : launch_attn_t<false, kG>(map, P, s, pdl);
}
}  // namespace

cudaError_t launch_attention_decode(const DecodeAttn& P, bool rope, cudaStream_t s, bool pdl) {
  if (P.B <= 0) return cudaSuccess;
  const int G = P.n_head / P.n_kv;
  if (P.n_head % P.n_kv || G > kAttnMaxG || P.splits < 1 ||
      P.splits * attn_nw(attn_kg(G)) > kAttnMaxRecs)
    return cudaErrorInvalidValue;
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return cudaErrorNotSupported;
  // the K cache as rows of 128 floats, boxes of 32 rows x 32 floats (128 B),
  // 128-byte swizzle
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)kHeadDim, (cuuint64_t)P.B * P.n_kv * P.tmax};
  const cuuint64_t strides[1] = {(cuuint64_t)kHeadDim * sizeof(float)};
  const cuuint32_t box[2] = {32u, (cuuint32_t)kAttnP};
  const cuuint32_t estr[2] = {1u, 1u};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, P.kcache, dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  switch (attn_kg(G)) {
    case 1: return launch_attn_g<1>(map, P, rope, s, pdl);
    case 2: return launch_attn_g<2>(map, P, rope, s, pdl);
    case 4: return launch_attn_g<4>(map, P, rope, s, pdl);
    default: return launch_attn_g<8>(map, P, rope, s, pdl);
  }
}

}  // namespace ouroq
