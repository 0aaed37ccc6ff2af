// decode.cu -- the step either side of the ternary path in a decode layer
// (cluster/src/infer/mod.rs:298-336), fused into a few kernels:
//   rmsnorm_kernel        y = rmsnorm(x + r) * w, optionally h = x + r (residual)
//   swiglu_norm_kernel    y = rmsnorm(silu(gate) * up) * w
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
constexpr int kMaxGroup = 8;  // query heads per KV head

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
// grid (B, n_kv, S), block (G + 1) warps, G = n_head / n_kv query heads per
// KV head. The CTA takes cache positions [t0, t1) of the causal range
// [0, pos], cut into S equal slices from the device-side position. Warp G
// (one lane) streams the slice's K and V rows into a ring of shared-memory
// stages with bulk copies; warp g < G serves query head g. Per stage a lane
// scores one position against the head's query (rows read at a rotated
// float4 offset, so the 8 lanes of each shared-memory phase hit distinct
// banks), the warp updates its online softmax (running max m, sum l), and
// then lane l accumulates dims 4l..4l+3 of P.V. The slice's (m, l, acc) goes
// to a partial record; the last CTA of the (sequence, KV head) to finish --
// counted with an atomic -- merges the S records into the output and resets
// the counter for the next launch.
//
// kRope: q and k arrive un-rotated; every CTA rotates its G query heads, and
// the CTA whose slice holds pos rotates k and writes k and v to the cache at
// pos. That CTA's staged copy of row pos may predate the write, so it scores
// the new key from registers and substitutes the new value row in P.V.
constexpr int kAttnP = 32;  // cache positions per stage
constexpr int kAttnStages = 3;
constexpr int kAttnRec = 132;  // floats per partial record: m, l, 2 unused, acc[128]
constexpr int kAttnMaxSplits = 64;

struct AttnShared {
  float ring[kAttnStages][2][kAttnP][kHeadDim];  // K rows then V rows, 32 KB a stage
  float q[kMaxGroup][kHeadDim];
  float p[kMaxGroup][kAttnP];
  uint64_t full[kAttnStages];
  uint64_t empty[kAttnStages];
  int issued;
  int last;
};
// the merge's scratch reuses the ring once every stage is drained
static_assert(kAttnMaxSplits * kMaxGroup * sizeof(float) <= sizeof(float) * kAttnP * kHeadDim,
              "merge weights fit in one stage");

template <bool kRope>
__global__ void __launch_bounds__((kMaxGroup + 1) * 32) attn_decode_kernel(DecodeAttn P) {
  extern __shared__ __align__(128) unsigned char attn_smem[];
  AttnShared& S = *reinterpret_cast<AttnShared*>(attn_smem);
  const int b = blockIdx.x, kh = blockIdx.y, sidx = blockIdx.z;
  const int G = P.n_head / P.n_kv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();
  pdl_wait();
  const long long pos = *P.pos;
  float* out = P.out + ((size_t)b * P.n_head + (size_t)kh * G) * kHeadDim;
  if (pos < 0 || pos >= P.tmax) {
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
  const size_t head_off = ((size_t)b * P.n_kv + kh) * P.tmax * kHeadDim;
  const float* kbase = P.kcache + head_off;
  const float* vbase = P.vcache + head_off;
  if (threadIdx.x == 0) {
    for (int st = 0; st < kAttnStages; ++st) {
      mbar_init(&S.full[st], 1);
      mbar_init(&S.empty[st], G);
    }
    S.issued = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == G) {
    if (lane == 0) {
      int c = 0;
      for (; c < nchunks; ++c) {
        const int st = c % kAttnStages;
        if (c >= kAttnStages && !mbar_wait(&S.empty[st], ((c / kAttnStages) - 1) & 1, P.status))
          break;
        const int rows = min(kAttnP, n - c * kAttnP);
        const uint32_t bytes = (uint32_t)rows * kHeadDim * sizeof(float);
        const size_t at = (size_t)(t0 + c * kAttnP) * kHeadDim;
        mbar_arrive_expect_tx(&S.full[st], 2 * bytes);
        bulk_g2s(&S.ring[st][0][0][0], kbase + at, bytes, &S.full[st]);
        bulk_g2s(&S.ring[st][1][0][0], vbase + at, bytes, &S.full[st]);
      }
      S.issued = c;
    }
  } else {
    const int g = warp;
    const float* qg = P.q + ((size_t)b * P.n_head + (size_t)kh * G + g) * kHeadDim;
    if (kRope) {
      for (int i = lane; i < 64; i += 32) {
        float c, s;
        rope_cs(pos, i, P.rope_base, c, s);
        const float x0 = qg[i], x1 = qg[i + 64];
        S.q[g][i] = x0 * c - x1 * s;
        S.q[g][i + 64] = x1 * c + x0 * s;
      }
    } else {
      reinterpret_cast<float4*>(S.q[g])[lane] = reinterpret_cast<const float4*>(qg)[lane];
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
      if (g == 0) {
        float* kc = P.kcache + head_off + (size_t)pos * kHeadDim;
        kc[lane] = kr0;
        kc[lane + 32] = kr1;
        kc[lane + 64] = kr2;
        kc[lane + 96] = kr3;
        reinterpret_cast<float4*>(P.vcache + head_off + (size_t)pos * kHeadDim)[lane] = vnew;
      }
    }
    __syncwarp();
    // its score, taken here: the staged copy of row pos predates this write
    float s_new = 0.0f;
    if (pos_chunk >= 0) {
      const float d = S.q[g][lane] * kr0 + S.q[g][lane + 32] * kr1 + S.q[g][lane + 64] * kr2 +
                      S.q[g][lane + 96] * kr3;
      s_new = warp_sum_f(d) * P.scale;
    }
    float m = -INFINITY, l = 0.0f;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    const float4* qr = reinterpret_cast<const float4*>(S.q[g]);
    for (int c = 0; c < nchunks; ++c) {
      const int st = c % kAttnStages;
      if (!mbar_wait(&S.full[st], (c / kAttnStages) & 1, P.status)) break;
      const int rows = min(kAttnP, n - c * kAttnP);
      float(*Ks)[kHeadDim] = S.ring[st][0];
      float(*Vs)[kHeadDim] = S.ring[st][1];
      const int rnew = c == pos_chunk ? (int)(pos - t0) - c * kAttnP : -1;
      float sc = -INFINITY;
      if (lane < rows) {
        const float4* kr = reinterpret_cast<const float4*>(Ks[lane]);
        float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll 8
        for (int i = 0; i < kHeadDim / 4; ++i) {
          const int j = (i + lane) & (kHeadDim / 4 - 1);
          const float4 kk = kr[j], qq = qr[j];
          d0 += qq.x * kk.x;
          d1 += qq.y * kk.y;
          d2 += qq.z * kk.z;
          d3 += qq.w * kk.w;
        }
        sc = ((d0 + d1) + (d2 + d3)) * P.scale;
        if (lane == rnew) sc = s_new;
      }
      const float mn = fmaxf(m, warp_max(sc));  // finite: lane 0 holds a position
      const float corr = expf(m - mn);
      const float p = lane < rows ? expf(sc - mn) : 0.0f;
      l = l * corr + warp_sum_f(p);
      m = mn;
      S.p[g][lane] = p;
      __syncwarp();
      a0 *= corr;
      a1 *= corr;
      a2 *= corr;
      a3 *= corr;
      const float4* vcol = reinterpret_cast<const float4*>(&Vs[0][0]) + lane;
#pragma unroll 4
      for (int t = 0; t < rows; ++t) {
        const float pt = S.p[g][t];
        const float4 vv = t == rnew ? vnew : vcol[t * (kHeadDim / 4)];
        a0 += pt * vv.x;
        a1 += pt * vv.y;
        a2 += pt * vv.z;
        a3 += pt * vv.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[st]);
    }
    float* rec = P.part +
                 ((((size_t)b * P.n_kv + kh) * P.splits + sidx) * G + g) * (size_t)kAttnRec;
    if (lane == 0) {
      rec[0] = m;
      rec[1] = l;
    }
    reinterpret_cast<float4*>(rec + 4)[lane] = make_float4(a0, a1, a2, a3);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    // no bulk copy may still be landing when the ring is reused or the CTA
    // exits: wait (bounded) for the last copy issued into each stage
    const int issued = S.issued;
    for (int st = 0; st < kAttnStages && st < issued; ++st) {
      const int c_last = st + ((issued - 1 - st) / kAttnStages) * kAttnStages;
      mbar_wait(&S.full[st], (c_last / kAttnStages) & 1, P.status);
    }
    const unsigned prev = atomicAdd(&P.counter[(size_t)b * P.n_kv + kh], 1u);
    S.last = prev == (unsigned)P.splits - 1;
  }
  __syncthreads();
  if (!S.last) return;
  __threadfence();
  // merge: out_g = sum_s acc_sg e^(m_sg - M_g) / sum_s l_sg e^(m_sg - M_g);
  // warp g reduces head g's S (m, l) pairs, lane s taking slices s, s + 32
  float* sm_e = &S.ring[0][0][0][0];  // [S][G] merge weights
  const float* recs =
      P.part + (((size_t)b * P.n_kv + kh) * P.splits) * G * (size_t)kAttnRec;
  if (warp < G) {
    const int g = warp;
    const bool h0 = lane < P.splits, h1 = lane + 32 < P.splits;
    const float* r0 = recs + ((size_t)lane * G + g) * kAttnRec;
    const float* r1 = recs + ((size_t)(lane + 32) * G + g) * kAttnRec;
    const float m0 = h0 ? __ldcg(r0) : -INFINITY, l0 = h0 ? __ldcg(r0 + 1) : 0.0f;
    const float m1 = h1 ? __ldcg(r1) : -INFINITY, l1 = h1 ? __ldcg(r1 + 1) : 0.0f;
    const float M = warp_max(fmaxf(m0, m1));  // finite: slice 0 is never empty
    const float e0 = m0 == -INFINITY ? 0.0f : expf(m0 - M);
    const float e1 = m1 == -INFINITY ? 0.0f : expf(m1 - M);
    const float L = warp_sum_f(l0 * e0 + l1 * e1);
    const float invL = L > 0.0f ? 1.0f / L : 0.0f;
    if (h0) sm_e[lane * G + g] = e0 * invL;
    if (h1) sm_e[(lane + 32) * G + g] = e1 * invL;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * (kHeadDim / 4); i += blockDim.x) {
    const int g = i / (kHeadDim / 4), c4 = i % (kHeadDim / 4);
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 16
    for (int s = 0; s < P.splits; ++s) {
      const float e = sm_e[s * G + g];
      const float4 a =
          __ldcg(reinterpret_cast<const float4*>(recs + (size_t)(s * G + g) * kAttnRec + 4) + c4);
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

int attn_splits(int B, int n_kv, int tmax, int num_sms) {
  // about one CTA per SM, at least one stage of positions per slice
  int S = (num_sms + B * n_kv - 1) / (B * n_kv);
  const int max_s = (tmax + kAttnP - 1) / kAttnP;
  if (S > max_s) S = max_s;
  if (S > kAttnMaxSplits) S = kAttnMaxSplits;
  return S < 1 ? 1 : S;
}

size_t attn_part_floats(int B, int n_head, int splits) {
  return (size_t)B * n_head * splits * kAttnRec;
}

cudaError_t launch_attention_decode(const DecodeAttn& P, bool rope, cudaStream_t s, bool pdl) {
  if (P.B <= 0) return cudaSuccess;
  if (P.splits < 1 || P.splits > kAttnMaxSplits || P.n_head % P.n_kv ||
      P.n_head / P.n_kv > kMaxGroup)
    return cudaErrorInvalidValue;
  const int G = P.n_head / P.n_kv;
  const dim3 grid(P.B, P.n_kv, P.splits);
  const size_t smem = sizeof(AttnShared);
  cudaError_t e = rope ? ensure_max_smem<attn_decode_kernel<true>>()
                        : ensure_max_smem<attn_decode_kernel<false>>();
  if (e != cudaSuccess) return e;
  return launch_k(rope ? attn_decode_kernel<true> : attn_decode_kernel<false>, grid,
                  dim3((G + 1) * 32), smem, s, pdl, P);
}

}  // namespace ouroq
