// hadamard.cuh -- blockwise Walsh-Hadamard butterflies on a shared-memory row,
// shared by the stand-alone quantiser (quant.cu) and the GEMV prologue
// (gemv.cu).
//
// Reference: cluster/src/infer/hadamard.rs:15-66. The network pairs element i
// with i + h for h = 1, 2, 4, ... (lower index <- a + b, upper <- a - b), the
// same pairs in the same stage order as wht_inplace, so every output is the
// same sequence of IEEE adds and the rotation is bit-identical. Explicit _rn
// intrinsics keep the compiler from contracting anything into an FMA.
//
// A warp rotates spans of 32*E elements (E = max(1, block/32) per lane):
// stages h < E run in registers, stages h >= E exchange with lane ^ (h/E)
// through shuffles.
#pragma once

#include <cuda_runtime.h>

namespace ouroq {

template <int E>
__device__ __forceinline__ void wht_span(float* v, int lane, int block) {
  // in-register stages (element distance h inside a lane; blocks narrower
  // than E lanes-worth stop early)
#pragma unroll
  for (int h = 1; h < E; h <<= 1) {
    if (h >= block) break;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      if ((i & h) == 0) {
        float a = v[i], b = v[i + h];
        v[i] = __fadd_rn(a, b);
        v[i + h] = __fsub_rn(a, b);
      }
    }
  }
  for (int m = 1; m * E < block; m <<= 1) {
    const bool hi = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      float other = __shfl_xor_sync(0xffffffffu, v[i], m);
      v[i] = hi ? __fsub_rn(other, v[i]) : __fadd_rn(v[i], other);
    }
  }
}

// mode 0/1: rotate_fwd (v *= s; WHT; v *= scale); mode 2: rotate_inv (WHT; v *= s*scale).
// Executed by `nwarps` warps; `warp` is this warp's index among them.
template <int E>
__device__ void rotate_row(float* row, const float* signs, int K, int block, float scale, int mode,
                           int warp, int nwarps) {
  const int lane = threadIdx.x & 31;
  const int span = 32 * E;
  for (int base = warp * span; base < K; base += nwarps * span) {
    float v[E];
    const int off = base + lane * E;
    // only spans narrower than 32 elements (block < 32) can overhang K; the
    // overhanging lanes form whole blocks of their own and never mix with
    // valid elements in the shuffles
    const bool valid = off < K;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      float t = valid ? row[off + i] : 0.0f;
      if (valid && mode != 2 && signs) t = __fmul_rn(t, signs[off + i]);
      v[i] = t;
    }
    wht_span<E>(v, lane, block);
    if (valid) {
#pragma unroll
      for (int i = 0; i < E; ++i) {
        float t = v[i];
        if (mode == 2)
          t = __fmul_rn(t, __fmul_rn(signs ? signs[off + i] : 1.0f, scale));
        else
          t = __fmul_rn(t, scale);
        row[off + i] = t;
      }
    }
  }
}

__device__ __forceinline__ void rotate_dispatch(float* row, const float* signs, int K, int block,
                                                float scale, int mode, int warp, int nwarps) {
  switch (block) {
    case 2: case 4: case 8: case 16: case 32:
      rotate_row<1>(row, signs, K, block, scale, mode, warp, nwarps); break;
    case 64: rotate_row<2>(row, signs, K, block, scale, mode, warp, nwarps); break;
    case 128: rotate_row<4>(row, signs, K, block, scale, mode, warp, nwarps); break;
    case 256: rotate_row<8>(row, signs, K, block, scale, mode, warp, nwarps); break;
    case 512: rotate_row<16>(row, signs, K, block, scale, mode, warp, nwarps); break;
    case 1024: rotate_row<32>(row, signs, K, block, scale, mode, warp, nwarps); break;
    default: break;  // rejected on the host
  }
}

// Per-token absmax int8 code of one value (s_x = absmax / 127 computed by the caller):
// q = clamp(rint(v / s), -127, 127); s == 0 -> 0. `rs` = __frcp_rn(s).
// Fast path: t = v * rs differs from the exact quotient by less than 2^-16
// (|v / s| <= 127, two correctly rounded operations), and the correctly
// rounded quotient by less than 2^-15. Both therefore round to the same
// integer unless t lies within 2^-14 of a half-integer; only then (or when rs
// overflowed) is the IEEE division evaluated. The result is always
// rint(__fdiv_rn(v, s)), bit for bit.
__device__ __forceinline__ int quant_code(float v, float s, float rs) {
  if (s == 0.0f) return 0;
  const float t = __fmul_rn(v, rs);
  float r = rintf(t);
  if (!(fabsf(__fsub_rn(t, r)) < 0.5f - 0x1p-14f)) r = rintf(__fdiv_rn(v, s));
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return (int)r;
}

}  // namespace ouroq
