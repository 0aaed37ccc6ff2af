// kernels.h -- host-side launch interface between the C ABI (api.cpp) and the
// CUDA kernels. Plain structs and pointers; no torch types anywhere.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace ouroq {

// Device weight layouts (produced by the repack kernels at upload time).
//
// kTern2: one 32-bit word per 16 weights of a row (k = 16t .. 16t+15); in
//   word t, byte b, bits (2j, 2j+1) hold code c = w + 1 of k = 16t + 4j + b.
//   Masking a word with 0x03030303 << 2j therefore yields four bytes whose
//   values are c * 4^j for four consecutive k, ready for dp4a against four
//   consecutive int8 activations.
// kSign1: one 32-bit word per 32 weights (k = 32t .. 32t+31); in word t,
//   byte b, bit j holds the sign bit of k = 32t + 4j + b. Group scales stay
//   fp16, stored [M][gpad] with gpad = K/128 rounded up to a multiple of 16
//   (zero padding) so every 16-group slice of a row starts 16-byte aligned.
enum DevFormat : int { kTern2 = 1, kSign1 = 2 };

// One matrix-times-activations job of a (possibly grouped) GEMV launch.
struct GemvJob {
  const uint8_t* w;         // device layout, [M][row_bytes]
  const uint16_t* scales;   // kSign1: fp16 [M][gpad] (rows padded to 16 groups); else null
  const int8_t* q;          // [B][K] int8 activations (16-byte aligned)
  const float* s_x;         // [B] per-token scales
  float* y;                 // [B][ldy] fp32 outputs, row b at y + b*ldy
  int32_t* acc;             // optional debug: tern [B][M]; sign [B][M][K/128]
  float w_scale;            // kTern2 per-tensor scale
  int M, K, ldy;
  int gpad;                 // kSign1: scale row pitch in fp16 elements (multiple of 16)
  int tile_begin;           // first global tile index of this job
};

constexpr int kMaxGemvJobs = 8;

struct GemvLaunch {
  GemvJob jobs[kMaxGemvJobs];
  int njobs;
  int ntiles;               // total 32-row tiles over all jobs
  int B;                    // tokens (same for all jobs)
  int fmt;                  // DevFormat (same for all jobs)
  unsigned* status;         // device status word
};

// One activation-quantisation job (fp32 [B][K] -> int8 [B][K] + s_x[B]).
struct QuantJob {
  const float* x;
  const float* signs;       // nullable (all +1)
  int8_t* q;
  float* s_x;
  float* x_rot;             // nullable: rotated fp32 copy (debug / rotate API)
  int K;
  int had_block;            // 0 = no rotation
  float had_scale;          // 1/sqrt(had_block), computed on the host
};

constexpr int kMaxQuantJobs = 8;

struct QuantLaunch {
  QuantJob jobs[kMaxQuantJobs];
  int njobs;
  int B;
};

// Launchers. All return cudaError_t from the launch itself.
cudaError_t launch_quantize(const QuantLaunch& L, cudaStream_t s, bool pdl);
cudaError_t launch_rotate(const float* x, float* out, const float* signs, int B, int K,
                          int block, float scale, int inverse, cudaStream_t s);
cudaError_t launch_gemv(const GemvLaunch& L, int num_sms, cudaStream_t s, bool pdl);
size_t gemv_smem_bytes(int fmt, int B, int maxK);
cudaError_t launch_repack_tern2(const uint8_t* canon, uint8_t* dev, int M, int K, cudaStream_t s);
cudaError_t launch_repack_sign1(const uint8_t* canon, uint8_t* dev, int M, int K, cudaStream_t s);

// Limits of the small-batch GEMV path.
constexpr int kGemvMaxB = 8;
constexpr size_t kGemvMaxXBytes = 64 * 1024;  // B*K int8 resident in shared memory

}  // namespace ouroq
