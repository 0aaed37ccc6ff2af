// kernels.h -- host-side launch interface between the C ABI (api.cpp) and the
// CUDA kernels. Plain structs and pointers; no torch types anywhere.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace ouroq {

// Device weight layouts (produced by the repack kernels at upload time).
//
// Rows are grouped in tiles of kTileRows = 32. A row is cut into 16-byte
// chunks (64 ternary or 128 sign weights each), and a tile is stored
// chunk-major: byte offset of (tile t, chunk c, row r) =
//   (t * C + c) * 512 + r * 16,     C = row_bytes / 16.
// Any run of chunks of a tile is therefore one contiguous block (one large
// bulk copy per pipeline stage), and 32 lanes reading chunk c of rows 0..31
// touch 512 contiguous bytes of shared memory (no bank conflicts).
// Rows past M in the last tile are zero.
//
// Within each 32-bit word the bits are permuted so that one mask exposes four
// consecutive k in the four byte lanes:
// kTern2: word t of a row covers k = 16t .. 16t+15; byte b, bits (2j, 2j+1)
//   hold code c = w + 1 of k = 16t + 4j + b. Masking with 0x03030303 << 2j
//   yields four bytes c * 4^j for k = 16t+4j .. 16t+4j+3, ready for dp4a.
// kSign1: word t covers k = 32t .. 32t+31; byte b, bit j holds the sign bit
//   of k = 32t + 4j + b. fp16 group scales are tiled the same way:
//   [tile][group][32 rows].
enum DevFormat : int { kTern2 = 1, kSign1 = 2, kPtq1 = 3, kTq1 = 4 };

// Error codes written to the status word by a kernel that gave up waiting.
enum : unsigned {
  kDevOk = 0,
  kDevWaitTimeout = 1,  // an mbarrier wait ran past its iteration limit
  kDevBadTile = 2,      // a tile index outside the job table (never expected)
  kDevPeerTimeout = 3,  // a sharded gather waited too long for a peer's rows
  kDevBadPosition = 4,  // a decode position outside the KV cache (nothing written)
};

constexpr int kTileRows = 32;

// One matrix-times-activations job of a (possibly grouped) GEMV launch.
struct GemvJob {
  const uint8_t* w;         // tiled device layout
  const uint16_t* scales;   // kSign1: tiled fp16 group scales; else null
  const int8_t* q;          // [B][K] int8 activations (16-byte aligned), unfused mode
  const float* s_x;         // [B] per-token scales, unfused mode
  const float* xf;          // [B][K] fp32 activations (16-byte aligned), fused mode
  const float* signs;       // fused mode: rotation signs [K] or null (all +1)
  float* y;                 // [B][ldy] fp32 outputs, row b at y + b*ldy
  int32_t* acc;             // optional debug: tern [B][M]; sign [B][M][K/128]
  float w_scale;            // kTern2 per-tensor scale
  float had_scale;          // fused mode: 1/sqrt(had_block)
  int M, K, ldy;
  int had_block;            // fused mode: Hadamard block, 0 = no rotation
  int tile_begin;           // first global tile index of this job
};

constexpr int kMaxGemvJobs = 8;
constexpr int kMaxGemvCtas = 160;  // >= SM count of the device (148 on B200)
constexpr int kMaxGemvStages = 13;

// Fused RMSNorm ahead of a fused GEMV (infer/mod.rs:303-333): every job of the
// launch reads the same K-wide row per token, v = x + r (mode 0, r nullable) or
// v = silu(x) * r (mode 1), a = v * inv * w with inv = 1 / sqrt(mean(v^2) + eps),
// quantised once per CTA; h (mode 0, nullable) receives v (written by CTA 0).
// Disabled while w is null.
struct NormSpec {
  const float* x;
  const float* r;
  const float* w;
  float* h;
  float eps;
  int mode;
  int K;
};
// Rows the fused norm keeps entirely in registers: B * K / 128 units at most.
constexpr int kNormFusedMaxUnits = 90;

struct GemvLaunch {
  GemvJob jobs[kMaxGemvJobs];
  NormSpec norm;
  int njobs;
  int ntiles;               // total 32-row tiles over all jobs
  int B;                    // tokens (same for all jobs)
  int fmt;                  // DevFormat (same for all jobs)
  int fused;                // 1: jobs carry fp32 activations and quantise in the prologue
  int stages;               // weight ring depth (2..kMaxGemvStages), sized to shared memory
  int xcap;                 // bytes of int8 activations one CTA keeps resident (its jobs)
  int gcap;                 // per-group activation sums one CTA keeps resident (ints)
  int defer;                // ternary: > 0 = tile slots for the end-of-CTA reduction
  unsigned* status;         // device status word
  // L2 prefetch of the weights the next launch reads (gemv_stream_kernel):
  // npf ranges, 16-byte aligned, multiples of 16 bytes, split evenly over the
  // CTAs and issued after each CTA's own copies; nothing waits for them.
  const uint8_t* pf_ptr[kMaxGemvJobs];
  uint32_t pf_bytes[kMaxGemvJobs];
  int npf;
  int cluster;              // gemv_stream_kernel: CTAs per cluster sharing the quantisation
  // CTA c owns tiles [cta_tile[c], cta_tile[c+1]): ranges balanced by weight
  // bytes on the host, so the kernel does no 64-bit division at start-up.
  uint16_t cta_tile[kMaxGemvCtas + 1];
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
// Fills L.ntiles, tile_begin, the CTA ranges, xcap/gcap and stages; returns
// false when the activations of one CTA's jobs cannot be kept in shared memory.
bool gemv_prepare(GemvLaunch& L, int num_sms, int smem_optin, int* grid, size_t* smem);
cudaError_t launch_gemv(GemvLaunch& L, int num_sms, int smem_optin, cudaStream_t s, bool pdl);
// Contiguous tile ranges per CTA (L.cta_tile[0..grid]) that minimise the
// heaviest CTA's load: its weight chunks, plus unit_q / 4 chunks x B per
// 128-value unit of each distinct input it quantises (0: weights only); needs
// L.ntiles and the jobs' tile_begin.
void balance_tiles(GemvLaunch& L, int grid, int per_chunk, int unit_q);
// The streaming decode GEMV (gemv_stream.cu): fused ternary launches of one or
// two tokens without rotation or norm. prepare returns false when the launch
// is not of that kind (the caller then uses launch_gemv).
bool gemv_stream_prepare(GemvLaunch& L, int num_sms, int* grid, size_t* smem);
cudaError_t launch_gemv_stream(GemvLaunch& L, int grid, size_t smem, cudaStream_t s, bool pdl);
size_t tiled_weight_bytes(int fmt, int M, int K);
size_t tiled_scale_bytes(int M, int K);
cudaError_t launch_repack(int fmt, const uint8_t* canon, uint8_t* dev, int M, int K, cudaStream_t s);
cudaError_t launch_repack_scales(const uint16_t* canon, uint16_t* dev, int M, int K,
                                 cudaStream_t s);

// One tensor-core GEMM launch (ternary): 128 weight rows per CTA x N tokens.
struct TcLaunch {
  const uint8_t* w;   // tiled device layout (kTern2 or kSign1)
  const uint16_t* scales;  // kSign1: tiled fp16 group scales; else null
  float* y;           // [tokens][ldy]
  int32_t* acc;       // optional debug: kTern2 [tokens][M]; kSign1 [tokens][M][K/128]
  const float* s_x;   // [tokens]
  float w_scale;
  int M, K, ldy;
  int tok0;           // first token of this launch
  int N;              // tokens per CTA tile (multiple of 16, 16..256), filled by the launcher
  int nvalid;         // valid tokens from tok0 (all token tiles)
  int stages;         // filled by the launcher
  int ksplit;         // CTAs of a cluster splitting K (1, 2 or 4), filled by the launcher
  unsigned* status;
};

// A grouped tensor-core launch: up to kMaxTcJobs ternary products
// y_j = W_j . q_j with the same batch, in ONE launch (the projections of a
// layer). The grid's x covers the 128-row tiles of every job in order.
constexpr int kMaxTcJobs = 8;
struct TcJob {
  const uint8_t* w;
  float* y;
  int32_t* acc;       // optional debug [tokens][M]
  const float* s_x;   // [tokens]
  float w_scale;
  int M, K, ldy;
};
struct TcGroup {
  CUtensorMap maps[kMaxTcJobs];    // each job's activations [Btot][K] int8
  TcJob jobs[kMaxTcJobs];
  int tile_begin[kMaxTcJobs + 1];  // job j: 128-row tiles [tile_begin[j], tile_begin[j + 1])
  int njobs;
};

bool gemm_tc_supported(int fmt, int M, int K, int B);
size_t gemm_tc_smem_bytes(int N, int stages);
// q: int8 activations [Btot][K] (16-byte aligned rows). One launch; the grid
// covers (128-row tiles) x (token tiles) x (parts of K), sizes chosen by the
// launcher.
// pdl: programmatic dependent launch (the weight copies and the set-up
// overlap the previous kernel; the activations are read after it).
cudaError_t launch_gemm_tc(const TcLaunch& L, const int8_t* q, int Btot, int smem_optin,
                           int num_sms, cudaStream_t s, bool pdl);
// n jobs (same K % 128 == 0 rule, ternary) in one launch: q[j] int8 [Btot][K_j];
// L carries the batch (nvalid, tok0) and the status word.
cudaError_t launch_gemm_tc_group(const TcLaunch& L, const TcJob* jobs, const int8_t* const* q, int n,
                                 int Btot, int smem_optin, int num_sms, cudaStream_t s, bool pdl);
// Sign weights (kSign1) on the tensor cores: one group accumulator per 128 k,
// the fp32 fold in ascending group order. The grid covers (128-row tiles) x
// (token tiles of 16 or 32) x (parts of the groups, a cluster chaining the
// fold), sizes chosen by the launcher.
bool gemm_sign_tc_supported(int M, int K, int B);
cudaError_t launch_gemm_sign_tc(const TcLaunch& L, const int8_t* q, int Btot, int smem_optin,
                                int num_sms, cudaStream_t s, bool pdl);

// The reference's own shard formats (PTQ1_0 "Tl1", TQ1_0), stored on the device
// exactly as in the shard (row-major, no repack): fp32 x [B][K] -> y [B][ldy].
struct RefLaunch {
  int fmt;            // kPtq1 or kTq1
  const uint8_t* w;   // payload, rows of K/128*28 (kPtq1) or K/256*54 (kTq1) bytes
  const float* x;
  float* y;
  int M, K, B, ldy;
};
size_t tl1_smem_bytes(int K, int R);
int tl1_rows_per_cta(int K, int M, int num_sms);
size_t tq1_smem_bytes(int K);
cudaError_t launch_refmt_matvec(const RefLaunch& P, int num_sms, cudaStream_t s);
// PTQ1_0 x K columns (x [B][K] -> y [B][ldy], B = columns) in matmul_tl1's
// K-column order rather than the per-column matvec order.
cudaError_t launch_tl1_columns(const RefLaunch& P, cudaStream_t s);

// 16-bit weights (F16 / BF16 shards, the tied lm_head): fp32 x [B][K] ->
// y [B][ldy] in the reference's per-row order; with tokens set, also the
// finite argmax of each sequence's logits (y may then be null).
struct HeadLaunch {
  const uint16_t* w;          // [M][K] as stored in the shard
  const float* x;
  float* y;                   // optional when tokens is set
  int M, K, B, ldy;
  int bf16;                   // 0: f16, 1: bf16
  int vec;                    // K % 8 == 0, w and x 16-byte aligned
  int num_sms;
  unsigned long long* key;    // [B] argmax keys, zero between launches
  unsigned* counter;          // CTAs finished, zero between launches
  long long* tokens;          // [B] or null (no argmax)
};
cudaError_t launch_head(const HeadLaunch& L, cudaStream_t s, bool pdl);

// Limits of the small-batch GEMV path.
constexpr int kGemvMaxB = 8;
// Largest batch of the stream GEMV (gemv_stream_kernel, fused quantisation).
constexpr int kStreamMaxB = 8;
// Above this batch the fp32-activation entry points quantise once in a separate
// launch instead of in every GEMV CTA's prologue (which repeats it per CTA).
constexpr int kFusedMaxB = 2;
constexpr size_t kGemvMaxXBytes = 64 * 1024;  // B*K int8 resident in shared memory

// Row-sharded matmul, peer-store transport. Each rank's landing buffer (one
// cudaMalloc, opened by every peer through CUDA IPC) holds two parities of
// [G][B][R] 64-bit words, each (step << 32 | fp32 bits).
constexpr int kShardMaxRanks = 8;
constexpr int kShardGatherCtas = 64;
struct ShardGather {
  const float* staging;                       // this rank's rows [B][R]
  unsigned long long* peers[kShardMaxRanks];  // landing buffer of every rank (own included)
  float* y;                                   // [B][G*R]
  unsigned* step;                             // this rank's step counter (device, starts at 0)
  unsigned* done;                             // last-CTA counter (device, starts at 0)
  unsigned* status;
  int rank, G, B, R;
  unsigned long long timeout_ns;
};
cudaError_t launch_shard_gather(const ShardGather& P, cudaStream_t s, bool pdl);

// Row-sharded matmul, NCCL transport: gather [G][B][R] -> y [B][G*R].
cudaError_t launch_shard_interleave(const float* gather, float* y, int B, int R, int G,
                                    cudaStream_t s);

// The decode step around the ternary path (decode.cu). Head dim 128; up to 8
// query heads per KV head. KV cache [B][n_kv][tmax][128] fp32 per layer.
struct DecodeAttn {
  float* q;                  // [B][n_head][128] (rotated in place by rope_append)
  const float* k;            // [B][n_kv][128] new keys (before RoPE)
  const float* v;            // [B][n_kv][128] new values
  float* kcache;             // [B][n_kv][tmax][128]
  float* vcache;
  const long long* pos;      // device: the position being decoded
  float* out;                // [B][n_head][128]
  float* part;               // [B][n_kv][splits][warps][group][132] partial records
  unsigned* counter;         // [B][n_kv] slices finished (zero between launches)
  unsigned* status;
  int B, n_head, n_kv, tmax, splits;
  float rope_base, scale;
};
cudaError_t launch_rmsnorm(const float* x, const float* r, float* h, const float* w, float* y,
                           int B, int n, float eps, cudaStream_t s, bool pdl);
cudaError_t launch_swiglu_norm(const float* g, const float* u, const float* w, float* y, int B,
                               int n, float eps, cudaStream_t s, bool pdl);
cudaError_t launch_rope_append(const DecodeAttn& P, cudaStream_t s, bool pdl);
int attn_splits(int B, int n_head, int n_kv, int tmax, int num_sms);
size_t attn_part_floats(int B, int n_head, int n_kv, int splits);
// rope: q, k un-rotated; k and v appended to the cache at pos in the same launch
cudaError_t launch_attention_decode(const DecodeAttn& P, bool rope, cudaStream_t s, bool pdl);

// Fixed scratch of ouroq_gemm_f32act_noalloc (one copy per device): int8
// codes for up to 4 MiB of B*K, then fp32 scales for up to 4096 tokens.
constexpr size_t kNoAllocQBytes = 4u << 20;
constexpr int kNoAllocMaxTokens = 4096;
constexpr size_t kNoAllocScratchBytes = kNoAllocQBytes + (size_t)kNoAllocMaxTokens * sizeof(float);
// Device address of that scratch on the current device (first use per device
// loads this library's kernels there).
cudaError_t noalloc_scratch_address(void** ptr);

}  // namespace ouroq
