/*
 * ouroq.h -- C ABI of the B200 (sm_100a) quantized-weight matmul path.
 *
 * This is the drop-in boundary for OuroborOS's packed-weight matmul operators.
 * The reference calls them from Rust (crate ouro-cluster, cluster/src/infer/):
 *
 *   ops::matvec_q(payload, kind, out_len, in_len, x) -> Vec<f32>   ops.rs:76-84
 *   ops::matmul_q(payload, kind, out_len, in_len, x[k][in], k)     ops.rs:219-230
 *       -> y[k][out] ("column-major": y[c*out_len + r], ops.rs:158-161)
 *   hadamard::rotate_fwd(x, signs, block) / rotate_inv             hadamard.rs:41-66
 *   Stage::wm / wmat_batched (per named tensor, width check)       infer/mod.rs:138-167
 *
 * Plain C types only (no CUDA or torch types): streams are passed as void*
 * holding a cudaStream_t, device buffers as plain pointers. Every function
 * returns an ouroq_status; nothing throws or aborts across the ABI. A context
 * is bound to one device and is not thread-safe: callers serialise, as the
 * reference serialises calls through its per-process stage Mutex
 * (agent/src/stage.rs:11-14).
 *
 * Formats accepted by ouroq_weight_upload (host layouts, row-major [M][*]):
 *   OUROQ_FMT_TERNARY2   codes c = w + 1 in {0,1,2}, 4 per byte, element k of a
 *                        row in byte k/4 bits 2*(k%4); one fp32 scale per tensor.
 *   OUROQ_FMT_SIGN1G128  bit = 1 -> +1, bit = 0 -> -1, 8 per byte, element k in
 *                        byte k/8 bit k%8; fp16 scales [M][K/128].
 * Activation arithmetic for both: per-token absmax int8 (s_x = absmax/127,
 * q = clamp(rint(x/s_x), -127, 127)), int32 accumulation, fp32 epilogue
 *   ternary: y = ((float)acc * w_scale) * s_x
 *   sign:    y = (sum over groups g ascending of (float)acc_g * scale_g) * s_x
 */
#ifndef OUROQ_H
#define OUROQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OUROQ_ABI_VERSION 1

typedef enum {
  OUROQ_OK = 0,
  OUROQ_ERR_BAD_SHAPE = 1,    /* dimensions not supported (reference: assert!/bail!) */
  OUROQ_ERR_BAD_ALIGN = 2,    /* pointer not 16-byte aligned where required */
  OUROQ_ERR_CUDA = 3,         /* CUDA runtime error; see ouroq_last_error */
  OUROQ_ERR_NCCL = 4,         /* NCCL error in the sharded path */
  OUROQ_ERR_TIMEOUT = 5,      /* a bounded device or collective wait expired */
  OUROQ_ERR_UNSUPPORTED = 6,  /* format / batch combination not implemented */
  OUROQ_ERR_BAD_ARG = 7,      /* null handle or pointer, bad enum value */
  OUROQ_ERR_NO_DEVICE = 8,    /* no CUDA device / not sm_100 */
  OUROQ_ERR_OOM = 9           /* device allocation failed */
} ouroq_status;

typedef enum {
  OUROQ_FMT_TERNARY2 = 1,
  OUROQ_FMT_SIGN1G128 = 2,
  /* The reference's own shard formats, uploaded byte for byte (no scales
   * argument, w_scale ignored) and used with fp32 activations only
   * (ouroq_gemm_f32act, ouroq_matvec_q, ouroq_matmul_q, ouroq_gemm_sharded):
   *   PTQ1_0 ("Tl1", QuantKind::Tl1, dequant.rs:123-171): per 128 weights
   *     28 bytes qs[24] | qh[2] | f16 d; K multiple of 128. Results are
   *     bit-identical to matvec_tl1's x86 order (ops.rs:499-584) for one
   *     token (ouroq_matvec_q, B = 1), and to matmul_tl1's x86 K-column order
   *     (ops.rs:381-481) for B > 1 and for every ouroq_matmul_q call.
   *   TQ1_0 (QuantKind::Tq1_0, dequant.rs:50-105): per 256 weights 54 bytes
   *     qs[48] | qh[4] | f16 d; K multiple of 256. Results are bit-identical
   *     to matvec_qblock (dequantise, then dot in element order, ops.rs:53-60). */
  OUROQ_FMT_PTQ1_0 = 3,
  OUROQ_FMT_TQ1_0 = 4,
  /* 16-bit weights as stored in the shard, rows of K little-endian values,
   * any K >= 1: F16 (QuantKind::F16, ops.rs:131-153) and BF16
   * (QuantKind::Bf16, ops.rs:600-620). Each row is one fp32 chain in element
   * order with every product and sum rounded, bit-identical to the
   * reference (a NaN keeps its position, not necessarily its payload). */
  OUROQ_FMT_F16 = 5,
  OUROQ_FMT_BF16 = 6
} ouroq_format;

typedef struct ouroq_ctx ouroq_ctx;
typedef struct ouroq_weight ouroq_weight;

/* ---- library / context ---- */
int ouroq_abi_version(void);
const char *ouroq_status_string(ouroq_status s);

/* Create a context on CUDA device `device` (sm_100 required). */
ouroq_status ouroq_ctx_create(int device, ouroq_ctx **out);
ouroq_status ouroq_ctx_destroy(ouroq_ctx *ctx);
/* Text of the last error on this context ("" if none). Valid until the next call. */
const char *ouroq_last_error(const ouroq_ctx *ctx);
/* Read and clear the device status word that kernels write on a fault they
 * refuse to act on (synchronises the device). OUROQ_ERR_TIMEOUT if a bounded
 * wait gave up, OUROQ_ERR_BAD_SHAPE if a decode position lay outside the KV
 * cache. */
ouroq_status ouroq_check_device(ouroq_ctx *ctx);
/* Where a buffer lives. Host-buffer entry points (ouroq_matvec_q,
 * ouroq_matmul_q, ouroq_rotate_fwd/inv) and device-buffer entry points
 * (ouroq_gemm*, ouroq_quantize_act, the decode ops) are separate; a caller
 * holding a pointer of unknown origin asks here which one applies. */
typedef enum {
  OUROQ_PTR_HOST = 0,    /* pageable or pinned host memory */
  OUROQ_PTR_DEVICE = 1,  /* device memory of some GPU */
  OUROQ_PTR_MANAGED = 2  /* unified (managed) memory */
} ouroq_ptr_kind_t;
ouroq_status ouroq_ptr_kind(const void *p, int *kind, int *device);
/* Number of kernels this context has launched (for bench accounting). */
uint64_t ouroq_launch_count(const ouroq_ctx *ctx);
/* 1 = launch GEMV kernels with programmatic dependent launch (default), 0 = off. */
ouroq_status ouroq_set_pdl(ouroq_ctx *ctx, int enable);
/* New (the reference's matvec_q streams each payload when it is called):
 * the weights the call after the next GEMV launch will read. That launch
 * prefetches them into L2 once its own weight copies are issued, so the
 * next call streams from L2 instead of waiting on HBM at its start. A
 * caller that knows its next projection (the next group of a layer, the
 * next layer) sets it before each call; the list is consumed by the next
 * GEMV launch (at most 8 ranges, weights and scales); n = 0 clears it. A
 * hint: results never depend on it. */
ouroq_status ouroq_set_prefetch(ouroq_ctx *ctx, int n, const ouroq_weight *const *w);

/* ---- weights ----
 * Upload a packed matrix (HOST pointers, canonical layout above) to device
 * memory owned by the context, converting it to the device layout.
 * Replaces the per-call borrowed payload of matvec_q (ops.rs:76) and the
 * Weight{payload, kind, in_len, out_len} record (infer/mod.rs:95-100):
 * M = out_len, K = in_len. K must be a multiple of 128.
 *   TERNARY2:  scales = NULL, w_scale = per-tensor scale.
 *   SIGN1G128: scales = uint16_t fp16 [M][K/128], w_scale ignored. */
ouroq_status ouroq_weight_upload(ouroq_ctx *ctx, ouroq_format fmt, const void *packed, int M, int K,
                                 const void *scales, float w_scale, ouroq_weight **out);
/* Same, from DEVICE pointers holding the canonical layout. */
ouroq_status ouroq_weight_upload_device(ouroq_ctx *ctx, ouroq_format fmt, const void *packed_dev,
                                        int M, int K, const void *scales_dev, float w_scale,
                                        ouroq_weight **out);
ouroq_status ouroq_weight_free(ouroq_ctx *ctx, ouroq_weight *w);
ouroq_status ouroq_weight_info(const ouroq_weight *w, int *fmt, int *M, int *K,
                               size_t *device_bytes);

/* ---- stream-ordered device API (all buffers DEVICE pointers) ---- */

/* K1: per-token absmax int8 quantisation of x [B][K], optionally preceded by
 * the blockwise rotation of hadamard::rotate_fwd (hadamard.rs:41-53) with
 * `hadamard_block` (power of two 2..1024 dividing K; 0 = no rotation) and
 * `signs` (fp32 +-1 [K], NULL = all +1). q [B][K] int8, s_x [B] fp32.
 * x, q: 16-byte aligned; K multiple of 4 (of 32 when hadamard_block < 32). */
ouroq_status ouroq_quantize_act(ouroq_ctx *ctx, const float *x, int B, int K, const float *signs,
                                int hadamard_block, int8_t *q, float *s_x, void *stream);

/* Grouped K1: quantise n (<= 8) independent activation sets in ONE launch.
 * Set i: x[i] [B][K[i]] -> q[i] [B][K[i]], s_x[i] [B]; optional rotation per
 * set (signs[i] nullable, blocks[i] = 0 for none). signs / blocks may be NULL. */
ouroq_status ouroq_quantize_group(ouroq_ctx *ctx, int n, const float *const *x, const int *K,
                                  const float *const *signs, const int *blocks, int B,
                                  int8_t *const *q, float *const *s_x, void *stream);

/* rotate_fwd (inverse = 0) / rotate_inv (inverse = 1) of hadamard.rs:41-66 on
 * B rows of K floats; out may equal x. */
ouroq_status ouroq_rotate(ouroq_ctx *ctx, const float *x, float *out, int B, int K,
                          const float *signs, int block, int inverse, void *stream);

/* y [B][M] = W . q for pre-quantised activations q [B][K] (16-byte aligned)
 * and scales s_x [B]. acc_debug (nullable) receives the exact int32
 * accumulators: TERNARY2 [B][M], SIGN1G128 [B][M][K/128]. */
ouroq_status ouroq_gemm(ouroq_ctx *ctx, const ouroq_weight *w, const int8_t *q, const float *s_x,
                        int B, float *y, int32_t *acc_debug, void *stream);

/* Grouped product: n (<= 8) independent products y_i = W_i . q_i, all weights
 * of one format. Up to 8 tokens one GEMV launch; from 9 tokens TERNARY2
 * weights run as ONE tensor-core launch over every matrix's row tiles (the
 * projections of a layer), SIGN1G128 weights one tensor-core launch each.
 * Used for the projections of a layer. */
ouroq_status ouroq_gemm_group(ouroq_ctx *ctx, int n, const ouroq_weight *const *w,
                              const int8_t *const *q, const float *const *s_x, int B,
                              float *const *y, void *stream);

/* Grouped GEMV with the quantisation fused in: n (<= 8) products
 * y_i = W_i . quant(rotate(x_i)) in ONE launch, x_i fp32 [B][K_i] (16-byte
 * aligned). Per entry optional rotation: signs[i] (nullable) and blocks[i]
 * (0 = none, else 32, 64 or 128, the same for every entry); both arrays may be
 * NULL. Beyond 8 tokens the distinct inputs are quantised in one launch and the
 * products run as in ouroq_gemm_group. OUROQ_ERR_UNSUPPORTED when B <= 8 and
 * the activations of the matrices
 * one CTA covers do not fit in shared memory. */
ouroq_status ouroq_gemm_group_f32act(ouroq_ctx *ctx, int n, const ouroq_weight *const *w,
                                     const float *const *x, int B, const float *const *signs,
                                     const int *blocks, float *const *y, void *stream);

/* fp32 activations in, fp32 outputs out: quantise (with optional rotation)
 * and multiply. Mirrors matvec_q / matmul_q's "f32 x in, f32 y out" contract
 * on device buffers. Small batches run as one fused launch; otherwise the
 * activations are quantised into context-owned scratch first. */
ouroq_status ouroq_gemm_f32act(ouroq_ctx *ctx, const ouroq_weight *w, const float *x, int B,
                               const float *signs, int hadamard_block, float *y, void *stream);

/* ouroq_gemm_f32act for callers that must not allocate device memory while
 * they run. This entry point has no counterpart in the reference.
 *
 * Who needs it: ouroq_gemm_f32act quantises batches it cannot fuse (B > 2)
 * into a context-owned buffer, and grows that buffer with cudaMalloc, freeing
 * the old one, the first time a larger batch arrives. A serving loop that
 * reserved the GPU's memory up front for weights and caches cannot take that
 * (the late cudaMalloc can fail), nor can one on a latency budget (cudaFree
 * waits for the whole device). This variant allocates nothing: it uses a
 * fixed scratch area compiled into the library, one per device.
 *
 * Limits (TERNARY2 / SIGN1G128): B <= 4096 and B * K <= 4 MiB (4194304);
 * larger batches return OUROQ_ERR_BAD_SHAPE with nothing launched; split them
 * into calls that fit. The reference formats (PTQ1_0, TQ1_0, F16, BF16) are
 * not quantised and take any batch, but PTQ1_0 / TQ1_0 with a rotation
 * (hadamard_block != 0) return OUROQ_ERR_UNSUPPORTED: rotate the activations
 * first (ouroq_rotate), then call this.
 * The first call on a device does one-time set-up (loads this library's
 * kernels on that device and looks up the scratch address); make it before
 * any stream capture. All calls on one device share the one scratch area,
 * whatever context or stream they use: two calls in flight at the same time
 * overwrite each other's activations. Order them on one stream, or wait for
 * one to finish before starting the next. Results are identical to
 * ouroq_gemm_f32act's. */
ouroq_status ouroq_gemm_f32act_noalloc(ouroq_ctx *ctx, const ouroq_weight *w, const float *x,
                                       int B, const float *signs, int hadamard_block, float *y,
                                       void *stream);

/* ---- row-sharded matmul across the GPUs of one node (one process per GPU) ----
 * New: the reference runs each matrix on one host. The rows of a large matrix
 * (e.g. 28672x8192 / 8192x28672) are split evenly over G ranks; every rank
 * computes its rows and an in-place NCCL all-gather over NVLink assembles the
 * full y on every rank. NCCL is loaded at run time (libnccl.so.2). */
#define OUROQ_SHARD_ID_BYTES 128
/* Rank 0 makes the group id (OUROQ_SHARD_ID_BYTES bytes) and the caller hands
 * the bytes to every rank over any channel it has. */
ouroq_status ouroq_shard_unique_id(void *id_out);
/* Join the group as `rank` of `world` on the context's device. Collective:
 * every rank calls it with the same id. */
ouroq_status ouroq_shard_init(ouroq_ctx *ctx, const void *id, int world, int rank);
/* How ouroq_gemm_sharded moves the rows between ranks:
 *   OUROQ_SHARD_PEER (default): one small kernel per call stores each rank's
 *     rows straight into every rank's landing buffer over NVLink (CUDA IPC
 *     mappings); each 64-bit word carries its step number, so readers wait on
 *     the data itself. Every wait is bounded.
 *   OUROQ_SHARD_NCCL: in-place ncclAllGather, then an interleave kernel. */
#define OUROQ_SHARD_PEER 0
#define OUROQ_SHARD_NCCL 1
ouroq_status ouroq_shard_set_transport(ouroq_ctx *ctx, int transport);
/* Leave the group (aborts it instead if a sync timed out or NCCL failed). */
ouroq_status ouroq_shard_finalize(ouroq_ctx *ctx);
/* Rows [*row0, *row0 + *rows) of an M-row matrix that `rank` owns; M must
 * divide evenly (OUROQ_ERR_BAD_SHAPE otherwise). Host-only, no device needed. */
ouroq_status ouroq_shard_rows(int M, int world, int rank, int *row0, int *rows);
/* Upload this rank's rows of a full matrix given in the canonical host layout
 * (same arguments as ouroq_weight_upload, full M). */
ouroq_status ouroq_weight_upload_shard(ouroq_ctx *ctx, ouroq_format fmt, const void *packed_full,
                                       int M, int K, const void *scales_full, float w_scale,
                                       ouroq_weight **out);
/* y [B][M] (full M, on every rank) = W . quant(rotate(x)), x fp32 [B][K]
 * identical on every rank. Every rank must make the same sequence of calls. */
ouroq_status ouroq_gemm_sharded(ouroq_ctx *ctx, const ouroq_weight *w_shard, const float *x,
                                int B, const float *signs, int hadamard_block, float *y,
                                void *stream);
/* Wait until `stream` has finished, at most timeout_ms (< 0: no bound).
 * OUROQ_ERR_TIMEOUT or OUROQ_ERR_NCCL marks the group failed: later sharded
 * calls return OUROQ_ERR_NCCL and finalize aborts the communicator. */
ouroq_status ouroq_shard_sync(ouroq_ctx *ctx, void *stream, int timeout_ms);

/* ---- the decode step either side of the path (infer/mod.rs:298-336) ----
 * fp32, stream-ordered, device buffers. These replace the reference's host
 * ops around the projections so that a decode step stays on the GPU.
 * rmsnorm (ops.rs:12-17): h = x + r (r, h nullable: no residual / not
 * stored), y[b] = h[b] / sqrt(mean(h[b]^2) + eps) * w, B rows of n. */
ouroq_status ouroq_rmsnorm(ouroq_ctx *ctx, const float *x, const float *r, float *h, const float *w,
                           float *y, int B, int n, float eps, void *stream);
/* y = rmsnorm(silu(gate) * up) * w (ops.rs:34-36, the FFN sub-norm). */
ouroq_status ouroq_swiglu_rmsnorm(ouroq_ctx *ctx, const float *gate, const float *up,
                                  const float *w, float *y, int B, int n, float eps, void *stream);
/* NeoX RoPE (ops.rs:21-33, rot = head_dim = 128) of q [B][n_head][128] in
 * place and of k [B][n_kv][128] at position *pos (a device int64), then k and
 * v appended to the caches [B][n_kv][tmax][128] at *pos. */
ouroq_status ouroq_rope_kv_append(ouroq_ctx *ctx, float *q, const float *k, const float *v,
                                  float *kcache, float *vcache, const int64_t *pos, int B,
                                  int n_head, int n_kv, int tmax, float rope_base, void *stream);
/* Causal GQA attention of q [B][n_head][128] over cache positions 0..*pos
 * (mod.rs:337-365, scale 1/sqrt(128)): out [B][n_head][128]. n_head a
 * multiple of n_kv, at most 8 query heads per KV head; every buffer 16-byte
 * aligned. A *pos outside [0, tmax) writes zeros to out, leaves the caches
 * alone and leaves a code in the status word. The slice partials live in
 * the context: calls on one context must not overlap in time. */
ouroq_status ouroq_attention_decode(ouroq_ctx *ctx, const float *q, const float *kcache,
                                    const float *vcache, const int64_t *pos, float *out, int B,
                                    int n_head, int n_kv, int tmax, void *stream);
/* ouroq_rope_kv_append followed by ouroq_attention_decode, in one launch: q
 * and k arrive un-rotated (q is left as it is), k and v are written to the
 * caches at *pos, and out is the attention of the rotated q. */
ouroq_status ouroq_rope_attention_decode(ouroq_ctx *ctx, const float *q, const float *k,
                                         const float *v, float *kcache, float *vcache,
                                         const int64_t *pos, float *out, int B, int n_head,
                                         int n_kv, int tmax, float rope_base, void *stream);

/* The norm in front of a projection group, fused into it (infer/mod.rs:303-333:
 * attn_norm before q/k/v, attn_sub_norm before o, ffn_norm before gate/up,
 * ffn_sub_norm before down): y_i = W_i . (rmsnorm(v) * norm_w) for the n
 * matrices w[i] (one format, one K), with v = x + residual (mode 0; residual
 * may be NULL; h, if not NULL, receives v) or v = silu(x) * residual (mode 1:
 * x the gate projection, residual the up projection, h NULL). x, residual,
 * h: device [B][K] fp32, h overlapping neither x nor residual; y[i]: device
 * [B][M_i]. Up to 2 tokens with rows of
 * up to 11520 values run as one launch (the norm in the GEMV prologue);
 * otherwise the norm kernel writes a context scratch row and the grouped
 * product reads it -- the same results either way up to the order of the sum
 * of squares. */
ouroq_status ouroq_gemm_norm_f32act(ouroq_ctx *ctx, int n, const ouroq_weight *const *w,
                                    const float *x, const float *residual, int mode,
                                    const float *norm_w, float eps, float *h, int B,
                                    float *const *y, void *stream);

/* argmax_token (infer/mod.rs:190-194): the tied lm_head of an F16 or BF16
 * weight [vocab][K] applied to the final hidden states x [B][K] (device
 * fp32), then finite_argmax (mod.rs:70-83: NaN skipped, first maximum wins,
 * 0 when every logit is NaN) of each sequence, in one launch. tokens [B]
 * device int64; logits [B][vocab] device fp32 or NULL. Calls on one context
 * must not overlap in time (the reduction scratch lives in the context). */
ouroq_status ouroq_argmax_token(ouroq_ctx *ctx, const ouroq_weight *w, const float *x, int B,
                                float *logits, int64_t *tokens, void *stream);

/* ---- BMTS v1 shard files (cluster/src/bmts.rs:1-14, 171-209) ----
 * BmtsShard::open: the file is memory-mapped and its header and JSON tensor
 * table parsed; version 2 (Cap'n Proto meta) is refused. Spans are views into
 * the mapping, valid until ouroq_bmts_close. `err` (nullable, err_len bytes)
 * receives the reason of a failure. */
typedef struct ouroq_bmts ouroq_bmts;
ouroq_status ouroq_bmts_open(const char *path, ouroq_bmts **out, char *err, size_t err_len);
ouroq_status ouroq_bmts_close(ouroq_bmts *f);
/* node, tensor count, data-section file offset, sum of declared tensor lengths (data_len) */
ouroq_status ouroq_bmts_info(const ouroq_bmts *f, int *node, int *n_tensors, uint64_t *data_start,
                             uint64_t *data_len);
/* Entry i of the tensor table; shape4 receives up to four dimensions. */
ouroq_status ouroq_bmts_tensor(const ouroq_bmts *f, int i, const char **name, int *rank,
                               uint64_t *shape4, uint32_t *dtype, uint64_t *offset,
                               uint64_t *length);
/* read_span (bmts.rs:286-309): bytes [offset, offset + length) of tensor
 * `name`; a span past the tensor's declared length is refused, never cut. */
ouroq_status ouroq_bmts_span(const ouroq_bmts *f, const char *name, uint64_t offset,
                             uint64_t length, const void **out, char *err, size_t err_len);
/* Stage::from_shard for one tensor (infer/mod.rs:110-123) plus the device
 * upload: dtype 143 (Tl1) -> OUROQ_FMT_PTQ1_0, 34 (TQ1_0) -> OUROQ_FMT_TQ1_0,
 * 1 (F16) -> OUROQ_FMT_F16, 30 (BF16) -> OUROQ_FMT_BF16; GGUF shape [in, out]
 * -> K = shape[0], M = shape[1]. Other dtypes: OUROQ_ERR_UNSUPPORTED. */
ouroq_status ouroq_bmts_upload(ouroq_ctx *ctx, const ouroq_bmts *f, const char *name,
                               ouroq_weight **out, char *err, size_t err_len);

/* ---- host-buffer mirrors of the reference operators (synchronous) ---- */

/* ops::matvec_q (ops.rs:76-84): x_host [K] fp32 -> y_host [M] fp32. */
ouroq_status ouroq_matvec_q(ouroq_ctx *ctx, const ouroq_weight *w, const float *x_host,
                            float *y_host);
/* ops::matmul_q (ops.rs:219-230): x_host [k][K] -> y_host [k][M]
 * (= the reference's y[c*out_len + r]); PTQ1_0 in matmul_tl1's K-column
 * order for every k, as matmul_q gives. Both mirrors are synchronous: x is
 * copied in, y copied back -- or, for TERNARY2 / SIGN1G128 weights at
 * k <= 8 with a page-locked mapped y_host that covers its [k][M] floats in
 * one allocation, stored into y_host by the kernel directly. */
ouroq_status ouroq_matmul_q(ouroq_ctx *ctx, const ouroq_weight *w, const float *x_host, int k,
                            float *y_host);
/* The projections of one stage call in one round trip: Stage::wm /
 * wmat_batched (infer/mod.rs:138-167) run once per named tensor of a layer
 * (q, k, v, o, gate, up, down: run_layer, infer/mod.rs:305-335), each a
 * matvec_q / matmul_q. Here n (<= 8) such products go in one call:
 * y_host[i] [k][M_i] = W_i . x_host[i] [k][K_i], entries may share an input.
 * Results are those of ouroq_matmul_q on each entry (ouroq_matvec_q's for
 * k = 1). Synchronous. Page-locked host buffers (cudaHostAlloc /
 * cudaHostRegister) are copied by DMA directly, and buffers that sit back to
 * back in memory cross in one copy; pageable ones go through the context's
 * page-locked staging buffer. When k <= 8, the weights are TERNARY2 or
 * SIGN1G128 and every y_host[i] is page-locked, mapped and covers its
 * [k][M_i] floats inside one allocation, the kernel stores the results into
 * y_host directly (no staging buffer, no copy back); otherwise y goes
 * through the device stage. Either way y_host holds the results when the
 * call returns OUROQ_OK. */
ouroq_status ouroq_matmul_q_group(ouroq_ctx *ctx, int n, const ouroq_weight *const *w,
                                  const float *const *x_host, int k, float *const *y_host);
/* hadamard::rotate_fwd (hadamard.rs:41-53) in place on a host buffer of n floats. */
ouroq_status ouroq_rotate_fwd(ouroq_ctx *ctx, float *x_host, const float *signs_host, size_t n,
                              size_t block);
/* hadamard::rotate_inv (hadamard.rs:57-66) in place on a host buffer. */
ouroq_status ouroq_rotate_inv(ouroq_ctx *ctx, float *x_host, const float *signs_host, size_t n,
                              size_t block);

#ifdef __cplusplus
}
#endif
#endif /* OUROQ_H */
