/*
 * oracle.h -- CPU restatement of OuroborOS's quantized-weight matmul path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the shipped library links, loads or
 * calls this code. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference leg use it, and only as the checker or the
 * timed CPU baseline.
 *
 * Two families of functions live here.
 *
 *  1. Restatements of the reference's own Rust code (parity pinned by the
 *     reference's own unit tests, ported as known-answer tests in
 *     tests/test_oracle_kat.py):
 *       - f16 decode              cluster/src/infer/dequant.rs:21-47
 *       - TQ1_0 block decode      cluster/src/infer/dequant.rs:50-105
 *       - PTQ1_0 (Tl1) group      cluster/src/infer/dequant.rs:123-195
 *       - WHT rotate_fwd / inv    cluster/src/infer/hadamard.rs:15-66
 *       - matvec_tl1 (scalar)     cluster/src/infer/ops.rs:294-363
 *       - matvec_tl1 (SSE4.1)     cluster/src/infer/ops.rs:499-584
 *       - matmul_tl1 (scalar K)   cluster/src/infer/ops.rs:162-286
 *       - matmul_tl1 (SSE4.1 K)   cluster/src/infer/ops.rs:162-215,381-481
 *       - matvec_qblock (TQ1_0)   cluster/src/infer/ops.rs:53-60,101-128
 *       - mt_threads chunking     cluster/src/infer/ops.rs:63-73,104-105
 *       - rmsnorm, rope_neox, silu, softmax, dot   ops.rs:11-60
 *       - attend (causal GQA)     cluster/src/infer/mod.rs:338-365
 *
 *  2. The int8-activation arithmetic of BitNet b1.58 that this library
 *     targets but the reference does not contain (it lives in the un-vendored bitnet-cpp submodule,
 *     .gitmodules:1-3, commit unknown). PARITY UNPINNED: no reference test
 *     or golden vector covers it. Every free choice is fixed here in writing:
 *       - s_x = absmax / 127.0f (one fp32 divide); absmax == 0 -> s_x = 0, q = 0
 *       - q = clamp(rintf(x / s_x), -127, 127), round-to-nearest-even
 *       - TERNARY2: code c = w + 1 in {0,1,2}, 4 per byte, row-major,
 *         k % 4 -> bits 2*(k % 4) (LSB first); one fp32 w_scale per tensor
 *       - SIGN1G128: bit 1 -> +1, bit 0 -> -1, 8 per byte, row-major,
 *         k % 8 -> bit k % 8 (LSB first); fp16 scale per 128 along K, [M][K/128]
 *       - ternary epilogue: y = ((float)acc * w_scale) * s_x
 *       - sign epilogue: sum = 0; for g ascending: sum += (float)acc_g * scale_g;
 *         y = sum * s_x   (separate fp32 mul and add, no fused multiply-add)
 *       - optional blockwise WHT before quantisation = rotate_fwd above.
 *
 * Compile with -ffp-contract=off and no fast-math: every float operation here
 * is one IEEE binary32 operation with round-to-nearest-even.
 */
#ifndef OUROQ_ORACLE_H
#define OUROQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded generators (LCG of ouro-wgpu/tests/l1_parity.rs:7-15) ---- */
uint64_t orc_lcg_step(uint64_t *st);
void orc_lcg_bytes(uint64_t seed, uint8_t *out, size_t n);
void orc_normals(uint64_t seed, float *out, size_t n);
void orc_ternary(uint64_t seed, int8_t *w, size_t n);      /* p(-1,0,1) = .25,.5,.25 */
void orc_signs(uint64_t seed, int8_t *w, size_t n);        /* p(-1,+1) = .5,.5 */
void orc_outliers(uint64_t seed, float *x, size_t n, double frac, float mult);
void orc_group_scales(uint64_t seed, uint16_t *scales, size_t n, float sigma);

/* ---- f16 ---- */
float orc_f16_to_f32(uint16_t bits);
uint16_t orc_f32_to_f16(float v); /* round to nearest even; used by generators only */

/* ---- canonical packers (host layouts of the C ABI) ---- */
void orc_pack_tern2(const int8_t *w, int M, int K, uint8_t *packed);
void orc_pack_sign1(const int8_t *w, int M, int K, uint8_t *packed);
float orc_absmean_scale(const int8_t *w, size_t n, float base); /* mean|w*base| */

/* ---- Hadamard rotation (hadamard.rs) ---- */
void orc_wht_inplace(float *x, size_t n);
int orc_rotate_fwd(float *x, const float *signs, size_t n, size_t block);
int orc_rotate_inv(float *x, const float *signs, size_t n, size_t block);

/* ---- per-token absmax int8 quantisation (optionally after rotate_fwd) ---- */
int orc_quantize_act(const float *x, int B, int K, const float *signs, int had_block,
                     int8_t *q, float *s_x, float *x_rot /* nullable, [B][K] */);

/* ---- int8-activation GEMM on the TERNARY2 / SIGN1G128 formats ---- */
int orc_gemm_tern2(const uint8_t *packed, int M, int K, float w_scale, const int8_t *q,
                   const float *s_x, int B, int32_t *acc /* nullable [B][M] */, float *y);
int orc_gemm_sign1(const uint8_t *packed, const uint16_t *scales, int M, int K,
                   const int8_t *q, const float *s_x, int B,
                   int32_t *acc_g /* nullable [B][M][K/128] */, float *y);
/* Same arithmetic, output rows chunked over `threads` pthreads like ops.rs:104-105. */
int orc_gemm_tern2_mt(const uint8_t *packed, int M, int K, float w_scale, const int8_t *q,
                      const float *s_x, int B, float *y, int threads);
int orc_gemm_sign1_mt(const uint8_t *packed, const uint16_t *scales, int M, int K,
                      const int8_t *q, const float *s_x, int B, float *y, int threads);

/* ---- the reference's own formats (dequant.rs / ops.rs) ---- */
void orc_tq1_block(const uint8_t *bytes, float *out);      /* 54 B -> 256 */
void orc_tl1_group(const uint8_t *bytes, float *out);      /* 28 B -> 128 */
int orc_matvec_tl1_scalar(const uint8_t *payload, int out_len, int in_len, const float *x,
                          float *y);
int orc_matvec_tl1_sse(const uint8_t *payload, int out_len, int in_len, const float *x,
                       float *y, int threads);
int orc_matmul_tl1_scalar(const uint8_t *payload, int out_len, int in_len, const float *x,
                          int k, float *y /* [k][out_len] */);
/* matmul_tl1's x86 K-column path (tl1_rows_avx2_k), rows threaded as ops.rs:166-167 */
int orc_matmul_tl1_sse(const uint8_t *payload, int out_len, int in_len, const float *x, int k,
                       float *y /* [k][out_len] */, int threads);
int orc_matvec_tq1(const uint8_t *payload, int out_len, int in_len, const float *x, float *y,
                   int threads);
/* 16-bit weights (QuantKind::F16 / Bf16) and the greedy pick */
float orc_bf16_to_f32(uint16_t bits);
int orc_matvec_half(const uint8_t *payload, int out_len, int in_len, const float *x, float *y,
                    int bf16, int threads);
int orc_finite_argmax(const float *l, int n);

/* ---- the decode step's host ops (ops.rs:11-60, infer/mod.rs:338-365), fp32 ---- */
void orc_rmsnorm(const float *x, const float *w, int n, float eps, float *y);
void orc_rope_neox(float *v, long long t, int rot, float base); /* in place, one head */
float orc_silu(float x);
void orc_swiglu(const float *gate, const float *up, int n, float *out); /* silu(g) * u */
void orc_softmax(float *v, int n);                                /* in place */
float orc_dot(const float *a, const float *b, int n);
int orc_attend(const float *q, const float *k, const float *v, int seq, int n_head, int n_kv,
               int hd, float *out); /* k, v [seq][n_kv*hd]; q, out [n_head*hd] */
int orc_hw_threads(void);

#ifdef __cplusplus
}
#endif
#endif
