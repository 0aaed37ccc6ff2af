// api.cpp -- implementation of the C ABI declared in include/ouroq.h.
//
// Host-side responsibilities: argument validation with the reference's error
// rules (shape / width mismatches are errors, never silent), device memory
// ownership for uploaded weights, dispatch to the kernels, and the
// host-buffer mirrors of ops::matvec_q / matmul_q / hadamard::rotate_*.
// No exception or abort crosses the ABI.
#include "ouroq.h"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "kernels.h"

using namespace ouroq;

// A planned stream-GEMV launch (tile split, shared-memory plan) for one set
// of shapes: planning balances hundreds of tiles on the host (tens of
// microseconds), so each context keeps the plans of the shapes it saw last.
// The key is everything gemv_stream_prepare reads besides the pointers: the
// format, batch, per job M, K and rotation, and which jobs share an input.
struct StreamPlan {
  bool used = false, ok = false;
  int fmt = 0, B = 0, njobs = 0, nsms = 0;
  int M[ouroq::kMaxGemvJobs], K[ouroq::kMaxGemvJobs], had[ouroq::kMaxGemvJobs],
      cls[ouroq::kMaxGemvJobs];
  // results
  int grid = 0, ntiles = 0, xcap = 0, defer = 0, stages = 0, cluster = 1;
  size_t smem = 0;
  int tile_begin[ouroq::kMaxGemvJobs];
  uint16_t cta_tile[ouroq::kMaxGemvCtas + 1];
};
constexpr int kStreamPlans = 16;

struct ouroq_ctx {
  int device = 0;
  int num_sms = 0;
  int smem_optin = 0;  // opt-in shared memory per block (bytes)
  bool pdl = true;
  bool use_tc = true;  // tensor-core path for batches >= 16
  bool stream_gemv = true;  // fused one/two-token ternary launches on gemv_stream_kernel
  // weights the next GEMV launch prefetches into L2 (ouroq_set_prefetch)
  std::vector<std::pair<const uint8_t*, uint32_t>> prefetch;
  StreamPlan plans[kStreamPlans];  // recent stream-GEMV plans, replaced round robin
  int next_plan = 0;
  std::string err;
  unsigned* d_status = nullptr;
  uint64_t launches = 0;
  cudaStream_t host_stream = nullptr;  // stream of the host-buffer mirrors
  // quantisation scratch of ouroq_gemm_f32act / the host mirrors
  int8_t* q_scratch = nullptr;
  size_t q_cap = 0;
  float* s_scratch = nullptr;
  size_t s_cap = 0;
  // staging for host-buffer calls
  float* x_stage = nullptr;
  size_t x_cap = 0;
  float* y_stage = nullptr;
  size_t y_cap = 0;
  float* sign_stage = nullptr;
  size_t sign_cap = 0;
  // page-locked host staging of the host-buffer calls (pageable inputs/outputs)
  float* hx_stage = nullptr;
  size_t hx_cap = 0;
  float* hy_stage = nullptr;
  size_t hy_cap = 0;
  // rotated fp32 activations for the reference formats (hadamard_block != 0)
  float* rot_scratch = nullptr;
  float* norm_scratch = nullptr;  // normalised activations when the norm is not fused
  size_t norm_cap = 0;
  size_t rot_cap = 0;
  // slice partials of the decode attention
  float* attn_part = nullptr;
  size_t attn_cap = 0;
  unsigned* attn_ctr = nullptr;  // zeroed on allocation; each launch leaves it zero
  size_t attn_ctr_cap = 0;
  unsigned long long* head_key = nullptr;  // argmax keys [B] + 1 counter word,
  size_t head_key_cap = 0;                 // zeroed on allocation, left zero
  // row-sharded group (NCCL communicator, opaque here)
  void* comm = nullptr;
  int shard_world = 1, shard_rank = 0;
  bool comm_failed = false;
  float* gather = nullptr;  // NCCL transport: [G][B][R]; peer transport: staging [B][R]
  size_t gather_cap = 0;
  int transport = OUROQ_SHARD_PEER;
  unsigned long long* landing = nullptr;  // peer transport: two parities of [G][B][R] words
  size_t landing_words = 0;               // per parity
  unsigned long long* peer_ptr[kShardMaxRanks] = {};
  unsigned* shard_ctr = nullptr;  // step, done
  unsigned long long peer_timeout_ns = 2000000000ull;
};

struct ouroq_weight {
  int fmt = 0;
  int M = 0, K = 0;
  uint8_t* w = nullptr;        // device layout
  uint16_t* scales = nullptr;  // sign: tiled fp16 group scales
  float w_scale = 0.0f;
  size_t bytes = 0;
  int shard_M = 0;     // full row count of a row-sharded matrix (0 = not sharded)
  int shard_row0 = 0;  // first full-matrix row held here
};

namespace {

__attribute__((format(printf, 3, 4)))
ouroq_status fail(ouroq_ctx* ctx, ouroq_status st, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    ctx->err = buf;
  }
  return st;
}

ouroq_status cuda_fail(ouroq_ctx* ctx, cudaError_t e, const char* what) {
  if (e == cudaErrorMemoryAllocation)
    return fail(ctx, OUROQ_ERR_OOM, "%s: %s", what, cudaGetErrorString(e));
  return fail(ctx, OUROQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define CU(ctx, call, what)                                   \
  do {                                                        \
    cudaError_t e_ = (call);                                  \
    if (e_ != cudaSuccess) return cuda_fail((ctx), e_, what); \
  } while (0)

// Makes ctx->device current for the scope, restoring the caller's device.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename T>
ouroq_status grow(ouroq_ctx* ctx, T*& buf, size_t& cap, size_t n, const char* what) {
  if (n <= cap) return OUROQ_OK;
  if (buf) cudaFree(buf);
  buf = nullptr;
  cap = 0;
  size_t want = n < 256 ? 256 : n;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&buf), want * sizeof(T));
  if (e != cudaSuccess) return cuda_fail(ctx, e, what);
  cap = want;
  return OUROQ_OK;
}

bool valid_block(int b) { return b >= 2 && b <= 1024 && (b & (b - 1)) == 0; }

ouroq_status check_quant_args(ouroq_ctx* ctx, int B, int K, int block) {
  if (B < 0 || K <= 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d K=%d", B, K);
  if (K % 4) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "K=%d not a multiple of 4", K);
  if (block != 0) {
    if (!valid_block(block))
      return fail(ctx, OUROQ_ERR_BAD_SHAPE, "hadamard block %d not a power of two in [2,1024]",
                  block);
    if (K % block) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "len %d not multiple of block %d", K, block);
    if (block < 32 && K % 32)
      return fail(ctx, OUROQ_ERR_BAD_SHAPE, "K=%d must be a multiple of 32 for block %d", K, block);
  }
  if ((size_t)K * 4 > 200 * 1024)
    return fail(ctx, OUROQ_ERR_BAD_SHAPE, "K=%d too wide for the quantiser (max 51200)", K);
  return OUROQ_OK;
}

// Largest token batch per small-batch GEMV launch for this K.
int gemv_chunk(int K) {
  int c = (int)(kGemvMaxXBytes / (size_t)K);
  return c > kGemvMaxB ? kGemvMaxB : c;
}

// Can this GEMV launch keep each CTA's activations in shared memory?
bool gemv_fits(const ouroq_ctx* ctx, GemvLaunch L) {
  int grid = 0;
  size_t smem = 0;
  return gemv_prepare(L, ctx->num_sms, ctx->smem_optin, &grid, &smem);
}

GemvJob make_job(const ouroq_weight* w, const int8_t* q, const float* s_x, float* y, int32_t* acc) {
  GemvJob j{};
  j.w = w->w;
  j.scales = w->scales;
  j.q = q;
  j.s_x = s_x;
  j.y = y;
  j.acc = acc;
  j.w_scale = w->w_scale;
  j.M = w->M;
  j.K = w->K;
  j.ldy = w->M;
  return j;
}

// The stream-GEMV plan of these shapes, from the context's recent plans or
// made now; null when the launch is not one the stream kernel takes
// (ternary, fused quantisation, no rotation, no fused norm, 1..8 tokens).
StreamPlan* stream_plan(ouroq_ctx* ctx, const GemvLaunch& L) {
  if (!ctx->stream_gemv || L.fmt != kTern2 || !L.fused || L.norm.w || L.B < 1 || L.B > kStreamMaxB)
    return nullptr;
  StreamPlan key;
  key.fmt = L.fmt;
  key.B = L.B;
  key.njobs = L.njobs;
  key.nsms = ctx->num_sms;
  for (int j = 0; j < L.njobs; ++j) {
    key.M[j] = L.jobs[j].M;
    key.K[j] = L.jobs[j].K;
    key.had[j] = L.jobs[j].had_block;
    int c = 0;
    while (c < j && !(L.jobs[c].xf == L.jobs[j].xf && L.jobs[c].K == L.jobs[j].K)) ++c;
    key.cls[j] = c;
  }
  auto same = [&](const StreamPlan& p) {
    if (!p.used || p.fmt != key.fmt || p.B != key.B || p.njobs != key.njobs || p.nsms != key.nsms)
      return false;
    for (int j = 0; j < key.njobs; ++j)
      if (p.M[j] != key.M[j] || p.K[j] != key.K[j] || p.had[j] != key.had[j] || p.cls[j] != key.cls[j])
        return false;
    return true;
  };
  for (StreamPlan& p : ctx->plans)
    if (same(p)) return &p;
  GemvLaunch S = L;
  int grid = 0;
  size_t smem = 0;
  StreamPlan* plan = &ctx->plans[ctx->next_plan];
  ctx->next_plan = (ctx->next_plan + 1) % kStreamPlans;
  *plan = key;
  plan->used = true;
  plan->ok = gemv_stream_prepare(S, ctx->num_sms, &grid, &smem);
  if (plan->ok) {
    plan->grid = grid;
    plan->smem = smem;
    plan->ntiles = S.ntiles;
    plan->xcap = S.xcap;
    plan->defer = S.defer;
    plan->stages = S.stages;
    plan->cluster = S.cluster;
    for (int j = 0; j < L.njobs; ++j) plan->tile_begin[j] = S.jobs[j].tile_begin;
    std::memcpy(plan->cta_tile, S.cta_tile, sizeof(plan->cta_tile));
  }
  return plan;
}

// Does a fused launch of more than kFusedMaxB tokens run on the stream
// kernel (one launch, each distinct input quantised once per CTA or
// cluster)? Otherwise such batches are quantised in a launch of their own.
bool stream_takes(ouroq_ctx* ctx, const GemvLaunch& L) {
  const StreamPlan* p = stream_plan(ctx, L);
  return p && p->ok;
}

ouroq_status run_gemv(ouroq_ctx* ctx, GemvLaunch& L, cudaStream_t s) {
  L.status = ctx->d_status;
  L.npf = 0;
  for (const auto& r : ctx->prefetch) {
    if (L.npf == kMaxGemvJobs) break;
    L.pf_ptr[L.npf] = r.first;
    L.pf_bytes[L.npf++] = r.second;
  }
  ctx->prefetch.clear();
  if (L.njobs == 0 || L.B == 0) return OUROQ_OK;
  if (StreamPlan* plan = stream_plan(ctx, L)) {
    if (plan->ok) {
      GemvLaunch S = L;
      S.ntiles = plan->ntiles;
      S.xcap = plan->xcap;
      S.defer = plan->defer;
      S.stages = plan->stages;
      S.cluster = plan->cluster;
      for (int j = 0; j < L.njobs; ++j) S.jobs[j].tile_begin = plan->tile_begin[j];
      std::memcpy(S.cta_tile, plan->cta_tile, sizeof(S.cta_tile));
      CU(ctx, launch_gemv_stream(S, plan->grid, plan->smem, s, ctx->pdl), "gemv launch");
      if (S.ntiles > 0) ctx->launches++;
      return OUROQ_OK;
    }
  }
  if (!gemv_fits(ctx, L))
    return fail(ctx, OUROQ_ERR_UNSUPPORTED,
                "B=%d: the activations of one CTA's matrices do not fit in shared memory", L.B);
  CU(ctx, launch_gemv(L, ctx->num_sms, ctx->smem_optin, s, ctx->pdl), "gemv launch");
  if (L.ntiles > 0) ctx->launches++;
  return OUROQ_OK;
}

// Token batches from this size up run on the tensor cores (ternary and sign weights).
// (From 9 tokens one tensor-core launch, its token tile of 16 padded with
// zero rows by the TMA, beats the two GEMV launches that 9-15 tokens take.)
constexpr int kTcMinBatch = 9;

ouroq_status gemm_impl(ouroq_ctx* ctx, const ouroq_weight* w, const int8_t* q, const float* s_x,
                       int B, float* y, int32_t* acc, cudaStream_t s) {
  const int dfmt = w->fmt == OUROQ_FMT_TERNARY2 ? kTern2 : kSign1;
  if (dfmt == kSign1 && B >= kTcMinBatch && ctx->use_tc && gemm_sign_tc_supported(w->M, w->K, B)) {
    TcLaunch L{};
    L.w = w->w;
    L.scales = w->scales;
    L.y = y;
    L.acc = acc;
    L.s_x = s_x;
    L.M = w->M;
    L.K = w->K;
    L.ldy = w->M;
    L.tok0 = 0;
    L.nvalid = B;
    L.status = ctx->d_status;
    CU(ctx, launch_gemm_sign_tc(L, q, B, ctx->smem_optin, ctx->num_sms, s, ctx->pdl), "sign tensor-core gemm launch");
    ctx->launches++;
    return OUROQ_OK;
  }
  if (B >= kTcMinBatch && ctx->use_tc && gemm_tc_supported(dfmt, w->M, w->K, B)) {
    TcLaunch L{};
    L.w = w->w;
    L.y = y;
    L.acc = acc;
    L.s_x = s_x;
    L.w_scale = w->w_scale;
    L.M = w->M;
    L.K = w->K;
    L.ldy = w->M;
    L.tok0 = 0;
    L.nvalid = B;
    L.status = ctx->d_status;
    CU(ctx, launch_gemm_tc(L, q, B, ctx->smem_optin, ctx->num_sms, s, ctx->pdl), "tensor-core gemm launch");
    ctx->launches++;
    return OUROQ_OK;
  }
  const int chunk = gemv_chunk(w->K);
  if (chunk < 1) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "K=%d too wide for the GEMV path", w->K);
  const int G = w->K / 128;
  for (int b0 = 0; b0 < B; b0 += chunk) {
    const int nb = B - b0 < chunk ? B - b0 : chunk;
    GemvLaunch L{};
    L.njobs = 1;
    L.B = nb;
    L.fmt = w->fmt == OUROQ_FMT_TERNARY2 ? kTern2 : kSign1;
    int32_t* a = nullptr;
    if (acc) a = acc + (size_t)b0 * w->M * (w->fmt == OUROQ_FMT_TERNARY2 ? 1 : G);
    L.jobs[0] = make_job(w, q + (size_t)b0 * w->K, s_x + b0, y + (size_t)b0 * w->M, a);
    ouroq_status st = run_gemv(ctx, L, s);
    if (st != OUROQ_OK) return st;
  }
  return OUROQ_OK;
}

// y_i = W_i . q_i (pre-quantised, L.jobs[i].q / s_x / y) for the n weights
// of a group and B tokens: up to kGemvMaxB tokens one grouped GEMV launch;
// from kTcMinBatch ternary weights one grouped tensor-core launch; otherwise
// one product per weight.
ouroq_status group_product(ouroq_ctx* ctx, GemvLaunch& L, const ouroq_weight* const* w, int n, int B,
                           cudaStream_t s) {
  if (B <= kGemvMaxB) return run_gemv(ctx, L, s);
  bool tc = B >= kTcMinBatch && ctx->use_tc;
  for (int i = 0; i < n && tc; ++i)
    tc = w[i]->fmt == OUROQ_FMT_TERNARY2 && gemm_tc_supported(kTern2, w[i]->M, w[i]->K, B) &&
         aligned16(L.jobs[i].q);
  if (tc && n > 1) {
    TcJob jobs[kMaxTcJobs];
    const int8_t* qs[kMaxTcJobs];
    for (int i = 0; i < n; ++i) {
      const GemvJob& J = L.jobs[i];
      jobs[i] = TcJob{J.w, J.y, J.acc, J.s_x, J.w_scale, J.M, J.K, J.ldy};
      qs[i] = J.q;
    }
    TcLaunch T{};
    T.tok0 = 0;
    T.nvalid = B;
    T.status = ctx->d_status;
    CU(ctx, launch_gemm_tc_group(T, jobs, qs, n, B, ctx->smem_optin, ctx->num_sms, s, ctx->pdl),
       "grouped tensor-core gemm launch");
    ctx->launches++;
    return OUROQ_OK;
  }
  for (int i = 0; i < n; ++i) {
    const GemvJob& J = L.jobs[i];
    ouroq_status st = gemm_impl(ctx, w[i], J.q, J.s_x, B, J.y, J.acc, s);
    if (st != OUROQ_OK) return st;
  }
  return OUROQ_OK;
}

ouroq_status quantize_impl(ouroq_ctx* ctx, const float* x, int B, int K, const float* signs,
                           int block, int8_t* q, float* s_x, cudaStream_t s) {
  QuantLaunch L{};
  L.njobs = 1;
  L.B = B;
  QuantJob& J = L.jobs[0];
  J.x = x;
  J.signs = signs;
  J.q = q;
  J.s_x = s_x;
  J.x_rot = nullptr;
  J.K = K;
  J.had_block = block;
  J.had_scale = block ? 1.0f / std::sqrt((float)block) : 1.0f;
  if (B == 0) return OUROQ_OK;
  CU(ctx, launch_quantize(L, s, ctx->pdl), "quantize launch");
  ctx->launches++;
  return OUROQ_OK;
}

bool is_half_format(int fmt) { return fmt == OUROQ_FMT_F16 || fmt == OUROQ_FMT_BF16; }
bool is_ref_format(int fmt) {
  return fmt == OUROQ_FMT_PTQ1_0 || fmt == OUROQ_FMT_TQ1_0 || is_half_format(fmt);
}

// Bytes of one row of a reference-format payload (dequant.rs:123-130, 50-53;
// 2 bytes per element for F16 / BF16).
size_t ref_row_bytes(int fmt, int K) {
  if (is_half_format(fmt)) return (size_t)K * 2;
  return fmt == OUROQ_FMT_PTQ1_0 ? (size_t)K / 128 * 28 : (size_t)K / 256 * 54;
}

ouroq_status check_weight_shape(ouroq_ctx* ctx, ouroq_format fmt, int M, int K) {
  if (fmt != OUROQ_FMT_TERNARY2 && fmt != OUROQ_FMT_SIGN1G128 && !is_ref_format(fmt))
    return fail(ctx, OUROQ_ERR_BAD_ARG, "unknown format %d", (int)fmt);
  if (M <= 0 || K <= 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "M=%d K=%d", M, K);
  if (is_half_format(fmt)) return OUROQ_OK;
  if (K % 128) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "K=%d not a multiple of 128", K);
  if (fmt == OUROQ_FMT_TQ1_0 && K % 256)
    return fail(ctx, OUROQ_ERR_BAD_SHAPE, "TQ1_0: K=%d not a multiple of 256", K);
  return OUROQ_OK;
}

// Reference formats are kept on the device byte for byte as in the shard.
ouroq_status upload_ref(ouroq_ctx* ctx, ouroq_format fmt, const void* packed, int M, int K,
                        ouroq_weight** out, bool from_device) {
  ouroq_weight* w = new (std::nothrow) ouroq_weight;
  if (!w) return fail(ctx, OUROQ_ERR_OOM, "host allocation");
  w->fmt = fmt;
  w->M = M;
  w->K = K;
  const size_t bytes = ref_row_bytes(fmt, K) * (size_t)M;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&w->w), bytes);
  if (e != cudaSuccess) {
    delete w;
    return cuda_fail(ctx, e, "weight alloc");
  }
  e = cudaMemcpyAsync(w->w, packed, bytes,
                      from_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                      ctx->host_stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->host_stream);
  if (e != cudaSuccess) {
    cudaFree(w->w);
    delete w;
    return cuda_fail(ctx, e, "weight upload");
  }
  w->bytes = bytes;
  *out = w;
  return OUROQ_OK;
}

// fp32 x [B][K] -> y [B][M] for the reference formats (no quantisation).
// columns: PTQ1_0 in matmul_tl1's K-column order (the reference's matmul_q)
// instead of matvec_tl1's order per token (its matvec_q); the other formats
// have one order for both.
ouroq_status ref_matvec(ouroq_ctx* ctx, const ouroq_weight* w, const float* x, int B, float* y,
                        cudaStream_t s, bool columns) {
  if (is_half_format(w->fmt)) {
    if ((size_t)B > 65535 * 8) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d too large", B);
    HeadLaunch L{};
    L.w = reinterpret_cast<const uint16_t*>(w->w);
    L.x = x;
    L.y = y;
    L.M = w->M;
    L.K = w->K;
    L.B = B;
    L.ldy = w->M;
    L.bf16 = w->fmt == OUROQ_FMT_BF16;
    L.vec = w->K % 8 == 0 && aligned16(w->w) && aligned16(x);
    L.num_sms = ctx->num_sms;
    CU(ctx, launch_head(L, s, ctx->pdl), "16-bit matvec launch");
    ctx->launches++;
    return OUROQ_OK;
  }
  RefLaunch P{};
  P.fmt = w->fmt == OUROQ_FMT_PTQ1_0 ? kPtq1 : kTq1;
  P.w = w->w;
  P.x = x;
  P.y = y;
  P.M = w->M;
  P.K = w->K;
  P.B = B;
  P.ldy = w->M;
  if (P.fmt == kPtq1 && columns) {
    CU(ctx, launch_tl1_columns(P, s), "PTQ1_0 K-column launch");
    ctx->launches++;
    return OUROQ_OK;
  }
  const size_t smem = P.fmt == kPtq1 ? tl1_smem_bytes(w->K, tl1_rows_per_cta(w->K, w->M, ctx->num_sms))
                                     : tq1_smem_bytes(w->K);
  if (smem > (size_t)ctx->smem_optin)
    return fail(ctx, OUROQ_ERR_UNSUPPORTED, "K=%d too wide for the reference-format kernels", w->K);
  if ((size_t)B > 65535) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d (max 65535)", B);
  CU(ctx, launch_refmt_matvec(P, ctx->num_sms, s), "reference-format matvec launch");
  ctx->launches++;
  return OUROQ_OK;
}

ouroq_status upload_impl(ouroq_ctx* ctx, ouroq_format fmt, const void* packed, int M, int K,
                         const void* scales, float w_scale, ouroq_weight** out, bool from_device) {
  if (!ctx || !packed || !out) return fail(ctx, OUROQ_ERR_BAD_ARG, "null argument");
  *out = nullptr;
  ouroq_status st = check_weight_shape(ctx, fmt, M, K);
  if (st != OUROQ_OK) return st;
  if (fmt == OUROQ_FMT_SIGN1G128 && !scales)
    return fail(ctx, OUROQ_ERR_BAD_ARG, "SIGN1G128 needs group scales");
  DeviceGuard g(ctx->device);
  // device-side inputs may still be in flight on the caller's streams
  if (from_device) CU(ctx, cudaDeviceSynchronize(), "upload input sync");
  if (is_ref_format(fmt)) return upload_ref(ctx, fmt, packed, M, K, out, from_device);
  ouroq_weight* w = new (std::nothrow) ouroq_weight;
  if (!w) return fail(ctx, OUROQ_ERR_OOM, "host allocation");
  w->fmt = fmt;
  w->M = M;
  w->K = K;
  w->w_scale = w_scale;
  const int dfmt = fmt == OUROQ_FMT_TERNARY2 ? kTern2 : kSign1;
  const size_t rb = fmt == OUROQ_FMT_TERNARY2 ? (size_t)K / 4 : (size_t)K / 8;
  const size_t canon_bytes = rb * (size_t)M;
  const size_t canon_sbytes = (size_t)M * (K / 128) * 2;
  const size_t wbytes = tiled_weight_bytes(dfmt, M, K);
  uint8_t* canon = nullptr;
  uint16_t* canon_s = nullptr;
  cudaStream_t s = ctx->host_stream;
  auto cleanup = [&](ouroq_status r) {
    if (!from_device) {
      if (canon) cudaFree(canon);
      if (canon_s) cudaFree(canon_s);
    }
    if (r != OUROQ_OK) {
      if (w->w) cudaFree(w->w);
      if (w->scales) cudaFree(w->scales);
      delete w;
    }
    return r;
  };
  if (from_device && ((reinterpret_cast<uintptr_t>(packed) & 3u) ||
                      (scales && (reinterpret_cast<uintptr_t>(scales) & 1u))))
    return cleanup(fail(ctx, OUROQ_ERR_BAD_ALIGN, "device weights must be 4-byte aligned"));
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&w->w), wbytes);
  if (e != cudaSuccess) return cleanup(cuda_fail(ctx, e, "weight alloc"));
  if (from_device) {
    canon = static_cast<uint8_t*>(const_cast<void*>(packed));
    canon_s = static_cast<uint16_t*>(const_cast<void*>(scales));
  } else {
    e = cudaMalloc(reinterpret_cast<void**>(&canon), canon_bytes);
    if (e != cudaSuccess) return cleanup(cuda_fail(ctx, e, "staging alloc"));
    e = cudaMemcpyAsync(canon, packed, canon_bytes, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return cleanup(cuda_fail(ctx, e, "weight upload"));
    if (scales) {
      e = cudaMalloc(reinterpret_cast<void**>(&canon_s), canon_sbytes);
      if (e != cudaSuccess) return cleanup(cuda_fail(ctx, e, "staging alloc"));
      e = cudaMemcpyAsync(canon_s, scales, canon_sbytes, cudaMemcpyHostToDevice, s);
      if (e != cudaSuccess) return cleanup(cuda_fail(ctx, e, "scale upload"));
    }
  }
  e = launch_repack(dfmt, canon, w->w, M, K, s);
  if (e != cudaSuccess) return cleanup(cuda_fail(ctx, e, "repack"));
  ctx->launches++;
  w->bytes = wbytes;
  if (fmt == OUROQ_FMT_SIGN1G128) {
    const size_t sbytes = tiled_scale_bytes(M, K);
    e = cudaMalloc(reinterpret_cast<void**>(&w->scales), sbytes);
    if (e != cudaSuccess) return cleanup(cuda_fail(ctx, e, "scale alloc"));
    e = launch_repack_scales(canon_s, w->scales, M, K, s);
    if (e != cudaSuccess) return cleanup(cuda_fail(ctx, e, "scale repack"));
    ctx->launches++;
    w->bytes += sbytes;
  }
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cleanup(cuda_fail(ctx, e, "upload sync"));
  *out = w;
  return cleanup(OUROQ_OK);
}

// ---- NCCL, resolved at run time: the library does not link it, so a process
// that never shards needs no NCCL at all, and one that imported PyTorch first
// shares the copy PyTorch already loaded.
struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api = [] {
    NcclApi a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      const char* e = dlerror();
      a.why = std::string("libnccl.so.2 not loadable: ") + (e ? e : "?");
      return a;
    }
    auto sym = [&](const char* name) { return dlsym(h, name); };
    a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(sym("ncclGetUniqueId"));
    a.CommInitRank = reinterpret_cast<decltype(a.CommInitRank)>(sym("ncclCommInitRank"));
    a.AllGather = reinterpret_cast<decltype(a.AllGather)>(sym("ncclAllGather"));
    a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(sym("ncclCommDestroy"));
    a.CommAbort = reinterpret_cast<decltype(a.CommAbort)>(sym("ncclCommAbort"));
    a.CommGetAsyncError =
        reinterpret_cast<decltype(a.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
    a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(sym("ncclGetErrorString"));
    a.ok = a.GetUniqueId && a.CommInitRank && a.AllGather && a.CommDestroy && a.CommAbort &&
           a.CommGetAsyncError && a.GetErrorString;
    if (!a.ok) a.why = "libnccl.so.2 lacks a required symbol";
    return a;
  }();
  return api;
}

ouroq_status nccl_fail(ouroq_ctx* ctx, ncclResult_t r, const char* what) {
  return fail(ctx, OUROQ_ERR_NCCL, "%s: %s", what, nccl().GetErrorString(r));
}

void shard_release(ouroq_ctx* ctx) {
  // The communicator goes first: aborting it ends any collective still
  // waiting on a peer, so the frees below (which synchronise the device)
  // cannot block on it. A peer-store gather ends by itself (bounded wait).
  if (ctx->comm) {
    ncclComm_t c = static_cast<ncclComm_t>(ctx->comm);
    if (ctx->comm_failed)
      nccl().CommAbort(c);
    else
      nccl().CommDestroy(c);
    ctx->comm = nullptr;
  }
  if (ctx->landing) cudaDeviceSynchronize();
  for (int g = 0; g < kShardMaxRanks; ++g) {
    if (ctx->peer_ptr[g] && ctx->peer_ptr[g] != ctx->landing) cudaIpcCloseMemHandle(ctx->peer_ptr[g]);
    ctx->peer_ptr[g] = nullptr;
  }
  cudaFree(ctx->landing);
  ctx->landing = nullptr;
  ctx->landing_words = 0;
  cudaFree(ctx->shard_ctr);
  ctx->shard_ctr = nullptr;
  cudaFree(ctx->gather);
  ctx->gather = nullptr;
  ctx->gather_cap = 0;
  ctx->shard_world = 1;
  ctx->shard_rank = 0;
  ctx->comm_failed = false;
}

// Wait for `s` with a bound, watching the communicator for asynchronous
// errors. On expiry or an NCCL error the group is marked failed.
ouroq_status stream_wait_bounded(ouroq_ctx* ctx, cudaStream_t s, int timeout_ms) {
  const ncclComm_t comm = static_cast<ncclComm_t>(ctx->comm);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess) return OUROQ_OK;
    if (q != cudaErrorNotReady) return cuda_fail(ctx, q, "stream query");
    ncclResult_t ar = ncclSuccess;
    if (comm && nccl().CommGetAsyncError(comm, &ar) == ncclSuccess && ar != ncclSuccess &&
        ar != ncclInProgress) {
      ctx->comm_failed = true;
      return nccl_fail(ctx, ar, "shard group");
    }
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0)
                        .count();
    if (timeout_ms >= 0 && ms > timeout_ms) {
      ctx->comm_failed = true;  // the group is aborted, not destroyed, on release
      return fail(ctx, OUROQ_ERR_TIMEOUT, "sharded work not done after %d ms", timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// Bound of the set-up exchange (landing buffer handles) between ranks.
constexpr int kShardSetupTimeoutMs = 60000;

// (Re)allocate this rank's landing buffer for `words` per parity and open
// every peer's through CUDA IPC. Collective: every rank reaches it on the same
// call (all ranks make the same sequence of sharded calls with the same sizes).
ouroq_status ensure_landing(ouroq_ctx* ctx, size_t words, cudaStream_t s) {
  if (words <= ctx->landing_words) return OUROQ_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  CU(ctx, cudaStreamIsCapturing(s, &cs), "capture query");
  if (cs != cudaStreamCaptureStatusNone)
    return fail(ctx, OUROQ_ERR_UNSUPPORTED,
                "the first sharded call of a given size must come before stream capture");
  const int G = ctx->shard_world, me = ctx->shard_rank;
  CU(ctx, cudaDeviceSynchronize(), "landing sync");
  for (int g = 0; g < kShardMaxRanks; ++g) {
    if (ctx->peer_ptr[g] && ctx->peer_ptr[g] != ctx->landing) cudaIpcCloseMemHandle(ctx->peer_ptr[g]);
    ctx->peer_ptr[g] = nullptr;
  }
  unsigned long long* old = ctx->landing;
  ctx->landing = nullptr;
  ctx->landing_words = 0;
  const size_t bytes = 2 * words * sizeof(unsigned long long);
  unsigned long long* buf = nullptr;
  CU(ctx, cudaMalloc(reinterpret_cast<void**>(&buf), bytes), "landing alloc");
  // zeroed in stream order before the exchange: peers store here only after it
  cudaError_t e = cudaMemsetAsync(buf, 0, bytes, s);
  cudaIpcMemHandle_t mine;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&mine, buf);
  uint8_t* dh = nullptr;
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&dh), hb * G);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dh + hb * me, &mine, hb, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) {
    cudaFree(dh);
    cudaFree(buf);
    cudaFree(old);
    return cuda_fail(ctx, e, "landing set-up");
  }
  const ncclResult_t nr = nccl().AllGather(dh + hb * me, dh, hb, ncclUint8,
                                           static_cast<ncclComm_t>(ctx->comm), s);
  if (nr != ncclSuccess) {
    ctx->comm_failed = true;
    return nccl_fail(ctx, nr, "landing handle exchange");  // freed with the group
  }
  const ouroq_status ws = stream_wait_bounded(ctx, s, kShardSetupTimeoutMs);
  if (ws != OUROQ_OK) return ws;  // buffers stay allocated until the group is released
  std::vector<cudaIpcMemHandle_t> all(G);
  e = cudaMemcpy(all.data(), dh, hb * G, cudaMemcpyDeviceToHost);
  cudaFree(dh);
  cudaFree(old);  // every peer closed its mapping of it before joining the exchange above
  if (e != cudaSuccess) {
    cudaFree(buf);
    return cuda_fail(ctx, e, "landing handle exchange");
  }
  for (int g = 0; g < G; ++g) {
    if (g == me) {
      ctx->peer_ptr[g] = buf;
      continue;
    }
    void* p = nullptr;
    e = cudaIpcOpenMemHandle(&p, all[g], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int h = 0; h < g; ++h)
        if (h != me && ctx->peer_ptr[h]) cudaIpcCloseMemHandle(ctx->peer_ptr[h]);
      for (int h = 0; h < kShardMaxRanks; ++h) ctx->peer_ptr[h] = nullptr;
      cudaFree(buf);
      ctx->comm_failed = true;  // the peers hold a mapping of nothing usable
      return cuda_fail(ctx, e, "open peer landing buffer");
    }
    ctx->peer_ptr[g] = static_cast<unsigned long long*>(p);
  }
  ctx->landing = buf;
  ctx->landing_words = words;
  return OUROQ_OK;
}

ouroq_status shard_rows_impl(ouroq_ctx* ctx, int M, int world, int rank, int* row0, int* rows) {
  if (world < 1 || rank < 0 || rank >= world)
    return fail(ctx, OUROQ_ERR_BAD_ARG, "rank %d of world %d", rank, world);
  if (M <= 0 || M % world)
    return fail(ctx, OUROQ_ERR_BAD_SHAPE, "M=%d rows do not split evenly over %d ranks", M, world);
  *rows = M / world;
  *row0 = rank * *rows;
  return OUROQ_OK;
}

}  // namespace

extern "C" {

int ouroq_abi_version(void) { return OUROQ_ABI_VERSION; }

const char* ouroq_status_string(ouroq_status s) {
  switch (s) {
    case OUROQ_OK: return "ok";
    case OUROQ_ERR_BAD_SHAPE: return "bad shape";
    case OUROQ_ERR_BAD_ALIGN: return "bad alignment";
    case OUROQ_ERR_CUDA: return "cuda error";
    case OUROQ_ERR_NCCL: return "nccl error";
    case OUROQ_ERR_TIMEOUT: return "timeout";
    case OUROQ_ERR_UNSUPPORTED: return "unsupported";
    case OUROQ_ERR_BAD_ARG: return "bad argument";
    case OUROQ_ERR_NO_DEVICE: return "no device";
    case OUROQ_ERR_OOM: return "out of memory";
  }
  return "unknown status";
}

ouroq_status ouroq_ctx_create(int device, ouroq_ctx** out) {
  if (!out) return OUROQ_ERR_BAD_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return OUROQ_ERR_NO_DEVICE;
  if (device < 0 || device >= n) return OUROQ_ERR_NO_DEVICE;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return OUROQ_ERR_NO_DEVICE;
  if (prop.major != 10) return OUROQ_ERR_NO_DEVICE;  // built for sm_100a only
  ouroq_ctx* ctx = new (std::nothrow) ouroq_ctx;
  if (!ctx) return OUROQ_ERR_OOM;
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  ctx->smem_optin = (int)prop.sharedMemPerBlockOptin;
  DeviceGuard g(device);
  if (cudaMalloc(reinterpret_cast<void**>(&ctx->d_status), sizeof(unsigned)) != cudaSuccess ||
      cudaMemset(ctx->d_status, 0, sizeof(unsigned)) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ctx->host_stream, cudaStreamNonBlocking) != cudaSuccess) {
    if (ctx->d_status) cudaFree(ctx->d_status);
    delete ctx;
    return OUROQ_ERR_CUDA;
  }
  *out = ctx;
  return OUROQ_OK;
}

ouroq_status ouroq_ctx_destroy(ouroq_ctx* ctx) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  DeviceGuard g(ctx->device);
  cudaStreamSynchronize(ctx->host_stream);
  cudaStreamDestroy(ctx->host_stream);
  cudaFree(ctx->d_status);
  cudaFree(ctx->q_scratch);
  cudaFree(ctx->s_scratch);
  cudaFree(ctx->x_stage);
  cudaFree(ctx->y_stage);
  cudaFree(ctx->sign_stage);
  cudaFreeHost(ctx->hx_stage);
  cudaFreeHost(ctx->hy_stage);
  cudaFree(ctx->rot_scratch);
  cudaFree(ctx->attn_part);
  cudaFree(ctx->attn_ctr);
  cudaFree(ctx->norm_scratch);
  cudaFree(ctx->head_key);
  shard_release(ctx);
  delete ctx;
  return OUROQ_OK;
}

const char* ouroq_last_error(const ouroq_ctx* ctx) { return ctx ? ctx->err.c_str() : ""; }

uint64_t ouroq_launch_count(const ouroq_ctx* ctx) { return ctx ? ctx->launches : 0; }

ouroq_status ouroq_set_pdl(ouroq_ctx* ctx, int enable) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  ctx->pdl = enable != 0;
  return OUROQ_OK;
}

ouroq_status ouroq_set_prefetch(ouroq_ctx* ctx, int n, const ouroq_weight* const* w) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (n < 0 || (n > 0 && !w)) return fail(ctx, OUROQ_ERR_BAD_ARG, "bad prefetch list");
  ctx->prefetch.clear();
  // whole 16-byte units only (a hint: a ragged tail is left out, never overrun)
  auto add = [&](const void* p, size_t bytes) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    bytes &= ~size_t{15};
    while (bytes > 0) {
      const size_t n1 = bytes < 0x40000000u ? bytes : 0x40000000u;
      ctx->prefetch.emplace_back(b, (uint32_t)n1);
      b += n1;
      bytes -= n1;
    }
  };
  for (int i = 0; i < n; ++i) {
    if (!w[i]) return fail(ctx, OUROQ_ERR_BAD_ARG, "null weight %d in the prefetch list", i);
    size_t wb = w[i]->bytes;
    if (w[i]->scales) {
      const size_t sb = tiled_scale_bytes(w[i]->M, w[i]->K);
      wb -= sb;
      add(w[i]->scales, sb);
    }
    add(w[i]->w, wb);
  }
  return OUROQ_OK;
}

ouroq_status ouroq_ptr_kind(const void* p, int* kind, int* device) {
  if (!p || !kind) return OUROQ_ERR_BAD_ARG;
  cudaPointerAttributes a{};
  const cudaError_t e = cudaPointerGetAttributes(&a, p);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();  // not a pointer CUDA knows: ordinary host memory
    *kind = OUROQ_PTR_HOST;
    if (device) *device = -1;
    return OUROQ_OK;
  }
  *kind = a.type == cudaMemoryTypeDevice    ? OUROQ_PTR_DEVICE
          : a.type == cudaMemoryTypeManaged ? OUROQ_PTR_MANAGED
                                            : OUROQ_PTR_HOST;
  if (device) *device = a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged ? a.device : -1;
  return OUROQ_OK;
}

ouroq_status ouroq_check_device(ouroq_ctx* ctx) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  DeviceGuard g(ctx->device);
  CU(ctx, cudaDeviceSynchronize(), "device sync");
  unsigned v = 0;
  CU(ctx, cudaMemcpy(&v, ctx->d_status, sizeof v, cudaMemcpyDeviceToHost), "status read");
  if (v != 0) {
    CU(ctx, cudaMemset(ctx->d_status, 0, sizeof v), "status clear");
    switch (v) {
      case kDevBadTile:
        return fail(ctx, OUROQ_ERR_CUDA, "tile index outside the job table (code %u)", v);
      case kDevBadPosition:
        return fail(ctx, OUROQ_ERR_BAD_SHAPE, "decode position outside the KV cache (code %u)", v);
      case kDevPeerTimeout:
        return fail(ctx, OUROQ_ERR_TIMEOUT, "peer rows did not arrive in time (code %u)", v);
      default:
        return fail(ctx, OUROQ_ERR_TIMEOUT, "device wait expired (code %u)", v);
    }
  }
  return OUROQ_OK;
}

ouroq_status ouroq_weight_upload(ouroq_ctx* ctx, ouroq_format fmt, const void* packed, int M, int K,
                                 const void* scales, float w_scale, ouroq_weight** out) {
  return upload_impl(ctx, fmt, packed, M, K, scales, w_scale, out, false);
}

ouroq_status ouroq_weight_upload_device(ouroq_ctx* ctx, ouroq_format fmt, const void* packed_dev,
                                        int M, int K, const void* scales_dev, float w_scale,
                                        ouroq_weight** out) {
  return upload_impl(ctx, fmt, packed_dev, M, K, scales_dev, w_scale, out, true);
}

ouroq_status ouroq_weight_free(ouroq_ctx* ctx, ouroq_weight* w) {
  if (!ctx || !w) return fail(ctx, OUROQ_ERR_BAD_ARG, "null argument");
  DeviceGuard g(ctx->device);
  cudaFree(w->w);
  cudaFree(w->scales);
  delete w;
  return OUROQ_OK;
}

ouroq_status ouroq_weight_info(const ouroq_weight* w, int* fmt, int* M, int* K,
                               size_t* device_bytes) {
  if (!w) return OUROQ_ERR_BAD_ARG;
  if (fmt) *fmt = w->fmt;
  if (M) *M = w->M;
  if (K) *K = w->K;
  if (device_bytes) *device_bytes = w->bytes;
  return OUROQ_OK;
}

ouroq_status ouroq_quantize_act(ouroq_ctx* ctx, const float* x, int B, int K, const float* signs,
                                int hadamard_block, int8_t* q, float* s_x, void* stream) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (B > 0 && (!x || !q || !s_x)) return fail(ctx, OUROQ_ERR_BAD_ARG, "null buffer");
  ouroq_status st = check_quant_args(ctx, B, K, hadamard_block);
  if (st != OUROQ_OK) return st;
  if (!aligned16(x) || !aligned16(q)) return fail(ctx, OUROQ_ERR_BAD_ALIGN, "x/q not 16-byte aligned");
  DeviceGuard g(ctx->device);
  return quantize_impl(ctx, x, B, K, signs, hadamard_block, q, s_x,
                       static_cast<cudaStream_t>(stream));
}

ouroq_status ouroq_quantize_group(ouroq_ctx* ctx, int n, const float* const* x, const int* K,
                                  const float* const* signs, const int* blocks, int B,
                                  int8_t* const* q, float* const* s_x, void* stream) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (n < 0 || n > kMaxQuantJobs)
    return fail(ctx, OUROQ_ERR_BAD_SHAPE, "group size %d (max %d)", n, kMaxQuantJobs);
  if (B < 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d", B);
  if (n == 0 || B == 0) return OUROQ_OK;
  if (!x || !K || !q || !s_x) return fail(ctx, OUROQ_ERR_BAD_ARG, "null array");
  QuantLaunch L{};
  L.njobs = n;
  L.B = B;
  for (int i = 0; i < n; ++i) {
    const int blk = blocks ? blocks[i] : 0;
    ouroq_status st = check_quant_args(ctx, B, K[i], blk);
    if (st != OUROQ_OK) return st;
    if (!x[i] || !q[i] || !s_x[i]) return fail(ctx, OUROQ_ERR_BAD_ARG, "null entry %d", i);
    if (!aligned16(x[i]) || !aligned16(q[i]))
      return fail(ctx, OUROQ_ERR_BAD_ALIGN, "x[%d]/q[%d] not 16-byte aligned", i, i);
    QuantJob& J = L.jobs[i];
    J.x = x[i];
    J.signs = signs ? signs[i] : nullptr;
    J.q = q[i];
    J.s_x = s_x[i];
    J.x_rot = nullptr;
    J.K = K[i];
    J.had_block = blk;
    J.had_scale = blk ? 1.0f / std::sqrt((float)blk) : 1.0f;
  }
  DeviceGuard g(ctx->device);
  CU(ctx, launch_quantize(L, static_cast<cudaStream_t>(stream), ctx->pdl), "quantize launch");
  ctx->launches++;
  return OUROQ_OK;
}

ouroq_status ouroq_rotate(ouroq_ctx* ctx, const float* x, float* out, int B, int K,
                          const float* signs, int block, int inverse, void* stream) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (B > 0 && (!x || !out)) return fail(ctx, OUROQ_ERR_BAD_ARG, "null buffer");
  if (!valid_block(block)) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "block %d", block);
  ouroq_status st = check_quant_args(ctx, B, K, block);
  if (st != OUROQ_OK) return st;
  DeviceGuard g(ctx->device);
  const float scale = 1.0f / std::sqrt((float)block);
  CU(ctx, launch_rotate(x, out, signs, B, K, block, scale, inverse, static_cast<cudaStream_t>(stream)),
     "rotate launch");
  if (B > 0) ctx->launches++;
  return OUROQ_OK;
}

ouroq_status ouroq_gemm(ouroq_ctx* ctx, const ouroq_weight* w, const int8_t* q, const float* s_x,
                        int B, float* y, int32_t* acc_debug, void* stream) {
  if (!ctx || !w) return fail(ctx, OUROQ_ERR_BAD_ARG, "null handle");
  if (B < 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d", B);
  if (B == 0) return OUROQ_OK;
  if (!q || !s_x || !y) return fail(ctx, OUROQ_ERR_BAD_ARG, "null buffer");
  if (is_ref_format(w->fmt))
    return fail(ctx, OUROQ_ERR_UNSUPPORTED, "PTQ1_0 / TQ1_0 weights take fp32 activations");
  if (!aligned16(q)) return fail(ctx, OUROQ_ERR_BAD_ALIGN, "q not 16-byte aligned");
  DeviceGuard g(ctx->device);
  return gemm_impl(ctx, w, q, s_x, B, y, acc_debug, static_cast<cudaStream_t>(stream));
}

ouroq_status ouroq_gemm_group(ouroq_ctx* ctx, int n, const ouroq_weight* const* w,
                              const int8_t* const* q, const float* const* s_x, int B,
                              float* const* y, void* stream) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (n < 0 || n > kMaxGemvJobs) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "group size %d (max %d)", n, kMaxGemvJobs);
  if (B < 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d", B);
  if (n == 0 || B == 0) return OUROQ_OK;
  if (!w || !q || !s_x || !y) return fail(ctx, OUROQ_ERR_BAD_ARG, "null array");
  GemvLaunch L{};
  L.njobs = n;
  L.B = B;
  for (int i = 0; i < n; ++i) {
    if (!w[i] || !q[i] || !s_x[i] || !y[i]) return fail(ctx, OUROQ_ERR_BAD_ARG, "null entry %d", i);
    if (is_ref_format(w[i]->fmt))
      return fail(ctx, OUROQ_ERR_UNSUPPORTED, "grouped calls take TERNARY2 / SIGN1G128 weights");
    if (w[i]->fmt != w[0]->fmt) return fail(ctx, OUROQ_ERR_UNSUPPORTED, "mixed formats in a group");
    if (B <= kGemvMaxB && (size_t)B * w[i]->K > kGemvMaxXBytes)
      return fail(ctx, OUROQ_ERR_UNSUPPORTED, "B*K=%zu exceeds the grouped GEMV limit",
                  (size_t)B * w[i]->K);
    if (!aligned16(q[i])) return fail(ctx, OUROQ_ERR_BAD_ALIGN, "q[%d] not 16-byte aligned", i);
    L.jobs[i] = make_job(w[i], q[i], s_x[i], y[i], nullptr);
  }
  L.fmt = w[0]->fmt == OUROQ_FMT_TERNARY2 ? kTern2 : kSign1;
  DeviceGuard g(ctx->device);
  return group_product(ctx, L, w, n, B, static_cast<cudaStream_t>(stream));
}

ouroq_status ouroq_gemm_group_f32act(ouroq_ctx* ctx, int n, const ouroq_weight* const* w,
                                     const float* const* x, int B, const float* const* signs,
                                     const int* blocks, float* const* y, void* stream) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (n < 0 || n > kMaxGemvJobs)
    return fail(ctx, OUROQ_ERR_BAD_SHAPE, "group size %d (max %d)", n, kMaxGemvJobs);
  if (B < 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d", B);
  if (n == 0 || B == 0) return OUROQ_OK;
  if (!w || !x || !y) return fail(ctx, OUROQ_ERR_BAD_ARG, "null array");
  GemvLaunch L{};
  L.njobs = n;
  L.B = B;
  L.fused = 1;
  int maxK = 0;
  for (int i = 0; i < n; ++i) {
    if (!w[i] || !x[i] || !y[i]) return fail(ctx, OUROQ_ERR_BAD_ARG, "null entry %d", i);
    if (is_ref_format(w[i]->fmt))
      return fail(ctx, OUROQ_ERR_UNSUPPORTED, "grouped calls take TERNARY2 / SIGN1G128 weights");
    if (w[i]->fmt != w[0]->fmt) return fail(ctx, OUROQ_ERR_UNSUPPORTED, "mixed formats in a group");
    const int blk = blocks ? blocks[i] : 0;
    ouroq_status st = check_quant_args(ctx, B, w[i]->K, blk);
    if (st != OUROQ_OK) return st;
    if (blk != 0 && (blk < 32 || blk > 128))
      return fail(ctx, OUROQ_ERR_UNSUPPORTED, "fused rotation needs a hadamard block of 32..128");
    if (blk != (blocks ? blocks[0] : 0))
      return fail(ctx, OUROQ_ERR_UNSUPPORTED, "all entries of a fused group share one hadamard block");
    if (!aligned16(x[i])) return fail(ctx, OUROQ_ERR_BAD_ALIGN, "x[%d] not 16-byte aligned", i);
    L.jobs[i] = make_job(w[i], nullptr, nullptr, y[i], nullptr);
    L.jobs[i].xf = x[i];
    L.jobs[i].signs = signs ? signs[i] : nullptr;
    L.jobs[i].had_block = blk;
    L.jobs[i].had_scale = blk ? 1.0f / std::sqrt((float)blk) : 1.0f;
    maxK = w[i]->K > maxK ? w[i]->K : maxK;
  }
  L.fmt = w[0]->fmt == OUROQ_FMT_TERNARY2 ? kTern2 : kSign1;
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // ternary without rotation, up to kStreamMaxB tokens: one stream-GEMV launch
  if (B <= kGemvMaxB && stream_takes(ctx, L)) return run_gemv(ctx, L, s);
  if (B <= kGemvMaxB && !gemv_fits(ctx, L))
    return fail(ctx, OUROQ_ERR_UNSUPPORTED,
                "B=%d, K=%d: activations do not fit the fused GEMV (use quantize + gemm_group)",
                B, maxK);
  if (B <= kFusedMaxB) return run_gemv(ctx, L, s);
  // Larger batches off the stream kernel: every CTA would quantise all tokens
  // of its matrices again, so quantise each distinct activation set once (one
  // launch) into scratch and run the grouped GEMV on the int8 codes.
  QuantLaunch Q{};
  Q.B = B;
  int set_of[kMaxGemvJobs];
  size_t qoff[kMaxQuantJobs], soff[kMaxQuantJobs], qtot = 0, stot = 0;
  for (int i = 0; i < n; ++i) {
    int k = 0;
    while (k < Q.njobs && !(Q.jobs[k].x == x[i] && Q.jobs[k].signs == L.jobs[i].signs &&
                            Q.jobs[k].had_block == L.jobs[i].had_block && Q.jobs[k].K == w[i]->K))
      ++k;
    if (k == Q.njobs) {
      QuantJob& J = Q.jobs[Q.njobs++];
      J.x = x[i];
      J.signs = L.jobs[i].signs;
      J.x_rot = nullptr;
      J.K = w[i]->K;
      J.had_block = L.jobs[i].had_block;
      J.had_scale = L.jobs[i].had_scale;
      qoff[k] = qtot;
      soff[k] = stot;
      qtot += ((size_t)B * w[i]->K + 15) / 16 * 16;
      stot += (size_t)B;
    }
    set_of[i] = k;
  }
  ouroq_status st = grow(ctx, ctx->q_scratch, ctx->q_cap, qtot, "q scratch");
  if (st != OUROQ_OK) return st;
  st = grow(ctx, ctx->s_scratch, ctx->s_cap, stot, "s scratch");
  if (st != OUROQ_OK) return st;
  for (int k = 0; k < Q.njobs; ++k) {
    Q.jobs[k].q = ctx->q_scratch + qoff[k];
    Q.jobs[k].s_x = ctx->s_scratch + soff[k];
  }
  CU(ctx, launch_quantize(Q, s, ctx->pdl), "quantize launch");
  ctx->launches++;
  L.fused = 0;
  for (int i = 0; i < n; ++i) {
    L.jobs[i].q = Q.jobs[set_of[i]].q;
    L.jobs[i].s_x = Q.jobs[set_of[i]].s_x;
    L.jobs[i].xf = nullptr;
  }
  return group_product(ctx, L, w, n, B, s);
}

// PTQ1_0 order of an fp32-activation product: kAuto = matvec_tl1's for one
// token, matmul_tl1's K-column order for several (what matvec_q / matmul_q
// give); the host mirrors pin it to the operator they mirror.
enum class Tl1Order { kAuto, kMatvec, kColumns };

static ouroq_status f32act_impl(ouroq_ctx* ctx, const ouroq_weight* w, const float* x, int B,
                                const float* signs, int hadamard_block, float* y, void* stream,
                                Tl1Order order) {
  if (!ctx || !w) return fail(ctx, OUROQ_ERR_BAD_ARG, "null handle");
  if (B < 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d", B);
  if (B == 0) return OUROQ_OK;
  if (!x || !y) return fail(ctx, OUROQ_ERR_BAD_ARG, "null buffer");
  // 16-bit weights read x element by element and need neither the
  // quantiser's shape rules nor alignment, unless x is rotated first
  const bool plain_half = is_half_format(w->fmt) && hadamard_block == 0;
  ouroq_status st = plain_half ? OUROQ_OK : check_quant_args(ctx, B, w->K, hadamard_block);
  if (st != OUROQ_OK) return st;
  if (!plain_half && !aligned16(x)) return fail(ctx, OUROQ_ERR_BAD_ALIGN, "x not 16-byte aligned");
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (is_ref_format(w->fmt)) {
    // the reference rotates x first (Qwen35Stage::wh, qwen35.rs:683-692), then matvec_q
    const float* xin = x;
    if (hadamard_block) {
      st = grow(ctx, ctx->rot_scratch, ctx->rot_cap, (size_t)B * w->K, "rotation scratch");
      if (st != OUROQ_OK) return st;
      CU(ctx,
         launch_rotate(x, ctx->rot_scratch, signs, B, w->K, hadamard_block,
                       1.0f / std::sqrt((float)hadamard_block), 0, s),
         "rotate launch");
      ctx->launches++;
      xin = ctx->rot_scratch;
    }
    const bool columns = order == Tl1Order::kColumns || (order == Tl1Order::kAuto && B > 1);
    return ref_matvec(ctx, w, xin, B, y, s, columns);
  }
  const int dfmt = w->fmt == OUROQ_FMT_TERNARY2 ? kTern2 : kSign1;
  if (B <= kGemvMaxB && (hadamard_block == 0 || (hadamard_block >= 32 && hadamard_block <= 128))) {
    // one launch: rotate + quantise in the GEMV prologue (up to kFusedMaxB
    // tokens; larger batches only on the stream kernel, which quantises each
    // input once per CTA or cluster, else they quantise once, below)
    GemvLaunch L{};
    L.njobs = 1;
    L.B = B;
    L.fmt = dfmt;
    L.fused = 1;
    L.jobs[0] = make_job(w, nullptr, nullptr, y, nullptr);
    L.jobs[0].xf = x;
    L.jobs[0].signs = signs;
    L.jobs[0].had_block = hadamard_block;
    L.jobs[0].had_scale = hadamard_block ? 1.0f / std::sqrt((float)hadamard_block) : 1.0f;
    if (stream_takes(ctx, L) || (B <= kFusedMaxB && gemv_fits(ctx, L))) return run_gemv(ctx, L, s);
  }
  st = grow(ctx, ctx->q_scratch, ctx->q_cap, (size_t)B * w->K, "q scratch");
  if (st != OUROQ_OK) return st;
  st = grow(ctx, ctx->s_scratch, ctx->s_cap, (size_t)B, "s scratch");
  if (st != OUROQ_OK) return st;
  st = quantize_impl(ctx, x, B, w->K, signs, hadamard_block, ctx->q_scratch, ctx->s_scratch, s);
  if (st != OUROQ_OK) return st;
  return gemm_impl(ctx, w, ctx->q_scratch, ctx->s_scratch, B, y, nullptr, s);
}

ouroq_status ouroq_gemm_f32act(ouroq_ctx* ctx, const ouroq_weight* w, const float* x, int B,
                               const float* signs, int hadamard_block, float* y, void* stream) {
  return f32act_impl(ctx, w, x, B, signs, hadamard_block, y, stream, Tl1Order::kAuto);
}

// Address of the fixed scratch on each device, looked up the first time a call
// runs there (with that device current) and reused afterwards.
static std::mutex g_noalloc_mu;
static void* g_noalloc_addr[64] = {};

static ouroq_status noalloc_scratch(ouroq_ctx* ctx, uint8_t** out) {
  if (ctx->device < 0 || ctx->device >= 64)
    return fail(ctx, OUROQ_ERR_UNSUPPORTED, "device %d: fixed scratch covers devices 0..63",
                ctx->device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[ctx->device]) {
    void* p = nullptr;
    CU(ctx, noalloc_scratch_address(&p), "fixed scratch address");
    g_noalloc_addr[ctx->device] = p;
  }
  *out = static_cast<uint8_t*>(g_noalloc_addr[ctx->device]);
  return OUROQ_OK;
}

// Same result as ouroq_gemm_f32act, for callers that must not allocate device
// memory mid-run; the activation codes go to the library's fixed per-device
// scratch instead of a buffer grown with cudaMalloc / cudaFree.
ouroq_status ouroq_gemm_f32act_noalloc(ouroq_ctx* ctx, const ouroq_weight* w, const float* x,
                                       int B, const float* signs, int hadamard_block, float* y,
                                       void* stream) {
  if (!ctx || !w) return fail(ctx, OUROQ_ERR_BAD_ARG, "null handle");
  if (B < 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d", B);
  if (B == 0) return OUROQ_OK;
  if (!x || !y) return fail(ctx, OUROQ_ERR_BAD_ARG, "null buffer");
  if (is_half_format(w->fmt) && hadamard_block == 0) {
    DeviceGuard g(ctx->device);  // no quantisation, no scratch
    return ref_matvec(ctx, w, x, B, y, static_cast<cudaStream_t>(stream), false);
  }
  ouroq_status st = check_quant_args(ctx, B, w->K, hadamard_block);
  if (st != OUROQ_OK) return st;
  if (!aligned16(x)) return fail(ctx, OUROQ_ERR_BAD_ALIGN, "x not 16-byte aligned");
  DeviceGuard g(ctx->device);
  if (is_ref_format(w->fmt)) {
    // no quantisation, so no scratch and no batch limit; the rotation would
    // need a buffer
    if (hadamard_block)
      return fail(ctx, OUROQ_ERR_UNSUPPORTED,
                  "PTQ1_0 / TQ1_0 with a rotation needs scratch: rotate first, or use ouroq_gemm_f32act");
    return ref_matvec(ctx, w, x, B, y, static_cast<cudaStream_t>(stream), B > 1);
  }
  if (B > kNoAllocMaxTokens || (size_t)B * w->K > kNoAllocQBytes)
    return fail(ctx, OUROQ_ERR_BAD_SHAPE,
                "B=%d, K=%d: the fixed scratch holds at most %d tokens and B*K <= %zu "
                "(split the batch, or use ouroq_gemm_f32act)",
                B, w->K, kNoAllocMaxTokens, kNoAllocQBytes);
  uint8_t* scratch = nullptr;
  st = noalloc_scratch(ctx, &scratch);
  if (st != OUROQ_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (B <= kGemvMaxB && (hadamard_block == 0 || (hadamard_block >= 32 && hadamard_block <= 128))) {
    // one launch, no scratch: rotate + quantise in the GEMV prologue (the
    // batches ouroq_gemm_f32act fuses; larger ones quantise once, below)
    GemvLaunch L{};
    L.njobs = 1;
    L.B = B;
    L.fmt = w->fmt == OUROQ_FMT_TERNARY2 ? kTern2 : kSign1;
    L.fused = 1;
    L.jobs[0] = make_job(w, nullptr, nullptr, y, nullptr);
    L.jobs[0].xf = x;
    L.jobs[0].signs = signs;
    L.jobs[0].had_block = hadamard_block;
    L.jobs[0].had_scale = hadamard_block ? 1.0f / std::sqrt((float)hadamard_block) : 1.0f;
    if (stream_takes(ctx, L) || (B <= kFusedMaxB && gemv_fits(ctx, L))) return run_gemv(ctx, L, s);
  }
  int8_t* q = reinterpret_cast<int8_t*>(scratch);
  float* s_x = reinterpret_cast<float*>(scratch + kNoAllocQBytes);
  st = quantize_impl(ctx, x, B, w->K, signs, hadamard_block, q, s_x, s);
  if (st != OUROQ_OK) return st;
  return gemm_impl(ctx, w, q, s_x, B, y, nullptr, s);
}

static bool host_mapped(const void* p, size_t bytes);

// The host-buffer mirrors: x staged in, the product, y copied back (or, for
// the quantised formats at k <= 8, whose GEMV stores y with plain stores,
// stored straight into a page-locked mapped y_host), synchronous.
static ouroq_status host_product(ouroq_ctx* ctx, const ouroq_weight* w, const float* x_host, int k,
                                 float* y_host, Tl1Order order) {
  if (!ctx || !w) return fail(ctx, OUROQ_ERR_BAD_ARG, "null handle");
  if (k < 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "k=%d", k);
  if (k == 0) return OUROQ_OK;
  if (!x_host || !y_host) return fail(ctx, OUROQ_ERR_BAD_ARG, "null buffer");
  DeviceGuard g(ctx->device);
  ouroq_status st = grow(ctx, ctx->x_stage, ctx->x_cap, (size_t)k * w->K, "x stage");
  if (st != OUROQ_OK) return st;
  const bool y_direct = !is_ref_format(w->fmt) && !is_half_format(w->fmt) && k <= kGemvMaxB &&
                        host_mapped(y_host, (size_t)k * w->M * 4);
  if (!y_direct) {
    st = grow(ctx, ctx->y_stage, ctx->y_cap, (size_t)k * w->M, "y stage");
    if (st != OUROQ_OK) return st;
  }
  cudaStream_t s = ctx->host_stream;
  CU(ctx, cudaMemcpyAsync(ctx->x_stage, x_host, (size_t)k * w->K * 4, cudaMemcpyHostToDevice, s),
     "x upload");
  st = f32act_impl(ctx, w, ctx->x_stage, k, nullptr, 0, y_direct ? y_host : ctx->y_stage, s, order);
  if (st != OUROQ_OK) return st;
  if (!y_direct)
    CU(ctx, cudaMemcpyAsync(y_host, ctx->y_stage, (size_t)k * w->M * 4, cudaMemcpyDeviceToHost, s),
       "y download");
  CU(ctx, cudaStreamSynchronize(s), "stream sync");
  return OUROQ_OK;
}

// ops::matmul_q: PTQ1_0 in matmul_tl1's K-column order for every k, k = 1 included
ouroq_status ouroq_matmul_q(ouroq_ctx* ctx, const ouroq_weight* w, const float* x_host, int k,
                            float* y_host) {
  return host_product(ctx, w, x_host, k, y_host, Tl1Order::kColumns);
}

// ops::matvec_q: PTQ1_0 in matvec_tl1's order
ouroq_status ouroq_matvec_q(ouroq_ctx* ctx, const ouroq_weight* w, const float* x_host,
                            float* y_host) {
  return host_product(ctx, w, x_host, 1, y_host, Tl1Order::kMatvec);
}

// Page-locked host memory (cudaHostAlloc / cudaHostRegister): DMA-able as it is.
static bool host_pinned(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();  // clear the error an unknown pointer leaves
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// cuPointerGetAttributes, resolved once through the runtime (no libcuda link).
using PointerAttrsFn = CUresult (*)(unsigned int, CUpointer_attribute*, void**, CUdeviceptr);
static PointerAttrsFn pointer_attrs_fn() {
  static PointerAttrsFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuPointerGetAttributes", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return static_cast<PointerAttrsFn>(nullptr);
    }
    return reinterpret_cast<PointerAttrsFn>(p);
  }();
  return fn;
}

// A page-locked host buffer that kernels address at its host address, with
// [p, p + bytes) inside one allocation: a product may store into it directly.
// Any doubt (unknown pointer, a different device address, a range the
// allocation does not cover, a refused query) answers no.
static bool host_mapped(const void* p, size_t bytes) {
  PointerAttrsFn fn = pointer_attrs_fn();
  if (!fn || !p) return false;
  unsigned int type = 0;
  CUdeviceptr dev = 0, start = 0;
  size_t size = 0;
  CUpointer_attribute at[4] = {CU_POINTER_ATTRIBUTE_MEMORY_TYPE, CU_POINTER_ATTRIBUTE_DEVICE_POINTER,
                               CU_POINTER_ATTRIBUTE_RANGE_START_ADDR, CU_POINTER_ATTRIBUTE_RANGE_SIZE};
  void* out[4] = {&type, &dev, &start, &size};
  const CUdeviceptr a = static_cast<CUdeviceptr>(reinterpret_cast<uintptr_t>(p));
  if (fn(4, at, out, a) != CUDA_SUCCESS) return false;
  return type == CU_MEMORYTYPE_HOST && dev == a && size > 0 && start <= a && bytes <= size &&
         a - start <= size - bytes;
}

static ouroq_status grow_pinned(ouroq_ctx* ctx, float*& buf, size_t& cap, size_t n,
                                const char* what) {
  if (n <= cap) return OUROQ_OK;
  if (buf) cudaFreeHost(buf);
  buf = nullptr;
  cap = 0;
  const size_t want = n < 4096 ? 4096 : n;
  cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&buf), want * sizeof(float),
                                cudaHostAllocDefault);
  if (e != cudaSuccess) return cuda_fail(ctx, e, what);
  cap = want;
  return OUROQ_OK;
}

// One host<->device transfer of a host-buffer call: `host` is the caller's
// buffer, `dev_off` the float offset of its slot in the device stage.
struct HostSeg {
  float* host;
  size_t dev_off, n;
  bool pinned;
};

// Issue the copies of `segs` (in stage order) on s: pinned buffers directly,
// pageable ones through the page-locked stage `hstage` (same offsets), and
// runs that sit back to back on both sides as one copy.
static ouroq_status copy_segs(ouroq_ctx* ctx, std::vector<HostSeg>& segs, float* dstage,
                              float* hstage, bool to_device, cudaStream_t s) {
  size_t i = 0;
  while (i < segs.size()) {
    float* h0 = segs[i].pinned ? segs[i].host : hstage + segs[i].dev_off;
    const size_t off0 = segs[i].dev_off;
    size_t n = segs[i].n, j = i + 1;
    while (j < segs.size()) {
      float* hj = segs[j].pinned ? segs[j].host : hstage + segs[j].dev_off;
      if (hj != h0 + n || segs[j].dev_off != off0 + n) break;
      n += segs[j].n;
      ++j;
    }
    if (to_device)
      CU(ctx, cudaMemcpyAsync(dstage + off0, h0, n * 4, cudaMemcpyHostToDevice, s), "x upload");
    else
      CU(ctx, cudaMemcpyAsync(h0, dstage + off0, n * 4, cudaMemcpyDeviceToHost, s), "y download");
    i = j;
  }
  return OUROQ_OK;
}

ouroq_status ouroq_matmul_q_group(ouroq_ctx* ctx, int n, const ouroq_weight* const* w,
                                  const float* const* x_host, int k, float* const* y_host) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (n < 0 || n > kMaxGemvJobs)
    return fail(ctx, OUROQ_ERR_BAD_SHAPE, "group size %d (max %d)", n, kMaxGemvJobs);
  if (k < 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "k=%d", k);
  if (n == 0 || k == 0) return OUROQ_OK;
  if (!w || !x_host || !y_host) return fail(ctx, OUROQ_ERR_BAD_ARG, "null array");
  for (int i = 0; i < n; ++i)
    if (!w[i] || !x_host[i] || !y_host[i]) return fail(ctx, OUROQ_ERR_BAD_ARG, "null entry %d", i);
  DeviceGuard g(ctx->device);
  // distinct inputs (same pointer and width) share one slot of the device stage
  std::vector<HostSeg> xs, ys;
  int slot[kMaxGemvJobs];
  size_t xtot = 0, ytot = 0;
  for (int i = 0; i < n; ++i) {
    int j = 0;
    while (j < i && !(x_host[j] == x_host[i] && w[j]->K == w[i]->K)) ++j;
    if (j < i) {
      slot[i] = slot[j];
    } else {
      slot[i] = (int)xs.size();
      xs.push_back({const_cast<float*>(x_host[i]), xtot, (size_t)k * w[i]->K, false});
      xtot += ((size_t)k * w[i]->K + 3) / 4 * 4;  // slots start 16-byte aligned
    }
    ys.push_back({y_host[i], ytot, (size_t)k * w[i]->M, false});
    ytot += ((size_t)k * w[i]->M + 3) / 4 * 4;
  }
  ouroq_status st = grow(ctx, ctx->x_stage, ctx->x_cap, xtot, "x stage");
  if (st != OUROQ_OK) return st;
  st = grow(ctx, ctx->y_stage, ctx->y_cap, ytot, "y stage");
  if (st != OUROQ_OK) return st;
  bool same_fmt = true;
  for (int i = 0; i < n; ++i) same_fmt &= w[i]->fmt == w[0]->fmt;
  // the quantised formats at small k: one grouped GEMV launch (as
  // ouroq_gemm_group_f32act), whose kernels store y with plain stores; when
  // every output is page-locked and mapped, they store into it directly (no
  // stage, no download)
  const bool grouped =
      same_fmt && !is_ref_format(w[0]->fmt) && !is_half_format(w[0]->fmt) && k <= kGemvMaxB;
  bool y_direct = grouped;
  for (const HostSeg& sg : ys) y_direct = y_direct && host_mapped(sg.host, sg.n * 4);
  bool x_staged = false, y_staged = false;
  for (HostSeg& sg : xs) x_staged |= !(sg.pinned = host_pinned(sg.host));
  if (!y_direct)
    for (HostSeg& sg : ys) y_staged |= !(sg.pinned = host_pinned(sg.host));
  if (x_staged) {
    st = grow_pinned(ctx, ctx->hx_stage, ctx->hx_cap, xtot, "pinned x stage");
    if (st != OUROQ_OK) return st;
    for (const HostSeg& sg : xs)
      if (!sg.pinned) std::memcpy(ctx->hx_stage + sg.dev_off, sg.host, sg.n * 4);
  }
  if (y_staged) {
    st = grow_pinned(ctx, ctx->hy_stage, ctx->hy_cap, ytot, "pinned y stage");
    if (st != OUROQ_OK) return st;
  }
  cudaStream_t s = ctx->host_stream;
  st = copy_segs(ctx, xs, ctx->x_stage, ctx->hx_stage, true, s);
  if (st != OUROQ_OK) return st;
  const float* xd[kMaxGemvJobs];
  float* yd[kMaxGemvJobs];
  for (int i = 0; i < n; ++i) {
    xd[i] = ctx->x_stage + xs[slot[i]].dev_off;
    yd[i] = y_direct ? y_host[i] : ctx->y_stage + ys[i].dev_off;
  }
  bool done = false;
  if (grouped) {
    // UNSUPPORTED is answered before any launch that stores y
    st = ouroq_gemm_group_f32act(ctx, n, w, xd, k, nullptr, nullptr, yd, s);
    if (st == OUROQ_OK) done = true;
    else if (st != OUROQ_ERR_UNSUPPORTED) return st;
  }
  if (!done && y_direct) {  // other routes write the device stage
    y_direct = false;
    for (HostSeg& sg : ys) y_staged |= !(sg.pinned = host_pinned(sg.host));
    if (y_staged) {
      st = grow_pinned(ctx, ctx->hy_stage, ctx->hy_cap, ytot, "pinned y stage");
      if (st != OUROQ_OK) return st;
    }
    for (int i = 0; i < n; ++i) yd[i] = ctx->y_stage + ys[i].dev_off;
  }
  for (int i = 0; i < n && !done; ++i) {
    st = f32act_impl(ctx, w[i], xd[i], k, nullptr, 0, yd[i], s, Tl1Order::kAuto);
    if (st != OUROQ_OK) return st;
  }
  if (!y_direct) {
    st = copy_segs(ctx, ys, ctx->y_stage, ctx->hy_stage, false, s);
    if (st != OUROQ_OK) return st;
  }
  CU(ctx, cudaStreamSynchronize(s), "stream sync");
  if (!y_direct)
    for (const HostSeg& sg : ys)
      if (!sg.pinned) std::memcpy(sg.host, ctx->hy_stage + sg.dev_off, sg.n * 4);
  return OUROQ_OK;
}

static ouroq_status rotate_host(ouroq_ctx* ctx, float* x_host, const float* signs_host, size_t n,
                                size_t block, int inverse) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (n == 0) return OUROQ_OK;
  if (!x_host) return fail(ctx, OUROQ_ERR_BAD_ARG, "null buffer");
  // hadamard.rs:33-37: block must be a power of two and divide the length
  if (!valid_block((int)block) || n % block)
    return fail(ctx, OUROQ_ERR_BAD_SHAPE, "len %zu not multiple of block %zu", n, block);
  // one row per block-aligned segment of at most 32768 elements
  size_t K = n;
  while (K > 32768) K /= 2;
  if (n % K || K % block) K = block;
  const int B = (int)(n / K);
  DeviceGuard g(ctx->device);
  ouroq_status st = grow(ctx, ctx->x_stage, ctx->x_cap, n, "x stage");
  if (st != OUROQ_OK) return st;
  cudaStream_t s = ctx->host_stream;
  CU(ctx, cudaMemcpyAsync(ctx->x_stage, x_host, n * 4, cudaMemcpyHostToDevice, s), "x upload");
  const float* sd = nullptr;
  if (signs_host) {
    st = grow(ctx, ctx->sign_stage, ctx->sign_cap, n, "sign stage");
    if (st != OUROQ_OK) return st;
    CU(ctx, cudaMemcpyAsync(ctx->sign_stage, signs_host, n * 4, cudaMemcpyHostToDevice, s),
       "signs upload");
    sd = ctx->sign_stage;
  }
  // rows of K elements; the sign vector repeats per row only when rows == 1,
  // so for B > 1 pass per-row sign slices by launching row by row.
  const float scale = 1.0f / std::sqrt((float)block);
  for (int b = 0; b < B; ++b) {
    CU(ctx,
       launch_rotate(ctx->x_stage + (size_t)b * K, ctx->x_stage + (size_t)b * K,
                     sd ? sd + (size_t)b * K : nullptr, 1, (int)K, (int)block, scale, inverse, s),
       "rotate launch");
    ctx->launches++;
  }
  CU(ctx, cudaMemcpyAsync(x_host, ctx->x_stage, n * 4, cudaMemcpyDeviceToHost, s), "x download");
  CU(ctx, cudaStreamSynchronize(s), "stream sync");
  return OUROQ_OK;
}

ouroq_status ouroq_rotate_fwd(ouroq_ctx* ctx, float* x_host, const float* signs_host, size_t n,
                              size_t block) {
  return rotate_host(ctx, x_host, signs_host, n, block, 0);
}

ouroq_status ouroq_rotate_inv(ouroq_ctx* ctx, float* x_host, const float* signs_host, size_t n,
                              size_t block) {
  return rotate_host(ctx, x_host, signs_host, n, block, 1);
}

// ---------------------------------------------------------------- row sharding
// Output rows of a large matrix split evenly over the GPUs of one node, one
// process per GPU; an in-place NCCL all-gather over NVLink assembles y on
// every rank. Activations are identical on all ranks and each rank quantises
// them itself (no extra collective).

ouroq_status ouroq_shard_unique_id(void* id_out) {
  if (!id_out) return OUROQ_ERR_BAD_ARG;
  const NcclApi& n = nccl();
  if (!n.ok) return OUROQ_ERR_NCCL;
  ncclUniqueId id;
  if (n.GetUniqueId(&id) != ncclSuccess) return OUROQ_ERR_NCCL;
  std::memcpy(id_out, &id, sizeof id);
  return OUROQ_OK;
}

ouroq_status ouroq_shard_init(ouroq_ctx* ctx, const void* id, int world, int rank) {
  if (!ctx || !id) return fail(ctx, OUROQ_ERR_BAD_ARG, "null argument");
  if (world < 1 || rank < 0 || rank >= world)
    return fail(ctx, OUROQ_ERR_BAD_ARG, "rank %d of world %d", rank, world);
  if (ctx->comm) return fail(ctx, OUROQ_ERR_BAD_ARG, "context already joined a shard group");
  if (world > kShardMaxRanks)
    return fail(ctx, OUROQ_ERR_UNSUPPORTED, "at most %d ranks per shard group", kShardMaxRanks);
  const NcclApi& n = nccl();
  if (!n.ok) return fail(ctx, OUROQ_ERR_NCCL, "%s", n.why.c_str());
  DeviceGuard g(ctx->device);
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof uid);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = n.CommInitRank(&comm, world, uid, rank);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclCommInitRank");
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&ctx->shard_ctr), 4 * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(ctx->shard_ctr, 0, 4 * sizeof(unsigned));
  if (e != cudaSuccess) {
    n.CommDestroy(comm);
    cudaFree(ctx->shard_ctr);
    ctx->shard_ctr = nullptr;
    return cuda_fail(ctx, e, "shard counters");
  }
  ctx->comm = comm;
  ctx->shard_world = world;
  ctx->shard_rank = rank;
  ctx->comm_failed = false;
  return OUROQ_OK;
}

ouroq_status ouroq_shard_finalize(ouroq_ctx* ctx) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  DeviceGuard g(ctx->device);
  shard_release(ctx);
  return OUROQ_OK;
}

ouroq_status ouroq_shard_rows(int M, int world, int rank, int* row0, int* rows) {
  if (!row0 || !rows) return OUROQ_ERR_BAD_ARG;
  return shard_rows_impl(nullptr, M, world, rank, row0, rows);
}

ouroq_status ouroq_weight_upload_shard(ouroq_ctx* ctx, ouroq_format fmt, const void* packed_full,
                                       int M, int K, const void* scales_full, float w_scale,
                                       ouroq_weight** out) {
  if (!ctx || !packed_full || !out) return fail(ctx, OUROQ_ERR_BAD_ARG, "null argument");
  if (!ctx->comm) return fail(ctx, OUROQ_ERR_BAD_ARG, "context has not joined a shard group");
  ouroq_status st = check_weight_shape(ctx, fmt, M, K);
  if (st != OUROQ_OK) return st;
  int row0 = 0, rows = 0;
  st = shard_rows_impl(ctx, M, ctx->shard_world, ctx->shard_rank, &row0, &rows);
  if (st != OUROQ_OK) return st;
  const size_t rb = is_ref_format(fmt) ? ref_row_bytes(fmt, K)
                                       : (fmt == OUROQ_FMT_TERNARY2 ? (size_t)K / 4 : (size_t)K / 8);
  const uint8_t* p = static_cast<const uint8_t*>(packed_full) + (size_t)row0 * rb;
  const uint16_t* sc =
      scales_full ? static_cast<const uint16_t*>(scales_full) + (size_t)row0 * (K / 128) : nullptr;
  st = upload_impl(ctx, fmt, p, rows, K, sc, w_scale, out, false);
  if (st != OUROQ_OK) return st;
  (*out)->shard_M = M;
  (*out)->shard_row0 = row0;
  return OUROQ_OK;
}

ouroq_status ouroq_gemm_sharded(ouroq_ctx* ctx, const ouroq_weight* w, const float* x, int B,
                                const float* signs, int hadamard_block, float* y, void* stream) {
  if (!ctx || !w) return fail(ctx, OUROQ_ERR_BAD_ARG, "null handle");
  if (!ctx->comm) return fail(ctx, OUROQ_ERR_BAD_ARG, "context has not joined a shard group");
  if (w->shard_M == 0) return fail(ctx, OUROQ_ERR_BAD_ARG, "weight was not uploaded as a shard");
  if (w->shard_M != w->M * ctx->shard_world)
    return fail(ctx, OUROQ_ERR_BAD_ARG, "weight shard belongs to another group size");
  if (B < 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d", B);
  if (B == 0) return OUROQ_OK;
  if (!x || !y) return fail(ctx, OUROQ_ERR_BAD_ARG, "null buffer");
  if (ctx->comm_failed) return fail(ctx, OUROQ_ERR_NCCL, "shard group failed earlier");
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int R = w->M, G = ctx->shard_world, r = ctx->shard_rank;
  if (G == 1) return ouroq_gemm_f32act(ctx, w, x, B, signs, hadamard_block, y, stream);
  if (ctx->transport == OUROQ_SHARD_PEER) {
    ouroq_status st = ensure_landing(ctx, (size_t)G * B * R, s);
    if (st != OUROQ_OK) return st;
    st = grow(ctx, ctx->gather, ctx->gather_cap, (size_t)B * R, "staging buffer");
    if (st != OUROQ_OK) return st;
    st = ouroq_gemm_f32act(ctx, w, x, B, signs, hadamard_block, ctx->gather, stream);
    if (st != OUROQ_OK) return st;
    ShardGather P{};
    P.staging = ctx->gather;
    for (int i = 0; i < G; ++i) P.peers[i] = ctx->peer_ptr[i];
    P.y = y;
    P.step = ctx->shard_ctr;
    P.done = ctx->shard_ctr + 1;
    P.status = ctx->d_status;
    P.rank = r;
    P.G = G;
    P.B = B;
    P.R = R;
    P.timeout_ns = ctx->peer_timeout_ns;
    CU(ctx, launch_shard_gather(P, s, ctx->pdl), "peer gather launch");
    ctx->launches++;
    return OUROQ_OK;
  }
  const ncclComm_t comm = static_cast<ncclComm_t>(ctx->comm);
  float* slot;
  float* recv;
  if (B == 1) {
    // slot order is the output order: compute into y's own rows, gather in place
    recv = y;
    slot = y + (size_t)r * R;
  } else {
    ouroq_status st = grow(ctx, ctx->gather, ctx->gather_cap, (size_t)G * B * R, "gather buffer");
    if (st != OUROQ_OK) return st;
    recv = ctx->gather;
    slot = ctx->gather + (size_t)r * B * R;
  }
  ouroq_status st = ouroq_gemm_f32act(ctx, w, x, B, signs, hadamard_block, slot, stream);
  if (st != OUROQ_OK) return st;
  const ncclResult_t nr = nccl().AllGather(slot, recv, (size_t)B * R, ncclFloat32, comm, s);
  if (nr != ncclSuccess) {
    ctx->comm_failed = true;
    return nccl_fail(ctx, nr, "ncclAllGather");
  }
  if (B > 1) {
    CU(ctx, launch_shard_interleave(ctx->gather, y, B, R, G, s), "interleave launch");
    ctx->launches++;
  }
  return OUROQ_OK;
}

ouroq_status ouroq_shard_set_transport(ouroq_ctx* ctx, int transport) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (transport != OUROQ_SHARD_PEER && transport != OUROQ_SHARD_NCCL)
    return fail(ctx, OUROQ_ERR_BAD_ARG, "unknown transport %d", transport);
  ctx->transport = transport;
  return OUROQ_OK;
}

ouroq_status ouroq_shard_sync(ouroq_ctx* ctx, void* stream, int timeout_ms) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (!ctx->comm) return fail(ctx, OUROQ_ERR_BAD_ARG, "context has not joined a shard group");
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ouroq_status st = stream_wait_bounded(ctx, s, timeout_ms);
  if (st != OUROQ_OK) return st;
  unsigned v = 0;
  CU(ctx, cudaMemcpyAsync(&v, ctx->d_status, sizeof v, cudaMemcpyDeviceToHost, s), "status read");
  CU(ctx, cudaStreamSynchronize(s), "status read");
  if (v == kDevPeerTimeout) {
    CU(ctx, cudaMemsetAsync(ctx->d_status, 0, sizeof v, s), "status clear");
    ctx->comm_failed = true;
    return fail(ctx, OUROQ_ERR_TIMEOUT, "a peer's rows did not arrive in time");
  }
  return OUROQ_OK;
}


// ---------------------------------------------------------------- decode step
ouroq_status ouroq_rmsnorm(ouroq_ctx* ctx, const float* x, const float* r, float* h, const float* w,
                           float* y, int B, int n, float eps, void* stream) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (B < 0 || n <= 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d n=%d", B, n);
  if (B == 0) return OUROQ_OK;
  if (!x || !w || !y) return fail(ctx, OUROQ_ERR_BAD_ARG, "null buffer");
  DeviceGuard g(ctx->device);
  CU(ctx, launch_rmsnorm(x, r, h, w, y, B, n, eps, static_cast<cudaStream_t>(stream), ctx->pdl),
     "rmsnorm launch");
  ctx->launches++;
  return OUROQ_OK;
}

ouroq_status ouroq_swiglu_rmsnorm(ouroq_ctx* ctx, const float* gate, const float* up,
                                  const float* w, float* y, int B, int n, float eps, void* stream) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (B < 0 || n <= 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d n=%d", B, n);
  if (B == 0) return OUROQ_OK;
  if (!gate || !up || !w || !y) return fail(ctx, OUROQ_ERR_BAD_ARG, "null buffer");
  DeviceGuard g(ctx->device);
  CU(ctx, launch_swiglu_norm(gate, up, w, y, B, n, eps, static_cast<cudaStream_t>(stream), ctx->pdl),
     "swiglu launch");
  ctx->launches++;
  return OUROQ_OK;
}

static ouroq_status check_attn_shape(ouroq_ctx* ctx, int B, int n_head, int n_kv, int tmax) {
  if (B < 0 || n_head <= 0 || n_kv <= 0 || tmax <= 0)
    return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d n_head=%d n_kv=%d tmax=%d", B, n_head, n_kv, tmax);
  if (n_head % n_kv || n_head / n_kv > 8)
    return fail(ctx, OUROQ_ERR_UNSUPPORTED, "%d query heads over %d KV heads (group of at most 8)",
                n_head, n_kv);
  if (B > 65535 || n_kv > 65535) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "grid too large");
  return OUROQ_OK;
}

ouroq_status ouroq_rope_kv_append(ouroq_ctx* ctx, float* q, const float* k, const float* v,
                                  float* kcache, float* vcache, const int64_t* pos, int B,
                                  int n_head, int n_kv, int tmax, float rope_base, void* stream) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  ouroq_status st = check_attn_shape(ctx, B, n_head, n_kv, tmax);
  if (st != OUROQ_OK || B == 0) return st;
  if (!q || !k || !v || !kcache || !vcache || !pos)
    return fail(ctx, OUROQ_ERR_BAD_ARG, "null buffer");
  DecodeAttn P{};
  P.q = q;
  P.k = k;
  P.v = v;
  P.kcache = kcache;
  P.vcache = vcache;
  P.pos = reinterpret_cast<const long long*>(pos);
  P.status = ctx->d_status;
  P.B = B;
  P.n_head = n_head;
  P.n_kv = n_kv;
  P.tmax = tmax;
  P.rope_base = rope_base;
  DeviceGuard g(ctx->device);
  CU(ctx, launch_rope_append(P, static_cast<cudaStream_t>(stream), ctx->pdl), "rope launch");
  ctx->launches++;
  return OUROQ_OK;
}

static ouroq_status attention_common(ouroq_ctx* ctx, DecodeAttn& P, bool rope, void* stream) {
  if (!aligned16(P.q) || !aligned16(P.kcache) || !aligned16(P.vcache) || !aligned16(P.out) ||
      (rope && (!aligned16(P.k) || !aligned16(P.v))))
    return fail(ctx, OUROQ_ERR_BAD_ALIGN, "attention buffers not 16-byte aligned");
  DeviceGuard g(ctx->device);
  P.status = ctx->d_status;
  P.splits = attn_splits(P.B, P.n_head, P.n_kv, P.tmax, ctx->num_sms);
  P.scale = 1.0f / std::sqrt(128.0f);
  ouroq_status st = grow(ctx, ctx->attn_part, ctx->attn_cap,
                         attn_part_floats(P.B, P.n_head, P.n_kv, P.splits), "attention partials");
  if (st != OUROQ_OK) return st;
  const size_t nctr = (size_t)P.B * P.n_kv;
  if (nctr > ctx->attn_ctr_cap) {
    st = grow(ctx, ctx->attn_ctr, ctx->attn_ctr_cap, nctr, "attention counters");
    if (st != OUROQ_OK) return st;
    CU(ctx, cudaMemset(ctx->attn_ctr, 0, ctx->attn_ctr_cap * sizeof(unsigned)),
       "attention counters");
  }
  P.part = ctx->attn_part;
  P.counter = ctx->attn_ctr;
  CU(ctx, launch_attention_decode(P, rope, static_cast<cudaStream_t>(stream), ctx->pdl),
     "attention launch");
  ctx->launches++;
  return OUROQ_OK;
}

ouroq_status ouroq_attention_decode(ouroq_ctx* ctx, const float* q, const float* kcache,
                                    const float* vcache, const int64_t* pos, float* out, int B,
                                    int n_head, int n_kv, int tmax, void* stream) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  ouroq_status st = check_attn_shape(ctx, B, n_head, n_kv, tmax);
  if (st != OUROQ_OK || B == 0) return st;
  if (!q || !kcache || !vcache || !pos || !out) return fail(ctx, OUROQ_ERR_BAD_ARG, "null buffer");
  DecodeAttn P{};
  P.q = const_cast<float*>(q);
  P.kcache = const_cast<float*>(kcache);
  P.vcache = const_cast<float*>(vcache);
  P.pos = reinterpret_cast<const long long*>(pos);
  P.out = out;
  P.B = B;
  P.n_head = n_head;
  P.n_kv = n_kv;
  P.tmax = tmax;
  return attention_common(ctx, P, false, stream);
}

ouroq_status ouroq_rope_attention_decode(ouroq_ctx* ctx, const float* q, const float* k,
                                         const float* v, float* kcache, float* vcache,
                                         const int64_t* pos, float* out, int B, int n_head,
                                         int n_kv, int tmax, float rope_base, void* stream) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  ouroq_status st = check_attn_shape(ctx, B, n_head, n_kv, tmax);
  if (st != OUROQ_OK || B == 0) return st;
  if (!q || !k || !v || !kcache || !vcache || !pos || !out)
    return fail(ctx, OUROQ_ERR_BAD_ARG, "null buffer");
  DecodeAttn P{};
  P.q = const_cast<float*>(q);
  P.k = k;
  P.v = v;
  P.kcache = kcache;
  P.vcache = vcache;
  P.pos = reinterpret_cast<const long long*>(pos);
  P.out = out;
  P.B = B;
  P.n_head = n_head;
  P.n_kv = n_kv;
  P.tmax = tmax;
  P.rope_base = rope_base;
  return attention_common(ctx, P, true, stream);
}

ouroq_status ouroq_argmax_token(ouroq_ctx* ctx, const ouroq_weight* w, const float* x, int B,
                                float* logits, int64_t* tokens, void* stream) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (!w || !x || !tokens) return fail(ctx, OUROQ_ERR_BAD_ARG, "null argument");
  if (!is_half_format(w->fmt))
    return fail(ctx, OUROQ_ERR_UNSUPPORTED, "argmax_token needs an F16 or BF16 head (format %d)",
                (int)w->fmt);
  if (B < 0 || (size_t)B > 65535 * 8) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d", B);
  if (B == 0) return OUROQ_OK;
  DeviceGuard g(ctx->device);
  const size_t need = (size_t)B + 1;  // keys, then the CTA counter
  if (need > ctx->head_key_cap) {
    ouroq_status st = grow(ctx, ctx->head_key, ctx->head_key_cap, need, "argmax scratch");
    if (st != OUROQ_OK) return st;
    CU(ctx, cudaMemset(ctx->head_key, 0, ctx->head_key_cap * sizeof(unsigned long long)),
       "argmax scratch");
  }
  HeadLaunch L{};
  L.w = reinterpret_cast<const uint16_t*>(w->w);
  L.x = x;
  L.y = logits;
  L.M = w->M;
  L.K = w->K;
  L.B = B;
  L.ldy = w->M;
  L.bf16 = w->fmt == OUROQ_FMT_BF16;
  L.vec = w->K % 8 == 0 && aligned16(w->w) && aligned16(x);
  L.num_sms = ctx->num_sms;
  // the counter word sits after the keys of the largest B seen so far
  L.key = ctx->head_key;
  L.counter = reinterpret_cast<unsigned*>(ctx->head_key + ctx->head_key_cap - 1);
  L.tokens = reinterpret_cast<long long*>(tokens);
  CU(ctx, launch_head(L, static_cast<cudaStream_t>(stream), ctx->pdl), "argmax_token launch");
  ctx->launches++;
  return OUROQ_OK;
}

ouroq_status ouroq_gemm_norm_f32act(ouroq_ctx* ctx, int n, const ouroq_weight* const* w,
                                    const float* x, const float* residual, int mode,
                                    const float* norm_w, float eps, float* h, int B,
                                    float* const* y, void* stream) {
  if (!ctx) return OUROQ_ERR_BAD_ARG;
  if (n < 1 || n > kMaxGemvJobs)
    return fail(ctx, OUROQ_ERR_BAD_SHAPE, "group size %d (1..%d)", n, kMaxGemvJobs);
  if (B < 0) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "B=%d", B);
  if (B == 0) return OUROQ_OK;
  if (!w || !x || !norm_w || !y) return fail(ctx, OUROQ_ERR_BAD_ARG, "null argument");
  if (mode != 0 && mode != 1) return fail(ctx, OUROQ_ERR_BAD_ARG, "mode %d", mode);
  if (mode == 1 && (!residual || h))
    return fail(ctx, OUROQ_ERR_BAD_ARG, "mode 1 takes the up projection and no h");
  for (int i = 0; i < n; ++i) {
    if (!w[i] || !y[i]) return fail(ctx, OUROQ_ERR_BAD_ARG, "null entry %d", i);
    if (is_ref_format(w[i]->fmt) || w[i]->fmt != w[0]->fmt)
      return fail(ctx, OUROQ_ERR_UNSUPPORTED, "one TERNARY2 or SIGN1G128 format per group");
    if (w[i]->K != w[0]->K) return fail(ctx, OUROQ_ERR_BAD_SHAPE, "entries read one row width");
  }
  const int K = w[0]->K;
  // one CTA writes h while the others still read x and the residual
  const size_t row_bytes = (size_t)B * K * sizeof(float);
  auto overlap = [&](const void* a, const void* b) {
    const char* pa = static_cast<const char*>(a);
    const char* pb = static_cast<const char*>(b);
    return a && b && pa < pb + row_bytes && pb < pa + row_bytes;
  };
  if (h && (overlap(h, x) || overlap(h, residual)))
    return fail(ctx, OUROQ_ERR_BAD_ARG, "h must not overlap x or the residual");
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool aligned = aligned16(x) && (!residual || aligned16(residual)) && aligned16(norm_w) &&
                       (!h || aligned16(h));
  if (B <= kFusedMaxB && aligned && K % 128 == 0 && B * (K / 128) <= kNormFusedMaxUnits) {
    GemvLaunch L{};
    L.njobs = n;
    L.B = B;
    L.fused = 1;
    L.fmt = w[0]->fmt == OUROQ_FMT_TERNARY2 ? kTern2 : kSign1;
    for (int i = 0; i < n; ++i) {
      L.jobs[i] = make_job(w[i], nullptr, nullptr, y[i], nullptr);
      L.jobs[i].xf = x;
    }
    L.norm.x = x;
    L.norm.r = residual;
    L.norm.w = norm_w;
    L.norm.h = h;
    L.norm.eps = eps;
    L.norm.mode = mode;
    L.norm.K = K;
    if (gemv_fits(ctx, L)) return run_gemv(ctx, L, s);
  }
  // not fused: the norm kernel into scratch, then the grouped product
  ouroq_status st = grow(ctx, ctx->norm_scratch, ctx->norm_cap, (size_t)B * K, "norm scratch");
  if (st != OUROQ_OK) return st;
  float* a = ctx->norm_scratch;
  if (mode == 0)
    CU(ctx, launch_rmsnorm(x, residual, h, norm_w, a, B, K, eps, s, ctx->pdl), "rmsnorm launch");
  else
    CU(ctx, launch_swiglu_norm(x, residual, norm_w, a, B, K, eps, s, ctx->pdl), "swiglu launch");
  ctx->launches++;
  if (B <= kGemvMaxB) {
    const float* xs[kMaxGemvJobs];
    for (int i = 0; i < n; ++i) xs[i] = a;
    return ouroq_gemm_group_f32act(ctx, n, w, xs, B, nullptr, nullptr, y, stream);
  }
  st = grow(ctx, ctx->q_scratch, ctx->q_cap, (size_t)B * K, "q scratch");
  if (st != OUROQ_OK) return st;
  st = grow(ctx, ctx->s_scratch, ctx->s_cap, (size_t)B, "s scratch");
  if (st != OUROQ_OK) return st;
  st = ouroq_quantize_act(ctx, a, B, K, nullptr, 0, ctx->q_scratch, ctx->s_scratch, stream);
  if (st != OUROQ_OK) return st;
  // the group's products on the shared codes (one tensor-core launch for ternary weights)
  const int8_t* qs[kMaxGemvJobs];
  const float* ss[kMaxGemvJobs];
  for (int i = 0; i < n; ++i) {
    qs[i] = ctx->q_scratch;
    ss[i] = ctx->s_scratch;
  }
  return ouroq_gemm_group(ctx, n, w, qs, ss, B, y, stream);
}

}  // extern "C"
