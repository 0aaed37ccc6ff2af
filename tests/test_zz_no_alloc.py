"""ouroq_gemm_f32act_noalloc: the entry point that allocates no device memory.

Who it is for: callers that cannot allocate device memory while they run --
a serving loop that reserved the GPU's memory up front for weights and caches
(a late cudaMalloc can fail there), or one on a latency budget (cudaFree waits
for the whole device). ouroq_gemm_f32act grows a scratch buffer with cudaMalloc
when a larger batch arrives; the no-alloc variant uses a fixed scratch area
compiled into the library instead (B <= 4096, B*K <= 4 MiB per call).

Each case calls the new entry point twice in a row, with different inputs,
through the C ABI and checks both results bit for bit against
ouroq_gemm_f32act on the same inputs and against the CPU oracle; free device
memory must not change across the two calls. The file is named to run last,
and passes on its own in a fresh process too: the first no-alloc call, which does the one-time set-up
on the device, happens in the `setup_call` fixture before anything is measured.
"""
import numpy as np
import pytest

import ouroboros_b200 as oq

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module")
def setup_call(ctx, oracle):
    """One small no-alloc call: the first call on a device does set-up."""
    import torch
    M, K = 64, 128
    w = ctx.upload(oq.TERNARY2, oracle.pack_tern2(oracle.ternary(5, M * K).reshape(M, K)), M, K,
                   w_scale=0.5)
    x = _dev(oracle.normals(6, 2 * K).reshape(2, K))
    y = torch.empty((2, M), dtype=torch.float32, device="cuda")
    ctx.gemm_f32act_noalloc(w, x, y)
    torch.cuda.synchronize()
    w.free()
    return True


def _ref_payload(oracle, fmt, M, K, seed):
    """A PTQ1_0 / TQ1_0 shard payload (random trits, |N(0, 0.02)| f16 scales)."""
    gb, per = (28, 128) if fmt == oq.PTQ1_0 else (54, 256)
    p = oracle.lcg_bytes(seed, M * (K // per) * gb).reshape(-1, gb)
    sc = np.array([oracle.f32_to_f16(v) for v in
                   np.abs(oracle.normals(seed + 1, p.shape[0])) * 0.02], np.uint16)
    p[:, gb - 2] = sc & 0xFF
    p[:, gb - 1] = sc >> 8
    return p.reshape(-1)


def _weight(ctx, oracle, fmt, M, K, seed):
    """Upload a weight; returns (handle, oracle(x, signs, block) -> y [B][M])."""
    if fmt == oq.TERNARY2:
        t = oracle.ternary(seed, M * K).reshape(M, K)
        packed, ws = oracle.pack_tern2(t), float(oracle.absmean_scale(t, 0.02))

        def ref(x, sg, block):
            q, s = oracle.quantize_act(x, sg, block)
            return oracle.gemm_tern2_mt(packed, M, K, ws, q, s)
        return ctx.upload(oq.TERNARY2, packed, M, K, w_scale=ws), ref
    if fmt == oq.SIGN1G128:
        packed = oracle.pack_sign1(oracle.signs(seed, M * K).reshape(M, K))
        sc = oracle.group_scales(seed + 1, M * (K // 128), 0.02)

        def ref(x, sg, block):
            q, s = oracle.quantize_act(x, sg, block)
            return oracle.gemm_sign1_mt(packed, sc, M, K, q, s)
        return ctx.upload(oq.SIGN1G128, packed, M, K, scales=sc), ref
    if fmt == oq.F16:
        emb = (oracle.normals(seed, M * K) * np.float32(0.02)).astype(np.float16).view(np.uint16)

        def ref(x, sg, block):
            return np.stack([oracle.matvec_half(emb, M, K, x[b]) for b in range(x.shape[0])])
        return ctx.upload(oq.F16, emb, M, K), ref
    payload = _ref_payload(oracle, fmt, M, K, seed)

    def ref(x, sg, block):
        B = x.shape[0]
        if fmt == oq.TQ1_0:
            return np.stack([oracle.matvec_tq1(payload, M, K, x[b]) for b in range(B)])
        if B == 1:  # one token: matvec_tl1's order; several: matmul_tl1's K columns
            return oracle.matvec_tl1_sse(payload, M, K, x[0])[None]
        return oracle.matmul_tl1_sse(payload, M, K, x, B).reshape(B, M)
    return ctx.upload(fmt, payload, M, K), ref


# (format, M, K, B, hadamard block): ternary weights without a rotation up to
# 8 tokens take the single fused launch (no scratch); the other batches go
# through the fixed scratch (tensor cores from 9 tokens, several token passes
# at B = 300); the reference formats and F16 need no scratch (matvec_tl1's
# order for one token, matmul_tl1's K columns for several).
CASES = [
    (oq.TERNARY2, 2560, 2560, 2, 0),
    (oq.TERNARY2, 2560, 2560, 4, 0),
    (oq.TERNARY2, 6912, 2560, 32, 0),
    (oq.TERNARY2, 2560, 6912, 300, 0),
    (oq.TERNARY2, 512, 1024, 12, 0),
    (oq.SIGN1G128, 4096, 4096, 12, 64),
    (oq.SIGN1G128, 2048, 1024, 40, 1024),
    (oq.PTQ1_0, 512, 2560, 1, 0),
    (oq.PTQ1_0, 512, 2560, 5, 0),
    (oq.TQ1_0, 384, 2560, 3, 0),
    (oq.F16, 1024, 2560, 2, 0),
]


@pytest.mark.parametrize("fmt,M,K,B,block", CASES)
def test_noalloc_matches_gemm_f32act_twice(ctx, oracle, setup_call, fmt, M, K, B, block):
    import torch
    w, ref = _weight(ctx, oracle, fmt, M, K, seed=M + K + B)
    sgh = oracle.signs(91, K).astype(np.float32) if block else None
    sg = _dev(sgh) if block else None
    xh = [oracle.outliers(B + i, oracle.normals(K + i, B * K), 0.01, 20.0).reshape(B, K)
          for i in range(2)]
    xs = [_dev(x) for x in xh]
    want = [_host(ctx.gemm_f32act(w, x, signs=sg, hadamard_block=block)) for x in xs]
    for x, yr in zip(xh, want):  # the existing entry point is itself the oracle's result
        assert np.array_equal(ref(x, sgh, block), yr)
    ys = [torch.full((B, M), float("nan"), dtype=torch.float32, device="cuda") for _ in xs]
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for x, y in zip(xs, ys):
        ctx.gemm_f32act_noalloc(w, x, y, signs=sg, hadamard_block=block)
    torch.cuda.synchronize()
    free_after = torch.cuda.mem_get_info()[0]
    for y, yr in zip(ys, want):
        assert np.array_equal(_host(y), yr)
    assert free_after == free_before
    w.free()


def test_noalloc_refuses_a_rotated_reference_format(ctx, oracle, setup_call):
    # PTQ1_0 with a rotation would need a buffer for the rotated activations:
    # refused as unsupported, nothing launched, y untouched
    import torch
    M, K = 256, 1024
    w, _ = _weight(ctx, oracle, oq.PTQ1_0, M, K, seed=8)
    x = _dev(oracle.normals(9, 2 * K).reshape(2, K))
    y = torch.full((2, M), 7.0, dtype=torch.float32, device="cuda")
    sg = _dev(oracle.signs(10, K).astype(np.float32))
    before = ctx.launch_count()
    with pytest.raises(oq.OuroqError) as ei:
        ctx.gemm_f32act_noalloc(w, x, y, signs=sg, hadamard_block=64)
    assert ei.value.status == 6  # OUROQ_ERR_UNSUPPORTED
    assert ctx.launch_count() == before
    torch.cuda.synchronize()
    assert bool(torch.all(y == 7.0))
    w.free()


@pytest.mark.parametrize("B,K", [(2048, 4096), (4097, 128)])
def test_noalloc_rejects_batches_beyond_the_fixed_scratch(ctx, oracle, setup_call, B, K):
    import torch
    M = 256
    w, _ = _weight(ctx, oracle, oq.TERNARY2, M, K, seed=3)
    x = torch.zeros((B, K), dtype=torch.float32, device="cuda")
    y = torch.full((B, M), 7.0, dtype=torch.float32, device="cuda")
    before = ctx.launch_count()
    with pytest.raises(oq.OuroqError) as ei:
        ctx.gemm_f32act_noalloc(w, x, y)
    assert ei.value.status == 1  # OUROQ_ERR_BAD_SHAPE
    assert "fixed scratch" in str(ei.value)
    assert ctx.launch_count() == before
    torch.cuda.synchronize()
    assert bool(torch.all(y == 7.0))
    w.free()
