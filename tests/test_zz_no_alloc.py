"""ouroq_gemm_f32act_noalloc: the entry point that allocates no device memory.

Who it is for: callers that cannot allocate device memory while they run --
a serving loop that reserved the GPU's memory up front for weights and caches
(a late cudaMalloc can fail there), or one on a latency budget (cudaFree waits
for the whole device). ouroq_gemm_f32act grows a scratch buffer with cudaMalloc
when a larger batch arrives; the no-alloc variant uses a fixed scratch area
compiled into the library instead (B <= 4096, B*K <= 4 MiB per call).

Each case calls the new entry point twice in a row, with different inputs,
through the C ABI and checks both results bit for bit against
ouroq_gemm_f32act on the same inputs; free device memory must not change
across the two calls. The file is named to run last, and passes on its own in
a fresh process too: the first no-alloc call, which does the one-time set-up
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


def _weight(ctx, oracle, fmt, M, K, seed):
    if fmt == oq.TERNARY2:
        t = oracle.ternary(seed, M * K).reshape(M, K)
        return ctx.upload(oq.TERNARY2, oracle.pack_tern2(t), M, K,
                          w_scale=float(oracle.absmean_scale(t, 0.02)))
    s = oracle.signs(seed, M * K).reshape(M, K)
    sc = oracle.group_scales(seed + 1, M * (K // 128), 0.02)
    return ctx.upload(oq.SIGN1G128, oracle.pack_sign1(s), M, K, scales=sc)


# (format, M, K, B, hadamard block): B <= 8 takes the single fused launch,
# larger batches go through the fixed scratch (tensor cores for ternary
# B >= 16, several token passes at B = 300; GEMV chunks for sign weights).
CASES = [
    (oq.TERNARY2, 2560, 2560, 4, 0),
    (oq.TERNARY2, 6912, 2560, 32, 0),
    (oq.TERNARY2, 2560, 6912, 300, 0),
    (oq.TERNARY2, 512, 1024, 12, 0),
    (oq.SIGN1G128, 4096, 4096, 12, 64),
    (oq.SIGN1G128, 2048, 1024, 40, 1024),
]


@pytest.mark.parametrize("fmt,M,K,B,block", CASES)
def test_noalloc_matches_gemm_f32act_twice(ctx, oracle, setup_call, fmt, M, K, B, block):
    import torch
    w = _weight(ctx, oracle, fmt, M, K, seed=M + K + B)
    sg = _dev(oracle.signs(91, K).astype(np.float32)) if block else None
    xs = [_dev(oracle.outliers(B + i, oracle.normals(K + i, B * K), 0.01, 20.0).reshape(B, K))
          for i in range(2)]
    want = [_host(ctx.gemm_f32act(w, x, signs=sg, hadamard_block=block)) for x in xs]
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


@pytest.mark.parametrize("B,K", [(2048, 4096), (4097, 128)])
def test_noalloc_rejects_batches_beyond_the_fixed_scratch(ctx, oracle, setup_call, B, K):
    import torch
    M = 256
    w = _weight(ctx, oracle, oq.TERNARY2, M, K, seed=3)
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
