"""16-bit weights (F16 / BF16) behind matvec_q and the greedy tied lm_head.

The kernels keep the reference's order (one fp32 chain per row, element
order, product and sum rounded separately: ops.rs:131-153, 600-620), so the
comparison with the oracle is exact -- NaN compared by position, since the
reference and the hardware may give a NaN different payload bits.
argmax_token (infer/mod.rs:190-194) must return finite_argmax of exactly
those logits (mod.rs:70-83: NaN skipped, first maximum wins, 0 if all NaN).
"""
import numpy as np
import pytest

import ouroboros_b200 as oq
from test_oracle_kat import matmul_fallback_payload

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    return t.detach().cpu().numpy()


def half_payload(oracle, M, K, seed, bf16):
    """Random 16-bit weights of magnitude ~0.02, as the shard stores them."""
    v = (oracle.normals(seed, M * K) * np.float32(0.02)).astype(np.float32)
    if bf16:
        return (v.view(np.uint32) >> 16).astype(np.uint16)
    return v.astype(np.float16).view(np.uint16)


def _same(got, want):
    nan = np.isnan(want)
    return np.array_equal(np.isnan(got), nan) and np.array_equal(got[~nan], want[~nan])


def test_reference_matmul_fallback_vectors(ctx, oracle):
    # ops.rs:782-798: K = 2 columns through matmul_q equal matvec_f16 per column
    out_len, in_len = 16, 32
    payload = matmul_fallback_payload(out_len, in_len)
    x = ((np.arange(2 * in_len) % 7) * 0.5).astype(np.float32)
    w = ctx.upload(oq.F16, payload, out_len, in_len)
    y = ctx.matmul_q(w, x.reshape(2, in_len))
    for c in range(2):
        want = oracle.matvec_half(payload, out_len, in_len, x[c * in_len:(c + 1) * in_len])
        assert _same(y[c], want)
    w.free()


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("M,K,B", [(1000, 2560, 1), (513, 2560, 2), (300, 1001, 3), (257, 520, 5),
                                   (700, 1536, 8), (129, 2560, 9), (64, 8, 17)])
def test_half_matches_reference_order(ctx, oracle, bf16, M, K, B):
    fmt = oq.BF16 if bf16 else oq.F16
    payload = half_payload(oracle, M, K, seed=M + K + bf16, bf16=bf16)
    x = oracle.normals(K + B, B * K).reshape(B, K)
    w = ctx.upload(fmt, payload, M, K)
    y = _host(ctx.gemm_f32act(w, _dev(x)))
    for b in range(B):
        want = oracle.matvec_half(payload, M, K, x[b], bf16=bf16)
        assert _same(y[b], want), int(np.sum(y[b] != want))
    w.free()


def test_half_special_values(ctx, oracle):
    # inf, NaN and subnormal weights: the chain carries them like the reference
    M, K = 64, 256
    payload = half_payload(oracle, M, K, seed=3, bf16=False)
    payload[5 * K + 7] = 0x7C00    # +inf
    payload[9 * K + 100] = 0x7E00  # NaN
    payload[11 * K: 12 * K] = 0x0001  # smallest subnormal
    payload[12 * K + 3] = 0xFC00   # -inf
    payload[12 * K + 4] = 0x7C00   # +inf in the same row -> NaN
    x = oracle.normals(4, K)
    x[3] = x[4] = 1.0  # -inf + inf in row 12
    w = ctx.upload(oq.F16, payload, M, K)
    y = ctx.matvec_q(w, x)
    want = oracle.matvec_half(payload, M, K, x)
    assert np.isnan(want[9]) and np.isnan(want[12]) and np.isinf(want[5])
    assert _same(y, want)
    w.free()


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("B", [1, 2, 5, 11])
def test_argmax_token_matches_finite_argmax(ctx, oracle, bf16, B):
    import torch
    M, K = 50000, 2560
    fmt = oq.BF16 if bf16 else oq.F16
    payload = half_payload(oracle, M, K, seed=21 + bf16, bf16=bf16)
    x = oracle.normals(22, B * K).reshape(B, K)
    w = ctx.upload(fmt, payload, M, K)
    logits = torch.empty((B, M), device="cuda")
    tok = _host(ctx.argmax_token(w, _dev(x), logits=logits))
    lg = _host(logits)
    for b in range(B):
        want = oracle.matvec_half(payload, M, K, x[b], bf16=bf16)
        assert _same(lg[b], want)
        assert tok[b] == oracle.finite_argmax(want)
    # without logits, and again (the reduction scratch is left clear)
    for _ in range(2):
        assert np.array_equal(_host(ctx.argmax_token(w, _dev(x))), tok)
    w.free()


def test_argmax_token_ties_nan_and_all_nan(ctx, oracle):
    M, K = 3000, 512
    payload = half_payload(oracle, M, K, seed=31, bf16=False)
    x = np.abs(oracle.normals(32, K)).astype(np.float32)
    # the best row, copied to a later row (tie: the earlier wins) and an
    # earlier row made NaN (skipped)
    want0 = oracle.matvec_half(payload, M, K, x)
    best = int(np.nanargmax(want0))
    payload = payload.reshape(M, K)
    payload[M - 5] = payload[best]
    payload[max(best - 1, 0), 17] = 0x7E00
    payload = payload.reshape(-1)
    w = ctx.upload(oq.F16, payload, M, K)
    xs = np.stack([x, np.full(K, np.nan, np.float32)])
    tok = _host(ctx.argmax_token(w, _dev(xs)))
    want = oracle.matvec_half(payload, M, K, x)
    assert tok[0] == oracle.finite_argmax(want) == best
    assert tok[1] == 0  # every logit NaN
    w.free()


def test_argmax_token_rejects_other_formats(ctx, oracle):
    from test_gpu_refmt import tl1_payload
    w = ctx.upload(oq.PTQ1_0, tl1_payload(oracle, 128, 256, seed=1), 128, 256)
    with pytest.raises(oq.OuroqError):
        ctx.argmax_token(w, _dev(oracle.normals(1, 256).reshape(1, 256)))
    w.free()


def test_ptr_kind(ctx):
    import torch
    d = torch.empty(16, device="cuda")
    pinned = torch.empty(16).pin_memory()
    pageable = np.empty(16, np.float32)
    assert oq.ptr_kind(d.data_ptr()) == (oq.PTR_DEVICE, 0)
    assert oq.ptr_kind(pinned.data_ptr())[0] == oq.PTR_HOST
    assert oq.ptr_kind(pageable.ctypes.data) == (oq.PTR_HOST, -1)
