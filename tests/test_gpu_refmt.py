"""GPU decode of the reference's own shard formats against the oracle.

PTQ1_0 ("Tl1") and TQ1_0 weights are uploaded byte for byte and multiplied by
fp32 activations. The kernels repeat the reference's floating-point order, so
every comparison with the oracle restatement of that order is exact:
  PTQ1_0: matvec_tl1's x86 order (cluster/src/infer/ops.rs:499-584) for one
          token (matvec_q); matmul_tl1's x86 K-column order (ops.rs:381-481)
          for a batch and for every host matmul_q call (ops.rs:219-230)
  TQ1_0:  matvec_qblock = dequantise then dot (ops.rs:101-128, 53-60), per
          token in both cases (matmul_q runs K matvecs for it)
The two PTQ1_0 orders differ within the tolerance the reference's own test
states (ops.rs:721-750), checked here too.
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


def tl1_payload(oracle, M, K, seed):
    p = oracle.lcg_bytes(seed, M * (K // 128) * 28).reshape(-1, 28)
    sc = np.array([oracle.f32_to_f16(v) for v in
                   np.abs(oracle.normals(seed + 1, p.shape[0])) * 0.02], np.uint16)
    p[:, 26] = sc & 0xFF
    p[:, 27] = sc >> 8
    return p.reshape(-1)


def tq1_payload(oracle, M, K, seed):
    p = oracle.lcg_bytes(seed, M * (K // 256) * 54).reshape(-1, 54)
    sc = np.array([oracle.f32_to_f16(v) for v in
                   np.abs(oracle.normals(seed + 1, p.shape[0])) * 0.02], np.uint16)
    p[:, 52] = sc & 0xFF
    p[:, 53] = sc >> 8
    return p.reshape(-1)


@pytest.mark.parametrize("M,K,B", [(37, 384, 1), (200, 2560, 3), (6912, 2560, 1), (2560, 6912, 2),
                                   (1024, 8192, 1)])
def test_tl1_matches_reference_order(ctx, oracle, M, K, B):
    payload = tl1_payload(oracle, M, K, seed=M + K)
    x = oracle.normals(K + 5, B * K).reshape(B, K)
    w = ctx.upload(oq.PTQ1_0, payload, M, K)
    y = _host(ctx.gemm_f32act(w, _dev(x)))
    if B == 1:
        want = oracle.matvec_tl1_sse(payload, M, K, x[0]).reshape(1, M)
    else:
        want = oracle.matmul_tl1_sse(payload, M, K, x, B).reshape(B, M)
    assert np.array_equal(y, want), int(np.sum(y != want))
    w.free()


@pytest.mark.parametrize("M,K,B", [(19, 512, 1), (300, 2560, 2), (6912, 2560, 1), (2560, 6912, 1)])
def test_tq1_matches_reference_order(ctx, oracle, M, K, B):
    payload = tq1_payload(oracle, M, K, seed=3 * M + K)
    x = oracle.normals(K + 9, B * K).reshape(B, K)
    w = ctx.upload(oq.TQ1_0, payload, M, K)
    y = _host(ctx.gemm_f32act(w, _dev(x)))
    for b in range(B):
        assert np.array_equal(y[b], oracle.matvec_tq1(payload, M, K, x[b]))
    w.free()


def test_tl1_reference_test_vectors(ctx, oracle):
    # payload and x of ops.rs:801-838 (37 x 384); the reference accepts its two
    # orders within 1e-5 relative of each other, ours equals the x86 order
    out_len, in_len = 37, 384
    n = out_len * (in_len // 128) * 28
    i = np.arange(n, dtype=np.uint64)
    payload = ((i * (0x9B ^ (i >> np.uint64(7)))) & np.uint64(0xFF)).astype(np.uint8)
    g = payload.reshape(-1, 28)
    g[:, 26], g[:, 27] = 0x10, 0x38
    x = np.array([((k % 7) - 3.0) * 0.5 for k in range(in_len)], np.float32)
    w = ctx.upload(oq.PTQ1_0, payload, out_len, in_len)
    y = ctx.matvec_q(w, x)
    assert np.array_equal(y, oracle.matvec_tl1_sse(payload, out_len, in_len, x))
    scalar = oracle.matvec_tl1_scalar(payload, out_len, in_len, x)
    assert np.all(np.abs(y - scalar) / np.maximum(np.abs(scalar), 1e-9) < 1e-5)
    w.free()


def test_tl1_k_columns(ctx, oracle):
    # matmul_q on host buffers, K = 4 columns (ops.rs:721-750 shapes)
    out_len, in_len, k = 97, 384, 4
    payload = tl1_payload(oracle, out_len, in_len, seed=41)
    x = oracle.normals(42, k * in_len).reshape(k, in_len)
    w = ctx.upload(oq.PTQ1_0, payload, out_len, in_len)
    y = ctx.matmul_q(w, x)
    kcol = oracle.matmul_tl1_sse(payload, out_len, in_len, x, k).reshape(k, out_len)
    assert np.array_equal(y, kcol)
    for c in range(k):
        want = oracle.matvec_tl1_sse(payload, out_len, in_len, x[c])
        assert np.all(np.abs(y[c] - want) <= 1e-3 * np.maximum(np.abs(want), 1.0))
    # one column through matmul_q keeps the K-column order; matvec_q the matvec order
    y1 = ctx.matmul_q(w, x[:1])
    assert np.array_equal(y1[0], oracle.matmul_tl1_sse(payload, out_len, in_len, x[0], 1))
    assert np.array_equal(ctx.matvec_q(w, x[0]), oracle.matvec_tl1_sse(payload, out_len, in_len, x[0]))
    w.free()


@pytest.mark.parametrize("out_len,in_len,k", [(130, 2560, 9), (64, 1152, 2), (33, 128, 8)])
def test_tl1_k_columns_blocks(ctx, oracle, out_len, in_len, k):
    # from two columns on, the K-column kernel decodes each group once for up
    # to eight columns (a second block of one column at k = 9, x staged in
    # chunks of eight groups, rows off the 64-row tile): still matmul_tl1's
    # order bit for bit
    payload = tl1_payload(oracle, out_len, in_len, seed=out_len + k)
    x = oracle.normals(in_len + k, k * in_len).reshape(k, in_len)
    w = ctx.upload(oq.PTQ1_0, payload, out_len, in_len)
    y = ctx.matmul_q(w, x)
    assert np.array_equal(y, oracle.matmul_tl1_sse(payload, out_len, in_len, x, k).reshape(k, out_len))
    w.free()


def test_tl1_with_rotation(ctx, oracle):
    # Qwen35Stage::wh: rotate_fwd(x, signs, block) then the product (two tokens: matmul_q)
    M, K, B, block = 256, 4096, 2, 128
    payload = tl1_payload(oracle, M, K, seed=77)
    x = oracle.outliers(78, oracle.normals(79, B * K), 0.01, 20.0).reshape(B, K)
    sg = oracle.signs(80, K).astype(np.float32)
    w = ctx.upload(oq.PTQ1_0, payload, M, K)
    y = _host(ctx.gemm_f32act(w, _dev(x), signs=_dev(sg), hadamard_block=block))
    xr = np.stack([oracle.rotate_fwd(x[b], sg, block) for b in range(B)])
    assert np.array_equal(y, oracle.matmul_tl1_sse(payload, M, K, xr, B).reshape(B, M))
    w.free()


def test_reference_formats_golden(ctx):
    from pathlib import Path
    with np.load(Path(__file__).resolve().parent / "golden" / "refformat.npz") as z:
        g = {k: z[k] for k in z.files}
    o, i = (int(v) for v in g["tl1_shape"])
    w = ctx.upload(oq.PTQ1_0, g["tl1_payload"], o, i)
    assert np.array_equal(ctx.matvec_q(w, g["tl1_x"]), g["tl1_sse"])
    assert np.array_equal(ctx.matmul_q(w, g["tl1_xk"].reshape(3, i)).reshape(-1),
                          g["tl1_matmul_sse_k3"])
    w.free()
    o, i = (int(v) for v in g["tq1_shape"])
    w = ctx.upload(oq.TQ1_0, g["tq1_payload"], o, i)
    assert np.array_equal(ctx.matvec_q(w, g["tq1_x"]), g["tq1_y"])
    w.free()


def test_reference_formats_reject_int8_activations(ctx, oracle):
    import torch
    payload = tq1_payload(oracle, 32, 256, seed=5)
    w = ctx.upload(oq.TQ1_0, payload, 32, 256)
    q = torch.zeros((1, 256), dtype=torch.int8, device="cuda")
    s = torch.ones((1,), dtype=torch.float32, device="cuda")
    with pytest.raises(oq.OuroqError) as ei:
        ctx.gemm(w, q, s)
    assert ei.value.status == 6
    with pytest.raises(oq.OuroqError) as ei:
        ctx.upload(oq.TQ1_0, payload, 16, 128 * 3)  # K not a multiple of 256
    assert ei.value.status == 1
    w.free()
