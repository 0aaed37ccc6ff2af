"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Tolerances (the target's): int32 accumulators bit-exact; fp32 outputs and the
Hadamard transform within 1e-5 relative. The kernels are built to reproduce
the oracle's IEEE operation sequence, so every comparison below is exact
equality, which implies both bounds; `assert_rel` states the 1e-5 bound
explicitly where it is the contract.
"""
import numpy as np
import pytest

import ouroboros_b200 as oq

pytestmark = pytest.mark.gpu

REL_TOL = 1e-5


def assert_rel(got, want, tol=REL_TOL):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    scale = np.maximum(np.abs(want), np.finfo(np.float32).tiny)
    assert np.all(np.abs(got - want) <= tol * scale), float(np.max(np.abs(got - want) / scale))


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def tern_case(oracle, M, K, B, seed):
    w = oracle.ternary(seed, M * K).reshape(M, K)
    x = oracle.normals(seed + 1, B * K).reshape(B, K)
    ws = oracle.absmean_scale(w, 0.02)
    return oracle.pack_tern2(w), ws, x


def sign_case(oracle, M, K, B, seed):
    w = oracle.signs(seed, M * K).reshape(M, K)
    sc = oracle.group_scales(seed + 1, M * (K // 128), 0.02)
    x = oracle.outliers(seed + 2, oracle.normals(seed + 3, B * K), 0.01, 20.0).reshape(B, K)
    return oracle.pack_sign1(w), sc, x


# ---------------------------------------------------------------- K1
@pytest.mark.parametrize("B,K", [(1, 2560), (8, 2560), (3, 6912), (64, 2560), (2, 128), (5, 4096)])
def test_quantize_matches_oracle(ctx, oracle, B, K):
    x = oracle.normals(100 + B, B * K).reshape(B, K)
    x[0, 3] = 40.0
    if B > 2:
        x[1] = 0.0
        x[2] = -0.25
    q, s = ctx.quantize_act(dev(x))
    qr, sr = oracle.quantize_act(x)
    assert np.array_equal(host(s), sr)
    assert np.array_equal(host(q), qr)


@pytest.mark.parametrize("block", [16, 32, 64, 128, 256, 1024])
@pytest.mark.parametrize("B", [1, 32])
def test_quantize_hadamard_matches_oracle(ctx, oracle, B, block):
    K = 4096
    x = oracle.outliers(7, oracle.normals(8 + block, B * K), 0.01, 20.0).reshape(B, K)
    sg = oracle.signs(9, K).astype(np.float32)
    q, s = ctx.quantize_act(dev(x), signs=dev(sg), hadamard_block=block)
    qr, sr, xr = oracle.quantize_act(x, sg, block, want_rot=True)
    assert np.array_equal(host(s), sr)
    assert np.array_equal(host(q), qr)
    rot = host(ctx.rotate(dev(x), signs=dev(sg), block=block))
    assert np.array_equal(rot, xr)  # bit-identical butterfly network
    assert_rel(rot[np.abs(xr) > 1e-6], xr[np.abs(xr) > 1e-6])


@pytest.mark.parametrize("block", [16, 64, 128, 1024])
def test_rotate_inv_matches_oracle(ctx, oracle, block):
    K = 2048
    x = oracle.normals(21, 3 * K).reshape(3, K)
    sg = oracle.signs(22, K).astype(np.float32)
    got = host(ctx.rotate(dev(x), signs=dev(sg), block=block, inverse=True))
    for b in range(3):
        assert np.array_equal(got[b], oracle.rotate_inv(x[b], sg, block))


def test_rotate_host_mirror_reference_kats(ctx, oracle):
    # hadamard.rs:96-141 inputs through the host-buffer mirror of rotate_fwd / rotate_inv
    n = 16
    x = np.array([((i * 11) % 7) - 3.0 for i in range(n)], np.float32)
    s = np.array([-1.0 if i % 3 == 0 else 1.0 for i in range(n)], np.float32)
    assert np.array_equal(ctx.rotate_fwd(x.copy(), s, 16), oracle.rotate_fwd(x, s, 16))
    x = np.array([((i * 91) % 23) * 0.37 - 4.0 for i in range(128)], np.float32)
    s = np.array([-1.0 if (i // 5) % 2 == 0 else 1.0 for i in range(128)], np.float32)
    y = ctx.rotate_fwd(ctx.rotate_inv(x.copy(), s, 64), s, 64)
    assert np.all(np.abs(x - y) < 1e-3)
    with pytest.raises(oq.OuroqError):
        ctx.rotate_fwd(np.zeros(96, np.float32), None, 48)


# ---------------------------------------------------------------- K2 ternary
TERN_SHAPES = [
    (6912, 2560, 1),   # C1
    (3840, 2560, 1), (2560, 2560, 1), (6912, 2560, 8), (2560, 6912, 1), (2560, 6912, 8),  # C2
    (37, 384, 1), (1, 128, 1), (33, 256, 3), (100, 640, 5), (32, 128, 7),  # ragged / tiny
]


@pytest.mark.parametrize("M,K,B", TERN_SHAPES)
def test_gemm_tern2_matches_oracle(ctx, oracle, M, K, B):
    packed, ws, x = tern_case(oracle, M, K, B, seed=M * 7 + K + B)
    qr, sr = oracle.quantize_act(x)
    accr, yr = oracle.gemm_tern2(packed, M, K, ws, qr, sr)
    w = ctx.upload(oq.TERNARY2, packed, M, K, w_scale=ws)
    import torch
    acc = torch.empty((B, M), dtype=torch.int32, device="cuda")
    y = ctx.gemm(w, dev(qr), dev(sr), acc=acc)
    assert np.array_equal(host(acc), accr)
    assert np.array_equal(host(y), yr)
    assert_rel(host(y)[yr != 0], yr[yr != 0])
    w.free()


@pytest.mark.parametrize("B", [16, 64])
def test_gemm_tern2_batched_c2(ctx, oracle, B):
    M, K = 6912, 2560
    packed, ws, x = tern_case(oracle, M, K, B, seed=5 + B)
    qr, sr = oracle.quantize_act(x)
    accr, yr = oracle.gemm_tern2(packed, M, K, ws, qr, sr)
    w = ctx.upload(oq.TERNARY2, packed, M, K, w_scale=ws)
    import torch
    acc = torch.empty((B, M), dtype=torch.int32, device="cuda")
    y = ctx.gemm(w, dev(qr), dev(sr), acc=acc)
    assert np.array_equal(host(acc), accr)
    assert np.array_equal(host(y), yr)
    w.free()


# B >= 9: tcgen05 tensor-core path (u8 codes x s8 activations, TMEM accumulators)
@pytest.mark.parametrize("M,K,B", [(128, 128, 16), (256, 256, 17), (200, 384, 33), (96, 512, 64), (300, 640, 9),
                                   (1000, 2560, 12),
                                   (6912, 2560, 64), (2560, 6912, 100), (3840, 2560, 256),
                                   (1000, 1024, 300), (2560, 2560, 512)])
def test_gemm_tern2_tensor_core(ctx, oracle, M, K, B):
    import torch
    packed, ws, x = tern_case(oracle, M, K, B, seed=M + 3 * K + B)
    qr, sr = oracle.quantize_act(x)
    accr, yr = oracle.gemm_tern2(packed, M, K, ws, qr, sr)
    w = ctx.upload(oq.TERNARY2, packed, M, K, w_scale=ws)
    acc = torch.empty((B, M), dtype=torch.int32, device="cuda")
    y = ctx.gemm(w, dev(qr), dev(sr), acc=acc)
    assert np.array_equal(host(acc), accr)
    assert np.array_equal(host(y), yr)
    w.free()
    ctx.check_device()


def test_gemm_tern2_zero_and_extreme_activations(ctx, oracle):
    M, K, B = 96, 512, 4
    packed, ws, x = tern_case(oracle, M, K, B, seed=77)
    x[0] = 0.0            # s_x = 0 -> y = 0
    x[1] = 1.0            # all codes 127
    x[2, ::2] = -1e6      # saturating negatives
    qr, sr = oracle.quantize_act(x)
    accr, yr = oracle.gemm_tern2(packed, M, K, ws, qr, sr)
    w = ctx.upload(oq.TERNARY2, packed, M, K, w_scale=ws)
    q, s = ctx.quantize_act(dev(x))
    assert np.array_equal(host(q), qr)
    y = ctx.gemm(w, q, s)
    assert np.array_equal(host(y), yr)
    assert np.all(host(y)[0] == 0)


# ---------------------------------------------------------------- K3 sign
@pytest.mark.parametrize("M,K,B", [(4096, 4096, 1), (11008, 4096, 1), (4096, 4096, 8),
                                   (77, 256, 3), (50, 2176, 2), (16, 128, 1)])
def test_gemm_sign1_hadamard_matches_oracle(ctx, oracle, M, K, B):
    packed, sc, x = sign_case(oracle, M, K, B, seed=M + K + B)
    sg = oracle.signs(1234, K).astype(np.float32)
    qr, sr = oracle.quantize_act(x, sg, 128)
    accr, yr = oracle.gemm_sign1(packed, sc, M, K, qr, sr)
    w = ctx.upload(oq.SIGN1G128, packed, M, K, scales=sc)
    q, s = ctx.quantize_act(dev(x), signs=dev(sg), hadamard_block=128)
    assert np.array_equal(host(q), qr) and np.array_equal(host(s), sr)
    import torch
    acc = torch.empty((B, M, K // 128), dtype=torch.int32, device="cuda")
    y = ctx.gemm(w, q, s, acc=acc)
    assert np.array_equal(host(acc), accr)
    assert np.array_equal(host(y), yr)
    w.free()


@pytest.mark.parametrize("M", [4096, 11008])
def test_gemm_sign1_c3_batch32(ctx, oracle, M):
    K, B = 4096, 32
    packed, sc, x = sign_case(oracle, M, K, B, seed=M)
    qr, sr = oracle.quantize_act(x, None, 128)
    _, yr = oracle.gemm_sign1(packed, sc, M, K, qr, sr)
    w = ctx.upload(oq.SIGN1G128, packed, M, K, scales=sc)
    y = ctx.gemm_f32act(w, dev(x), hadamard_block=128)
    assert np.array_equal(host(y), yr)
    w.free()


@pytest.mark.parametrize("M,K,B", [(4096, 4096, 32), (11008, 4096, 32), (300, 384, 17), (77, 128, 16), (200, 512, 9),
                                   (256, 2176, 40), (128, 512, 100)])
def test_gemm_sign1_tensor_core(ctx, oracle, M, K, B):
    # batches from 9 tokens run the sign tensor-core kernel (one launch): the
    # per-group accumulators and the ascending-group fp32 fold must equal the
    # oracle's bit for bit; row counts off the 128-row tile, K off the 512-k
    # stage (a last stage of one group), token tiles of 16 and 32 with padding
    import torch
    packed, sc, x = sign_case(oracle, M, K, B, seed=3 * M + K + B)
    qr, sr = oracle.quantize_act(x, None, 0)
    accr, yr = oracle.gemm_sign1(packed, sc, M, K, qr, sr)
    w = ctx.upload(oq.SIGN1G128, packed, M, K, scales=sc)
    acc = torch.empty((B, M, K // 128), dtype=torch.int32, device="cuda")
    n0 = ctx.launch_count()
    y = ctx.gemm(w, dev(qr), dev(sr), acc=acc)
    assert ctx.launch_count() - n0 == 1
    assert np.array_equal(host(acc), accr)
    assert np.array_equal(host(y), yr)
    ctx.check_device()
    w.free()


@pytest.mark.parametrize("M,K,B,Z", [(256, 1664, 32, 4), (300, 2048, 17, 2), (128, 1152, 16, 4),
                                     (4096, 4096, 32, 4), (77, 512, 40, 4), (200, 1024, 64, 2),
                                     (128, 256, 16, 4), (256, 4096, 32, 2)])
def test_gemm_sign1_tensor_core_split(ctx, oracle, monkeypatch, M, K, B, Z):
    # the groups split over a cluster of Z CTAs (forced through
    # OUROQ_SIGN_KSPLIT), the fp32 fold chained from CTA to CTA: still the
    # oracle's order bit for bit. Ragged splits (13 groups over 4, 9 over 4),
    # token tiles of 16 and 32, two token tiles, one group per CTA, and splits
    # the launcher refuses (more CTAs than groups; more groups per CTA than
    # tensor memory holds) falling back to one CTA per row tile. With and
    # without the debug accumulators (two instantiations of the kernel).
    import torch
    monkeypatch.setenv("OUROQ_SIGN_KSPLIT", str(Z))
    packed, sc, x = sign_case(oracle, M, K, B, seed=5 * M + K + B + Z)
    qr, sr = oracle.quantize_act(x, None, 0)
    accr, yr = oracle.gemm_sign1(packed, sc, M, K, qr, sr)
    w = ctx.upload(oq.SIGN1G128, packed, M, K, scales=sc)
    acc = torch.empty((B, M, K // 128), dtype=torch.int32, device="cuda")
    y1 = ctx.gemm(w, dev(qr), dev(sr), acc=acc)
    y2 = ctx.gemm(w, dev(qr), dev(sr))
    assert np.array_equal(host(acc), accr)
    assert np.array_equal(host(y1), yr)
    assert np.array_equal(host(y2), yr)
    ctx.check_device()
    w.free()


# ---------------------------------------------------------------- grouped / host mirrors
def test_gemm_group_c2_layer(ctx, oracle):
    shapes = [(3840, 2560), (2560, 2560), (6912, 2560), (6912, 2560), (2560, 6912)]
    B = 1
    ws_, qs, ss, ys, want = [], [], [], [], []
    import torch
    for i, (M, K) in enumerate(shapes):
        packed, wsc, x = tern_case(oracle, M, K, B, seed=300 + i)
        qr, sr = oracle.quantize_act(x)
        want.append(oracle.gemm_tern2(packed, M, K, wsc, qr, sr)[1])
        ws_.append(ctx.upload(oq.TERNARY2, packed, M, K, w_scale=wsc))
        qs.append(dev(qr))
        ss.append(dev(sr))
        ys.append(torch.empty((B, M), dtype=torch.float32, device="cuda"))
    ctx.gemm_group(ws_, qs, ss, ys)
    for y, yr in zip(ys, want):
        assert np.array_equal(host(y), yr)
    for w in ws_:
        w.free()


@pytest.mark.parametrize("B", [1, 2, 3, 4, 5, 8])
def test_gemm_group_f32act_c2_layer(ctx, oracle, B):
    # up to eight tokens: one fused stream-GEMV launch for the five projections
    # (fp32 activations quantised in the prologue, each distinct input once per
    # CTA or cluster; four tiles a stage up to two tokens, two up to four, one
    # beyond)
    import torch
    shapes = [(3840, 2560), (2560, 2560), (6912, 2560), (6912, 2560), (2560, 6912)]
    inputs = [oracle.normals(400 + i, B * k).reshape(B, k) for i, k in enumerate([2560, 2560, 2560, 6912])]
    dev_inputs = [dev(x) for x in inputs]  # gate and up share one input buffer
    input_of = [0, 1, 2, 2, 3]
    ws_, xs, ys, want = [], [], [], []
    for i, (M, K) in enumerate(shapes):
        packed, wsc, _ = tern_case(oracle, M, K, 1, seed=500 + i)
        x = inputs[input_of[i]]
        qr, sr = oracle.quantize_act(x)
        want.append(oracle.gemm_tern2(packed, M, K, wsc, qr, sr)[1])
        ws_.append(ctx.upload(oq.TERNARY2, packed, M, K, w_scale=wsc))
        xs.append(dev_inputs[input_of[i]])
        ys.append(torch.empty((B, M), dtype=torch.float32, device="cuda"))
    n0 = ctx.launch_count()
    ctx.gemm_group_f32act(ws_, xs, ys)
    assert ctx.launch_count() - n0 == 1
    for y, yr in zip(ys, want):
        assert np.array_equal(host(y), yr)
    for w in ws_:
        w.free()


@pytest.mark.parametrize("B", [11, 16, 64, 100])
def test_gemm_group_tensor_core_c2_layer(ctx, oracle, B):
    # from 9 tokens the five projections of a layer run as ONE tensor-core
    # launch over every matrix's row tiles (each CTA finds its matrix, K of
    # 2560 and 6912 in one grid); the fp32 entry quantises the four distinct
    # inputs in one launch first
    import torch
    shapes = [(3840, 2560), (2560, 2560), (6912, 2560), (6912, 2560), (2560, 6912)]
    inputs = [oracle.normals(700 + i, B * k).reshape(B, k) for i, k in enumerate([2560, 2560, 2560, 6912])]
    input_of = [0, 1, 2, 2, 3]
    ws_, want, qs, ss = [], [], [], []
    for i, (M, K) in enumerate(shapes):
        packed, wsc, _ = tern_case(oracle, M, K, 1, seed=800 + i)
        qr, sr = oracle.quantize_act(inputs[input_of[i]])
        want.append(oracle.gemm_tern2(packed, M, K, wsc, qr, sr)[1])
        ws_.append(ctx.upload(oq.TERNARY2, packed, M, K, w_scale=wsc))
        qs.append(dev(qr))
        ss.append(dev(sr))
    ys = [torch.empty((B, M), dtype=torch.float32, device="cuda") for M, _ in shapes]
    n0 = ctx.launch_count()
    ctx.gemm_group(ws_, qs, ss, ys)
    assert ctx.launch_count() - n0 == 1
    for y, yr in zip(ys, want):
        assert np.array_equal(host(y), yr)
    xd = [dev(x) for x in inputs]
    ys2 = [torch.empty((B, M), dtype=torch.float32, device="cuda") for M, _ in shapes]
    n0 = ctx.launch_count()
    ctx.gemm_group_f32act(ws_, [xd[input_of[i]] for i in range(len(shapes))], ys2)
    assert ctx.launch_count() - n0 == 2  # quantise + one grouped tensor-core launch
    for y, yr in zip(ys2, want):
        assert np.array_equal(host(y), yr)
    for w in ws_:
        w.free()
    ctx.check_device()


def test_gemm_group_sign_tensor_core(ctx, oracle):
    # sign weights from 9 tokens in a group: one tensor-core launch per matrix
    import torch
    B = 32
    shapes = [(300, 1024), (4096, 4096)]
    ws_, want, qs, ss = [], [], [], []
    for i, (M, K) in enumerate(shapes):
        packed, sc, x = sign_case(oracle, M, K, B, seed=900 + i)
        qr, sr = oracle.quantize_act(x, None, 0)
        want.append(oracle.gemm_sign1(packed, sc, M, K, qr, sr)[1])
        ws_.append(ctx.upload(oq.SIGN1G128, packed, M, K, scales=sc))
        qs.append(dev(qr))
        ss.append(dev(sr))
    ys = [torch.empty((B, M), dtype=torch.float32, device="cuda") for M, _ in shapes]
    ctx.gemm_group(ws_, qs, ss, ys)
    for y, yr in zip(ys, want):
        assert np.array_equal(host(y), yr)
    for w in ws_:
        w.free()


@pytest.mark.parametrize("M,K,B", [(300, 2560, 3), (77, 6912, 6), (1000, 1152, 7), (33, 128, 8)])
def test_stream_gemv_batches_exact(ctx, oracle, M, K, B):
    # three to eight tokens through the one-launch stream GEMV: rows off the
    # 32-row tile, K of one 128-value unit, a token of zeros (scale 0) and
    # outliers; codes, sums and outputs equal the oracle's bit for bit
    x = oracle.outliers(M + B, oracle.normals(K + B, B * K), 0.01, 20.0).reshape(B, K)
    x[B - 1] = 0.0
    packed, ws, _ = tern_case(oracle, M, K, 1, seed=M * B + K)
    qr, sr = oracle.quantize_act(x)
    _, yr = oracle.gemm_tern2(packed, M, K, ws, qr, sr)
    w = ctx.upload(oq.TERNARY2, packed, M, K, w_scale=ws)
    n0 = ctx.launch_count()
    y = ctx.gemm_f32act(w, dev(x))
    assert ctx.launch_count() - n0 == 1
    assert np.array_equal(host(y), yr)
    w.free()


@pytest.mark.parametrize("block", [64, 128, 1024])
@pytest.mark.parametrize("M,K,B", [(4096, 4096, 1), (11008, 4096, 1), (300, 2048, 3)])
def test_fused_hadamard_sign_gemv(ctx, oracle, M, K, B, block):
    packed, sc, x = sign_case(oracle, M, K, B, seed=M + block)
    sg = oracle.signs(77, K).astype(np.float32)
    qr, sr = oracle.quantize_act(x, sg, block)
    _, yr = oracle.gemm_sign1(packed, sc, M, K, qr, sr)
    w = ctx.upload(oq.SIGN1G128, packed, M, K, scales=sc)
    y = ctx.gemm_f32act(w, dev(x), signs=dev(sg), hadamard_block=block)
    assert np.array_equal(host(y), yr)
    w.free()


@pytest.mark.parametrize("M,K,B", [(8192, 28672, 1), (1024, 28672, 2), (2048, 8192, 2), (1024, 28672, 4)])
def test_fused_wide_rows_exact(ctx, oracle, M, K, B):
    # one fused launch quantising rows too wide for one round of loads per
    # warp (28672 values = 224 units of 128): the later rounds must give the
    # same codes, scales and sums as the oracle's quantiser
    packed, ws, x = tern_case(oracle, M, K, B, seed=M + K + B)
    qr, sr = oracle.quantize_act(x)
    _, yr = oracle.gemm_tern2(packed, M, K, ws, qr, sr)
    w = ctx.upload(oq.TERNARY2, packed, M, K, w_scale=ws)
    xd = dev(x)
    n0 = ctx.launch_count()
    y = ctx.gemm_f32act(w, xd)
    assert ctx.launch_count() - n0 == 1  # the fused path, not quantise + gemm
    assert np.array_equal(host(y), yr)
    w.free()


@pytest.mark.parametrize("B", [1, 2])
def test_fused_group_cluster_shared_quantisation(ctx, oracle, B):
    # rows of 28672 and 12800 values: the one-token GEMV quantises them once per
    # cluster of CTAs (each CTA a quarter of the units, codes, maxima and sums
    # exchanged through distributed shared memory). Clusters here mix inputs
    # (x0 and x1, x0 and x2) and the last one holds an empty CTA (11 tiles);
    # token 1 of x1 is all zeros (scale 0) and x0 carries outliers
    import torch
    shapes = [(100, 28672, 0), (70, 12800, 1), (40, 28672, 0), (33, 384, 2)]
    xs = [oracle.outliers(600, oracle.normals(601, B * 28672), 0.01, 20.0).reshape(B, 28672),
          oracle.normals(602, B * 12800).reshape(B, 12800),
          oracle.normals(603, B * 384).reshape(B, 384)]
    if B >= 2:
        xs[1][1] = 0.0
    xd = [dev(x) for x in xs]
    ws_, ys, want = [], [], []
    for i, (M, K, xi) in enumerate(shapes):
        packed, wsc, _ = tern_case(oracle, M, K, 1, seed=610 + i)
        qr, sr = oracle.quantize_act(xs[xi])
        want.append(oracle.gemm_tern2(packed, M, K, wsc, qr, sr)[1])
        ws_.append(ctx.upload(oq.TERNARY2, packed, M, K, w_scale=wsc))
        ys.append(torch.empty((B, M), dtype=torch.float32, device="cuda"))
    n0 = ctx.launch_count()
    ctx.gemm_group_f32act(ws_, [xd[xi] for _, _, xi in shapes], ys)
    assert ctx.launch_count() - n0 == 1
    for y, yr in zip(ys, want):
        assert np.array_equal(host(y), yr)
    for w in ws_:
        w.free()
    ctx.check_device()


def test_fused_group_rejects_oversized_activations(ctx, oracle):
    import torch
    packed, wsc, _ = tern_case(oracle, 64, 28672, 1, seed=3)
    w = ctx.upload(oq.TERNARY2, packed, 64, 28672, w_scale=wsc)
    x = torch.zeros((8, 28672), device="cuda")
    y = torch.empty((8, 64), device="cuda")
    with pytest.raises(oq.OuroqError) as e:
        ctx.gemm_group_f32act([w], [x], [y])
    assert e.value.status == 6
    w.free()


def test_host_mirrors_matvec_matmul(ctx, oracle):
    M, K = 1000, 2560
    packed, ws, x = tern_case(oracle, M, K, 5, seed=42)
    w = ctx.upload(oq.TERNARY2, packed, M, K, w_scale=ws)
    y1 = ctx.matvec_q(w, x[0])
    qr, sr = oracle.quantize_act(x)
    _, yr = oracle.gemm_tern2(packed, M, K, ws, qr, sr)
    assert np.array_equal(y1, yr[0])
    yk = ctx.matmul_q(w, x)
    assert yk.shape == (5, M)
    assert np.array_equal(yk, yr)
    with pytest.raises(oq.OuroqError):
        ctx.matvec_q(w, x[0, :100])
    w.free()


@pytest.mark.parametrize("fmt,k", [("tern", 1), ("tern", 5), ("tern", 12), ("sign", 1), ("sign", 3)])
def test_host_mirrors_page_locked_outputs(ctx, oracle, fmt, k):
    # ouroq_matvec_q / ouroq_matmul_q through the C ABI with page-locked host
    # buffers (as a caller that registers its buffers passes them): up to
    # k = 8 the kernel stores into y directly, from 9 y is copied back; the
    # NaN fill shows every element is written
    import torch
    M, K = 700, 2560
    if fmt == "tern":
        packed, ws, x = tern_case(oracle, M, K, k, seed=300 + k)
        qr, sr = oracle.quantize_act(x)
        yr = oracle.gemm_tern2(packed, M, K, ws, qr, sr)[1]
        w = ctx.upload(oq.TERNARY2, packed, M, K, w_scale=ws)
    else:
        packed, sc, x = sign_case(oracle, M, K, k, seed=400 + k)
        qr, sr = oracle.quantize_act(x)
        yr = oracle.gemm_sign1(packed, sc, M, K, qr, sr)[1]
        w = ctx.upload(oq.SIGN1G128, packed, M, K, scales=sc)
    xh = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).pin_memory()
    yh = torch.full((k, M), float("nan"), dtype=torch.float32).pin_memory()
    ctx._check(ctx.lib.ouroq_matmul_q(ctx.ctx, w.handle, xh.data_ptr(), k, yh.data_ptr()))
    assert np.array_equal(yh.numpy(), yr)
    if k == 1:
        yh.fill_(float("nan"))
        ctx._check(ctx.lib.ouroq_matvec_q(ctx.ctx, w.handle, xh.data_ptr(), yh.data_ptr()))
        assert np.array_equal(yh.numpy(), yr)
    w.free()
    ctx.check_device()


@pytest.mark.parametrize("k", [1, 2, 5, 20])
def test_host_group_call_matches_oracle(ctx, oracle, k):
    # ouroq_matmul_q_group: the projections of one layer call (shapes of the
    # BitNet-2B layer scaled down in rows, gate and up sharing their input) in
    # one synchronous host-buffer call; every entry equals the oracle's
    # product, with pageable numpy buffers and with page-locked buffers that
    # sit back to back (the bench's e2e path)
    import torch
    shapes = [(384, 2560, 0), (256, 2560, 1), (700, 2560, 2), (700, 2560, 2), (256, 6912, 3)]
    xs = [oracle.normals(90 + i, k * K).reshape(k, K) for i, K in enumerate([2560, 2560, 2560, 6912])]
    ws, want = [], []
    for i, (M, K, xi) in enumerate(shapes):
        wt = oracle.ternary(70 + i, M * K).reshape(M, K)
        wsc = oracle.absmean_scale(wt, 0.02)
        ws.append(ctx.upload(oq.TERNARY2, oracle.pack_tern2(wt), M, K, w_scale=wsc))
        qr, sr = oracle.quantize_act(xs[xi])
        want.append(oracle.gemm_tern2(oracle.pack_tern2(wt), M, K, wsc, qr, sr)[1])
    got = ctx.matmul_q_group(ws, [xs[xi] for _, _, xi in shapes])
    for g, r in zip(got, want):
        assert np.array_equal(g, r)
    xcat = torch.from_numpy(np.concatenate([x.reshape(-1) for x in xs])).pin_memory()
    off = np.cumsum([0] + [x.size for x in xs])
    ycat = torch.empty(sum(k * M for M, _, _ in shapes), dtype=torch.float32).pin_memory()
    yoff = np.cumsum([0] + [k * M for M, _, _ in shapes])
    ys = [ycat[yoff[i]:yoff[i + 1]] for i in range(len(shapes))]
    ctx.matmul_q_group(ws, [xcat[off[xi]:off[xi + 1]] for _, _, xi in shapes], ys)
    for y, r in zip(ys, want):
        assert np.array_equal(y.numpy().reshape(r.shape), r)
    # page-locked outputs but one pageable: the call stages them all instead
    # of storing into the page-locked ones directly
    ycat.zero_()
    mixed = ys[:-1] + [np.empty((k, shapes[-1][0]), dtype=np.float32)]
    ctx.matmul_q_group(ws, [xcat[off[xi]:off[xi + 1]] for _, _, xi in shapes], mixed)
    for y, r in zip(mixed, want):
        yn = y if isinstance(y, np.ndarray) else y.numpy()
        assert np.array_equal(yn.reshape(r.shape), r)
    # page-locked inputs off the 16-byte grid (the device stage's slots stay
    # aligned for the kernels)
    xodd = torch.empty(xcat.numel() + 1, dtype=torch.float32).pin_memory()
    xodd[1:].copy_(xcat)
    ycat.zero_()
    ctx.matmul_q_group(ws, [xodd[1 + off[xi]:1 + off[xi + 1]] for _, _, xi in shapes], ys)
    for y, r in zip(ys, want):
        assert np.array_equal(y.numpy().reshape(r.shape), r)
    with pytest.raises(oq.OuroqError):
        ctx.matmul_q_group(ws[:1], [xs[0][:, :100]])
    for w in ws:
        w.free()
    ctx.check_device()


def test_empty_batch_is_a_no_op(ctx, oracle):
    # matmul_q with k = 0 columns returns an empty vector (ops.rs:219-230)
    import torch
    packed, ws, _ = tern_case(oracle, 64, 256, 1, seed=2)
    w = ctx.upload(oq.TERNARY2, packed, 64, 256, w_scale=ws)
    assert ctx.matmul_q(w, np.empty((0, 256), np.float32)).shape == (0, 64)
    assert ctx.gemm_f32act(w, torch.empty((0, 256), device="cuda")).shape == (0, 64)
    q = torch.empty((0, 256), dtype=torch.int8, device="cuda")
    assert ctx.gemm(w, q, torch.empty(0, device="cuda")).shape == (0, 64)
    w.free()
    ctx.check_device()


# ---------------------------------------------------------------- C5 sizes
@pytest.mark.parametrize("M,K", [(28672, 8192), (8192, 28672)])
def test_c5_shapes_batch1_exact(ctx, oracle, M, K):
    packed, ws, x = tern_case(oracle, M, K, 1, seed=M ^ K)
    qr, sr = oracle.quantize_act(x)
    accr, yr = oracle.gemm_tern2(packed, M, K, ws, qr, sr)
    w = ctx.upload(oq.TERNARY2, packed, M, K, w_scale=ws)
    import torch
    acc = torch.empty((1, M), dtype=torch.int32, device="cuda")
    y = ctx.gemm(w, dev(qr), dev(sr), acc=acc)
    assert np.array_equal(host(acc), accr)
    assert np.array_equal(host(y), yr)
    w.free()


def _epilogue(acc, w_scale, s_x):
    """The oracle's fp32 epilogue y = ((float)acc * w_scale) * s_x, each product
    rounded to fp32 on its own (oracle/oracle.h)."""
    a = acc.astype(np.float32)
    return ((a * np.float32(w_scale)).astype(np.float32) * s_x[:, None].astype(np.float32)).astype(np.float32)


@pytest.mark.parametrize("M,K,B", [(8192, 28672, 16), (28672, 8192, 16), (8192, 28672, 256),
                                   (28672, 8192, 256)])
def test_c5_batched_exact(ctx, oracle, M, K, B):
    # configuration 5 at its full size through the batched paths (B = 16 and
    # 256: the tensor-core GEMM). acc must equal the exact integer product
    # (float64 on the GPU: every partial sum is an integer below 2^53) and y
    # the oracle's epilogue applied to it, bit for bit.
    import torch
    wt = oracle.ternary(555 + B, M * K).reshape(M, K)
    ws = float(oracle.absmean_scale(wt, 0.02))
    x = oracle.normals(556 + B, B * K).reshape(B, K)
    qr, sr = oracle.quantize_act(x)
    w = ctx.upload(oq.TERNARY2, oracle.pack_tern2(wt), M, K, w_scale=ws)
    acc = torch.empty((B, M), dtype=torch.int32, device="cuda")
    y = ctx.gemm(w, dev(qr), dev(sr), acc=acc)
    wd = dev(wt).double()
    exact = dev(qr).double() @ wd.T
    del wd
    assert torch.equal(acc.double(), exact)
    assert np.array_equal(host(y), _epilogue(host(acc), ws, sr))
    w.free()
    ctx.check_device()


@pytest.mark.parametrize("M,K", [(3840, 2560), (2560, 2560), (6912, 2560), (2560, 6912)])
def test_c2_layer_shapes_batch512(ctx, oracle, M, K):
    # configuration 2 at its largest batch, every projection shape of the layer
    # (gate and up share 6912 x 2560), against the oracle (threaded GEMM for y,
    # exact integer product for acc)
    import torch
    B = 512
    packed, ws, x = tern_case(oracle, M, K, B, seed=M + K + 512)
    qr, sr = oracle.quantize_act(x)
    yr = oracle.gemm_tern2_mt(packed, M, K, ws, qr, sr)
    wt = oracle.ternary(M + K + 512, M * K).reshape(M, K)
    w = ctx.upload(oq.TERNARY2, packed, M, K, w_scale=ws)
    acc = torch.empty((B, M), dtype=torch.int32, device="cuda")
    y = ctx.gemm(w, dev(qr), dev(sr), acc=acc)
    assert torch.equal(acc.double(), dev(qr).double() @ dev(wt).double().T)
    assert np.array_equal(host(y), yr)
    assert np.array_equal(host(ctx.gemm_f32act(w, dev(x))), yr)
    w.free()


# ---------------------------------------------------------------- errors
def test_error_behaviour(ctx, oracle):
    with pytest.raises(oq.OuroqError) as e:
        ctx.upload(oq.TERNARY2, np.zeros((4, 25), np.uint8), 4, 100)
    assert e.value.status == 1
    packed, ws, x = tern_case(oracle, 64, 256, 1, seed=1)
    w = ctx.upload(oq.TERNARY2, packed, 64, 256, w_scale=ws)
    import torch
    qbuf = torch.zeros(2 * 256 + 16, dtype=torch.int8, device="cuda")
    q_mis = qbuf[1:257].view(1, 256)
    s = torch.ones(1, device="cuda")
    with pytest.raises(oq.OuroqError) as e:
        ctx.gemm(w, q_mis, s)
    assert e.value.status == 2
    with pytest.raises(oq.OuroqError) as e:
        ctx.quantize_act(dev(np.zeros((1, 384), np.float32)), hadamard_block=256)
    assert e.value.status == 1
    w.free()
    ctx.check_device()
