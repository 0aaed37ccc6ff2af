"""Pins the CPU oracle to the reference's own known-answer tests (CPU only).

Each test restates one unit test of the reference, with the same generator,
inputs and tolerance, and runs it against oracle/oracle.c:

  hadamard.rs:96-172   five rotation tests
  dequant.rs:564-603   PTQ1_0 group decode vs an independent transcription
  dequant.rs:608-664   PTQ1_0 round trip vs the transcribed C quantiser (64 LCG groups)
  dequant.rs:667-677   PTQ1_0 trits in range
  dequant.rs:680-690   bf16 known values
  dequant.rs:693-702   f16 known values (incl. subnormal)
  ops.rs:782-798       F16 matmul_q == K x matvec_f16 (its payload restated)
  dequant.rs:705-726   TQ1_0 zero block and value set
  ops.rs:721-750       matmul_tl1 K=4 == K x matvec_tl1 (scalar and x86 K-column paths)
  ops.rs:801-838       fused matvec_tl1 == decode-then-dot

The int8-activation arithmetic has no reference test (it lives in the absent
bitnet-cpp submodule): it is checked here against an independent numpy
restatement instead, and marked parity-unpinned in the oracle header.
"""
import math

import numpy as np
import pytest


# ---------------------------------------------------------------- hadamard.rs
def naive_matrix(n, block):
    """hadamard.rs:72-87: H[i][j] = (-1)^popcount(i&j) / sqrt(N), block diagonal."""
    scale = np.float32(1.0) / np.sqrt(np.float32(block))
    m = np.zeros((n, n), np.float32)
    for start in range(0, n, block):
        for r in range(block):
            for c in range(block):
                p = bin(r & c).count("1")
                m[start + r, start + c] = -scale if p & 1 else scale
    return m


def mat_vec(m, x):
    return np.array([sum(float(m[r, c]) * float(x[c]) for c in range(len(x)))
                     for r in range(len(x))], np.float32)


def test_fwd_is_h_times_diag_s(oracle):
    # hadamard.rs:96-110
    block = n = 16
    x = np.array([((i * 11) % 7) - 3.0 for i in range(n)], np.float32)
    s = np.array([-1.0 if i % 3 == 0 else 1.0 for i in range(n)], np.float32)
    fast = oracle.rotate_fwd(x, s, block)
    ref = mat_vec(naive_matrix(n, block), x * s)
    assert np.all(np.abs(fast - ref) < 1e-4)


def test_inv_is_diag_s_times_h(oracle):
    # hadamard.rs:112-126
    block = n = 16
    x = np.array([((i * 5) % 9) - 4.0 for i in range(n)], np.float32)
    s = np.array([-1.0 if i % 4 == 0 else 1.0 for i in range(n)], np.float32)
    fast = oracle.rotate_inv(x, s, block)
    ref = mat_vec(naive_matrix(n, block), x) * s
    assert np.all(np.abs(fast - ref) < 1e-4)


def _roundtrip_inputs(n):
    x = np.array([((i * 91) % 23) * 0.37 - 4.0 for i in range(n)], np.float32)
    s = np.array([-1.0 if (i // 5) % 2 == 0 else 1.0 for i in range(n)], np.float32)
    return x, s


def test_fwd_inv_roundtrip_identity(oracle):
    # hadamard.rs:128-141
    block = 64
    x, s = _roundtrip_inputs(block * 2)
    y = oracle.rotate_fwd(oracle.rotate_inv(x, s, block), s, block)
    assert np.all(np.abs(x - y) < 1e-3)


def test_rotation_preserves_l2_norm(oracle):
    # hadamard.rs:143-158
    block = 64
    x, s = _roundtrip_inputs(block * 3)
    n0 = float(np.sum(x * x, dtype=np.float32))
    for y in (oracle.rotate_fwd(x, s, block), oracle.rotate_inv(x, s, block)):
        n1 = float(np.sum(y * y, dtype=np.float32))
        assert abs(n0 - n1) / n0 < 1e-4


def test_blockwise_independence(oracle):
    # hadamard.rs:160-172
    block = 32
    n = block * 2
    x = np.array([((i * 7) % 17) - 8.0 for i in range(n)], np.float32)
    s = np.ones(n, np.float32)
    a = oracle.rotate_fwd(x, s, block)
    xb = x.copy()
    xb[3] += 5.0
    b = oracle.rotate_fwd(xb, s, block)
    assert np.array_equal(a[block:], b[block:])


def test_rotate_rejects_bad_block(oracle):
    # hadamard.rs:33-37 (assert! on power-of-two block dividing the length)
    with pytest.raises(ValueError):
        oracle.rotate_fwd(np.zeros(96, np.float32), None, 48)
    with pytest.raises(ValueError):
        oracle.rotate_fwd(np.zeros(100, np.float32), None, 64)


# ---------------------------------------------------------------- dequant.rs
def _dig(byte, n, d):
    q = (byte * (1, 3, 9, 27, 81, 243)[n]) & 0xFF
    xi = (q * 3) >> 8
    return np.float32(xi - 1) * np.float32(d)


def test_tl1_group_matches_c_reference(oracle):
    # dequant.rs:564-603
    buf = np.zeros(28, np.uint8)
    for i in range(26):
        buf[i] = (i * 131 + 7) & 0xFF
    buf[26], buf[27] = 0x35, 0x3A
    fast = oracle.tl1_group(buf)
    d = oracle.f16_to_f32(int(buf[26]) | (int(buf[27]) << 8))
    qs, qh = buf[0:24], buf[24:26]
    expect = np.zeros(128, np.float32)
    for n in range(5):
        for m in range(16):
            expect[n * 16 + m] = _dig(int(qs[m]), n, d)
    for n in range(5):
        for m in range(8):
            expect[80 + n * 8 + m] = _dig(int(qs[16 + m]), n, d)
    for n in range(4):
        for h in range(2):
            expect[120 + n * 2 + h] = _dig(int(qh[h]), n, d)
    assert np.array_equal(fast, expect)
    assert np.all(np.isfinite(fast))


def quantize_group_ref(x):
    """dequant.rs:610-641: transcription of quantize_row_ptq1_0_ref (d = 1.0)."""
    blk = np.zeros(28, np.uint8)
    blk[27] = 0x3C
    xi = [int(round(v)) + 1 for v in x]

    def enc(q):
        return (q * 256 + 242) // 243

    for m in range(16):
        q = 0
        for n in range(5):
            q = q * 3 + xi[m + n * 16]
        blk[m] = enc(q)
    for m in range(8):
        q = 0
        for n in range(5):
            q = q * 3 + xi[80 + m + n * 8]
        blk[16 + m] = enc(q)
    for h in range(2):
        q = 0
        for m in range(4):
            q = q * 3 + xi[120 + h + m * 2]
        q *= 3
        blk[24 + h] = enc(q)
    return blk


def test_ptq1_roundtrip_vs_c_quantizer(oracle):
    # dequant.rs:608-664: 64 LCG groups, seed 0x12345678, then the all-zero group
    lcg = 0x12345678
    for _ in range(64):
        x = np.zeros(128, np.float32)
        for i in range(128):
            lcg = (lcg * 1664525 + 1013904223) & 0xFFFFFFFF
            x[i] = (-1.0, 0.0, 1.0)[(lcg >> 16) % 3]
        out = oracle.tl1_group(quantize_group_ref(x))
        assert np.array_equal(out, x), "roundtrip must be bit-exact"
    out = oracle.tl1_group(quantize_group_ref(np.zeros(128, np.float32)))
    assert np.all(out == 0.0)


def test_tl1_group_trits_in_range(oracle):
    # dequant.rs:667-677
    buf = np.zeros(28, np.uint8)
    for i in range(26):
        buf[i] = ((i * 29) & 0xFF) ^ ((i * 7) & 0xFF)
    buf[26], buf[27] = 0x00, 0x3C
    out = oracle.tl1_group(buf)
    assert np.all(np.isin(out, [-1.0, 0.0, 1.0]))


def test_f16_known_values(oracle):
    # dequant.rs:693-702
    f = oracle.f16_to_f32
    assert f(0x0000) == 0.0
    assert f(0x3C00) == 1.0
    assert f(0xBC00) == -1.0
    assert f(0x3800) == 0.5
    assert f(0x7C00) == math.inf
    # the reference compares in f32 arithmetic
    assert abs(np.float32(f(0x3555)) - np.float32(0.33325195)) < np.float32(1e-9)
    assert abs(np.float32(f(0x0001)) - np.float32(5.9604645e-8)) < np.float32(1e-12)


def test_f16_decode_matches_numpy_for_all_finite_patterns(oracle):
    bits = np.arange(0, 1 << 16, dtype=np.uint32)
    ref = bits.astype(np.uint16).view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(b)) for b in bits[::97]], np.float32)
    r = ref[::97]
    fin = np.isfinite(r)
    assert np.array_equal(got[fin], r[fin])


def test_bf16_known_values(oracle):
    # dequant.rs:680-690
    f = oracle.bf16_to_f32
    assert f(0x0000) == 0.0
    assert f(0x3F80) == 1.0
    assert f(0xBF80) == -1.0
    assert f(0x7F80) == math.inf
    assert f(0x4000) == 2.0
    assert abs(np.float32(f(0x3EAA)) - np.float32(0.33203125)) < np.float32(1e-6)


def _matvec_half_loop(payload, out_len, in_len, x, bf16):
    """matvec_f16 / matvec_bf16 (ops.rs:131-153, 600-620) as plain float32
    steps: s = s + w * x, the product and the sum rounded separately."""
    bits = np.ascontiguousarray(payload).view(np.uint16).reshape(out_len, in_len)
    if bf16:
        w = (bits.astype(np.uint32) << 16).view(np.float32)
    else:
        w = bits.view(np.float16).astype(np.float32)
    y = np.zeros(out_len, np.float32)
    for r in range(out_len):
        s = np.float32(0.0)
        for i in range(in_len):
            s = np.float32(s + np.float32(w[r, i] * np.float32(x[i])))
        y[r] = s
    return y


def matmul_fallback_payload(out_len, in_len):
    """ops.rs:785-790: the low two bytes of ((i % 17) - 8) * 0.25 as f32."""
    v = ((np.arange(out_len * in_len) % 17).astype(np.float32) - 8.0) * np.float32(0.25)
    return (v.view(np.uint32) & 0xFFFF).astype(np.uint16)


def test_matmul_q_fallback_payload(oracle):
    # ops.rs:782-798: x[i] = (i % 7) * 0.5 over two columns; each column is matvec_f16
    out_len, in_len = 16, 32
    payload = matmul_fallback_payload(out_len, in_len)
    x = ((np.arange(2 * in_len) % 7) * 0.5).astype(np.float32)
    for c in range(2):
        xc = x[c * in_len:(c + 1) * in_len]
        got = oracle.matvec_half(payload, out_len, in_len, xc)
        assert np.array_equal(got, _matvec_half_loop(payload, out_len, in_len, xc, False))


@pytest.mark.parametrize("bf16", [False, True])
def test_matvec_half_matches_loop(oracle, bf16):
    out_len, in_len = 23, 70
    payload = oracle.lcg_bytes(7 + bf16, out_len * in_len * 2).view(np.uint16).copy()
    # keep exponents tame so the chain stays finite (no NaN or inf patterns)
    payload = (payload & 0x807F) | 0x3F00 if bf16 else (payload & 0x83FF) | 0x3800
    x = oracle.normals(9, in_len)
    got = oracle.matvec_half(payload, out_len, in_len, x, bf16=bf16)
    want = _matvec_half_loop(payload, out_len, in_len, x, bf16)
    assert np.array_equal(got, want)


def test_finite_argmax_rules(oracle):
    # infer/mod.rs:70-83: NaN skipped, first maximum wins, 0 if all NaN
    nan, inf = float("nan"), float("inf")
    assert oracle.finite_argmax([1.0, 3.0, 2.0, 3.0]) == 1
    assert oracle.finite_argmax([nan, 0.5, nan, 0.7]) == 3
    assert oracle.finite_argmax([nan, nan, nan]) == 0
    assert oracle.finite_argmax([-inf, -inf]) == 0
    assert oracle.finite_argmax([-0.0, 0.0]) == 0
    assert oracle.finite_argmax([0.0, -0.0, -1.0]) == 0
    assert oracle.finite_argmax([-2.0, nan, inf, inf]) == 2


def test_tq1_values_are_ternary_scaled(oracle):
    # dequant.rs:705-715: zero qs with d = 1.0 decodes to -1 everywhere
    block = np.zeros(54, np.uint8)
    block[52], block[53] = 0x00, 0x3C
    v = oracle.tq1_block(block)
    assert v.size == 256 and np.all(v == -1.0)


def test_tq1_all_values_in_set(oracle):
    # dequant.rs:717-726
    block = np.zeros(54, np.uint8)
    for i in range(52):
        block[i] = (i * 7 + 3) & 0xFF
    block[52], block[53] = 0x00, 0x40
    v = oracle.tq1_block(block)
    assert np.all(np.isin(v, [-2.0, 0.0, 2.0]))


# ---------------------------------------------------------------- ops.rs
def _tl1_payload(out_len, in_len, shift):
    n = out_len * (in_len // 128) * 28
    i = np.arange(n, dtype=np.uint64)
    p = ((i * (0x9B ^ (i >> np.uint64(shift)))) & np.uint64(0xFF)).astype(np.uint8)
    g = p.reshape(-1, 28)
    g[:, 26] = 0x10
    g[:, 27] = 0x38
    return p


def test_matvec_tl1_fused_matches_reference(oracle):
    # ops.rs:801-838 (37 x 384, rel 1e-5), for both restated accumulation orders
    out_len, in_len = 37, 384
    payload = _tl1_payload(out_len, in_len, 7)
    x = np.array([((i % 7) - 3.0) * 0.5 for i in range(in_len)], np.float32)
    groups = in_len // 128
    for fused in (oracle.matvec_tl1_scalar(payload, out_len, in_len, x),
                  oracle.matvec_tl1_sse(payload, out_len, in_len, x)):
        for row in range(out_len):
            flat = np.concatenate([oracle.tl1_group(payload[(row * groups + g) * 28:(row * groups + g + 1) * 28])
                                   for g in range(groups)])
            want = np.float32(0.0)
            for a, b in zip(flat, x):
                want = np.float32(want + a * b)
            assert abs(fused[row] - want) / max(abs(want), 1e-9) < 1e-5


def test_matmul_tl1_k_columns_matches_matvec(oracle):
    # ops.rs:721-750 (97 x 384, K = 4, tol 1e-3 * max(|want|, 1))
    out_len, in_len, k = 97, 384, 4
    payload = _tl1_payload(out_len, in_len, 5)
    x = np.array([((i % 11) - 5.0) * 0.25 for i in range(k * in_len)], np.float32)
    scalar_k = oracle.matmul_tl1_scalar(payload, out_len, in_len, x, k)
    sse_k = oracle.matmul_tl1_sse(payload, out_len, in_len, x, k)
    for batched in (scalar_k, sse_k):
        for c in range(k):
            want = oracle.matvec_tl1_sse(payload, out_len, in_len, x[c * in_len:(c + 1) * in_len])
            got = batched[c * out_len:(c + 1) * out_len]
            assert np.all(np.abs(got - want) <= 1e-3 * np.maximum(np.abs(want), 1.0))
    # every partial sum of this fixture is a multiple of 129/1024 below 2^18
    # of them, exact in fp32: all accumulation orders agree bit for bit, which
    # pins the K-column path's decode and indexing
    assert np.array_equal(sse_k, scalar_k)


def _tl1_k_lanes(oracle, payload, out_len, in_len, x, k):
    """numpy statement of tl1_rows_avx2_k's order (ops.rs:381-481): two 4-lane
    accumulators per column over the whole row, a scalar tail sum, and
    y = tail + (hsum(lo) + hsum(hi)) with hsum(v) = (v0 + v2) + (v1 + v3)."""
    f32 = np.float32
    gpr = in_len // 128
    x = x.reshape(k, in_len)
    y = np.empty(k * out_len, f32)
    hs = lambda v: f32(f32(v[0] + v[2]) + f32(v[1] + v[3]))  # noqa: E731
    for r in range(out_len):
        lo = np.zeros((k, 4), f32)
        hi = np.zeros((k, 4), f32)
        tail = np.zeros(k, f32)
        for g in range(gpr):
            w = oracle.tl1_group(payload[(r * gpr + g) * 28:(r * gpr + g + 1) * 28])
            xg = x[:, g * 128:(g + 1) * 128]
            for n in range(5):
                for base, acc in ((n * 16, lo), (n * 16 + 4, hi), (n * 16 + 8, lo),
                                  (n * 16 + 12, hi), (80 + n * 8, lo), (80 + n * 8 + 4, hi)):
                    acc[:] = (w[base:base + 4] * xg[:, base:base + 4]) + acc
            for n in range(4):
                for m in range(2):
                    i = 120 + n * 2 + m
                    tail[:] = tail + w[i] * xg[:, i]
        for c in range(k):
            y[c * out_len + r] = f32(tail[c] + f32(hs(lo[c]) + hs(hi[c])))
    return y


def test_matmul_tl1_sse_k_order(oracle):
    # random scales and activations: the K-column order differs from the
    # per-group matvec order, and the restatement must follow it exactly
    out_len, in_len, k = 23, 512, 3
    payload = oracle.lcg_bytes(123, out_len * (in_len // 128) * 28)
    g = payload.reshape(-1, 28)
    g[:, 27] &= 0x3B  # finite f16 scales below 1
    x = oracle.normals(124, k * in_len)
    got = oracle.matmul_tl1_sse(payload, out_len, in_len, x, k, threads=3)
    assert np.array_equal(got, _tl1_k_lanes(oracle, payload, out_len, in_len, x, k))


def test_matvec_tq1_matches_decode_then_dot(oracle):
    # ops.rs:101-128 restated: dequant_tq1_row then dot, threaded over rows
    out_len, in_len = 19, 512
    payload = oracle.lcg_bytes(99, out_len * (in_len // 256) * 54)
    blocks = payload.reshape(-1, 54)
    blocks[:, 53] %= 0x70  # keep the f16 scale finite, like l1_parity.rs:18-25
    x = oracle.normals(5, in_len)
    y = oracle.matvec_tq1(payload, out_len, in_len, x, threads=3)
    for r in range(out_len):
        row = np.concatenate([oracle.tq1_block(blocks[r * 2 + b]) for b in range(2)])
        s = np.float32(0.0)
        for a, b in zip(row, x):
            s = np.float32(s + a * b)
        assert y[r] == s


# ------------------------------------------- int8 path (parity unpinned)
def np_quantize(x):
    amax = np.max(np.abs(x), axis=1).astype(np.float32)
    s = (amax / np.float32(127.0)).astype(np.float32)
    q = np.zeros_like(x, dtype=np.int8)
    nz = s != 0
    r = np.rint((x[nz] / s[nz, None]).astype(np.float32))
    q[nz] = np.clip(r, -127, 127).astype(np.int8)
    return q, s


def test_quantize_matches_numpy(oracle):
    x = oracle.normals(11, 5 * 640).reshape(5, 640)
    x[1] = 0.0                     # zero row -> s = 0, q = 0
    x[2, 7] = 1e4                  # one huge outlier
    x[3, :] = 0.5                  # constant row (ties at exactly 127)
    q, s = oracle.quantize_act(x)
    qr, sr = np_quantize(x)
    assert np.array_equal(s, sr)
    assert np.array_equal(q, qr)
    assert s[1] == 0 and np.all(q[1] == 0)
    assert np.all(q[3] == 127)


def test_quantize_with_rotation_matches_numpy(oracle):
    K, block = 512, 128
    x = oracle.outliers(3, oracle.normals(12, 2 * K), 0.01, 20.0).reshape(2, K)
    sg = oracle.signs(4, K).astype(np.float32)
    q, s, xr = oracle.quantize_act(x, sg, block, want_rot=True)
    for b in range(2):
        assert np.array_equal(xr[b], oracle.rotate_fwd(x[b], sg, block))
    H = naive_matrix(K, block).astype(np.float64)
    exact = (H @ (x * sg).T.astype(np.float64)).T
    assert np.allclose(xr, exact, rtol=1e-5, atol=1e-5 * np.abs(exact).max())
    qr, sr = np_quantize(xr)
    assert np.array_equal(q, qr) and np.array_equal(s, sr)


def test_gemm_tern2_matches_numpy(oracle):
    M, K, B = 67, 384, 3
    w = oracle.ternary(21, M * K).reshape(M, K)
    x = oracle.normals(22, B * K).reshape(B, K)
    q, s = oracle.quantize_act(x)
    ws = oracle.absmean_scale(w, 0.02)
    acc, y = oracle.gemm_tern2(oracle.pack_tern2(w), M, K, ws, q, s)
    ref = q.astype(np.int64) @ w.astype(np.int64).T
    assert np.array_equal(acc, ref)
    yr = (acc.astype(np.float32) * np.float32(ws)).astype(np.float32) * s[:, None]
    assert np.array_equal(y, yr.astype(np.float32))
    ymt = oracle.gemm_tern2_mt(oracle.pack_tern2(w), M, K, ws, q, s, threads=4)
    assert np.array_equal(ymt, y)


def test_gemm_sign1_matches_numpy(oracle):
    M, K, B = 45, 512, 2
    G = K // 128
    w = oracle.signs(31, M * K).reshape(M, K)
    sc = oracle.group_scales(32, M * G, 0.02)
    x = oracle.normals(33, B * K).reshape(B, K)
    q, s = oracle.quantize_act(x)
    acc, y = oracle.gemm_sign1(oracle.pack_sign1(w), sc, M, K, q, s)
    ref = np.einsum("mgk,bgk->bmg", w.reshape(M, G, 128).astype(np.int64),
                    q.reshape(B, G, 128).astype(np.int64))
    assert np.array_equal(acc, ref)
    scf = sc.view(np.float16).astype(np.float32).reshape(M, G)
    yr = np.zeros((B, M), np.float32)
    for g in range(G):
        yr = (yr + (acc[:, :, g].astype(np.float32) * scf[None, :, g]).astype(np.float32)).astype(np.float32)
    yr = (yr * s[:, None]).astype(np.float32)
    assert np.array_equal(y, yr)
    ymt = oracle.gemm_sign1_mt(oracle.pack_sign1(w), sc, M, K, q, s, threads=3)
    assert np.array_equal(ymt, y)


def test_packers_bit_order(oracle):
    w = np.array([[-1, 0, 1, 1, 0, 0, -1, 1] * 16], np.int8)  # K = 128
    p = oracle.pack_tern2(w)
    # element k in byte k/4, bits 2*(k%4), code = w + 1
    assert p[0, 0] == (0 | 1 << 2 | 2 << 4 | 2 << 6)
    assert p[0, 1] == (1 | 1 << 2 | 0 << 4 | 2 << 6)
    sg = np.where(w > 0, 1, -1).astype(np.int8)
    ps = oracle.pack_sign1(sg)
    bits = [1 if v > 0 else 0 for v in sg[0, :8]]
    assert ps[0, 0] == sum(b << i for i, b in enumerate(bits))
