"""Golden fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py).

CPU: the oracle still reproduces every committed array bit for bit, so a
change to the oracle cannot silently move the parity target.
GPU: the CUDA path, called through the C ABI, reproduces the same arrays:
int32 accumulators bit-exact, fp32 outputs and rotations exactly (which is
within the 1e-5 relative bound of the contract).
"""
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


# ---------------------------------------------------------------- CPU: oracle pinned
def test_oracle_reproduces_quant(oracle):
    g = load("quant")
    for blk in (0, 64, 128):
        q, s = oracle.quantize_act(g["x"], g["signs"] if blk else None, blk)
        assert np.array_equal(q, g[f"q_b{blk}"])
        assert np.array_equal(s, g[f"s_b{blk}"])
    assert np.all(g["q_b0"][2] == 0) and g["s_b0"][2] == 0.0


def test_oracle_reproduces_rotate(oracle):
    g = load("rotate")
    for blk in (32, 128, 1024):
        assert np.array_equal(oracle.rotate_fwd(g[f"x_b{blk}"], g[f"signs_b{blk}"], blk),
                              g[f"fwd_b{blk}"])
        assert np.array_equal(oracle.rotate_inv(g[f"x_b{blk}"], g[f"signs_b{blk}"], blk),
                              g[f"inv_b{blk}"])


def test_oracle_reproduces_products(oracle):
    g = load("tern2")
    for tag in ("a", "b"):
        M, K, _ = (int(v) for v in g[f"{tag}_shape"])
        acc, y = oracle.gemm_tern2(g[f"{tag}_packed"], M, K, float(g[f"{tag}_w_scale"]),
                                   g[f"{tag}_q"], g[f"{tag}_s"])
        assert np.array_equal(acc, g[f"{tag}_acc"]) and np.array_equal(y, g[f"{tag}_y"])
    s = load("sign1")
    M, K, _ = (int(v) for v in s["shape"])
    acc, y = oracle.gemm_sign1(s["packed"], s["scales"], M, K, s["q"], s["s"])
    assert np.array_equal(acc, s["acc"]) and np.array_equal(y, s["y"])


def test_oracle_reproduces_reference_formats(oracle):
    g = load("refformat")
    o, i = (int(v) for v in g["tl1_shape"])
    assert np.array_equal(oracle.matvec_tl1_scalar(g["tl1_payload"], o, i, g["tl1_x"]),
                          g["tl1_scalar"])
    assert np.array_equal(oracle.matvec_tl1_sse(g["tl1_payload"], o, i, g["tl1_x"], 1),
                          g["tl1_sse"])
    assert np.array_equal(oracle.matmul_tl1_scalar(g["tl1_payload"], o, i, g["tl1_xk"], 3),
                          g["tl1_matmul_k3"])
    assert np.array_equal(oracle.matmul_tl1_sse(g["tl1_payload"], o, i, g["tl1_xk"], 3, 1),
                          g["tl1_matmul_sse_k3"])
    # the reference's own tolerance between the two accumulation orders (ops.rs:829)
    np.testing.assert_allclose(g["tl1_sse"], g["tl1_scalar"], rtol=1e-5, atol=1e-5)
    o, i = (int(v) for v in g["tq1_shape"])
    assert np.array_equal(oracle.matvec_tq1(g["tq1_payload"], o, i, g["tq1_x"], 1), g["tq1_y"])


# ---------------------------------------------------------------- GPU: kernels vs fixtures
def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    return t.detach().cpu().numpy()


@pytest.mark.gpu
def test_gpu_quant_golden(ctx):
    g = load("quant")
    for blk in (0, 64, 128):
        q, s = ctx.quantize_act(_dev(g["x"]), signs=_dev(g["signs"]) if blk else None,
                                hadamard_block=blk)
        assert np.array_equal(_host(q), g[f"q_b{blk}"])
        assert np.array_equal(_host(s), g[f"s_b{blk}"])


@pytest.mark.gpu
def test_gpu_rotate_golden(ctx):
    g = load("rotate")
    for blk in (32, 128, 1024):
        x = _dev(g[f"x_b{blk}"][None, :])
        sg = _dev(g[f"signs_b{blk}"])
        assert np.array_equal(_host(ctx.rotate(x, signs=sg, block=blk))[0], g[f"fwd_b{blk}"])
        assert np.array_equal(_host(ctx.rotate(x, signs=sg, block=blk, inverse=True))[0],
                              g[f"inv_b{blk}"])


@pytest.mark.gpu
def test_gpu_tern2_golden(ctx):
    import torch
    import ouroboros_b200 as oq
    g = load("tern2")
    for tag in ("a", "b"):  # b: B = 16 runs on the tensor cores
        M, K, B = (int(v) for v in g[f"{tag}_shape"])
        w = ctx.upload(oq.TERNARY2, g[f"{tag}_packed"], M, K, w_scale=float(g[f"{tag}_w_scale"]))
        acc = torch.empty((B, M), dtype=torch.int32, device="cuda")
        y = ctx.gemm(w, _dev(g[f"{tag}_q"]), _dev(g[f"{tag}_s"]), acc=acc)
        assert np.array_equal(_host(acc), g[f"{tag}_acc"])
        assert np.array_equal(_host(y), g[f"{tag}_y"])
        y2 = ctx.gemm_f32act(w, _dev(g[f"{tag}_x"]))
        assert np.array_equal(_host(y2), g[f"{tag}_y"])
        w.free()


@pytest.mark.gpu
def test_gpu_sign1_golden(ctx):
    import torch
    import ouroboros_b200 as oq
    s = load("sign1")
    M, K, B = (int(v) for v in s["shape"])
    w = ctx.upload(oq.SIGN1G128, s["packed"], M, K, scales=s["scales"])
    acc = torch.empty((B, M, K // 128), dtype=torch.int32, device="cuda")
    y = ctx.gemm(w, _dev(s["q"]), _dev(s["s"]), acc=acc)
    assert np.array_equal(_host(acc), s["acc"])
    assert np.array_equal(_host(y), s["y"])
    y2 = ctx.gemm_f32act(w, _dev(s["x"]), signs=_dev(s["signs"]), hadamard_block=int(s["block"]))
    assert np.array_equal(_host(y2), s["y"])
    w.free()
