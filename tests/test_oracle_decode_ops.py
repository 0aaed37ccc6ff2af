"""The oracle's restatement of the decode step's host ops (ops.rs:11-60,
infer/mod.rs:338-365), pinned by the reference's own unit tests (ops.rs:629-694),
and the anchor that ties the GPU decode tests to the reference's order: those
tests compare the kernels with float64 torch formulas (`_ref_rms`,
`_rope_ref`, `_attn_ref` in tests/test_gpu_decode.py); here each formula is
checked against the fp32 restatement of the reference's own order on the
same inputs, within a fifth of the tolerance the GPU test allows, so a kernel
inside the GPU tolerance of the formula is inside 1.2 times it of the
reference."""
import math

import numpy as np
import pytest
import torch

from test_gpu_decode import _attn_ref, _ref_rms, _rope_ref


# ---------------------------------------------------------------- ops.rs:629-694
def test_rmsnorm_basic(oracle):
    y = oracle.rmsnorm([1.0, 2.0, 3.0, 4.0], [1.0] * 4, 1e-5)
    ms = np.float32((1.0 + 4.0 + 9.0 + 16.0) / 4.0)
    inv = np.float32(1.0) / np.sqrt(ms + np.float32(1e-5))
    assert abs(y[0] - 1.0 * inv) < 1e-6 and abs(y[3] - 4.0 * inv) < 1e-6


def test_rmsnorm_weight_scale(oracle):
    y = oracle.rmsnorm([3.0, 3.0], [2.0, 0.5], 0.0)
    assert abs(y[0] - 2.0) < 1e-6 and abs(y[1] - 0.5) < 1e-6


def test_rope_preserves_norm(oracle):
    v0 = np.array([0.1 * i + 0.05 for i in range(8)], np.float32)
    v = oracle.rope_neox(v0, 5, 8, 500000.0)
    assert abs(float(np.sum(v0 * v0)) - float(np.sum(v * v))) < 1e-4
    assert not np.array_equal(v, v0)


def test_rope_position_zero_is_identity(oracle):
    v0 = np.array([0.25 * i for i in range(8)], np.float32)
    assert np.all(np.abs(oracle.rope_neox(v0, 0, 8, 500000.0) - v0) < 1e-5)


def test_dot(oracle):
    assert oracle.dot([1.0, 2.0], [5.0, 6.0]) == 17.0
    assert oracle.dot([0.0] * 4, [1.0] * 4) == 0.0


def test_softmax_sums_to_one(oracle):
    v = oracle.softmax([1.0, 2.0, 3.0, -10.0])
    assert abs(float(v.sum()) - 1.0) < 1e-6 and v[3] < 1e-4 and v[2] > v[0]


def test_silu(oracle):
    assert abs(oracle.silu(0.0)) < 1e-9
    assert abs(oracle.silu(10.0) - 10.0) < 1e-3
    assert abs(oracle.silu(-10.0)) < 1e-3


# ---------------------------------------------------------------- anchors
@pytest.mark.parametrize("n", [2560, 6912])
def test_rmsnorm_formula_matches_reference_order(oracle, n):
    g = torch.Generator().manual_seed(n)
    x = torch.randn((3, n), generator=g)
    r = torch.randn((3, n), generator=g)
    w = 1 + 0.02 * torch.randn(n, generator=g)
    got = _ref_rms(x + r, w)  # the GPU test's formula (rtol 1e-5, atol 1e-6 there)
    v = (x + r).numpy()
    want = np.stack([oracle.rmsnorm(v[b], w.numpy(), 1e-5) for b in range(3)])
    np.testing.assert_allclose(got.numpy(), want, rtol=2e-6, atol=2e-7)


def test_swiglu_norm_formula_matches_reference_order(oracle):
    n = 6912
    g = torch.Generator().manual_seed(5)
    gate = 3 * torch.randn((2, n), generator=g)
    up = torch.randn((2, n), generator=g)
    w = 1 + 0.02 * torch.randn(n, generator=g)
    a = gate.double() / (1 + torch.exp(-gate.double())) * up.double()
    got = _ref_rms(a.float(), w)
    for b in range(2):
        act = np.array([oracle.silu(float(gv)) for gv in gate[b].numpy()], np.float32) * up[b].numpy()
        want = oracle.rmsnorm(act, w.numpy(), 1e-5)
        np.testing.assert_allclose(got[b].numpy(), want, rtol=2e-6, atol=2e-7)


@pytest.mark.parametrize("pos", [0, 1, 700, 1279])
def test_rope_formula_matches_reference_order(oracle, pos):
    g = torch.Generator().manual_seed(pos + 1)
    v = torch.randn((4, 128), generator=g)
    got = _rope_ref(v, pos)  # rtol = atol = 1e-5 there
    want = np.stack([oracle.rope_neox(v[h].numpy(), pos, 128, 500000.0) for h in range(4)])
    np.testing.assert_allclose(got.numpy(), want, rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("pos", [0, 63, 1023])
def test_attention_formula_matches_reference_order(oracle, pos):
    n_head, n_kv, tmax, B = 20, 5, 1024, 1
    g = torch.Generator().manual_seed(pos + 7)
    q = torch.randn((B, n_head * 128), generator=g)
    kc = torch.randn((B, n_kv, tmax, 128), generator=g)
    vc = torch.randn((B, n_kv, tmax, 128), generator=g)
    got = _attn_ref(q, kc, vc, pos, n_head, n_kv)  # rtol 1e-4, atol 1e-5 there
    k = kc[0, :, :pos + 1].permute(1, 0, 2).reshape(pos + 1, n_kv * 128).numpy()
    v = vc[0, :, :pos + 1].permute(1, 0, 2).reshape(pos + 1, n_kv * 128).numpy()
    want = oracle.attend(q[0].numpy(), k, v, n_head, n_kv)
    np.testing.assert_allclose(got[0].numpy(), want, rtol=2e-5, atol=2e-6)
    assert math.isfinite(float(np.abs(want).max()))
