#!/usr/bin/env python3
"""Generate the golden fixtures of the packed-weight matmul path.

The fixtures are small oracle outputs (oracle/, the CPU restatement) on seeded
inputs, stored with their inputs so that a test needs neither the generator
nor the oracle to know the expected bytes:

  quant.npz      per-token absmax int8 quantisation, plain and after the
                 blockwise Walsh-Hadamard rotation (blocks 64 and 128)
  rotate.npz     rotate_fwd / rotate_inv of hadamard.rs:41-66 (blocks 32, 128, 1024)
  tern2.npz      TERNARY2 x int8 products: int32 accumulators and fp32 outputs
  sign1.npz      SIGN1G128 x int8 products after a block-128 rotation:
                 per-group int32 accumulators and fp32 outputs
  refformat.npz  the reference's own formats: matvec_tl1 (PTQ1_0, scalar and
                 SSE4.1 accumulation orders), matmul_tl1 (K = 3 columns, scalar and
                 x86 K-column orders) and
                 matvec_qblock (TQ1_0) on payloads built with the generators of
                 the reference's tests (ops.rs:721-750, 801-838)

Run from the repository root:  python tests/golden/make_golden.py
The CPU suite (tests/test_golden.py) checks that the oracle still reproduces
every array bit for bit; the GPU suite checks the CUDA kernels against them.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import pyoracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent


def quant_cases():
    d = {}
    x = O.outliers(101, O.normals(100, 4 * 512), 0.01, 20.0).reshape(4, 512)
    x[2] = 0.0  # an all-zero token: s_x = 0, q = 0
    sg = O.signs(102, 512).astype(np.float32)
    d["x"], d["signs"] = x, sg
    for blk in (0, 64, 128):
        q, s = O.quantize_act(x, sg if blk else None, blk)
        d[f"q_b{blk}"], d[f"s_b{blk}"] = q, s
    return d


def rotate_cases():
    d = {}
    for blk in (32, 128, 1024):
        x = O.normals(200 + blk, 2048)
        sg = O.signs(300 + blk, 2048).astype(np.float32)
        d[f"x_b{blk}"], d[f"signs_b{blk}"] = x, sg
        d[f"fwd_b{blk}"] = O.rotate_fwd(x, sg, blk)
        d[f"inv_b{blk}"] = O.rotate_inv(x, sg, blk)
    return d


def tern2_cases():
    d = {}
    for tag, (M, K, B) in {"a": (96, 512, 3), "b": (200, 1024, 16)}.items():
        w = O.ternary(400 + M, M * K).reshape(M, K)
        ws = O.absmean_scale(w, 0.02)
        x = O.normals(500 + M, B * K).reshape(B, K)
        q, s = O.quantize_act(x)
        acc, y = O.gemm_tern2(O.pack_tern2(w), M, K, ws, q, s)
        d.update({f"{tag}_packed": O.pack_tern2(w), f"{tag}_w_scale": np.float32(ws),
                  f"{tag}_x": x, f"{tag}_q": q, f"{tag}_s": s, f"{tag}_acc": acc, f"{tag}_y": y,
                  f"{tag}_shape": np.array([M, K, B], np.int32)})
    return d


def sign1_cases():
    d = {}
    M, K, B = 80, 1024, 4
    w = O.signs(600, M * K).reshape(M, K)
    sc = O.group_scales(601, M * (K // 128), 0.02)
    x = O.outliers(603, O.normals(602, B * K), 0.01, 20.0).reshape(B, K)
    sg = O.signs(604, K).astype(np.float32)
    q, s = O.quantize_act(x, sg, 128)
    acc, y = O.gemm_sign1(O.pack_sign1(w), sc, M, K, q, s)
    d.update({"packed": O.pack_sign1(w), "scales": sc, "x": x, "signs": sg, "block": np.int32(128),
              "q": q, "s": s, "acc": acc, "y": y, "shape": np.array([M, K, B], np.int32)})
    return d


def refformat_cases():
    d = {}
    # PTQ1_0 payload generator of ops.rs:721-750: byte i = (i * (0x9B ^ (i >> 5))) mod 256,
    # fp16 scale bytes 0x10, 0x38 at offsets 26..28 of every 28-byte group
    out_len, in_len = 24, 384
    n = out_len * (in_len // 128) * 28
    i = np.arange(n, dtype=np.uint64)
    pay = ((i * (0x9B ^ (i >> 5))) % 256).astype(np.uint8)
    g = pay.reshape(-1, 28)
    g[:, 26], g[:, 27] = 0x10, 0x38
    x = (((np.arange(in_len) % 11) - 5) * 0.25).astype(np.float32)
    d["tl1_payload"], d["tl1_x"] = pay, x
    d["tl1_shape"] = np.array([out_len, in_len], np.int32)
    d["tl1_scalar"] = O.matvec_tl1_scalar(pay, out_len, in_len, x)
    d["tl1_sse"] = O.matvec_tl1_sse(pay, out_len, in_len, x, 1)
    xk = O.normals(700, 3 * in_len)
    d["tl1_xk"] = xk
    d["tl1_matmul_k3"] = O.matmul_tl1_scalar(pay, out_len, in_len, xk, 3)
    d["tl1_matmul_sse_k3"] = O.matmul_tl1_sse(pay, out_len, in_len, xk, 3, 1)
    # TQ1_0 payload generator of ops.rs:801-838: byte i = (i * (0x9B ^ (i >> 7))) mod 256
    out_len, in_len = 16, 512
    n = out_len * (in_len // 256) * 54
    i = np.arange(n, dtype=np.uint64)
    pay = ((i * (0x9B ^ (i >> 7))) % 256).astype(np.uint8)
    b = pay.reshape(-1, 54)
    b[:, 52], b[:, 53] = 0x10, 0x38
    x = (((np.arange(in_len) % 7) - 3) * 0.5).astype(np.float32)
    d["tq1_payload"], d["tq1_x"] = pay, x
    d["tq1_shape"] = np.array([out_len, in_len], np.int32)
    d["tq1_y"] = O.matvec_tq1(pay, out_len, in_len, x, 1)
    return d


CASES = {"quant": quant_cases, "rotate": rotate_cases, "tern2": tern2_cases,
         "sign1": sign1_cases, "refformat": refformat_cases}


def main():
    for name, fn in CASES.items():
        np.savez_compressed(OUT / f"{name}.npz", **fn())
        print(f"wrote {OUT / (name + '.npz')}")


if __name__ == "__main__":
    main()
