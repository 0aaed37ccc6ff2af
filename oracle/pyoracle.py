"""ctypes wrapper of the CPU oracle (oracle/_build/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference leg of bench.py, and only as the checker or
the timed CPU baseline. The product library never loads it.

See oracle/oracle.h for which reference function each routine restates and
for the int8-activation conventions (parity unpinned: the reference holds no
test or vector for that arithmetic).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

_lib = None

_u8p = ctypes.POINTER(ctypes.c_uint8)
_i8p = ctypes.POINTER(ctypes.c_int8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)
_sz = ctypes.c_size_t
_i = ctypes.c_int
_u64 = ctypes.c_uint64


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        srcs = [HERE / "oracle.c", HERE / "oracle.h"]
        if not LIB_PATH.exists() or any(
                f.exists() and f.stat().st_mtime > LIB_PATH.stat().st_mtime for f in srcs):
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        sig = {
            "orc_lcg_bytes": (None, [_u64, _u8p, _sz]),
            "orc_normals": (None, [_u64, _f32p, _sz]),
            "orc_ternary": (None, [_u64, _i8p, _sz]),
            "orc_signs": (None, [_u64, _i8p, _sz]),
            "orc_outliers": (None, [_u64, _f32p, _sz, ctypes.c_double, ctypes.c_float]),
            "orc_group_scales": (None, [_u64, _u16p, _sz, ctypes.c_float]),
            "orc_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "orc_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
            "orc_pack_tern2": (None, [_i8p, _i, _i, _u8p]),
            "orc_pack_sign1": (None, [_i8p, _i, _i, _u8p]),
            "orc_absmean_scale": (ctypes.c_float, [_i8p, _sz, ctypes.c_float]),
            "orc_wht_inplace": (None, [_f32p, _sz]),
            "orc_rotate_fwd": (_i, [_f32p, _f32p, _sz, _sz]),
            "orc_rotate_inv": (_i, [_f32p, _f32p, _sz, _sz]),
            "orc_quantize_act": (_i, [_f32p, _i, _i, _f32p, _i, _i8p, _f32p, _f32p]),
            "orc_gemm_tern2": (_i, [_u8p, _i, _i, ctypes.c_float, _i8p, _f32p, _i, _i32p, _f32p]),
            "orc_gemm_sign1": (_i, [_u8p, _u16p, _i, _i, _i8p, _f32p, _i, _i32p, _f32p]),
            "orc_gemm_tern2_mt": (_i, [_u8p, _i, _i, ctypes.c_float, _i8p, _f32p, _i, _f32p, _i]),
            "orc_gemm_sign1_mt": (_i, [_u8p, _u16p, _i, _i, _i8p, _f32p, _i, _f32p, _i]),
            "orc_tq1_block": (None, [_u8p, _f32p]),
            "orc_tl1_group": (None, [_u8p, _f32p]),
            "orc_matvec_tl1_scalar": (_i, [_u8p, _i, _i, _f32p, _f32p]),
            "orc_matvec_tl1_sse": (_i, [_u8p, _i, _i, _f32p, _f32p, _i]),
            "orc_matmul_tl1_scalar": (_i, [_u8p, _i, _i, _f32p, _i, _f32p]),
            "orc_matmul_tl1_sse": (_i, [_u8p, _i, _i, _f32p, _i, _f32p, _i]),
            "orc_matvec_tq1": (_i, [_u8p, _i, _i, _f32p, _f32p, _i]),
            "orc_bf16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "orc_matvec_half": (_i, [_u8p, _i, _i, _f32p, _f32p, _i, _i]),
            "orc_finite_argmax": (_i, [_f32p, _i]),
            "orc_rmsnorm": (None, [_f32p, _f32p, _i, ctypes.c_float, _f32p]),
            "orc_rope_neox": (None, [_f32p, ctypes.c_longlong, _i, ctypes.c_float]),
            "orc_silu": (ctypes.c_float, [ctypes.c_float]),
            "orc_swiglu": (None, [_f32p, _f32p, _i, _f32p]),
            "orc_softmax": (None, [_f32p, _i]),
            "orc_dot": (ctypes.c_float, [_f32p, _f32p, _i]),
            "orc_attend": (_i, [_f32p, _f32p, _f32p, _i, _i, _i, _i, _f32p]),
            "orc_hw_threads": (_i, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t) if a is not None else None


def _chk(rc: int, what: str) -> None:
    if rc != 0:
        raise ValueError(f"oracle {what} rejected its arguments")


# ---- generators ----
def lcg_bytes(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.uint8)
    lib().orc_lcg_bytes(seed, _p(out, _u8p), n)
    return out


def normals(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_normals(seed, _p(out, _f32p), n)
    return out


def ternary(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.int8)
    lib().orc_ternary(seed, _p(out, _i8p), n)
    return out


def signs(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.int8)
    lib().orc_signs(seed, _p(out, _i8p), n)
    return out


def outliers(seed: int, x: np.ndarray, frac: float, mult: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).copy()
    lib().orc_outliers(seed, _p(x, _f32p), x.size, frac, mult)
    return x


def group_scales(seed: int, n: int, sigma: float) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().orc_group_scales(seed, _p(out, _u16p), n, sigma)
    return out


def f16_to_f32(bits: int) -> float:
    return lib().orc_f16_to_f32(bits)


def f32_to_f16(v: float) -> int:
    return lib().orc_f32_to_f16(v)


# ---- packers ----
def pack_tern2(w: np.ndarray) -> np.ndarray:
    M, K = w.shape
    w = np.ascontiguousarray(w, np.int8)
    out = np.empty((M, K // 4), np.uint8)
    lib().orc_pack_tern2(_p(w, _i8p), M, K, _p(out, _u8p))
    return out


def pack_sign1(w: np.ndarray) -> np.ndarray:
    M, K = w.shape
    w = np.ascontiguousarray(w, np.int8)
    out = np.empty((M, K // 8), np.uint8)
    lib().orc_pack_sign1(_p(w, _i8p), M, K, _p(out, _u8p))
    return out


def absmean_scale(w: np.ndarray, base: float) -> float:
    w = np.ascontiguousarray(w, np.int8)
    return float(lib().orc_absmean_scale(_p(w, _i8p), w.size, base))


# ---- Hadamard ----
def wht(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).copy()
    lib().orc_wht_inplace(_p(x, _f32p), x.size)
    return x


def rotate_fwd(x: np.ndarray, signs_: np.ndarray | None, block: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).copy()
    s = None if signs_ is None else np.ascontiguousarray(signs_, np.float32)
    _chk(lib().orc_rotate_fwd(_p(x, _f32p), _p(s, _f32p), x.size, block), "rotate_fwd")
    return x


def rotate_inv(x: np.ndarray, signs_: np.ndarray | None, block: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).copy()
    s = None if signs_ is None else np.ascontiguousarray(signs_, np.float32)
    _chk(lib().orc_rotate_inv(_p(x, _f32p), _p(s, _f32p), x.size, block), "rotate_inv")
    return x


# ---- quantisation / GEMM ----
def quantize_act(x: np.ndarray, signs_: np.ndarray | None = None, had_block: int = 0,
                 want_rot: bool = False):
    x = np.ascontiguousarray(x, np.float32)
    B, K = x.shape
    q = np.empty((B, K), np.int8)
    s = np.empty(B, np.float32)
    xr = np.empty((B, K), np.float32) if want_rot else None
    sg = None if signs_ is None else np.ascontiguousarray(signs_, np.float32)
    _chk(lib().orc_quantize_act(_p(x, _f32p), B, K, _p(sg, _f32p), had_block, _p(q, _i8p),
                                _p(s, _f32p), _p(xr, _f32p)), "quantize_act")
    return (q, s, xr) if want_rot else (q, s)


def gemm_tern2(packed: np.ndarray, M: int, K: int, w_scale: float, q: np.ndarray, s_x: np.ndarray):
    packed = np.ascontiguousarray(packed, np.uint8)
    q = np.ascontiguousarray(q, np.int8)
    s_x = np.ascontiguousarray(s_x, np.float32)
    B = q.shape[0]
    acc = np.empty((B, M), np.int32)
    y = np.empty((B, M), np.float32)
    _chk(lib().orc_gemm_tern2(_p(packed, _u8p), M, K, w_scale, _p(q, _i8p), _p(s_x, _f32p), B,
                              _p(acc, _i32p), _p(y, _f32p)), "gemm_tern2")
    return acc, y


def gemm_sign1(packed: np.ndarray, scales: np.ndarray, M: int, K: int, q: np.ndarray,
               s_x: np.ndarray):
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = np.ascontiguousarray(scales, np.uint16)
    q = np.ascontiguousarray(q, np.int8)
    s_x = np.ascontiguousarray(s_x, np.float32)
    B = q.shape[0]
    acc = np.empty((B, M, K // 128), np.int32)
    y = np.empty((B, M), np.float32)
    _chk(lib().orc_gemm_sign1(_p(packed, _u8p), _p(scales, _u16p), M, K, _p(q, _i8p),
                              _p(s_x, _f32p), B, _p(acc, _i32p), _p(y, _f32p)), "gemm_sign1")
    return acc, y


def gemm_tern2_mt(packed, M, K, w_scale, q, s_x, threads=0):
    B = q.shape[0]
    y = np.empty((B, M), np.float32)
    _chk(lib().orc_gemm_tern2_mt(_p(packed, _u8p), M, K, w_scale, _p(q, _i8p), _p(s_x, _f32p), B,
                                 _p(y, _f32p), threads), "gemm_tern2_mt")
    return y


def gemm_sign1_mt(packed, scales, M, K, q, s_x, threads=0):
    B = q.shape[0]
    y = np.empty((B, M), np.float32)
    _chk(lib().orc_gemm_sign1_mt(_p(packed, _u8p), _p(scales, _u16p), M, K, _p(q, _i8p),
                                 _p(s_x, _f32p), B, _p(y, _f32p), threads), "gemm_sign1_mt")
    return y


# ---- the reference's own formats ----
def tq1_block(block: np.ndarray) -> np.ndarray:
    block = np.ascontiguousarray(block, np.uint8)
    out = np.empty(256, np.float32)
    lib().orc_tq1_block(_p(block, _u8p), _p(out, _f32p))
    return out


def tl1_group(group: np.ndarray) -> np.ndarray:
    group = np.ascontiguousarray(group, np.uint8)
    out = np.empty(128, np.float32)
    lib().orc_tl1_group(_p(group, _u8p), _p(out, _f32p))
    return out


def matvec_tl1_scalar(payload, out_len, in_len, x):
    payload = np.ascontiguousarray(payload, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(out_len, np.float32)
    _chk(lib().orc_matvec_tl1_scalar(_p(payload, _u8p), out_len, in_len, _p(x, _f32p),
                                     _p(y, _f32p)), "matvec_tl1_scalar")
    return y


def matvec_tl1_sse(payload, out_len, in_len, x, threads=0):
    payload = np.ascontiguousarray(payload, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(out_len, np.float32)
    _chk(lib().orc_matvec_tl1_sse(_p(payload, _u8p), out_len, in_len, _p(x, _f32p), _p(y, _f32p),
                                  threads), "matvec_tl1_sse")
    return y


def matmul_tl1_scalar(payload, out_len, in_len, x, k):
    payload = np.ascontiguousarray(payload, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(k * out_len, np.float32)
    _chk(lib().orc_matmul_tl1_scalar(_p(payload, _u8p), out_len, in_len, _p(x, _f32p), k,
                                     _p(y, _f32p)), "matmul_tl1_scalar")
    return y


def matmul_tl1_sse(payload, out_len, in_len, x, k, threads=0):
    """matmul_tl1's x86 K-column path: x [k][in_len] -> y [k * out_len] (y[c*out_len + r])."""
    payload = np.ascontiguousarray(payload, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(k * out_len, np.float32)
    _chk(lib().orc_matmul_tl1_sse(_p(payload, _u8p), out_len, in_len, _p(x, _f32p), k,
                                  _p(y, _f32p), threads), "matmul_tl1_sse")
    return y


def matvec_tq1(payload, out_len, in_len, x, threads=0):
    payload = np.ascontiguousarray(payload, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(out_len, np.float32)
    _chk(lib().orc_matvec_tq1(_p(payload, _u8p), out_len, in_len, _p(x, _f32p), _p(y, _f32p),
                              threads), "matvec_tq1")
    return y


def bf16_to_f32(bits: int) -> float:
    return float(lib().orc_bf16_to_f32(bits))


def matvec_half(payload, out_len, in_len, x, bf16=False, threads=0):
    """matvec_f16 / matvec_bf16 (ops.rs:131-153, 600-620) on the shard bytes."""
    payload = np.ascontiguousarray(payload).view(np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert payload.size == out_len * in_len * 2 and x.size == in_len
    y = np.empty(out_len, dtype=np.float32)
    _chk(lib().orc_matvec_half(_p(payload, _u8p), out_len, in_len, _p(x, _f32p), _p(y, _f32p),
                               int(bool(bf16)), threads), "matvec_half")
    return y


def finite_argmax(logits) -> int:
    """infer/mod.rs:70-83."""
    l = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().orc_finite_argmax(_p(l, _f32p), l.size))


# ---- the decode step's host ops (ops.rs:11-60, infer/mod.rs:338-365) ----
def rmsnorm(x, w, eps: float) -> np.ndarray:
    """ops.rs:12-17 on one row."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty_like(x)
    lib().orc_rmsnorm(_p(x, _f32p), _p(w, _f32p), x.size, eps, _p(y, _f32p))
    return y


def rope_neox(v, t: int, rot: int, base: float) -> np.ndarray:
    """ops.rs:21-33 on one head vector (returns a rotated copy)."""
    v = np.ascontiguousarray(v, np.float32).copy()
    lib().orc_rope_neox(_p(v, _f32p), int(t), rot, base)
    return v


def silu(x: float) -> float:
    return float(lib().orc_silu(x))


def swiglu(gate, up) -> np.ndarray:
    """silu(gate) * up element by element (infer/mod.rs:330)."""
    gate = np.ascontiguousarray(gate, np.float32)
    up = np.ascontiguousarray(up, np.float32)
    out = np.empty_like(gate)
    lib().orc_swiglu(_p(gate, _f32p), _p(up, _f32p), gate.size, _p(out, _f32p))
    return out


def softmax(v) -> np.ndarray:
    v = np.ascontiguousarray(v, np.float32).copy()
    lib().orc_softmax(_p(v, _f32p), v.size)
    return v


def dot(a, b) -> float:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return float(lib().orc_dot(_p(a, _f32p), _p(b, _f32p), a.size))


def attend(q, k, v, n_head: int, n_kv: int, hd: int = 128) -> np.ndarray:
    """infer/mod.rs:338-365 for one sequence: q [n_head*hd], k/v [seq][n_kv*hd]."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    seq = k.size // (n_kv * hd)
    out = np.empty(n_head * hd, np.float32)
    _chk(lib().orc_attend(_p(q, _f32p), _p(k, _f32p), _p(v, _f32p), seq, n_head, n_kv, hd,
                          _p(out, _f32p)), "attend")
    return out


def hw_threads() -> int:
    return int(lib().orc_hw_threads())
