"""ouroboros_b200 -- B200-native packed-weight matmul path of OuroborOS.

Python mirror of the C ABI in include/ouroq.h, loaded from the in-tree
libouroq.so with ctypes. The shipped compute path is the CUDA library; there
is no CPU fallback: if the library is missing or no sm_100 device is present,
every entry point raises.

The operator names follow the reference's Rust API (crate ouro-cluster):
  matvec_q   cluster/src/infer/ops.rs:76-84
  matmul_q   cluster/src/infer/ops.rs:219-230  (output [k][out_len])
  rotate_fwd cluster/src/infer/hadamard.rs:41-53
  rotate_inv cluster/src/infer/hadamard.rs:57-66
Errors raise OuroqError, the counterpart of the reference's assert!/bail!
(hadamard.rs:33-37, infer/mod.rs:139-145).

torch is used only to own device memory and streams (plumbing).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

__all__ = [
    "OuroqError", "Context", "Weight", "TERNARY2", "SIGN1G128", "PTQ1_0", "TQ1_0", "F16", "BF16",
    "load_library",
    "LIB_PATH",
    "ABI_FUNCTIONS", "SHARD_ID_BYTES", "shard_unique_id", "shard_rows",
]

LIB_PATH = Path(__file__).resolve().parent / "libouroq.so"

TERNARY2 = 1
SIGN1G128 = 2
PTQ1_0 = 3  # the reference's Tl1 shard format (28 B per 128 weights), fp32 activations
TQ1_0 = 4   # the reference's TQ1_0 shard format (54 B per 256 weights), fp32 activations
F16 = 5     # 16-bit shard weights (QuantKind::F16, e.g. the tied token_embd), fp32 activations
BF16 = 6    # QuantKind::Bf16
SHARD_ID_BYTES = 128

OK = 0
_STATUS = {
    0: "ok", 1: "bad shape", 2: "bad alignment", 3: "cuda error", 4: "nccl error", 5: "timeout",
    6: "unsupported", 7: "bad argument", 8: "no device", 9: "out of memory",
}

_p = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); every function declared in include/ouroq.h
ABI_FUNCTIONS = {
    "ouroq_abi_version": (_i, []),
    "ouroq_status_string": (ctypes.c_char_p, [_i]),
    "ouroq_ctx_create": (_i, [_i, ctypes.POINTER(_p)]),
    "ouroq_ctx_destroy": (_i, [_p]),
    "ouroq_last_error": (ctypes.c_char_p, [_p]),
    "ouroq_check_device": (_i, [_p]),
    "ouroq_ptr_kind": (_i, [_p, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "ouroq_launch_count": (ctypes.c_uint64, [_p]),
    "ouroq_set_pdl": (_i, [_p, _i]),
    "ouroq_set_prefetch": (_i, [_p, _i, _p]),
    "ouroq_weight_upload": (_i, [_p, _i, _p, _i, _i, _p, _f, ctypes.POINTER(_p)]),
    "ouroq_weight_upload_device": (_i, [_p, _i, _p, _i, _i, _p, _f, ctypes.POINTER(_p)]),
    "ouroq_weight_free": (_i, [_p, _p]),
    "ouroq_weight_info": (_i, [_p, ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i),
                               ctypes.POINTER(_sz)]),
    "ouroq_quantize_act": (_i, [_p, _p, _i, _i, _p, _i, _p, _p, _p]),
    "ouroq_quantize_group": (_i, [_p, _i, _p, _p, _p, _p, _i, _p, _p, _p]),
    "ouroq_rotate": (_i, [_p, _p, _p, _i, _i, _p, _i, _i, _p]),
    "ouroq_gemm": (_i, [_p, _p, _p, _p, _i, _p, _p, _p]),
    "ouroq_gemm_group": (_i, [_p, _i, _p, _p, _p, _i, _p, _p]),
    "ouroq_gemm_group_f32act": (_i, [_p, _i, _p, _p, _i, _p, _p, _p, _p]),
    "ouroq_gemm_f32act": (_i, [_p, _p, _p, _i, _p, _i, _p, _p]),
    "ouroq_gemm_f32act_noalloc": (_i, [_p, _p, _p, _i, _p, _i, _p, _p]),
    "ouroq_shard_unique_id": (_i, [_p]),
    "ouroq_shard_init": (_i, [_p, _p, _i, _i]),
    "ouroq_shard_set_transport": (_i, [_p, _i]),
    "ouroq_shard_finalize": (_i, [_p]),
    "ouroq_shard_rows": (_i, [_i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "ouroq_weight_upload_shard": (_i, [_p, _i, _p, _i, _i, _p, _f, ctypes.POINTER(_p)]),
    "ouroq_gemm_sharded": (_i, [_p, _p, _p, _i, _p, _i, _p, _p]),
    "ouroq_shard_sync": (_i, [_p, _p, _i]),
    "ouroq_rmsnorm": (_i, [_p, _p, _p, _p, _p, _p, _i, _i, _f, _p]),
    "ouroq_swiglu_rmsnorm": (_i, [_p, _p, _p, _p, _p, _i, _i, _f, _p]),
    "ouroq_rope_kv_append": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _f, _p]),
    "ouroq_attention_decode": (_i, [_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p]),
    "ouroq_rope_attention_decode": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i,
                                         ctypes.c_float, _p]),
    "ouroq_argmax_token": (_i, [_p, _p, _p, _i, _p, _p, _p]),
    "ouroq_gemm_norm_f32act": (_i, [_p, _i, _p, _p, _p, _i, _p, ctypes.c_float, _p, _i, _p, _p]),
    "ouroq_bmts_open": (_i, [ctypes.c_char_p, ctypes.POINTER(_p), ctypes.c_char_p, _sz]),
    "ouroq_bmts_close": (_i, [_p]),
    "ouroq_bmts_info": (_i, [_p, ctypes.POINTER(_i), ctypes.POINTER(_i),
                             ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]),
    "ouroq_bmts_tensor": (_i, [_p, _i, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_i),
                               ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint32),
                               ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]),
    "ouroq_bmts_span": (_i, [_p, ctypes.c_char_p, ctypes.c_uint64, ctypes.c_uint64,
                             ctypes.POINTER(_p), ctypes.c_char_p, _sz]),
    "ouroq_bmts_upload": (_i, [_p, _p, ctypes.c_char_p, ctypes.POINTER(_p), ctypes.c_char_p, _sz]),
    "ouroq_matvec_q": (_i, [_p, _p, _p, _p]),
    "ouroq_matmul_q": (_i, [_p, _p, _p, _i, _p]),
    "ouroq_matmul_q_group": (_i, [_p, _i, _p, _p, _i, _p]),
    "ouroq_rotate_fwd": (_i, [_p, _p, _p, _sz, _sz]),
    "ouroq_rotate_inv": (_i, [_p, _p, _p, _sz, _sz]),
}

_lib = None


PTR_HOST, PTR_DEVICE, PTR_MANAGED = 0, 1, 2


def ptr_kind(ptr: int) -> tuple[int, int]:
    """(kind, device) of a raw pointer: PTR_HOST / PTR_DEVICE / PTR_MANAGED,
    device -1 for host memory."""
    lib = load_library()
    kind, dev = ctypes.c_int(), ctypes.c_int()
    st = lib.ouroq_ptr_kind(ctypes.c_void_p(ptr), ctypes.byref(kind), ctypes.byref(dev))
    if st != OK:
        raise OuroqError(st, "ptr_kind")
    return kind.value, dev.value


class OuroqError(RuntimeError):
    def __init__(self, status: int, msg: str = ""):
        self.status = status
        super().__init__(f"{_STATUS.get(status, status)}: {msg}" if msg else _STATUS.get(status, str(status)))


def load_library(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load libouroq.so and declare every C-ABI signature. Raises if absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise OuroqError(6, f"{p} not built (run python -m ouroboros_b200.build)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in ABI_FUNCTIONS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def _ptr(t) -> int | None:
    """Device/host address of a torch tensor or numpy array (None passes through)."""
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        if not t.flags.c_contiguous:
            raise OuroqError(7, "array must be C-contiguous")
        return t.ctypes.data
    if not t.is_contiguous():
        raise OuroqError(7, "tensor must be contiguous")
    return t.data_ptr()


def _dev(t, dtype: str, numel: int | None, what: str, optional: bool = False) -> int | None:
    """Address of a contiguous CUDA tensor of `dtype` ("float32", "int8", ...)
    holding exactly `numel` elements (None: at least one). The C ABI takes bare
    device pointers with no lengths, so a wrong dtype, size or layout is
    caught here and raised like the reference's width check (Stage::wm,
    infer/mod.rs:139-145) instead of becoming an out-of-bounds access."""
    if t is None:
        if optional:
            return None
        raise OuroqError(7, f"{what}: missing")
    if isinstance(t, np.ndarray) or not getattr(t, "is_cuda", False):
        raise OuroqError(7, f"{what}: expected a CUDA tensor")
    if str(t.dtype) != "torch." + dtype:
        raise OuroqError(7, f"{what}: dtype {t.dtype}, expected {dtype}")
    if not t.is_contiguous():
        raise OuroqError(7, f"{what}: not contiguous")
    n = t.numel()
    if (numel is None and n < 1) or (numel is not None and n != numel):
        raise OuroqError(1, f"{what}: {n} elements, expected {numel if numel is not None else '>= 1'}")
    return t.data_ptr()


def _ndim(t) -> int:
    """Dimensions of a tensor (-1 for anything else)."""
    return t.dim() if hasattr(t, "dim") else -1


def _rows(x, width: int, what: str) -> int:
    """Rows of an activation tensor [B][width] (a 1-D x of `width` is one row)."""
    if not hasattr(x, "numel"):
        raise OuroqError(7, f"{what}: expected a CUDA tensor")
    n = x.numel()
    if width <= 0 or n % width:
        raise OuroqError(1, f"{what}: {n} elements is not a whole number of rows of {width}")
    return n // width


def _stream_ptr(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def shard_unique_id() -> bytes:
    """A new shard-group id (rank 0 makes it; every rank passes it to shard_init)."""
    lib = load_library()
    buf = ctypes.create_string_buffer(SHARD_ID_BYTES)
    st = lib.ouroq_shard_unique_id(ctypes.cast(buf, _p))
    if st != OK:
        raise OuroqError(st, "ouroq_shard_unique_id")
    return buf.raw


def shard_rows(M: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of an M-row matrix owned by `rank` of `world`."""
    lib = load_library()
    r0, n = _i(), _i()
    st = lib.ouroq_shard_rows(M, world, rank, ctypes.byref(r0), ctypes.byref(n))
    if st != OK:
        raise OuroqError(st, f"ouroq_shard_rows(M={M}, world={world}, rank={rank})")
    return r0.value, n.value


class Weight:
    """A packed matrix resident on the device (ouroq_weight handle)."""

    def __init__(self, ctx: "Context", handle: int, fmt: int, M: int, K: int):
        self.ctx, self.handle, self.fmt, self.M, self.K = ctx, handle, fmt, M, K
        self.w_scale = 0.0
        # rows held on this device: M, or this rank's share of a row-sharded
        # matrix (what the unsharded products write; gemm_sharded writes M)
        self.rows = M

    @property
    def out_len(self) -> int:
        return self.M

    @property
    def in_len(self) -> int:
        return self.K

    def device_bytes(self) -> int:
        n = _sz()
        self.ctx._check(self.ctx.lib.ouroq_weight_info(self.handle, None, None, None, ctypes.byref(n)))
        return n.value

    def free(self) -> None:
        if self.handle:
            self.ctx._check(self.ctx.lib.ouroq_weight_free(self.ctx.ctx, self.handle))
            self.handle = None


class Context:
    """One ouroq context per CUDA device (not thread-safe, like the reference's stage slot)."""

    def __init__(self, device: int = 0, lib_path=None):
        self.lib = load_library(lib_path)
        self.device = device
        h = _p()
        st = self.lib.ouroq_ctx_create(device, ctypes.byref(h))
        if st != OK:
            raise OuroqError(st, f"ouroq_ctx_create(device={device})")
        self.ctx = h.value

    # -- plumbing --
    def _check(self, st: int) -> None:
        if st != OK:
            raise OuroqError(st, (self.lib.ouroq_last_error(self.ctx) or b"").decode())

    def close(self) -> None:
        if getattr(self, "ctx", None):
            self.lib.ouroq_ctx_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def launch_count(self) -> int:
        return int(self.lib.ouroq_launch_count(self.ctx))

    def set_pdl(self, enable: bool) -> None:
        self._check(self.lib.ouroq_set_pdl(self.ctx, 1 if enable else 0))

    def set_prefetch(self, ws) -> None:
        """The weights the call after the next GEMV launch reads: that launch
        prefetches them into L2 (a hint; results never depend on it)."""
        n = len(ws)
        arr = (_p * max(n, 1))(*[w.handle for w in ws])
        self._check(self.lib.ouroq_set_prefetch(self.ctx, n, arr))

    def check_device(self) -> None:
        self._check(self.lib.ouroq_check_device(self.ctx))

    # -- weights --
    def upload(self, fmt: int, packed: np.ndarray, M: int, K: int, scales: np.ndarray | None = None,
               w_scale: float = 1.0) -> Weight:
        if fmt in (F16, BF16) and np.asarray(packed).dtype.itemsize == 2:
            packed = np.ascontiguousarray(packed).view(np.uint8)  # the shard's bytes
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        if scales is not None:
            scales = np.ascontiguousarray(scales, dtype=np.uint16)
        h = _p()
        self._check(self.lib.ouroq_weight_upload(self.ctx, fmt, _ptr(packed), M, K, _ptr(scales),
                                                 float(w_scale), ctypes.byref(h)))
        w = Weight(self, h.value, fmt, M, K)
        w.w_scale = float(w_scale)
        return w

    def upload_device(self, fmt: int, packed_dev, M: int, K: int, scales_dev=None,
                      w_scale: float = 1.0) -> Weight:
        h = _p()
        self._check(self.lib.ouroq_weight_upload_device(self.ctx, fmt, _ptr(packed_dev), M, K,
                                                        _ptr(scales_dev), float(w_scale),
                                                        ctypes.byref(h)))
        w = Weight(self, h.value, fmt, M, K)
        w.w_scale = float(w_scale)
        return w

    # -- device API (torch CUDA tensors) --
    def quantize_act(self, x, signs=None, hadamard_block: int = 0, q=None, s_x=None, stream=None):
        import torch
        if _ndim(x) != 2:
            raise OuroqError(1, "x must be a [B][K] CUDA tensor")
        B, K = x.shape
        if q is None:
            q = torch.empty((B, K), dtype=torch.int8, device=x.device)
        if s_x is None:
            s_x = torch.empty((B,), dtype=torch.float32, device=x.device)
        self._check(self.lib.ouroq_quantize_act(
            self.ctx, _dev(x, "float32", B * K, "x"), B, K,
            _dev(signs, "float32", K, "signs", True), hadamard_block,
            _dev(q, "int8", B * K, "q"), _dev(s_x, "float32", B, "s_x"), _stream_ptr(stream)))
        return q, s_x

    def quantize_group(self, xs, qs, sxs, signs=None, blocks=None, stream=None):
        """One launch quantising several activation sets (same batch B)."""
        n = len(xs)
        if any(_ndim(x) != 2 for x in xs):
            raise OuroqError(1, "every x must be a [B][K] CUDA tensor")
        B = xs[0].shape[0] if n else 0
        if any(x.shape[0] != B for x in xs):
            raise OuroqError(1, "every x must have the same B")
        K = [x.shape[1] for x in xs]
        arr = lambda vals: (_p * max(n, 1))(*vals)  # noqa: E731
        Ks = (_i * max(n, 1))(*K)
        sg = (arr([_dev(sv, "float32", K[i], f"signs[{i}]", True) for i, sv in enumerate(signs)])
              if signs is not None else None)
        bl = (_i * max(n, 1))(*blocks) if blocks is not None else None
        self._check(self.lib.ouroq_quantize_group(
            self.ctx, n, arr([_dev(x, "float32", B * K[i], f"x[{i}]") for i, x in enumerate(xs)]),
            Ks, sg, bl, B, arr([_dev(q, "int8", B * K[i], f"q[{i}]") for i, q in enumerate(qs)]),
            arr([_dev(sv, "float32", B, f"s_x[{i}]") for i, sv in enumerate(sxs)]),
            _stream_ptr(stream)))
        return qs, sxs

    def rotate(self, x, signs=None, block: int = 128, inverse: bool = False, out=None, stream=None):
        import torch
        if _ndim(x) != 2:
            raise OuroqError(1, "x must be a [B][K] CUDA tensor")
        B, K = x.shape
        if out is None:
            out = torch.empty_like(x)
        self._check(self.lib.ouroq_rotate(
            self.ctx, _dev(x, "float32", B * K, "x"), _dev(out, "float32", B * K, "out"), B, K,
            _dev(signs, "float32", K, "signs", True), block, 1 if inverse else 0,
            _stream_ptr(stream)))
        return out

    def gemm(self, w: Weight, q, s_x, y=None, acc=None, stream=None):
        import torch
        B = _rows(q, w.K, "q")
        if y is None:
            y = torch.empty((B, w.rows), dtype=torch.float32, device=q.device)
        nacc = B * w.rows * (w.K // 128 if w.fmt == SIGN1G128 else 1)
        self._check(self.lib.ouroq_gemm(
            self.ctx, w.handle, _dev(q, "int8", B * w.K, "q"), _dev(s_x, "float32", B, "s_x"), B,
            _dev(y, "float32", B * w.rows, "y"), _dev(acc, "int32", nacc, "acc", True),
            _stream_ptr(stream)))
        return y

    def gemm_group(self, ws, qs, sxs, ys, stream=None):
        n = len(ws)
        B = _rows(qs[0], ws[0].K, "q[0]") if n else 0
        arr = lambda vals: (_p * max(n, 1))(*vals)  # noqa: E731
        self._check(self.lib.ouroq_gemm_group(
            self.ctx, n, arr([w.handle for w in ws]),
            arr([_dev(q, "int8", B * w.K, f"q[{i}]") for i, (w, q) in enumerate(zip(ws, qs))]),
            arr([_dev(sv, "float32", B, f"s_x[{i}]") for i, sv in enumerate(sxs)]), B,
            arr([_dev(y, "float32", B * w.rows, f"y[{i}]") for i, (w, y) in enumerate(zip(ws, ys))]),
            _stream_ptr(stream)))
        return ys

    def gemm_group_f32act(self, ws, xs, ys, signs=None, blocks=None, stream=None):
        """One launch: fused quantisation (+ optional rotation) and GEMV for each (W, x)."""
        n = len(ws)
        B = _rows(xs[0], ws[0].K, "x[0]") if n else 0
        arr = lambda vals: (_p * max(n, 1))(*vals)  # noqa: E731
        sg = (arr([_dev(sv, "float32", w.K, f"signs[{i}]", True)
                   for i, (w, sv) in enumerate(zip(ws, signs))]) if signs is not None else None)
        bl = (_i * max(n, 1))(*blocks) if blocks is not None else None
        self._check(self.lib.ouroq_gemm_group_f32act(
            self.ctx, n, arr([w.handle for w in ws]),
            arr([_dev(x, "float32", B * w.K, f"x[{i}]") for i, (w, x) in enumerate(zip(ws, xs))]),
            B, sg, bl,
            arr([_dev(y, "float32", B * w.rows, f"y[{i}]") for i, (w, y) in enumerate(zip(ws, ys))]),
            _stream_ptr(stream)))
        return ys

    def gemm_f32act(self, w: Weight, x, signs=None, hadamard_block: int = 0, y=None, stream=None):
        import torch
        B = _rows(x, w.K, "x")
        if y is None:
            y = torch.empty((B, w.rows), dtype=torch.float32, device=x.device)
        self._check(self.lib.ouroq_gemm_f32act(
            self.ctx, w.handle, _dev(x, "float32", B * w.K, "x"), B,
            _dev(signs, "float32", w.K, "signs", True), hadamard_block,
            _dev(y, "float32", B * w.rows, "y"), _stream_ptr(stream)))
        return y

    def gemm_f32act_noalloc(self, w: Weight, x, y, signs=None, hadamard_block: int = 0, stream=None):
        """gemm_f32act for callers that must not allocate device memory mid-run
        (memory reserved up front, or no room for cudaFree's device-wide wait).
        The library allocates nothing here, and neither does this wrapper: the
        caller passes the output y [B][M] fp32. Limits B <= 4096, B*K <= 4 MiB;
        all calls on one device share one scratch area, so two calls in flight at
        once race. The first call on a device does set-up: make it before any
        stream capture."""
        B = _rows(x, w.K, "x")
        self._check(self.lib.ouroq_gemm_f32act_noalloc(
            self.ctx, w.handle, _dev(x, "float32", B * w.K, "x"), B,
            _dev(signs, "float32", w.K, "signs", True), hadamard_block,
            _dev(y, "float32", B * w.rows, "y"), _stream_ptr(stream)))
        return y

    # -- row-sharded matmul (one process per GPU, NCCL all-gather) --
    def shard_init(self, group_id: bytes, world: int, rank: int) -> None:
        """Join the shard group; `group_id` comes from shard_unique_id() on rank 0."""
        buf = ctypes.create_string_buffer(bytes(group_id), SHARD_ID_BYTES)
        self._check(self.lib.ouroq_shard_init(self.ctx, ctypes.cast(buf, _p), world, rank))

    def shard_set_transport(self, transport: str) -> None:
        """'peer' (stores into every rank's buffer over NVLink) or 'nccl' (all-gather)."""
        self._check(self.lib.ouroq_shard_set_transport(self.ctx, {"peer": 0, "nccl": 1}[transport]))

    def shard_finalize(self) -> None:
        self._check(self.lib.ouroq_shard_finalize(self.ctx))

    def upload_shard(self, fmt: int, packed_full: np.ndarray, M: int, K: int,
                     scales_full: np.ndarray | None = None, w_scale: float = 1.0) -> Weight:
        """Upload this rank's rows of a full matrix (canonical host layout, full M)."""
        packed_full = np.ascontiguousarray(packed_full, dtype=np.uint8)
        if scales_full is not None:
            scales_full = np.ascontiguousarray(scales_full, dtype=np.uint16)
        h = _p()
        self._check(self.lib.ouroq_weight_upload_shard(self.ctx, fmt, _ptr(packed_full), M, K,
                                                       _ptr(scales_full), float(w_scale),
                                                       ctypes.byref(h)))
        w = Weight(self, h.value, fmt, M, K)
        w.w_scale = float(w_scale)
        rows = _i()
        self._check(self.lib.ouroq_weight_info(w.handle, None, ctypes.byref(rows), None, None))
        w.rows = rows.value
        return w

    def gemm_sharded(self, w: Weight, x, y=None, signs=None, hadamard_block: int = 0, stream=None):
        """y [B][M] (full M, every rank) from this rank's rows + an all-gather."""
        import torch
        B = _rows(x, w.K, "x")
        if y is None:
            y = torch.empty((B, w.M), dtype=torch.float32, device=x.device)
        self._check(self.lib.ouroq_gemm_sharded(
            self.ctx, w.handle, _dev(x, "float32", B * w.K, "x"), B,
            _dev(signs, "float32", w.K, "signs", True), hadamard_block,
            _dev(y, "float32", B * w.M, "y"), _stream_ptr(stream)))
        return y

    def shard_sync(self, stream=None, timeout_ms: int = 10000) -> None:
        self._check(self.lib.ouroq_shard_sync(self.ctx, _stream_ptr(stream), int(timeout_ms)))

    # -- the decode step around the projections (fp32 device tensors) --
    def rmsnorm(self, x, w, y=None, residual=None, h=None, eps: float = 1e-5, stream=None):
        """y = rmsnorm(x + residual) * w; h (optional) receives x + residual."""
        import torch
        n = w.numel()
        B = _rows(x, n, "x")
        if y is None:
            y = torch.empty_like(x)
        self._check(self.lib.ouroq_rmsnorm(
            self.ctx, _dev(x, "float32", B * n, "x"), _dev(residual, "float32", B * n, "residual", True),
            _dev(h, "float32", B * n, "h", True), _dev(w, "float32", n, "w"),
            _dev(y, "float32", B * n, "y"), B, n, eps, _stream_ptr(stream)))
        return y

    def swiglu_rmsnorm(self, gate, up, w, y=None, eps: float = 1e-5, stream=None):
        import torch
        n = w.numel()
        B = _rows(gate, n, "gate")
        if y is None:
            y = torch.empty_like(gate)
        self._check(self.lib.ouroq_swiglu_rmsnorm(
            self.ctx, _dev(gate, "float32", B * n, "gate"), _dev(up, "float32", B * n, "up"),
            _dev(w, "float32", n, "w"), _dev(y, "float32", B * n, "y"), B, n, eps,
            _stream_ptr(stream)))
        return y

    def rope_kv_append(self, q, k, v, kcache, vcache, pos, n_head: int, n_kv: int,
                       rope_base: float = 500000.0, stream=None):
        B, tmax = _rows(q, n_head * 128, "q"), kcache.shape[-2]
        kv = B * n_kv * 128
        self._check(self.lib.ouroq_rope_kv_append(
            self.ctx, _dev(q, "float32", B * n_head * 128, "q"), _dev(k, "float32", kv, "k"),
            _dev(v, "float32", kv, "v"), _dev(kcache, "float32", kv * tmax, "kcache"),
            _dev(vcache, "float32", kv * tmax, "vcache"), _dev(pos, "int64", None, "pos"), B,
            n_head, n_kv, tmax, rope_base, _stream_ptr(stream)))

    def attention_decode(self, q, kcache, vcache, pos, n_head: int, n_kv: int, out=None, stream=None):
        import torch
        B, tmax = _rows(q, n_head * 128, "q"), kcache.shape[-2]
        if out is None:
            out = torch.empty((B, n_head * 128), dtype=torch.float32, device=q.device)
        cache = B * n_kv * tmax * 128
        self._check(self.lib.ouroq_attention_decode(
            self.ctx, _dev(q, "float32", B * n_head * 128, "q"),
            _dev(kcache, "float32", cache, "kcache"), _dev(vcache, "float32", cache, "vcache"),
            _dev(pos, "int64", None, "pos"), _dev(out, "float32", B * n_head * 128, "out"), B,
            n_head, n_kv, tmax, _stream_ptr(stream)))
        return out

    def gemm_norm_f32act(self, ws, x, norm_w, ys, residual=None, swiglu=False, h=None,
                         eps: float = 1e-5, stream=None):
        """ys[i] = W_i (rmsnorm(x + residual) * norm_w), or with swiglu=True
        W_i (rmsnorm(silu(x) * residual) * norm_w); h receives x + residual."""
        n = len(ws)
        if n == 0:
            raise OuroqError(1, "no matrices")
        K = ws[0].K
        B = _rows(x, K, "x")
        arr = lambda vals: (_p * n)(*vals)  # noqa: E731
        self._check(self.lib.ouroq_gemm_norm_f32act(
            self.ctx, n, arr([w.handle for w in ws]), _dev(x, "float32", B * K, "x"),
            _dev(residual, "float32", B * K, "residual", not swiglu), 1 if swiglu else 0,
            _dev(norm_w, "float32", K, "norm_w"), eps, _dev(h, "float32", B * K, "h", True), B,
            arr([_dev(y, "float32", B * w.rows, f"y[{i}]") for i, (w, y) in enumerate(zip(ws, ys))]),
            _stream_ptr(stream)))
        return ys

    def argmax_token(self, w: Weight, x, tokens=None, logits=None, stream=None):
        """Greedy next token of each row of x [B][K] through the F16 / BF16 head w
        (the reference's argmax_token); logits [B][M] are written if given."""
        import torch
        B = _rows(x, w.K, "x")
        if tokens is None:
            tokens = torch.empty((B,), dtype=torch.long, device=x.device)
        self._check(self.lib.ouroq_argmax_token(
            self.ctx, w.handle, _dev(x, "float32", B * w.K, "x"), B,
            _dev(logits, "float32", B * w.rows, "logits", True), _dev(tokens, "int64", B, "tokens"),
            _stream_ptr(stream)))
        return tokens

    def rope_attention_decode(self, q, k, v, kcache, vcache, pos, n_head: int, n_kv: int,
                              rope_base: float = 500000.0, out=None, stream=None):
        """rope_kv_append + attention_decode in one launch; q is not modified."""
        import torch
        B, tmax = _rows(q, n_head * 128, "q"), kcache.shape[-2]
        if out is None:
            out = torch.empty((B, n_head * 128), dtype=torch.float32, device=q.device)
        kv = B * n_kv * 128
        self._check(self.lib.ouroq_rope_attention_decode(
            self.ctx, _dev(q, "float32", B * n_head * 128, "q"), _dev(k, "float32", kv, "k"),
            _dev(v, "float32", kv, "v"), _dev(kcache, "float32", kv * tmax, "kcache"),
            _dev(vcache, "float32", kv * tmax, "vcache"), _dev(pos, "int64", None, "pos"),
            _dev(out, "float32", B * n_head * 128, "out"), B, n_head, n_kv, tmax, rope_base,
            _stream_ptr(stream)))
        return out

    # -- host-buffer mirrors of the reference operators (numpy in, numpy out) --
    def matvec_q(self, w: Weight, x: np.ndarray) -> np.ndarray:
        """ops::matvec_q: y[out_len] = W . x[in_len] (fp32)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.shape != (w.K,):
            raise OuroqError(1, f"in_len {w.K} != x len {x.size}")
        y = np.empty(w.rows, dtype=np.float32)
        self._check(self.lib.ouroq_matvec_q(self.ctx, w.handle, _ptr(x), _ptr(y)))
        return y

    def matmul_q(self, w: Weight, x: np.ndarray) -> np.ndarray:
        """ops::matmul_q: x [k][in_len] -> y [k][out_len] (= y[c*out_len + r])."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim != 2 or x.shape[1] != w.K:
            raise OuroqError(1, f"in_len {w.K} != x width {x.shape[-1]}")
        k = x.shape[0]
        y = np.empty((k, w.rows), dtype=np.float32)
        self._check(self.lib.ouroq_matmul_q(self.ctx, w.handle, _ptr(x), k, _ptr(y)))
        return y

    def matmul_q_group(self, ws, xs, ys=None):
        """Several matmul_q products in one synchronous round trip: ys[i] [k][M_i]
        = W_i . xs[i] [k][K_i] (host buffers: numpy arrays or CPU tensors; page-locked
        ones are copied by DMA directly). Entries may share an input. Returns ys."""
        n = len(ws)
        if len(xs) != n or (ys is not None and len(ys) != n):
            raise OuroqError(1, "one input and one output per weight")

        def size_of(a):
            return a.size if isinstance(a, np.ndarray) else a.numel()

        def f32(a):
            return str(getattr(a, "dtype", "")) in ("float32", "torch.float32")
        k = None
        for w, x in zip(ws, xs):
            if getattr(x, "is_cuda", False):
                raise OuroqError(7, "matmul_q_group takes host buffers")
            if w.K <= 0 or size_of(x) % w.K or not f32(x):
                raise OuroqError(1, f"in_len {w.K}: input of {size_of(x)} values is not [k][{w.K}] float32")
            rows = size_of(x) // w.K
            if k is not None and rows != k:
                raise OuroqError(1, "every input has the same number of columns k")
            k = rows
        if ys is None:
            ys = [np.empty((k, w.rows), dtype=np.float32) for w in ws]
        for w, y in zip(ws, ys):
            if getattr(y, "is_cuda", False) or size_of(y) != k * w.rows or not f32(y):
                raise OuroqError(1, f"output of {size_of(y)} values, expected host [{k}][{w.rows}] float32")
        W = (_p * n)(*[w.handle for w in ws])
        X = (_p * n)(*[_ptr(x) for x in xs])
        Y = (_p * n)(*[_ptr(y) for y in ys])
        self._check(self.lib.ouroq_matmul_q_group(self.ctx, n, W, X, k or 0, Y))
        return ys

    def rotate_fwd(self, x: np.ndarray, signs: np.ndarray | None, block: int) -> np.ndarray:
        """hadamard::rotate_fwd in place on a host fp32 buffer (returns it)."""
        return self._rotate_host(x, signs, block, self.lib.ouroq_rotate_fwd)

    def rotate_inv(self, x: np.ndarray, signs: np.ndarray | None, block: int) -> np.ndarray:
        return self._rotate_host(x, signs, block, self.lib.ouroq_rotate_inv)

    def _rotate_host(self, x, signs, block, fn):
        if x.dtype != np.float32 or not x.flags.c_contiguous:
            raise OuroqError(7, "x must be a contiguous float32 array")
        if signs is not None:
            signs = np.ascontiguousarray(signs, dtype=np.float32)
            if signs.size != x.size:
                raise OuroqError(1, "sign vector must match activation")
        self._check(fn(self.ctx, _ptr(x), _ptr(signs), x.size, block))
        return x
