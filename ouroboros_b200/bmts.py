"""BMTS v1 shard files: the reference's per-stage tensor shard format.

Host mirror of cluster/src/bmts.rs over the C ABI (ouroq_bmts_*):

    shard = BmtsShard("shard_1.bmts")          # BmtsShard::open (bmts.rs:171-209)
    shard.node, shard.tensors                  # header and tensor table
    shard.read_tensor("blk.0.attn_q.weight")   # bytes (bmts.rs:278-281)
    shard.read_span(name, offset, length)      # size-stamp checked (bmts.rs:286-309)
    w = shard.upload(ctx, "blk.0.ffn_up.weight")  # Stage::from_shard + device upload

`write_shard` writes a v1 file the way bmts.rs:312-325 does (used by tools and
tests).
"""
from __future__ import annotations

import ctypes
import json
import struct
from dataclasses import dataclass

import numpy as np

from . import OuroqError, Weight, load_library, PTQ1_0, TQ1_0, F16, BF16

BMTS_MAGIC = 0x4F55524F
BMTS_VERSION = 1
DTYPE_TQ1_0 = 34   # QuantKind::Tq1_0 (dequant.rs:344)
DTYPE_TL1 = 143    # QuantKind::Tl1 (dequant.rs:345)
DTYPE_F16 = 1      # QuantKind::F16 (dequant.rs:337)
DTYPE_BF16 = 30    # QuantKind::Bf16 (dequant.rs:338)


@dataclass
class BmtsTensor:
    name: str
    shape: list
    dtype: int
    offset: int
    length: int


def write_shard(path: str, node: int, tensors: list[BmtsTensor], data: bytes) -> None:
    """Header, compact JSON tensor table (field order of BmtsTensor), data."""
    meta = json.dumps([{"name": t.name, "shape": list(t.shape), "dtype": t.dtype,
                        "offset": t.offset, "length": t.length} for t in tensors],
                      separators=(",", ":")).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<IHHII", BMTS_MAGIC, BMTS_VERSION, node, len(tensors), len(meta)))
        f.write(meta)
        f.write(bytes(data))


class BmtsShard:
    """A memory-mapped BMTS v1 shard (closed with close() or on deletion)."""

    def __init__(self, path: str):
        self.lib = load_library()
        err = ctypes.create_string_buffer(512)
        h = ctypes.c_void_p()
        st = self.lib.ouroq_bmts_open(path.encode(), ctypes.byref(h), err, len(err))
        if st != 0:
            raise OuroqError(st, err.value.decode(errors="replace"))
        self.handle = h.value
        node, n = ctypes.c_int(), ctypes.c_int()
        start, dlen = ctypes.c_uint64(), ctypes.c_uint64()
        self.lib.ouroq_bmts_info(self.handle, ctypes.byref(node), ctypes.byref(n),
                                 ctypes.byref(start), ctypes.byref(dlen))
        self.node, self.data_start, self.data_len = node.value, start.value, dlen.value
        self.tensors = []
        for i in range(n.value):
            name = ctypes.c_char_p()
            rank = ctypes.c_int()
            shape = (ctypes.c_uint64 * 4)()
            dtype = ctypes.c_uint32()
            off, ln = ctypes.c_uint64(), ctypes.c_uint64()
            self.lib.ouroq_bmts_tensor(self.handle, i, ctypes.byref(name), ctypes.byref(rank), shape,
                                       ctypes.byref(dtype), ctypes.byref(off), ctypes.byref(ln))
            self.tensors.append(BmtsTensor(name.value.decode(), list(shape[:rank.value]),
                                           dtype.value, off.value, ln.value))

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.ouroq_bmts_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def read_span(self, name: str, offset: int, length: int) -> np.ndarray:
        err = ctypes.create_string_buffer(512)
        p = ctypes.c_void_p()
        st = self.lib.ouroq_bmts_span(self.handle, name.encode(), offset, length, ctypes.byref(p),
                                      err, len(err))
        if st != 0:
            raise OuroqError(st, err.value.decode(errors="replace"))
        if length == 0:
            return np.zeros(0, np.uint8)
        return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_uint8)),
                                     shape=(length,)).copy()

    def read_tensor(self, name: str) -> np.ndarray:
        t = next((t for t in self.tensors if t.name == name), None)
        if t is None:
            raise OuroqError(7, f"tensor {name} not in shard")
        return self.read_span(name, 0, t.length)

    def upload(self, ctx, name: str) -> Weight:
        """Device copy of a Tl1 / TQ1_0 / F16 / BF16 tensor, shape [in, out] -> (M = out, K = in)."""
        err = ctypes.create_string_buffer(512)
        h = ctypes.c_void_p()
        st = self.lib.ouroq_bmts_upload(ctx.ctx, self.handle, name.encode(), ctypes.byref(h), err,
                                        len(err))
        if st != 0:
            raise OuroqError(st, err.value.decode(errors="replace"))
        t = next(t for t in self.tensors if t.name == name)
        fmt = {DTYPE_TL1: PTQ1_0, DTYPE_TQ1_0: TQ1_0, DTYPE_F16: F16, DTYPE_BF16: BF16}[t.dtype]
        return Weight(ctx, h.value, fmt, int(t.shape[1]), int(t.shape[0]))
