"""BMTS v1 shard reader (cluster/src/bmts.rs) through the C ABI.

CPU: the reference's own tests restated (test_bmts_roundtrip bmts.rs:433-497,
test_bmts_bad_magic bmts.rs:498-509) plus the other refusals of
BmtsShard::open (short file, truncated meta, count mismatch, version 2,
ranges past the file). GPU: a shard holding Tl1 and TQ1_0 tensors is uploaded
by name and multiplied, bit-identical to the oracle's reference-order matvec.
"""
import struct

import numpy as np
import pytest

import ouroboros_b200 as oq
from ouroboros_b200.bmts import (BMTS_MAGIC, DTYPE_TL1, DTYPE_TQ1_0, BmtsShard, BmtsTensor,
                                 write_shard)


def test_bmts_roundtrip(tmp_path):
    path = str(tmp_path / "shard_1.bmts")
    blob = bytes(range(64))
    tensors = [BmtsTensor("blk.0.attn_q.weight", [8, 8], 34, 0, 32),
               BmtsTensor("blk.0.attn_k.weight", [8, 8], 34, 32, 32)]
    write_shard(path, 1, tensors, blob)
    shard = BmtsShard(path)
    assert shard.node == 1
    assert len(shard.tensors) == 2
    assert shard.data_len == 64
    assert shard.tensors == tensors
    assert bytes(shard.read_tensor("blk.0.attn_q.weight")) == blob[0:32]
    assert bytes(shard.read_tensor("blk.0.attn_k.weight")) == blob[32:64]
    with pytest.raises(oq.OuroqError):
        shard.read_tensor("missing")
    # range fetch of a sub-span, size-stamp checked
    assert bytes(shard.read_span("blk.0.attn_q.weight", 8, 16)) == blob[8:24]
    assert bytes(shard.read_span("blk.0.attn_q.weight", 0, 32)) == blob[0:32]
    with pytest.raises(oq.OuroqError):
        shard.read_span("blk.0.attn_q.weight", 0, 33)
    shard.close()


def test_bmts_bad_magic(tmp_path):
    path = tmp_path / "bad.bmts"
    path.write_bytes(bytes(32))
    with pytest.raises(oq.OuroqError) as ei:
        BmtsShard(str(path))
    assert "magic" in str(ei.value)


def _header(version=1, node=1, n=1, meta_len=0):
    return struct.pack("<IHHII", BMTS_MAGIC, version, node, n, meta_len)


@pytest.mark.parametrize("case", ["short", "meta_truncated", "count", "v2", "not_json"])
def test_bmts_refusals(tmp_path, case):
    path = tmp_path / f"{case}.bmts"
    meta = b'[{"name":"a","shape":[128,4],"dtype":143,"offset":0,"length":112}]'
    if case == "short":
        path.write_bytes(b"OURO")
    elif case == "meta_truncated":
        path.write_bytes(_header(meta_len=len(meta) + 10) + meta)
    elif case == "count":
        path.write_bytes(_header(n=2, meta_len=len(meta)) + meta + bytes(112))
    elif case == "v2":
        path.write_bytes(_header(version=2, meta_len=len(meta)) + meta + bytes(112))
    else:
        path.write_bytes(_header(meta_len=7) + b"not [{}" + bytes(112))
    with pytest.raises(oq.OuroqError):
        BmtsShard(str(path))


def test_bmts_tensor_past_end_of_file(tmp_path):
    path = str(tmp_path / "short_data.bmts")
    write_shard(path, 3, [BmtsTensor("w", [128, 4], DTYPE_TL1, 0, 112)], bytes(50))
    shard = BmtsShard(path)
    assert shard.node == 3
    with pytest.raises(oq.OuroqError) as ei:
        shard.read_tensor("w")
    assert "exceeds file" in str(ei.value)


def test_bmts_json_extras_and_escapes(tmp_path):
    # serde_json output may escape characters and a v1 table may carry extra keys
    path = tmp_path / "extras.bmts"
    meta = (b'[ {"name": "blk.0.\\u0061ttn\\"q", "shape": [8, 8], "dtype": 34, '
            b'"offset": 0, "length": 16, "extra": {"a": [1, 2, {"b": null}], "c": true}} ]')
    path.write_bytes(_header(meta_len=len(meta)) + meta + bytes(range(16)))
    shard = BmtsShard(str(path))
    assert shard.tensors[0].name == 'blk.0.attn"q'
    assert bytes(shard.read_tensor('blk.0.attn"q')) == bytes(range(16))


def _one_entry(extra: bytes, name: bytes = b'"w"') -> bytes:
    return (b'[{"name":' + name + b',"shape":[8,8],"dtype":34,"offset":0,"length":16'
            + extra + b'}]')


def test_bmts_string_escapes_follow_json(tmp_path):
    # a surrogate pair becomes one code point (U+1F600), as serde_json decodes it
    path = tmp_path / "pair.bmts"
    meta = _one_entry(b"", b'"w\\ud83d\\ude00\\/x"')
    path.write_bytes(_header(meta_len=len(meta)) + meta + bytes(16))
    assert BmtsShard(str(path)).tensors[0].name == "w\U0001F600/x"


@pytest.mark.parametrize("case,meta", [
    ("lone_high_surrogate", _one_entry(b"", b'"w\\ud83d"')),
    ("lone_low_surrogate", _one_entry(b"", b'"w\\ude00"')),
    ("unknown_escape", _one_entry(b"", b'"w\\q"')),
    ("raw_control_char", _one_entry(b"", b'"w\tx"')),
    ("nul_in_name", _one_entry(b"", b'"w\\u0000x"')),
    ("invalid_utf8", _one_entry(b"", b'"w\xc3\x28"')),
    ("overlong_utf8", _one_entry(b"", b'"w\xc0\xaf"')),
    ("bad_literal", _one_entry(b',"x":tru')),
    ("bad_number", _one_entry(b',"x":1.e5')),
    ("deep_nesting", _one_entry(b',"x":' + b"[" * 100000 + b"]" * 100000)),
])
def test_bmts_refuses_malformed_json(tmp_path, case, meta):
    # serde_json refuses all of these; so does the reader, without reading past
    # the table or recursing without bound
    path = tmp_path / f"{case}.bmts"
    path.write_bytes(_header(meta_len=len(meta)) + meta + bytes(16))
    with pytest.raises(oq.OuroqError):
        BmtsShard(str(path))


def test_bmts_unknown_values_of_every_json_kind(tmp_path):
    path = tmp_path / "kinds.bmts"
    meta = _one_entry(b',"a":-1.5e3,"b":0,"c":false,"d":null,"e":"s","f":[],"g":{},'
                      b'"h":' + b"[" * 100 + b"]" * 100)
    path.write_bytes(_header(meta_len=len(meta)) + meta + bytes(16))
    assert BmtsShard(str(path)).tensors[0].name == "w"


@pytest.mark.gpu
def test_bmts_upload_and_matvec(ctx, oracle, tmp_path):
    # a small stage shard: one Tl1 and one TQ1_0 projection, GGUF shape [in, out]
    from test_gpu_refmt import tl1_payload, tq1_payload
    k1, m1, k2, m2 = 2560, 384, 512, 96
    p1 = tl1_payload(oracle, m1, k1, seed=11)
    p2 = tq1_payload(oracle, m2, k2, seed=12)
    tensors = [BmtsTensor("blk.0.ffn_up.weight", [k1, m1], DTYPE_TL1, 0, p1.size),
               BmtsTensor("blk.0.attn_k.weight", [k2, m2], DTYPE_TQ1_0, p1.size, p2.size)]
    path = str(tmp_path / "stage.bmts")
    write_shard(path, 2, tensors, p1.tobytes() + p2.tobytes())
    shard = BmtsShard(path)
    w1 = shard.upload(ctx, "blk.0.ffn_up.weight")
    w2 = shard.upload(ctx, "blk.0.attn_k.weight")
    assert (w1.M, w1.K, w2.M, w2.K) == (m1, k1, m2, k2)
    x1 = oracle.normals(13, k1)
    x2 = oracle.normals(14, k2)
    assert np.array_equal(ctx.matvec_q(w1, x1), oracle.matvec_tl1_sse(p1, m1, k1, x1))
    assert np.array_equal(ctx.matvec_q(w2, x2), oracle.matvec_tq1(p2, m2, k2, x2))
    w1.free()
    w2.free()
    shard.close()


def test_bmts_span_arithmetic_does_not_wrap(tmp_path):
    # offsets and lengths near 2^64: a span whose end wraps around must be
    # refused, not mapped onto the start of the file
    path = tmp_path / "wrap.bmts"
    big = 2**64 - 1
    meta = (b'[{"name":"w","shape":[8,8],"dtype":34,"offset":%d,"length":%d}]'
            % (2**64 - 8, big))
    path.write_bytes(_header(meta_len=len(meta)) + meta + bytes(64))
    shard = BmtsShard(str(path))
    for off, ln in ((0, 8), (2**64 - 100, 50), (big, 0), (16, 8)):
        with pytest.raises(oq.OuroqError):
            shard.read_span("w", off, ln)
    shard.close()
    # data offset 0, a huge declared length: a span offset chosen so that
    # data_start + offset wraps to byte 4 of the file (inside its header)
    meta = b'[{"name":"w","shape":[8,8],"dtype":34,"offset":0,"length":%d}]' % big
    path.write_bytes(_header(meta_len=len(meta)) + meta + bytes(64))
    shard = BmtsShard(str(path))
    assert bytes(shard.read_span("w", 0, 16)) == bytes(16)
    with pytest.raises(oq.OuroqError):
        shard.read_span("w", 2**64 - shard.data_start + 4, 8)
    shard.close()
