"""Malformed BMTS shards: the C++ reader (csrc/bmts.cpp, BmtsShard::open of
cluster/src/bmts.rs:171-209) must refuse them with a status, never crash or
read past the file. Seeded mutations of a valid shard -- byte flips in the
header and the JSON tensor table, truncations, random bytes spliced into the
table, grown lengths and offsets -- are opened, listed and read span by span
in a child process, so a crash fails the test instead of killing the runner."""
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

CHILD = r"""
import os, random, sys, tempfile
sys.path.insert(0, sys.argv[1])
import ouroboros_b200 as oq
from ouroboros_b200.bmts import BmtsShard, BmtsTensor, write_shard

rng = random.Random(int(sys.argv[2]))
n_cases = int(sys.argv[3])
tmp = tempfile.mkdtemp()
base_path = os.path.join(tmp, "base.bmts")
tensors = [BmtsTensor("blk.0.ffn_up.weight", [128, 4], 143, 0, 112),
           BmtsTensor("blk.0.attn_k.weight", [256, 2], 34, 112, 108),
           BmtsTensor("token_embd.weight", [8, 4], 1, 220, 64)]
write_shard(base_path, 3, tensors, bytes(range(256)) + bytes(28))
base = open(base_path, "rb").read()
meta_end = 16 + int.from_bytes(base[12:16], "little")
opened = refused = 0
for i in range(n_cases):
    b = bytearray(base)
    kind = rng.randrange(5)
    if kind == 0:    # flip bytes anywhere in header + table
        for _ in range(rng.randint(1, 4)):
            b[rng.randrange(meta_end)] = rng.randrange(256)
    elif kind == 1:  # truncate
        del b[rng.randrange(len(b)):]
    elif kind == 2:  # printable noise inside the JSON table
        for _ in range(rng.randint(1, 6)):
            b[rng.randrange(16, meta_end)] = ord(rng.choice('{}[]":,0123456789-e.ab\\\\'))
    elif kind == 3:  # splice random bytes into the table, fixing up the declared length
        at = rng.randrange(16, meta_end)
        ins = bytes(rng.randrange(256) for _ in range(rng.randint(1, 12)))
        b[at:at] = ins
        b[12:16] = (meta_end - 16 + len(ins)).to_bytes(4, "little")
    else:            # huge numbers for offsets / lengths / shapes
        s = b[16:meta_end].decode("latin-1")
        for key in ('"offset":', '"length":', '"shape":['):
            j = s.find(key)
            if j >= 0 and rng.random() < 0.7:
                k = j + len(key)
                s = s[:k] + str(rng.choice([2**63, 2**64 - 1, 2**32, 10**30, -1])) + s[k:]
        meta = s.encode("latin-1")
        b = b[:12] + len(meta).to_bytes(4, "little") + meta + b[meta_end:]
    path = os.path.join(tmp, "m.bmts")
    with open(path, "wb") as f:
        f.write(bytes(b))
    try:
        sh = BmtsShard(path)
    except oq.OuroqError:
        refused += 1
        continue
    opened += 1
    for t in sh.tensors:
        for off, ln in ((0, t.length), (0, 1), (t.length, 0), (1, t.length)):
            try:
                sh.read_span(t.name, off, ln)
            except oq.OuroqError:
                pass
    sh.close()
print("done", opened, refused)
"""


def test_malformed_shards_are_refused_not_crashed():
    out = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), "20261202", "1500"],
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, (out.returncode, out.stderr[-2000:])
    words = out.stdout.split()
    assert words[0] == "done", out.stdout[-500:]
    opened, refused = int(words[1]), int(words[2])
    assert refused > 100 and opened + refused == 1500
