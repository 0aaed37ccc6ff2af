"""Row-sharded matmul on 2 GPUs: ouroq_gemm_sharded against the oracle.

Each case runs as two child processes, one per GPU. They exchange the group
id over a gloo process group (host only), join the library's NCCL group, and
upload only their own rows of the same full matrix. The full y on every rank
must equal the unsharded oracle result bit for bit. NVLink SHARP (NVLS) is off
in the children, as required for tests where a rank may leave a group.

Skipped when fewer than two GPUs are visible.
"""
import os
import socket

import numpy as np
import pytest

import ouroboros_b200 as oq

pytestmark = pytest.mark.gpu

CASES = [  # (format, M, K, B, hadamard block)
    (oq.TERNARY2, 4096, 2048, 1, 0),
    (oq.TERNARY2, 4096, 2048, 5, 0),
    (oq.TERNARY2, 2048, 4096, 16, 0),   # tensor-core path on each rank
    (oq.SIGN1G128, 2048, 1024, 3, 128),
    (oq.TERNARY2, 28672, 8192, 1, 0),   # config-5 up/gate shape
]


def _need_gpus(n):
    import torch
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case_data(O, fmt, M, K, B, block, seed):
    x = O.outliers(seed + 2, O.normals(seed + 3, B * K), 0.01, 20.0).reshape(B, K)
    sg = O.signs(seed + 4, K).astype(np.float32) if block else None
    if fmt == oq.TERNARY2:
        w = O.ternary(seed, M * K).reshape(M, K)
        return O.pack_tern2(w), None, O.absmean_scale(w, 0.02), x, sg
    w = O.signs(seed, M * K).reshape(M, K)
    sc = O.group_scales(seed + 1, M * (K // 128), 0.02)
    return O.pack_sign1(w), sc, 1.0, x, sg


def _worker(rank, world, port, mode, out_q, transport="peer"):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import torch
    import torch.distributed as dist
    from oracle import pyoracle as O
    from ouroboros_b200 import shard
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    ctx = oq.Context(rank)
    try:
        shard.join(ctx)
        ctx.shard_set_transport(transport)
        if mode == "cases":
            for i, (fmt, M, K, B, block) in enumerate(CASES):
                packed, sc, ws, x, sg = _case_data(O, fmt, M, K, B, block, 100 + i)
                w = ctx.upload_shard(fmt, packed, M, K, sc, ws)
                xd = torch.from_numpy(x).cuda()
                sgd = torch.from_numpy(sg).cuda() if sg is not None else None
                y = ctx.gemm_sharded(w, xd, signs=sgd, hadamard_block=block)
                ctx.shard_sync(timeout_ms=30000)
                out_q.put(("y", rank, i, y.cpu().numpy()))
                w.free()
            ctx.shard_finalize()
        else:
            # rank 1 leaves between steps: it never enters the second product.
            # Rank 0's gather cannot complete; its bounded sync must report
            # a timeout and mark the group failed, and finalize then aborts it.
            fmt, M, K, B, block = CASES[0]
            packed, sc, ws, x, sg = _case_data(O, fmt, M, K, B, block, 100)
            w = ctx.upload_shard(fmt, packed, M, K, sc, ws)
            xd = torch.from_numpy(x).cuda()
            ctx.gemm_sharded(w, xd)
            ctx.shard_sync(timeout_ms=30000)
            status = 0
            if rank == 0:
                ctx.gemm_sharded(w, xd)
                try:
                    ctx.shard_sync(timeout_ms=1500)
                except oq.OuroqError as e:
                    status = e.status
                try:
                    ctx.gemm_sharded(w, xd)
                    later = 0
                except oq.OuroqError as e:
                    later = e.status
                ctx.shard_finalize()
                out_q.put(("timeout", rank, status, later))
            dist.barrier()
            if rank != 0:
                ctx.shard_finalize()
                out_q.put(("timeout", rank, 0, 0))
            w.free()
    finally:
        ctx.close()
        dist.destroy_process_group()


def _run(world, mode, transport="peer"):
    import torch.multiprocessing as mp
    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    port = _free_port()
    procs = [mctx.Process(target=_worker, args=(r, world, port, mode, q, transport))
             for r in range(world)]
    for p in procs:
        p.start()
    n_expected = world * len(CASES) if mode == "cases" else world
    out = [q.get(timeout=600) for _ in range(n_expected)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return out


@pytest.mark.parametrize("transport", ["peer", "nccl"])
def test_sharded_matches_oracle_on_two_gpus(oracle, transport):
    _need_gpus(2)
    out = _run(2, "cases", transport)
    for i, (fmt, M, K, B, block) in enumerate(CASES):
        packed, sc, ws, x, sg = _case_data(oracle, fmt, M, K, B, block, 100 + i)
        q, s = oracle.quantize_act(x, sg, block)
        if fmt == oq.TERNARY2:
            _, want = oracle.gemm_tern2(packed, M, K, ws, q, s)
        else:
            _, want = oracle.gemm_sign1(packed, sc, M, K, q, s)
        got = [y for kind, r, j, y in out if kind == "y" and j == i]
        assert len(got) == 2
        for y in got:
            assert np.array_equal(y, want), f"case {i}"


@pytest.mark.parametrize("transport", ["peer", "nccl"])
def test_sharded_sync_times_out_when_a_rank_leaves(oracle, transport):
    _need_gpus(2)
    out = _run(2, "timeout", transport)
    r0 = [o for o in out if o[1] == 0][0]
    assert r0[2] == 5  # OUROQ_ERR_TIMEOUT
    assert r0[3] == 4  # later calls: OUROQ_ERR_NCCL (group marked failed)
