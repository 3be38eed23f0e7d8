"""Multi-rank host logic on CPU (gloo, world size 2): row partition, sharded
row ops equal to the unsharded op, the single all-reduce of per-rank
reduction partials, and failure detection when a rank dies (no GPU involved:
the per-rank compute is the CPU oracle)."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import PKG, ROOT


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_row_range_covers_rows_once():
    from oxide_b200.dist import row_range

    for rows in (0, 1, 7, 8, 131072, 1000003):
        for world in (1, 2, 3, 4, 8):
            blocks = [row_range(rows, r, world) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == rows
            assert all(blocks[i][1] == blocks[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in blocks]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        row_range(10, 2, 2)


def _worker(rank, world, port, q, mode):
    sys.path[:0] = [ROOT, PKG]
    import datetime

    import torch
    import torch.distributed as dist

    from oracle import oracle as orc
    from oxide_b200.dist import combine_partial, row_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        rng = np.random.default_rng(4)
        rows, cols = 37, 256
        x = rng.standard_normal((rows, cols), dtype=np.float32)
        w = rng.uniform(0.5, 1.5, cols).astype(np.float32)
        lo, hi = row_range(rows, rank, world)
        if mode == "ops":
            y = orc.rms_norm(x[lo:hi], w, 1e-5)
            got = [None] * world
            dist.all_gather_object(got, (lo, y))
            full = np.concatenate([blk for _, blk in sorted(got, key=lambda t: t[0])])
            ok_rows = np.array_equal(full, orc.rms_norm(x, w, 1e-5))
            res = {}
            for op in (0, 1, 2):
                part = torch.tensor([orc.reduce(op, x[lo:hi])], dtype=torch.float64)
                total = float(combine_partial(part.view(()), op))
                res[op] = total
            q.put((rank, ok_rows, res, {op: orc.reduce(op, x) for op in (0, 1, 2)}))
        else:  # "fail": rank 1 dies before the collective; rank 0 must error, not hang
            if rank == 1:
                os._exit(3)
            part = torch.tensor(1.0, dtype=torch.float64)
            try:
                combine_partial(part, 0)
                q.put((rank, "no error"))
            except Exception as e:  # the collective reports the lost peer
                q.put((rank, f"error: {type(e).__name__}"))
    finally:
        if mode == "ops":
            dist.destroy_process_group()


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    for _ in range(world if mode == "ops" else 1):
        out.append(q.get(timeout=120))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_sharded_rows_and_reductions_match_unsharded():
    results = _run("ops")
    assert len(results) == 2
    for rank, ok_rows, res, ref in results:
        assert ok_rows, f"rank {rank}: sharded RMSNorm differs from the unsharded op"
        assert res[1] == ref[1]  # max is exact
        for op in (0, 2):
            assert abs(res[op] - ref[op]) <= 1e-12 * max(1.0, abs(ref[op]))


def test_dead_rank_is_detected_by_collective_timeout():
    (rank, status), = _run("fail")
    assert rank == 0 and status.startswith("error"), status
