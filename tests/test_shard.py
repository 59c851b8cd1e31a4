"""Program-id sharding (easy_as_b200.shard) on CPU: 2 gloo ranks, each computes its
slice of the add kernel with the CPU oracle, then the slices are gathered to rank 0
and compared with one whole-grid oracle run."""

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from easy_as_b200.shard import element_range, gather, program_range


def test_program_range_is_a_partition():
    for total in (0, 1, 7, 1031, 2 ** 18):
        for world in (1, 2, 3, 4, 8):
            ranges = [program_range(total, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [hi - lo for lo, hi in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_element_range_whole_programs():
    n, block = 1031, 256
    rs = [element_range(n, block, r, 2) for r in range(2)]
    assert rs == [(0, 512), (512, 1031)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent
    sys.path[:0] = [str(root.parent), str(root)]
    import goldens
    from oracle.interp import execute

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = goldens.case("add_c1")  # N = 1031, BLOCK = 256: uneven split (2 + 3 programs)
        ir = goldens.ir_from_json(c["opt"])
        rng = np.random.default_rng(0)
        n = 1031
        a = rng.standard_normal(n, dtype=np.float32)
        b = rng.standard_normal(n, dtype=np.float32)
        lo, hi = element_range(n, 256, rank, world)
        out_local = np.zeros(hi - lo, np.float32)
        execute(ir, {"a": a[lo:hi].copy(), "b": b[lo:hi].copy(), "c": out_local, "N": hi - lo})
        counts = [element_range(n, 256, r, world)[1] - element_range(n, 256, r, world)[0] for r in range(world)]
        full = torch.zeros(n) if rank == 0 else None
        gather(torch.from_numpy(out_local), full, counts, dst=0)
        if rank == 0:
            ref = np.zeros(n, np.float32)
            execute(ir, {"a": a, "b": b, "c": ref, "N": n})
            result["ok"] = bool(np.array_equal(full.numpy(), ref))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_shard_and_gather():
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert result.get("ok") is True
