"""The multi-process host logic of bench.py on CPU (gloo, world size 2): the timing reduction takes the slowest
rank, every rank gets it, and the reference arm runs on rank 0 alone."""
import os
import sys

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    sys.path.insert(0, ROOT)
    import datetime
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        got = bench.max_over_ranks(10.0 + 5.0 * rank, dist, "cpu")
        out[rank] = got
        # the reference arm: ranks other than 0 return at once, without timing anything
        if rank != 0:
            class A:
                steps, warmup, gpus = 1, 1, world
            out[world + rank] = bench.reference_arm(A())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_gloo():
    world = 2
    port = 29500 + os.getpid() % 2000
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    procs = [ctx.Process(target=_rank, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert out[0] == out[1] == 15.0
    assert out[world + 1] == 0


def test_max_over_ranks_single():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.max_over_ranks(3.5, None, "cpu") == 3.5


def test_cpu_accept_reference_leg():
    """The acceptance microbench's CPU leg (bench.py --workload cfg5: its cpu_baseline and its --impl reference arm):
    the reference engine's greedy rule and the rejection-sampling port over a small sample give positive rates in the
    GPU line's unit."""
    import bench
    cb = bench.cpu_accept_reference(seqs=3)
    assert cb["unit"] == bench.ACCEPT_UNIT and cb["value"] > 0 and cb["rejection_port_sequences_per_s"] > 0
    assert cb["kind"] in ("reference", "port") and cb["cores"] == 1
