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


def test_step_bytes_match_the_hand_computed_figures():
    """The roofline's algorithmic bytes per verify step (bench.step_bytes) against figures worked out by hand from the
    model shapes: an expert block is gate_up q4 [1024][2048] + down q4 [2048][512] = 1 769 472 B; the LM head
    248320 x 2048 at 9/16 B = 286 064 640 B; cfg 3 = 925 MB dense + 37.6 experts x 40 layers + 67 MB of recurrent
    and conv state (read and written) + 170 MB of KV at 8192 positions = 3.82 GB; cfg 2 = 1.11 GB of weights + 40 MB
    state + 51 MB KV = 1.20 GB; cfg 1 = 67 MB of weights, 69 MB in all."""
    import bench
    from geode_b200 import synth
    s3 = synth.baseline_shape(3)
    q4 = lambda r, c: r * c * 9 // 16
    assert q4(2 * s3.moe_ff, s3.hidden) + q4(s3.hidden, s3.moe_ff) == 1769472
    assert q4(s3.vocab, s3.hidden) == 286064640
    b3 = bench.step_bytes(s3, 37.6, 8192)
    assert abs(b3["experts"] - 37.6 * 40 * 1769472) <= 40   # (rounded to a byte per layer)
    assert abs(b3["total"] / 3.82e9 - 1) < 0.005 and abs(b3["dense"] / 925e6 - 1) < 0.002
    assert abs(b3["kv"] / 170e6 - 1) < 0.01 and abs(b3["state"] / 67e6 - 1) < 0.01
    b2 = bench.step_bytes(synth.baseline_shape(2), 0, 4096)
    assert abs(b2["total"] / 1.20e9 - 1) < 0.01 and abs(b2["state"] / 40e6 - 1) < 0.02
    b1 = bench.step_bytes(synth.baseline_shape(1), 0, 1024)
    assert abs(b1["dense"] / 67.3e6 - 1) < 0.01 and abs(b1["total"] / 69.0e6 - 1) < 0.01
