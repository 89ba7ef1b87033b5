"""The expert-parallel exchange on CPU (gloo ranks, world size 2): the scheme gcuda_set_ep runs on the device, restated
with numpy on the host. Each rank fills the rows of the picks whose expert it owns (expert e on rank e % world) and
leaves the others zero; a sum all-reduce then gives every rank every row exactly (one non-zero term per element), and
the rank-order combine gives the same bits as one rank holding everything. A rank that fails before the exchange
makes the other's collective end with an error at the group's timeout, instead of waiting for good."""
import datetime
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

N, K, H, E = 5, 8, 64, 32


def _routes():
    rng = np.random.default_rng(7)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(N)])             # [N][K] picks
    w = rng.random((N, K)).astype(np.float32)
    y = (rng.standard_normal((N * K, H)) * 3).astype(np.float32)                     # every pick's expert output
    return ids, w, y


def _combine(ids, w, eout):
    x = np.zeros((N, H), np.float32)
    for t in range(N):
        o = np.zeros(H, np.float32)
        for k in range(K):
            o = (o + w[t, k] * eout[t * K + k]).astype(np.float32)   # rank order
        x[t] = o
    return x


def _rank(rank, world, port, out, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        ids, w, y = _routes()
        mine = (ids.reshape(-1) % world) == rank
        eout = np.where(mine[:, None], y, np.float32(0)).astype(np.float32)
        if rank == fail_rank:
            raise RuntimeError("planted failure before the exchange")
        t = torch.from_numpy(eout)
        dist.all_reduce(t)
        out[rank] = (t.numpy().copy(), _combine(ids, w, t.numpy()))
    except RuntimeError as e:
        out[rank] = str(e)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(fail_rank):
    world = 2
    port = 29600 + os.getpid() % 2000 + (0 if fail_rank < 0 else 7)
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    procs = [ctx.Process(target=_rank, args=(r, world, port, out, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode is not None
    return dict(out)


def test_exchange_is_exact():
    out = _run(-1)
    ids, w, y = _routes()
    ref = _combine(ids, w, y)
    for r in range(2):
        eout, x = out[r]
        assert np.array_equal(eout.view(np.uint32), y.view(np.uint32))
        assert np.array_equal(x.view(np.uint32), ref.view(np.uint32))


def test_failed_rank_ends_the_exchange():
    out = _run(1)
    assert "planted failure" in out[1]
    assert isinstance(out[0], str)   # rank 0's all-reduce ended with an error (no peer), it did not wait for good
