"""The expert-parallel exchange on CPU (two spawned ranks): the scheme gcuda_set_ep runs on the device (k_ep_tick,
k_ep_exchange in geode_b200/csrc/ep_exchange.cuh), restated on the host with a torch.distributed TCPStore standing in
for the peers' mapped memory. Per step the epoch advances and every rank meets every peer at the step-start flags;
per MoE layer each rank stores the rows of the picks whose expert it owns (expert e on rank e % world) into every
peer's slot for that layer, then raises its flag for the layer in every peer (the epoch, after the rows), then waits -
bounded - until every peer's flag holds the epoch. Every pick's row then comes from exactly one rank, and the
rank-order combine gives the same bits as one rank holding everything, over several steps and layers. A rank that
never arrives makes the other's bounded wait give up with an error (the device's kErrWaitTimeout) instead of waiting
for good."""
import datetime
import os
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

N, K, H, E = 5, 8, 64, 32
LAYERS, STEPS = 3, 2
WAIT_S = 3.0


def _routes(step, layer):
    rng = np.random.default_rng(1000 * step + layer)
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


def _wait_flag(store, key, epoch, what):
    """The bounded acquire wait: poll the flag until it holds the epoch, give up after WAIT_S."""
    end = time.monotonic() + WAIT_S
    while not (store.check([key]) and int(store.get(key)) == epoch):
        if time.monotonic() > end:
            raise TimeoutError(f"wait gave up: {what}")
        time.sleep(1e-3)


def _tick(store, rank, world, epoch):
    for dst in range(world):
        if dst != rank:
            store.set(f"flag/{dst}/tick/{rank}", str(epoch))
    for src in range(world):
        if src != rank:
            _wait_flag(store, f"flag/{rank}/tick/{src}", epoch, f"rank {src} at the start of step {epoch}")


def _exchange(store, rank, world, layer, epoch, ids, y):
    owner = ids.reshape(-1) % world
    eout = np.zeros_like(y)
    eout[owner == rank] = y[owner == rank]                 # this rank's own picks, computed here
    for dst in range(world):                               # the peer stores, then the release of the flag
        if dst == rank:
            continue
        for p in np.nonzero(owner == rank)[0]:
            store.set(f"slot/{dst}/{layer}/{p}", eout[p].tobytes())
        store.set(f"flag/{dst}/{layer}/{rank}", str(epoch))
    for src in range(world):
        if src == rank:
            continue
        _wait_flag(store, f"flag/{rank}/{layer}/{src}", epoch, f"rank {src} at layer {layer} of step {epoch}")
        for p in np.nonzero(owner == src)[0]:
            eout[p] = np.frombuffer(store.get(f"slot/{rank}/{layer}/{p}"), np.float32)
    return eout


def _rank(rank, world, port, out, fail_rank):
    try:
        store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
        res = []
        for step in range(1, STEPS + 1):
            if rank == fail_rank and step == STEPS:
                raise RuntimeError("planted failure: this rank leaves before the step")
            _tick(store, rank, world, step)
            for layer in range(LAYERS):
                ids, w, y = _routes(step, layer)
                eout = _exchange(store, rank, world, layer, step, ids, y)
                res.append((eout, _combine(ids, w, eout)))
        out[rank] = res
        if rank == 0:
            time.sleep(0.5)   # (the store's host stays up until the peer has read its last rows)
    except (RuntimeError, TimeoutError) as e:
        out[rank] = str(e)


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
    for r in range(2):
        assert not isinstance(out[r], str), out[r]
        i = 0
        for step in range(1, STEPS + 1):
            for layer in range(LAYERS):
                ids, w, y = _routes(step, layer)
                eout, x = out[r][i]
                i += 1
                assert np.array_equal(eout.view(np.uint32), y.view(np.uint32))
                assert np.array_equal(x.view(np.uint32), _combine(ids, w, y).view(np.uint32))


def test_missing_rank_ends_the_wait():
    out = _run(1)
    assert "planted failure" in out[1]
    assert isinstance(out[0], str) and "wait gave up" in out[0], out[0]   # bounded: rank 0 did not wait for good
