"""Expert parallelism over two GPUs (gcuda_set_ep, include/geode_cuda.h): each rank computes the routed experts it
owns (expert e on rank e % 2), stores those picks' rows into the other rank's expert-output buffer over NVLink and
waits for the other's (k_ep_exchange: peer memory mapped through CUDA IPC, per-layer flags with bounded waits), and
every rank combines in rank order - so the logits of a verify batch equal the one-GPU step's bit for bit, on both
ranks.
Skipped with fewer than two GPUs. The ranks are child processes; a host barrier before the first collective keeps a
rank whose set-up failed from leaving the other inside one."""
import multiprocessing as mp
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from geode_b200 import synth  # noqa: E402

pytestmark = pytest.mark.gpu


def _shape():
    return synth.ModelShape("wide-moe", "qwen35moe", 1024, 4, 4096, synth.hybrid_types(4), n_heads=4, n_kv_heads=2,
                            head_dim=256, gdn_k_heads=2, gdn_v_heads=4, gdn_k_dim=128, gdn_v_dim=128, n_experts=64,
                            top_k=8, moe_ff=256, shared_ff=256, ctx=600)


def _rank(rank, world, uid, pack_dir, ctx, batches, barrier, q):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    from geode_b200.backend import Backend
    be = None
    try:
        be = Backend(pack_dir, context=ctx, max_tokens=5, device=rank, ep=(rank, world, uid))
        ok = True
    except Exception as e:  # (set-up failed: tell the others at the barrier, then leave)
        q.put((rank, "setup: " + repr(e)))
        ok = False
    try:
        barrier.wait(timeout=120)
    except Exception:
        ok = False
    if not ok:
        barrier.abort()
        return
    out = []
    for toks in batches:
        logits, _ = be.verify(np.asarray(toks, np.int32))
        out.append(logits.copy())
        be.keep(2)
    q.put((rank, out))
    be.close()


def test_ep_two_gpus_bit_exact(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from geode_b200.backend import Backend, ep_unique_id
    shape = _shape()
    d = str(tmp_path / "pack")
    synth.write_pack(d, shape, seed=11)
    rng = np.random.default_rng(3)
    batches = [rng.integers(0, shape.vocab, 5).tolist() for _ in range(3)]
    one = Backend(d, context=shape.ctx, max_tokens=5, device=0)
    ref = []
    for toks in batches:
        logits, _ = one.verify(np.asarray(toks, np.int32))
        ref.append(logits.copy())
        one.keep(2)
    one.close()
    uid = ep_unique_id()
    ctx = mp.get_context("spawn")
    q, barrier = ctx.Queue(), ctx.Barrier(2)
    procs = [ctx.Process(target=_rank, args=(r, 2, uid, d, shape.ctx, batches, barrier, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(2):
            r, v = q.get(timeout=300)
            got[r] = v
    finally:
        for p in procs:
            p.join(60)
            if p.is_alive():
                p.kill()
    for r in range(2):
        assert not isinstance(got[r], str), got[r]
        for a, b in zip(got[r], ref):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
