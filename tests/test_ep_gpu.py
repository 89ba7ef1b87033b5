"""Expert parallelism over two GPUs (gcuda_set_ep, include/geode_cuda.h): each rank computes the routed experts it
owns (expert e on rank e % 2); the down kernel's epilogue stores those picks' rows into the other rank's slot for the
layer over NVLink and its last CTA meets the other rank at the layer's flag (peer memory mapped through CUDA IPC,
bounded waits), and every rank combines in rank order - so the logits of a verify batch equal the one-GPU step's bit
for bit, on both ranks. With the MTP layer, the drafts after each kept step (the MTP layer's own MoE exchanged the
same way) equal the one-GPU drafts bit for bit too.
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


def _steps(be, batches, mtp):
    """verify each batch, keep 2 of its rows; with the MTP layer, then draft over the 2 kept positions (hidden NULL)"""
    out = []
    for toks in batches:
        pos = be.pos
        logits, _ = be.verify(np.asarray(toks, np.int32))
        out.append(logits.copy())
        be.keep(2)
        if mtp:
            d, pr, lg = be.draft(np.array([toks[1], toks[4]], np.int32), pos, logits=True)
            out.append(np.array([d], np.int64))
            out.append(np.array([pr], np.float32))
            out.append(lg.copy())
    return out


def _rank(rank, world, uid, pack_dir, ctx, batches, barrier, q, mtp=False):
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
    out = _steps(be, batches, mtp)
    q.put((rank, out))
    be.close()


@pytest.mark.parametrize("mtp", [False, True])
def test_ep_two_gpus_bit_exact(tmp_path, mtp):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from geode_b200.backend import Backend, ep_unique_id
    shape = _shape()
    d = str(tmp_path / "pack")
    synth.write_pack(d, shape, seed=11, mtp=mtp)
    rng = np.random.default_rng(3)
    batches = [rng.integers(0, shape.vocab, 5).tolist() for _ in range(3)]
    one = Backend(d, context=shape.ctx, max_tokens=5, device=0)
    ref = _steps(one, batches, mtp)
    one.close()
    uid = ep_unique_id()
    ctx = mp.get_context("spawn")
    q, barrier = ctx.Queue(), ctx.Barrier(2)
    procs = [ctx.Process(target=_rank, args=(r, 2, uid, d, shape.ctx, batches, barrier, q, mtp)) for r in range(2)]
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
        assert len(got[r]) == len(ref)
        for a, b in zip(got[r], ref):
            assert np.array_equal(a, b) and np.array_equal(np.ascontiguousarray(a).view(np.uint8),
                                                           np.ascontiguousarray(b).view(np.uint8))
