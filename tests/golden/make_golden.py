"""Regenerates the golden fixtures in this folder from the REFERENCE engine's own code (oracle/_ref/libgeode_ref.so,
compiled from the reference sources by oracle/Makefile): every output here was computed by the reference, not by the
restatement, so tests/test_oracle.py pins the restatement to the reference wherever the reference build is absent
(the GPU box). Run from the repository root: python tests/golden/make_golden.py

- kernels.npz: the E4M3 table, quantize_activation, matvec_rows_q_multi, matvec_rows_bf16_multi, route_topk, rmsnorm,
  fast_exp (engine/src/kernels.cpp, engine/src/model.cpp:4021), the q4 block quantizer (engine/src/yue2_q4.cpp:88) and
  the sampler's uniform stream (std::mt19937_64 + generate_canonical, engine/src/sampler.cpp:45);
- accept.npz: the acceptance rule (engine/src/geode.cpp:327-350) around geode::Sampler, greedy and sampled;
- accept_seen.npz: the same with geode_generate's presence penalty (engine/src/geode.cpp:234-255);
- model_moe.npz / model_dense.npz: Model::forward_batch over a prompt and a 5-token verify batch on a tiny synthetic
  pack (written by geode_b200/synth.py with the seed stored), every logit and the per-layer trace;
- state_file.npz: Model::save_state's file (engine/src/state.cpp) after a 20-token prompt on a tiny synthetic pack,
  with that pack's geode.json (the state's fingerprint hashes it) and the shapes the state records;
- state_file_mtp.npz: the same on a pack with the MTP layer (the model opened with drafting on), after the prompt and
  the MTP layer over all its positions (the last one fed the token after the prompt): the file with the layer's KV
  slot and the last hidden row, the reference's hidden rows and that next token;
- mtp_moe.npz / mtp_dense.npz: the MTP drafting layer (Model::forward_mtp, engine/src/model.cpp:4965-5039) on a tiny
  pack with one: the main model's hidden rows after a prompt, the MTP pass over the prompt's positions (logits and
  normed output of the last), then one chained position fed its own draft.

Run with names (kernels, accept, accept_seen, model, state, state_mtp, mtp) to regenerate only those fixtures.
"""
import ctypes as C
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from geode_b200 import synth  # noqa: E402
import oracle_py as op  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def kernels(R):
    rng = np.random.default_rng(20261201)
    g = {}
    g["e4m3"] = np.array([R.ref_e4m3_value(b) for b in range(256)], np.float32)
    x = (rng.standard_normal(512) * 3).astype(np.float32)
    x[:16] = 0.0
    q, s, b = np.zeros(512, np.int8), np.zeros(32, np.float32), np.zeros(32, np.int32)
    R.ref_quantize_activation(x.ctypes.data, 512, q.ctypes.data, s.ctypes.data, b.ctypes.data)
    g.update(act_x=x, act_q=q, act_scale=s, act_bsum=b)
    w, gl = synth.q4_quantize((rng.standard_normal((32, 512)) * 0.02).astype(np.float32))
    xs = rng.standard_normal((5, 512)).astype(np.float32)
    y = np.zeros((5, 32), np.float32)
    R.ref_matvec_q(w.ctypes.data, 32, 512, C.c_float(gl), 6, 5, xs.ctypes.data, y.ctypes.data)
    g.update(w_packed=w, w_rows=32, w_cols=512, w_global=np.float32(gl), w_x=xs, w_y=y)
    bw = synth.bf16_bits((rng.standard_normal((33, 256)) * 0.05).astype(np.float32))
    bx = rng.standard_normal((5, 256)).astype(np.float32)
    by = np.zeros((5, 33), np.float32)
    R.ref_matvec_bf16_multi(bw.ctypes.data, 33, 256, 5, bx.ctypes.data, by.ctypes.data)
    g.update(bf_w=bw, bf_x=bx, bf_y=by)
    lg = (rng.standard_normal((8, 256)) * 2).astype(np.float32)
    ids, wt = np.zeros((8, 8), np.int32), np.zeros((8, 8), np.float32)
    for t in range(8):
        R.ref_route_topk(lg[t].ctypes.data, 256, 8, ids[t].ctypes.data, wt[t].ctypes.data)
    g.update(rt_logits=lg, rt_k=8, rt_ids=ids, rt_w=wt)
    rx = (rng.standard_normal(2048) * 4).astype(np.float32)
    rw = (rng.standard_normal(2048) * 0.1).astype(np.float32)
    ry = np.zeros(2048, np.float32)
    R.ref_rmsnorm(rx.ctypes.data, rw.ctypes.data, ry.ctypes.data, 2048, C.c_float(1e-6), 1)
    g.update(rn_x=rx, rn_w=rw, rn_y=ry)
    fx = np.concatenate([rng.standard_normal(200) * 20, [-100.0, 100.0, 0.0, -87.0, 88.0, 1e-8]]).astype(np.float32)
    g.update(fe_x=fx, fe_y=np.array([R.ref_fast_exp(float(v)) for v in fx], np.float32))
    u = np.zeros(16, np.float64)
    R.ref_uniforms(C.c_uint64(1234), 16, u.ctypes.data)
    g.update(mt_seed=1234, mt_u=u)
    # the q4 quantizer: blocks through the reference's q4_block, assembled into the pack's row layout
    qw = (rng.standard_normal((8, 256)) * 0.02).astype(np.float32)
    qw[0, :16] = 0.0
    s2 = np.float32(np.float32(np.abs(qw).max()) * np.float32(1.25) / np.float32(15.0 * 448.0))
    packed = np.zeros((8, 256 // 16 * 9), np.uint8)
    for r in range(8):
        for blk in range(16):
            sb = C.c_uint8(0)
            codes = np.zeros(16, np.uint8)
            R.ref_q4_block(np.ascontiguousarray(qw[r, 16 * blk: 16 * blk + 16]).ctypes.data, C.c_float(s2), C.byref(sb),
                           codes.ctypes.data)
            packed[r, 8 * blk: 8 * blk + 8] = codes[0::2] | (codes[1::2] << 4)
            packed[r, 128 + blk] = sb.value
    g.update(qz_w=qw, qz_s2=s2, qz_packed=packed)
    np.savez_compressed(os.path.join(OUT, "kernels.npz"), **g)


def accept(R):
    rng = np.random.default_rng(77)
    V = 4096
    cases = [(0.0, 1.0, 0), (0.7, 0.95, 20), (0.7, 1.0, 0), (1.3, 0.8, 40), (0.5, 0.9, 0), (0.0, 1.0, 0)]
    rows = (rng.standard_normal((len(cases), 5, V)) * 3).astype(np.float32)
    batch = rng.integers(0, V, (len(cases), 5)).astype(np.int32)
    params, kept, nxt, samples = [], [], [], []
    for c, (T, P, K) in enumerate(cases):
        for i in range(c % 5):   # planted drafts that stand (greedy rows)
            batch[c, i + 1] = int(np.argmax(rows[c, i]))
        seed = int(rng.integers(0, 2 ** 40))
        n = C.c_int(0)
        s = np.zeros(5, np.int32)
        k = R.ref_accept(rows[c].ctypes.data, 5, V, batch[c].ctypes.data, T, P, K, C.c_uint64(seed), None, 0, C.byref(n),
                         s.ctypes.data)
        params.append((T, P, K, seed))
        kept.append(k)
        nxt.append(n.value)
        samples.append(s)
    np.savez_compressed(os.path.join(OUT, "accept.npz"), rows=rows, batch=batch, params=np.array(params, np.float64),
                        kept=np.array(kept), next=np.array(nxt), samples=np.array(samples))


def accept_seen(R):
    """The acceptance with geode_generate's presence penalty (engine/src/geode.cpp:234-255): seen lists that hold
    some rows' greedy maxima, drafts planted as the penalised greedy samples (they stand only under the penalty), a
    draft repeated and one already seen."""
    rng = np.random.default_rng(91)
    V = 4096
    cases = [(0.0, 1.0, 0, 2.5), (0.7, 0.95, 20, 1.5), (0.0, 1.0, 0, -0.75), (1.1, 0.9, 40, 3.0), (0.0, 1.0, 0, 0.0),
             (0.7, 1.0, 0, 0.5)]
    rows = (rng.standard_normal((len(cases), 5, V)) * 3).astype(np.float32)
    batch = rng.integers(0, V, (len(cases), 5)).astype(np.int32)
    params, seen_in, n_in, kept, nxt, samples, seen_out, n_out = [], [], [], [], [], [], [], []
    for c, (T, P, K, pen) in enumerate(cases):
        seen = list(rng.choice(V, 12, replace=False))
        seen[0] = int(np.argmax(rows[c, 0]))   # row 0's maximum is penalised
        seen[1] = int(np.argmax(rows[c, 2]))
        op.plant_penalized_drafts(rows[c], batch[c], seen, pen, 1 + c % 4)
        if c == 2:
            batch[c, 4] = batch[c, 3]   # a draft repeated (it joins seen once)
        if c == 3:
            batch[c, 1] = seen[5]       # a draft already seen
        seed = int(rng.integers(0, 2 ** 40))
        k, n, s, so = op.accept_seen(R, rows[c], batch[c], T, P, K, seed, pen, seen, fn="ref_accept_seen")
        params.append((T, P, K, seed, pen))
        seen_in.append(np.pad(np.array(seen, np.int32), (0, 8)))
        n_in.append(len(seen))
        kept.append(k)
        nxt.append(n)
        samples.append(s)
        seen_out.append(np.pad(so, (0, 20 - len(so))))
        n_out.append(len(so))
    np.savez_compressed(os.path.join(OUT, "accept_seen.npz"), rows=rows, batch=batch,
                        params=np.array(params, np.float64), seen=np.array(seen_in), n_seen=np.array(n_in),
                        kept=np.array(kept), next=np.array(nxt), samples=np.array(samples),
                        seen_out=np.array(seen_out), n_seen_out=np.array(n_out))


def model(arch, name, seed=21, attn_block=64):
    shape = synth.tiny_shape(arch, n_layers=4, ctx=640)
    with tempfile.TemporaryDirectory() as d:
        synth.write_pack(d, shape, seed=seed)
        ref = op.Reference(d, threads=4, ctx=shape.ctx, attn_block=attn_block)
        rng = np.random.default_rng(seed + 1)
        prompt = rng.integers(0, shape.vocab, 100).astype(np.int32)
        toks = rng.integers(0, shape.vocab, 5).astype(np.int32)
        r1 = ref.forward(prompt)
        r2 = ref.forward(toks, trace=True)
        out = dict(seed=seed, attn_block=attn_block, prompt=prompt, toks=toks, prompt_logits=r1["logits"],
                   logits=r2["logits"])
        for k in ("x", "mixer", "moe", "out", "ids", "weights"):
            out["trace_" + k] = r2["trace"][k]
        ref.close()
    np.savez_compressed(os.path.join(OUT, name + ".npz"), **out)


def state_file(seed=31):
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    with tempfile.TemporaryDirectory() as d:
        synth.write_pack(d, shape, seed=seed)
        ref = op.Reference(d, threads=1, ctx=shape.ctx)
        prompt = np.random.default_rng(seed + 1).integers(0, shape.vocab, 20).astype(np.int32)
        ref.forward(prompt, all_logits=False)
        path = os.path.join(d, "s.state")
        ref.save_state(path)
        ref.close()
        ora = op.Oracle(d)
        c = ora.cfg
        conv_dim = 2 * c.gdn_k_heads * c.gdn_k_dim + c.gdn_v_heads * c.gdn_v_dim
        shapes = np.array([ora.n_attn, c.n_kv_heads, c.n_kv_heads * c.head_dim, c.hidden, c.n_layers,
                           ora.n_gdn * conv_dim * (c.conv_kernel - 1),
                           ora.n_gdn * c.gdn_v_heads * c.gdn_k_dim * c.gdn_v_dim], np.uint64)
        manifest = np.frombuffer(open(os.path.join(d, "geode.json"), "rb").read(), np.uint8)
        state = np.frombuffer(open(path, "rb").read(), np.uint8)
    np.savez_compressed(os.path.join(OUT, "state_file.npz"), seed=seed, prompt=prompt, shapes=shapes,
                        manifest=manifest, state=state)


def state_file_mtp(seed=33):
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    with tempfile.TemporaryDirectory() as d:
        synth.write_pack(d, shape, seed=seed, mtp=True)
        ref = op.Reference(d, threads=1, ctx=shape.ctx, draft=True)
        toks = np.random.default_rng(seed + 1).integers(0, shape.vocab, 21).astype(np.int32)
        prompt, nxt = toks[:20], int(toks[20])
        ref.forward(prompt, all_logits=False)
        hid = ref.hidden_rows(len(prompt))
        ref.mtp(np.append(prompt[1:], nxt), hid, 0, logits=False)   # (every position's MTP KV row written)
        path = os.path.join(d, "s.state")
        ref.save_state(path)
        ref.close()
        ora = op.Oracle(d)
        c = ora.cfg
        conv_dim = 2 * c.gdn_k_heads * c.gdn_k_dim + c.gdn_v_heads * c.gdn_v_dim
        shapes = np.array([ora.n_attn + 1, c.n_kv_heads, c.n_kv_heads * c.head_dim, c.hidden, c.n_layers,
                           ora.n_gdn * conv_dim * (c.conv_kernel - 1),
                           ora.n_gdn * c.gdn_v_heads * c.gdn_k_dim * c.gdn_v_dim, 1], np.uint64)
        manifest = np.frombuffer(open(os.path.join(d, "geode.json"), "rb").read(), np.uint8)
        state = np.frombuffer(open(path, "rb").read(), np.uint8)
    np.savez_compressed(os.path.join(OUT, "state_file_mtp.npz"), seed=seed, prompt=prompt, next=nxt, hidden=hid,
                        shapes=shapes, manifest=manifest, state=state)


def mtp(arch, name, seed=41):
    shape = synth.tiny_shape(arch, n_layers=4, ctx=640)
    with tempfile.TemporaryDirectory() as d:
        synth.write_pack(d, shape, seed=seed, mtp=True)
        ref = op.Reference(d, threads=1, ctx=shape.ctx, draft=True)
        prompt = np.random.default_rng(seed + 1).integers(0, shape.vocab, 40).astype(np.int32)
        ref.forward(prompt, all_logits=False)
        hid = ref.hidden_rows(len(prompt))
        lg1, h1 = ref.mtp(prompt[1:], hid[:-1], 0)
        draft = int(np.argmax(lg1))
        lg2, h2 = ref.mtp([draft], h1[None], len(prompt) - 1)
        ref.close()
    np.savez_compressed(os.path.join(OUT, name + ".npz"), seed=seed, prompt=prompt, hidden=hid, logits1=lg1,
                        mtp_hidden1=h1, draft=draft, logits2=lg2, mtp_hidden2=h2)


if __name__ == "__main__":
    if not op.have_reference():
        sys.exit("build the reference first: make -C oracle ref")
    R = op.reference_lib()
    which = set(sys.argv[1:]) or {"kernels", "accept", "accept_seen", "model", "state", "state_mtp", "mtp"}
    if "kernels" in which:
        kernels(R)
    if "accept" in which:
        accept(R)
    if "accept_seen" in which:
        accept_seen(R)
    if "model" in which:
        model("qwen35moe", "model_moe")
        model("qwen35", "model_dense")
    if "state" in which:
        state_file()
    if "state_mtp" in which:
        state_file_mtp()
    if "mtp" in which:
        mtp("qwen35moe", "mtp_moe")
        mtp("qwen35", "mtp_dense")
    print("written to", OUT)
