#!/usr/bin/env python
"""Benchmark of the speculative-decoding verify step at the Qwen3.6-35B-A3B shape (BASELINE cfg 3): 40 layers in the
3:1 Gated DeltaNet : gated attention pattern, hidden 2048, 256 routed experts top-8 + a shared expert (ff 512), vocab
248320, q4 weights (the engine's E4M3-scaled 16-value blocks), 1 accepted token + 4 drafts verified per step against
a context of 8192 positions.

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]

A step = the verify forward of 5 tokens (every row's logits), the greedy acceptance of the rows and the rollback of
the Gated DeltaNet states to the last accepted token, chained on the device (gcuda_step_device). `value`: verified
tokens/s of the whole job with the weights resident in HBM; `e2e`: the same through the C ABI with host buffers
(gcuda_verify: tokens in, every logit out to pinned host memory; gcuda_accept; gcuda_keep). Weights are random q4
bytes made on the device (the weights' values do not change the bytes streamed); the 8192-position KV cache and the
recurrent states are random. `--impl reference` times the reference engine's own CPU path (oracle/_ref, compiled
from the reference sources) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "verify tok/s at 35B-A3B shape, 4 drafts, 1/2/4/8 B200; % of HBM roofline"
UNIT = "verified tokens/s"
CTX = 8192
NTOK = 5


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def step_bytes(shape, union_per_layer: float, ctx: float, n: int = NTOK) -> dict:
    """Algorithmic bytes of one verify step: every weight byte the step must read once (q4 at 9/16 byte per value,
    the routed experts actually picked), the KV rows attended and written, the recurrent and conv states read and
    written, the logits written. Rollback copies are excluded (implementation overhead)."""
    s = shape
    H = s.hidden
    q4 = lambda r, c: r * c * 9 // 16
    kd, vd = s.gdn_k_heads * s.gdn_k_dim, s.gdn_v_heads * s.gdn_v_dim
    conv_dim = 2 * kd + vd
    kv_pos = 2 * (s.n_kv_heads * s.head_dim + 4 * s.n_kv_heads)
    expert = q4(2 * s.moe_ff, H) + q4(H, s.moe_ff)
    b = {"dense": 0, "experts": 0, "kv": 0, "state": 0, "logits": 0}
    for t in s.layer_types:
        b["dense"] += 2 * H * 4
        if t == "full_attention":
            b["dense"] += q4(2 * s.n_heads * s.head_dim, H) + 2 * q4(s.n_kv_heads * s.head_dim, H) + \
                q4(H, s.n_heads * s.head_dim) + 2 * s.head_dim * 4
            b["kv"] += int(ctx * kv_pos) + n * kv_pos
        else:
            b["dense"] += q4(conv_dim, H) + 2 * q4(vd, H) + 2 * s.gdn_v_heads * H * 2 + conv_dim * s.conv_kernel * 4 + \
                s.gdn_v_dim * 4 + 2 * s.gdn_v_heads * 4
            b["state"] += 2 * s.gdn_v_heads * s.gdn_k_dim * s.gdn_v_dim * 4 + 2 * conv_dim * (s.conv_kernel - 1) * 4
        if s.dense:
            b["dense"] += 2 * q4(s.shared_ff, H) + q4(H, s.shared_ff)
        else:
            b["dense"] += (s.n_experts + 1) * H * 2 + 2 * q4(s.shared_ff, H) + q4(H, s.shared_ff)
            b["experts"] += int(round(union_per_layer * expert))
    b["dense"] += q4(s.vocab, H) + H * 4 + n * (H // 16) * 9
    b["logits"] = n * s.vocab * 4
    b["total"] = sum(v for k, v in b.items())
    return b


class Clocks:
    """nvidia-smi sampled every 200 ms while running: median SM clock, max clock, the throttle reasons seen."""

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        q = "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
            "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, mx, reasons = [], 0.0, set()
        for r in self.rows:
            try:
                sm.append(float(r[0]))
                mx = max(mx, float(r[1]))
                for i, nm in enumerate(names):
                    if r[4 + i].lower().startswith("active"):
                        reasons.add(nm)
            except Exception:
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------- the CPU path ----
def cpu_reference(steps: int = 5, warmup: int = 1, distinct: int = 4, threads: int = 0) -> dict:
    """The reference engine's own CPU verify path (oracle/_ref: Model::forward_batch with every row's logits, then the
    acceptance rule around geode::Sampler) on the cfg-3 workload at its full depth: the same shapes (hidden 2048,
    40 layers, 256 experts top-8, vocab 248320, the 8192-position int8 KV cache). The pack holds `distinct` layers'
    bytes (3 GDN : 1 attention) that the 40 layers name in turn (synth.write_pack's distinct_layers), so every layer
    reads as many bytes as a distinct one (the 2.4 GB pack is far larger than the host's caches) while the pack is
    written in seconds. `warmup` untimed steps (they read the routed experts in), then the median of `steps`."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_py as op  # (the baseline leg only: the reference's code timed on the host)
    from geode_b200 import synth

    kind = "reference" if op.have_reference() else "port"
    shape = synth.baseline_shape(3)
    threads = threads or os.cpu_count() or 1
    with tempfile.TemporaryDirectory() as d:
        synth.write_pack(d, shape, seed=1, fill="random", distinct_layers=distinct)
        if kind != "reference":
            return {"kind": "port", "value": None, "unit": UNIT, "cores": 1,
                    "sample": "the reference build is missing: no CPU number"}
        ref = op.Reference(d, threads=threads, ctx=CTX + 64)
        ref.forward([1, 2, 3])
        ref.save_state(os.path.join(d, "t.state"))
        op.write_long_state(os.path.join(d, "t.state"), os.path.join(d, "l.state"), CTX)
        lib = op.reference_lib()
        rng = np.random.default_rng(3)
        times = []
        import ctypes as C

        for it in range(warmup + steps):
            ref.load_state(os.path.join(d, "l.state"))
            toks = rng.integers(0, shape.vocab, NTOK).astype(np.int32)
            t0 = time.perf_counter()
            out = ref.forward(toks, all_logits=True)
            nxt = C.c_int(0)
            samples = np.zeros(NTOK, np.int32)
            lib.ref_accept(out["logits"].ctypes.data, NTOK, shape.vocab, toks.ctypes.data, 0.0, 1.0, 0, C.c_uint64(1),
                           None, 0, C.byref(nxt), samples.ctypes.data)
            t1 = time.perf_counter()
            if it >= warmup:
                times.append(t1 - t0)
        ref.close()
    t = statistics.median(times)
    return {"kind": kind, "value": NTOK / t, "unit": UNIT, "cores": threads, "steps": steps, "warmup": warmup,
            "layers": shape.n_layers,
            "sample": f"all 40 layers (3 GDN : 1 attention; {distinct} layers' bytes named in turn) + lm_head, ctx {CTX}, "
                      f"5 rows, greedy acceptance; median of {steps} steps after {warmup} warm-up = {t * 1e3:.0f} ms/step "
                      f"(state reloaded before each step)"}


ACCEPT_METRIC = "acceptance rows/s (cfg5: 256 sequences x (8+1) rows, vocab 248320)"
ACCEPT_UNIT = "verified rows/s (greedy)"


def cpu_accept_reference(seqs: int = 24, seed: int = 5) -> dict:
    """The acceptance microbench's CPU side on a bounded sample (`seqs` of its 256 sequences, the same shapes: 8+1
    target rows and 8 draft rows of N(0, 3) logits over vocab 248320, drafts = the draft rows' argmax): greedy with the
    reference engine's own rule (oracle/_ref: geode_generate's acceptance around geode::Sampler at temperature 0, one
    sequence after another on one thread), and rejection sampling (T 0.7, top-k 20, top-p 0.95, Philox 1234) with
    the oracle's port - the reference has none. value = the greedy rate in the GPU line's unit: the 9 rows of a
    sequence per sequence (the rule reads only up to the first failed draft, as the GPU call's rows are counted)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ctypes as C
    import oracle_py as op  # (the baseline leg only: the reference's code timed on the host)
    S, K, V = seqs, 8, 248320
    rng = np.random.default_rng(seed)
    target = (rng.standard_normal((S, K + 1, V), dtype=np.float32) * 3).astype(np.float32)
    draft = (rng.standard_normal((S, K, V), dtype=np.float32) * 3).astype(np.float32)
    drafts = np.ascontiguousarray(np.argmax(draft, axis=2).astype(np.int32))
    kind = "reference" if op.have_reference() else "port"
    lib = op.reference_lib() if kind == "reference" else op.oracle_lib()
    accept = lib.ref_accept if kind == "reference" else lib.go_accept
    samples = np.zeros(K + 1, np.int32)
    nxt = C.c_int(0)
    t0 = time.perf_counter()
    for s_ in range(S):
        batch = np.ascontiguousarray(np.concatenate([[0], drafts[s_]]).astype(np.int32))
        accept(np.ascontiguousarray(target[s_]).ctypes.data, K + 1, V, batch.ctypes.data, 0.0, 1.0, 0, C.c_uint64(0), None,
               0, C.byref(nxt), samples.ctypes.data)
    t_greedy = time.perf_counter() - t0
    O = op.oracle_lib()
    n_rej = max(1, S // 3)
    t0 = time.perf_counter()
    for s_ in range(n_rej):
        O.go_spec_reject(np.ascontiguousarray(target[s_]).ctypes.data, np.ascontiguousarray(draft[s_]).ctypes.data, K, V,
                         np.ascontiguousarray(drafts[s_]).ctypes.data, 0.7, 0.95, 20, C.c_uint64(1234), s_, C.byref(nxt))
    t_rej = time.perf_counter() - t0
    return {"kind": kind, "value": S * (K + 1) / t_greedy, "unit": ACCEPT_UNIT, "cores": 1,
            "sample": f"{S} of the 256 sequences (seeded N(0, 3) logits, drafts = the draft rows' argmax): greedy by the "
                      f"{'reference engine' if kind == 'reference' else 'oracle port'}'s rule {t_greedy * 1e3:.1f} ms; "
                      f"rejection sampling by the oracle port (no reference code) on {n_rej} sequences "
                      f"{t_rej * 1e3:.0f} ms",
            "rejection_port_sequences_per_s": n_rej / t_rej}


def max_over_ranks(value: float, dist, device) -> float:
    """The largest of every rank's value (every rank takes the same collective; a lone process returns its own)."""
    if dist is None:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    t0 = time.perf_counter()
    if args.workload == "cfg5":
        cb = cpu_accept_reference()
        v = cb["value"]
        print(json.dumps({"impl": "reference", "metric": ACCEPT_METRIC, "value": v, "unit": ACCEPT_UNIT,
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": 256 * 9 / v * 1e3, "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                          "config": {"workload": "cfg5: acceptance microbench, 256 x 8 drafts, V 248320, greedy"},
                          "cpu_baseline": cb,
                          "e2e": {"value": v, "unit": ACCEPT_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                          "wall_s": time.perf_counter() - t0}))
        return 0
    # (each step about a second on 16 cores: at most 5 timed steps after 1 warm-up, so the run stays within minutes)
    steps, warmup = max(1, min(args.steps, 5)), 1
    cb = cpu_reference(steps=steps, warmup=warmup)
    if cb.get("value") is None:
        print(json.dumps({"impl": "reference", "unavailable": cb["sample"]}))
        return 0
    v = cb["value"]
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
            "warmup": warmup, "ms_per_step": NTOK / v * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q4xint8->f32", "data": "synthetic",
            "config": {"workload": "cfg3: MoE 35B-A3B shape verify (40 layers, 256 experts top-8 + shared, vocab "
                                   "248320), 1 accepted + 4 drafts, ctx 8192, greedy acceptance", "global_batch": NTOK,
                       "seq_len": CTX, "parallelism": "cpu", "layers": 40,
                       "requested": {"steps": args.steps, "warmup": args.warmup}},
            "cpu_baseline": cb, "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": time.perf_counter() - t0}
    print(json.dumps(line))
    return 0


# ------------------------------------------------------------------------------------------- the GPU path ----
# dram__bytes_read.sum + dram__bytes_write.sum of one LM-head launch of k_gemv_static (one ncu capture, the command in
# profiles/k_gemv_static_lmhead_cfg3.md): 287.9 MB + 20.8 MB
LMHEAD_TRAFFIC = 307.97e6


def gemv_roofline(L, peak_gbs, reps: int = 20) -> dict:
    """The dominant kernel's roofline, measured live: the q4 GEMV (k_gemv_static, the kernel of every dense product and
    the LM head) on the LM head's shape, 248320 x 2048, 5 token rows; CUDA events on its stream."""
    import torch
    rows, cols, n = 248320, 2048, NTOK
    tb = L.gcuda_op_q4_tiled_bytes(rows, cols)
    pack = torch.randint(0, 256, (rows, cols // 16 * 9), dtype=torch.uint8, device="cuda")
    pack[:, cols // 2:] = torch.randint(0x30, 0x49, (rows, cols // 16), dtype=torch.uint8, device="cuda")
    tiles = torch.empty(tb, dtype=torch.uint8, device="cuda")
    L.gcuda_op_q4_relayout(pack.data_ptr(), rows, cols, tiles.data_ptr(), None)
    del pack
    x = torch.randn(n, cols, device="cuda")
    q = torch.empty(n, cols, dtype=torch.int8, device="cuda")
    sc = torch.empty(n, cols // 16, device="cuda")
    bs = torch.empty(n, cols // 16, dtype=torch.int32, device="cuda")
    y = torch.empty(n, rows, device="cuda")
    L.gcuda_op_quantize(x.data_ptr(), n, cols, q.data_ptr(), sc.data_ptr(), bs.data_ptr(), None)
    st = torch.cuda.current_stream()
    for _ in range(3):
        L.gcuda_op_q4_gemv(tiles.data_ptr(), rows, cols, 1e-3, q.data_ptr(), sc.data_ptr(), bs.data_ptr(), n, y.data_ptr(),
                           st.cuda_stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        L.gcuda_op_q4_gemv(tiles.data_ptr(), rows, cols, 1e-3, q.data_ptr(), sc.data_ptr(), bs.data_ptr(), n, y.data_ptr(),
                           st.cuda_stream)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    alg = rows * cols * 9 // 16 + n * cols + n * (cols // 16) * 8 + n * rows * 4
    ach = alg / (ms * 1e-3) / 1e9
    return {"kernel": "k_gemv_static (q4 GEMV, lm_head 248320x2048, 5 rows)", "bound": "hbm", "achieved": ach,
            "peak": peak_gbs, "unit": "GB/s", "frac": ach / peak_gbs, "traffic": LMHEAD_TRAFFIC, "ms": ms,
            "algorithmic_bytes": alg, "traffic_source": "ncu, profiles/k_gemv_static_lmhead_cfg3.md"}


KT_NAMES = ["gate_up", "down", "lm_head", "dense"]
# ncu figures of the dominant kernel, per launch (the capture's command and numbers: this file)
GATEUP_PROFILE = os.path.join(ROOT, "profiles", "k_experts_lane_gateup_cfg3.md")


def profiled_traffic(path: str, blocks: float):
    """dram bytes read + written of one launch, from a committed ncu summary's `traffic_per_launch_bytes:` and
    `expert_blocks_in_launch:` lines, scaled to a launch that reads `blocks` expert blocks (the traffic grows in
    proportion to the blocks read)."""
    got = {}
    try:
        with open(path) as f:
            for line in f:
                k, _, v = line.strip().partition(":")
                if k in ("traffic_per_launch_bytes", "expert_blocks_in_launch"):
                    got[k] = float(v.split()[0])
    except OSError:
        return None
    if len(got) != 2 or not blocks:
        return None
    return got["traffic_per_launch_bytes"] * blocks / got["expert_blocks_in_launch"]


def kernel_rooflines(be, shape, toks, peak_gbs, reps: int = 5) -> dict:
    """Per kind of launch inside the step (gcuda_debug_kernel_times: eager steps, no programmatic overlap, CUDA events
    around each launch): device ms per step, launches, algorithmic bytes per launch and GB/s. The expert products'
    algorithmic bytes: the q4 weights of the routed experts the layer's union names plus the shared expert's (9/16
    byte per value); the activations and outputs (< 0.2%) are left out."""
    import ctypes as C
    L = be.L
    L.gcuda_debug_kernel_times.restype = C.c_int
    L.gcuda_debug_kernel_times.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                           C.c_void_p, C.c_void_p]
    ms = np.zeros(4, np.float32)
    nl = np.zeros(4, np.int32)
    step_ms = C.c_float(0)
    usum = C.c_int(0)
    t = np.ascontiguousarray(toks, dtype=np.int32)
    be._rc(L.gcuda_debug_kernel_times(be.g, t.ctypes.data, len(t), reps, ms.ctypes.data, nl.ctypes.data,
                                      C.byref(step_ms), C.byref(usum)), "kernel_times")
    H, q4 = shape.hidden, (lambda r, c: r * c * 9 // 16)
    n_moe = 0 if shape.dense else shape.n_layers
    union = usum.value / max(1, n_moe)
    per = {
        "gate_up": (union * q4(2 * shape.moe_ff, H) + q4(2 * shape.shared_ff, H)) if n_moe else 0,
        "down": (union * q4(H, shape.moe_ff) + q4(H, shape.shared_ff)) if n_moe else 0,
        "lm_head": q4(shape.vocab, H),
        "dense": None,
    }
    out = {"timing": "eager steps, kernel by kernel (no programmatic overlap), CUDA events around each launch; "
                     f"mean of {reps} steps", "eager_step_ms": step_ms.value, "union_per_layer": union}
    for k, name in enumerate(KT_NAMES):
        d = {"ms_per_step": float(ms[k]), "launches_per_step": int(nl[k]),
             "share_of_eager_step": float(ms[k]) / step_ms.value if step_ms.value else None}
        if per[name] and nl[k]:
            ms_launch = float(ms[k]) / nl[k]
            ach = per[name] / (ms_launch * 1e-3) / 1e9
            d.update(ms_per_launch=ms_launch, algorithmic_bytes_per_launch=int(per[name]), achieved_gbs=ach,
                     frac=ach / peak_gbs)
        out[name] = d
    return out


def accept_bench(args) -> int:
    """The acceptance microbench (BASELINE cfg 5): 256 sequences x 8 drafts, vocab 248320, target and draft logits
    N(0, 3) fp32 resident on the device (4.3 GB, larger than L2), drafts = the draft rows' argmax. Times, with CUDA
    events on the launching stream, the greedy acceptance of all sequences in one call (gcuda_op_greedy_verify: every
    target row's first maximum, then the rule) and rejection sampling at temperature 0.7, top-k 20, top-p 0.95,
    Philox seed 1234 (gcuda_op_spec_reject_static, whose results reach the host inside the timed call)."""
    import ctypes as C
    import torch
    from geode_b200 import cuda_lib
    from geode_b200.backend import GSampling, _sig
    S, K, V = 256, 8, 248320
    L = cuda_lib()
    _sig(L)
    L.gcuda_op_spec_reject_static.restype = C.c_int
    L.gcuda_op_spec_reject_static.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                              C.c_uint64, C.c_void_p, C.c_void_p, C.c_void_p]
    peak, peak_kind = measured_peaks()
    gen = torch.Generator(device="cuda").manual_seed(5)
    target = torch.randn((S, K + 1, V), generator=gen, device="cuda") * 3
    draft = torch.randn((S, K, V), generator=gen, device="cuda") * 3
    drafts = draft.argmax(dim=2).to(torch.int32).contiguous()
    h_drafts = drafts.cpu().numpy()
    scratch = torch.empty(S * (K + 1), dtype=torch.int64, device="cuda")
    acc = torch.empty(S, dtype=torch.int32, device="cuda")
    nxt = torch.empty(S, dtype=torch.int32, device="cuda")
    h_acc, h_nxt = np.zeros(S, np.int32), np.zeros(S, np.int32)
    st = torch.cuda.current_stream()
    sp = GSampling(0.7, 0.95, 20)

    def greedy():
        assert L.gcuda_op_greedy_verify(target.data_ptr(), drafts.data_ptr(), S, K, V, scratch.data_ptr(), acc.data_ptr(),
                                        nxt.data_ptr(), st.cuda_stream) == 0

    def reject():
        assert L.gcuda_op_spec_reject_static(target.data_ptr(), draft.data_ptr(), h_drafts.ctypes.data, S, K, V,
                                             C.byref(sp), 1234, h_acc.ctypes.data, h_nxt.ctypes.data, st.cuda_stream) == 0

    def timed(fn, steps):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    steps = max(3, min(args.steps, 50))
    with Clocks(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        ms_g = timed(greedy, steps)
        ms_r = timed(reject, steps)
    a = h_acc.copy()
    rows = S * (K + 1)
    bytes_g = rows * V * 4 + S * K * 4 + S * 8
    # rejection sampling reads, per sequence, the target rows 0..accepted and the draft rows 0..min(accepted, K-1)
    rows_r = int(np.sum(np.minimum(a + 1, K + 1) + np.minimum(a + 1, K)))
    bytes_r = rows_r * V * 4
    ach = bytes_g / (ms_g * 1e-3) / 1e9
    line = {
        "metric": ACCEPT_METRIC, "value": rows / (ms_g * 1e-3), "unit": ACCEPT_UNIT, "n_gpus": 1, "steps": steps, "warmup": max(3, args.warmup),
        "ms_per_step": ms_g, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (logits N(0, 3) made on the device, seed 5; drafts = the draft rows' argmax)",
        "config": {"workload": "cfg5: acceptance microbench, 256 x 8 drafts, V 248320, T 0.7, top-k 20, top-p 0.95, "
                               "Philox(1234)", "l2": "inputs larger than L2 (4.3 GB of logits; no flush)"},
        "roofline": {"kernel": "k_argmax_rows (+ k_greedy_decide)", "bound": "hbm", "achieved": ach, "peak": peak,
                     "unit": "GB/s", "frac": ach / peak, "traffic": None, "algorithmic_bytes": bytes_g},
        "rejection": {"ms_per_call": ms_r, "sequences_per_s": S / (ms_r * 1e-3), "rows_read": rows_r,
                      "achieved_gbs": bytes_r / (ms_r * 1e-3) / 1e9, "mean_accepted": float(a.mean()),
                      "accepted_hist": np.bincount(a, minlength=K + 1).tolist()},
        "cpu_baseline": None if args.no_cpu_baseline else cpu_accept_reference(), "e2e": None,
        "clocks": clk.summary(), "peak_kind": peak_kind,
    }
    print(json.dumps(line))
    return 0


CFG4_METRIC = "MoE expert stage of the batched verify (cfg4: 64 sequences x 5 rows, 256 experts top-8, Zipf picks)"
CFG4_UNIT = "verified rows/s through the 40 layers' routed experts"


def zipf_picks(rng, n: int, E: int, K: int, s: float = 1.0) -> np.ndarray:
    """n rows of K distinct experts each, expert popularity Zipf(s) over a random ranking of the E experts (the
    router-logit bias BASELINE cfg 4 describes, drawn directly)."""
    rank = rng.permutation(E)
    p = 1.0 / (np.arange(1, E + 1, dtype=np.float64) ** s)
    p = p[np.argsort(rank)]
    p /= p.sum()
    return np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(n)]).astype(np.int32)


def cfg4_bench(args) -> int:
    """The batched configuration's routed experts on the tensor core (gcuda_op_moe_umma): 320 token rows (64
    sequences x 5), top-8 of 256 experts with Zipf(1.0) picks, hidden 2048, expert ff 512, 40 layers - each layer's
    picks grouped by expert on the device, the grouped gate_up, SwiGLU + quantize and the grouped down, exact per pick.
    A step = the 40 layers' expert stages one after another (the attention / Gated DeltaNet of 64 sequences and the
    combine are not built for this configuration). Weights: random U-layout bytes made on the device (18 GB, far
    above L2; no flush), activations random."""
    import ctypes as C
    import torch
    from geode_b200 import cuda_lib
    L = cuda_lib()
    peak, peak_kind = measured_peaks()
    n_seq, rows_per, E, K, H, ff = 64, NTOK, 256, 8, 2048, 512
    layers = max(1, min(args.layers, 40))   # (fewer only for profiling)
    n = n_seq * rows_per
    rng = np.random.default_rng(4)
    eb = L.gcuda_op_moe_umma_expert_bytes(H, ff)
    gu_code = 2 * ff * H // 2
    gu_bytes = 2 * ff * H * 9 // 16
    dn_code = H * ff // 2
    gen = torch.Generator(device="cuda").manual_seed(4)
    experts = []
    for _ in range(layers):   # random codes, scale bytes in 0x30..0x48 (sane E4M3 values)
        u = torch.randint(0, 256, (E, eb), dtype=torch.uint8, device="cuda", generator=gen)
        u[:, gu_code:gu_bytes] = torch.randint(0x30, 0x49, (E, gu_bytes - gu_code), dtype=torch.uint8, device="cuda", generator=gen)
        u[:, gu_bytes + dn_code:] = torch.randint(0x30, 0x49, (E, eb - gu_bytes - dn_code), dtype=torch.uint8, device="cuda", generator=gen)
        experts.append(u)
    globs = torch.full((E, 2), 1e-3, dtype=torch.float32, device="cuda")
    ids = [torch.from_numpy(zipf_picks(rng, n, E, K)).cuda() for _ in range(layers)]
    union = [int(torch.unique(i).numel()) for i in ids]
    x = torch.randn(n, H, device="cuda", generator=gen)
    q = torch.empty(n, H, dtype=torch.int8, device="cuda")
    sc = torch.empty(n, H // 16, device="cuda")
    bs = torch.empty(n, H // 16, dtype=torch.int32, device="cuda")
    L.gcuda_op_quantize(x.data_ptr(), n, H, q.data_ptr(), sc.data_ptr(), bs.data_ptr(), None)
    wb = L.gcuda_op_moe_umma_work_bytes(n, K, E, H, ff)
    work = torch.empty(wb, dtype=torch.uint8, device="cuda")
    out = torch.empty(n * K, H, device="cuda")
    st = torch.cuda.current_stream()

    def step():
        for l in range(layers):
            rc = L.gcuda_op_moe_umma(experts[l].data_ptr(), globs.data_ptr(), E, H, ff, q.data_ptr(), sc.data_ptr(),
                                     bs.data_ptr(), n, ids[l].data_ptr(), K, out.data_ptr(), work.data_ptr(), wb,
                                     st.cuda_stream)
            assert rc == 0, rc

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    assert L.gcuda_op_status(1) == 0
    steps = max(3, min(args.steps, 20))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        e0.record(st)
        for _ in range(steps):
            step()
        e1.record(st)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    wbytes = sum(union) * eb           # the routed experts' weights each step reads once
    ach = wbytes / (ms * 1e-3) / 1e9
    macs = n * K * (2 * ff * H + H * ff) * layers   # the picks' products (useful multiply-adds)
    cb = None
    if not args.no_cpu_baseline:
        cb = cpu_moe_port(layers)
    line = {
        "metric": CFG4_METRIC, "value": n * 1e3 / ms, "unit": CFG4_UNIT, "n_gpus": 1, "steps": steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q4xint8->f32 (tcgen05 kind::i8, exact per pick)",
        "data": "synthetic (random U-layout q4 bytes and activations made on the device; Zipf(1.0) picks)",
        "config": {"workload": "cfg4: routed-expert stage only (gcuda_op_moe_umma per layer), 320 rows, 40 layers",
                   "global_batch": n, "seq_len": None, "parallelism": "1 GPU",
                   "l2": "inputs larger than L2 (18 GB of expert weights; no flush)", "layers": layers},
        "roofline": {"kernel": "k_umma_gemm (grouped, tcgen05 int8 MMAs + exact float chain) with the plan and SwiGLU "
                               "kernels", "bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                     "frac": ach / peak, "traffic": None, "algorithmic_bytes_per_step": wbytes,
                     "experts_per_layer": sum(union) / layers},
        "tensor": {"useful_tops": 2 * macs / (ms * 1e-3) / 1e12, "note": "2 x the picks' multiply-adds / time; the MMAs "
                   "do twice that (each K = 32 step holds two blocks' zero-padded columns)"},
        "cpu_baseline": cb, "e2e": None, "gpu_launches": 4 * layers, "clocks": clk.summary(), "peak_kind": peak_kind,
    }
    print(json.dumps(line))
    return 0


def cpu_moe_port(layers: int, picks: int = 48) -> dict:
    """The CPU side of the cfg4 line: the oracle's port of the reference's per-pick expert product (go_expert_pair,
    engine/src/model.cpp:4496-4543; one thread) on a sample of `picks` picks, scaled to the step's 320 x 8 x 40."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_py as op
    from geode_b200 import synth
    O = op.oracle_lib()
    rng = np.random.default_rng(5)
    H, ff = 2048, 512
    gu, g0 = synth.q4_random(rng, 2 * ff, H)
    dn, g1 = synth.q4_random(rng, H, ff)
    blk = np.ascontiguousarray(np.concatenate([gu.reshape(-1), dn.reshape(-1)]))
    h = rng.standard_normal(H).astype(np.float32)
    y = np.zeros(H, np.float32)
    t0 = time.perf_counter()
    for _ in range(picks):
        O.go_expert_pair(blk.ctypes.data, g0, g1, H, ff, h.ctypes.data, y.ctypes.data)
    t = (time.perf_counter() - t0) / picks
    step = t * 320 * 8 * layers
    return {"kind": "port", "value": 320 / step, "unit": CFG4_UNIT, "cores": 1,
            "sample": f"{picks} picks of the oracle's port of the per-pick expert product, {t * 1e3:.2f} ms each, "
                      f"scaled to 320 rows x 8 picks x {layers} layers = {step:.1f} s a step"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=40)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=40, help="(smaller cases for profiling)")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: each GPU verifies its own sequence (replicas, weak scaling); without it (the default) "
                         "one sequence runs over all GPUs with the routed experts striped over them (expert "
                         "parallelism, gcuda_set_ep; strong scaling)")
    ap.add_argument("--workload", default="cfg3", choices=["cfg3", "cfg4", "cfg5"],
                    help="cfg3: the verify step (the headline); cfg4: the batched configuration's routed experts on the "
                         "tensor core (one GPU); cfg5: the acceptance microbench (one GPU)")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)
    if args.workload in ("cfg4", "cfg5"):
        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        return accept_bench(args) if args.workload == "cfg5" else cfg4_bench(args)

    import torch
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    from geode_b200 import synth
    from geode_b200.backend import synthetic, ep_unique_id
    from geode_b200 import cuda_lib
    ep = None
    if not args.replicas and world > 1:
        obj = [ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ep = (rank, world, obj[0])

    peak, peak_kind = measured_peaks()
    shape = synth.baseline_shape(3)
    if args.layers != 40:
        shape.n_layers = args.layers
        shape.layer_types = synth.hybrid_types(args.layers)
    context = CTX + args.warmup + args.steps + args.e2e_steps + 64
    t_build = time.perf_counter()
    # (expert parallel: every rank the same model, state and tokens - one sequence)
    seed = 0 if ep else rank
    be = synthetic(shape, context=context, max_tokens=NTOK, device=local, seed=seed, ep=ep)
    be.randomize_state(CTX, seed=7 + seed)
    t_build = time.perf_counter() - t_build
    rng = np.random.default_rng(seed)
    toks = rng.integers(0, shape.vocab, NTOK).astype(np.int32)
    launches0 = be.launches()

    # ---- value: the device-resident step, K steps back to back
    stream = torch.cuda.ExternalStream(be.stream())
    be.begin_device_loop(toks)
    for _ in range(args.warmup):
        be.step_device(NTOK)
    be.sync_step()
    be.begin_device_loop(toks)   # (counters from zero for the timed steps)
    pos0 = be.pos
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    lc0 = be.launches()
    with Clocks(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            be.step_device(NTOK)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    steps_done, union_sum, _ = be.sync_step()
    launches_timed = be.launches() - lc0
    ms = max_over_ranks(ms, dist, "cuda")
    ms_step = ms / args.steps
    n_moe = 0 if shape.dense else shape.n_layers
    union_layer = union_sum / max(1, steps_done * n_moe) if n_moe else 0.0
    mean_ctx = (pos0 + be.pos) / 2
    b = step_bytes(shape, union_layer, mean_ctx)
    seqs = 1 if ep else world   # sequences the job verifies at once
    value = seqs * NTOK * args.steps / (ms * 1e-3)

    # ---- e2e: the C ABI with host buffers, every step synchronous (tokens in, logits out, accept, keep)
    pinned = torch.empty((NTOK, shape.vocab), dtype=torch.float32, pin_memory=True).numpy()
    for i in range(3):
        be.verify(toks, logits=False)
        kept, nxt, _ = be.accept(0.0)
        if kept < NTOK:
            be.keep(kept)
    import ctypes as C
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.e2e_steps):
        be._rc(be.L.gcuda_verify(be.g, toks.ctypes.data, NTOK, pinned.ctypes.data, None), "verify")
        be._last_n = NTOK
        kept, nxt, _ = be.accept(0.0)
        if kept < NTOK:
            be.keep(kept)
        toks[0] = nxt
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    e2e_s = max_over_ranks(e2e_s, dist, "cuda")
    e2e = seqs * NTOK * args.e2e_steps / e2e_s

    lm_op = gemv_roofline(cuda_lib(), peak)
    kr = kernel_rooflines(be, shape, toks, peak)
    gu = kr["gate_up"]
    roof = {"kernel": "k_experts_lane gate_up (the union's routed experts + the shared expert, a lane a weight row, "
                      "SwiGLU + quantize epilogue): the step's largest kernel by device time", "bound": "hbm",
            "achieved": gu.get("achieved_gbs"), "peak": peak, "unit": "GB/s", "frac": gu.get("frac"),
            "traffic": profiled_traffic(GATEUP_PROFILE, kr["union_per_layer"] + 1), "ms": gu.get("ms_per_launch"),
            "algorithmic_bytes": gu.get("algorithmic_bytes_per_launch"), "launches_per_step": gu["launches_per_step"],
            "timing": kr["timing"], "traffic_source": "ncu, " + os.path.relpath(GATEUP_PROFILE, ROOT) +
            " (a 41-block launch, scaled to this run's mean union + the shared expert)"}
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cb = cpu_reference()
        except Exception as ex:   # (the baseline must not sink the GPU number)
            cb = {"kind": "reference", "value": None, "unit": UNIT, "cores": os.cpu_count(), "sample": f"failed: {ex}"}
    step_ach = b["total"] / (ms_step * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong" if ep else "weak", "vs_baseline": None,
        "dtype": "q4xint8->f32", "data": "synthetic (random q4 codes / E4M3 scales made on the device; random 8192-position KV)",
        "config": {"workload": "cfg3: MoE 35B-A3B shape verify (40 layers, 256 experts top-8 + shared, vocab 248320), "
                               "1 accepted + 4 drafts, ctx 8192, greedy acceptance + GDN rollback",
                   "global_batch": NTOK * seqs, "seq_len": CTX,
                   "parallelism": f"ep{world}" if ep else f"replicas x{world}" if world > 1 else "1 GPU",
                   "l2": "inputs larger than L2 (20 GB of weights per GPU; no flush)", "layers": shape.n_layers},
        "roofline": roof,
        "kernels": kr,
        "lm_head_operator": lm_op,
        "step_roofline": {"bound": "hbm", "achieved": step_ach, "peak": peak, "unit": "GB/s", "frac": step_ach / peak,
                          "peak_kind": peak_kind, "algorithmic_bytes_per_step": b, "experts_per_layer": union_layer,
                          "per_gpu": "bytes and experts of one GPU (under expert parallelism each reads its own experts "
                                     "and every dense weight)",
                          "mean_context": mean_ctx},
        "cpu_baseline": cb,
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": NTOK * 4,
                "d2h_bytes_per_step": NTOK * shape.vocab * 4 + NTOK * 4, "steps": args.e2e_steps},
        "gpu_launches": int(launches_timed),
        "clocks": clk.summary(),
        "build_s": t_build,
        "peak_kind": peak_kind,
    }
    if rank == 0:
        print(json.dumps(line))
    be.close()
    if dist:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
