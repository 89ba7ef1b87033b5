"""Python driver of libgeode_cuda.so's backend (include/geode_cuda.h): adopts a geode-pack's tensors into a gcuda
handle and exposes verify / keep / accept / state. It mirrors what the C++ host (libgeode_host.so) does for the
engine; the tests and the benchmark use it to reach the backend from Python. No CPU fallback: every call goes to
the CUDA library, and a missing library or device raises.
"""
from __future__ import annotations

import ctypes as C
import json
import os
from typing import Optional

import numpy as np

from . import cuda_lib


class GShape(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "n_layers", "vocab")] + [("eps", C.c_float)] + \
               [(n, C.c_int) for n in ("n_heads", "n_kv_heads", "head_dim", "rope_dim")] + [("rope_theta", C.c_float)] + \
               [(n, C.c_int) for n in ("gdn_k_heads", "gdn_v_heads", "gdn_k_dim", "gdn_v_dim", "conv_kernel",
                                       "n_experts", "top_k", "moe_ff", "shared_ff", "dense", "context", "max_tokens")]


class GLayer(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("attn", "in_norm", "post_norm", "qkv", "z", "out", "a", "b", "A_log", "dt_bias",
                                       "conv", "gnorm", "q", "k", "v", "o", "q_norm", "k_norm", "sh_gate", "sh_up",
                                       "sh_down", "router", "shared_gate", "experts")]


class GSampling(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int), ("presence_penalty", C.c_float)]


def _sig(L):
    vp, i32, i64, f32, sz = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t
    sigs = {
        "gcuda_open": (vp, [i32, C.c_char_p, i32]),
        "gcuda_close": (None, [vp]),
        "gcuda_last_error": (i32, [vp, C.c_char_p, i32]),
        "gcuda_adopt_q4": (i32, [vp, vp, i64, i64, sz, f32]),
        "gcuda_adopt_raw": (i32, [vp, vp, sz]),
        "gcuda_adopt_embedding": (i32, [vp, vp, i64, i64, f32]),
        "gcuda_adopt_experts": (i32, [vp, vp, i32, sz, vp]),
        "gcuda_setup": (i32, [vp, vp, vp, i32, i32, i32]),
        "gcuda_verify": (i32, [vp, vp, i32, vp, vp]),
        "gcuda_verify_device": (i32, [vp, vp, i32]),
        "gcuda_keep": (i32, [vp, i32]),
        "gcuda_position": (i32, [vp]),
        "gcuda_reset": (i32, [vp]),
        # g, sampling, uniforms, stops, n_stops, seen, n_seen, kept, next, samples
        "gcuda_accept": (i32, [vp, vp, vp, vp, i32, vp, i32, vp, vp, vp]),
        "gcuda_spec_reject": (i32, [vp, vp, vp, vp, i32, i32, i32, vp, C.c_uint64, vp, vp]),
        "gcuda_state_get": (i32, [vp, vp, vp, vp, vp, i32]),
        "gcuda_state_put": (i32, [vp, vp, vp, vp, vp, i32]),
        "gcuda_device_logits": (vp, [vp]),
        "gcuda_last_ms": (f32, [vp]),
        "gcuda_launches": (C.c_uint64, [vp]),
        "gcuda_debug_read": (i32, [vp, i32, vp, sz]),
        "gcuda_debug_step_eager": (i32, [vp, vp, i32, i32]),
        "gcuda_debug_trace": (i32, [vp, vp, i32, vp, vp, vp, vp, vp, vp]),
        "gcuda_debug_expf_table": (i32, [C.c_uint32, i64, vp, vp]),
        "gcuda_synth_q4": (i32, [vp, i64, i64, f32, C.c_uint64]),
        "gcuda_ep_unique_id": (i32, [vp]),
        "gcuda_set_ep": (i32, [vp, i32, i32, vp]),
        "gcuda_synth_raw": (i32, [vp, sz, i32, f32, f32, C.c_uint64]),
        "gcuda_synth_embedding": (i32, [vp, i64, i64, f32, C.c_uint64]),
        "gcuda_synth_experts": (i32, [vp, i32, i32, i32, f32, C.c_uint64]),
        "gcuda_state_randomize": (i32, [vp, i32, C.c_uint64]),
        "gcuda_step_device": (i32, [vp, i32]),
        "gcuda_step_device_reject": (i32, [vp, i32, vp, vp, C.c_uint64]),
        "gcuda_begin_device_loop": (i32, [vp, vp, i32]),
        "gcuda_sync_step": (i32, [vp, vp, vp, vp]),
        "gcuda_stream": (vp, [vp]),
        "gcuda_set_mtp": (i32, [vp, i32, i32, i32, i32, vp]),
        "gcuda_set_draft_head": (i32, [vp, i32, vp, i32]),
        "gcuda_draft_rows": (i32, [vp]),
        "gcuda_draft": (i32, [vp, vp, i32, i32, vp, vp, vp, vp]),
        "gcuda_draft_next": (i32, [vp, i32, i32, vp, vp, vp]),
    }
    for name, (res, args) in sigs.items():
        if hasattr(L, name):
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def draft_vocab(pack_dir: str, vocab: int):
    """The pack's draft vocabulary (draft_vocab.bin: int32 token ids) as the engine's GPU branch takes it
    (engine/src/model.cpp:2135-2161): the ids inside the vocabulary in file order, padded to whole tiles of 32 rows
    with copies of the first; None without the file or a valid id."""
    path = os.path.join(pack_dir, "draft_vocab.bin")
    if not os.path.exists(path):
        return None
    ids = np.fromfile(path, dtype="<i4")
    ids = ids[(ids >= 0) & (ids < vocab)]
    if ids.size == 0:
        return None
    pad = (-ids.size) % 32
    return np.ascontiguousarray(np.concatenate([ids, np.full(pad, ids[0])]).astype(np.int32))


class GcudaError(RuntimeError):
    pass


class Backend:
    """One gcuda handle over a geode-pack directory (or, with pack_dir None, a synthetic model: see synthetic())."""

    def __init__(self, pack_dir: Optional[str], context: int, max_tokens: int = 5, device: int = 0,
                 ep: Optional[tuple] = None):
        """ep: (rank, world, id) - this handle's rank in an expert-parallel group (gcuda_set_ep; id from ep_unique_id()
        on one rank, the same bytes on every rank)."""
        self.L = L = cuda_lib()
        _sig(L)
        err = C.create_string_buffer(512)
        self.g = L.gcuda_open(device, err, 512)
        if not self.g:
            raise GcudaError("gcuda_open: " + err.value.decode())
        if ep is not None:
            rank, world, uid = ep
            buf = C.create_string_buffer(bytes(uid), len(uid))
            if L.gcuda_set_ep(self.g, rank, world, buf) != 0:
                msg = self.error()
                L.gcuda_close(self.g)
                self.g = None
                raise GcudaError("set_ep: " + msg)
        if pack_dir is None:
            return
        with open(os.path.join(pack_dir, "geode.json")) as f:
            m = json.load(f)
        self.manifest = m
        files = {fi["name"]: np.memmap(os.path.join(pack_dir, fi["name"]), dtype=np.uint8, mode="r") for fi in m["files"]}
        c = m["config"]
        dense = m["arch"] == "qwen35"
        T = m["tensors"]

        def check(rc, what):
            if rc < 0:
                raise GcudaError(f"{what}: {self.error()}")
            return rc

        def tensor_bytes(name):
            t = T[name]
            buf = files[t["file"]]
            n = int(np.prod(t["shape"]))
            if t["type"] == "f32":
                size = 4 * n
            elif t["type"] == "bf16":
                size = 2 * n
            else:
                size = t["shape"][0] * int(np.prod(t["shape"][1:])) // 16 * 9
            return np.ascontiguousarray(buf[t["offset"]: t["offset"] + size]), t

        def q4(name):
            b, t = tensor_bytes(name)
            rows, cols = t["shape"][0], int(np.prod(t["shape"][1:]))
            return check(L.gcuda_adopt_q4(self.g, _ptr(b), rows, cols, cols // 16 * 9, t.get("global", 1.0)), name)

        def raw(name):
            b, _ = tensor_bytes(name)
            return check(L.gcuda_adopt_raw(self.g, _ptr(b), b.nbytes), name)

        attn = [t == "full_attention" for t in c["layer_types"]]

        def layer(x, p, is_attn, experts):
            """one decoder layer's tensors under prefix p (layers.{l}. or mtp.layers.0.)"""
            for f_ in GLayer._fields_:
                setattr(x, f_[0], -1)
            x.attn = 1 if is_attn else 0
            x.in_norm, x.post_norm = raw(p + "input_layernorm.weight"), raw(p + "post_attention_layernorm.weight")
            if is_attn:
                x.q, x.k, x.v, x.o = (q4(p + f"self_attn.{n}_proj.weight") for n in "qkvo")
                x.q_norm, x.k_norm = raw(p + "self_attn.q_norm.weight"), raw(p + "self_attn.k_norm.weight")
            else:
                x.qkv = q4(p + "linear_attn.in_proj_qkv.weight")
                x.z = q4(p + "linear_attn.in_proj_z.weight")
                x.out = q4(p + "linear_attn.out_proj.weight")
                x.a, x.b = raw(p + "linear_attn.in_proj_a.weight"), raw(p + "linear_attn.in_proj_b.weight")
                x.A_log, x.dt_bias = raw(p + "linear_attn.A_log"), raw(p + "linear_attn.dt_bias")
                x.conv, x.gnorm = raw(p + "linear_attn.conv1d.weight"), raw(p + "linear_attn.norm.weight")
            if dense:
                x.sh_gate, x.sh_up, x.sh_down = (q4(p + f"mlp.{n}_proj.weight") for n in ("gate", "up", "down"))
            else:
                x.sh_gate, x.sh_up, x.sh_down = (q4(p + f"mlp.shared_expert.{n}_proj.weight") for n in ("gate", "up", "down"))
                x.router, x.shared_gate = raw(p + "mlp.gate.weight"), raw(p + "mlp.shared_expert_gate.weight")
                buf = files[experts["file"]]
                E = c["num_experts"]
                blocks = np.ascontiguousarray(buf[experts["offset"]: experts["offset"] + E * experts["stride"]])
                sc, _ = tensor_bytes(p + "mlp.experts.scales")
                x.experts = check(L.gcuda_adopt_experts(self.g, _ptr(blocks), E, experts["stride"], _ptr(sc)),
                                  p + "experts")

        layers = (GLayer * c["num_hidden_layers"])()
        for l in range(c["num_hidden_layers"]):
            layer(layers[l], f"layers.{l}.", attn[l], None if dense else m["experts"]["layers"][l])
        self.has_mtp = "mtp" in m
        if self.has_mtp:
            # the MTP drafting layer (engine/src/model.cpp:175-191): fc, its norms, one attention decoder layer
            mt = GLayer()
            layer(mt, "mtp.layers.0.", True, None if dense else m["mtp"]["experts"])
            check(L.gcuda_set_mtp(self.g, q4("mtp.fc.weight"), raw("mtp.pre_fc_norm_embedding.weight"),
                                  raw("mtp.pre_fc_norm_hidden.weight"), raw("mtp.norm.weight"), C.addressof(mt)),
                  "set_mtp")
            ids = draft_vocab(pack_dir, c["vocab_size"])
            if ids is not None:
                hb, ht = tensor_bytes("lm_head.weight")
                rb = ht["shape"][1] // 16 * 9
                rows = np.ascontiguousarray(hb.reshape(-1, rb)[ids])
                dh = check(L.gcuda_adopt_q4(self.g, _ptr(rows), len(ids), ht["shape"][1], rb, ht.get("global", 1.0)),
                           "draft head")
                check(L.gcuda_set_draft_head(self.g, dh, _ptr(ids), len(ids)), "set_draft_head")
        eb, et = tensor_bytes("embed_tokens.weight")
        embed = check(L.gcuda_adopt_embedding(self.g, _ptr(eb), et["shape"][0], et["shape"][1], et.get("global", 1.0)), "embed")
        head = q4("lm_head.weight")
        norm = raw("norm.weight")
        rope = c.get("rope_parameters", {})
        s = GShape(hidden=c["hidden_size"], n_layers=c["num_hidden_layers"], vocab=c["vocab_size"],
                   eps=c.get("rms_norm_eps", 1e-6), n_heads=c["num_attention_heads"], n_kv_heads=c["num_key_value_heads"],
                   head_dim=c["head_dim"], rope_dim=int(c["head_dim"] * rope.get("partial_rotary_factor", 1.0)),
                   rope_theta=rope.get("rope_theta", 10000.0), gdn_k_heads=c.get("linear_num_key_heads", 0),
                   gdn_v_heads=c.get("linear_num_value_heads", 0), gdn_k_dim=c.get("linear_key_head_dim", 0),
                   gdn_v_dim=c.get("linear_value_head_dim", 0), conv_kernel=c.get("linear_conv_kernel_dim", 0),
                   n_experts=c.get("num_experts", 0), top_k=c.get("num_experts_per_tok", 0),
                   moe_ff=c.get("moe_intermediate_size", 0),
                   shared_ff=c["intermediate_size"] if dense else c["shared_expert_intermediate_size"],
                   dense=1 if dense else 0, context=context, max_tokens=max_tokens)
        self.shape = s
        check(L.gcuda_setup(self.g, C.addressof(s), C.addressof(layers), embed, head, norm), "setup")
        self.vocab, self.hidden = s.vocab, s.hidden
        self.n_attn = sum(attn)
        self.n_gdn = s.n_layers - self.n_attn

    def error(self) -> str:
        buf = C.create_string_buffer(1024)
        self.L.gcuda_last_error(self.g, buf, 1024)
        return buf.value.decode()

    def _rc(self, rc, what):
        if rc != 0:
            raise GcudaError(f"{what} ({rc}): {self.error()}")

    def close(self):
        if getattr(self, "g", None):
            self.L.gcuda_close(self.g)
            self.g = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def pos(self) -> int:
        return self.L.gcuda_position(self.g)

    def verify(self, toks, logits: bool = True, hidden: bool = False):
        toks = np.ascontiguousarray(np.asarray(toks, dtype=np.int32))
        n = len(toks)
        lg = np.zeros((n, self.vocab), np.float32) if logits else None
        hd = np.zeros((n, self.hidden), np.float32) if hidden else None
        self._rc(self.L.gcuda_verify(self.g, _ptr(toks), n, _ptr(lg) if lg is not None else None,
                                     _ptr(hd) if hd is not None else None), "verify")
        self._last_n = n
        return lg, hd

    def keep(self, kept: int):
        self._rc(self.L.gcuda_keep(self.g, kept), "keep")

    def draft(self, toks, pos: int, hidden=None, logits: bool = False):
        """gcuda_draft: the MTP pass over positions pos.. (toks: the next tokens; hidden: their rows, or None for the
        last verified batch's); (draft, prob, the last position's logits or None - over the draft head's rows when the
        pack has a draft vocabulary, see draft_vocab)."""
        toks = np.ascontiguousarray(np.asarray(toks, dtype=np.int32))
        hd = None if hidden is None else np.ascontiguousarray(hidden, dtype=np.float32)
        d, pr = C.c_int(0), C.c_float(0.0)
        lg = np.zeros(self.L.gcuda_draft_rows(self.g), np.float32) if logits else None
        self._rc(self.L.gcuda_draft(self.g, _ptr(toks), len(toks), pos, _ptr(hd) if hd is not None else None,
                                    C.byref(d), C.byref(pr), _ptr(lg) if lg is not None else None), "draft")
        return d.value, pr.value, lg

    def draft_next(self, tok: int, pos: int, logits: bool = False):
        """gcuda_draft_next: one chained MTP position; (draft, prob, logits or None)."""
        d, pr = C.c_int(0), C.c_float(0.0)
        lg = np.zeros(self.L.gcuda_draft_rows(self.g), np.float32) if logits else None
        self._rc(self.L.gcuda_draft_next(self.g, int(tok), pos, C.byref(d), C.byref(pr),
                                         _ptr(lg) if lg is not None else None), "draft_next")
        return d.value, pr.value, lg

    def reset(self):
        self._rc(self.L.gcuda_reset(self.g), "reset")

    def state_put(self, conv, gdn, kv, kvs, pos: int):
        self._rc(self.L.gcuda_state_put(self.g, _ptr(conv), _ptr(gdn), _ptr(kv), _ptr(kvs), pos), "state_put")

    def state_get(self, conv, gdn, kv, kvs, positions: int):
        self._rc(self.L.gcuda_state_get(self.g, _ptr(conv), _ptr(gdn), _ptr(kv), _ptr(kvs), positions), "state_get")

    def accept(self, temperature=0.0, top_p=1.0, top_k=0, uniforms=None, stops=(), presence_penalty=0.0, seen=()):
        """The acceptance of the last verified batch (its own tokens are the drafts): (kept, next, samples). With a
        presence penalty, seen lists the answer's sampled tokens so far (distinct); the device logits are penalised in
        place."""
        n = self._last_n
        u = np.ascontiguousarray(np.zeros(n) if uniforms is None else np.asarray(uniforms, dtype=np.float64))
        st = np.ascontiguousarray(np.asarray(list(stops) or [0], dtype=np.int32))
        sn = np.ascontiguousarray(np.asarray(list(seen) or [0], dtype=np.int32))
        kept, nxt = C.c_int(0), C.c_int(0)
        samples = np.zeros(n, np.int32)
        sp = GSampling(temperature, top_p, top_k, presence_penalty)
        self._rc(self.L.gcuda_accept(self.g, C.addressof(sp), _ptr(u), _ptr(st), len(stops), _ptr(sn), len(seen),
                                     C.byref(kept), C.byref(nxt), _ptr(samples)), "accept")
        return kept.value, nxt.value, samples

    def trace(self, toks):
        """One step with the per-layer trace (gcuda_debug_trace): x [L+1][n][H]; for MoE models router_logits
        [L][n][E+1], ids / weights [L][n][K], gate [L][n], n_union [L]. The logits stay on the device."""
        toks = np.ascontiguousarray(np.asarray(toks, dtype=np.int32))
        sh = self.shape
        n, L_, H = len(toks), sh.n_layers, sh.hidden
        out = {"x": np.zeros((L_ + 1, n, H), np.float32)}
        moe = sh.n_experts > 0 and not sh.dense
        if moe:
            E, K = sh.n_experts, sh.top_k
            out.update(router_logits=np.zeros((L_, n, E + 1), np.float32), ids=np.zeros((L_, n, K), np.int32),
                       weights=np.zeros((L_, n, K), np.float32), gate=np.zeros((L_, n), np.float32),
                       n_union=np.zeros(L_, np.int32))
        p = (lambda k: _ptr(out[k]) if moe else None)
        self._rc(self.L.gcuda_debug_trace(self.g, _ptr(toks), n, _ptr(out["x"]), p("router_logits"), p("ids"),
                                          p("weights"), p("gate"), p("n_union")), "debug_trace")
        self._last_n = n
        return out

    def randomize_state(self, pos: int, seed: int = 1):
        self._rc(self.L.gcuda_state_randomize(self.g, pos, C.c_uint64(seed)), "state_randomize")

    def begin_device_loop(self, toks):
        toks = np.ascontiguousarray(np.asarray(toks, dtype=np.int32))
        self._rc(self.L.gcuda_begin_device_loop(self.g, _ptr(toks), len(toks)), "begin_device_loop")

    def step_device(self, n: int):
        self._rc(self.L.gcuda_step_device(self.g, n), "step_device")

    def step_device_reject(self, n: int, d_draft: int, temperature: float, top_p: float = 1.0, top_k: int = 0,
                           seed: int = 1234):
        """gcuda_step_device with rejection sampling against the draft rows at d_draft ([n-1][vocab] f32, device)."""
        sp = GSampling(temperature, top_p, top_k)
        self._rc(self.L.gcuda_step_device_reject(self.g, n, C.c_void_p(d_draft), C.byref(sp), C.c_uint64(seed)),
                 "step_device_reject")

    def sync_step(self):
        steps, usum, kept = C.c_int(0), C.c_int(0), C.c_int(0)
        self._rc(self.L.gcuda_sync_step(self.g, C.byref(steps), C.byref(usum), C.byref(kept)), "sync_step")
        return steps.value, usum.value, kept.value

    def stream(self) -> int:
        return int(self.L.gcuda_stream(self.g) or 0)

    def last_ms(self) -> float:
        return self.L.gcuda_last_ms(self.g)

    def launches(self) -> int:
        return int(self.L.gcuda_launches(self.g))


def ep_unique_id() -> bytes:
    """NCCL's 128-byte id for a new expert-parallel group (made on one rank, handed to all)."""
    L = cuda_lib()
    _sig(L)
    buf = C.create_string_buffer(128)
    if L.gcuda_ep_unique_id(buf) != 0:
        raise GcudaError("ep_unique_id: NCCL unavailable")
    return buf.raw


def synthetic(shape, context: int, max_tokens: int = 5, device: int = 0, seed: int = 0,
              ep: Optional[tuple] = None) -> Backend:
    """A backend over a model of `shape` (geode_b200.synth.ModelShape) whose q4 weights are random bytes made on the
    device (gcuda_synth_*: random codes, E4M3 scales 0x30..0x48) - the same bytes a pack of that shape streams, for
    measuring at full size without writing ~20 GB of pack first."""
    be = Backend(None, context, max_tokens, device, ep=ep)
    L, g = be.L, be.g
    k = [seed]

    def nxt():
        k[0] += 1
        return C.c_uint64(k[0] * 0x9E3779B9 + 17)

    def chk(rc, what):
        if rc < 0:
            raise GcudaError(f"{what}: {be.error()}")
        return rc

    s = shape
    H = s.hidden
    q4 = lambda rows, cols: chk(L.gcuda_synth_q4(g, rows, cols, 0.02 / 14.7, nxt()), "synth_q4")
    f32 = lambda count, mean, std: chk(L.gcuda_synth_raw(g, count, 0, mean, std, nxt()), "synth_raw")
    bf16 = lambda count, std: chk(L.gcuda_synth_raw(g, count, 1, 0.0, std, nxt()), "synth_raw")
    layers = (GLayer * s.n_layers)()
    for l in range(s.n_layers):
        x = layers[l]
        for f_ in GLayer._fields_:
            setattr(x, f_[0], -1)
        attn = s.layer_types[l] == "full_attention"
        x.attn = 1 if attn else 0
        x.in_norm, x.post_norm = f32(H, 0.0, 0.1), f32(H, 0.0, 0.1)
        if attn:
            x.q, x.k = q4(s.n_heads * s.head_dim * 2, H), q4(s.n_kv_heads * s.head_dim, H)
            x.v, x.o = q4(s.n_kv_heads * s.head_dim, H), q4(H, s.n_heads * s.head_dim)
            x.q_norm, x.k_norm = f32(s.head_dim, 0.0, 0.1), f32(s.head_dim, 0.0, 0.1)
        else:
            vd = s.gdn_v_heads * s.gdn_v_dim
            x.qkv, x.z, x.out = q4(s.conv_dim, H), q4(vd, H), q4(H, vd)
            x.a, x.b = bf16(s.gdn_v_heads * H, 0.05), bf16(s.gdn_v_heads * H, 0.05)
            x.A_log, x.dt_bias = f32(s.gdn_v_heads, 1.4, 0.5), f32(s.gdn_v_heads, 0.0, 0.1)
            x.conv, x.gnorm = f32(s.conv_dim * s.conv_kernel, 0.0, 0.3), f32(s.gdn_v_dim, 1.0, 0.1)
        if s.dense:
            x.sh_gate, x.sh_up, x.sh_down = q4(s.shared_ff, H), q4(s.shared_ff, H), q4(H, s.shared_ff)
        else:
            x.sh_gate, x.sh_up, x.sh_down = q4(s.shared_ff, H), q4(s.shared_ff, H), q4(H, s.shared_ff)
            x.router, x.shared_gate = bf16(s.n_experts * H, 0.05), bf16(H, 0.05)
            x.experts = chk(L.gcuda_synth_experts(g, s.n_experts, H, s.moe_ff, 0.02 / 14.7, nxt()), "synth_experts")
    embed = chk(L.gcuda_synth_embedding(g, s.vocab, H, 1.0 / 14.7, nxt()), "synth_embedding")
    head = q4(s.vocab, H)
    norm = f32(H, 0.0, 0.1)
    gs = GShape(hidden=H, n_layers=s.n_layers, vocab=s.vocab, eps=s.eps, n_heads=s.n_heads, n_kv_heads=s.n_kv_heads,
                head_dim=s.head_dim, rope_dim=s.rope_dim, rope_theta=s.rope_theta, gdn_k_heads=s.gdn_k_heads,
                gdn_v_heads=s.gdn_v_heads, gdn_k_dim=s.gdn_k_dim, gdn_v_dim=s.gdn_v_dim, conv_kernel=s.conv_kernel,
                n_experts=s.n_experts, top_k=s.top_k, moe_ff=s.moe_ff, shared_ff=s.shared_ff, dense=1 if s.dense else 0,
                context=context, max_tokens=max_tokens)
    be.shape = gs
    chk(L.gcuda_setup(g, C.addressof(gs), C.addressof(layers), embed, head, norm), "setup")
    be.vocab, be.hidden = gs.vocab, gs.hidden
    be.n_attn = s.n_attn
    be.n_gdn = s.n_gdn
    return be
