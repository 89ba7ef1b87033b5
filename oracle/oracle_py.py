"""TEST INFRASTRUCTURE: Python bindings (ctypes) for the two CPU checkers under oracle/.

- ``Oracle``: the C restatement (oracle/liboracle.so, built from geode_oracle.c) over a geode-pack.
- ``Reference``: the reference engine's own code (oracle/_ref/libgeode_ref.so, compiled from the reference sources
  by oracle/Makefile), present only where it was built.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module, and only to check or to
time the CPU path beside the CUDA one.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libgeode_ref.so")


def build_oracle() -> str:
    """Compiles liboracle.so (gcc, seconds) when it is missing or older than its source."""
    src = os.path.join(HERE, "geode_oracle.c")
    if not os.path.exists(ORACLE_SO) or os.path.getmtime(ORACLE_SO) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", HERE, "oracle"])
    return ORACLE_SO


def have_reference() -> bool:
    return os.path.exists(REF_SO)


class GoQ4(C.Structure):
    _fields_ = [("data", C.c_void_p), ("rows", C.c_int64), ("cols", C.c_int64), ("global_", C.c_float)]


class GoConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "n_layers", "vocab")] + [("eps", C.c_float)] + \
               [(n, C.c_int) for n in ("n_heads", "n_kv_heads", "head_dim", "rope_dim")] + [("rope_theta", C.c_float)] + \
               [(n, C.c_int) for n in ("gdn_k_heads", "gdn_v_heads", "gdn_k_dim", "gdn_v_dim", "conv_kernel",
                                       "n_experts", "top_k", "moe_ff", "shared_ff", "dense", "attn_block")]


class GoLayer(C.Structure):
    _fields_ = [("attn", C.c_int), ("in_norm", C.c_void_p), ("post_norm", C.c_void_p),
                ("qkv", GoQ4), ("z", GoQ4), ("out", GoQ4), ("a", C.c_void_p), ("b", C.c_void_p),
                ("A_log", C.c_void_p), ("dt_bias", C.c_void_p), ("conv", C.c_void_p), ("gnorm", C.c_void_p),
                ("q", GoQ4), ("k", GoQ4), ("v", GoQ4), ("o", GoQ4), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p),
                ("sh_gate", GoQ4), ("sh_up", GoQ4), ("sh_down", GoQ4), ("router", C.c_void_p),
                ("shared_gate", C.c_void_p), ("experts", C.c_void_p), ("expert_stride", C.c_uint64),
                ("expert_scales", C.c_void_p)]


class GoModel(C.Structure):
    _fields_ = [("cfg", GoConfig), ("layers", C.c_void_p), ("embed", GoQ4), ("lm_head", GoQ4), ("final_norm", C.c_void_p)]


class GoState(C.Structure):
    _fields_ = [("pos", C.c_int), ("ctx", C.c_int), ("conv", C.c_void_p), ("gdn", C.c_void_p), ("kv", C.c_void_p),
                ("kvs", C.c_void_p)]


class GoMtp(C.Structure):
    _fields_ = [("layer", GoLayer), ("fc", GoQ4), ("norm", C.c_void_p), ("pre_e", C.c_void_p), ("pre_h", C.c_void_p)]


class GoTrace(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("x", "mixer", "moe", "out", "ids", "weights", "gate")]


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class Pack:
    """A geode-pack read into memory (numpy arrays over dense.bin and the expert file)."""

    def __init__(self, pack_dir: str):
        self.dir = pack_dir
        with open(os.path.join(pack_dir, "geode.json")) as f:
            self.manifest = json.load(f)
        self.files = {f["name"]: np.fromfile(os.path.join(pack_dir, f["name"]), dtype=np.uint8)
                      for f in self.manifest["files"]}
        c = self.manifest["config"]
        self.arch = self.manifest["arch"]
        self.cfg = c
        self.hidden = c["hidden_size"]
        self.n_layers = c["num_hidden_layers"]
        self.vocab = c["vocab_size"]
        self.attn = [t == "full_attention" for t in c["layer_types"]]

    def tensor(self, name: str):
        t = self.manifest["tensors"][name]
        return t, self.files[t["file"]]

    def raw(self, name: str) -> np.ndarray:
        t, buf = self.tensor(name)
        n = int(np.prod(t["shape"]))
        off = t["offset"]
        if t["type"] == "f32":
            return buf[off: off + 4 * n].view(np.float32)
        if t["type"] == "bf16":
            return buf[off: off + 2 * n].view(np.uint16)
        rows, cols = t["shape"][0], int(np.prod(t["shape"][1:]))
        return buf[off: off + rows * cols // 16 * 9].reshape(rows, cols // 16 * 9)

    def q4(self, name: str):
        t, _ = self.tensor(name)
        return self.raw(name), t["shape"][0], int(np.prod(t["shape"][1:])), float(t.get("global", 1.0))


class OracleState:
    def __init__(self, ora: "Oracle", ctx: int):
        c = ora.model.cfg
        nk, nv, dk, dv, K = c.gdn_k_heads, c.gdn_v_heads, c.gdn_k_dim, c.gdn_v_dim, c.conv_kernel
        conv_dim = 2 * nk * dk + nv * dv
        n_gdn, n_attn = ora.n_gdn, ora.n_attn
        kv_row = c.n_kv_heads * c.head_dim
        self.ctx = ctx
        self.pos = 0
        self.conv = np.zeros(max(1, n_gdn * conv_dim * max(K - 1, 0)), np.float32)
        self.gdn = np.zeros(max(1, n_gdn * nv * dk * dv), np.float32)
        self.kv = np.zeros(max(1, n_attn * 2 * ctx * kv_row), np.int8)
        self.kvs = np.zeros(max(1, n_attn * 2 * ctx * c.n_kv_heads), np.float32)
        # the MTP layer's own KV slot (after the main attention layers' in the engine's cache)
        self.mtp_kv = np.zeros(2 * ctx * kv_row if ora.has_mtp else 1, np.int8)
        self.mtp_kvs = np.zeros(2 * ctx * c.n_kv_heads if ora.has_mtp else 1, np.float32)

    def copy(self) -> "OracleState":
        s = object.__new__(OracleState)
        s.ctx, s.pos = self.ctx, self.pos
        s.conv, s.gdn, s.kv, s.kvs = self.conv.copy(), self.gdn.copy(), self.kv.copy(), self.kvs.copy()
        s.mtp_kv, s.mtp_kvs = self.mtp_kv.copy(), self.mtp_kvs.copy()
        return s

    def struct(self) -> GoState:
        return GoState(self.pos, self.ctx, _ptr(self.conv), _ptr(self.gdn), _ptr(self.kv), _ptr(self.kvs))


class Oracle:
    """The C restatement of the verify pass over one pack."""

    def __init__(self, pack_dir: str, attn_block: int = 1024):
        self.lib = C.CDLL(build_oracle())
        self.pack = p = Pack(pack_dir)
        c = p.cfg
        self.n_attn = sum(p.attn)
        self.n_gdn = p.n_layers - self.n_attn
        rope = c.get("rope_parameters", {})
        cfg = GoConfig(hidden=p.hidden, n_layers=p.n_layers, vocab=p.vocab, eps=c.get("rms_norm_eps", 1e-6),
                       n_heads=c["num_attention_heads"], n_kv_heads=c["num_key_value_heads"], head_dim=c["head_dim"],
                       rope_dim=int(c["head_dim"] * rope.get("partial_rotary_factor", 1.0)),
                       rope_theta=rope.get("rope_theta", 10000.0), gdn_k_heads=c.get("linear_num_key_heads", 0),
                       gdn_v_heads=c.get("linear_num_value_heads", 0), gdn_k_dim=c.get("linear_key_head_dim", 0),
                       gdn_v_dim=c.get("linear_value_head_dim", 0), conv_kernel=c.get("linear_conv_kernel_dim", 0),
                       n_experts=c.get("num_experts", 0), top_k=c.get("num_experts_per_tok", 0),
                       moe_ff=c.get("moe_intermediate_size", 0),
                       shared_ff=c["intermediate_size"] if p.arch == "qwen35" else c["shared_expert_intermediate_size"],
                       dense=1 if p.arch == "qwen35" else 0, attn_block=attn_block)
        self.cfg = cfg
        L = (GoLayer * p.n_layers)()
        keep = []

        def q4(name):
            raw, rows, cols, g = p.q4(name)
            keep.append(raw)
            return GoQ4(_ptr(raw), rows, cols, g)

        def arr(name):
            a = p.raw(name)
            keep.append(a)
            return _ptr(a)

        ex = self.pack.manifest["experts"]["layers"]

        def fill(x, pre, attn, e):
            x.attn = 1 if attn else 0
            x.in_norm, x.post_norm = arr(pre + "input_layernorm.weight"), arr(pre + "post_attention_layernorm.weight")
            if attn:
                x.q, x.k, x.v, x.o = (q4(pre + "self_attn." + n + "_proj.weight") for n in "qkvo")
                x.q_norm, x.k_norm = arr(pre + "self_attn.q_norm.weight"), arr(pre + "self_attn.k_norm.weight")
            else:
                x.qkv = q4(pre + "linear_attn.in_proj_qkv.weight")
                x.z = q4(pre + "linear_attn.in_proj_z.weight")
                x.out = q4(pre + "linear_attn.out_proj.weight")
                x.a, x.b = arr(pre + "linear_attn.in_proj_a.weight"), arr(pre + "linear_attn.in_proj_b.weight")
                x.A_log, x.dt_bias = arr(pre + "linear_attn.A_log"), arr(pre + "linear_attn.dt_bias")
                x.conv, x.gnorm = arr(pre + "linear_attn.conv1d.weight"), arr(pre + "linear_attn.norm.weight")
            if p.arch == "qwen35":
                x.sh_gate, x.sh_up, x.sh_down = (q4(pre + f"mlp.{n}_proj.weight") for n in ("gate", "up", "down"))
            else:
                x.sh_gate, x.sh_up, x.sh_down = (q4(pre + f"mlp.shared_expert.{n}_proj.weight")
                                                 for n in ("gate", "up", "down"))
                x.router, x.shared_gate = arr(pre + "mlp.gate.weight"), arr(pre + "mlp.shared_expert_gate.weight")
                buf = p.files[e["file"]]
                x.experts = _ptr(buf) + e["offset"]
                x.expert_stride = e["stride"]
                x.expert_scales = arr(pre + "mlp.experts.scales")

        for l in range(p.n_layers):
            fill(L[l], f"layers.{l}.", p.attn[l], ex[l] if l < len(ex) else None)
        # the MTP drafting layer, when the pack has one (engine/src/model.cpp:175-191, engine/src/pack.cpp:300-305)
        self.has_mtp = "mtp" in p.manifest
        self.mtp = None
        if self.has_mtp:
            self.mtp = GoMtp()
            fill(self.mtp.layer, "mtp.layers.0.", True, p.manifest["mtp"].get("experts"))
            self.mtp.fc = q4("mtp.fc.weight")
            self.mtp.norm, self.mtp.pre_e = arr("mtp.norm.weight"), arr("mtp.pre_fc_norm_embedding.weight")
            self.mtp.pre_h = arr("mtp.pre_fc_norm_hidden.weight")
            self.lib.go_forward_mtp.restype = C.c_int
            self.lib.go_forward_mtp.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                                C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        self._keep = keep
        self._layers = L
        self.model = GoModel(cfg, C.addressof(L), q4("embed_tokens.weight"), q4("lm_head.weight"), arr("norm.weight"))
        self.lib.go_forward.restype = C.c_int
        self.lib.go_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]

    def new_state(self, ctx: int) -> OracleState:
        return OracleState(self, ctx)

    def forward_mtp(self, state: OracleState, next_toks, hidden, pos: int, logits: bool = True):
        """go_forward_mtp over the state's MTP KV slot (state.mtp_kv / mtp_kvs): position i from pos takes hidden[i]
        and the embedding of next_toks[i]; the last position's logits and its output after mtp.norm (or None)."""
        if not self.has_mtp:
            raise RuntimeError("the pack has no MTP layer")
        next_toks = np.ascontiguousarray(np.asarray(next_toks, dtype=np.int32))
        hidden = np.ascontiguousarray(hidden, dtype=np.float32)
        n = len(next_toks)
        lg = np.zeros(self.pack.vocab, np.float32) if logits else None
        mh = np.zeros(self.pack.hidden, np.float32) if logits else None
        rc = self.lib.go_forward_mtp(C.addressof(self.model), C.addressof(self.mtp), _ptr(state.mtp_kv),
                                     _ptr(state.mtp_kvs), state.ctx, _ptr(next_toks), _ptr(hidden), n, pos,
                                     _ptr(lg) if logits else None, _ptr(mh) if logits else None)
        if rc != 0:
            raise RuntimeError("oracle forward_mtp failed")
        return lg, mh

    def forward(self, state: OracleState, toks, logits: bool = True, hidden: bool = False, trace: bool = False):
        toks = np.ascontiguousarray(np.asarray(toks, dtype=np.int32))
        n = len(toks)
        V, H = self.pack.vocab, self.pack.hidden
        lg = np.zeros((n, V), np.float32) if logits else None
        hd = np.zeros((n, H), np.float32) if hidden else None
        st = state.struct()
        tr = None
        trd = None
        if trace:
            K = max(1, self.cfg.top_k)
            Ls = self.pack.n_layers
            trd = {k: np.zeros((Ls, n, H), np.float32) for k in ("x", "mixer", "moe", "out")}
            trd["ids"] = np.full((Ls, n, K), -1, np.int32)
            trd["weights"] = np.zeros((Ls, n, K), np.float32)
            trd["gate"] = np.zeros((Ls, n), np.float32)
            tr = GoTrace(*[_ptr(trd[k]) for k in ("x", "mixer", "moe", "out", "ids", "weights", "gate")])
        rc = self.lib.go_forward(C.addressof(self.model), C.addressof(st), _ptr(toks), n,
                                 _ptr(lg) if lg is not None else None, _ptr(hd) if hd is not None else None,
                                 C.addressof(tr) if tr is not None else None)
        if rc != 0:
            raise RuntimeError("oracle forward failed")
        state.pos = st.pos
        out = {"logits": lg, "hidden": hd}
        if trace:
            out["trace"] = trd
        return out


# ------------------------------------------------------------------------------------------ kernel wrappers ----
def oracle_lib():
    lib = C.CDLL(build_oracle())
    lib.go_e4m3_value.restype = C.c_float
    lib.go_e4m3_value.argtypes = [C.c_uint8]
    lib.go_fast_exp.restype = C.c_float
    lib.go_fast_exp.argtypes = [C.c_float]
    lib.go_canonical.restype = C.c_double
    lib.go_mt64_next.restype = C.c_uint64
    lib.go_sample.restype = C.c_int
    lib.go_sample.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_float, C.c_int, C.c_double]
    lib.go_accept.restype = C.c_int
    lib.go_accept.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_float, C.c_float, C.c_int, C.c_uint64,
                              C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
    lib.go_accept_seen.restype = C.c_int
    lib.go_accept_seen.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_float, C.c_float, C.c_int,
                                   C.c_uint64, C.c_void_p, C.c_int, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.c_void_p]
    lib.go_expf_restated.restype = C.c_float
    lib.go_expf_restated.argtypes = [C.c_float]
    lib.go_expf_mismatch.restype = C.c_uint64
    lib.go_expf_mismatch.argtypes = [C.c_uint64, C.c_uint64, C.c_int, C.c_int, C.c_void_p, C.c_int]
    lib.go_expf_check_table.restype = C.c_uint64
    lib.go_expf_check_table.argtypes = [C.c_uint64, C.c_uint64, C.c_void_p, C.c_int, C.c_void_p, C.c_int]
    lib.go_expert_pair.argtypes = [C.c_void_p, C.c_float, C.c_float, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    lib.go_spec_reject.restype = C.c_int
    lib.go_spec_reject.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_float, C.c_float,
                                   C.c_int, C.c_uint64, C.c_uint64, C.c_void_p]
    lib.go_quantize_q4.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_float, C.c_void_p, C.c_int]
    lib.go_q4_block.argtypes = [C.c_void_p, C.c_float, C.c_void_p, C.c_void_p]
    lib.go_quantize_activation.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p]
    lib.go_matvec_q.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64]
    lib.go_matvec_bf16.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_void_p, C.c_void_p]
    lib.go_rmsnorm.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_int]
    lib.go_route_topk.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    lib.go_dequant_row.argtypes = [C.c_void_p, C.c_int64, C.c_void_p]
    return lib


def oracle_quantize_activation(lib, x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32)
    cols = x.shape[-1]
    q = np.zeros(cols, np.int8)
    s = np.zeros(cols // 16, np.float32)
    b = np.zeros(cols // 16, np.int32)
    lib.go_quantize_activation(_ptr(x), cols, _ptr(q), _ptr(s), _ptr(b))
    return q, s, b


def oracle_matvec_q(lib, packed: np.ndarray, rows: int, cols: int, glob: float, xs: np.ndarray) -> np.ndarray:
    """y [n][rows] of the int8 path: each token's activation quantized, then the rows in order."""
    packed = np.ascontiguousarray(packed)
    w = GoQ4(_ptr(packed), rows, cols, glob)
    xs = np.atleast_2d(np.ascontiguousarray(xs, np.float32))
    ys = np.zeros((xs.shape[0], rows), np.float32)
    for t in range(xs.shape[0]):
        q, s, _ = oracle_quantize_activation(lib, xs[t])
        y = np.zeros(rows, np.float32)
        lib.go_matvec_q(C.addressof(w), _ptr(q), _ptr(s), _ptr(y), 0, rows)
        ys[t] = y
    return ys


class GoMt64(C.Structure):
    _fields_ = [("mt", C.c_uint64 * 312), ("mti", C.c_int)]


def oracle_uniforms(lib, seed: int, n: int) -> np.ndarray:
    """The first n draws the reference's Sampler makes from mt19937_64(seed): generate_canonical<double, 53>."""
    g = GoMt64()
    lib.go_mt64_seed(C.byref(g), C.c_uint64(seed))
    lib.go_canonical.argtypes = [C.c_void_p]
    return np.array([lib.go_canonical(C.byref(g)) for _ in range(n)], dtype=np.float64)


def oracle_route_topk(lib, logits: np.ndarray, K: int):
    logits = np.ascontiguousarray(logits, np.float32)
    E = logits.shape[-1]
    ids = np.zeros(K, np.int32)
    w = np.zeros(K, np.float32)
    lib.go_route_topk(_ptr(logits), E, K, _ptr(ids), _ptr(w))
    return ids, w


# ------------------------------------------------------------------------------------------ the reference ----
class Reference:
    """The reference engine's geode::Model over a pack (oracle/_ref/libgeode_ref.so)."""

    def __init__(self, pack_dir: str, threads: int = 1, ctx: int = 8192, attn_block: Optional[int] = None,
                 draft: bool = False):
        if not have_reference():
            raise RuntimeError("the reference build oracle/_ref/libgeode_ref.so is missing")
        if attn_block is not None:
            os.environ["GEODE_ATTN_BLOCK"] = str(attn_block)
        self.lib = lib = C.CDLL(REF_SO)
        lib.ref_open2.restype = C.c_void_p
        lib.ref_open2.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_char_p, C.c_int]
        lib.ref_hidden.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        lib.ref_mtp.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                C.c_char_p, C.c_int]
        lib.ref_close.argtypes = [C.c_void_p]
        lib.ref_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_char_p, C.c_int]
        lib.ref_position.argtypes = [C.c_void_p]
        lib.ref_save_state.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_int]
        lib.ref_load_state.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_int]
        lib.ref_trace.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int]
        lib.ref_trace_get.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        err = C.create_string_buffer(512)
        self.h = lib.ref_open2(pack_dir.encode(), threads, ctx, 1 if draft else 0, err, 512)
        if attn_block is not None:
            del os.environ["GEODE_ATTN_BLOCK"]
        if not self.h:
            raise RuntimeError("reference open failed: " + err.value.decode())
        with open(os.path.join(pack_dir, "geode.json")) as f:
            m = json.load(f)
        self.vocab = m["config"]["vocab_size"]
        self.hidden = m["config"]["hidden_size"]
        self.n_layers = m["config"]["num_hidden_layers"]
        self.top_k = m["config"].get("num_experts_per_tok", 0)

    def close(self):
        if self.h:
            self.lib.ref_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def pos(self) -> int:
        return self.lib.ref_position(self.h)

    def forward(self, toks, all_logits: bool = True, trace: bool = False):
        toks = np.ascontiguousarray(np.asarray(toks, dtype=np.int32))
        n = len(toks)
        lg = np.zeros((n if all_logits else 1, self.vocab), np.float32)
        if trace:
            self.lib.ref_trace(self.h, 1, self.n_layers, n)
        err = C.create_string_buffer(512)
        rc = self.lib.ref_forward(self.h, _ptr(toks), n, _ptr(lg), 1 if all_logits else 0, err, 512)
        out = {"logits": lg}
        if trace:
            K = max(1, self.top_k)
            tr = {}
            for i, k in enumerate(("x", "mixer", "moe", "out")):
                a = np.zeros((self.n_layers, n, self.hidden), np.float32)
                self.lib.ref_trace_get(self.h, i, _ptr(a))
                tr[k] = a
            tr["ids"] = np.zeros((self.n_layers, n, K), np.int32)
            self.lib.ref_trace_get(self.h, 4, _ptr(tr["ids"]))
            tr["weights"] = np.zeros((self.n_layers, n, K), np.float32)
            self.lib.ref_trace_get(self.h, 5, _ptr(tr["weights"]))
            tr["gate"] = np.zeros((self.n_layers, n), np.float32)
            self.lib.ref_trace_get(self.h, 6, _ptr(tr["gate"]))
            self.lib.ref_trace(self.h, 0, 0, 0)
            out["trace"] = tr
        if rc != 0:
            raise RuntimeError("reference forward failed: " + err.value.decode())
        return out

    def profile(self) -> str:
        buf = C.create_string_buffer(8192)
        self.lib.ref_profile.argtypes = [C.c_void_p, C.c_char_p, C.c_int]
        self.lib.ref_profile(self.h, buf, 8192)
        return buf.value.decode()

    def hidden_rows(self, n: int) -> np.ndarray:
        """Model::hidden(t) for the last forward_batch's first n tokens (after the final norm; MTP packs only)."""
        out = np.zeros((n, self.hidden), np.float32)
        for t in range(n):
            if self.lib.ref_hidden(self.h, t, out[t].ctypes.data) != 0:
                raise RuntimeError("the reference keeps no hidden rows (no MTP layer bound)")
        return out

    def mtp(self, next_toks, hidden, pos: int, logits: bool = True):
        """Model::forward_mtp: position i from pos takes hidden[i] and the embedding of next_toks[i]; the last
        position's logits and its normed output (Model::mtp_hidden), or (None, None)."""
        next_toks = np.ascontiguousarray(np.asarray(next_toks, dtype=np.int32))
        hidden = np.ascontiguousarray(hidden, dtype=np.float32)
        n = len(next_toks)
        lg = np.zeros(self.vocab, np.float32) if logits else None
        mh = np.zeros(self.hidden, np.float32) if logits else None
        err = C.create_string_buffer(512)
        if self.lib.ref_mtp(self.h, next_toks.ctypes.data, hidden.ctypes.data, n, pos,
                            lg.ctypes.data if logits else None, mh.ctypes.data if logits else None, err, 512) != 0:
            raise RuntimeError("reference forward_mtp: " + err.value.decode())
        return lg, mh

    def save_state(self, path: str):
        err = C.create_string_buffer(512)
        if self.lib.ref_save_state(self.h, path.encode(), err, 512) != 0:
            raise RuntimeError(err.value.decode())

    def load_state(self, path: str):
        err = C.create_string_buffer(512)
        if self.lib.ref_load_state(self.h, path.encode(), err, 512) != 0:
            raise RuntimeError(err.value.decode())


def reference_lib():
    lib = C.CDLL(REF_SO)
    lib.ref_quantize_activation.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p]
    lib.ref_matvec_q.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_float, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    lib.ref_dequant_row.argtypes = [C.c_void_p, C.c_int64, C.c_float, C.c_int, C.c_void_p]
    lib.ref_matvec_bf16_multi.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_void_p, C.c_void_p]
    lib.ref_rmsnorm.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_int]
    lib.ref_fast_exp.restype = C.c_float
    lib.ref_fast_exp.argtypes = [C.c_float]
    lib.ref_route_topk.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    lib.ref_q4_block.argtypes = [C.c_void_p, C.c_float, C.c_void_p, C.c_void_p]
    lib.ref_e4m3_value.restype = C.c_float
    lib.ref_e4m3_value.argtypes = [C.c_uint8]
    lib.ref_accept.restype = C.c_int
    lib.ref_accept.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_float, C.c_float, C.c_int, C.c_uint64,
                               C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
    lib.ref_accept_seen.restype = C.c_int
    lib.ref_accept_seen.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_float, C.c_float, C.c_int,
                                    C.c_uint64, C.c_void_p, C.c_int, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p]
    lib.ref_uniforms.argtypes = [C.c_uint64, C.c_int, C.c_void_p]
    return lib


# ------------------------------------------------------------------------------------------ state files ----
# The reference's conversation file (engine/src/state.cpp:5-17, 45-65, 192-207): a 4096-byte header (StateHeader, an
# FNV-1a checksum of its bytes last), the fixed part (gen, images, last hidden, conv states, GDN states, gen), then the
# KV cache in blocks of 256 positions: [K, V][attention layer][256][kv_row] int8, then [K, V][layer][256][kv_heads] f32.
_HDR = np.dtype([("magic", "S8"), ("version", "<u4"), ("header_size", "<u4"), ("fingerprint", "<u8"), ("conv_id", "<u8"),
                 ("gen", "<u8"), ("position", "<i4"), ("extra", "<i4"), ("rope_delta", "<i4"), ("n_images", "<u4"),
                 ("image_cap", "<u4"), ("kv_elem", "<u4"), ("n_attn", "<u4"), ("kv_heads", "<u4"), ("kv_row", "<u4"),
                 ("hidden", "<u4"), ("has_hidden", "<u4"), ("block", "<u4"), ("conv_n", "<u8"), ("gdn_n", "<u8"),
                 ("fixed_offset", "<u8"), ("fixed_bytes", "<u8"), ("kv_offset", "<u8"), ("block_bytes", "<u8"),
                 ("checksum", "<u8")])


def _fnv(data: bytes, h: int = 1469598103934665603) -> int:
    for b in data:
        h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def write_long_state(template: str, out: str, position: int, seed: int = 0):
    """A state file at `position` with random int8 KV rows (scales |N(0, 0.5)| / 127), from a template the reference
    saved for the same model (its header and fixed part kept; the position, the KV blocks and the checksum new)."""
    with open(template, "rb") as f:
        data = bytearray(f.read())
    h = np.frombuffer(bytes(data[:_HDR.itemsize]), dtype=_HDR)[0].copy()
    assert h["magic"] == b"GEODESTA" and h["kv_elem"] == 1, "an int8-KV state of the reference"
    h["position"] = position
    raw = bytearray(h.tobytes())
    raw[136:144] = _fnv(bytes(raw[:136])).to_bytes(8, "little")
    rng = np.random.default_rng(seed)
    B, n_attn, row, heads = int(h["block"]), int(h["n_attn"]), int(h["kv_row"]), int(h["kv_heads"])
    blocks = (position + B - 1) // B
    with open(out, "wb") as f:
        f.write(raw)
        f.write(bytes(data[len(raw): int(h["kv_offset"])]))
        for b in range(blocks):
            kv = rng.integers(-127, 128, 2 * n_attn * B * row, dtype=np.int8)
            sc = (np.abs(rng.standard_normal(2 * n_attn * B * heads)) * 0.5 / 127 + 1e-4).astype(np.float32)
            f.write(kv.tobytes())
            f.write(sc.tobytes())


def accept_seen(lib, rows, batch, temperature, top_p, top_k, seed, penalty, seen, stops=(), fn="go_accept_seen"):
    """The acceptance with the presence penalty through lib.<fn> (go_accept_seen of the oracle, ref_accept_seen of the
    reference build): (kept, next, samples, the seen list after it)."""
    rows = np.ascontiguousarray(rows, dtype=np.float32)
    n, V = rows.shape
    batch = np.ascontiguousarray(batch, dtype=np.int32)
    buf = np.zeros(len(seen) + n + 1, np.int32)
    buf[:len(seen)] = np.asarray(seen, dtype=np.int32)
    ns = C.c_int(len(seen))
    st = np.ascontiguousarray(np.asarray(list(stops) or [0], dtype=np.int32))
    nxt = C.c_int(0)
    samples = np.zeros(n, np.int32)
    kept = getattr(lib, fn)(rows.ctypes.data, n, V, batch.ctypes.data, temperature, top_p, top_k, C.c_uint64(seed),
                            st.ctypes.data, len(stops), penalty, buf.ctypes.data, C.byref(ns), C.byref(nxt),
                            samples.ctypes.data)
    return kept, nxt.value, samples, buf[:ns.value].copy()


def plant_penalized_drafts(rows, batch, seen, penalty, stand):
    """Sets batch[1..stand] to the greedy samples of rows 0..stand-1 under the presence penalty (each row's logits
    less the penalty at the tokens of seen and at the drafts planted before it, once each - the f32 subtraction the
    engine makes), so that those drafts stand under the penalty. Returns batch."""
    pen = np.float32(penalty)
    known = set(int(t) for t in seen)
    for i in range(stand):
        r = np.array(rows[i], dtype=np.float32, copy=True)
        idx = np.array(sorted(known), dtype=np.int64)
        if idx.size:
            r[idx] = r[idx] - pen
        y = int(np.argmax(r))
        batch[i + 1] = y
        known.add(y)
    return batch
