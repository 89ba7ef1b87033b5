"""Synthetic geode-pack writer and the model shapes of the benchmark configurations.

The reference engine reads a "geode-pack" v1 directory (engine/src/pack.cpp:40-317): ``geode.json`` (the manifest:
files, model config, tensor table, expert table), ``dense.bin`` (every non-expert tensor) and an expert file (one
block per routed expert and layer: gate_up rows then down rows, engine/src/pack.cpp:333-337). The pack builder of
the reference (tools/geodepack.py) is not part of its public tree, so this module writes the format from the
reader's side, with the tensor names the reference binds (engine/src/model.cpp:94-203).

q4 matrices are quantized with the reference's block quantizer (engine/src/yue2_q4.cpp:72-114, restated in
``q4_quantize``; the tests pin it bit for bit against the reference's own ``q4_block``) and the per-matrix global
``max|w| * 1.25 / (15 * 448)`` (engine/src/yue2_q4.cpp:343). ``fill="random"`` instead draws q4 codes and E4M3
scale bytes directly (the self-test weights of engine/src/gpu_check.cpp:51-63): the same bytes per matrix, for
timing runs whose values do not matter.
"""
from __future__ import annotations

import dataclasses
import json
import os
from typing import Dict, List, Optional

import numpy as np

KBLOCK = 16


# ----------------------------------------------------------------------------------------------- model shapes ----
@dataclasses.dataclass
class ModelShape:
    name: str
    arch: str  # "qwen35moe" or "qwen35" (dense)
    hidden: int
    n_layers: int
    vocab: int
    layer_types: List[str]
    n_heads: int = 16
    n_kv_heads: int = 4
    head_dim: int = 256
    partial_rotary: float = 0.25
    rope_theta: float = 1.0e7
    gdn_k_heads: int = 16
    gdn_v_heads: int = 16
    gdn_k_dim: int = 128
    gdn_v_dim: int = 128
    conv_kernel: int = 4
    n_experts: int = 0
    top_k: int = 0
    moe_ff: int = 0
    shared_ff: int = 0  # the MoE's shared expert, or the dense model's MLP width
    eps: float = 1e-6
    ctx: int = 8192

    @property
    def dense(self) -> bool:
        return self.arch == "qwen35"

    @property
    def n_attn(self) -> int:
        return sum(1 for t in self.layer_types if t == "full_attention")

    @property
    def n_gdn(self) -> int:
        return self.n_layers - self.n_attn

    @property
    def conv_dim(self) -> int:
        return 2 * self.gdn_k_heads * self.gdn_k_dim + self.gdn_v_heads * self.gdn_v_dim

    @property
    def rope_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary)


def hybrid_types(n_layers: int) -> List[str]:
    """Qwen3.5/3.6's 3:1 pattern: three Gated DeltaNet layers, then one full-attention layer."""
    return ["full_attention" if (l % 4) == 3 else "linear_attention" for l in range(n_layers)]


def baseline_shape(cfg: int) -> ModelShape:
    """The model shapes of the five benchmark configurations (cfg 1..5; 4 and 5 reuse 3's model)."""
    if cfg == 1:
        return ModelShape("cfg1-single-layer", "qwen35", 2048, 1, 32768, ["full_attention"], head_dim=128,
                          shared_ff=6144, ctx=1024 + 8)
    if cfg == 2:
        return ModelShape("cfg2-dense-2b", "qwen35", 2048, 24, 248320, hybrid_types(24), shared_ff=6144, ctx=4096 + 8)
    if cfg in (3, 4, 5):
        return ModelShape("cfg3-moe-35b-a3b", "qwen35moe", 2048, 40, 248320, hybrid_types(40), n_experts=256,
                          top_k=8, moe_ff=512, shared_ff=512, ctx=8192 + 8)
    raise ValueError(cfg)


def tiny_shape(arch: str = "qwen35moe", n_layers: int = 4, hidden: int = 256, vocab: int = 1024,
               n_experts: int = 16, top_k: int = 4, ctx: int = 640) -> ModelShape:
    """A small model of the same structure for parity tests (every dimension a multiple of the kernels' tiles)."""
    return ModelShape(f"tiny-{arch}-{n_layers}", arch, hidden, n_layers, vocab, hybrid_types(n_layers), n_heads=4,
                      n_kv_heads=2, head_dim=64, gdn_k_heads=2, gdn_v_heads=4, gdn_k_dim=32, gdn_v_dim=32,
                      n_experts=0 if arch == "qwen35" else n_experts, top_k=0 if arch == "qwen35" else top_k,
                      moe_ff=0 if arch == "qwen35" else 128, shared_ff=384 if arch == "qwen35" else 128, ctx=ctx)


# ----------------------------------------------------------------------------------------------- q4 format ----
def e4m3_table() -> np.ndarray:
    """E4M3fn byte -> float32 (engine/src/kernels.cpp:39-52)."""
    b = np.arange(256)
    sign, ex, man = b >> 7, (b >> 3) & 15, b & 7
    v = np.where(ex == 0, np.ldexp(man / 8.0, -6), np.ldexp(1.0 + man / 8.0, ex - 7)).astype(np.float32)
    v[(ex == 15) & (man == 7)] = np.nan
    return np.where(sign == 1, -v, v).astype(np.float32)


E4M3 = e4m3_table()
Q4_LEVELS = np.array([1, 3, 5, 7, 9, 11, 13, 15, -1, -3, -5, -7, -9, -11, -13, -15], dtype=np.int8)


def e4m3_byte(x: np.ndarray) -> np.ndarray:
    """Non-negative floats onto E4M3 codes 0..126: the nearer neighbour, ties to the even code
    (engine/src/yue2_q4.cpp:72-86)."""
    pos = E4M3[:127]
    x = np.asarray(x, dtype=np.float32)
    hi = np.searchsorted(pos, x, side="right")  # first code with value > x
    hi = np.clip(hi, 1, 126)
    lo = hi - 1
    dl = (x - pos[lo]).astype(np.float32)
    dh = (pos[hi] - x).astype(np.float32)
    out = np.where(dl < dh, lo, np.where(dh < dl, hi, np.where(lo % 2 == 0, lo, hi)))
    out = np.where(x >= pos[126], 126, out)
    out = np.where(x > 0, out, 0)
    return out.astype(np.int64)


def q4_quantize(w: np.ndarray, s2: Optional[float] = None):
    """[rows, cols] float32 -> (pack bytes [rows, cols*9/16] uint8, global s2). Per 16-value block the reference's
    candidate search: codes mapping amax onto 15 and onto 13, two either side, the least squared error (the first
    of equals), values onto the nearest odd magnitude (exact ties to the even index) (engine/src/yue2_q4.cpp:88-114)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    assert cols % KBLOCK == 0
    if s2 is None:
        s2 = np.float32(np.float32(np.abs(w).max()) * np.float32(1.25) / np.float32(15.0 * 448.0))
    s2 = np.float32(s2)
    x = w.reshape(-1, KBLOCK)
    amax = np.abs(x).max(axis=1)
    cands = []
    for t in (np.float32(15.0), np.float32(13.0)):
        b0 = e4m3_byte((amax / np.float32(t * s2)).astype(np.float32))
        for k in range(-2, 3):
            cands.append(np.clip(b0 + k, 0, 0x7E))
    cand = np.stack(cands, axis=1)  # [nb, 10]
    scale = (E4M3[cand] * s2).astype(np.float32)
    safe = np.where(scale == 0, np.float32(1.0), scale).astype(np.float32)
    y = (x[:, None, :] / safe[:, :, None]).astype(np.float32)  # [nb, 10, 16]
    a = np.minimum(np.abs(y), np.float32(15.0))
    idx = np.clip(np.rint((a - np.float32(1.0)) * np.float32(0.5)), 0, 7).astype(np.int64)
    neg = y < 0
    lev = np.where(neg, -(2 * idx + 1), 2 * idx + 1).astype(np.float32)
    q = (lev * scale[:, :, None]).astype(np.float32)
    d = (q - x[:, None, :]).astype(np.float32)
    err = np.zeros(d.shape[:2], dtype=np.float32)
    for i in range(KBLOCK):  # sequential, as the reference sums
        err = (err + d[:, :, i] * d[:, :, i]).astype(np.float32)
    best = np.argmin(err, axis=1)  # first of equal minima
    nb = x.shape[0]
    sel = np.arange(nb)
    codes = (idx[sel, best] + np.where(neg[sel, best], 8, 0)).astype(np.uint8)  # [nb, 16]
    sbyte = cand[sel, best].astype(np.uint8)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)  # [nb, 8]
    nbr = cols // KBLOCK
    out = np.concatenate([packed.reshape(rows, nbr * 8), sbyte.reshape(rows, nbr)], axis=1)
    return np.ascontiguousarray(out), float(s2)


def q4_random(rng: np.random.Generator, rows: int, cols: int, std: float = 0.02):
    """Random q4 bytes (uniform codes; E4M3 scale bytes 0x30..0x48, engine/src/gpu_check.cpp:51-63) with a global
    that gives the dequantized values roughly the given standard deviation."""
    nb = cols // KBLOCK
    codes = rng.integers(0, 256, size=(rows, nb * 8), dtype=np.uint8)
    scales = rng.integers(0x30, 0x49, size=(rows, nb), dtype=np.uint8)
    g = std / (np.sqrt(85.0) * 1.6)
    return np.ascontiguousarray(np.concatenate([codes, scales], axis=1)), float(g)


def q4_dequant(packed: np.ndarray, cols: int, glob: float) -> np.ndarray:
    """Pack bytes -> float32 values, (level * 1) * (e4m3 * global) (engine/src/kernels.cpp:1214-1228)."""
    rows = packed.shape[0]
    nb = cols // KBLOCK
    codes = packed[:, : nb * 8]
    sc = packed[:, nb * 8:]
    lo = Q4_LEVELS[codes & 15].astype(np.float32)
    hi = Q4_LEVELS[codes >> 4].astype(np.float32)
    lev = np.empty((rows, cols), dtype=np.float32)
    lev[:, 0::2] = lo
    lev[:, 1::2] = hi
    s = (E4M3[sc] * np.float32(glob)).astype(np.float32)
    return (lev.reshape(rows, nb, KBLOCK) * s[:, :, None]).astype(np.float32).reshape(rows, cols)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


# ----------------------------------------------------------------------------------------------- the pack ----
class _Writer:
    def __init__(self, path: str):
        self.f = open(path, "wb")
        self.off = 0

    def put(self, data: np.ndarray) -> int:
        pad = (-self.off) % 64
        if pad:
            self.f.write(b"\0" * pad)
            self.off += pad
        at = self.off
        b = np.ascontiguousarray(data).tobytes()
        self.f.write(b)
        self.off += len(b)
        return at

    def close(self):
        self.f.close()


def write_draft_vocab(pack_dir: str, ids) -> None:
    """The pack's draft vocabulary: draft_vocab.bin, the token ids as little-endian int32 in order (the file the engine
    reads for its draft head, engine/src/model.cpp:803-827)."""
    np.asarray(ids, dtype="<i4").tofile(os.path.join(pack_dir, "draft_vocab.bin"))


def write_pack(out_dir: str, shape: ModelShape, seed: int = 0, fill: str = "quantized",
               router_std: float = 0.05, weight_std: float = 0.02, mtp: bool = False, distinct_layers: int = 0) -> Dict:
    """Writes a geode-pack for ``shape`` into out_dir; returns the manifest. fill: "quantized" (N(0, weight_std)
    weights through the reference quantizer) or "random" (random q4 bytes). mtp: also the MTP drafting layer, as the
    engine reads it (engine/src/model.cpp:175-191, engine/src/pack.cpp:300-305): mtp.fc.weight [hidden, 2 hidden],
    the norms mtp.norm / mtp.pre_fc_norm_embedding / mtp.pre_fc_norm_hidden, a full-attention decoder layer under
    mtp.layers.0. with its MLP (routed experts after the last layer's, manifest "mtp": {"experts": ...}). Its tensors
    come after every other, so the rest of the pack is the same bytes with or without it. distinct_layers = k > 0:
    only layers 0..k-1 get bytes of their own; layer l >= k names layer l % k's bytes in the manifest (its tensors and
    its expert table entry at the same offsets; the layer kinds must repeat with period k) - a full-depth model whose
    every layer reads as many bytes as a distinct one would, on a pack of k layers' size."""
    os.makedirs(out_dir, exist_ok=True)
    rng = np.random.default_rng(seed)
    s = shape
    H = s.hidden
    tensors: Dict[str, Dict] = {}
    dense = _Writer(os.path.join(out_dir, "dense.bin"))

    def q4(name, rows, cols, std=weight_std):
        if fill == "random":
            b, g = q4_random(rng, rows, cols, std)
        else:
            w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std)
            b, g = q4_quantize(w)
        tensors[name] = {"file": "dense.bin", "offset": dense.put(b), "type": "q4", "shape": [rows, cols], "global": g}

    def f32(name, arr):
        arr = np.asarray(arr, dtype=np.float32)
        tensors[name] = {"file": "dense.bin", "offset": dense.put(arr), "type": "f32", "shape": list(arr.shape)}

    def bf16(name, rows, cols, std):
        w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std)
        tensors[name] = {"file": "dense.bin", "offset": dense.put(bf16_bits(w)), "type": "bf16", "shape": [rows, cols]}

    # the embedding rows are the "fp32 N(0, 1) activations" of the verified tokens
    q4("embed_tokens.weight", s.vocab, H, std=1.0)
    expert_layers = []
    ex_path = os.path.join(out_dir, "experts.bin")
    experts = _Writer(ex_path) if not s.dense else None
    row_b = lambda cols: cols // KBLOCK * 9

    def decoder_layer(p, attn):
        """A decoder layer's tensors under prefix p; its routed experts' table entry (None: dense)."""
        entry = None
        f32(p + "input_layernorm.weight", rng.standard_normal(H, dtype=np.float32) * np.float32(0.1))
        f32(p + "post_attention_layernorm.weight", rng.standard_normal(H, dtype=np.float32) * np.float32(0.1))
        if attn:
            q4(p + "self_attn.q_proj.weight", s.n_heads * s.head_dim * 2, H)
            q4(p + "self_attn.k_proj.weight", s.n_kv_heads * s.head_dim, H)
            q4(p + "self_attn.v_proj.weight", s.n_kv_heads * s.head_dim, H)
            q4(p + "self_attn.o_proj.weight", H, s.n_heads * s.head_dim)
            f32(p + "self_attn.q_norm.weight", rng.standard_normal(s.head_dim, dtype=np.float32) * np.float32(0.1))
            f32(p + "self_attn.k_norm.weight", rng.standard_normal(s.head_dim, dtype=np.float32) * np.float32(0.1))
        else:
            vd = s.gdn_v_heads * s.gdn_v_dim
            q4(p + "linear_attn.in_proj_qkv.weight", s.conv_dim, H)
            q4(p + "linear_attn.in_proj_z.weight", vd, H)
            q4(p + "linear_attn.out_proj.weight", H, vd)
            bf16(p + "linear_attn.in_proj_a.weight", s.gdn_v_heads, H, 0.05)
            bf16(p + "linear_attn.in_proj_b.weight", s.gdn_v_heads, H, 0.05)
            f32(p + "linear_attn.A_log", rng.uniform(0.0, np.log(16.0), s.gdn_v_heads).astype(np.float32))
            f32(p + "linear_attn.dt_bias", rng.standard_normal(s.gdn_v_heads, dtype=np.float32) * np.float32(0.1))
            f32(p + "linear_attn.conv1d.weight",
                rng.standard_normal(s.conv_dim * s.conv_kernel, dtype=np.float32) * np.float32(0.3))
            f32(p + "linear_attn.norm.weight", 1.0 + rng.standard_normal(s.gdn_v_dim, dtype=np.float32) * np.float32(0.1))
        if s.dense:
            q4(p + "mlp.gate_proj.weight", s.shared_ff, H)
            q4(p + "mlp.up_proj.weight", s.shared_ff, H)
            q4(p + "mlp.down_proj.weight", H, s.shared_ff)
        else:
            bf16(p + "mlp.gate.weight", s.n_experts, H, router_std)
            bf16(p + "mlp.shared_expert_gate.weight", 1, H, 0.05)
            q4(p + "mlp.shared_expert.gate_proj.weight", s.shared_ff, H)
            q4(p + "mlp.shared_expert.up_proj.weight", s.shared_ff, H)
            q4(p + "mlp.shared_expert.down_proj.weight", H, s.shared_ff)
            stride = 2 * s.moe_ff * row_b(H) + H * row_b(s.moe_ff)
            scales = np.zeros((s.n_experts, 2), dtype=np.float32)
            first = None
            for e in range(s.n_experts):
                if fill == "random":
                    gu, g0 = q4_random(rng, 2 * s.moe_ff, H, weight_std)
                    dn, g1 = q4_random(rng, H, s.moe_ff, weight_std)
                else:
                    gu, g0 = q4_quantize(rng.standard_normal((2 * s.moe_ff, H), dtype=np.float32) * np.float32(weight_std))
                    dn, g1 = q4_quantize(rng.standard_normal((H, s.moe_ff), dtype=np.float32) * np.float32(weight_std))
                blk = np.concatenate([gu.reshape(-1), dn.reshape(-1)])
                assert blk.size == stride
                if e == 0:
                    at = experts.put(blk)
                    first = at
                else:
                    experts.f.write(blk.tobytes())
                    experts.off += blk.size
                scales[e] = (g0, g1)
            f32(p + "mlp.experts.scales", scales)
            entry = {"file": "experts.bin", "offset": first, "stride": stride, "format": "q4"}
        return entry

    k = distinct_layers if 0 < distinct_layers < s.n_layers else s.n_layers
    for l in range(s.n_layers):
        if l < k:
            entry = decoder_layer(f"layers.{l}.", s.layer_types[l] == "full_attention")
            if entry is not None:
                expert_layers.append(entry)
            continue
        src = l % k
        if s.layer_types[l] != s.layer_types[src]:
            raise ValueError(f"layer {l} is not of layer {src}'s kind: the kinds must repeat every {k} layers")
        pre = f"layers.{src}."
        for name in [n_ for n_ in tensors if n_.startswith(pre)]:
            tensors[f"layers.{l}." + name[len(pre):]] = dict(tensors[name])
        if not s.dense:
            expert_layers.append(dict(expert_layers[src]))

    f32("norm.weight", rng.standard_normal(H, dtype=np.float32) * np.float32(0.1))
    q4("lm_head.weight", s.vocab, H)
    mtp_entry = None
    if mtp:
        q4("mtp.fc.weight", H, 2 * H)
        for n_ in ("mtp.norm.weight", "mtp.pre_fc_norm_embedding.weight", "mtp.pre_fc_norm_hidden.weight"):
            f32(n_, rng.standard_normal(H, dtype=np.float32) * np.float32(0.1))
        mtp_entry = decoder_layer("mtp.layers.0.", True)
    dense.close()
    files = [{"name": "dense.bin", "size": os.path.getsize(os.path.join(out_dir, "dense.bin"))}]
    if experts is not None:
        experts.close()
        files.append({"name": "experts.bin", "size": os.path.getsize(ex_path)})
    cfg = {
        "hidden_size": H, "num_hidden_layers": s.n_layers, "vocab_size": s.vocab, "rms_norm_eps": s.eps,
        "num_attention_heads": s.n_heads, "num_key_value_heads": s.n_kv_heads, "head_dim": s.head_dim,
        "rope_parameters": {"rope_theta": s.rope_theta, "partial_rotary_factor": s.partial_rotary},
        "linear_num_key_heads": s.gdn_k_heads, "linear_num_value_heads": s.gdn_v_heads,
        "linear_key_head_dim": s.gdn_k_dim, "linear_value_head_dim": s.gdn_v_dim,
        "linear_conv_kernel_dim": s.conv_kernel, "layer_types": s.layer_types,
    }
    if s.dense:
        cfg["intermediate_size"] = s.shared_ff
    else:
        cfg.update({"num_experts": s.n_experts, "num_experts_per_tok": s.top_k, "moe_intermediate_size": s.moe_ff,
                    "shared_expert_intermediate_size": s.shared_ff})
    manifest = {"format": "geode-pack", "version": 1, "arch": s.arch, "files": files, "config": cfg,
                "tensors": tensors, "experts": {"layers": expert_layers}, "formats": {"q4": {"layout": "rows"}}}
    if mtp:
        manifest["mtp"] = {"experts": mtp_entry} if mtp_entry is not None else {}
    with open(os.path.join(out_dir, "geode.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    return manifest
