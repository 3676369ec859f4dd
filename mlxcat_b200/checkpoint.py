"""MLX-format checkpoints for the device model (safetensors + config.json).

mlx-lm stores a 4-bit model as safetensors files next to a ``config.json``:
every quantized linear ``<name>`` is three tensors -- ``<name>.weight``
(uint32 [out][in/8], 8 nibbles per word, lowest first), ``<name>.scales`` and
``<name>.biases`` ([out][in/64], the model's float dtype) -- and the RMSNorm
weights are plain float vectors.  This module reads that layout (the
safetensors container is parsed here: an 8-byte little-endian header length, a
JSON header of {name: {dtype, shape, data_offsets}}, then the raw bytes) and
loads it into a ``Context`` through the C ABI (mlxcat_weights_set_q4 /
_set_bf16 / _set_norm); ``save_mlx_checkpoint`` writes a context's weights
back in the same layout.

Names follow mlx-lm's Llama / Qwen3 / Qwen3-MoE modules (un-vendored here):
``model.embed_tokens``, ``model.layers.{l}.self_attn.{q,k,v,o}_proj``,
``model.layers.{l}.self_attn.{q,k}_norm`` (Qwen3), ``model.layers.{l}.
{input,post_attention}_layernorm``, ``model.layers.{l}.mlp.{gate,up,down}_proj``,
MoE ``model.layers.{l}.mlp.gate`` (router) and ``model.layers.{l}.mlp.
switch_mlp.{gate,up,down}_proj`` (stacked [experts][out][in/8]), ``model.norm``,
``lm_head``.  Scales and biases are converted to fp16 (the kernels' format);
a quantized router is dequantised to bf16 (the router is kept bf16).
"""
from __future__ import annotations

import json
import mmap
import os
import struct
from typing import Dict, Tuple

import numpy as np

from .engine import Context, ModelConfig

_DTYPES = {"U32": np.uint32, "I32": np.int32, "F32": np.float32, "F16": np.float16, "BF16": np.uint16,
           "U16": np.uint16, "U8": np.uint8, "I64": np.int64}
_NAMES = {v: k for k, v in _DTYPES.items() if k not in ("BF16",)}

TENSOR_EMBED = 0xFFFF0000
TENSOR_LM_HEAD = 0xFFFF0001
_LINEARS = (("self_attn.q_proj", 0), ("self_attn.k_proj", 1), ("self_attn.v_proj", 2), ("self_attn.o_proj", 3),
            ("mlp.gate_proj", 4), ("mlp.up_proj", 5), ("mlp.down_proj", 6))
_SWITCH = (("mlp.switch_mlp.gate_proj", 0), ("mlp.switch_mlp.up_proj", 1), ("mlp.switch_mlp.down_proj", 2))
_NORMS = (("input_layernorm", 0), ("post_attention_layernorm", 1), ("self_attn.q_norm", 2),
          ("self_attn.k_norm", 3))


def tensor_expert(layer: int, expert: int, kind: int) -> int:
    return 0x40000000 | (layer << 12) | (expert << 2) | kind


# --------------------------------------------------------------------------- #
# safetensors container
# --------------------------------------------------------------------------- #
def read_safetensors(path: str) -> Tuple[Dict[str, np.ndarray], Dict[str, str], Dict[str, str]]:
    """(tensors, metadata, dtypes) of one file: numpy views of the mapped file
    (BF16 as uint16 bits), the header's __metadata__, and each tensor's dtype name."""
    # mapped, not read: a 70B checkpoint's shards are tens of GB, and each tensor
    # is a view of the mapping until it is copied to the device
    with open(path, "rb") as f:
        size = os.fstat(f.fileno()).st_size
        data = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) if size else b""
    if len(data) < 8:
        raise ValueError(f"{path}: not a safetensors file")
    (n,) = struct.unpack("<Q", data[:8])
    if 8 + n > len(data):
        raise ValueError(f"{path}: header length {n} past the end of the file")
    header = json.loads(bytes(data[8:8 + n]).decode("utf-8"))
    meta = header.pop("__metadata__", {}) or {}
    base = 8 + n
    out = {}
    for name, d in header.items():
        dt = _DTYPES.get(d["dtype"])
        if dt is None:
            raise ValueError(f"{path}: tensor {name} has unsupported dtype {d['dtype']}")
        b0, b1 = d["data_offsets"]
        shape = tuple(d["shape"])
        count = int(np.prod(shape)) if shape else 1
        if b1 - b0 != count * np.dtype(dt).itemsize or base + b1 > len(data):
            raise ValueError(f"{path}: tensor {name} has inconsistent offsets")
        a = np.frombuffer(data, dtype=dt, count=count, offset=base + b0).reshape(shape)
        out[name] = (a, d["dtype"])
    return {k: v[0] for k, v in out.items()}, meta, {k: v[1] for k, v in out.items()}


def write_safetensors(path: str, tensors: Dict[str, np.ndarray], metadata: Dict[str, str] | None = None,
                      bf16: Tuple[str, ...] = ()):
    """Tensors in name order; names in `bf16` are uint16 arrays of bf16 bits."""
    header, off, blobs = {}, 0, []
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name])
        dt = "BF16" if name in bf16 else _NAMES[a.dtype.type]
        b = a.tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode("utf-8")
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


# --------------------------------------------------------------------------- #
# config.json
# --------------------------------------------------------------------------- #
def config_from_mlx(c: dict, name: str = "mlx") -> ModelConfig:
    """ModelConfig of an mlx-lm config.json (model_type llama, qwen3 or qwen3_moe)."""
    mt = c.get("model_type", "llama")
    if mt not in ("llama", "qwen3", "qwen3_moe"):
        raise ValueError(f"model_type {mt!r} is not on this path (llama, qwen3, qwen3_moe)")
    q = c.get("quantization") or c.get("quantization_config") or {}
    if q.get("group_size", 64) != 64 or q.get("bits", 4) != 4:
        raise ValueError("only MLX affine 4-bit group-64 checkpoints are supported")
    H, heads = int(c["hidden_size"]), int(c["num_attention_heads"])
    moe = mt == "qwen3_moe"
    return ModelConfig(
        n_layers=int(c["num_hidden_layers"]), hidden=H, n_heads=heads,
        n_kv_heads=int(c.get("num_key_value_heads", heads)), head_dim=int(c.get("head_dim", H // heads)),
        intermediate=int(c["moe_intermediate_size"] if moe else c["intermediate_size"]),
        vocab=int(c["vocab_size"]), tie_embeddings=bool(c.get("tie_word_embeddings", False)),
        qk_norm=mt in ("qwen3", "qwen3_moe"), rms_eps=float(c.get("rms_norm_eps", 1e-5)),
        rope_theta=float(c.get("rope_theta", 10000.0)), name=name,
        n_experts=int(c.get("num_experts", 0)) if moe else 0,
        top_k=int(c.get("num_experts_per_tok", 0)) if moe else 0,
        norm_topk=bool(c.get("norm_topk_prob", True)) if moe else True)


def config_to_mlx(cfg: ModelConfig) -> dict:
    mt = "qwen3_moe" if cfg.n_experts else ("qwen3" if cfg.qk_norm else "llama")
    c = {"model_type": mt, "hidden_size": cfg.hidden, "num_hidden_layers": cfg.n_layers,
         "num_attention_heads": cfg.n_heads, "num_key_value_heads": cfg.n_kv_heads, "head_dim": cfg.head_dim,
         "vocab_size": cfg.vocab, "tie_word_embeddings": bool(cfg.tie_embeddings), "rms_norm_eps": cfg.rms_eps,
         "rope_theta": cfg.rope_theta, "quantization": {"group_size": 64, "bits": 4}}
    if cfg.n_experts:
        c.update(moe_intermediate_size=cfg.intermediate, num_experts=cfg.n_experts,
                 num_experts_per_tok=cfg.top_k, norm_topk_prob=bool(cfg.norm_topk))
    else:
        c["intermediate_size"] = cfg.intermediate
    return c


# --------------------------------------------------------------------------- #
# name <-> device tensor mapping
# --------------------------------------------------------------------------- #
def q4_tensors(cfg: ModelConfig):
    """(mlx name, device tensor id, out, in) of every dense q4 linear (the
    MoE experts are stacked per projection, see _SWITCH)."""
    H, D, I = cfg.hidden, cfg.head_dim, cfg.intermediate
    shapes = {0: (cfg.n_heads * D, H), 1: (cfg.n_kv_heads * D, H), 2: (cfg.n_kv_heads * D, H),
              3: (H, cfg.n_heads * D), 4: (I, H), 5: (I, H), 6: (H, I)}
    out = [("model.embed_tokens", TENSOR_EMBED, cfg.vocab, H)]
    for l in range(cfg.n_layers):
        for suffix, kind in _LINEARS:
            if cfg.n_experts and kind >= 4:
                continue
            out.append((f"model.layers.{l}.{suffix}", l * 16 + kind) + shapes[kind])
    if not cfg.tie_embeddings:
        out.append(("lm_head", TENSOR_LM_HEAD, cfg.vocab, H))
    return out


def norm_tensors(cfg: ModelConfig):
    """(mlx name, device norm id, length) of every RMSNorm weight."""
    out = []
    for l in range(cfg.n_layers):
        for suffix, kind in _NORMS:
            if kind >= 2 and not cfg.qk_norm:
                continue
            out.append((f"model.layers.{l}.{suffix}.weight", Context.norm_id(l, kind),
                        cfg.head_dim if kind >= 2 else cfg.hidden))
    out.append(("model.norm.weight", Context.NORM_FINAL, cfg.hidden))
    return out


def _f16(a: np.ndarray, dtype: str) -> np.ndarray:
    """scales / biases in the kernels' fp16, as uint16 bits"""
    if dtype == "F16":
        return np.ascontiguousarray(a).view(np.uint16)
    if dtype == "BF16":
        f = (a.astype(np.uint32) << 16).view(np.float32)
        return f.astype(np.float16).view(np.uint16)
    return np.asarray(a, np.float32).astype(np.float16).view(np.uint16)


def _f32(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "BF16":
        return (a.astype(np.uint32) << 16).view(np.float32)
    return np.asarray(a, np.float32)


def _bf16_bits(f: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even"""
    u = np.ascontiguousarray(f, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    return r.astype(np.uint16)


def _tp_slice(cfg: ModelConfig, tid: int, wq, s, b):
    """This tensor-parallel rank's part of a full q4 tensor: q/k/v heads and
    gate/up rows (column split), the matching input columns of o and down
    (row split, whole 64-column groups); embedding and lm_head replicated."""
    T, r, D = cfg.tp_size, cfg.tp_rank, cfg.head_dim
    if tid in (TENSOR_EMBED, TENSOR_LM_HEAD):
        return wq, s, b
    kind = tid % 16
    if kind in (0, 1, 2, 4, 5):
        n = {0: cfg.n_heads * D, 1: cfg.n_kv_heads * D, 2: cfg.n_kv_heads * D, 4: cfg.intermediate,
             5: cfg.intermediate}[kind] // T
        return wq[r * n:(r + 1) * n], s[r * n:(r + 1) * n], b[r * n:(r + 1) * n]
    k = (cfg.n_heads * D if kind == 3 else cfg.intermediate) // T
    if k % 64:
        raise ValueError("tensor-parallel slices must hold whole 64-column groups")
    return (wq[:, r * k // 8:(r + 1) * k // 8], s[:, r * k // 64:(r + 1) * k // 64],
            b[:, r * k // 64:(r + 1) * k // 64])


def _load_all(path: str):
    files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {path}")
    tensors, dtypes = {}, {}
    for f in files:
        t, _, d = read_safetensors(os.path.join(path, f))
        tensors.update(t)
        dtypes.update(d)
    return tensors, dtypes


def load_mlx_checkpoint(path: str, device: int = 0, **overrides) -> Context:
    """A Context on `device` holding the checkpoint in directory `path`
    (config.json + *.safetensors).  `overrides` replace ModelConfig fields
    (e.g. tp_size / tp_rank, ep_size / ep_rank: each rank loads its slice)."""
    import dataclasses
    with open(os.path.join(path, "config.json")) as f:
        cfg = config_from_mlx(json.load(f), name=os.path.basename(os.path.normpath(path)))
    if overrides:
        cfg = dataclasses.replace(cfg, **overrides)
    tensors, dtypes = _load_all(path)

    def need(name):
        if name not in tensors:
            raise KeyError(f"checkpoint lacks {name}")
        return tensors[name], dtypes[name]

    ctx = Context(cfg, device)
    try:
        for name, tid, n_out, n_in in q4_tensors(cfg):
            wq, wd = need(name + ".weight")
            s, sd = need(name + ".scales")
            b, bd = need(name + ".biases")
            if wd != "U32" or wq.shape != (n_out, n_in // 8) or s.shape != (n_out, n_in // 64):
                raise ValueError(f"{name}: expected uint32 [{n_out}][{n_in // 8}] with [{n_out}][{n_in // 64}] "
                                 f"scales, got {wd} {wq.shape} / {s.shape}")
            s, b = _f16(s, sd), _f16(b, bd)
            if cfg.tp_size > 1:
                wq, s, b = _tp_slice(cfg, tid, wq, s, b)
            ctx.set_q4(tid, wq, s, b)
        for l in range(cfg.n_layers if cfg.n_experts else 0):
            E, H, I = cfg.n_experts, cfg.hidden, cfg.intermediate
            rname = f"model.layers.{l}.mlp.gate"
            r, rd = need(rname + ".weight")
            if rd == "U32":   # a quantized router: dequantised, then kept bf16
                s, sd = need(rname + ".scales")
                b, bd = need(rname + ".biases")
                sh = np.repeat(_f16(s, sd).view(np.float16).astype(np.float32), 64, axis=1)
                bh = np.repeat(_f16(b, bd).view(np.float16).astype(np.float32), 64, axis=1)
                q = ((r[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 15).reshape(E, H).astype(np.float32)
                rbits = _bf16_bits(sh * q + bh)
            else:
                rbits = r.astype(np.uint16) if rd == "BF16" else _bf16_bits(_f32(r, rd))
            ctx.set_bf16(l * 16 + 7, rbits.reshape(E, H))
            for suffix, kind in _SWITCH:
                wq, _ = need(f"model.layers.{l}.{suffix}.weight")
                s, sd = need(f"model.layers.{l}.{suffix}.scales")
                b, bd = need(f"model.layers.{l}.{suffix}.biases")
                n_out, n_in = (I, H) if kind < 2 else (H, I)
                if wq.shape != (E, n_out, n_in // 8):
                    raise ValueError(f"{suffix} of layer {l}: expected [{E}][{n_out}][{n_in // 8}], got {wq.shape}")
                s16, b16 = _f16(s, sd).reshape(E, n_out, -1), _f16(b, bd).reshape(E, n_out, -1)
                lo = cfg.ep_rank * (E // cfg.ep_size) if cfg.ep_size > 1 else 0
                hi = lo + (E // cfg.ep_size if cfg.ep_size > 1 else E)
                for e in range(lo, hi):
                    ctx.set_q4(tensor_expert(l, e, kind), wq[e], s16[e], b16[e])
        for name, nid, n in norm_tensors(cfg):
            w, wd = need(name)
            if w.shape != (n,):
                raise ValueError(f"{name}: expected [{n}], got {w.shape}")
            ctx.set_norm(nid, _f32(w, wd))
    except Exception:
        ctx.close()
        raise
    return ctx


def save_mlx_checkpoint(ctx: Context, path: str, norms: Dict[int, np.ndarray] | None = None):
    """Write a (one-GPU) context's weights as an MLX checkpoint: config.json and
    model.safetensors (scales / biases fp16).  `norms` maps norm ids to their
    weights (the device holds them write-only; missing ones are written as 1)."""
    cfg = ctx.cfg
    if cfg.tp_size > 1 or cfg.ep_size > 1:
        raise ValueError("save a checkpoint from a one-GPU context")
    os.makedirs(path, exist_ok=True)
    t, bf16 = {}, []
    for name, tid, n_out, n_in in q4_tensors(cfg):
        wq, s, b = ctx.get_q4(tid, n_out, n_in)
        t[name + ".weight"] = wq
        t[name + ".scales"] = np.ascontiguousarray(s).view(np.float16)
        t[name + ".biases"] = np.ascontiguousarray(b).view(np.float16)
    for l in range(cfg.n_layers if cfg.n_experts else 0):
        E, H, I = cfg.n_experts, cfg.hidden, cfg.intermediate
        t[f"model.layers.{l}.mlp.gate.weight"] = ctx.get_bf16(l * 16 + 7, (E, H))
        bf16.append(f"model.layers.{l}.mlp.gate.weight")
        for suffix, kind in _SWITCH:
            n_out, n_in = (I, H) if kind < 2 else (H, I)
            parts = [ctx.get_q4(tensor_expert(l, e, kind), n_out, n_in) for e in range(E)]
            t[f"model.layers.{l}.{suffix}.weight"] = np.stack([p[0] for p in parts])
            t[f"model.layers.{l}.{suffix}.scales"] = np.stack([np.asarray(p[1]).view(np.float16) for p in parts])
            t[f"model.layers.{l}.{suffix}.biases"] = np.stack([np.asarray(p[2]).view(np.float16) for p in parts])
    for name, nid, n in norm_tensors(cfg):
        w = (norms or {}).get(nid)
        t[name] = np.ones(n, np.float32) if w is None else np.asarray(w, np.float32)
    write_safetensors(os.path.join(path, "model.safetensors"), t, {"format": "mlx"}, bf16=tuple(bf16))
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(config_to_mlx(cfg), f, indent=1)
