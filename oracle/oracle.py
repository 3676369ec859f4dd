"""ctypes wrapper over liboracle.so -- the CPU restatement of mlxcat's n-gram
speculative-decode path.

TEST INFRASTRUCTURE ONLY.  Loaded by tests/, by ``__graft_entry__.smoke()`` as
the checker, and by bench.py's CPU legs.  The product package never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

MODE_COMPAT = 0
MODE_PREFIX = 1
T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN, T_ROUTER = range(8)
TENSOR_EMBED = 0xFFFF0000
TENSOR_LM_HEAD = 0xFFFF0001


def tensor_expert(layer: int, expert: int, kind: int) -> int:
    """id of a MoE expert tensor (kind 0 gate, 1 up, 2 down)"""
    return 0x40000000 | (layer << 12) | (expert << 2) | kind


def build() -> str:
    """Compile liboracle.so with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class Config(C.Structure):
    _fields_ = [
        ("n_layers", C.c_int), ("hidden", C.c_int), ("n_heads", C.c_int),
        ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("intermediate", C.c_int),
        ("vocab", C.c_int), ("tie_embeddings", C.c_int), ("qk_norm", C.c_int),
        ("rms_eps", C.c_float), ("rope_theta", C.c_float),
        ("n_experts", C.c_int), ("top_k", C.c_int), ("norm_topk", C.c_int),
    ]


class Sampling(C.Structure):
    _fields_ = [
        ("temperature", C.c_float), ("top_p", C.c_float), ("seed", C.c_uint64),
        ("has_seed", C.c_int32), ("eos", C.c_int32 * 8), ("n_eos", C.c_int32),
        ("trigger", C.c_int32),
    ]


class SpecConfig(C.Structure):
    _fields_ = [
        ("mode", C.c_int), ("enabled", C.c_int), ("max_proposal", C.c_int),
        ("max_suffix", C.c_int), ("min_context", C.c_int),
    ]


class Stats(C.Structure):
    _fields_ = [
        ("proposed", C.c_int64), ("accepted", C.c_int64),
        ("proposal_batches", C.c_int64), ("rejected_batches", C.c_int64),
    ]


class Row(C.Structure):
    _fields_ = [
        ("hist", C.POINTER(C.c_int32)), ("hist_len", C.c_int), ("hist_cap", C.c_int),
        ("n_gen", C.c_int), ("max_new", C.c_int), ("active", C.c_int),
        ("sp", Sampling),
    ]


def _ptr(a, ctype):
    return a.ctypes.data_as(C.POINTER(ctype))


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    L = C.CDLL(_LIB_PATH)
    u32p, u16p, f32p, i32p = (C.POINTER(C.c_uint32), C.POINTER(C.c_uint16),
                              C.POINTER(C.c_float), C.POINTER(C.c_int32))
    L.orc_philox4x32_10.argtypes = [u32p, u32p, u32p]
    L.orc_set_threads.argtypes = [C.c_int]; L.orc_set_threads.restype = C.c_int
    L.orc_exp_neg.argtypes = [C.c_float]; L.orc_exp_neg.restype = C.c_float
    L.orc_log.argtypes = [C.c_float]; L.orc_log.restype = C.c_float
    L.orc_normal.argtypes = [C.c_uint64, C.c_uint32, C.c_uint64]; L.orc_normal.restype = C.c_float
    L.orc_uniform_u32.argtypes = [C.c_uint64, C.c_uint64, C.c_uint32]
    L.orc_uniform_u32.restype = C.c_uint32
    L.orc_q4_quantize_row.argtypes = [f32p, C.c_int, u32p, u16p, u16p]
    L.orc_q4_synth.argtypes = [C.c_uint64, C.c_uint32, C.c_float, C.c_int, C.c_int, u32p, u16p, u16p]
    L.orc_q4_dequant.argtypes = [u32p, u16p, u16p, C.c_int, C.c_int, f32p]
    L.orc_q4_linear.argtypes = [u32p, u16p, u16p, C.c_int, C.c_int, f32p, C.c_int, f32p]
    L.orc_propose_suffix.argtypes = [i32p, C.c_int, C.c_int, C.c_int, C.c_int, i32p]
    L.orc_propose_suffix.restype = C.c_int
    L.orc_argmax.argtypes = [f32p, C.c_int]; L.orc_argmax.restype = C.c_int
    L.orc_top_p_keep.argtypes = [f32p, C.c_int, C.c_float, C.POINTER(C.c_uint8)]
    L.orc_fixed_dist.argtypes = [f32p, C.c_int, C.c_float, C.c_float, u32p]
    L.orc_fixed_dist.restype = C.c_uint64
    L.orc_pick.argtypes = [u32p, C.c_int, C.c_uint64, C.c_uint32, C.c_int]
    L.orc_pick.restype = C.c_int
    L.orc_accept_row.argtypes = [C.c_int, f32p, C.c_int, i32p, C.c_int, C.POINTER(Sampling),
                                 C.c_uint64, i32p, C.POINTER(C.c_int)]
    L.orc_accept_row.restype = C.c_int
    L.orc_tensor_id.argtypes = [C.c_int, C.c_int]; L.orc_tensor_id.restype = C.c_uint32
    L.orc_model_synth.argtypes = [C.POINTER(Config), C.c_uint64, C.c_float]
    L.orc_model_synth.restype = C.c_void_p
    L.orc_model_table.argtypes = [i32p, C.c_int]; L.orc_model_table.restype = C.c_void_p
    L.orc_model_empty.argtypes = [C.POINTER(Config)]; L.orc_model_empty.restype = C.c_void_p
    L.orc_model_set_q4.argtypes = [C.c_void_p, C.c_uint32, u32p, u16p, u16p]
    L.orc_model_set_q4.restype = C.c_int
    L.orc_model_get_q4.argtypes = [C.c_void_p, C.c_uint32, C.POINTER(u32p), C.POINTER(u16p),
                                   C.POINTER(u16p), C.POINTER(C.c_int), C.POINTER(C.c_int)]
    L.orc_model_free.argtypes = [C.c_void_p]
    L.orc_kv_create.argtypes = [C.c_void_p, C.c_int, C.c_int]; L.orc_kv_create.restype = C.c_void_p
    L.orc_kv_free.argtypes = [C.c_void_p]
    L.orc_kv_len.argtypes = [C.c_void_p, C.c_int]; L.orc_kv_len.restype = C.c_int
    L.orc_kv_set_len.argtypes = [C.c_void_p, C.c_int, C.c_int]
    L.orc_kv_trim.argtypes = [C.c_void_p, C.c_int]; L.orc_kv_trim.restype = C.c_int
    L.orc_kv_k.argtypes = [C.c_void_p, C.c_int, C.c_int]; L.orc_kv_k.restype = f32p
    L.orc_kv_v.argtypes = [C.c_void_p, C.c_int, C.c_int]; L.orc_kv_v.restype = f32p
    L.orc_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int, i32p, i32p, i32p, f32p]
    L.orc_spec_step.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(Row), C.c_int,
                                C.POINTER(SpecConfig), i32p, i32p, C.POINTER(Stats)]
    L.orc_admit.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(Row), C.c_int, i32p, C.c_int, C.c_int]
    L.orc_admit.restype = C.c_int
    L.orc_router_synth.argtypes = [C.c_uint64, C.c_uint32, C.c_float, C.c_int, C.c_int, u16p]
    L.orc_model_set_router.argtypes = [C.c_void_p, C.c_int, u16p]
    L.orc_model_set_router.restype = C.c_int
    L.orc_model_set_norm.argtypes = [C.c_void_p, C.c_uint32, f32p]
    L.orc_model_set_norm.restype = C.c_int
    L.orc_moe_route.argtypes = [C.c_void_p, C.c_int, f32p, i32p, f32p]
    L.orc_moe_route.restype = C.c_float
    L.orc_moe_min_margin.argtypes = [C.c_int]
    L.orc_moe_min_margin.restype = C.c_float
    L.orc_f32_to_bf16.argtypes = [C.c_float]; L.orc_f32_to_bf16.restype = C.c_uint16
    L.orc_moe_force.argtypes = [C.c_int, C.c_int, C.c_int, i32p, f32p]
    L.orc_moe_force_deviation.argtypes = [C.c_int]
    L.orc_moe_force_deviation.restype = C.c_float
    L.orc_moe_force_weight_deviation.argtypes = [C.c_int]
    L.orc_moe_force_weight_deviation.restype = C.c_float
    L.orc_moe_mlp.argtypes = [C.c_void_p, C.c_int, f32p, C.c_int, f32p, i32p, f32p, f32p]
    _lib = L
    return L


# --------------------------------------------------------------------------- #
# thin numpy helpers
# --------------------------------------------------------------------------- #
def set_threads(n: int = 0) -> int:
    """OpenMP threads for the oracle's loops (0: every host core)"""
    return int(lib().orc_set_threads(n))


def philox(ctr, key):
    c = np.asarray(ctr, dtype=np.uint32)
    k = np.asarray(key, dtype=np.uint32)
    out = np.zeros(4, dtype=np.uint32)
    lib().orc_philox4x32_10(_ptr(c, C.c_uint32), _ptr(k, C.c_uint32), _ptr(out, C.c_uint32))
    return out


def exp_neg(x: float) -> float:
    return lib().orc_exp_neg(x)


def log(x: float) -> float:
    return lib().orc_log(x)


def normal(seed: int, tensor_id: int, index: int) -> float:
    return lib().orc_normal(seed, tensor_id, index)


def uniform_u32(seed: int, gen_index: int, purpose: int) -> int:
    return lib().orc_uniform_u32(seed, gen_index, purpose)


def q4_quantize(w: np.ndarray):
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    wq = np.zeros((N, K // 8), np.uint32)
    s = np.zeros((N, K // 64), np.uint16)
    b = np.zeros((N, K // 64), np.uint16)
    for n in range(N):
        lib().orc_q4_quantize_row(_ptr(w[n], C.c_float), K, _ptr(wq[n], C.c_uint32),
                                  _ptr(s[n], C.c_uint16), _ptr(b[n], C.c_uint16))
    return wq, s, b


def q4_synth(seed: int, tensor_id: int, stddev: float, N: int, K: int):
    wq = np.zeros((N, K // 8), np.uint32)
    s = np.zeros((N, K // 64), np.uint16)
    b = np.zeros((N, K // 64), np.uint16)
    lib().orc_q4_synth(seed, tensor_id, stddev, N, K, _ptr(wq, C.c_uint32),
                       _ptr(s, C.c_uint16), _ptr(b, C.c_uint16))
    return wq, s, b


def q4_dequant(wq, s, b):
    N = wq.shape[0]
    K = wq.shape[1] * 8
    w = np.zeros((N, K), np.float32)
    lib().orc_q4_dequant(_ptr(np.ascontiguousarray(wq), C.c_uint32),
                         _ptr(np.ascontiguousarray(s), C.c_uint16),
                         _ptr(np.ascontiguousarray(b), C.c_uint16), N, K, _ptr(w, C.c_float))
    return w


def q4_linear(wq, s, b, x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    N = wq.shape[0]
    y = np.zeros((M, N), np.float32)
    lib().orc_q4_linear(_ptr(np.ascontiguousarray(wq), C.c_uint32),
                        _ptr(np.ascontiguousarray(s), C.c_uint16),
                        _ptr(np.ascontiguousarray(b), C.c_uint16), N, K,
                        _ptr(x, C.c_float), M, _ptr(y, C.c_float))
    return y


def propose_suffix(ctx, max_suffix: int, min_ctx: int, limit: int):
    c = np.ascontiguousarray(ctx, dtype=np.int32)
    out = np.zeros(max(limit, 1), np.int32)
    n = lib().orc_propose_suffix(_ptr(c, C.c_int32), len(c), max_suffix, min_ctx, limit,
                                 _ptr(out, C.c_int32))
    return out[:n].tolist() if n > 0 else None


def argmax(logits) -> int:
    l = np.ascontiguousarray(logits, dtype=np.float32)
    return lib().orc_argmax(_ptr(l, C.c_float), l.shape[-1])


def top_p_keep(logits, top_p: float):
    l = np.ascontiguousarray(logits, dtype=np.float32)
    keep = np.zeros(l.shape[-1], np.uint8)
    lib().orc_top_p_keep(_ptr(l, C.c_float), l.shape[-1], top_p, _ptr(keep, C.c_uint8))
    return keep.astype(bool)


def fixed_dist(logits, temperature: float, top_p: float):
    l = np.ascontiguousarray(logits, dtype=np.float32)
    P = np.zeros(l.shape[-1], np.uint32)
    S = lib().orc_fixed_dist(_ptr(l, C.c_float), l.shape[-1], temperature, top_p,
                             _ptr(P, C.c_uint32))
    return P, S


def pick(P, S: int, u: int, skip: int = -1) -> int:
    P = np.ascontiguousarray(P, dtype=np.uint32)
    return lib().orc_pick(_ptr(P, C.c_uint32), len(P), S, u, skip)


def sampling(temperature=0.0, top_p=0.0, seed=None, eos=(), trigger=-1) -> Sampling:
    sp = Sampling()
    sp.temperature = temperature
    sp.top_p = top_p
    sp.seed = 0 if seed is None else seed
    sp.has_seed = 0 if seed is None else 1
    eos = list(eos)[:8]
    for i, e in enumerate(eos):
        sp.eos[i] = e
    sp.n_eos = len(eos)
    sp.trigger = trigger
    return sp


def accept_row(mode, logits, drafts, sp: Sampling, gen_index: int):
    l = np.ascontiguousarray(logits, dtype=np.float32)
    d = np.ascontiguousarray(drafts if len(drafts) else [0], dtype=np.int32)
    count = len(drafts)
    out = np.zeros(count + 1, np.int32)
    rej = C.c_int(0)
    n = lib().orc_accept_row(mode, _ptr(l, C.c_float), l.shape[-1], _ptr(d, C.c_int32), count,
                             C.byref(sp), gen_index, _ptr(out, C.c_int32), C.byref(rej))
    return out[:n].tolist(), bool(rej.value)


# --------------------------------------------------------------------------- #
# model / cache / generator
# --------------------------------------------------------------------------- #
def apply_allowed_mask(logits, allowed_ids):
    """applyAllowedTokenMask (Sources/MLXCat/TrackB/Sampling.swift:557-569):
    ids outside [0, vocab) are dropped; if none is left the logits come back
    unchanged, else every logit outside the allowed ids becomes -inf (fp32)."""
    out = np.array(logits, dtype=np.float32, copy=True)
    V = out.shape[-1]
    valid = sorted({int(t) for t in allowed_ids if 0 <= int(t) < V})
    if not valid:
        return out
    keep = np.zeros(V, dtype=bool)
    keep[valid] = True
    out[..., ~keep] = -np.inf
    return out


def make_config(n_layers, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab,
                tie_embeddings=True, qk_norm=False, rms_eps=1e-5, rope_theta=10000.0,
                n_experts=0, top_k=0, norm_topk=True) -> Config:
    return Config(n_layers, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab,
                  int(tie_embeddings), int(qk_norm), rms_eps, rope_theta, n_experts, top_k,
                  int(norm_topk))


def router_synth(seed: int, tensor_id: int, stddev: float, E: int, H: int):
    w = np.zeros((E, H), np.uint16)
    lib().orc_router_synth(seed, tensor_id, stddev, E, H, _ptr(w, C.c_uint16))
    return w


def moe_force(ids, weights=None):
    """Force the expert choices of the next forwards: ids [n_layers][M][top_k]
    (e.g. the device's routing of the same verify forward), and optionally their
    weights; None clears."""
    if ids is None:
        lib().orc_moe_force(0, 0, 0, None, None)
        return
    a = np.ascontiguousarray(ids, dtype=np.int32)
    w = None if weights is None else np.ascontiguousarray(weights, dtype=np.float32)
    lib().orc_moe_force(a.shape[0], a.shape[1], a.shape[2], _ptr(a, C.c_int32),
                        None if w is None else _ptr(w, C.c_float))


def moe_force_deviation(reset=True) -> float:
    """largest distance (bf16 steps) between a forced choice and the oracle's own"""
    return float(lib().orc_moe_force_deviation(int(reset)))


def moe_force_weight_deviation(reset=True) -> float:
    """largest relative difference between a forced routing weight and the oracle's own"""
    return float(lib().orc_moe_force_weight_deviation(int(reset)))


def moe_min_margin(reset=True) -> float:
    return float(lib().orc_moe_min_margin(int(reset)))


class Model:
    def __init__(self, handle, cfg: Config | None, vocab: int):
        self.h = handle
        self.cfg = cfg
        self.vocab = vocab

    @classmethod
    def synth(cls, cfg: Config, seed: int, stddev: float = 0.02):
        return cls(lib().orc_model_synth(C.byref(cfg), seed, stddev), cfg, cfg.vocab)

    @classmethod
    def table(cls, next_tokens):
        n = np.ascontiguousarray(next_tokens, dtype=np.int32)
        return cls(lib().orc_model_table(_ptr(n, C.c_int32), len(n)), None, len(n))

    @classmethod
    def empty(cls, cfg: Config):
        return cls(lib().orc_model_empty(C.byref(cfg)), cfg, cfg.vocab)

    def set_q4(self, tensor_id: int, wq, s, b):
        rc = lib().orc_model_set_q4(self.h, tensor_id, _ptr(np.ascontiguousarray(wq), C.c_uint32),
                                    _ptr(np.ascontiguousarray(s), C.c_uint16),
                                    _ptr(np.ascontiguousarray(b), C.c_uint16))
        if rc != 0:
            raise KeyError(tensor_id)

    def set_norm(self, norm_id: int, w):
        """RMSNorm weights (id layer*16 + {8 input, 9 post-attention, 10 q,
        11 k}, 0xFFFF0002 final)"""
        if lib().orc_model_set_norm(self.h, norm_id, _ptr(np.ascontiguousarray(w, np.float32), C.c_float)):
            raise KeyError(norm_id)

    def set_router(self, layer: int, w):
        if lib().orc_model_set_router(self.h, layer, _ptr(np.ascontiguousarray(w, np.uint16), C.c_uint16)):
            raise KeyError(layer)

    def route(self, layer: int, x):
        """(expert ids, weights, margin) of one token's normalised MLP input"""
        k = self.cfg.top_k
        ids = np.zeros(k, np.int32)
        w = np.zeros(k, np.float32)
        xv = np.ascontiguousarray(x, np.float32)
        mg = lib().orc_moe_route(self.h, layer, _ptr(xv, C.c_float), _ptr(ids, C.c_int32), _ptr(w, C.c_float))
        return ids, w, float(mg)

    def moe_mlp(self, layer: int, x):
        """(y, ids, weights, margins) of the MoE MLP of `layer` on x [M][hidden]"""
        xv = np.ascontiguousarray(x, np.float32)
        M = xv.shape[0]
        k = self.cfg.top_k
        y = np.zeros((M, self.cfg.hidden), np.float32)
        ids = np.zeros((M, k), np.int32)
        w = np.zeros((M, k), np.float32)
        mg = np.zeros(M, np.float32)
        lib().orc_moe_mlp(self.h, layer, _ptr(xv, C.c_float), M, _ptr(y, C.c_float), _ptr(ids, C.c_int32),
                          _ptr(w, C.c_float), _ptr(mg, C.c_float))
        return y, ids, w, mg

    def get_q4(self, tensor_id: int):
        wq, s, b = C.POINTER(C.c_uint32)(), C.POINTER(C.c_uint16)(), C.POINTER(C.c_uint16)()
        N, K = C.c_int(), C.c_int()
        lib().orc_model_get_q4(self.h, tensor_id, C.byref(wq), C.byref(s), C.byref(b),
                               C.byref(N), C.byref(K))
        N, K = N.value, K.value
        if N == 0:
            return None
        return (np.ctypeslib.as_array(wq, shape=(N, K // 8)).copy(),
                np.ctypeslib.as_array(s, shape=(N, K // 64)).copy(),
                np.ctypeslib.as_array(b, shape=(N, K // 64)).copy())

    def __del__(self):
        try:
            if self.h:
                lib().orc_model_free(self.h)
                self.h = None
        except Exception:
            pass


class KV:
    def __init__(self, model: Model, max_rows: int, max_len: int):
        self.h = lib().orc_kv_create(model.h, max_rows, max_len)
        self.max_rows = max_rows
        self.max_len = max_len

    def len(self, row):
        return lib().orc_kv_len(self.h, row)

    def set_len(self, row, n):
        lib().orc_kv_set_len(self.h, row, n)

    def trim(self, n):
        return lib().orc_kv_trim(self.h, n)

    def k(self, row, layer, n_kv, head_dim):
        p = lib().orc_kv_k(self.h, row, layer)
        return np.ctypeslib.as_array(p, shape=(n_kv, self.max_len, head_dim))

    def v(self, row, layer, n_kv, head_dim):
        p = lib().orc_kv_v(self.h, row, layer)
        return np.ctypeslib.as_array(p, shape=(n_kv, self.max_len, head_dim))

    def __del__(self):
        try:
            if self.h:
                lib().orc_kv_free(self.h)
                self.h = None
        except Exception:
            pass


def forward(model: Model, kv: KV, tokens, rows, pos, want_logits=True):
    t = np.ascontiguousarray(tokens, dtype=np.int32)
    r = np.ascontiguousarray(rows, dtype=np.int32)
    p = np.ascontiguousarray(pos, dtype=np.int32)
    M = len(t)
    logits = np.zeros((M, model.vocab), np.float32) if want_logits else None
    lib().orc_forward(model.h, kv.h, M, _ptr(t, C.c_int32), _ptr(r, C.c_int32),
                      _ptr(p, C.c_int32), _ptr(logits, C.c_float) if want_logits else None)
    return logits


class Generator:
    """Batched speculative decode on the CPU restatement (rows are slots)."""

    def __init__(self, model: Model, max_rows: int, max_len: int, spec: SpecConfig):
        self.model = model
        self.kv = KV(model, max_rows, max_len)
        self.rows = (Row * max_rows)()
        self.n_rows = max_rows
        self.spec = spec
        self.stats = Stats()
        self._hist_bufs = [None] * max_rows

    def admit(self, row: int, prompt, max_new: int, sp: Sampling, chunk: int = 256) -> int:
        cap = len(prompt) + max_new + 16
        buf = (C.c_int32 * cap)()
        self._hist_bufs[row] = buf
        R = self.rows[row]
        R.hist = C.cast(buf, C.POINTER(C.c_int32))
        R.hist_len = 0
        R.hist_cap = cap
        R.max_new = max_new
        R.sp = sp
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        return lib().orc_admit(self.model.h, self.kv.h, C.byref(R), row, _ptr(p, C.c_int32),
                               len(p), chunk)

    def set_row(self, row: int, history, n_gen: int, max_new: int, kv_len: int, sp: Sampling,
                active: bool = True):
        """Install a row's state without prefill (used to continue from a state
        produced elsewhere, e.g. copied from the device)."""
        cap = len(history) + max_new + 16
        buf = (C.c_int32 * cap)(*history)
        self._hist_bufs[row] = buf
        R = self.rows[row]
        R.hist = C.cast(buf, C.POINTER(C.c_int32))
        R.hist_len = len(history)
        R.hist_cap = cap
        R.n_gen = n_gen
        R.max_new = max_new
        R.active = int(active)
        R.sp = sp
        self.kv.set_len(row, kv_len)

    def step(self):
        K1 = self.spec.max_proposal + 1
        out = np.zeros((self.n_rows, K1), np.int32)
        n_out = np.zeros(self.n_rows, np.int32)
        lib().orc_spec_step(self.model.h, self.kv.h, self.rows, self.n_rows, C.byref(self.spec),
                            _ptr(out, C.c_int32), _ptr(n_out, C.c_int32), C.byref(self.stats))
        return [out[r, :n_out[r]].tolist() for r in range(self.n_rows)]

    def history(self, row):
        R = self.rows[row]
        return [R.hist[i] for i in range(R.hist_len)]

    def active(self, row):
        return bool(self.rows[row].active)
