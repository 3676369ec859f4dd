"""Host-side mirror of mlxcat's Track-B surface over the C ABI.

Names, argument meaning and error behaviour follow the Swift types of the
reference so that callers (and the parity tests) read like mlxcat's own:

* ``SpeculativeDecodingConfiguration`` / ``SpeculativeDecodingStats``
  -- Sources/MLXCat/TrackB/BatchGenerator.swift:10-38
* ``SamplingParameters`` (path subset) -- Sampling.swift:139-217
* ``Request`` / ``Response`` / ``FinishReason`` -- Request.swift,
  BatchGenerator.swift:40-67
* ``ContinuousBatchGenerator`` (insert / next / remove) -- BatchGenerator.swift:144-1035
* ``BatchKVCache`` (lengths / trim / extract) -- BatchCache.swift:37-433
* ``Scheduler`` (submit / step / is_idle / stats) -- Scheduler.swift:13-476

All arithmetic runs on the device inside libmlxcat_cuda.so; this module only
moves plain integers across the ABI.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import weakref
from collections import OrderedDict, deque
from typing import Dict, List, Optional

import numpy as np

from . import _abi as A


# --------------------------------------------------------------------------- #
# configuration types
# --------------------------------------------------------------------------- #
@dataclasses.dataclass(frozen=True)
class ModelConfig:
    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    tie_embeddings: bool = True
    qk_norm: bool = False
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    kind: int = A.MODEL_TRANSFORMER
    name: str = "custom"
    # sparse MoE MLP (Qwen3-MoE): experts per layer, experts per token,
    # renormalised routing weights; `intermediate` is then the expert width
    n_experts: int = 0
    top_k: int = 0
    norm_topk: bool = True
    # tensor parallelism: this context is rank tp_rank of tp_size (1 = off)
    tp_size: int = 1
    tp_rank: int = 0
    # expert parallelism (MoE): rank ep_rank of ep_size holds 1/ep_size of the experts
    ep_size: int = 1
    ep_rank: int = 0

    def to_c(self) -> A.ModelConfigC:
        return A.ModelConfigC(self.kind, self.n_layers, self.hidden, self.n_heads, self.n_kv_heads,
                              self.head_dim, self.intermediate, self.vocab, int(self.tie_embeddings),
                              int(self.qk_norm), self.rms_eps, self.rope_theta, 64, 4,
                              self.n_experts, self.top_k, int(self.norm_topk), self.tp_size, self.tp_rank,
                              self.ep_size, self.ep_rank)

    @staticmethod
    def table(vocab: int) -> "ModelConfig":
        return ModelConfig(0, 0, 0, 0, 0, 0, vocab, kind=A.MODEL_TABLE, name="table")


# The BASELINE configurations (architectures only).
TINY = ModelConfig(4, 512, 8, 2, 64, 1408, 32000, True, False, 1e-5, 500000.0, name="tiny-llama")
QWEN3_4B = ModelConfig(36, 2560, 32, 8, 128, 9728, 151936, True, True, 1e-6, 1e6, name="qwen3-4b")
LLAMA3_8B = ModelConfig(32, 4096, 32, 8, 128, 14336, 128256, False, False, 1e-5, 500000.0,
                        name="llama3-8b")
LLAMA3_70B = ModelConfig(80, 8192, 64, 8, 128, 28672, 128256, False, False, 1e-5, 500000.0,
                         name="llama3-70b")
QWEN3_30B_A3B = ModelConfig(48, 2048, 32, 4, 128, 768, 151936, False, True, 1e-6, 1e6,
                            name="qwen3-30b-a3b", n_experts=128, top_k=8, norm_topk=True)
CONFIGS = {c.name: c for c in (TINY, QWEN3_4B, LLAMA3_8B, QWEN3_30B_A3B, LLAMA3_70B)}


@dataclasses.dataclass
class SpeculativeDecodingConfiguration:
    """BatchGenerator.swift:10-29 (defaults and clamping as there) + mode."""
    enabled: bool = False
    max_proposal_tokens: int = 4
    max_suffix_tokens: int = 16
    min_context_tokens: int = 8
    mode: int = A.ACCEPT_COMPAT

    def __post_init__(self):
        self.max_proposal_tokens = max(0, self.max_proposal_tokens)
        self.max_suffix_tokens = max(1, self.max_suffix_tokens)
        self.min_context_tokens = max(2, self.min_context_tokens)
        if self.max_proposal_tokens > A.MAX_PROPOSAL:
            raise ValueError(f"max_proposal_tokens <= {A.MAX_PROPOSAL} on this path")

    def to_c(self) -> A.SpecConfigC:
        return A.SpecConfigC(self.mode, int(self.enabled), self.max_proposal_tokens,
                             self.max_suffix_tokens, self.min_context_tokens)


SpeculativeDecodingConfiguration.disabled = SpeculativeDecodingConfiguration(enabled=False)


@dataclasses.dataclass
class SpeculativeDecodingStats:
    proposed_token_count: int = 0
    accepted_token_count: int = 0
    proposal_batch_count: int = 0
    rejected_batch_count: int = 0


@dataclasses.dataclass
class SamplingParameters:
    """Subset of Sampling.swift:139-217 that the speculative path supports."""
    temperature: float = 0.0
    top_p: float = 0.0
    seed: Optional[int] = None
    eos_token_ids: tuple = ()
    tool_call_start_token_id: Optional[int] = None

    def to_c(self, default_seed: int = 0) -> A.SamplingC:
        s = A.SamplingC()
        s.temperature = self.temperature
        s.top_p = self.top_p
        s.seed = (self.seed if self.seed is not None else default_seed) & 0xFFFFFFFFFFFFFFFF
        s.has_seed = 0 if self.seed is None else 1
        eos = list(self.eos_token_ids)
        if len(eos) > A.MAX_EOS:
            raise ValueError("at most 8 EOS ids")
        for i, e in enumerate(eos):
            s.eos[i] = e
        s.n_eos = len(eos)
        s.trigger = -1 if self.tool_call_start_token_id is None else self.tool_call_start_token_id
        return s


class FinishReason:
    STOP = "stop"
    LENGTH = "length"
    CANCELLED = "cancelled"

    @staticmethod
    def failed(msg: str) -> str:
        return f"failed: {msg}"


@dataclasses.dataclass
class Response:
    uid: str
    token: int
    finish_reason: Optional[str] = None


@dataclasses.dataclass
class Request:
    uid: str
    tokens: List[int]
    max_tokens: int
    sampling: SamplingParameters = dataclasses.field(default_factory=SamplingParameters)


# --------------------------------------------------------------------------- #
# context / cache
# --------------------------------------------------------------------------- #
def allowed_next_token_ids(allowed_sequences, generated_tokens) -> Optional[List[int]]:
    """TokenSampler.allowedNextTokenIDs (Sources/MLXCat/TrackB/Sampling.swift:529-546):
    the next tokens of every allowed sequence that the generated tokens are a
    strict prefix of, sorted; None when there are no sequences or none of them
    continues (no constraint)."""
    if not allowed_sequences:
        return None
    g = list(generated_tokens)
    allowed = set()
    for seq in allowed_sequences:
        if len(g) >= len(seq) or list(seq[:len(g)]) != g:
            continue
        allowed.add(int(seq[len(g)]))
    return sorted(allowed) if allowed else None


def speculative_token_masks(row: int, allowed_sequences, generated_tokens, drafts) -> Dict:
    """The allowed sets of one choice-constrained row at each verify position:
    position p follows the generated tokens and drafts[:p] (what the row will
    have generated if the drafts before p are accepted).  The result feeds
    BatchKVCache.set_token_masks; unconstrained positions are left out."""
    out = {}
    for p in range(len(drafts) + 1):
        ids = allowed_next_token_ids(allowed_sequences, list(generated_tokens) + list(drafts[:p]))
        if ids is not None:
            out[(row, p)] = ids
    return out


class Context:
    """One model on one device (mlxcat_ctx)."""

    def __init__(self, cfg: ModelConfig, device: int = 0):
        self.L = A.lib()
        self.cfg = cfg
        self._caches = weakref.WeakSet()   # mlxcat_ctx_destroy frees them too
        h = C.c_void_p()
        c = cfg.to_c()
        A.check(self.L.mlxcat_ctx_create(C.byref(c), device, C.byref(h)))
        self.h = h

    def check(self, rc):
        return A.check(rc, self.h)

    @staticmethod
    def tp_unique_id() -> bytes:
        """a fresh NCCL id for a tensor-parallel group (create on one rank)"""
        buf = (C.c_uint8 * 128)()
        A.check(A.lib().mlxcat_tp_unique_id(buf))
        return bytes(buf)

    def tp_connect(self, uid: bytes):
        """join the tensor-parallel group (collective over its tp_size ranks)"""
        buf = (C.c_uint8 * 128).from_buffer_copy(uid)
        self.check(self.L.mlxcat_ctx_tp_connect(self.h, buf))

    def synth_weights(self, seed: int, stddev: float = 0.02):
        self.check(self.L.mlxcat_weights_synth(self.h, seed, stddev))

    def set_table(self, next_tokens):
        n = np.ascontiguousarray(next_tokens, dtype=np.int32)
        self.check(self.L.mlxcat_weights_set_table(self.h, n.ctypes.data, len(n)))

    def set_q4(self, tensor_id: int, wq, scales, biases):
        wq = np.ascontiguousarray(wq, dtype=np.uint32)
        s = np.ascontiguousarray(scales, dtype=np.uint16)
        b = np.ascontiguousarray(biases, dtype=np.uint16)
        self.check(self.L.mlxcat_weights_set_q4(self.h, tensor_id, wq.ctypes.data, s.ctypes.data,
                                                b.ctypes.data))

    def set_bf16(self, tensor_id: int, w):
        w = np.ascontiguousarray(w, dtype=np.uint16)
        self.check(self.L.mlxcat_weights_set_bf16(self.h, tensor_id, w.ctypes.data))

    def get_bf16(self, tensor_id: int, shape):
        w = np.zeros(shape, np.uint16)
        self.check(self.L.mlxcat_weights_get_bf16(self.h, tensor_id, w.ctypes.data))
        return w

    NORM_FINAL = 0xFFFF0002

    @staticmethod
    def norm_id(layer: int, kind: int) -> int:
        """id of an RMSNorm weight: kind 0 input_layernorm, 1 post_attention_layernorm,
        2 q_norm, 3 k_norm"""
        return layer * 16 + 8 + kind

    def set_norm(self, norm_id: int, w):
        a = np.ascontiguousarray(w, dtype=np.float32)
        self.check(self.L.mlxcat_weights_set_norm(self.h, norm_id, a.ctypes.data))

    def get_q4(self, tensor_id: int, N: int, K: int):
        wq = np.zeros((N, K // 8), np.uint32)
        s = np.zeros((N, K // 64), np.uint16)
        b = np.zeros((N, K // 64), np.uint16)
        self.check(self.L.mlxcat_weights_get_q4(self.h, tensor_id, wq.ctypes.data, s.ctypes.data,
                                                b.ctypes.data))
        return wq, s, b

    def weights_bytes(self) -> int:
        return int(self.L.mlxcat_weights_bytes(self.h))

    def stream(self) -> int:
        s = C.c_void_p()
        self.check(self.L.mlxcat_ctx_stream(self.h, C.byref(s)))
        return s.value or 0

    def synchronize(self):
        self.check(self.L.mlxcat_ctx_synchronize(self.h))

    def launch_count(self) -> int:
        return int(self.L.mlxcat_ctx_launch_count(self.h))

    def close(self):
        if getattr(self, "h", None):
            for c in list(getattr(self, "_caches", ())):
                c.close()   # before the context: a cache uses its stream and buffers
            self.L.mlxcat_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BatchKVCache:
    """Device KV cache + per-row generator state (mlxcat_cache)."""

    def __init__(self, ctx: Context, max_rows: int, max_len: int):
        self.ctx = ctx
        self.L = ctx.L
        self.max_rows = max_rows
        self.max_len = max_len
        h = C.c_void_p()
        ctx.check(self.L.mlxcat_cache_create(ctx.h, max_rows, max_len, C.byref(h)))
        self.h = h
        ctx._caches.add(self)

    PEER_HANDLE_BYTES = 128

    def peer_handle(self) -> bytes:
        """This rank's expert- or tensor-parallel handle (mlxcat_cache_peer_handle):
        the bytes every other rank needs to map this cache's exchange region."""
        buf = (C.c_uint8 * self.PEER_HANDLE_BYTES)()
        self.ctx.check(self.L.mlxcat_cache_peer_handle(self.h, buf))
        return bytes(buf)

    def peer_connect(self, handles):
        """Map every rank's region (handles: one per rank, in rank order)."""
        if any(len(h) != self.PEER_HANDLE_BYTES for h in handles):
            raise ValueError(f"peer handles are {self.PEER_HANDLE_BYTES} bytes each")
        buf = (C.c_uint8 * (self.PEER_HANDLE_BYTES * len(handles))).from_buffer_copy(b"".join(handles))
        self.ctx.check(self.L.mlxcat_cache_peer_connect(self.h, buf))

    def set_token_masks(self, k: int, allowed):
        """Grammar masks for the next accept(): allowed maps (row, position) to
        the token ids the row's grammar allows at that verify position (after
        the drafts before it); positions not in the map are unconstrained."""
        V = self.ctx.cfg.vocab
        W = (V + 31) // 32
        bits = np.zeros((self.max_rows, k + 1, W), np.uint32)
        on = np.zeros((self.max_rows, k + 1), np.uint8)
        for (r, p), ids in allowed.items():
            on[r, p] = 1
            for t in ids:
                if 0 <= t < V:
                    bits[r, p, t >> 5] |= np.uint32(1 << (t & 31))
        self.ctx.check(self.L.mlxcat_cache_set_token_masks(self.h, k, bits.ctypes.data, on.ctypes.data))

    def clear_token_masks(self):
        self.ctx.check(self.L.mlxcat_cache_set_token_masks(self.h, 0, None, None))

    def insert_row(self, row: int, prompt, max_new_tokens: int, sampling: SamplingParameters,
                   default_seed: int = 0) -> int:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        sp = sampling.to_c(default_seed)
        first = C.c_int32()
        self.ctx.check(self.L.mlxcat_cache_insert_row(self.h, row, p.ctypes.data, len(p), max_new_tokens,
                                                      C.byref(sp), C.byref(first)))
        return first.value

    def insert_row_prefix(self, row: int, prompt, k_prefix, v_prefix, max_new_tokens: int,
                          sampling: SamplingParameters, default_seed: int = 0) -> int:
        """Admission on a prefix-cache hit (Scheduler.prepareHitRow): k_prefix,
        v_prefix fp16 [n_layers][n_kv_heads][prefix_len][head_dim] hold the KV of
        the first prefix_len prompt tokens; the rest of the prompt is prefilled."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        k = np.ascontiguousarray(k_prefix, dtype=np.float16)
        v = np.ascontiguousarray(v_prefix, dtype=np.float16)
        if k.shape != v.shape or k.ndim != 4:
            raise ValueError("k_prefix / v_prefix must both be [n_layers][n_kv_heads][prefix_len][head_dim]")
        sp = sampling.to_c(default_seed)
        first = C.c_int32()
        self.ctx.check(self.L.mlxcat_cache_insert_row_prefix(self.h, row, p.ctypes.data, len(p), k.shape[2],
                                                             k.ctypes.data, v.ctypes.data, max_new_tokens,
                                                             C.byref(sp), C.byref(first)))
        return first.value

    def remove_row(self, row: int):
        self.ctx.check(self.L.mlxcat_cache_remove_row(self.h, row))

    def filter(self, keep):
        """BatchKVCache.filter(keeping:): rows not in keep are removed (slots are kept)"""
        k = np.ascontiguousarray(list(keep), dtype=np.int32)
        self.ctx.check(self.L.mlxcat_cache_filter(self.h, k.ctypes.data if len(k) else None, len(k)))

    def trim_row(self, row: int, n: int) -> int:
        t = C.c_int32()
        self.ctx.check(self.L.mlxcat_cache_trim_row(self.h, row, n, C.byref(t)))
        return t.value

    def trim(self, n: int) -> int:
        t = C.c_int32()
        self.ctx.check(self.L.mlxcat_cache_trim(self.h, n, C.byref(t)))
        return t.value

    def lengths(self) -> List[int]:
        out = np.zeros(self.max_rows, np.int32)
        self.ctx.check(self.L.mlxcat_cache_lengths(self.h, out.ctypes.data))
        return out.tolist()

    def active(self) -> List[bool]:
        out = np.zeros(self.max_rows, np.int32)
        self.ctx.check(self.L.mlxcat_cache_active(self.h, out.ctypes.data))
        return [bool(x) for x in out]

    def history(self, row: int) -> List[int]:
        n = C.c_int32()
        self.ctx.check(self.L.mlxcat_cache_history(self.h, row, None, 0, C.byref(n)))
        out = np.zeros(max(n.value, 1), np.int32)
        self.ctx.check(self.L.mlxcat_cache_history(self.h, row, out.ctypes.data, n.value, C.byref(n)))
        return out[:n.value].tolist()

    def extract_row(self, row: int, layer: int):
        cfg = self.ctx.cfg
        L = self.lengths()[row]
        k = np.zeros((cfg.n_kv_heads, L, cfg.head_dim), np.float16)
        v = np.zeros_like(k)
        self.ctx.check(self.L.mlxcat_cache_extract_row(self.h, row, layer, k.ctypes.data, v.ctypes.data))
        return k, v

    def moe_routing(self, layer: int):
        """(expert ids, weights) [M][top_k] of `layer` in the last forward (MoE models)"""
        tk = self.ctx.cfg.top_k
        m = C.c_int32()
        self.ctx.check(self.L.mlxcat_cache_moe_routing(self.h, layer, None, None, C.byref(m)))
        ids = np.zeros((m.value, tk), np.int32)
        w = np.zeros((m.value, tk), np.float32)
        self.ctx.check(self.L.mlxcat_cache_moe_routing(self.h, layer, ids.ctypes.data, w.ctypes.data,
                                                       C.byref(m)))
        return ids, w

    def draft(self, spec: SpeculativeDecodingConfiguration):
        k = spec.max_proposal_tokens if spec.enabled else 0
        d = np.zeros((self.max_rows, max(k, 1)), np.int32)
        cnt = np.zeros(self.max_rows, np.int32)
        sc = spec.to_c()
        self.ctx.check(self.L.mlxcat_draft(self.h, C.byref(sc), d.ctypes.data, cnt.ctypes.data))
        return [d[r, :cnt[r]].tolist() for r in range(self.max_rows)]

    def verify_forward(self, spec: SpeculativeDecodingConfiguration, want_logits=True):
        k = spec.max_proposal_tokens if spec.enabled else 0
        sc = spec.to_c()
        logits = np.zeros((self.max_rows, k + 1, self.ctx.cfg.vocab), np.float32) if want_logits else None
        self.ctx.check(self.L.mlxcat_verify_forward(self.h, C.byref(sc),
                                                    logits.ctypes.data if want_logits else None))
        return logits

    def accept(self, spec: SpeculativeDecodingConfiguration):
        return self._step(self.L.mlxcat_accept, spec)

    def spec_step(self, spec: SpeculativeDecodingConfiguration):
        return self._step(self.L.mlxcat_spec_step, spec)

    def _step(self, fn, spec):
        k = spec.max_proposal_tokens if spec.enabled else 0
        tok = np.zeros((self.max_rows, k + 1), np.int32)
        n = np.zeros(self.max_rows, np.int32)
        fin = np.zeros(self.max_rows, np.int32)
        st = A.StatsC()
        sc = spec.to_c()
        self.ctx.check(fn(self.h, C.byref(sc), tok.ctypes.data, n.ctypes.data, fin.ctypes.data,
                          C.byref(st)))
        stats = SpeculativeDecodingStats(st.proposed, st.accepted, st.proposal_batches,
                                         st.rejected_batches)
        return tok, n, fin, stats

    def set_profiling(self, enabled: bool):
        self.ctx.check(self.L.mlxcat_cache_set_profiling(self.h, int(enabled)))

    def profile(self):
        """(q4 linear ms, attention ms, q4 launches, attention launches) of the last step."""
        a, b = C.c_float(), C.c_float()
        na, nb = C.c_int32(), C.c_int32()
        self.ctx.check(self.L.mlxcat_cache_profile(self.h, C.byref(a), C.byref(b), C.byref(na),
                                                   C.byref(nb)))
        return a.value, b.value, na.value, nb.value

    def last_verify_ms(self) -> float:
        ms = C.c_float()
        self.ctx.check(self.L.mlxcat_last_verify_ms(self.h, C.byref(ms)))
        return ms.value

    def last_step_ms(self) -> float:
        ms = C.c_float()
        self.ctx.check(self.L.mlxcat_last_step_ms(self.h, C.byref(ms)))
        return ms.value

    def close(self):
        # a context that was closed first has destroyed this cache already
        if getattr(self, "h", None) and getattr(self.ctx, "h", None):
            self.L.mlxcat_cache_destroy(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# --------------------------------------------------------------------------- #
# generator / scheduler
# --------------------------------------------------------------------------- #
class ContinuousBatchGenerator:
    """Rows of a device BatchKVCache, addressed by request uid.

    ``next()`` runs one speculative step for every row at once (the reference
    speculates at width 1 only, BatchGenerator.swift:959; ``mode=ACCEPT_COMPAT``
    keeps exactly that gate) and returns the emitted tokens as Responses."""

    def __init__(self, ctx: Context, max_rows: int, max_len: int,
                 speculative_decoding: SpeculativeDecodingConfiguration = None,
                 base_seed: int = 0):
        self.ctx = ctx
        self.cache = BatchKVCache(ctx, max_rows, max_len)
        self.spec = speculative_decoding or SpeculativeDecodingConfiguration.disabled
        self.base_seed = base_seed
        self.row_of: "OrderedDict[str, int]" = OrderedDict()
        self.free = list(range(max_rows))
        self.stats = SpeculativeDecodingStats()
        self.decode_calls = 0

    @property
    def row_uids(self):
        return list(self.row_of.keys())

    def insert(self, uid: str, prompt, max_tokens: int, sampling: SamplingParameters) -> Response:
        if uid in self.row_of:
            raise ValueError(f"uid {uid} already running")
        if not self.free:
            raise RuntimeError("no free row")
        row = self.free.pop(0)
        first = self.cache.insert_row(row, prompt, max_tokens, sampling,
                                      default_seed=self.base_seed + row)
        self.row_of[uid] = row
        return Response(uid, first)

    def remove(self, uid: str):
        row = self.row_of.pop(uid, None)
        if row is not None:
            self.cache.remove_row(row)
            self.free.append(row)
            self.free.sort()

    def next(self) -> List[Response]:
        if not self.row_of:
            return []
        tok, n, fin, stats = self.cache.spec_step(self.spec)
        self.decode_calls += 1
        self.stats = stats
        out = []
        for uid, row in self.row_of.items():
            for i in range(int(n[row])):
                out.append(Response(uid, int(tok[row, i])))
        return out


class Scheduler:
    """Admission + step loop (Scheduler.swift:310-434, 599-668)."""

    def __init__(self, ctx: Context, max_concurrent_requests: int, max_len: int,
                 speculative_decoding: SpeculativeDecodingConfiguration = None, base_seed: int = 0):
        self.generator = ContinuousBatchGenerator(ctx, max_concurrent_requests, max_len,
                                                  speculative_decoding, base_seed)
        self.waiting: deque = deque()
        self.running: Dict[str, dict] = {}

    def submit(self, request: Request):
        self.waiting.append(request)

    @property
    def is_idle(self) -> bool:
        return not self.waiting and not self.running

    @property
    def speculative_decoding_stats(self) -> SpeculativeDecodingStats:
        return self.generator.stats

    def _finish(self, req: Request, token: int, count: int) -> Optional[str]:
        if token in req.sampling.eos_token_ids:
            return FinishReason.STOP
        if count >= req.max_tokens:
            return FinishReason.LENGTH
        return None

    def admit_waiting(self) -> List[Response]:
        """Admit waiting requests into free rows (Scheduler.admitWaiting /
        completeAdmission, Scheduler.swift:478, 599-668): prefill, first token."""
        out: List[Response] = []
        while self.waiting and self.generator.free:
            req = self.waiting.popleft()
            try:
                r = self.generator.insert(req.uid, req.tokens, req.max_tokens, req.sampling)
            except A.MlxcatError as e:
                out.append(Response(req.uid, -1, FinishReason.failed(str(e))))
                continue
            fr = self._finish(req, r.token, 1)
            out.append(Response(req.uid, r.token, fr))
            if fr:
                self.generator.remove(req.uid)
            else:
                self.running[req.uid] = {"req": req, "count": 1}
        return out

    def step(self) -> List[Response]:
        """One scheduler step: admissions, then one (speculative) decode step
        over every running row."""
        out = self.admit_waiting()
        if not self.running:
            return out
        finished = []
        for r in self.generator.next():
            st = self.running.get(r.uid)
            if st is None or r.uid in finished:
                continue
            st["count"] += 1
            fr = self._finish(st["req"], r.token, st["count"])
            out.append(Response(r.uid, r.token, fr))
            if fr:
                finished.append(r.uid)
        for uid in finished:
            self.generator.remove(uid)
            self.running.pop(uid, None)
        return out
