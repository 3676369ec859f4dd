"""ctypes declarations of the C ABI in include/mlxcat_cuda.h.

The shared library is built in-tree (``mlxcat_b200/libmlxcat_cuda.so``).  There
is no fallback: if the library is missing or a call fails, an exception is
raised.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmlxcat_cuda.so")

OK = 0
E_INVALID = -1
E_CUDA = -2
E_OOM = -3
E_STATE = -4

MODEL_TRANSFORMER = 0
MODEL_TABLE = 1
ACCEPT_COMPAT = 0
ACCEPT_PREFIX = 1
MAX_PROPOSAL = 8
MAX_EOS = 8
GEMM_STORE, GEMM_ADD, GEMM_SWIGLU = 0, 1, 2
TENSOR_EMBED = 0xFFFF0000
TENSOR_LM_HEAD = 0xFFFF0001


class ModelConfigC(C.Structure):
    _fields_ = [
        ("kind", C.c_int32), ("n_layers", C.c_int32), ("hidden", C.c_int32),
        ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32),
        ("intermediate", C.c_int32), ("vocab", C.c_int32), ("tie_embeddings", C.c_int32),
        ("qk_norm", C.c_int32), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
        ("group_size", C.c_int32), ("bits", C.c_int32),
        ("n_experts", C.c_int32), ("top_k", C.c_int32), ("norm_topk", C.c_int32),
        ("tp_size", C.c_int32), ("tp_rank", C.c_int32),
        ("ep_size", C.c_int32), ("ep_rank", C.c_int32),
    ]


class SamplingC(C.Structure):
    _fields_ = [
        ("temperature", C.c_float), ("top_p", C.c_float), ("seed", C.c_uint64),
        ("has_seed", C.c_int32), ("eos", C.c_int32 * MAX_EOS), ("n_eos", C.c_int32),
        ("trigger", C.c_int32),
    ]


class SpecConfigC(C.Structure):
    _fields_ = [
        ("mode", C.c_int32), ("enabled", C.c_int32), ("max_proposal", C.c_int32),
        ("max_suffix", C.c_int32), ("min_context", C.c_int32),
    ]


class StatsC(C.Structure):
    _fields_ = [
        ("proposed", C.c_int64), ("accepted", C.c_int64),
        ("proposal_batches", C.c_int64), ("rejected_batches", C.c_int64),
    ]


class RowsC(C.Structure):
    _fields_ = [
        ("hist", C.c_void_p), ("hist_cap", C.c_int32), ("rows", C.c_int32),
        ("hist_len", C.c_void_p), ("kv_len", C.c_void_p), ("n_gen", C.c_void_p),
        ("max_new", C.c_void_p), ("active", C.c_void_p), ("temperature", C.c_void_p),
        ("top_p", C.c_void_p), ("seed", C.c_void_p), ("has_seed", C.c_void_p),
        ("eos", C.c_void_p), ("n_eos", C.c_void_p), ("trigger", C.c_void_p),
    ]


# name -> (restype, argtypes)
_vp, _i32, _u32, _u64, _f32, _sz = C.c_void_p, C.c_int32, C.c_uint32, C.c_uint64, C.c_float, C.c_size_t
_vp3 = C.c_void_p * 3   # const T *const [3]: gate, up, down
PROTOTYPES = {
    "mlxcat_ctx_create": (C.c_int, [C.POINTER(ModelConfigC), _i32, C.POINTER(_vp)]),
    "mlxcat_ctx_destroy": (C.c_int, [_vp]),
    "mlxcat_tp_unique_id": (C.c_int, [_vp]),
    "mlxcat_ctx_tp_connect": (C.c_int, [_vp, _vp]),
    "mlxcat_last_error": (C.c_char_p, [_vp]),
    "mlxcat_ctx_stream": (C.c_int, [_vp, C.POINTER(_vp)]),
    "mlxcat_ctx_synchronize": (C.c_int, [_vp]),
    "mlxcat_ctx_launch_count": (C.c_int64, [_vp]),
    "mlxcat_weights_synth": (C.c_int, [_vp, _u64, _f32]),
    "mlxcat_weights_set_q4": (C.c_int, [_vp, _u32, _vp, _vp, _vp]),
    "mlxcat_weights_get_q4": (C.c_int, [_vp, _u32, _vp, _vp, _vp]),
    "mlxcat_weights_set_table": (C.c_int, [_vp, _vp, _i32]),
    "mlxcat_weights_set_bf16": (C.c_int, [_vp, _u32, _vp]),
    "mlxcat_weights_get_bf16": (C.c_int, [_vp, _u32, _vp]),
    "mlxcat_weights_set_norm": (C.c_int, [_vp, _u32, _vp]),
    "mlxcat_weights_bytes": (C.c_int64, [_vp]),
    "mlxcat_cache_create": (C.c_int, [_vp, _i32, _i32, C.POINTER(_vp)]),
    "mlxcat_cache_destroy": (C.c_int, [_vp]),
    "mlxcat_cache_peer_handle": (C.c_int, [_vp, _vp]),
    "mlxcat_cache_set_token_masks": (C.c_int, [_vp, _i32, _vp, _vp]),
    "mlxcat_cache_peer_connect": (C.c_int, [_vp, _vp]),
    "mlxcat_cache_insert_row": (C.c_int, [_vp, _i32, _vp, _i32, _i32, C.POINTER(SamplingC),
                                          C.POINTER(_i32)]),
    "mlxcat_op_dequant_q4": (C.c_int, [_vp, _vp, _vp, _i32, _i32, _vp, _vp]),
    "mlxcat_op_gemm_f16": (C.c_int, [_vp, _i32, _i32, _vp, _i32, _i32, _vp, _i32, _vp, _vp]),
    "mlxcat_cache_moe_routing": (C.c_int, [_vp, _i32, _vp, _vp, C.POINTER(_i32)]),
    "mlxcat_cache_insert_row_prefix": (C.c_int, [_vp, _i32, _vp, _i32, _i32, _vp, _vp, _i32,
                                                 C.POINTER(SamplingC), C.POINTER(_i32)]),
    "mlxcat_cache_remove_row": (C.c_int, [_vp, _i32]),
    "mlxcat_cache_filter": (C.c_int, [_vp, _vp, _i32]),
    "mlxcat_cache_trim_row": (C.c_int, [_vp, _i32, _i32, C.POINTER(_i32)]),
    "mlxcat_cache_trim": (C.c_int, [_vp, _i32, C.POINTER(_i32)]),
    "mlxcat_cache_lengths": (C.c_int, [_vp, _vp]),
    "mlxcat_cache_history": (C.c_int, [_vp, _i32, _vp, _i32, C.POINTER(_i32)]),
    "mlxcat_cache_extract_row": (C.c_int, [_vp, _i32, _i32, _vp, _vp]),
    "mlxcat_cache_active": (C.c_int, [_vp, _vp]),
    "mlxcat_draft": (C.c_int, [_vp, C.POINTER(SpecConfigC), _vp, _vp]),
    "mlxcat_verify_forward": (C.c_int, [_vp, C.POINTER(SpecConfigC), _vp]),
    "mlxcat_accept": (C.c_int, [_vp, C.POINTER(SpecConfigC), _vp, _vp, _vp, C.POINTER(StatsC)]),
    "mlxcat_spec_step": (C.c_int, [_vp, C.POINTER(SpecConfigC), _vp, _vp, _vp, C.POINTER(StatsC)]),
    "mlxcat_last_verify_ms": (C.c_int, [_vp, C.POINTER(_f32)]),
    "mlxcat_last_step_ms": (C.c_int, [_vp, C.POINTER(_f32)]),
    "mlxcat_cache_set_profiling": (C.c_int, [_vp, _i32]),
    "mlxcat_cache_profile": (C.c_int, [_vp, C.POINTER(_f32), C.POINTER(_f32), C.POINTER(_i32),
                                       C.POINTER(_i32)]),
    "mlxcat_op_last_error": (C.c_char_p, []),
    "mlxcat_op_q4_linear_workspace": (_sz, [_i32, _i32, _i32]),
    "mlxcat_op_q4_linear": (C.c_int, [_vp, _vp, _vp, _i32, _i32, _vp, _i32, _vp, _vp, _sz, _vp]),
    "mlxcat_op_attention_workspace": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "mlxcat_op_prefill_attention": (C.c_int, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp,
                                              _vp, _vp]),
    "mlxcat_op_attention": (C.c_int, [_vp, _vp, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
                                      _vp, _vp, _sz, _vp]),
    "mlxcat_op_attention_noalloc": (C.c_int, [_vp, _vp, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _i32,
                                              _i32, _vp, _vp]),
    "mlxcat_op_synth_q4": (C.c_int, [_u64, _u32, _f32, _i32, _i32, _vp, _vp, _vp, _vp]),
    "mlxcat_op_moe_workspace": (_sz, [_i32, _i32, _i32, _i32, _i32]),
    "mlxcat_op_moe": (C.c_int, [_vp, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp3, _vp3, _vp3,
                                _vp, _vp, _vp, _vp, _sz, _vp]),
    "mlxcat_op_draft": (C.c_int, [C.POINTER(RowsC), C.POINTER(SpecConfigC), _vp, _vp, _vp, _vp, _vp]),
    "mlxcat_op_accept_workspace": (_sz, [_i32, _i32]),
    "mlxcat_op_accept": (C.c_int, [C.POINTER(RowsC), C.POINTER(SpecConfigC), _vp, _vp, _vp, _i32,
                                   _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
}

_lib = None


class MlxcatError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"mlxcat error {code}: {msg}")
        self.code = code


def lib():
    """Load libmlxcat_cuda.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run __graft_entry__.build() "
                          "(there is no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    for name, (res, args) in PROTOTYPES.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def check(rc: int, ctx=None):
    if rc != OK:
        L = lib()
        msg = (L.mlxcat_last_error(ctx) if ctx else L.mlxcat_op_last_error()) or b""
        raise MlxcatError(rc, msg.decode(errors="replace"))
    return rc


def header_functions(header_path: str | None = None):
    """Names of every entry point declared in include/mlxcat_cuda.h."""
    import re
    if header_path is None:
        header_path = os.path.join(os.path.dirname(HERE), "include", "mlxcat_cuda.h")
    text = open(header_path).read()
    return sorted(set(re.findall(r"MLXCAT_API\s+[\w\s\*]+?\b(mlxcat_\w+)\s*\(", text)))
