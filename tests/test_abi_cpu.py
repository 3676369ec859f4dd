"""C-ABI checks that need no GPU: the library loads, exports every entry point
include/mlxcat_cuda.h declares, validates arguments before touching a device,
and the host mirror keeps the reference's configuration semantics."""
import ctypes as C
import os
import subprocess

import pytest

import mlxcat_b200 as M
from mlxcat_b200 import _abi as A

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def have_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def test_library_exports_every_header_function():
    declared = A.header_functions()
    assert len(declared) >= 30
    L = A.lib()
    for name in declared:
        assert hasattr(L, name), name
    assert sorted(A.PROTOTYPES) == declared
    out = subprocess.run(["nm", "-D", "--defined-only", A.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(declared) <= exported


def test_library_links_no_torch():
    out = subprocess.run(["ldd", A.LIB_PATH], capture_output=True, text=True).stdout
    assert "torch" not in out and "python" not in out


def test_invalid_config_rejected_before_device():
    cfg = M.ModelConfig(2, 500, 8, 2, 64, 1408, 32000)   # hidden not a multiple of 128
    h = C.c_void_p()
    c = cfg.to_c()
    rc = A.lib().mlxcat_ctx_create(C.byref(c), 0, C.byref(h))
    assert rc == A.E_INVALID
    assert b"multiple" in A.lib().mlxcat_op_last_error()
    c2 = M.TINY.to_c()
    c2.group_size = 32
    assert A.lib().mlxcat_ctx_create(C.byref(c2), 0, C.byref(h)) == A.E_INVALID


@pytest.mark.skipif(have_gpu(), reason="checks the no-device error path")
def test_no_device_fails_loudly():
    with pytest.raises(A.MlxcatError) as ei:
        M.Context(M.TINY, 0)
    assert ei.value.code == A.E_CUDA


def test_operator_argument_validation():
    L = A.lib()
    assert L.mlxcat_op_q4_linear(None, None, None, 128, 128, None, 1, None, None, 0, None) == A.E_INVALID
    assert L.mlxcat_op_q4_linear_workspace(128, 256, 4) >= 4 * 256 * 2
    assert L.mlxcat_op_attention_workspace(5, 5, 8, 2, 64, 600) > 0
    assert L.mlxcat_op_accept_workspace(8, 5) > 0
    # cache calls reject a null cache before any device work
    assert L.mlxcat_cache_filter(None, None, 0) == A.E_INVALID
    assert L.mlxcat_cache_trim_row(None, 0, 1, None) == A.E_INVALID
    # MoE operator: shapes outside the kernels' contract are refused up front
    assert L.mlxcat_op_moe_workspace(0, 2048, 768, 128, 8) == 0
    assert L.mlxcat_op_moe_workspace(320, 2048, 768, 128, 8) > 320 * 8 * 2048 * 4
    # tensor / expert parallel configurations are validated on the host
    h = C.c_void_p()
    bad = M.ModelConfig(2, 512, 8, 3, 64, 512, 4096, tp_size=2).to_c()      # 3 KV heads over 2 ranks
    assert L.mlxcat_ctx_create(C.byref(bad), 0, C.byref(h)) == A.E_INVALID
    bad = M.ModelConfig(2, 512, 8, 2, 64, 256, 4096, n_experts=32, top_k=4, ep_size=3).to_c()   # 32 % 3
    assert L.mlxcat_ctx_create(C.byref(bad), 0, C.byref(h)) == A.E_INVALID
    bad = M.ModelConfig(2, 512, 8, 2, 64, 256, 4096, n_experts=48, top_k=4).to_c()   # experts % 32
    assert L.mlxcat_ctx_create(C.byref(bad), 0, C.byref(h)) == A.E_INVALID


def test_spec_config_clamps_like_reference():
    # BatchGenerator.swift:16-27: maxProposal >= 0, maxSuffix >= 1, minContext >= 2
    s = M.SpeculativeDecodingConfiguration(True, -3, 0, 0)
    assert (s.max_proposal_tokens, s.max_suffix_tokens, s.min_context_tokens) == (0, 1, 2)
    d = M.SpeculativeDecodingConfiguration()
    assert (d.enabled, d.max_proposal_tokens, d.max_suffix_tokens, d.min_context_tokens) == (
        False, 4, 16, 8)
    with pytest.raises(ValueError):
        M.SpeculativeDecodingConfiguration(True, 99)


def test_baseline_configs_are_valid_shapes():
    for cfg in M.CONFIGS.values():
        c = cfg.to_c()
        for d in (c.hidden, c.intermediate, c.n_heads * c.head_dim, c.vocab):
            assert d % 128 == 0
        assert c.n_heads % c.n_kv_heads == 0


def test_ctypes_structs_match_the_header_layout(tmp_path):
    """Size and field offsets of every struct of the header, as the C compiler
    lays them out, equal the Python mirrors' (a Swift or ctypes binding reads
    the same bytes)."""
    structs = {"mlxcat_model_config": A.ModelConfigC, "mlxcat_sampling": A.SamplingC,
               "mlxcat_spec_config": A.SpecConfigC, "mlxcat_stats": A.StatsC, "mlxcat_rows": A.RowsC}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "mlxcat_cuda.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = {}
    for ln in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        cname, key, val = ln.split()
        got[(cname, key)] = int(val)
    for cname, py in structs.items():
        assert got[(cname, "size")] == C.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)


def test_oracle_structs_match_their_header(tmp_path):
    """The checker's own ctypes mirrors (oracle/oracle.py) against oracle.h."""
    from oracle import oracle as O
    structs = {"orc_config": O.Config, "orc_sampling": O.Sampling, "orc_spec_config": O.SpecConfig,
               "orc_stats": O.Stats, "orc_row": O.Row}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "oracle.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "olayout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "olayout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "oracle"), str(src), "-o", str(exe)], check=True)
    got = {}
    for ln in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        cname, key, val = ln.split()
        got[(cname, key)] = int(val)
    for cname, py in structs.items():
        assert got[(cname, "size")] == C.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)
