"""MLX checkpoint layout, no GPU: the safetensors container round trip, the
config.json mapping for the three model types on the path, and the tensor
names the loader expects (mlx-lm's module names)."""
import json

import numpy as np
import pytest

from mlxcat_b200 import checkpoint as K
from mlxcat_b200.engine import CONFIGS


def test_safetensors_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    t = {"a.weight": rng.integers(0, 2**32 - 1, size=(4, 8), dtype=np.uint32),
         "a.scales": rng.normal(size=(4, 1)).astype(np.float16),
         "n.weight": rng.normal(size=(7,)).astype(np.float32),
         "r.weight": rng.integers(0, 2**16 - 1, size=(3, 5), dtype=np.uint16)}
    p = tmp_path / "x.safetensors"
    K.write_safetensors(str(p), t, {"format": "mlx"}, bf16=("r.weight",))
    got, meta, dtypes = K.read_safetensors(str(p))
    assert meta == {"format": "mlx"}
    assert dtypes == {"a.weight": "U32", "a.scales": "F16", "n.weight": "F32", "r.weight": "BF16"}
    for k, v in t.items():
        np.testing.assert_array_equal(got[k], v)
    raw = p.read_bytes()
    n = int.from_bytes(raw[:8], "little")
    assert (8 + n) % 8 == 0 and json.loads(raw[8:8 + n])["a.weight"]["shape"] == [4, 8]


def test_truncated_file_is_rejected(tmp_path):
    p = tmp_path / "bad.safetensors"
    K.write_safetensors(str(p), {"w": np.zeros(16, np.float32)})
    p.write_bytes(p.read_bytes()[:-8])
    with pytest.raises(ValueError):
        K.read_safetensors(str(p))


@pytest.mark.parametrize("name", ["llama3-8b", "qwen3-4b", "qwen3-30b-a3b", "llama3-70b"])
def test_config_round_trip(name):
    cfg = CONFIGS[name]
    back = K.config_from_mlx(K.config_to_mlx(cfg), name=name)
    assert back == cfg


def test_config_rejects_other_quantizations():
    c = K.config_to_mlx(CONFIGS["llama3-8b"])
    c["quantization"] = {"group_size": 32, "bits": 4}
    with pytest.raises(ValueError):
        K.config_from_mlx(c)


def test_tensor_names_follow_mlx_lm():
    cfg = CONFIGS["qwen3-30b-a3b"]
    names = [n for n, *_ in K.q4_tensors(cfg)]
    assert names[0] == "model.embed_tokens" and names[-1] == "lm_head"
    assert "model.layers.3.self_attn.o_proj" in names and "model.layers.0.mlp.gate_proj" not in names
    norms = [n for n, *_ in K.norm_tensors(cfg)]
    assert "model.layers.47.self_attn.k_norm.weight" in norms and norms[-1] == "model.norm.weight"
    dense = [n for n, *_ in K.q4_tensors(CONFIGS["llama3-8b"])]
    assert "model.layers.31.mlp.down_proj" in dense and len(dense) == 1 + 32 * 7 + 1


def test_scale_conversion_from_bf16():
    f = np.array([1.5e-3, -2.25, 0.0], np.float32)
    bits = K._bf16_bits(f)
    h = K._f16(bits, "BF16").view(np.float16).astype(np.float32)
    np.testing.assert_allclose(h, f, rtol=8e-3)
