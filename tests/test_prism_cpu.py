"""Prism Hadamard checkpoints on CPU: the block Walsh-Hadamard transform
against scipy's Sylvester matrix, the module transforms of the reference's
synthetic artifact (Tests/MLXLMTests/Kernel/Cache/
PrismHadamardCheckpointKernelTests.swift), the artifact checks, and a whole
packed hybrid model against its dense equivalent."""
import copy
import json
import math
import os

import pytest
import torch
from scipy.linalg import hadamard

from mlx_swift_lm_b200 import DecoderLM
from mlx_swift_lm_b200.loader import prism
from mlx_swift_lm_b200.loader.load import CheckpointView, build_from_tensors, load_model
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.ops.rotation import HadamardTransform
from mlx_swift_lm_b200 import ops


def test_block_hadamard_matches_sylvester_matrix():
    torch.manual_seed(0)
    b, K = 64, 256
    s = (torch.randint(0, 2, (K,)) * 2 - 1).float()
    x = torch.randn(5, K, dtype=torch.float64)
    H = torch.tensor(hadamard(b), dtype=torch.float64) / math.sqrt(b)
    want = torch.cat([(x[:, i:i + b] * s[i:i + b].double()) @ H for i in range(0, K, b)], 1)
    tr = HadamardTransform(b, s)
    got = tr.rotate(x)
    assert torch.allclose(got, want, atol=1e-12)
    assert torch.allclose(tr.inverse(got), x, atol=1e-12)


SIGNS = [(-1.0 if i % 3 == 0 else 1.0) for i in range(512)]


def _config(**edit):
    c = {"schema_version": 2, "model_type": "prism_hadamard_qwen35", "base_model_type": "qwen3_5",
         "gdn_activation_layout": "grouped", "tensor_namespace": "mlx-vlm-qwen3_5", "hadamard_config": "hadamard.json",
         "components": {"text": True, "vision": False, "mtp": False},
         "quantization": {"bits": 2, "group_size": 128, "mode": "affine"},
         "text_config": {"mtp_num_hidden_layers": 0},
         "modules": [{"path": "model.embed_tokens", "block": 512, "embedding": True, "dtype": "float16"},
                     {"path": "lm_head", "block": 512, "embedding": False, "dtype": "float16"}]}
    c.update(edit)
    return c


def _meta(**edit):
    m = {"prism.hadamard.version": 1, "prism.hadamard.block_size": 512,
         "prism.hadamard.transform": "normalized-sylvester-walsh-hadamard",
         "prism.hadamard.axis": "input-last-dimension", "prism.hadamard.sign_mode": "explicit",
         "prism.hadamard.weight_names": ["language_model.lm_head.weight"],
         "prism.hadamard.inverse_weight_names": ["language_model.model.embed_tokens.weight"],
         "prism.hadamard.sign_widths": [512], "prism.hadamard.sign_values": SIGNS,
         "prism.hadamard.gdn_v_grouped": True}
    m.update(edit)
    return m


def _weights():
    """4 rows x 512 columns per module: codes 0, scales 1, row r bias r + 1."""
    w = {"language_model.model.layers.0.input_layernorm.weight": torch.ones(8),
         "language_model.model.layers.0.post_attention_layernorm.weight": torch.ones(8)}
    biases = torch.tensor([float(i // 4 + 1) for i in range(16)]).reshape(4, 4).half()
    for p in ("model.embed_tokens", "lm_head"):
        n = "language_model." + p
        w[n + ".weight"] = torch.zeros(4, 32, dtype=torch.int32)
        w[n + ".scales"] = torch.ones(4, 4, dtype=torch.float16)
        w[n + ".biases"] = biases.clone()
        w[n + ".signs"] = torch.tensor(SIGNS)
    return w


def test_installed_modules_apply_exact_transforms():
    info = prism.parse_config(_config())
    meta = prism.HadamardMetadata(_meta())
    w = _weights()
    prism.validate(info, meta, w)
    ck = CheckpointView(w, {"bits": 2, "group_size": 128, "mode": "affine"}, torch.float32, keep_quantized=True,
                        hadamard=meta)
    root = math.sqrt(512)
    emb = ck.embedding("embed_tokens")
    rows = emb[torch.tensor([2, 0])]
    # equal values v -> v * sqrt(512) at column 0 (then sign 0 = -1), exact zeros elsewhere
    assert abs(rows[0, 0] + 3 * root) < 1e-4 and abs(rows[1, 0] + root) < 1e-4
    assert torch.all(rows[:, 1:] == 0)
    head = ck.linear("lm_head")
    out = ops.gemm(torch.tensor(SIGNS)[None], head, epi="f32")
    assert out.shape == (1, 4)
    assert torch.allclose(out[0], torch.arange(1, 5).float() * root, atol=1e-3)


@pytest.mark.parametrize("edit,detail", [
    ({"gdn_activation_layout": "tiled"}, "unsupported architecture/packing contract"),
    ({"hadamard_config": "../hadamard.json"}, "unsupported architecture/packing contract"),
    ({"quantization": {"bits": 4, "group_size": 128, "mode": "affine"}}, "unsupported architecture/packing contract"),
    ({"text_config": {"num_experts": 8}}, "unsupported architecture/packing contract"),
    ({"modules": [{"path": "model.embed_tokens", "block": 256, "embedding": True, "dtype": "float16"}]},
     "invalid packed module declarations"),
    ({"modules": [{"path": "lm_head", "block": 512, "embedding": False, "dtype": "float16"}]},
     "invalid packed module declarations"),
    ({"modules": [{"path": "model..x", "block": 512, "embedding": False, "dtype": "float16"},
                  {"path": "model.embed_tokens", "block": 512, "embedding": True, "dtype": "float16"}]},
     "invalid packed module declarations"),
])
def test_rejects_other_contracts(edit, detail):
    with pytest.raises(prism.PrismCheckpointError) as e:
        prism.parse_config(_config(**edit))
    assert e.value.detail == detail
    assert str(e.value) == f"Invalid Prism Hadamard checkpoint: {detail}"


def _edit_weights(fn):
    w = _weights()
    fn(w)
    return w


LM = "language_model.lm_head"


@pytest.mark.parametrize("meta_edit,weights_edit,detail", [
    ({}, lambda w: w.__setitem__("language_model.model.layers.0.input_layernorm.weight", torch.ones(8).half()),
     "schema-2 native state requires the published FP32 normalizers"),
    ({"prism.hadamard.gdn_v_grouped": False}, None, "transform manifest disagrees with tensors"),
    ({"prism.hadamard.weight_names": ["language_model.model.other.weight"]}, None,
     "transform manifest disagrees with tensors"),
    ({"prism.hadamard.inverse_weight_names": []}, None, "transform manifest disagrees with tensors"),
    ({}, lambda w: w.__setitem__("language_model.model.extra.signs", torch.tensor(SIGNS)),
     "transform manifest disagrees with tensors"),
    ({}, lambda w: w.pop(LM + ".signs"), "transform manifest disagrees with tensors"),
    ({}, lambda w: w.__setitem__(LM + ".signs", torch.tensor(SIGNS).int()), "packed tensor shape/dtype mismatch"),
    ({}, lambda w: w.__setitem__(LM + ".signs", torch.tensor(SIGNS[:256])), "packed tensor shape/dtype mismatch"),
    ({}, lambda w: w.__setitem__(LM + ".scales", torch.ones(4, 4)), "packed tensor shape/dtype mismatch"),
    ({}, lambda w: w[LM + ".signs"].__setitem__(1, -1.0), "tensor signs disagree with metadata"),
])
def test_rejects_inconsistent_tensors(meta_edit, weights_edit, detail):
    info = prism.parse_config(_config())
    meta = prism.HadamardMetadata(_meta(**meta_edit))
    w = _edit_weights(weights_edit) if weights_edit else _weights()
    with pytest.raises(prism.PrismCheckpointError) as e:
        prism.validate(info, meta, w)
    assert e.value.detail == detail


def test_metadata_is_read_through_a_symlink_and_bounded(tmp_path):
    real = tmp_path / "blob.json"
    real.write_text(json.dumps(_meta()))
    d = tmp_path / "snap"
    d.mkdir()
    os.symlink(real, d / "hadamard.json")
    assert prism.HadamardMetadata.read(str(d)).block == 512
    with pytest.raises(prism.PrismCheckpointError):
        prism.HadamardMetadata.read(str(tmp_path / "missing"))
    with pytest.raises(prism.PrismCheckpointError, match="no transform signs for width 1024"):
        prism.HadamardMetadata(_meta()).transform(1024)


def prism_cfg():
    c = tiny_qwen3()
    c.model_type = "qwen3_5"
    c.layer_types = ["linear_attention", "linear_attention", "linear_attention", "full_attention"]
    c.attn_output_gate = True
    c.linear_num_key_heads, c.linear_num_value_heads = 2, 4
    c.linear_key_head_dim = c.linear_value_head_dim = 64
    c.tie_word_embeddings = False
    c.hidden_size, c.intermediate_size = 512, 1024  # input widths that are whole Hadamard blocks
    return c


def test_packed_model_matches_its_dense_equivalent(tmp_path):
    from mlx_swift_lm_b200.testing.prism import write_prism_checkpoint

    m = DecoderLM(prism_cfg(), "cpu", torch.float32).init_random(3, std=0.2)
    d = str(tmp_path / "prism")
    dense = write_prism_checkpoint(m, d, block=512)
    pm, hf = load_model(d, device="cpu", dtype=torch.float32)
    assert hf["model_type"] == "qwen3_5_text"
    from mlx_swift_lm_b200.ops.rotation import RotatedWeight

    assert isinstance(pm.lm_head, RotatedWeight) and isinstance(pm.layers[0].wqkv, RotatedWeight)
    ref_cfg = copy.deepcopy(pm.cfg)
    ref_cfg.quantization = None
    ref = build_from_tensors(ref_cfg, dense, "cpu", torch.float32)
    toks = torch.arange(3, 40) % m.cfg.vocab_size
    a = pm.forward_dense(toks, pm.new_cache())
    b = ref.forward_dense(toks, ref.new_cache())
    assert torch.allclose(a, b, atol=2e-3, rtol=1e-3), (a - b).abs().max()
