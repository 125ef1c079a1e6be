"""LoRA / DoRA adapters (fuse into the fused projection layouts, unload,
MLX and PEFT formats) and adapter training, on the tiny Qwen3 in fp32 on CPU."""
import json
import os

import torch

from mlx_swift_lm_b200 import DecoderLM
from mlx_swift_lm_b200.adapters import AdapterRegistry, LoRAConfiguration, LoRAContainer, LoRAParameters, load_adapter
from mlx_swift_lm_b200.api.tokenizer import ByteTokenizer
from mlx_swift_lm_b200.loader.safetensors import save_safetensors
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.train import TrainParameters, TrainableLoRA, iterate_batches, loss_fn, train, train_forward

ALL_KEYS = ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
            "mlp.up_proj", "mlp.down_proj"]


def _model(seed=0, **over):
    cfg = tiny_qwen3()
    for k, v in over.items():
        setattr(cfg, k, v)
    return DecoderLM(cfg, "cpu", torch.float32).init_random(seed, std=0.2)


def _adapter(m, ft="lora", seed=0, layers=2):
    conf = LoRAConfiguration(num_layers=layers, fine_tune_type=ft,
                             lora_parameters=LoRAParameters(rank=4, scale=2.0, keys=ALL_KEYS))
    ad = LoRAContainer.init_for(m, conf, seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    for ent in ad.tensors.values():  # non-zero B so the adapter changes the model
        ent["b"] = torch.randn(ent["b"].shape, generator=g) * 0.05
        if ent["m"] is not None:
            ent["m"] = ent["m"] * (1 + 0.1 * torch.randn(ent["m"].shape, generator=g))
    return ad


def _logits(m, toks):
    return m.forward_dense(torch.tensor(toks), m.new_cache())


def test_train_forward_matches_inference_forward():
    m = _model()
    toks = torch.randint(0, m.cfg.vocab_size, (1, 21), generator=torch.Generator().manual_seed(2))
    a = train_forward(m, toks, None, training=False)[0]
    b = _logits(m, toks[0].tolist())
    assert torch.allclose(a, b, atol=2e-4, rtol=1e-4)


def _check_fused_equals_unfused(ft):
    m = _model()
    toks = torch.randint(0, m.cfg.vocab_size, (1, 17), generator=torch.Generator().manual_seed(3))
    base = _logits(m, toks[0].tolist())
    ad = _adapter(m, ft)
    lora = TrainableLoRA(ad, "cpu")
    unfused = train_forward(m, toks, lora, training=False)[0].detach()
    ad.load(m)
    fused = _logits(m, toks[0].tolist())
    assert (fused - base).abs().max() > 1e-3, "adapter should change the logits"
    assert torch.allclose(fused, unfused, atol=5e-4, rtol=1e-3)
    ad.unload(m)
    assert torch.equal(_logits(m, toks[0].tolist()), base)


def test_lora_fused_equals_unfused_and_unload_restores():
    _check_fused_equals_unfused("lora")


def test_dora_fused_equals_unfused_and_unload_restores():
    _check_fused_equals_unfused("dora")


def test_fresh_adapter_is_identity():
    m = _model()
    conf = LoRAConfiguration(num_layers=4, lora_parameters=LoRAParameters(rank=8, keys=["q_proj", "v_proj"]))
    ad = LoRAContainer.init_for(m, conf)
    toks = list(range(5, 30))
    base = _logits(m, toks)
    ad.load(m)
    assert torch.allclose(_logits(m, toks), base, atol=1e-5)


def test_mlx_format_roundtrip_and_registry(tmp_path):
    m = _model()
    ad = _adapter(m)
    d = str(tmp_path / "ad")
    ad.save(d)
    cfg = json.load(open(os.path.join(d, "adapter_config.json")))
    assert cfg["fine_tune_type"] == "lora" and cfg["lora_parameters"]["rank"] == 4
    ad2 = load_adapter(d)
    assert set(ad2.tensors) == set(ad.tensors)
    for k in ad.tensors:
        assert torch.allclose(ad2.tensors[k]["a"], ad.tensors[k]["a"])
        assert torch.allclose(ad2.tensors[k]["b"], ad.tensors[k]["b"])
    toks = list(range(40, 60))
    base = _logits(m, toks)
    reg = AdapterRegistry(m)
    reg.register("a", d)
    reg.activate("a")
    with_a = _logits(m, toks)
    assert (with_a - base).abs().max() > 1e-3
    reg.activate(None)
    assert torch.equal(_logits(m, toks), base)


def test_peft_format(tmp_path):
    m = _model()
    ad = _adapter(m, layers=1)
    d = tmp_path / "peft"
    d.mkdir()
    r = 4
    json.dump({"peft_type": "LORA", "r": r, "lora_alpha": 2.0 * r, "lora_dropout": 0.0,
               "target_modules": ["q_proj", "down_proj"]}, open(d / "adapter_config.json", "w"))
    tens = {}
    for (li, k), ent in ad.tensors.items():
        if k in ("self_attn.q_proj", "mlp.down_proj"):
            base = f"base_model.model.model.layers.{li}.{k}"
            tens[base + ".lora_A.weight"] = ent["a"]
            tens[base + ".lora_B.weight"] = ent["b"]
    save_safetensors(str(d / "adapter_model.safetensors"), tens)
    p = load_adapter(str(d))
    assert p.configuration.lora_parameters.scale == 2.0
    assert set(k for _, k in p.tensors) == {"self_attn.q_proj", "mlp.down_proj"}
    li = next(iter(p.tensors))[0]
    assert torch.allclose(p.tensors[(li, "self_attn.q_proj")]["a"], ad.tensors[(li, "self_attn.q_proj")]["a"])


def test_training_reduces_loss(tmp_path):
    torch.manual_seed(0)
    m = _model(seed=1)
    tok = ByteTokenizer(m.cfg.vocab_size)
    data = ["the quick brown fox jumps over the lazy dog"] * 4 + ["hello world, hello adapters"] * 4
    conf = LoRAConfiguration(num_layers=2, lora_parameters=LoRAParameters(rank=8, scale=4.0, keys=ALL_KEYS))
    ad = LoRAContainer.init_for(m, conf)
    lora = TrainableLoRA(ad, "cpu")
    x, y, ln = next(iterate_batches(data, tok, 4, train=False))
    l0, n = loss_fn(m, lora, x, y, ln, training=False)
    assert n == int((ln - 1).sum())
    events = []
    params = TrainParameters(batch_size=4, iterations=30, steps_per_report=10, steps_per_eval=15,
                             validation_batches=1, save_every=15, adapter_path=str(tmp_path / "out"),
                             learning_rate=3e-3)
    train(m, ad, tok, data, data[:4], params, progress=lambda e: events.append(e) or True)
    lora2 = TrainableLoRA(ad, "cpu")
    l1, _ = loss_fn(m, lora2, x, y, ln, training=False)
    assert float(l1) < float(l0) - 0.5, (float(l0), float(l1))
    kinds = {e.kind for e in events}
    assert kinds == {"train", "validation", "save"}
    assert os.path.exists(tmp_path / "out" / "adapters.safetensors")
    # the saved adapter applied to the serving path reproduces the trained loss
    ad3 = load_adapter(str(tmp_path / "out"))
    ad3.load(m)
    lg = train_forward(m, x, None, training=False)
    ce = torch.nn.functional.cross_entropy(lg.reshape(-1, lg.shape[-1]), y.reshape(-1), reduction="none")
    mask = (torch.arange(x.shape[1])[None, :] < (ln[:, None] - 1)).reshape(-1)
    assert abs(float((ce * mask).sum() / mask.sum()) - float(l1)) < 1e-3
