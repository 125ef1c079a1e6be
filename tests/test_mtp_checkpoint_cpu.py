"""MTP heads stored in checkpoints: the Qwen 3.5 inline layout (mtp.*), the
DeepSeek V3 / GLM nextn layout (layers.{N}: enorm, hnorm, eh_proj,
shared_head) and MiMo's mtp_layers load into the draft module and compute
what the module they were exported from computes; a loaded head drives the
engine's MTP rounds with token-exact greedy output."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM, EngineConfig, EngineV2, SchedulerConfig
from mlx_swift_lm_b200.loader.convert import export_tensors
from mlx_swift_lm_b200.models.batch import ForwardBatch
from mlx_swift_lm_b200.models.config import tiny_qwen3
from mlx_swift_lm_b200.models.mtp import MTPModule, load_mtp, mtp_layout


def _export_head(mod, layout, L):
    t = export_tensors(mod.inner)
    layer = {k[len("model.layers.0."):]: v for k, v in t.items() if k.startswith("model.layers.0.")}
    fn = t["model.norm.weight"]
    if layout == "qwen35":
        out = {f"mtp.layers.0.{k}": v for k, v in layer.items()}
        out.update({"mtp.fc.weight": mod.fc.float(), "mtp.pre_fc_norm_embedding.weight": mod.norm_e.float(),
                    "mtp.pre_fc_norm_hidden.weight": mod.norm_h.float(), "mtp.norm.weight": fn})
    elif layout == "deepseek":
        p = f"model.layers.{L}."
        out = {p + k: v for k, v in layer.items()}
        out.update({p + "eh_proj.weight": mod.fc.float(), p + "enorm.weight": mod.norm_e.float(),
                    p + "hnorm.weight": mod.norm_h.float(), p + "shared_head.norm.weight": fn})
    else:
        p = "model.mtp_layers.0."
        out = {p + k: v for k, v in layer.items()}
        out.update({p + "input_proj.weight": mod.fc.float(), p + "token_layernorm.weight": mod.norm_e.float(),
                    p + "hidden_layernorm.weight": mod.norm_h.float(), p + "final_layernorm.weight": fn})
    return out


@pytest.mark.parametrize("layout", ["qwen35", "deepseek", "mimo"])
def test_mtp_head_roundtrip(layout):
    cfg = tiny_qwen3()
    target = DecoderLM(cfg, "cpu", torch.float32).init_random(0, std=0.2)
    ref = MTPModule(target).init_random(3, std=0.2)
    tens = _export_head(ref, layout, cfg.num_layers)
    tens["model.embed_tokens.weight"] = target.embed  # the rest of a checkpoint
    assert mtp_layout(tens, cfg.num_layers) == (layout, 1)
    got = load_mtp(target, tens)
    assert got.layout == layout
    T = 5
    ids = torch.tensor([3, 9, 27, 81, 5], dtype=torch.int32)
    hidden = torch.randn(T, cfg.hidden_size, generator=torch.Generator().manual_seed(1))

    def run(mod):
        kv = mod.new_kv(64)
        from mlx_swift_lm_b200.kv.paged import SequenceKV

        s = SequenceKV(kv)
        s.ensure(T)
        fb = ForwardBatch(input_ids=ids, positions=torch.arange(T, dtype=torch.int32),
                          slots=torch.tensor(s.slots(0, T), dtype=torch.int64), num_decode=0,
                          pf_cu_q=torch.tensor([0, T], dtype=torch.int32), pf_cu_q_host=[0, T],
                          pf_pos0=torch.tensor([0], dtype=torch.int32),
                          pf_page_table=torch.tensor([s.pages], dtype=torch.int32))
        return mod.forward(fb, kv, hidden)

    la, ha = run(ref)
    lb, hb = run(got)
    assert torch.allclose(la, lb, atol=1e-4, rtol=1e-4)
    assert torch.allclose(ha, hb, atol=1e-4, rtol=1e-4)


def test_loaded_head_drives_mtp_rounds():
    from mlx_swift_lm_b200.engine.mtp import MTPConfig

    cfg = tiny_qwen3()
    target = DecoderLM(cfg, "cpu", torch.float32).init_random(0, std=0.2)
    ref = MTPModule(target).init_random(3, std=0.2)
    tens = _export_head(ref, "qwen35", cfg.num_layers)
    head = load_mtp(target, tens)
    prompts = [[5, 7, 9, 11, 13], [2, 4, 6]]

    def eng():
        return EngineV2(target, config=EngineConfig(scheduler=SchedulerConfig(max_concurrent_requests=2),
                                                   max_model_len=128, use_cuda_graphs=False, window_ring=False))

    want = eng().generate(prompts, max_tokens=12)
    e = eng()
    e.enable_mtp(head, MTPConfig(k=2))
    assert e.generate(prompts, max_tokens=12) == want
