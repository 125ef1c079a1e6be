"""Model configuration resolution: local directories, the HF cache layout,
registry entries, tokenizer sources; loading a container through it."""
import os

import pytest
import torch

from mlx_swift_lm_b200.api.configuration import (LocalDownloader, ModelConfiguration, ModelNotFound, REGISTRY,
                                                  configuration)


def test_local_downloader_resolves_hf_cache(tmp_path):
    hub = tmp_path / "models--org--tiny"
    (hub / "snapshots" / "abc123").mkdir(parents=True)
    (hub / "refs").mkdir()
    (hub / "refs" / "main").write_text("abc123")
    (hub / "snapshots" / "abc123" / "config.json").write_text("{}")
    dl = LocalDownloader([str(tmp_path)])
    assert dl.download("org/tiny", "main", ["config.json"]).endswith("snapshots/abc123")
    with pytest.raises(ModelNotFound):
        dl.download("org/absent")
    plain = tmp_path / "org" / "plain"
    plain.mkdir(parents=True)
    (plain / "config.json").write_text("{}")
    assert dl.download("org/plain") == str(plain)


def test_configuration_fields():
    c = REGISTRY["openai/gpt-oss-120b"]
    assert c.tool_call_format == "harmony" and "<|return|>" in c.effective_stop_strings
    d = configuration("/definitely/not/here")
    assert d.id == "/definitely/not/here"
    m = ModelConfiguration(directory="/a/b/model")
    assert m.name == "b/model"


def test_container_loads_through_configuration(tmp_path):
    from mlx_swift_lm_b200 import DecoderLM
    from mlx_swift_lm_b200.api.container import ModelContainer
    from mlx_swift_lm_b200.loader.convert import save_model
    from mlx_swift_lm_b200.models.config import tiny_qwen3

    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(1)
    d = tmp_path / "models--me--tiny" / "snapshots" / "r1"
    save_model(m, str(d), dtype=torch.float32)
    c = ModelContainer.load(ModelConfiguration(id="me/tiny", revision="r1", eos_token_ids={3}), device="cpu",
                            downloader=LocalDownloader([str(tmp_path)]))
    assert c.model_id == "me/tiny" and 3 in c.eos
    assert os.path.samefile(c.configuration.model_directory, d)
