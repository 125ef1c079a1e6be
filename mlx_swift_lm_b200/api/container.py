"""ModelContainer: model + tokenizer + engine behind one object.

Parity: MLXLMCommon/ModelContainer.swift:53-262 (``perform``, ``prepare``,
``generate``, ``encode`` / ``decode``, chat template) and
``loadModelContainer`` (ModelFactory.swift:310).
"""
from __future__ import annotations

import threading

import torch

from ..engine.engine import EngineConfig, EngineV2
from ..engine.scheduler import SchedulerConfig
from .generate import GenerateParameters, generate, generate_stream
from .tokenizer import ByteTokenizer, as_tokenizer


class ModelContainer:
    def __init__(self, model, tokenizer=None, engine_config: EngineConfig | None = None, eos_token_ids=None,
                 model_id: str = "local", hf_config: dict | None = None):
        self.model = model
        self.tokenizer = as_tokenizer(tokenizer) or ByteTokenizer(model.cfg.vocab_size)
        eos = set(eos_token_ids or [])
        if getattr(self.tokenizer, "eos_token_id", None) is not None:
            eos.add(int(self.tokenizer.eos_token_id))
        self.eos = eos
        self.engine = EngineV2(model, self.tokenizer, engine_config or EngineConfig(), eos_token_ids=eos)
        self.model_id = model_id
        self.hf_config = hf_config or {}
        self.lock = threading.RLock()

    # ------------------------------------------------------------------ loading
    @classmethod
    def load(cls, path, device=None, dtype=torch.bfloat16, engine_config: EngineConfig | None = None,
             tp=None, downloader=None, tokenizer_loader=None):
        """`path`: a local directory, a hub id found on local disk, or a
        :class:`.configuration.ModelConfiguration` (resolved through
        `downloader`, default :class:`.configuration.LocalDownloader`)."""
        from ..loader.load import eos_token_ids, load_model
        from .configuration import HFTokenizerLoader, ModelConfiguration, configuration

        mc = path if isinstance(path, ModelConfiguration) else configuration(str(path))
        res = mc.resolve(downloader)
        device = device or ("cuda" if torch.cuda.is_available() else "cpu")
        if device == "cpu":
            dtype = torch.float32
        model, hf = load_model(res.model_directory, device, dtype, tp)
        tok = (tokenizer_loader or HFTokenizerLoader()).load(res.tokenizer_directory)
        eos = eos_token_ids(res.model_directory, hf, getattr(tok, "tok", None)) | set(res.eos_token_ids)
        for s in res.extra_eos_tokens:
            ids = tok.encode(s) if hasattr(tok, "encode") else []
            if len(ids) == 1:
                eos.add(ids[0])
        c = cls(model, tok, engine_config, eos, model_id=res.name, hf_config=hf)
        c.configuration = res
        c._resolve_image_markers()
        return c

    def _resolve_image_markers(self):
        """SmolVLM tiling needs the ids of its marker tokens (SmolVLM2.swift:179-232);
        without them images go in as one global tile."""
        m = self.model
        if getattr(m, "kind", None) != "idefics3" or not getattr(m, "tile_longest_edge", 0):
            return
        enc = getattr(self.tokenizer, "encode", None)
        if enc is None:
            return

        def one(text):
            ids = enc(text)
            return ids[0] if len(ids) == 1 else None

        fake = one("<fake_token_around_image>")
        if fake is None:
            return
        m.marker_ids = {"fake": fake, "global": enc("<global-img>"), "newline": enc("\n"),
                        "row": lambda r, c: enc(f"<row_{r + 1}_col_{c + 1}>")}

    @classmethod
    def random(cls, cfg, device="cpu", dtype=torch.float32, seed=0, std=0.02, engine_config=None, tokenizer=None):
        from ..models.decoder import DecoderLM

        m = DecoderLM(cfg, device, dtype).init_random(seed, std=std)
        return cls(m, tokenizer, engine_config or EngineConfig(scheduler=SchedulerConfig(),
                                                               use_cuda_graphs=torch.device(device).type == "cuda"))

    def replicate(self, devices: list, engine_config: EngineConfig | None = None):
        """Data parallelism: one more engine per extra device, each with a copy
        of the model, behind an :class:`..engine.replicas.EngineReplicas` router
        that becomes this container's engine (the server sees one engine)."""
        from ..engine.replicas import EngineReplicas

        cfg = engine_config or self.engine.cfg
        engines = [self.engine]
        for d in devices:
            m = self.model.clone_to(d, self.model.dtype)
            engines.append(EngineV2(m, self.tokenizer, cfg, eos_token_ids=self.eos))
        self.engine = EngineReplicas(engines)
        return self

    # ------------------------------------------------------------------ actor-style access
    def perform(self, fn):
        with self.lock:
            return fn(self)

    # ------------------------------------------------------------------ text <-> tokens
    def encode(self, text: str) -> list[int]:
        return self.tokenizer.encode(text)

    def decode(self, ids) -> str:
        return self.tokenizer.decode(ids)

    def apply_chat_template(self, messages, tools=None, add_generation_prompt=True, **kw) -> list[int]:
        out = self.tokenizer.apply_chat_template(messages, tools=tools, add_generation_prompt=add_generation_prompt,
                                                 tokenize=True, **kw)
        if isinstance(out, dict):
            out = out["input_ids"]
        return list(out)

    def prepare(self, prompt=None, messages=None, tools=None) -> list[int]:
        if messages is not None:
            return self.apply_chat_template(messages, tools=tools)
        if isinstance(prompt, str):
            return self.encode(prompt)
        return list(prompt)

    def prepare_media(self, toks: list[int], images=None, videos=None):
        """Vision-language models: expand the image / video placeholders of
        `toks` and encode the media (models.vlm.Qwen2VLModel.prepare)."""
        if not images and not videos:
            return toks, None
        if not hasattr(self.model, "prepare"):
            raise ValueError(f"{type(self.model).__name__} takes no image or video input")
        from .media import MediaInput

        return self.model.prepare(toks, MediaInput(list(images or []), list(videos or [])))

    # ------------------------------------------------------------------ generation
    def generate(self, prompt=None, messages=None, params: GenerateParameters | None = None, tools=None, images=None,
                 videos=None):
        toks, mm = self.prepare_media(self.prepare(prompt, messages, tools), images, videos)
        return generate(self.engine, toks, params, mm=mm)

    def stream(self, prompt=None, messages=None, params: GenerateParameters | None = None, tools=None, images=None,
               videos=None):
        toks, mm = self.prepare_media(self.prepare(prompt, messages, tools), images, videos)
        yield from generate_stream(self.engine, toks, params, mm=mm)

    # ------------------------------------------------------------------ embeddings
    @torch.no_grad()
    def embed(self, texts, pooling: str = "mean", normalize: bool = True) -> list[list[float]]:
        """Sentence embeddings from the final hidden states (mean or last-token
        pooling, L2-normalised), the decoder-embedder path of MLXEmbedders."""
        out = []
        for t in texts:
            toks = self.encode(t) if isinstance(t, str) else list(t)
            h = self.model.forward_dense(torch.tensor(toks, device=self.model.device), self.model.new_cache(),
                                         return_hidden=True).float()
            v = h.mean(0) if pooling == "mean" else h[-1]
            if normalize:
                v = v / v.norm().clamp(min=1e-12)
            out.append(v.cpu().tolist())
        return out
