"""SigLIP vision encoder on the decoder's kernels, and the Gemma 3
vision-language model built on it.

SigLIP (MLXVLM/Models/Gemma3.swift:478-780, the vision tower of Gemma 3,
PaliGemma, Idefics3): a Conv2d patch embedding whose kernel equals its stride
(one linear map of each flattened [C, p, p] patch) plus a learned position
embedding per patch; pre-norm encoder layers (LayerNorm, multi-head
self-attention with biased q / k / v / o over the whole image, LayerNorm,
GELU-tanh MLP with biases); a final LayerNorm.

Gemma 3's projector (Gemma3.swift:783-850): the patch grid average-pooled to
``mm_tokens_per_image`` tokens, a Gemma RMSNorm (weights stored as w - 1) and
a [vision, text] projection; the tokens replace the image placeholders of
the prompt (one placeholder expands to ``mm_tokens_per_image`` image tokens)
and the language model runs as usual (1-D positions, causal attention).

B200 path: GEMMs with bias / GELU epilogues, the fused residual + LayerNorm
kernel, and the tensor-core paged prefill kernel in bidirectional mode over a
scratch page pool (one row per image); head dims the kernels do not take
(SigLIP-so400m: 72) are zero-padded to the next one they do (q.k and the
kept output channels are unchanged).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops
from ..kv.paged import PAGE
from .decoder import DecoderLM
from .encoder import scratch_layout


@dataclass
class SiglipConfig:
    hidden_size: int = 1152
    intermediate_size: int = 4304
    num_layers: int = 27
    num_heads: int = 16
    image_size: int = 896
    patch_size: int = 14
    num_channels: int = 3
    eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def grid(self) -> int:
        return self.image_size // self.patch_size

    @classmethod
    def from_hf(cls, vc: dict) -> "SiglipConfig":
        return cls(hidden_size=vc.get("hidden_size", 1152), intermediate_size=vc.get("intermediate_size", 4304),
                   num_layers=vc.get("num_hidden_layers", 27), num_heads=vc.get("num_attention_heads", 16),
                   image_size=vc.get("image_size", 896), patch_size=vc.get("patch_size", 14),
                   num_channels=vc.get("num_channels", 3), eps=vc.get("layer_norm_eps", 1e-6))


_NAMES = {"ln1_w": "layer_norm1.weight", "ln1_b": "layer_norm1.bias", "q_w": "self_attn.q_proj.weight",
          "q_b": "self_attn.q_proj.bias", "k_w": "self_attn.k_proj.weight", "k_b": "self_attn.k_proj.bias",
          "v_w": "self_attn.v_proj.weight", "v_b": "self_attn.v_proj.bias", "o_w": "self_attn.out_proj.weight",
          "o_b": "self_attn.out_proj.bias", "ln2_w": "layer_norm2.weight", "ln2_b": "layer_norm2.bias",
          "fc1_w": "mlp.fc1.weight", "fc1_b": "mlp.fc1.bias", "fc2_w": "mlp.fc2.weight", "fc2_b": "mlp.fc2.bias"}


class SiglipVisionTower:
    def __init__(self, cfg: SiglipConfig, device="cpu", dtype=torch.float32):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.patch_w = self.patch_b = self.pos = None
        self.post_w = self.post_b = None
        self.layers: list[dict] = []

    def tensors(self):
        yield "patch_w", self.patch_w
        yield "patch_b", self.patch_b
        yield "pos", self.pos
        yield "post_w", self.post_w
        yield "post_b", self.post_b
        for i, L in enumerate(self.layers):
            for k, v in L.items():
                yield f"layers.{i}.{k}", v

    def to(self, device, dtype):
        self.device, self.dtype = torch.device(device), dtype
        for n in ("patch_w", "patch_b", "pos", "post_w", "post_b"):
            setattr(self, n, getattr(self, n).to(self.device, dtype).contiguous())
        for L in self.layers:
            for k in L:
                L[k] = L[k].to(self.device, dtype).contiguous()
        # fused q|k|v (and its bias) for one GEMM per layer
        for L in self.layers:
            L["qkv_w"] = torch.cat([L["q_w"], L["k_w"], L["v_w"]], 0).contiguous()
            L["qkv_b"] = torch.cat([L["q_b"], L["k_b"], L["v_b"]], 0).contiguous()
        return self

    def init_random(self, seed: int = 0, std: float = 0.02):
        c = self.cfg
        g = torch.Generator().manual_seed(seed)
        E, F = c.hidden_size, c.intermediate_size

        def rn(*shape):
            return torch.empty(shape).normal_(0.0, std, generator=g)

        self.patch_w, self.patch_b = rn(E, c.num_channels * c.patch_size ** 2), rn(E)
        self.pos = rn(c.grid * c.grid, E)
        self.post_w, self.post_b = torch.ones(E), rn(E)
        self.layers = []
        for _ in range(c.num_layers):
            L = {k: rn(E) for k in ("ln1_b", "q_b", "k_b", "v_b", "o_b", "ln2_b", "fc2_b")}
            L.update(ln1_w=torch.ones(E), ln2_w=torch.ones(E), q_w=rn(E, E), k_w=rn(E, E), v_w=rn(E, E),
                     o_w=rn(E, E), fc1_w=rn(F, E), fc1_b=rn(F), fc2_w=rn(E, F))
            self.layers.append(L)
        return self.to(self.device, self.dtype)

    @classmethod
    def from_tensors(cls, cfg: SiglipConfig, t: dict, device="cpu", dtype=torch.float32):
        pre = next((p for p in ("vision_tower.vision_model.", "model.vision_tower.vision_model.",
                                "vision_model.", "") if p + "embeddings.patch_embedding.weight" in t), None)
        if pre is None:
            raise KeyError("no SigLIP weights (vision_model.embeddings.patch_embedding.weight)")
        m = cls(cfg)

        def g(n):
            return t[pre + n].float()

        w = g("embeddings.patch_embedding.weight")
        if w.shape[-1] == cfg.num_channels and w.shape[1] != cfg.num_channels:  # MLX layout [out, p, p, C]
            w = w.permute(0, 3, 1, 2)
        m.patch_w, m.patch_b = w.reshape(w.shape[0], -1), g("embeddings.patch_embedding.bias")
        m.pos = g("embeddings.position_embedding.weight")
        m.post_w, m.post_b = g("post_layernorm.weight"), g("post_layernorm.bias")
        m.layers = [{k: g(f"encoder.layers.{i}.{n}") for k, n in _NAMES.items()} for i in range(cfg.num_layers)]
        return m.to(device, dtype)

    @staticmethod
    def patchify(pixels: torch.Tensor, p: int) -> torch.Tensor:
        """[B, C, S, S] -> [B * (S/p)^2, C*p*p], patches row-major, each flattened as [C, p, p]."""
        B, C, S, _ = pixels.shape
        n = S // p
        x = pixels.reshape(B, C, n, p, n, p).permute(0, 2, 4, 1, 3, 5)
        return x.reshape(B * n * n, C * p * p)

    @torch.no_grad()
    def forward(self, pixels: torch.Tensor) -> torch.Tensor:
        """pixels [B, C, S, S] (normalised) -> patch features [B, (S/p)^2, hidden]."""
        c = self.cfg
        dev, E, NH, D = self.device, c.hidden_size, c.num_heads, c.head_dim
        B = pixels.shape[0]
        P = c.grid * c.grid
        patches = self.patchify(pixels.to(dev, self.dtype), c.patch_size)
        w = self.patch_w
        K = w.shape[1]
        if patches.is_cuda and K % 8:
            # the GEMM's TMA rows need K * 2 bytes to be a multiple of 16: zero
            # columns pad both operands (C*14*14 = 588 for RGB patches of 14)
            K8 = (K + 7) // 8 * 8
            if getattr(self, "_patch_w8", None) is None or self._patch_w8.shape[1] != K8:
                self._patch_w8 = torch.nn.functional.pad(w, (0, K8 - K)).contiguous()
            w = self._patch_w8
            patches = torch.nn.functional.pad(patches, (0, K8 - K))
        x = ops.gemm(patches.contiguous(), w, bias=self.patch_b)
        x = (x.float() + self.pos.float().repeat(B, 1)).to(self.dtype)
        N = x.shape[0]
        Dk = D if D in (64, 128, 256) or not x.is_cuda else (64 if D < 64 else 128 if D < 128 else 256)
        pt, slots, cu, npages = scratch_layout([P] * B, dev)
        kc = torch.zeros(npages, NH, PAGE, Dk, dtype=self.dtype, device=dev)
        vc = torch.zeros_like(kc)
        cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
        pos0 = torch.zeros(B, dtype=torch.int32, device=dev)
        tok = torch.arange(N, dtype=torch.int32, device=dev)
        table = torch.zeros(1, max(Dk, 2), dtype=torch.float32, device=dev)
        delta = None
        for L in self.layers:
            h = ops.add_layernorm(x, delta, L["ln1_w"], L["ln1_b"], c.eps)
            qkv = ops.gemm(h, L["qkv_w"], bias=L["qkv_b"])
            if Dk != D:  # zero-pad every head to the kernels' head dim
                qkv = torch.nn.functional.pad(qkv.view(N, 3 * NH, D), (0, Dk - D)).reshape(N, 3 * NH * Dk)
            q = ops.qk_norm_rope_kv(qkv, tok * 0, slots, table, 0, False, None, None, c.eps, kc, vc, NH, NH, Dk)
            a = ops.paged_prefill(q, kc, vc, pt, cu_t, pos0, D ** -0.5, -1, cu_q_host=cu)
            if Dk != D:
                a = a[..., :D]
            d = ops.gemm(a.reshape(N, E).contiguous(), L["o_w"], bias=L["o_b"])
            h = ops.add_layernorm(x, d, L["ln2_w"], L["ln2_b"], c.eps)
            delta = ops.gemm(ops.gemm(h, L["fc1_w"], epi="gelu_tanh", bias=L["fc1_b"]), L["fc2_w"], bias=L["fc2_b"])
        out = ops.add_layernorm(x, delta, self.post_w, self.post_b, c.eps)
        return out.view(B, P, E)


def siglip_pixels(image, size: int, mean=(0.5, 0.5, 0.5), std=(0.5, 0.5, 0.5)) -> torch.Tensor:
    """An image (PIL, HWC uint8 / float array or CHW tensor) resized to size x
    size (bilinear), scaled to [0, 1] and normalised: [3, size, size] fp32."""
    import numpy as np

    if hasattr(image, "convert"):
        image = np.asarray(image.convert("RGB"))
    t = torch.as_tensor(np.asarray(image) if not torch.is_tensor(image) else image).float()
    if t.dim() == 3 and t.shape[-1] in (1, 3, 4) and t.shape[0] not in (1, 3):
        t = t[..., :3].permute(2, 0, 1)
    if t.max() > 1.5:
        t = t / 255.0
    t = torch.nn.functional.interpolate(t[None], size=(size, size), mode="bilinear", align_corners=False)[0]
    m = torch.tensor(mean)[:, None, None]
    s = torch.tensor(std)[:, None, None]
    return (t - m) / s


class Gemma3VLModel(DecoderLM):
    """Gemma 3 language model + SigLIP tower + pooled projector; multimodal
    requests carry ``Request.mm`` from :meth:`prepare`."""

    def __init__(self, cfg, vision_cfg: SiglipConfig, device="cpu", dtype=torch.float32,
                 image_token_id: int = 262144, mm_tokens: int = 256):
        super().__init__(cfg, device, dtype)
        self.vision = SiglipVisionTower(vision_cfg, device, dtype)
        self.image_token_id = image_token_id
        self.mm_tokens = mm_tokens
        self.proj_norm = None  # [vision hidden] (Gemma RMSNorm weight, stored w - 1)
        self.proj_w = None  # [vision hidden, text hidden]

    def init_random(self, seed: int = 0, std: float = 0.02, with_embeddings: bool = True, keep_layers=None):
        super().init_random(seed, std, with_embeddings, keep_layers)
        self.vision.init_random(seed + 17, std)
        g = torch.Generator().manual_seed(seed + 29)
        E = self.vision.cfg.hidden_size
        self.proj_norm = torch.zeros(E, device=self.device, dtype=self.dtype)
        self.proj_w = torch.empty(E, self.cfg.hidden_size).normal_(0.0, std, generator=g).to(self.device, self.dtype)
        return self

    def clone_to(self, device, dtype):
        m = super().clone_to(device, dtype)
        out = Gemma3VLModel(self.cfg, self.vision.cfg, device, dtype, self.image_token_id, self.mm_tokens)
        out.embed, out.norm, out.lm_head, out.layers = m.embed, m.norm, m.lm_head, m.layers
        v = SiglipVisionTower(self.vision.cfg)
        v.patch_w, v.patch_b, v.pos, v.post_w, v.post_b = (self.vision.patch_w, self.vision.patch_b, self.vision.pos,
                                                         self.vision.post_w, self.vision.post_b)
        v.layers = [{k: t for k, t in L.items() if k not in ("qkv_w", "qkv_b")} for L in self.vision.layers]
        out.vision = v.to(device, dtype)
        out.proj_norm, out.proj_w = self.proj_norm.to(device, dtype), self.proj_w.to(device, dtype)
        return out

    @torch.no_grad()
    def image_embeddings(self, pixels: torch.Tensor) -> torch.Tensor:
        """[B, C, S, S] -> [B * mm_tokens, text hidden]."""
        f = self.vision.forward(pixels)  # [B, P, E]
        B, P, E = f.shape
        n = self.vision.cfg.grid
        side = int(round(self.mm_tokens ** 0.5))
        k = n // side
        pooled = f.float().view(B, side, k, side, k, E).mean((2, 4)).reshape(B * side * side, E)
        h = ops.rmsnorm(pooled.to(self.dtype).contiguous(), self.proj_norm, self.vision.cfg.eps, True)
        return ops.gemm(h, self.proj_w.t().contiguous())

    @torch.no_grad()
    def prepare(self, prompt_tokens: list[int], media) -> tuple[list[int], dict | None]:
        """Expand each image placeholder to mm_tokens image tokens and encode
        the images. Returns (tokens, mm) with mm = {embeds, image_pos,
        prompt_len}; positions stay 1-D."""
        images = list(getattr(media, "images", None) or []) if media is not None else []
        if not images:
            return list(prompt_tokens), None
        size = self.vision.cfg.image_size
        pix = torch.stack([siglip_pixels(im, size) for im in images])
        emb = self.image_embeddings(pix)
        toks = []
        for t in prompt_tokens:
            toks.extend([t] * self.mm_tokens if t == self.image_token_id else [t])
        image_pos = [i for i, t in enumerate(toks) if t == self.image_token_id]
        assert len(image_pos) == emb.shape[0], "one image per placeholder token"
        return toks, {"embeds": emb, "image_pos": torch.tensor(image_pos), "prompt_len": len(toks), "delta": 0}

    def forward(self, fb, kv, return_hidden: bool = False, inputs_embeds=None, return_both=False,
                return_residual=False):
        states = getattr(fb, "row_states", None)
        rows = []
        if inputs_embeds is None and states:
            nd = fb.num_decode
            pf = fb.pf_cu_q_host or [0]
            for i, st in enumerate(states):
                mm = st.req.mm if st is not None else None
                if mm is None or i < nd:
                    continue
                a, n = nd + pf[i - nd], pf[i - nd + 1] - pf[i - nd]
                rows.append((a, n, int(fb.pf_pos0_host[i - nd]), mm))
        if not rows:
            return super().forward(fb, kv, return_hidden, inputs_embeds, return_both, return_residual)
        x = ops.embedding(fb.input_ids, self.embed, self.cfg.embed_scale).clone()
        for a, n, p0, mm in rows:
            ip = mm["image_pos"]
            sel = ((ip >= p0) & (ip < p0 + n)).nonzero()[:, 0]
            if len(sel):
                x[(ip[sel] - p0 + a).to(x.device)] = mm["embeds"][sel.to(mm["embeds"].device)].to(x.dtype)
        return super().forward(fb, kv, return_hidden, x, return_both, return_residual)
