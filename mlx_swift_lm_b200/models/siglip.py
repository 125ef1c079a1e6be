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
                                "vision_model.", "model.vision_model.", "vision_tower.", "model.vision_tower.", "")
                    if p + "embeddings.patch_embedding.weight" in t), None)
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


def _image_tensor(image) -> torch.Tensor:
    """An image (PIL, HWC uint8 / float array or CHW tensor) as [3, H, W] fp32 in [0, 1]."""
    import numpy as np

    if hasattr(image, "convert"):
        image = np.asarray(image.convert("RGB"))
    t = torch.as_tensor(np.asarray(image) if not torch.is_tensor(image) else image).float()
    if t.dim() == 3 and t.shape[-1] in (1, 3, 4) and t.shape[0] not in (1, 3):
        t = t[..., :3].permute(2, 0, 1)
    if t.max() > 1.5:
        t = t / 255.0
    return t


def _resize(t: torch.Tensor, h: int, w: int) -> torch.Tensor:
    if tuple(t.shape[-2:]) == (h, w):
        return t
    return torch.nn.functional.interpolate(t[None], size=(h, w), mode="bicubic", align_corners=False,
                                           antialias=True)[0].clamp(0.0, 1.0)


def smolvlm_tiles(image, tile: int, longest: int) -> tuple[list[torch.Tensor], int, int]:
    """SmolVLM's image split (SmolVLM2.swift:264-299): the image resized so its
    longest edge is min(longest, its own) and each side is a multiple of
    `tile` (aspect kept), cut into rows x cols tiles of `tile` pixels in
    row-major order, plus the whole image resized to tile x tile last.
    Returns ([3, tile, tile] tiles in [0, 1], rows, cols)."""
    t = _image_tensor(image)
    H, W = t.shape[-2:]
    edge = min(longest, max(H, W))
    if W >= H:
        w1 = edge
        h1 = edge * H / W
        w2 = -(-w1 // tile) * tile
        h2 = -(-int(round(w2 * H / W)) // tile) * tile
    else:
        h1 = edge
        w1 = edge * W / H
        h2 = -(-h1 // tile) * tile
        w2 = -(-int(round(h2 * W / H)) // tile) * tile
    h2, w2 = max(int(h2), tile), max(int(w2), tile)
    big = _resize(t, h2, w2)
    rows, cols = h2 // tile, w2 // tile
    tiles = [big[:, r * tile:(r + 1) * tile, c * tile:(c + 1) * tile] for r in range(rows) for c in range(cols)]
    tiles.append(_resize(t, tile, tile))
    return tiles, rows, cols


class SiglipVLM(DecoderLM):
    """A decoder language model with a SigLIP-family vision tower and one of
    the connectors built on it; multimodal requests carry ``Request.mm`` from
    :meth:`prepare` (image features replace the image placeholder rows).

    Connectors (``kind``):

    * ``gemma3`` (Gemma3.swift:783-850): the patch grid average-pooled to
      ``mm_tokens`` tokens, Gemma RMSNorm (weights stored w - 1), a
      [vision, text] projection; one placeholder expands to ``mm_tokens``.
    * ``paligemma`` (Paligemma.swift:505-600): a biased linear projection; the
      features are divided by sqrt(text hidden) and the decoder's embedding
      scale multiplies them back, so the rows are the projection itself; the
      prompt is ``mm_tokens`` image tokens then the text, and the whole prompt
      (image and text) attends both ways (prefix-LM: the prompt is prefilled
      in one chunk, generated tokens attend causally).
    * ``idefics3`` (Idefics3.swift:136-183, 629-760; SmolVLM2.swift for
      ``smolvlm``): pixel shuffle by ``scale_factor`` (each s x s block of
      patches concatenated into one token) and a bias-free linear projection;
      ``image_seq_len`` tokens per image (tile). A prompt without a
      placeholder gets the image tokens at its middle (the reference
      processor's rule). ``smolvlm`` also splits large images into tiles with
      row / column marker tokens when ``marker_ids`` are known.
    """

    def __init__(self, cfg, vision_cfg: SiglipConfig, device="cpu", dtype=torch.float32, kind: str = "gemma3",
                 image_token_id: int = 262144, mm_tokens: int = 256, scale_factor: int = 1):
        super().__init__(cfg, device, dtype)
        self.kind = kind
        self.vision = SiglipVisionTower(vision_cfg, device, dtype)
        self.image_token_id = image_token_id
        self.mm_tokens = mm_tokens
        self.scale_factor = scale_factor
        self.proj_norm = None  # gemma3: [vision hidden] (Gemma RMSNorm weight, stored w - 1)
        self.proj_w = None  # gemma3: [vision hidden, text hidden]; others: [text hidden, in] (nn.Linear)
        self.proj_b = None  # paligemma: [text hidden]
        self.image_mean = (0.5, 0.5, 0.5)
        self.image_std = (0.5, 0.5, 0.5)
        # smolvlm tiling: ids of '<fake_token_around_image>' ("fake"), '<global-img>' ("global"),
        # "\n" ("newline"), and row(r, c) -> ids of '<row_{r+1}_col_{c+1}>'
        self.marker_ids: dict | None = None
        self.tile_longest_edge = 0

    @property
    def prefix_lm(self) -> bool:
        return self.kind == "paligemma"

    def _proj_in(self) -> int:
        E = self.vision.cfg.hidden_size
        return E * self.scale_factor ** 2 if self.kind == "idefics3" else E

    def init_random(self, seed: int = 0, std: float = 0.02, with_embeddings: bool = True, keep_layers=None,
                    layer_hook=None):
        super().init_random(seed, std, with_embeddings, keep_layers, layer_hook)
        self.vision.init_random(seed + 17, std)
        g = torch.Generator().manual_seed(seed + 29)
        E, Hd = self.vision.cfg.hidden_size, self.cfg.hidden_size
        if self.kind == "gemma3":
            self.proj_norm = torch.zeros(E, device=self.device, dtype=self.dtype)
            self.proj_w = torch.empty(E, Hd).normal_(0.0, std, generator=g).to(self.device, self.dtype)
        else:
            self.proj_w = torch.empty(Hd, self._proj_in()).normal_(0.0, std, generator=g).to(self.device, self.dtype)
            if self.kind == "paligemma":
                self.proj_b = torch.empty(Hd).normal_(0.0, std, generator=g).to(self.device, self.dtype)
        return self

    def _same_kind(self, device, dtype):
        out = SiglipVLM(self.cfg, self.vision.cfg, device, dtype, self.kind, self.image_token_id, self.mm_tokens,
                        self.scale_factor)
        out.__class__ = self.__class__
        return out

    def clone_to(self, device, dtype):
        m = super().clone_to(device, dtype)
        out = self._same_kind(device, dtype)
        out.embed, out.norm, out.lm_head, out.layers = m.embed, m.norm, m.lm_head, m.layers
        v = SiglipVisionTower(self.vision.cfg)
        v.patch_w, v.patch_b, v.pos, v.post_w, v.post_b = (self.vision.patch_w, self.vision.patch_b, self.vision.pos,
                                                         self.vision.post_w, self.vision.post_b)
        v.layers = [{k: t for k, t in L.items() if k not in ("qkv_w", "qkv_b")} for L in self.vision.layers]
        out.vision = v.to(device, dtype)
        for n in ("proj_norm", "proj_w", "proj_b"):
            t = getattr(self, n)
            setattr(out, n, None if t is None else t.to(device, dtype))
        out.image_mean, out.image_std = self.image_mean, self.image_std
        out.marker_ids, out.tile_longest_edge = self.marker_ids, self.tile_longest_edge
        return out

    @staticmethod
    def pixel_shuffle(f: torch.Tensor, s: int) -> torch.Tensor:
        """[B, P, E] -> [B, P / s^2, E * s^2]: each s x s block of the patch
        grid becomes one token (Idefics3.swift:145-173)."""
        B, P, E = f.shape
        n = int(round(P ** 0.5))
        x = f.reshape(B, n, n // s, E * s).permute(0, 2, 1, 3)
        x = x.reshape(B, n // s, n // s, E * s * s).permute(0, 2, 1, 3)
        return x.reshape(B, P // (s * s), E * s * s)

    @torch.no_grad()
    def image_embeddings(self, pixels: torch.Tensor) -> torch.Tensor:
        """[B, C, S, S] -> [B * mm_tokens, text hidden]."""
        f = self.vision.forward(pixels)  # [B, P, E]
        B, P, E = f.shape
        if self.kind == "gemma3":
            n = self.vision.cfg.grid
            side = int(round(self.mm_tokens ** 0.5))
            k = n // side
            pooled = f.float().view(B, side, k, side, k, E).mean((2, 4)).reshape(B * side * side, E)
            h = ops.rmsnorm(pooled.to(self.dtype).contiguous(), self.proj_norm, self.vision.cfg.eps, True)
            return ops.gemm(h, self.proj_w.t().contiguous())
        if self.kind == "paligemma":
            y = ops.gemm(f.reshape(B * P, E).contiguous(), self.proj_w, bias=self.proj_b)
            # / sqrt(hidden) then the decoder's x sqrt(hidden): the rounded round trip of the reference
            sc = float(self.cfg.hidden_size) ** 0.5
            return ((y.float() / sc).to(self.dtype).float() * self.cfg.embed_scale).to(self.dtype)
        x = self.pixel_shuffle(f, self.scale_factor)
        return ops.gemm(x.reshape(-1, x.shape[-1]).contiguous(), self.proj_w)

    def _pixels(self, image) -> torch.Tensor:
        size = self.vision.cfg.image_size
        t = _resize(_image_tensor(image), size, size)
        m = torch.tensor(self.image_mean)[:, None, None]
        s = torch.tensor(self.image_std)[:, None, None]
        return (t - m) / s

    def _image_token_run(self, n_tiles: int, rows: int, cols: int) -> list[int]:
        """SmolVLM prompt of one tiled image (SmolVLM2.swift:208-232)."""
        mk = self.marker_ids
        run = []
        for r in range(rows):
            for c in range(cols):
                run += [mk["fake"]] + list(mk["row"](r, c)) + [self.image_token_id] * self.mm_tokens
            run += list(mk["newline"])
        run += list(mk["newline"]) + [mk["fake"]] + list(mk["global"]) + [self.image_token_id] * self.mm_tokens
        return run + [mk["fake"]]

    @torch.no_grad()
    def prepare(self, prompt_tokens: list[int], media) -> tuple[list[int], dict | None]:
        """Expand the image placeholders and encode the images. Returns
        (tokens, mm) with mm = {embeds, image_pos, prompt_len, delta[, prefix_lm]};
        positions stay 1-D."""
        images = list(getattr(media, "images", None) or []) if media is not None else []
        if not images:
            return list(prompt_tokens), None
        it = self.image_token_id
        toks = list(prompt_tokens)
        if self.kind == "idefics3" and self.marker_ids and self.tile_longest_edge:
            if len(images) != 1:
                raise ValueError("SmolVLM serves one image per request")
            tile = self.vision.cfg.image_size
            tiles, rows, cols = smolvlm_tiles(images[0], tile, self.tile_longest_edge)
            m = torch.tensor(self.image_mean)[:, None, None]
            s = torch.tensor(self.image_std)[:, None, None]
            pix = torch.stack([(t - m) / s for t in tiles])
            run = self._image_token_run(len(tiles), rows, cols) if rows * cols > 1 else (
                [self.marker_ids["fake"]] + list(self.marker_ids["global"]) + [it] * self.mm_tokens
                + [self.marker_ids["fake"]])
            if rows * cols == 1:
                pix = pix[-1:]
            if it in toks:
                j = toks.index(it)
                toks = toks[:j] + run + toks[j + 1:]
            else:
                j = len(toks) // 2
                toks = toks[:j] + run + toks[j:]
        else:
            pix = torch.stack([self._pixels(im) for im in images])
            n_ph = sum(1 for t in toks if t == it)
            if n_ph == 0:
                run = [it] * (self.mm_tokens * len(images))
                j = 0 if self.kind == "paligemma" else len(toks) // 2
                toks = toks[:j] + run + toks[j:]
            elif n_ph == len(images):
                out = []
                for t in toks:
                    out.extend([t] * self.mm_tokens if t == it else [t])
                toks = out
            elif n_ph != self.mm_tokens * len(images):
                raise ValueError(f"{n_ph} image tokens for {len(images)} images of {self.mm_tokens} tokens")
        emb = self.image_embeddings(pix)
        image_pos = [i for i, t in enumerate(toks) if t == it]
        if len(image_pos) != emb.shape[0]:
            raise ValueError(f"{len(image_pos)} image tokens for {emb.shape[0]} image features")
        mm = {"embeds": emb, "image_pos": torch.tensor(image_pos), "prompt_len": len(toks), "delta": 0}
        if self.prefix_lm:
            mm["prefix_lm"] = True
        return toks, mm

    def forward(self, fb, kv, return_hidden: bool = False, inputs_embeds=None, return_both=False,
                return_residual=False):
        states = getattr(fb, "row_states", None)
        rows = []
        whole_prompts = True
        if inputs_embeds is None and states:
            nd = fb.num_decode
            pf = fb.pf_cu_q_host or [0]
            for i, st in enumerate(states):
                if i < nd:
                    continue
                mm = st.req.mm if st is not None else None
                a, n = nd + pf[i - nd], pf[i - nd + 1] - pf[i - nd]
                p0 = int(fb.pf_pos0_host[i - nd])
                if mm is None or not mm.get("prefix_lm") or p0 != 0 or n != mm["prompt_len"]:
                    whole_prompts = False
                if mm is not None:
                    rows.append((a, n, p0, mm))
        if self.prefix_lm and rows and whole_prompts and fb.num_tokens > fb.num_decode:
            # prefix-LM: every prefill row is a whole image + text prompt
            fb.bidirectional = True
        if not rows:
            return super().forward(fb, kv, return_hidden, inputs_embeds, return_both, return_residual)
        x = ops.embedding(fb.input_ids, self.embed, self.cfg.embed_scale).clone()
        for a, n, p0, mm in rows:
            ip = mm["image_pos"]
            sel = ((ip >= p0) & (ip < p0 + n)).nonzero()[:, 0]
            if len(sel):
                x[(ip[sel] - p0 + a).to(x.device)] = mm["embeds"][sel.to(mm["embeds"].device)].to(x.dtype)
        try:
            return super().forward(fb, kv, return_hidden, x, return_both, return_residual)
        finally:
            if self.prefix_lm:
                fb.bidirectional = False


class Gemma3VLModel(SiglipVLM):
    """Gemma 3 language model + SigLIP tower + pooled projector."""

    def __init__(self, cfg, vision_cfg: SiglipConfig, device="cpu", dtype=torch.float32,
                 image_token_id: int = 262144, mm_tokens: int = 256):
        super().__init__(cfg, vision_cfg, device, dtype, "gemma3", image_token_id, mm_tokens)
