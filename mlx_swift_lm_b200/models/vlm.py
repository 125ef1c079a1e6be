"""Qwen2-VL / Qwen2.5-VL / Qwen3-VL vision-language models: the fused
decoder plus a vision tower, multimodal rows and M-RoPE.

Qwen3-VL (MLXVLM/Models/Qwen3VL.swift) interleaves the M-RoPE frequencies
(frequency i follows the h position when i % 3 == 1 and the w position when
i % 3 == 2, within 3 x section, else the t position) and adds the vision
tower's deepstack features to the hidden states of the image tokens after
the first decoder layers.

Parity: MLXVLM/Models/Qwen2VL.swift - ``getRopeIndex`` (:345: text runs get
equal (t, h, w) positions, an image of grid (t, h, w) / merge gets the 3-D
grid positions after the preceding text, later text resumes at max + 1; the
per-request delta max + 1 - length continues decoding), M-RoPE (:33: the
rotary frequencies split into sections driven by the t, h and w positions),
vision embeddings merged over the image placeholder tokens (QwenVL.swift:63),
and the placeholder expansion of the processor (:835). Multimodal rows of
the continuous-batching engine (ContinuousBatchingV2/MultimodalV2.swift:43).

In the engine a multimodal request carries ``Request.mm``
(:meth:`Qwen2VLModel.prepare`): the vision embeddings of its image tokens and
the 3-D positions of its prompt. A forward batch that holds any of its prompt
tokens gets (a) those embeddings written over the placeholder rows of the
token embeddings and (b) a per-token rotary table (``fb.rope_table``) from
the 3-D positions; generated tokens use the 1-D position p + delta, so decode
steps (and their CUDA graphs) need nothing special.
"""
from __future__ import annotations

import torch

from .. import ops
from ..api.media import MediaConfig, MediaInput, process_image, process_video
from .decoder import DecoderLM
from .vision import QwenVisionTower, VisionConfig


def get_rope_index(tokens: list[int], grids: list[tuple[int, int, int]], image_token: int, video_token: int,
                   merge: int) -> tuple[torch.Tensor, int]:
    """3-D positions [3, L] of a prompt and its decode delta. `grids` are the
    (t, h, w) patch grids of the prompt's images / videos in order."""
    L = len(tokens)
    out = torch.zeros(3, L, dtype=torch.long)
    st, nxt, gi = 0, 0, 0
    while st < L:
        ed = next((i for i in range(st, L) if tokens[i] in (image_token, video_token)), L)
        n = ed - st  # text run
        out[:, st:ed] = torch.arange(nxt, nxt + n)[None]
        nxt += n
        if ed >= L or gi >= len(grids):
            if ed < L:  # placeholders without a grid: positioned as text
                out[:, ed:] = torch.arange(nxt, nxt + L - ed)[None]
                nxt += L - ed
            break
        t, h, w = grids[gi]
        gi += 1
        lh, lw = h // merge, w // merge
        cnt = t * lh * lw
        tt = torch.arange(t)[:, None].expand(t, lh * lw).reshape(-1)
        hh = torch.arange(lh)[None, :, None].expand(t, lh, lw).reshape(-1)
        ww = torch.arange(lw)[None, None, :].expand(t, lh, lw).reshape(-1)
        out[:, ed:ed + cnt] = torch.stack([tt, hh, ww]) + nxt
        nxt = int(out[:, ed:ed + cnt].max()) + 1
        st = ed + cnt
    return out, int(out.max()) + 1 - L if L else 0


class Qwen2VLModel(DecoderLM):
    def __init__(self, cfg, vision_cfg: VisionConfig, device="cpu", dtype=torch.float32, image_token_id: int = 151655,
                 video_token_id: int = 151656, mrope_section=(16, 24, 24)):
        super().__init__(cfg, device, dtype)
        self.vision = QwenVisionTower(vision_cfg, device, dtype)
        self.image_token_id, self.video_token_id = image_token_id, video_token_id
        self.mrope_section = list(mrope_section)
        self.media_cfg = MediaConfig(patch_size=vision_cfg.patch_size,
                                     temporal_patch_size=vision_cfg.temporal_patch_size,
                                     merge_size=vision_cfg.spatial_merge_size)
        half = self.rot_dim // 2
        assert sum(self.mrope_section) == half, "mrope sections must cover the rotary half-dimension"
        base = cfg.rope_theta
        self._inv = 1.0 / (base ** (torch.arange(0, self.rot_dim, 2, dtype=torch.float64) / self.rot_dim))
        sec = torch.zeros(half, dtype=torch.long)
        o = 0
        for i, s in enumerate(self.mrope_section):
            sec[o:o + s] = i
            o += s
        self._sec = sec

    def init_random(self, seed: int = 0, std: float = 0.02, with_embeddings: bool = True, keep_layers=None):
        super().init_random(seed, std, with_embeddings, keep_layers)
        self.vision.init_random(seed + 17, std)
        return self

    def clone_to(self, device, dtype):
        m = super().clone_to(device, dtype)
        out = Qwen2VLModel(self.cfg, self.vision.cfg, device, dtype, self.image_token_id, self.video_token_id,
                           self.mrope_section)
        out.embed, out.norm, out.lm_head, out.layers = m.embed, m.norm, m.lm_head, m.layers
        out.vision = QwenVisionTower(self.vision.cfg)
        for n, t in self.vision.tensors():
            if t is None:
                continue
            if n.startswith("blocks."):
                _, i, s = n.split(".")
                from .vision import VisionBlock

                while len(out.vision.blocks) <= int(i):
                    out.vision.blocks.append(VisionBlock())
                setattr(out.vision.blocks[int(i)], s, t)
            else:
                setattr(out.vision, n, t)
        out.vision.to(device, dtype)
        return out

    # ------------------------------------------------------------------ requests
    @torch.no_grad()
    def prepare(self, prompt_tokens: list[int], media: MediaInput | None) -> tuple[list[int], dict | None]:
        """Expand each image / video placeholder token to its merged patch
        count, encode the media with the vision tower, and compute the 3-D
        positions. Returns (tokens, mm) with mm = {embeds [n, H], image_pos
        (prompt indices of the placeholder tokens), pos3 [3, L], delta}."""
        media = media or MediaInput()
        items = [("image", x) for x in media.images] + [("video", x) for x in media.videos]
        if not items:
            return list(prompt_tokens), None
        merge2 = self.vision.cfg.spatial_merge_size ** 2
        patches, grids, kinds = [], [], []
        imgs, vids = iter(media.images), iter(media.videos)
        toks = []
        for t in prompt_tokens:
            if t == self.image_token_id or t == self.video_token_id:
                src = next(imgs) if t == self.image_token_id else next(vids)
                p, g = (process_image(src, self.media_cfg) if t == self.image_token_id
                        else process_video(src, self.media_cfg))
                patches.append(p)
                grids.append(g)
                toks.extend([t] * (g[0] * g[1] * g[2] // merge2))
            else:
                toks.append(t)
        emb = self.vision.forward(torch.cat(patches), grids)
        pos3, delta = get_rope_index(toks, grids, self.image_token_id, self.video_token_id,
                                     self.vision.cfg.spatial_merge_size)
        image_pos = [i for i, t in enumerate(toks) if t in (self.image_token_id, self.video_token_id)]
        assert len(image_pos) == emb.shape[0]
        return toks, {"embeds": emb, "image_pos": torch.tensor(image_pos), "pos3": pos3, "delta": delta,
                      "prompt_len": len(toks)}

    def _rope_rows(self, pos3: torch.Tensor) -> torch.Tensor:
        """cos | sin [n, rot_dim] of 3-D positions [3, n] (sectioned frequencies)."""
        p = pos3.double()[self._sec]  # [half, n]: the position driving each frequency
        ang = p.t() * self._inv[None]
        return torch.cat([ang.cos(), ang.sin()], -1).float()

    # ------------------------------------------------------------------ forward
    def forward(self, fb, kv, return_hidden: bool = False, inputs_embeds=None, return_both=False,
                return_residual=False):
        states = getattr(fb, "row_states", None)
        mm_rows = []
        if inputs_embeds is None and states:
            nd = fb.num_decode
            pf = fb.pf_cu_q_host or [0]
            for i, st in enumerate(states):
                mm = st.req.mm if st is not None else None
                if mm is None or i < nd:
                    continue
                a = nd + pf[i - nd]
                n = pf[i - nd + 1] - pf[i - nd]
                p0 = int(fb.pf_pos0_host[i - nd]) if getattr(fb, "pf_pos0_host", None) else None
                mm_rows.append((a, n, p0, mm))
        if not mm_rows:
            return super().forward(fb, kv, return_hidden, inputs_embeds, return_both, return_residual)
        x = ops.embedding(fb.input_ids, self.embed, self.cfg.embed_scale).clone()
        # 1-D positions of every token, then 3-D rows for the multimodal prompt tokens
        pos_all = fb.positions.to("cpu").long()
        table = self._rope_rows(pos_all[None].expand(3, -1))
        for a, n, p0, mm in mm_rows:
            if p0 is None:
                p0 = int(pos_all[a])
            plen = mm["prompt_len"]
            k = min(n, max(0, plen - p0))
            if k:
                table[a:a + k] = self._rope_rows(mm["pos3"][:, p0:p0 + k])
            ip = mm["image_pos"]
            sel = ((ip >= p0) & (ip < p0 + n)).nonzero()[:, 0]
            if len(sel):
                rows = (ip[sel] - p0 + a).to(x.device)
                x[rows] = mm["embeds"][sel.to(mm["embeds"].device)].to(x.dtype)
        fb.rope_table = table.to(x.device)
        try:
            return super().forward(fb, kv, return_hidden, x, return_both, return_residual)
        finally:
            fb.rope_table = None


class Qwen3VLModel(Qwen2VLModel):
    """Qwen3-VL: interleaved M-RoPE and deepstack injection (see the module doc)."""

    def __init__(self, cfg, vision_cfg: VisionConfig, device="cpu", dtype=torch.float32, image_token_id: int = 151655,
                 video_token_id: int = 151656, mrope_section=(24, 20, 20)):
        super().__init__(cfg, vision_cfg, device, dtype, image_token_id, video_token_id, mrope_section)
        half = self.rot_dim // 2
        sec = torch.zeros(half, dtype=torch.long)
        for axis in (1, 2):
            for i in range(axis, 3 * self.mrope_section[axis], 3):
                sec[i] = axis
        self._sec = sec

    def clone_to(self, device, dtype):
        m = super().clone_to(device, dtype)
        out = Qwen3VLModel(self.cfg, self.vision.cfg, device, dtype, self.image_token_id, self.video_token_id,
                           self.mrope_section)
        out.embed, out.norm, out.lm_head, out.layers = m.embed, m.norm, m.lm_head, m.layers
        out.vision = m.vision
        out.vision.deep = [dict(d) for d in self.vision.deep]
        out.vision.patch_b, out.vision.pos_embed = self.vision.patch_b, self.vision.pos_embed
        out.vision.to(device, dtype)
        return out

    @torch.no_grad()
    def prepare(self, prompt_tokens: list[int], media: MediaInput | None) -> tuple[list[int], dict | None]:
        vis = self.vision
        fwd = vis.forward
        deep: list = []

        def forward(patches, grids):  # keep the deepstack features next to the merged embeddings
            out, d = fwd(patches, grids)
            deep.extend(d)
            return out

        vis.forward = forward
        try:
            toks, mm = super().prepare(prompt_tokens, media)
        finally:
            del vis.forward
        if mm is not None:
            mm["deep"] = deep
        return toks, mm

    def forward(self, fb, kv, return_hidden: bool = False, inputs_embeds=None, return_both=False,
                return_residual=False):
        states = getattr(fb, "row_states", None)
        rows = []
        if inputs_embeds is None and states:
            nd = fb.num_decode
            pf = fb.pf_cu_q_host or [0]
            for i, st in enumerate(states):
                mm = st.req.mm if st is not None else None
                if mm is None or i < nd or not mm.get("deep"):
                    continue
                a, n = nd + pf[i - nd], pf[i - nd + 1] - pf[i - nd]
                p0 = int(fb.pf_pos0_host[i - nd])
                ip = mm["image_pos"]
                sel = ((ip >= p0) & (ip < p0 + n)).nonzero()[:, 0]
                if len(sel):
                    rows.append(((ip[sel] - p0 + a), sel, mm["deep"]))
        if not rows:
            return super().forward(fb, kv, return_hidden, inputs_embeds, return_both, return_residual)
        n_deep = max(len(d) for _, _, d in rows)

        def hook(li, x, delta):
            if li >= n_deep:
                return x, delta
            x = (x.float() + delta.float()).to(x.dtype) if delta is not None else x
            for r, sel, d in rows:
                if li < len(d):
                    rr = r.to(x.device)
                    x[rr] = (x[rr].float() + d[li][sel.to(d[li].device)].float()).to(x.dtype)
            return x, None

        self._after_layer = hook
        try:
            return super().forward(fb, kv, return_hidden, inputs_embeds, return_both, return_residual)
        finally:
            self._after_layer = None
