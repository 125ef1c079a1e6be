"""Qwen2-VL, Qwen2.5-VL and Qwen3-VL vision towers on the decoder's kernels.

Qwen3-VL (MLXVLM/Models/Qwen3VL.swift) keeps Qwen2-VL's LayerNorm blocks and
2-D rotary embedding, adds a bias to the patch embedding and a learned
position embedding on a fixed square grid that is bilinearly resampled to
each image's patch grid, uses a GELU-tanh MLP (``linear_fc1`` / ``linear_fc2``),
normalises before the 2x2 merge, and taps the hidden states after its
``deepstack_visual_indexes`` blocks through extra mergers (normalising after
the merge): those "deepstack" features are added to the language model's
hidden states at the image positions after its first layers.

Qwen2.5-VL (MLXVLM/Models/Qwen25VL.swift) changes the blocks to RMSNorm and a
biased SwiGLU MLP, attends within windows of ``window_size`` pixels except in
its ``fullatt_block_indexes`` blocks (patches reordered window by window, in
units of merged 2x2 patches, and restored after the merger), and merges with
an RMSNorm.

Parity: MLXVLM/Models/Qwen2VL.swift:513-790 and QwenVL.swift:90-160 -
patch embedding (a Conv3d whose kernel equals its stride, i.e. one linear map
of each flattened [C, t, p, p] patch), pre-norm blocks (LayerNorm, fused qkv
with bias, 2-D rotary embedding over (row, column) patch positions with
rotate-half, bidirectional attention within each frame, quick-GELU MLP) and
the patch merger (LayerNorm, 2x2 neighbouring patches concatenated, GELU
MLP into the language model's hidden size).

B200 path: GEMMs with bias / GELU epilogues, the fused residual + LayerNorm
kernel, and the tensor-core paged prefill kernel in bidirectional mode over
a scratch page pool (one row per frame). The 2-D rotary angles of every
patch are tabulated per token and handed to the qk/RoPE/KV-write kernel as
its cos/sin table with positions 0..N-1.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops
from ..kv.paged import PAGE
from ..ops import reference as ref
from .encoder import scratch_layout


@dataclass
class VisionConfig:
    depth: int = 32
    embed_dim: int = 1280
    num_heads: int = 16
    mlp_ratio: float = 4.0
    patch_size: int = 14
    temporal_patch_size: int = 2
    spatial_merge_size: int = 2
    in_chans: int = 3
    hidden_size: int = 3584  # language model hidden size (merger output)
    eps: float = 1e-6
    kind: str = "qwen2"  # "qwen2" | "qwen2_5" | "qwen3"
    intermediate_size: int = 0  # qwen2_5: SwiGLU width
    window_size: int = 112  # qwen2_5: attention window in pixels
    fullatt_blocks: tuple = ()  # qwen2_5: blocks attending whole frames
    num_pos: int = 0  # qwen3: learned position embeddings (a square grid)
    deepstack: tuple = ()  # qwen3: blocks whose outputs feed the deepstack mergers

    @property
    def head_dim(self) -> int:
        return self.embed_dim // self.num_heads

    @property
    def patch_dim(self) -> int:
        return self.in_chans * self.temporal_patch_size * self.patch_size * self.patch_size

    @classmethod
    def from_hf(cls, vc: dict, text_hidden: int, kind: str = "qwen2") -> "VisionConfig":
        common = dict(depth=vc.get("depth", 32), num_heads=vc.get("num_heads", 16),
                      patch_size=vc.get("patch_size", 14), temporal_patch_size=vc.get("temporal_patch_size", 2),
                      spatial_merge_size=vc.get("spatial_merge_size", 2),
                      in_chans=vc.get("in_chans", vc.get("in_channels", 3)))
        if kind == "qwen3":
            return cls(embed_dim=vc.get("hidden_size", 1152), hidden_size=vc.get("out_hidden_size", text_hidden),
                       intermediate_size=vc.get("intermediate_size", 4304), num_pos=vc.get("num_position_embeddings",
                                                                                            2304),
                       deepstack=tuple(vc.get("deepstack_visual_indexes", ())), kind="qwen3", **common)
        if kind == "qwen2_5":  # hidden_size is the tower width, out_hidden_size the language model's
            return cls(embed_dim=vc.get("hidden_size", 1280), hidden_size=vc.get("out_hidden_size", text_hidden),
                       intermediate_size=vc.get("intermediate_size", 3420), window_size=vc.get("window_size", 112),
                       fullatt_blocks=tuple(vc.get("fullatt_block_indexes", (7, 15, 23, 31))), kind="qwen2_5",
                       **common)
        return cls(embed_dim=vc.get("embed_dim", 1280), mlp_ratio=vc.get("mlp_ratio", 4.0),
                   hidden_size=vc.get("hidden_size", text_hidden), **common)


def _swiglu(gate, up, gate_b, up_b, down):
    """Fused SwiGLU operands: gate/up rows (and biases) interleaved in 64-row
    blocks, the width padded with zero rows to a multiple of 64 (zero gate and
    up give a zero product, and the matching zero columns of down add nothing)."""
    I = gate.shape[0]
    pad = -I % 64
    if pad:
        z = lambda t: torch.cat([t, t.new_zeros((pad,) + tuple(t.shape[1:]))], 0)  # noqa: E731
        gate, up, gate_b, up_b = z(gate), z(up), z(gate_b), z(up_b)
        down = torch.cat([down, down.new_zeros(down.shape[0], pad)], 1)
    gu_w = ref.interleave_gate_up(gate, up)
    gu_b = ref.interleave_gate_up(gate_b[:, None], up_b[:, None])[:, 0].contiguous()
    return gu_w, gu_b, down.contiguous()


class VisionBlock:
    __slots__ = ("norm1_w", "norm1_b", "qkv_w", "qkv_b", "proj_w", "proj_b", "norm2_w", "norm2_b", "fc1_w", "fc1_b",
                 "fc2_w", "fc2_b",
                 # qwen2_5: SwiGLU gate/up (64-row interleaved, with biases) and down projections
                 "gu_w", "gu_b", "dn_w", "dn_b")

    def __init__(self):
        for s in self.__slots__:
            setattr(self, s, None)


class QwenVisionTower:
    def __init__(self, cfg: VisionConfig, device="cpu", dtype=torch.float32):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.patch_w = self.patch_b = self.pos_embed = None  # qwen3: patch bias, position grid
        self.deep: list[dict] = []  # qwen3: deepstack mergers (post-merge LayerNorm + GELU MLP)
        self.blocks: list[VisionBlock] = []
        self.ln_q_w = self.ln_q_b = None
        self.m1_w = self.m1_b = self.m2_w = self.m2_b = None
        d = cfg.head_dim // 2
        self.inv_freq = 1.0 / (10000.0 ** (torch.arange(0, d, 2, dtype=torch.float64) / d))

    def init_random(self, seed: int = 0, std: float = 0.02):
        c = self.cfg
        g = torch.Generator(device=self.device).manual_seed(seed)
        E, F = c.embed_dim, int(c.embed_dim * c.mlp_ratio)
        M = E * c.spatial_merge_size ** 2

        def rn(*shape):
            return torch.empty(shape, device=self.device, dtype=self.dtype).normal_(0.0, std, generator=g)

        def ones(n):
            return torch.ones(n, device=self.device, dtype=self.dtype)

        self.patch_w = rn(E, c.patch_dim)
        q3 = c.kind == "qwen3"
        if q3:
            F = c.intermediate_size
            self.patch_b, self.pos_embed = rn(E), rn(c.num_pos, E)
            self.deep = [{"norm_w": ones(M), "norm_b": rn(M), "fc1_w": rn(M, M), "fc1_b": rn(M),
                          "fc2_w": rn(c.hidden_size, M), "fc2_b": rn(c.hidden_size)} for _ in c.deepstack]
        self.blocks = []
        q25 = c.kind == "qwen2_5"
        for _ in range(c.depth):
            b = VisionBlock()
            b.qkv_w, b.qkv_b = rn(3 * E, E), rn(3 * E)
            b.proj_w, b.proj_b = rn(E, E), rn(E)
            if q25:
                I = c.intermediate_size
                b.norm1_w, b.norm2_w = ones(E), ones(E)
                b.gu_w, b.gu_b, b.dn_w = _swiglu(rn(I, E), rn(I, E), rn(I), rn(I), rn(E, I))
                b.dn_b = rn(E)
            else:
                b.norm1_w, b.norm1_b, b.norm2_w, b.norm2_b = ones(E), rn(E), ones(E), rn(E)
                b.fc1_w, b.fc1_b, b.fc2_w, b.fc2_b = rn(F, E), rn(F), rn(E, F), rn(E)
            self.blocks.append(b)
        self.ln_q_w, self.ln_q_b = ones(E), (None if q25 else rn(E))
        self.m1_w, self.m1_b, self.m2_w, self.m2_b = rn(M, M), rn(M), rn(c.hidden_size, M), rn(c.hidden_size)
        return self

    def tensors(self):
        for n in ("patch_w", "patch_b", "pos_embed", "ln_q_w", "ln_q_b", "m1_w", "m1_b", "m2_w", "m2_b"):
            yield n, getattr(self, n)
        for i, b in enumerate(self.blocks):
            for s in VisionBlock.__slots__:
                yield f"blocks.{i}.{s}", getattr(b, s)
        for j, d in enumerate(self.deep):
            for k, v in d.items():
                yield f"deep.{j}.{k}", v

    def to(self, device, dtype):
        self.device, self.dtype = torch.device(device), dtype
        for n, v in list(self.tensors()):
            if v is None:
                continue
            if n.startswith("blocks."):
                _, i, s = n.split(".")
                setattr(self.blocks[int(i)], s, v.to(self.device, dtype).contiguous())
            elif n.startswith("deep."):
                _, j, k = n.split(".")
                self.deep[int(j)][k] = v.to(self.device, dtype).contiguous()
            else:
                setattr(self, n, v.to(self.device, dtype).contiguous())
        return self

    # ------------------------------------------------------------------ positions
    def rotary_table(self, grids: list[tuple[int, int, int]]) -> torch.Tensor:
        """Per-patch cos | sin [N, head_dim] fp32 in patchify order: angles of
        the row position on the first quarter of the frequencies and of the
        column position on the second (rotate-half over the head)."""
        m = self.cfg.spatial_merge_size
        hs, ws = [], []
        for t, h, w in grids:
            hp = torch.arange(h)[:, None].expand(h, w).reshape(h // m, m, w // m, m).permute(0, 2, 1, 3).reshape(-1)
            wp = torch.arange(w)[None, :].expand(h, w).reshape(h // m, m, w // m, m).permute(0, 2, 1, 3).reshape(-1)
            hs.append(hp.repeat(t))
            ws.append(wp.repeat(t))
        hp, wp = torch.cat(hs).double(), torch.cat(ws).double()
        ang = torch.cat([hp[:, None] * self.inv_freq[None], wp[:, None] * self.inv_freq[None]], -1)
        return torch.cat([ang.cos(), ang.sin()], -1).float().to(self.device)

    def position_rows(self, grids: list[tuple[int, int, int]]) -> torch.Tensor:
        """qwen3: learned position embedding of every patch [N, E] in patchify
        order: the square grid of ``num_pos`` embeddings bilinearly resampled
        to the frame's h x w patches (corner-aligned sample points), repeated
        over frames, in merge-window order."""
        c = self.cfg
        n = int(round(c.num_pos ** 0.5))
        m = c.spatial_merge_size
        grid = self.pos_embed.float().view(n, n, -1)
        out = []
        for t, h, w in grids:
            hy = torch.linspace(0, n - 1, h, dtype=torch.float32)
            wx = torch.linspace(0, n - 1, w, dtype=torch.float32)
            h0, w0 = hy.long(), wx.long()
            h1, w1 = (h0 + 1).clamp(max=n - 1), (w0 + 1).clamp(max=n - 1)
            dh, dw = (hy - h0)[:, None, None].to(grid.device), (wx - w0)[None, :, None].to(grid.device)
            e = ((1 - dh) * (1 - dw) * grid[h0][:, w0] + (1 - dh) * dw * grid[h0][:, w1]
                 + dh * (1 - dw) * grid[h1][:, w0] + dh * dw * grid[h1][:, w1])  # [h, w, E]
            e = e.reshape(h // m, m, w // m, m, -1).permute(0, 2, 1, 3, 4).reshape(h * w, -1)
            out.append(e.repeat(t, 1))
        return torch.cat(out).to(self.dtype)

    def window_index(self, grids: list[tuple[int, int, int]]):
        """(order of the merged units window by window, window lengths in
        patches): units of each frame grouped into windows of
        window_size / merge / patch units per side, row-major over windows."""
        c = self.cfg
        m = c.spatial_merge_size
        ws = c.window_size // m // c.patch_size
        order, lens, base = [], [], 0
        for t, h, w in grids:
            gh, gw = h // m, w // m
            idx = torch.arange(t * gh * gw).reshape(t, gh, gw)
            nh, nw = -(-gh // ws), -(-gw // ws)
            for ti in range(t):
                for wi in range(nh):
                    for wj in range(nw):
                        blk = idx[ti, wi * ws:(wi + 1) * ws, wj * ws:(wj + 1) * ws].reshape(-1)
                        if blk.numel():
                            order.append(blk + base)
                            lens.append(blk.numel() * m * m)
            base += t * gh * gw
        return torch.cat(order), lens

    # ------------------------------------------------------------------ forward
    @torch.no_grad()
    def forward(self, patches: torch.Tensor, grids: list[tuple[int, int, int]]) -> torch.Tensor:
        """patches [N, C*tp*p*p] -> merged embeddings [N / merge^2, hidden]."""
        c = self.cfg
        dev, E, NH, D = self.device, c.embed_dim, c.num_heads, c.head_dim
        q25 = c.kind == "qwen2_5"
        q3 = c.kind == "qwen3"
        U = c.spatial_merge_size ** 2
        x = ops.gemm(patches.to(dev, self.dtype).contiguous(), self.patch_w, bias=self.patch_b)
        N = x.shape[0]
        if q3:
            x = (x.float() + self.position_rows(grids).float()).to(self.dtype)
        deep = []
        table = self.rotary_table(grids)
        frames = [h * w for t, h, w in grids for _ in range(t)]  # attention within each frame

        def layout(lens):
            pt, slots, cu, npages = scratch_layout(lens, dev)
            return (pt, slots, cu, torch.tensor(cu, dtype=torch.int32, device=dev),
                    torch.zeros(len(lens), dtype=torch.int32, device=dev), npages)

        full = layout(frames)
        if q25:  # window order of merged units; the full-attention frames stay contiguous in it
            order, wlens = self.window_index(grids)
            order = order.to(dev)
            perm = (order[:, None] * U + torch.arange(U, device=dev)[None]).reshape(-1)
            x = x.index_select(0, perm).contiguous()
            table = table.index_select(0, perm).contiguous()
            win = layout(wlens)
        npages = max(full[5], win[5]) if q25 else full[5]
        kc = torch.zeros(npages, NH, PAGE, D, dtype=self.dtype, device=dev)
        vc = torch.zeros_like(kc)
        tok = torch.arange(N, dtype=torch.int32, device=dev)
        delta = None
        for i, b in enumerate(self.blocks):
            pt, slots, cu, cu_t, pos0, _ = win if q25 and i not in c.fullatt_blocks else full
            if q25:
                h = ops.add_rmsnorm(x, delta, b.norm1_w, c.eps)
            else:
                h = ops.add_layernorm(x, delta, b.norm1_w, b.norm1_b, c.eps)
            qkv = ops.gemm(h, b.qkv_w, bias=b.qkv_b)
            q = ops.qk_norm_rope_kv(qkv, tok, slots, table, D, False, None, None, c.eps, kc, vc, NH, NH, D)
            a = ops.paged_prefill(q, kc, vc, pt, cu_t, pos0, D ** -0.5, -1, cu_q_host=cu)
            d = ops.gemm(a.reshape(N, E), b.proj_w, bias=b.proj_b)
            if q25:
                h = ops.add_rmsnorm(x, d, b.norm2_w, c.eps)
                delta = ops.gemm(ops.gemm(h, b.gu_w, epi="swiglu", bias=b.gu_b), b.dn_w, bias=b.dn_b)
            else:
                h = ops.add_layernorm(x, d, b.norm2_w, b.norm2_b, c.eps)
                act = "gelu_tanh" if q3 else "quick_gelu"
                delta = ops.gemm(ops.gemm(h, b.fc1_w, epi=act, bias=b.fc1_b), b.fc2_w, bias=b.fc2_b)
            if q3 and i in c.deepstack:  # the block's output through its deepstack merger
                dm = self.deep[c.deepstack.index(i)]
                y = (x.float() + delta.float()).to(self.dtype).reshape(N // U, -1).contiguous()
                y = ops.add_layernorm(y, None, dm["norm_w"], dm["norm_b"], c.eps)
                deep.append(ops.gemm(ops.gemm(y, dm["fc1_w"], epi="gelu", bias=dm["fc1_b"]), dm["fc2_w"],
                                     bias=dm["fc2_b"]))
        if q25:
            hq = ops.add_rmsnorm(x, delta, self.ln_q_w, c.eps)
        else:
            hq = ops.add_layernorm(x, delta, self.ln_q_w, self.ln_q_b, c.eps)
        hq = hq.reshape(N // U, -1).contiguous()
        out = ops.gemm(ops.gemm(hq, self.m1_w, epi="gelu", bias=self.m1_b), self.m2_w, bias=self.m2_b)
        if q25:  # back to patchify order
            out = out.index_select(0, torch.argsort(order)).contiguous()
        if q3:
            return out, deep
        return out

    # ------------------------------------------------------------------ loading
    @classmethod
    def from_tensors(cls, cfg: VisionConfig, t: dict, device="cpu", dtype=torch.float32) -> "QwenVisionTower":
        pre = next((p for p in ("visual.", "model.visual.", "vision_tower.") if p + "patch_embed.proj.weight" in t),
                   None)
        if pre is None:
            raise KeyError("no Qwen VL vision tower weights (visual.patch_embed.proj.weight)")
        m = cls(cfg)

        def g(n):
            return t[pre + n].float()

        w = g("patch_embed.proj.weight")
        if w.dim() == 5 and w.shape[-1] == cfg.in_chans:  # MLX layout [out, t, p, p, C]
            w = w.permute(0, 4, 1, 2, 3)
        m.patch_w = w.reshape(w.shape[0], -1)
        q25 = cfg.kind == "qwen2_5"
        q3 = cfg.kind == "qwen3"
        if q3:
            m.patch_b, m.pos_embed = g("patch_embed.proj.bias"), g("pos_embed.weight")
            m.deep = [{"norm_w": g(f"deepstack_merger_list.{j}.norm.weight"),
                       "norm_b": g(f"deepstack_merger_list.{j}.norm.bias"),
                       "fc1_w": g(f"deepstack_merger_list.{j}.linear_fc1.weight"),
                       "fc1_b": g(f"deepstack_merger_list.{j}.linear_fc1.bias"),
                       "fc2_w": g(f"deepstack_merger_list.{j}.linear_fc2.weight"),
                       "fc2_b": g(f"deepstack_merger_list.{j}.linear_fc2.bias")} for j in range(len(cfg.deepstack))]
        for i in range(cfg.depth):
            p = f"blocks.{i}."
            b = VisionBlock()
            b.qkv_w, b.qkv_b = g(p + "attn.qkv.weight"), g(p + "attn.qkv.bias")
            b.proj_w, b.proj_b = g(p + "attn.proj.weight"), g(p + "attn.proj.bias")
            if q25:
                b.norm1_w, b.norm2_w = g(p + "norm1.weight"), g(p + "norm2.weight")
                b.gu_w, b.gu_b, b.dn_w = _swiglu(g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight"),
                                                 g(p + "mlp.gate_proj.bias"), g(p + "mlp.up_proj.bias"),
                                                 g(p + "mlp.down_proj.weight"))
                b.dn_b = g(p + "mlp.down_proj.bias")
            else:
                b.norm1_w, b.norm1_b = g(p + "norm1.weight"), g(p + "norm1.bias")
                b.norm2_w, b.norm2_b = g(p + "norm2.weight"), g(p + "norm2.bias")
                fc = ("mlp.linear_fc1", "mlp.linear_fc2") if q3 else ("mlp.fc1", "mlp.fc2")
                b.fc1_w, b.fc1_b = g(p + fc[0] + ".weight"), g(p + fc[0] + ".bias")
                b.fc2_w, b.fc2_b = g(p + fc[1] + ".weight"), g(p + fc[1] + ".bias")
            m.blocks.append(b)
        if q3:
            m.ln_q_w, m.ln_q_b = g("merger.norm.weight"), g("merger.norm.bias")
            m.m1_w, m.m1_b = g("merger.linear_fc1.weight"), g("merger.linear_fc1.bias")
            m.m2_w, m.m2_b = g("merger.linear_fc2.weight"), g("merger.linear_fc2.bias")
            return m.to(device, dtype)
        m.ln_q_w = g("merger.ln_q.weight")
        m.ln_q_b = None if q25 else g("merger.ln_q.bias")
        m.m1_w, m.m1_b = g("merger.mlp.0.weight"), g("merger.mlp.0.bias")
        m.m2_w, m.m2_b = g("merger.mlp.2.weight"), g("merger.mlp.2.bias")
        return m.to(device, dtype)
