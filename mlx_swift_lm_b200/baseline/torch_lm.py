"""Stock-PyTorch build of the decoder: the comparison bar for the sm_100a kernels.

The same weights (the same seeded initialisation as :class:`DecoderLM`), the
same engine (scheduler, page pool, page tables, packed step inputs, CUDA-graph
decode buckets) and the same paged K/V slab, but every model op is a library
call, as a plain PyTorch serving build would write it:

* GEMMs: ``torch.nn.functional.linear`` (cuBLAS / cuBLASLt);
* RMSNorm, SiLU, RoPE, residual adds: torch elementwise ops;
* K/V append: ``index_put_`` into the page slab;
* attention on CUDA: FlashAttention-2 as built by vLLM
  (``vllm.vllm_flash_attn.flash_attn_varlen_func``, ``fa_version=2``),
  reading the page slab in place through the page table (page size 16): one
  call for the decode rows, one for the prefill chunks. This is the
  attention a stock PyTorch serving stack runs; its compiled kernels need no
  JIT. On CPU (tests): ``scaled_dot_product_attention`` over each row's
  pages gathered into a contiguous buffer;
* tensor parallelism: NCCL ``all_reduce`` after the row-parallel projections;
* greedy tokens: ``torch.argmax``.

Scope: dense attention models without sinks or logit softcaps (what the
headline benchmark runs). The reference engine's own comparison arm is its
stock MLX path (Sources/BenchCBv2Core/BenchCBv2RealModel.swift:278-359); this
class plays that role on the B200.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..models.batch import ForwardBatch
from ..models.decoder import DecoderLM

PAGE = 16


class TorchDecoderLM(DecoderLM):
    """:class:`DecoderLM` with every op replaced by a PyTorch / cuBLAS / NCCL call."""

    supports_window_ring = False  # attention reads the row-wide page tables only

    scratch_page = None
    graph_sampling = False  # its engine sampler is greedy-only

    # ------------------------------------------------------------------ engine hooks
    def bind_engine(self, engine):
        """Reserve one page of the engine's pool as the write target of padding
        rows (slot -1) of captured decode graphs, which torch indexing cannot
        skip; the scheduler never hands that page out."""
        self.check_supported()
        self.scratch_page = int(engine.kv.pool.alloc(1)[0])
        engine.sampler = GreedyTorchSampler()
        if engine.graphs is not None:
            engine.graphs.gather_fn = self.gather_tokens
        return self

    def check_supported(self):
        cfg = self.cfg
        bad = [name for name, on in (
            ("attention sinks", cfg.attention_sinks), ("logit softcap", cfg.attn_logit_softcap > 0),
            ("MoE layers", any(L.moe for L in self.layers)), ("linear-attention layers", any(L.linear for L in self.layers)),
            ("LayerNorm", cfg.norm_kind != "rmsnorm"), ("(1 + w) norms", cfg.norm_offset_one),
            ("post-sublayer norms", cfg.post_norms), ("parallel blocks", cfg.parallel_block),
            ("attention output gate", cfg.attn_output_gate), ("interleaved RoPE", cfg.rope_interleaved),
            ("non-SwiGLU MLP", cfg.glu_epi != "swiglu"), ("final softcap", cfg.final_logit_softcap > 0)) if on]
        if bad:
            raise ValueError("the PyTorch baseline serves plain dense decoders; unsupported: " + ", ".join(bad))

    @staticmethod
    def gather_tokens(prev_out, src, host_ids, ids, B):
        """Input ids of a chained decode step: the previous step's device token
        where ``src >= 0``, else the host-supplied id."""
        s = src[:B].long()
        ids[:B] = torch.where(s >= 0, prev_out[s.clamp(min=0)], host_ids[:B])

    # ------------------------------------------------------------------ ops
    def _norm(self, x, delta, w, b=None):
        if delta is not None:
            x.add_(delta)
        return F.rms_norm(x, (x.shape[-1],), w, self.cfg.rms_norm_eps)

    def _linear(self, x, w, b=None):
        return F.linear(x, w, b)

    def _attn_out(self, L, attn2d):
        delta = F.linear(attn2d, L.wo, L.bo if self.tp.rank == 0 else None)
        return self.tp.reduce(delta)

    def _mlp(self, L, h):
        gu = F.linear(h, L.wgu, L.bgu)
        T = gu.shape[0]
        # gate and up rows alternate in blocks of 64 (the fused-epilogue layout of the shared weights)
        g4 = gu.view(T, -1, 2, 64)
        act = (F.silu(g4[:, :, 0]) * g4[:, :, 1]).reshape(T, -1)
        delta = F.linear(act, L.wd, L.bd if self.tp.rank == 0 else None)
        return self.tp.reduce(delta)

    def _rope(self, x, positions):
        """x [T, heads, D] rotated in place over the first rot_dim channels (non-interleaved halves)."""
        rd = self.rot_dim
        if rd == 0:
            return x
        half = rd // 2
        cs = self.cos_sin[positions.long()]
        cos, sin = cs[:, None, :half], cs[:, None, half:]
        x1, x2 = x[..., :half].float(), x[..., half:rd].float()
        r1 = x1 * cos - x2 * sin
        r2 = x2 * cos + x1 * sin
        return torch.cat([r1.to(x.dtype), r2.to(x.dtype), x[..., rd:]], dim=-1)

    def _write_kv(self, cache, slots, vals):
        valid = slots >= 0
        s = torch.where(valid, slots, torch.full_like(slots, self.scratch_page * PAGE))
        pg, off = s // PAGE, s % PAGE
        heads = torch.arange(vals.shape[1], device=vals.device)
        cache.index_put_((pg[:, None], heads[None, :], off[:, None]), vals)

    def _gather(self, cache, pages):
        """cache [P, KVH, 16, D], pages [R, n] -> [R, KVH, n * 16, D] contiguous (one gather)."""
        P, KVH, S, D = cache.shape
        R, n = pages.shape
        flat = cache.view(P * KVH, S, D)
        idx = pages.long()[:, None, :] * KVH + torch.arange(KVH, device=cache.device)[None, :, None]
        return flat[idx.reshape(-1)].view(R, KVH, n * S, D)

    # ------------------------------------------------------------------ attention
    def _attention(self, L, h, fb: ForwardBatch, kv, li: int, attn: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        T, nd = fb.num_tokens, fb.num_decode
        H, KVH, D = self.H, self.KVH, self.D
        G = H // KVH
        ki = self.kv_index[li] if self.kv_index else li
        qkv = F.linear(h, L.wqkv, L.bqkv)
        q = qkv[:, :H * D].view(T, H, D)
        k = qkv[:, H * D:(H + KVH) * D].view(T, KVH, D)
        v = qkv[:, (H + KVH) * D:(H + 2 * KVH) * D].view(T, KVH, D)
        if L.q_norm is not None:
            q = F.rms_norm(q, (D,), L.q_norm, cfg.rms_norm_eps)
            k = F.rms_norm(k, (D,), L.k_norm, cfg.rms_norm_eps)
        q = self._rope(q, fb.positions)
        k = self._rope(k, fb.positions)
        kc, vc = kv.layer(ki)
        self._write_kv(kc, fb.slots, k)
        self._write_kv(vc, fb.slots, v)
        win = cfg.window(li)
        out = attn.view(T, H, D)
        if q.is_cuda:
            self._attention_fa(q, kc, vc, fb, win, out)
            return self._attn_out(L, attn.view(T, H * D))
        if nd:
            pt = fb.dec_page_table[:nd]
            kg, vg = self._gather(kc, pt), self._gather(vc, pt)
            Lk = kg.shape[2]
            kp = torch.arange(Lk, device=q.device)
            sl = fb.dec_seq_lens[:nd].long().clamp(min=1)[:, None]
            mask = kp[None, :] < sl
            if win > 0:
                mask &= kp[None, :] >= sl - win
            # GQA: the group's query heads are the query rows of one KV head
            qd = q[:nd].view(nd, KVH, G, D)
            o = F.scaled_dot_product_attention(qd, kg, vg, attn_mask=mask[:, None, None, :], scale=cfg.scale)
            out[:nd] = o.reshape(nd, H, D)
        if T > nd:
            cu = fb.pf_cu_q_host
            pos0 = fb.pf_pos0_host if fb.pf_pos0_host is not None else fb.pf_pos0.tolist()
            for r in range(len(cu) - 1):
                a, b = nd + cu[r], nd + cu[r + 1]
                Lq, p0 = b - a, int(pos0[r])
                n = p0 + Lq
                npg = (n + PAGE - 1) // PAGE
                pages = fb.pf_page_table[r:r + 1, :npg]
                kg = self._gather(kc, pages)[:, :, :n]
                vg = self._gather(vc, pages)[:, :, :n]
                qr = q[a:b].transpose(0, 1)[None]  # [1, H, Lq, D]
                if p0 == 0 and win <= 0:
                    o = F.scaled_dot_product_attention(qr, kg, vg, is_causal=True, scale=cfg.scale, enable_gqa=True)
                else:
                    qp = torch.arange(p0, n, device=q.device)[:, None]
                    kp = torch.arange(n, device=q.device)[None, :]
                    mask = kp <= qp
                    if win > 0:
                        mask &= kp > qp - win
                    o = F.scaled_dot_product_attention(qr, kg, vg, attn_mask=mask, scale=cfg.scale, enable_gqa=True)
                out[a:b] = o[0].transpose(0, 1)
        return self._attn_out(L, attn.view(T, H * D))

    def _attention_fa(self, q, kc, vc, fb: ForwardBatch, win: int, out):
        from vllm.vllm_flash_attn import flash_attn_varlen_func

        T, nd = fb.num_tokens, fb.num_decode
        # [pages, KVH, 16, D] viewed as [pages, 16, KVH, D]: the kernel takes the strides
        kn, vn = kc.permute(0, 2, 1, 3), vc.permute(0, 2, 1, 3)
        wsz = (win - 1, 0) if win > 0 else (-1, -1)
        if nd:
            if self._dec_cu is None or self._dec_cu.shape[0] < nd + 1 or self._dec_cu.device != q.device:
                self._dec_cu = torch.arange(1024 + 1, dtype=torch.int32, device=q.device)
            flash_attn_varlen_func(
                q[:nd], kn, vn, out=out[:nd], max_seqlen_q=1, cu_seqlens_q=self._dec_cu[:nd + 1],
                max_seqlen_k=fb.dec_page_table.shape[1] * PAGE, seqused_k=fb.dec_seq_lens[:nd].clamp(min=1),
                block_table=fb.dec_page_table[:nd], causal=True, softmax_scale=self.cfg.scale, window_size=wsz,
                fa_version=2)
        if T > nd:
            cu = fb.pf_cu_q_host
            pos0 = fb.pf_pos0_host if fb.pf_pos0_host is not None else fb.pf_pos0.tolist()
            lens = [cu[r + 1] - cu[r] for r in range(len(cu) - 1)]
            kv_lens = [int(p0) + n for p0, n in zip(pos0, lens)]
            flash_attn_varlen_func(
                q[nd:], kn, vn, out=out[nd:], max_seqlen_q=max(lens), cu_seqlens_q=fb.pf_cu_q, max_seqlen_k=max(kv_lens),
                seqused_k=fb.pf_pos0 + (fb.pf_cu_q[1:] - fb.pf_cu_q[:-1]), block_table=fb.pf_page_table,
                causal=True, softmax_scale=self.cfg.scale, window_size=wsz, fa_version=2)

    _dec_cu = None

    # ------------------------------------------------------------------ forward
    def forward(self, fb: ForwardBatch, kv, return_hidden: bool = False, inputs_embeds=None, return_both=False,
                return_residual=False):
        cfg = self.cfg
        T = fb.num_tokens
        x = F.embedding(fb.input_ids.long(), self.embed)
        if cfg.embed_scale != 1.0:
            x = x * cfg.embed_scale
        attn = torch.empty((T, self.H, self.D), dtype=x.dtype, device=x.device)
        delta = None
        for li, L in enumerate(self.layers):
            h = self._norm(x, delta, L.ln1)
            delta = self._attention(L, h, fb, kv, li, attn)
            h = self._norm(x, delta, L.ln2)
            delta = self._mlp(L, h)
        x.add_(delta)
        if fb.logit_idx is not None:
            x = x[fb.logit_idx]
        h = F.rms_norm(x, (x.shape[-1],), self.norm, cfg.rms_norm_eps)
        if return_hidden:
            return h
        logits = F.linear(h, self.lm_head).float()
        return (logits, h) if return_both else logits

    def forward_decode_tokens(self, fb: ForwardBatch, kv, out: torch.Tensor, out2=None, flags=None):
        logits = self.forward(fb, kv)
        out.copy_(torch.argmax(logits, dim=-1).to(torch.int32))
        if flags is not None:
            flags.copy_((~torch.isfinite(logits)).any(-1).to(torch.int32))
        return out


class GreedyTorchSampler:
    """Greedy-only engine sampler built on ``torch.argmax`` (the baseline's
    eager steps: prefill completions)."""

    def sample(self, logits, states, out=None):
        if any(not st.req.sampling.greedy for st in states):
            raise ValueError("the PyTorch baseline arm samples greedily only")
        toks = torch.argmax(logits, dim=-1).to(torch.int32)
        if out is not None:
            out.copy_(toks)
            toks = out
        return toks, None

    @staticmethod
    def logprob_entries(lp_info, toks_host, states):
        return [None] * len(states)
