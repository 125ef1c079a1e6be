"""Plain-PyTorch fp32 restatements of every kernel (the CPU oracles).

These define the semantics the sm_100a kernels must match: the GPU numerics
tests compare each kernel against the function of the same name here, and the
CPU execution path of the framework (benchmark config 1: tiny Qwen3 on CPU in
fp32) runs on them directly. Rounding points mirror the kernels: wherever a
kernel rounds an intermediate to the activation dtype, the oracle rounds to
the input tensor's dtype (a no-op for fp32 tensors).
"""
from __future__ import annotations

import math

import numpy as np
import torch

PAGE = 16
DECODE_PART_TOKENS = 256


# --------------------------------------------------------------------------
# GEMM
# --------------------------------------------------------------------------
def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, block: int = 64) -> torch.Tensor:
    """[F, K] gate and up weights -> [2F, K] with alternating 64-row blocks
    (the layout the fused SwiGLU GEMM epilogue consumes)."""
    F, K = gate.shape
    assert F % block == 0, f"intermediate size {F} must be a multiple of {block}"
    g = gate.reshape(F // block, block, K)
    u = up.reshape(F // block, block, K)
    return torch.stack([g, u], dim=1).reshape(2 * F, K).contiguous()


def deinterleave_gate_up(w: torch.Tensor, block: int = 64):
    F2, K = w.shape
    t = w.reshape(F2 // (2 * block), 2, block, K)
    return t[:, 0].reshape(-1, K), t[:, 1].reshape(-1, K)


def glu_act_ref(epi, g, u):
    if epi == "geglu":
        return torch.nn.functional.gelu(g, approximate="tanh") * u
    if epi == "swiglu_oai":
        g = g.clamp(max=7.0)
        u = u.clamp(-7.0, 7.0)
        return (u + 1.0) * g * torch.sigmoid(1.702 * g)
    return torch.nn.functional.silu(g) * u


def gemm_ref(x, w, epi="none", residual=None, out_dtype=None, bias=None):
    """y = epi(x @ w.T + bias) computed in fp32.
    epi: none | swiglu | geglu | swiglu_oai | f32 | add | gelu | gelu_tanh | quick_gelu | relu2."""
    acc = x.float() @ w.float().t()
    if bias is not None:
        acc = acc + bias.float()
    dt = out_dtype or x.dtype
    if epi in ("swiglu", "geglu", "swiglu_oai"):
        F2 = acc.shape[-1]
        t = acc.reshape(*acc.shape[:-1], F2 // 128, 2, 64)
        g = t[..., 0, :].to(x.dtype).float()
        u = t[..., 1, :].to(x.dtype).float()
        y = glu_act_ref(epi, g, u)
        return y.reshape(*acc.shape[:-1], F2 // 2).to(dt)
    if epi == "f32":
        return acc
    if epi == "add":
        return (acc.to(x.dtype).float() + residual.float()).to(dt)
    if epi in ("gelu", "gelu_tanh"):
        return torch.nn.functional.gelu(acc, approximate="tanh" if epi == "gelu_tanh" else "none").to(dt)
    if epi == "quick_gelu":
        return (acc * torch.sigmoid(1.702 * acc)).to(dt)
    if epi == "relu2":
        return torch.relu(acc).square().to(dt)
    return acc.to(dt)


# --------------------------------------------------------------------------
# norms / rope / embedding
# --------------------------------------------------------------------------
def add_rmsnorm_ref(x, delta, w, eps, offset_one=False):
    """Returns (new_x, normed). new_x = round(x + delta)."""
    if delta is not None:
        r = (x.float() + delta.float()).to(x.dtype)
    else:
        r = x
    rf = r.float()
    inv = torch.rsqrt(rf.pow(2).mean(-1, keepdim=True) + eps)
    ww = w.float() + (1.0 if offset_one else 0.0)
    return r, (rf * inv * ww).to(x.dtype)


def rope_cos_sin(inv_freq: torch.Tensor, max_pos: int, mscale: float = 1.0) -> torch.Tensor:
    """[max_pos, rot_dim] fp32 table: cos then sin, computed in fp64."""
    pos = torch.arange(max_pos, dtype=torch.float64)
    ang = pos[:, None] * inv_freq.double()[None, :]
    return torch.cat([ang.cos() * mscale, ang.sin() * mscale], dim=-1).float().contiguous()


def apply_rope_ref(x, positions, cos_sin, rot_dim, interleaved=False):
    """x: [T, nh, D] float. Returns rotated float tensor (rot_dim 0: unchanged)."""
    if rot_dim == 0:
        return x.float()
    half = rot_dim // 2
    cs = cos_sin[positions.long()]  # [T, rot_dim]
    cos, sin = cs[:, None, :half], cs[:, None, half:]
    out = x.clone()
    if interleaved:
        x1 = x[..., 0:rot_dim:2]
        x2 = x[..., 1:rot_dim:2]
        out[..., 0:rot_dim:2] = x1 * cos - x2 * sin
        out[..., 1:rot_dim:2] = x2 * cos + x1 * sin
    else:
        x1 = x[..., :half]
        x2 = x[..., half:rot_dim]
        out[..., :half] = x1 * cos - x2 * sin
        out[..., half:rot_dim] = x2 * cos + x1 * sin
    return out


def kv_page_write_ref(cache, slots, vals, scale=None):
    """cache [P, KVH, 16, D]; vals [T, KVH, D]; slots [T] (-1 = skip)."""
    for t in range(vals.shape[0]):
        s = int(slots[t])
        if s < 0:
            continue
        v = vals[t].float()
        if scale is not None:
            v = v / scale.float()[:, None]
        cache[s // PAGE, :, s % PAGE, :] = v.to(cache.dtype)


def qk_norm_rope_kv_ref(qkv, positions, slots, cos_sin, rot_dim, interleaved, qw, kw, eps,
                        k_cache, v_cache, H, KVH, D, k_scale=None, v_scale=None):
    T = qkv.shape[0]
    dt = qkv.dtype
    q = qkv[:, : H * D].reshape(T, H, D).float()
    k = qkv[:, H * D:(H + KVH) * D].reshape(T, KVH, D).float()
    v = qkv[:, (H + KVH) * D:(H + 2 * KVH) * D].reshape(T, KVH, D)
    if qw is not None:
        q = (q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + eps) * qw.float()).to(dt).float()
    if kw is not None:
        k = (k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + eps) * kw.float()).to(dt).float()
    q = apply_rope_ref(q, positions, cos_sin, rot_dim, interleaved).to(dt)
    k = apply_rope_ref(k, positions, cos_sin, rot_dim, interleaved).to(dt)
    if slots is not None and k_cache is not None:
        kv_page_write_ref(k_cache, slots, k, k_scale)
        kv_page_write_ref(v_cache, slots, v, v_scale)
    return q, k, v


# --------------------------------------------------------------------------
# attention
# --------------------------------------------------------------------------
def gather_pages(cache, page_ids, n_tokens, scale=None):
    """cache [P, KVH, 16, D] -> [n_tokens, KVH, D] float."""
    if n_tokens == 0:
        return cache.new_zeros((0, cache.shape[1], cache.shape[3]), dtype=torch.float32)
    npg = (n_tokens + PAGE - 1) // PAGE
    pages = cache[torch.as_tensor(page_ids[:npg], dtype=torch.long, device=cache.device)]  # [npg, KVH, 16, D]
    x = pages.permute(0, 2, 1, 3).reshape(npg * PAGE, cache.shape[1], cache.shape[3])[:n_tokens].float()
    if scale is not None:
        x = x * scale.float()[None, :, None]
    return x


def attention_rows_ref(q, k, v, q_pos, kv_len, scale, window=0, sinks=None, softcap=0.0, k_pos=None,
                       extra_mask=None):
    """q [Tq, H, D] float at absolute positions q_pos [Tq]; k,v [kv_len, KVH, D].
    Causal with optional sliding window (window > 0); window < 0 is
    bidirectional over all kv_len keys (encoders). Sinks are
    denominator-only logits."""
    Tq, H, D = q.shape
    KVH = k.shape[1]
    G = H // KVH
    kk = k.repeat_interleave(G, dim=1)  # [L, H, D]
    vv = v.repeat_interleave(G, dim=1)
    s = torch.einsum("thd,lhd->thl", q.float(), kk.float()) * scale
    if softcap > 0:
        s = softcap * torch.tanh(s / softcap)
    kp = torch.arange(kv_len, device=q.device) if k_pos is None else k_pos.to(q.device).long()
    qp = q_pos.to(q.device).long()[:, None]
    mask = kp[None, :] <= qp
    if extra_mask is not None:  # e.g. chunked attention: same chunk only
        mask = mask & extra_mask(qp[:, 0], kp)
    if window < 0:
        mask = torch.ones_like(mask)
    if window > 0:
        mask = mask & (kp[None, :] > qp - window)
    s = s.masked_fill(~mask[:, None, :], float("-inf"))
    if sinks is not None:
        sk = sinks.float().to(q.device)[None, :, None].expand(Tq, H, 1)
        s = torch.cat([s, sk], dim=-1)
        p = torch.softmax(s, dim=-1)[..., :-1]
    else:
        p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    return torch.einsum("thl,lhd->thd", p, vv.float())


def paged_decode_ref(q, k_cache, v_cache, page_table, seq_lens, scale, window=0, sinks=None, softcap=0.0,
                     k_scale=None, v_scale=None):
    """q [B, H, D]; returns [B, H, D] in q.dtype."""
    B = q.shape[0]
    out = torch.zeros_like(q, dtype=torch.float32)
    for b in range(B):
        L = int(seq_lens[b])
        if L <= 0:
            continue
        pids = page_table[b].tolist()
        k = gather_pages(k_cache, pids, L, k_scale)
        v = gather_pages(v_cache, pids, L, v_scale)
        qpos = torch.tensor([L - 1])
        out[b] = attention_rows_ref(q[b:b + 1].float(), k, v, qpos, L, scale, window, sinks, softcap)[0]
    return out.to(q.dtype)


def paged_selected_decode_ref(q, k_cache, v_cache, page_table, seq_lens, sel, scale):
    """Attention of q [B, H, D] over the positions sel[b] (-1 / out of range
    ignored) of each row's pages; returns [B, H, D] in q.dtype."""
    B, H, D = q.shape
    KVH = k_cache.shape[1]
    out = torch.zeros(B, H, D, dtype=torch.float32)
    for b in range(B):
        L = int(seq_lens[b])
        pos = [int(t) for t in sel[b].tolist() if 0 <= int(t) < L]
        if not pos:
            continue
        pids = page_table[b].tolist()
        k = gather_pages(k_cache, pids, L).float()[pos]  # [n, KVH, D]
        v = gather_pages(v_cache, pids, L).float()[pos]
        kk = k.repeat_interleave(H // KVH, 1)
        vv = v.repeat_interleave(H // KVH, 1)
        s = torch.einsum("hd,nhd->hn", q[b].float(), kk) * scale
        out[b] = torch.einsum("hn,nhd->hd", torch.softmax(s, -1), vv)
    return out.to(q.dtype)


def paged_prefill_ref(q, k_cache, v_cache, page_table, cu_q, q_pos0, scale, window=0, sinks=None, softcap=0.0,
                      k_scale=None, v_scale=None):
    """q [T, H, D] (rows' chunks concatenated); returns [T, H, D]."""
    out = torch.zeros_like(q, dtype=torch.float32)
    R = len(cu_q) - 1
    for r in range(R):
        a, b = int(cu_q[r]), int(cu_q[r + 1])
        if b <= a:
            continue
        p0 = int(q_pos0[r])
        L = p0 + (b - a)
        pids = page_table[r].tolist()
        k = gather_pages(k_cache, pids, L, k_scale)
        v = gather_pages(v_cache, pids, L, v_scale)
        qpos = torch.arange(p0, L)
        out[a:b] = attention_rows_ref(q[a:b].float(), k, v, qpos, L, scale, window, sinks, softcap)
    return out.to(q.dtype)


# --------------------------------------------------------------------------
# sampling
# --------------------------------------------------------------------------
_M0, _M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = np.uint64(0x9E3779B9), np.uint64(0xBB67AE85)
_MASK32 = np.uint64(0xFFFFFFFF)


def philox_u32(key: int, step: int, idx: np.ndarray) -> np.ndarray:
    """Vectorised Philox-4x32-10; same stream as the CUDA sampler."""
    idx = np.asarray(idx, dtype=np.uint64)
    c0 = idx & _MASK32
    c1 = np.full_like(c0, np.uint64(step & 0xFFFFFFFF))
    c2 = np.full_like(c0, np.uint64((step >> 32) & 0xFFFFFFFF))
    c3 = np.full_like(c0, np.uint64(0x42323030))
    k0 = np.uint64(key & 0xFFFFFFFF)
    k1 = np.uint64((key >> 32) & 0xFFFFFFFF)
    with np.errstate(over="ignore"):
        for _ in range(10):
            p0 = _M0 * c0
            p1 = _M1 * c2
            hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK32
            hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK32
            n0 = (hi1 ^ c1 ^ k0) & _MASK32
            n2 = (hi0 ^ c3 ^ k1) & _MASK32
            c0, c1, c2, c3 = n0, lo1, n2, lo0
            k0 = (k0 + _W0) & _MASK32
            k1 = (k1 + _W1) & _MASK32
    return c0.astype(np.uint32)


def philox_uniform(key: int, step: int, idx: np.ndarray) -> np.ndarray:
    x = philox_u32(key, step, idx)
    return ((x >> 8).astype(np.float32) + np.float32(0.5)) * np.float32(1.0 / 16777216.0)


def mix_key(seed: int, request_id: int) -> int:
    """RNG key of a request: seed mixed with its id (splitmix64 finaliser)."""
    z = (seed ^ (request_id * 0x9E3779B97F4A7C15)) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return z ^ (z >> 31)


def process_logits_ref(logits, bias=None, rep_ids=None, rep_penalty=1.0, out_ids=None, freq=0.0, pres=0.0,
                       allow=None):
    """One row. bias: dict id->val; rep_ids: recent-context ids; out_ids: generated ids;
    allow: bool tensor [V] (True = allowed) or None."""
    lg = logits.clone().float()
    V = lg.shape[0]
    if bias:
        for i, b in bias.items():
            if 0 <= i < V:
                lg[i] += b
    if rep_ids is not None and rep_penalty != 1.0:
        for i in sorted(set(int(t) for t in rep_ids if 0 <= int(t) < V)):
            x = lg[i].item()
            lg[i] = x / rep_penalty if x > 0 else x * rep_penalty
    if out_ids is not None and (freq != 0.0 or pres != 0.0):
        counts = {}
        for t in out_ids:
            t = int(t)
            if 0 <= t < V:
                counts[t] = counts.get(t, 0) + 1
        for i, c in counts.items():
            lg[i] = lg[i] - (np.float32(c) * np.float32(freq) + np.float32(pres))
    if allow is not None:
        lg = lg.masked_fill(~allow, float("-inf"))
    return lg


def _fkey(x: np.ndarray) -> np.ndarray:
    b = x.astype(np.float32).view(np.uint32)
    return np.where(b & np.uint32(0x80000000), ~b, b | np.uint32(0x80000000)).astype(np.uint32)


def sample_ref(logits, temperature, top_k=0, top_p=1.0, min_p=0.0, key=0, step=0):
    """One row of processed logits -> token id (same rule as the kernel)."""
    lg = logits.float().cpu().numpy()
    if temperature <= 0 or not np.isfinite(lg.max()):
        return int(np.argmax(lg))
    s = (lg * np.float32(1.0 / temperature)).astype(np.float32)
    mx = np.float32(lg.max() * np.float32(1.0 / temperature))
    keys = _fkey(s)
    thr = np.uint32(0)
    V = s.shape[0]
    if 0 < top_k < V:
        thr = np.sort(keys)[::-1][top_k - 1]
    if top_p < 1.0:
        w = np.rint(np.exp2((s - mx) * np.float32(1.4426950408889634)) * np.float32(1073741824.0)).astype(np.uint64)
        kept = keys >= thr
        tot = int(w[kept].sum())
        target = max(1, math.ceil(float(top_p) * float(tot)))
        order = np.argsort(-keys[kept].astype(np.int64), kind="stable")
        kk = keys[kept][order]
        ww = w[kept][order]
        # cumulative mass over distinct key values (ties share a value)
        cum = np.cumsum(ww)
        idx = int(np.searchsorted(cum, target))
        idx = min(idx, len(kk) - 1)
        thr = max(thr, kk[idx])
    if min_p > 0:
        thr = max(thr, _fkey(np.array([mx + np.float32(math.log(min_p))], dtype=np.float32))[0])
    keep = (keys >= thr) & np.isfinite(s)
    u = philox_uniform(key, step, np.arange(V))
    g = -np.log(-np.log(u))
    v = np.where(keep, s + g, -np.inf)
    return int(np.argmax(v))


# --------------------------------------------------------------------------
# gated DeltaNet (linear attention)
# --------------------------------------------------------------------------
def gdn_layer_ref(P, cu, fresh, slot, conv_state, ssm_state, conv_w, A_log, dt_bias, norm_w, Hk, Dk, Hv, Dv, eps):
    """Gated DeltaNet layer body over a flattened batch of rows (fp32).
    P [T, C + Hv*Dv + 2*Hv] = q | k | v | z | b | a (C = 2*Hk*Dk + Hv*Dv);
    rows r cover tokens cu[r]..cu[r+1]-1 with state slot slot[r] (zero state
    when fresh[r]). Updates conv_state [S, 3, C] and ssm_state [S, Hv, Dv, Dk]
    in place; returns rmsnorm(y) * norm_w * silu(z) [T, Hv*Dv] in P.dtype.
    Semantics of MLXLMCommon/GatedDelta.swift (gated_delta_step) and
    MLXLLM/Models/Qwen3Next.swift (conv + SiLU, q/k scaling, RMSNormGated)."""
    T = P.shape[0]
    C = 2 * Hk * Dk + Hv * Dv
    taps = conv_w.shape[1]
    out = torch.zeros(T, Hv * Dv, dtype=torch.float32, device=P.device)
    cu = [int(c) for c in cu]
    rep = Hv // Hk
    for r in range(len(cu) - 1):
        s0, s1 = cu[r], cu[r + 1]
        n = s1 - s0
        if n <= 0:
            continue
        sl = int(slot[r])
        x = P[s0:s1, :C].float()
        prev = torch.zeros(taps - 1, C, device=P.device) if int(fresh[r]) else conv_state[sl].float()
        xx = torch.cat([prev, x], 0)
        conv = torch.zeros(n, C, device=P.device)
        for j in range(taps):
            conv += conv_w[:, j].float() * xx[j:j + n]
        y = conv * torch.sigmoid(conv)
        q = y[:, :Hk * Dk].reshape(n, Hk, Dk)
        k = y[:, Hk * Dk:2 * Hk * Dk].reshape(n, Hk, Dk)
        v = y[:, 2 * Hk * Dk:].reshape(n, Hv, Dv)
        q = q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + eps) / Dk
        k = k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + eps) / math.sqrt(Dk)
        zb = C + Hv * Dv
        b = P[s0:s1, zb:zb + Hv].float()
        a = P[s0:s1, zb + Hv:zb + 2 * Hv].float()
        g = torch.exp(-torch.exp(A_log.float()) * torch.nn.functional.softplus(a + dt_bias.float()))
        beta = torch.sigmoid(b)
        S = torch.zeros(Hv, Dv, Dk, device=P.device) if int(fresh[r]) else ssm_state[sl].float().clone()
        o = torch.zeros(n, Hv, Dv, device=P.device)
        for t in range(n):
            kh = k[t].repeat_interleave(rep, 0)
            qh = q[t].repeat_interleave(rep, 0)
            S = S * g[t][:, None, None]
            kv = (S * kh[:, None, :]).sum(-1)
            delta = (v[t] - kv) * beta[t][:, None]
            S = S + kh[:, None, :] * delta[:, :, None]
            o[t] = (S * qh[:, None, :]).sum(-1)
        ssm_state[sl] = S.to(ssm_state.dtype)
        conv_state[sl] = xx[-(taps - 1):].to(conv_state.dtype)
        z = P[s0:s1, C:C + Hv * Dv].float().reshape(n, Hv, Dv)
        on = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + eps) * norm_w.float() * (z * torch.sigmoid(z))
        out[s0:s1] = on.reshape(n, -1)
    return out.to(P.dtype)


def mamba_layer_ref(P, cu, fresh, slot, conv_state, ssm_state, conv_w, conv_b, A_log, dt_bias, D, norm_w, G, N, H,
                    Pd, eps, norm_group, dt_limits=(0.0, float("inf"))):
    """Mamba-2 mixer body over a flattened batch of rows (fp32).
    P [T, C + H*Pd + H] = C | B | x (conv channels, C = 2*G*N + H*Pd) | z | dt;
    conv with bias + SiLU; dt = clip(softplus(dt + dt_bias)); per head h of
    group g = h // (H // G): S <- exp(-exp(A_log) dt) S + dt x B^T,
    y = S C + D x; out = rmsnorm over groups of `norm_group` channels of
    (y * silu(z)) * norm_w. States as in :func:`gdn_layer_ref` with
    ssm_state [S, H, Pd, N]. Semantics of MLXLLM/Models/SSM.swift and
    MLXLLM/Models/NemotronH.swift (RMSNormGated with group_size)."""
    T = P.shape[0]
    C = 2 * G * N + H * Pd
    taps = conv_w.shape[1]
    out = torch.zeros(T, H * Pd, dtype=torch.float32, device=P.device)
    rep = H // G
    for r in range(len(cu) - 1):
        s0, s1 = int(cu[r]), int(cu[r + 1])
        n = s1 - s0
        if n <= 0:
            continue
        sl = int(slot[r])
        x = P[s0:s1, :C].float()
        prev = torch.zeros(taps - 1, C, device=P.device) if int(fresh[r]) else conv_state[sl].float()
        xx = torch.cat([prev, x], 0)
        conv = torch.zeros(n, C, device=P.device) + (conv_b.float() if conv_b is not None else 0.0)
        for j in range(taps):
            conv += conv_w[:, j].float() * xx[j:j + n]
        yv = conv * torch.sigmoid(conv)
        Cm = yv[:, :G * N].reshape(n, G, N)
        Bm = yv[:, G * N:2 * G * N].reshape(n, G, N)
        xh = yv[:, 2 * G * N:].reshape(n, H, Pd)
        dt = torch.nn.functional.softplus(P[s0:s1, C + H * Pd:C + H * Pd + H].float() + dt_bias.float())
        dt = dt.clamp(dt_limits[0], dt_limits[1])
        dA = torch.exp(-torch.exp(A_log.float()) * dt)
        S = torch.zeros(H, Pd, N, device=P.device) if int(fresh[r]) else ssm_state[sl].float().clone()
        o = torch.zeros(n, H, Pd, device=P.device)
        for t in range(n):
            Bh = Bm[t].repeat_interleave(rep, 0)
            Ch = Cm[t].repeat_interleave(rep, 0)
            S = S * dA[t][:, None, None] + (xh[t] * dt[t][:, None])[:, :, None] * Bh[:, None, :]
            o[t] = (S * Ch[:, None, :]).sum(-1) + D.float()[:, None] * xh[t]
        ssm_state[sl] = S.to(ssm_state.dtype)
        conv_state[sl] = xx[-(taps - 1):].to(conv_state.dtype)
        z = P[s0:s1, C:C + H * Pd].float()
        v = o.reshape(n, -1) * (z * torch.sigmoid(z))
        vg = v.reshape(n, -1, norm_group)
        vg = vg * torch.rsqrt(vg.pow(2).mean(-1, keepdim=True) + eps)
        out[s0:s1] = vg.reshape(n, -1) * norm_w.float()
    return out.to(P.dtype)


def short_conv_ref(P, cu, fresh, slot, conv_state, conv_w, conv_b):
    """LFM2 short convolution over a flattened batch of rows (fp32 math):
    P [T, 3C] = B | C | x; y = C * (conv over Bx = B * x with the row's
    conv state [S, taps-1, C] before its chunk); updates the state in place."""
    C, taps = conv_w.shape
    T = P.shape[0]
    out = torch.zeros(T, C, dtype=torch.float32, device=P.device)
    for r in range(len(cu) - 1):
        s0, s1 = int(cu[r]), int(cu[r + 1])
        n = s1 - s0
        if n <= 0:
            continue
        sl = int(slot[r])
        bx = (P[s0:s1, :C].float() * P[s0:s1, 2 * C:3 * C].float()).to(P.dtype).float()
        prev = torch.zeros(taps - 1, C, device=P.device) if int(fresh[r]) else conv_state[sl].float()
        xx = torch.cat([prev, bx], 0)
        acc = torch.zeros(n, C, device=P.device) + (conv_b.float() if conv_b is not None else 0.0)
        for j in range(taps):
            acc += conv_w[:, j].float() * xx[j:j + n]
        out[s0:s1] = P[s0:s1, C:2 * C].float() * acc
        conv_state[sl] = xx[-(taps - 1):].to(conv_state.dtype)
    return out.to(P.dtype)


def xielu_ref(x, params):
    """xIELU: a_p = softplus(alpha_p), a_n = beta + softplus(alpha_n);
    x > 0 -> a_p x^2 + beta x, else a_n (exp(min(x, eps)) - 1) - a_n x + beta x."""
    p = params.float()
    ap = torch.nn.functional.softplus(p[0])
    an = p[2] + torch.nn.functional.softplus(p[1])
    beta, eps = p[2], p[3]
    xf = x.float()
    y = torch.where(xf > 0, ap * xf * xf + beta * xf, an * torch.expm1(torch.minimum(xf, eps)) - an * xf + beta * xf)
    return y.to(x.dtype)
