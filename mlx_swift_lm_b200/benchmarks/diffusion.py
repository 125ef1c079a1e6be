"""Block mask-diffusion decoding throughput (Nemotron-Labs-Diffusion-3B
shape, random weights, synthetic prompts): committed tokens per second and
forward passes per committed token for R concurrent requests, diffusion
(threshold commits) and linear self-speculation modes.

    python -m mlx_swift_lm_b200.benchmarks.diffusion [--rows 32] [--prompt 512] [--new 128]

Wall-clock over whole requests (prefill included) after one warm-up request
set, with a device synchronize on both sides; the host commit policy and the
per-forward device-to-host read are part of what is timed.
"""
from __future__ import annotations

import argparse
import time

import torch

from ..engine.block_diffusion import BlockDiffusionEngine, DiffusionConfig, DiffusionRequest
from ..models.config import DecoderConfig
from ..models.decoder import DecoderLM


def nemotron_labs_diffusion_3b(layers: int = 26) -> DecoderConfig:
    c = DecoderConfig(model_type="nemotron_labs_diffusion", vocab_size=131072, hidden_size=3072, num_layers=layers,
                      num_heads=32, num_kv_heads=8, head_dim=128, intermediate_size=9216, rms_norm_eps=1e-5,
                      rope_theta=1e6, max_position_embeddings=262144)
    c.extra.update(mask_token_id=100, diffusion_block=32, attn_pos_scale=(0.1, 16384))
    return c


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=32)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--new", type=int, default=128)
    ap.add_argument("--block", type=int, default=32)
    ap.add_argument("--threshold", type=float, default=0.9)
    ap.add_argument("--layers", type=int, default=26)
    a = ap.parse_args(argv)
    torch.manual_seed(0)
    m = DecoderLM(nemotron_labs_diffusion_3b(a.layers), "cuda", torch.bfloat16).init_random(0, std=0.02)
    g = torch.Generator().manual_seed(1)
    for mode, thr in (("diffusion", a.threshold), ("linear_spec", 0.0)):
        eng = BlockDiffusionEngine(m, DiffusionConfig(max_rows=a.rows, kv_tokens=a.rows * (a.prompt + a.new + 64)))

        def reqs():
            return [DiffusionRequest(torch.randint(200, 131072, (a.prompt,), generator=g).tolist(), a.new, a.block,
                                     thr, mode) for _ in range(a.rows)]

        eng.generate(reqs()[:2])  # warm-up
        rs = reqs()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = eng.generate(rs)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        new = sum(len(t) - a.prompt for t, _ in out)
        nfe = sum(n for _, n in out) / len(out)
        print(f"{mode} rows={a.rows} prompt={a.prompt} new={a.new} block={a.block}: {new / dt:.0f} tok/s, "
              f"{eng.forwards} forwards ({nfe:.1f} per request), {dt * 1e3:.0f} ms")


if __name__ == "__main__":
    main()
