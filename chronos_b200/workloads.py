"""Seeded synthetic inputs of the benchmark configurations (shared by bench.py and the parity tests, so that the tests
check the very batches the bench times). No dataset is involved anywhere: every tensor is drawn from a seeded generator.
"""
from __future__ import annotations

import torch

from .layout import FoldedLayerConfig

DECODE = dict(hidden=4096, inter=1536, n_experts=288, group_size=4, rank=64, top_k=8)  # the decode / prefill / stack layer
TOKENS_PER_STREAM = 3      # 1 bonus + 2 draft tokens of a speculative verify step
STREAM_CORR = 0.67         # shared share of variance of a stream's tokens -> ~30 % top-8 overlap at 288 experts
N_BATCHES = 8              # distinct routed batches a timed loop rotates through


def decode_batches(cfg: FoldedLayerConfig, streams: int, device, seed: int = 1, n_batches: int = N_BATCHES) -> list[torch.Tensor]:
    """Seeded activation batches [streams * 3, H] bf16: the 3 tokens of a stream share a common component (correlation
    0.67 of their router logits), which makes their top-8 sets overlap by about 30 %."""
    gen = torch.Generator(device=device).manual_seed(seed)
    out = []
    for _ in range(n_batches):
        base = torch.randn(streams, 1, cfg.hidden, generator=gen, device=device)
        eps = torch.randn(streams, TOKENS_PER_STREAM, cfg.hidden, generator=gen, device=device)
        out.append((STREAM_CORR ** 0.5 * base + (1.0 - STREAM_CORR) ** 0.5 * eps).reshape(-1, cfg.hidden).to(torch.bfloat16).contiguous())
    return out


def zipf_prefill_batch(layer, n_tokens: int, seed: int = 2, exponent: float = 1.1) -> torch.Tensor:
    """Prefill-shaped batch [n_tokens, H] bf16 ~ N(0, 1) whose routing follows a Zipf(`exponent`) expert popularity over a
    seeded permutation of the experts. N(0, 1) activations carry no direction a router bias could ride on, so the bias
    log p_e enters through one input channel: x[:, 0] = 1 and router_w[:, 0] = log p_e (the layer's router table is
    modified in place)."""
    cfg = layer.cfg
    dev = layer.device
    gen = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(n_tokens, cfg.hidden, generator=gen, device=dev).to(torch.bfloat16)
    perm = torch.randperm(cfg.n_experts, generator=torch.Generator().manual_seed(seed))
    p_e = torch.arange(1, cfg.n_experts + 1, dtype=torch.float64) ** -exponent
    p_e = (p_e / p_e.sum())[torch.argsort(perm)]
    layer.packed.t["router_w"][:, 0] = torch.log(p_e).to(torch.float32).to(dev)
    x[:, 0] = 1.0
    return x
