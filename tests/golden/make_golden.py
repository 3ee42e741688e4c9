#!/usr/bin/env python3
"""Generates the golden fixtures in this folder by running the REFERENCE's own code.

Run where the Chronos reference checkout is importable:

    PYTHONPATH=/path/to/Chronos python tests/golden/make_golden.py

For every case it folds seeded synthetic experts with the reference converter
(`chronos_1t.models.glm53_holo.convert_expert_group`), then records what the reference's runtime
functions return on those bytes:
  * `unpack_nvfp4` of both banks of slot 0                       (fp32, bit-exact target)
  * `expert_keys` of selected (slot, member)                      (integer, bit-exact target)
  * `reconstruct_group_experts(include_tail=False / True)`        (fp32 reconstruction)
  * `pack_nvfp4` of a seeded matrix incl. an all-tiny block       (byte-exact target)
  * softmax-top-k and sigmoid-noaux_tc routers (torch CPU)        (ids exact, gates fp32)
  * the routed layer output, grouped dense loop in fp32 torch     (layer tolerance target)
plus one router-only case at the benchmark's shape (288 experts x hidden 4096 x 512 tokens): logits, ids and gates of
the softmax, sigmoid `noaux_tc` and sqrt-softplus `noaux_tc` routers as the reference computes them.
The fixtures are small `.npz` files; fp8 tensors are stored as uint8 bit patterns.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

from chronos_1t.converter.convert_glm53_flash_colab import pack_nvfp4, unpack_nvfp4
from chronos_1t.models import glm53_holo as G

HERE = Path(__file__).resolve().parent

CASES = {
    # name: hidden, inter, experts, group size K, healer rank, top_k, tokens, seed, tail bits (gu, down)
    "k4_h256_i128": dict(hidden=256, inter=128, experts=8, k=4, rank=16, top_k=2, tokens=5, seed=0, tails=(2, 2)),
    "k8_h384_i128": dict(hidden=384, inter=128, experts=16, k=8, rank=32, top_k=4, tokens=4, seed=1, tails=(1, 2)),
}


def _np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy().copy()
    return t.numpy().copy()


def make_case(name: str, c: dict) -> None:
    h, i, e, k, r = c["hidden"], c["inter"], c["experts"], c["k"], c["rank"]
    gen = torch.Generator().manual_seed(c["seed"])
    gate = torch.randn(e, i, h, generator=gen) * 0.02
    up = torch.randn(e, i, h, generator=gen) * 0.02
    down = torch.randn(e, h, i, generator=gen) * 0.02
    router_w = torch.randn(e, h, generator=gen) * 0.02
    e_bias = torch.randn(e, generator=gen) * 0.05
    x = torch.randn(c["tokens"], h, generator=gen)
    n_slots = e // k
    # the converter indexes router rows by g*8 (its hard-coded group stride): give it a table laid out that way
    rw_conv = torch.zeros(8 * n_slots, h)
    for g in range(n_slots):
        rw_conv[g * 8 : g * 8 + k] = router_w[g * k : (g + 1) * k]
    v_sub, s_sub = G.router_subspace(router_w)
    out: dict[str, np.ndarray] = {
        "meta": np.array([h, i, e, k, r, c["top_k"], c["tokens"]], dtype=np.int64),
        "router_w": _np(router_w), "e_bias": _np(e_bias), "x": _np(x),
    }
    groups = []
    for g in range(n_slots):
        tens, _ = G.convert_expert_group(
            gate[g * k : (g + 1) * k], up[g * k : (g + 1) * k], down[g * k : (g + 1) * k], rw_conv, v_sub, s_sub, g,
            svd_rank=r, gu_tail_bits=c["tails"][0], down_tail_bits=c["tails"][1],
        )
        groups.append(tens)
        for sfx, t in tens.items():
            out[f"g{g}.{sfx}"] = _np(t)

    g0 = groups[0]
    out["ref.dequant_gu_g0"] = _np(unpack_nvfp4(g0["s_gu.weight"], g0["s_gu.weight_scale"], g0["s_gu.weight_scale_2"]))
    out["ref.dequant_down_g0"] = _np(unpack_nvfp4(g0["s_down.weight"], g0["s_down.weight_scale"], g0["s_down.weight_scale_2"]))

    for (g, m) in ((0, 0), (n_slots - 1, k - 1)):
        sg, sd = G.group_seed_bases(g)
        for tag, rows, cols, sb in (("gu", 2 * i, h, sg), ("down", h, i, sd)):
            keys = G.expert_keys(rows, cols, m, sb, torch.device("cpu"))
            for nm, t in zip(("r_s1", "r_perm", "r_inv", "r_s2", "c_s1", "c_perm", "c_inv", "c_s2"), keys):
                out[f"ref.keys.{tag}.g{g}.m{m}.{nm}"] = _np(t).astype(np.int8 if "s" in nm.split("_")[1] else np.int32)

    for (g, m, tail) in ((0, 0, False), (n_slots - 1, k - 1, False), (0, k - 1, True)):
        gu, dn = G.reconstruct_group_experts(groups[g], g, [m], h, i, include_tail=tail)[0]
        tg = "tail" if tail else "notail"
        out[f"ref.recon_{tg}.g{g}.m{m}.gu"] = _np(gu)
        out[f"ref.recon_{tg}.g{g}.m{m}.down"] = _np(dn)

    # pack_nvfp4 known-answer incl. a block of tiny values (scale code rounds to 0 -> saturated nibbles, signed zeros)
    wp = torch.randn(16, 64, generator=gen) * 0.02
    wp[3, 16:32] = torch.randn(16, generator=gen) * 1e-9
    wp[5, :16] = 0.0
    p, s, s2 = pack_nvfp4(wp)
    out["ref.pack.in"], out["ref.pack.packed"], out["ref.pack.scale"], out["ref.pack.scale2"] = _np(wp), _np(p), _np(s), _np(s2)
    out["ref.pack.dequant"] = _np(unpack_nvfp4(p, s, s2))

    # routers: chronos_1t/models/vllm_chronos_moe.py:310-314 and chronos_1t/models/glm53_chronos_moe.py:392-399
    logits = F.linear(x.float(), router_w.float())
    tv, ti = torch.topk(logits, k=c["top_k"], dim=-1)
    out["ref.router.logits"], out["ref.router.softmax_ids"] = _np(logits), _np(ti)
    out["ref.router.softmax_gates"] = _np(F.softmax(tv, dim=-1))
    scores = torch.sigmoid(x.float() @ router_w.T)
    _, si = torch.topk(scores + e_bias, c["top_k"], dim=-1)
    sw = scores.gather(1, si)
    sw = sw / (sw.sum(-1, keepdim=True) + 1e-20)
    out["ref.router.sigmoid_ids"], out["ref.router.sigmoid_gates"] = _np(si), _np(sw * 2.5)

    # layer output: grouped dense loop, chronos_1t/models/glm53_chronos_moe.py:452-472, fp32 reconstruction w/o tail
    for tag, ids, w in (("softmax", ti, F.softmax(tv, dim=-1)), ("sigmoid", si, sw * 2.5)):
        y = torch.zeros(c["tokens"], h)
        flat_ids, flat_w = ids.reshape(-1), w.reshape(-1)
        tok_of = torch.arange(c["tokens"]).repeat_interleave(c["top_k"])
        for eid in torch.unique(flat_ids).tolist():
            sel = torch.nonzero(flat_ids == eid).flatten()
            gu_w, dn_w = G.reconstruct_group_experts(groups[eid // k], eid // k, [eid % k], h, i, include_tail=False)[0]
            xs = x[tok_of[sel]]
            gu = F.linear(xs, gu_w)
            act = F.silu(gu[:, :i]) * gu[:, i:]
            y.index_add_(0, tok_of[sel], F.linear(act, dn_w) * flat_w[sel].unsqueeze(-1))
        out[f"ref.layer_y.{tag}"] = _np(y)

    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(name, "->", (HERE / f"{name}.npz").stat().st_size, "bytes")


ROUTER_CASE = dict(name="router_e288_h4096", experts=288, hidden=4096, tokens=512, top_k=8, seed=11)


def router_case_inputs(c: dict = ROUTER_CASE):
    """Seeded inputs of the router-only case (torch CPU generator): bf16-rounded activations, router table, bias.
    The tests regenerate them from the seed, so the fixture only stores what the reference computed from them."""
    gen = torch.Generator().manual_seed(c["seed"])
    x = torch.randn(c["tokens"], c["hidden"], generator=gen).to(torch.bfloat16).float()
    router_w = torch.randn(c["experts"], c["hidden"], generator=gen) * 0.02
    e_bias = torch.randn(c["experts"], generator=gen) * 0.05
    return x, router_w, e_bias


def make_router_case(c: dict = ROUTER_CASE) -> None:
    """Router at the benchmark's own shape (288 experts, hidden 4096), the three flavours exactly as the reference
    writes them: chronos_1t/models/vllm_chronos_moe.py:310-314, chronos_1t/models/glm53_chronos_moe.py:392-399,
    chronos_1t/models/dsv41_chronos_moe.py:3402-3410. Stores logits, ids and gates only."""
    x, router_w, e_bias = router_case_inputs(c)
    k = c["top_k"]
    out: dict[str, np.ndarray] = {"meta": np.array([c["experts"], c["hidden"], c["tokens"], k, c["seed"]], dtype=np.int64)}
    logits = F.linear(x.float(), router_w.float())
    tv, ti = torch.topk(logits, k=k, dim=-1)
    out["logits"] = _np(logits)
    out["softmax_ids"], out["softmax_gates"] = _np(ti).astype(np.int16), _np(F.softmax(tv, dim=-1))
    scores = torch.sigmoid(x.float() @ router_w.T)
    _, si = torch.topk(scores + e_bias, k, dim=-1)
    sw = scores.gather(1, si)
    sw = sw / (sw.sum(-1, keepdim=True) + 1e-20)
    out["sigmoid_ids"], out["sigmoid_gates"] = _np(si).astype(np.int16), _np(sw * 2.5)
    raw = F.linear(x, router_w).float()
    sc = F.softplus(raw).sqrt()
    _, qi = torch.topk(sc + e_bias.unsqueeze(0), k=k, dim=-1)
    qw = sc.gather(1, qi)
    out["sqrt_softplus_ids"] = _np(qi).astype(np.int16)
    out["sqrt_softplus_gates"] = _np((qw / (qw.sum(dim=-1, keepdim=True) + 1e-20)) * 1.5)
    np.savez_compressed(HERE / f"{c['name']}.npz", **out)
    print(c["name"], "->", (HERE / f"{c['name']}.npz").stat().st_size, "bytes")


def make_fp8_block_case() -> None:
    """Stock 128x128 block-FP8 weights (the format the reference keeps the shared expert in,
    chronos_1t/models/glm53_chronos_moe.py:170-181): `dequant_fp8_block` (chronos_1t/models/glm53_tiers.py:74-95) of seeded
    bytes, and the shared expert's output the way `shared_forward` (:401-404) computes it for a batch above its GEMV
    threshold (dequantise, then F.linear), in fp32."""
    from chronos_1t.models.glm53_tiers import dequant_fp8_block

    gen = torch.Generator().manual_seed(21)
    h, i, n_tok = 256, 128, 6
    out: dict[str, np.ndarray] = {"meta": np.array([h, i, n_tok], dtype=np.int64)}
    tens = {}
    for name, (rows, cols) in (("gate_proj", (i, h)), ("up_proj", (i, h)), ("down_proj", (h, i))):
        w = torch.randint(0, 256, (rows, cols), generator=gen, dtype=torch.uint8)
        w[(w & 0x7F) == 0x7F] = 0x3A  # no NaN codes
        s = torch.rand((rows // 128, cols // 128), generator=gen) * 0.02 + 0.001
        tens[name] = (w, s)
        out[f"{name}.weight"], out[f"{name}.weight_scale_inv"] = _np(w), _np(s)
        out[f"ref.dequant.{name}"] = _np(dequant_fp8_block(w, s, dtype=torch.float32))
    x = torch.randn(n_tok, h, generator=gen)
    out["x"] = _np(x)
    gu_w = torch.cat([dequant_fp8_block(*tens["gate_proj"], dtype=torch.float32), dequant_fp8_block(*tens["up_proj"], dtype=torch.float32)], 0)
    gu = F.linear(x, gu_w)
    act = F.silu(gu[:, :i]) * gu[:, i:]
    out["ref.shared_y"] = _np(F.linear(act, dequant_fp8_block(*tens["down_proj"], dtype=torch.float32)))
    np.savez_compressed(HERE / "fp8_block_shared.npz", **out)
    print("fp8_block_shared ->", (HERE / "fp8_block_shared.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    torch.set_num_threads(4)
    for nm, cfg in CASES.items():
        if len(sys.argv) < 2 or nm in sys.argv[1:]:
            make_case(nm, cfg)
    if len(sys.argv) < 2 or ROUTER_CASE["name"] in sys.argv[1:]:
        make_router_case()
    if len(sys.argv) < 2 or "fp8_block_shared" in sys.argv[1:]:
        make_fp8_block_case()
