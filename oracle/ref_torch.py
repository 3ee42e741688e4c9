"""The reference's own PyTorch path for the folded MoE layer, driven from `oracle/_ref` (TEST INFRASTRUCTURE).

Only the bench's reference arm / CPU-baseline leg and the tests may import this module. It adds nothing of its own to
the arithmetic: weights come from the reference's `reconstruct_group_experts(include_tail=False)`
(chronos_1t/models/glm53_holo.py:336-368), the shared expert from its `unpack_nvfp4`
(chronos_1t/converter/convert_glm53_flash_colab.py:81-89), and the loop around them is the grouped dense loop of
chronos_1t/models/glm53_chronos_moe.py:452-472 (sort pairs by expert, one reconstruction per distinct expert,
`F.linear` -> SwiGLU -> `F.linear` -> gate-weighted `index_add_`), with the softmax router of
chronos_1t/models/vllm_chronos_moe.py:310-314. The reference's block classes cannot be instantiated for other shapes
than their own (hard-coded group size and dimensions), which is why the loop is restated here.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

_REF = Path(__file__).resolve().parent / "_ref"
_FP8 = ("s_gu.weight_scale", "s_down.weight_scale", "healer.u_gu", "healer.v_gu", "healer.u_down", "healer.v_down")


def available() -> bool:
    return (_REF / "chronos_1t" / "models" / "glm53_holo.py").exists()


def modules():
    """(glm53_holo, convert_glm53_flash_colab) of the reference, imported from oracle/_ref."""
    if not available():
        raise RuntimeError("oracle/_ref is empty: run oracle/build_ref.py where the reference checkout is present")
    if str(_REF) not in sys.path:
        sys.path.insert(0, str(_REF))
    from chronos_1t.converter import convert_glm53_flash_colab as conv
    from chronos_1t.models import glm53_holo as holo

    return holo, conv


def group_to_torch(g: dict, device: str = "cpu") -> dict:
    """Slot dict of numpy arrays (fp8 as uint8) -> the tensors the reference functions take."""
    out = {}
    for k, v in g.items():
        t = torch.from_numpy(np.ascontiguousarray(v)) if isinstance(v, np.ndarray) else torch.as_tensor(v)
        if k in _FP8 or k.endswith("_scale") and t.dtype == torch.uint8:
            t = t.view(torch.float8_e4m3fn)
        out[k] = t.to(device)
    return out


@torch.no_grad()
def layer_forward(x: torch.Tensor, groups: dict | list, router_w: torch.Tensor, top_k: int, hidden: int, inter: int, group_size: int,
                  shared: dict | None = None, ids: torch.Tensor | None = None, gates: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 layer output [n, H] on x's device. `groups[g]` = slot g as torch tensors (see group_to_torch); `shared` = the
    plain-NVFP4 always-on expert as {sh_gu_w, sh_gu_s, sh_gu_s2, sh_dn_w, sh_dn_s, sh_dn_s2} tensors or None."""
    holo, conv = modules()
    x = x.float()
    n_tok = x.shape[0]
    if ids is None:
        logits = F.linear(x, router_w.float())
        tv, ids = torch.topk(logits, k=top_k, dim=-1)
        gates = F.softmax(tv, dim=-1)
    y = torch.zeros((n_tok, hidden), dtype=torch.float32, device=x.device)
    flat_ids, flat_w = ids.reshape(-1), gates.reshape(-1).float()
    tok_of = torch.arange(n_tok, device=x.device).repeat_interleave(ids.shape[1])
    order = torch.argsort(flat_ids)
    uniq, counts = torch.unique_consecutive(flat_ids[order], return_counts=True)
    start = 0
    for eid, cnt in zip(uniq.tolist(), counts.tolist()):
        sel = order[start:start + cnt]
        start += cnt
        if eid < 0:
            continue
        g_idx, m = eid // group_size, eid % group_size
        gu_w, dn_w = holo.reconstruct_group_experts(groups[g_idx], g_idx, [m], hidden, inter, include_tail=False)[0]
        xs = x[tok_of[sel]]
        gu = F.linear(xs, gu_w)
        act = F.silu(gu[:, :inter]) * gu[:, inter:]
        y.index_add_(0, tok_of[sel], F.linear(act, dn_w) * flat_w[sel].unsqueeze(-1))
    if shared is not None:
        i = inter
        fp8 = lambda t: t.view(torch.float8_e4m3fn) if t.dtype == torch.uint8 else t
        gate = conv.unpack_nvfp4(shared["sh_gu_w"][:i], fp8(shared["sh_gu_s"][:i]), shared["sh_gu_s2"][0])
        up = conv.unpack_nvfp4(shared["sh_gu_w"][i:], fp8(shared["sh_gu_s"][i:]), shared["sh_gu_s2"][1])
        down = conv.unpack_nvfp4(shared["sh_dn_w"], fp8(shared["sh_dn_s"]), shared["sh_dn_s2"][0])
        y += F.linear(F.silu(F.linear(x, gate)) * F.linear(x, up), down)
    return y
