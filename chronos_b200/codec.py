"""Codec probes with the reference's function names and argument meaning, executed by the CUDA library.

`unpack_nvfp4` mirrors chronos_1t/converter/convert_glm53_flash_colab.py:81-89 (fp32, bit-exact);
`reconstruct_group_experts` mirrors chronos_1t/models/glm53_holo.py:336-368 (with or without the tail lattice).
Inputs must live on a CUDA device; there is no CPU implementation behind these calls.
"""
from __future__ import annotations

from typing import Mapping

import torch

from . import _lib
from .layout import FoldedLayerConfig, PackedLayer


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise _lib.ChronosError(f"{name} must be a CUDA tensor: chronos_b200 has no CPU path")


def unpack_nvfp4(packed: torch.Tensor, scale_fp8: torch.Tensor, scale_2: torch.Tensor) -> torch.Tensor:
    """packed u8 [rows, cols/2], scale_fp8 e4m3 [rows, cols/16], scale_2 f32 [] -> f32 [rows, cols]."""
    _need_cuda(packed, "packed")
    rows, half = packed.shape
    cols = half * 2
    scale_u8 = scale_fp8.view(torch.uint8) if scale_fp8.dtype == torch.float8_e4m3fn else scale_fp8
    if tuple(scale_u8.shape) != (rows, cols // 16):
        raise ValueError(f"weight_scale has shape {tuple(scale_u8.shape)}, expected {(rows, cols // 16)}")
    packed = packed.contiguous()
    scale_u8 = scale_u8.to(packed.device).contiguous()
    s2 = scale_2.to(device=packed.device, dtype=torch.float32).reshape(1).contiguous()
    out = torch.empty((rows, cols), dtype=torch.float32, device=packed.device)
    _lib.check(_lib.lib().chronos_b200_dequant_nvfp4(packed.data_ptr(), scale_u8.data_ptr(), s2.data_ptr(), out.data_ptr(),
                                                   rows, cols, _stream()))
    return out


def reconstruct_experts(layer: PackedLayer, experts: list[int]) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """fp32 (gate_up [2I, H], down [H, I]) = beta * unbind(bank) + U.V (+ tail when the layer carries it) for the
    given global expert ids."""
    c = layer.cfg
    out = []
    scratch = torch.empty(max(2 * c.inter * c.hidden, c.hidden * c.inter), dtype=torch.float32, device=layer.device)
    for e in experts:
        gu = torch.empty((2 * c.inter, c.hidden), dtype=torch.float32, device=layer.device)
        dn = torch.empty((c.hidden, c.inter), dtype=torch.float32, device=layer.device)
        _lib.check(_lib.lib().chronos_b200_unfold_expert_fp32(layer.ptr, e, 0, gu.data_ptr(), scratch.data_ptr(), _stream()))
        _lib.check(_lib.lib().chronos_b200_unfold_expert_fp32(layer.ptr, e, 1, dn.data_ptr(), scratch.data_ptr(), _stream()))
        out.append((gu, dn))
    return out


def reconstruct_group_experts(g: Mapping[str, torch.Tensor], g_idx: int, members: list[int], hidden: int, inter: int,
                              include_tail: bool = False, dtype: torch.dtype = torch.float32,
                              device: torch.device | str = "cuda") -> list[tuple[torch.Tensor, torch.Tensor]]:
    """Same call shape as the reference function; `g` holds one slot's tensors. `include_tail=True` adds the tail
    lattice term (chronos_1t/models/glm53_holo.py:362-366); the slot must then carry the `tail.*` tensors."""
    k = int(g["s_gu.beta"].shape[0])
    rank = int(g["healer.u_gu"].shape[-1])
    # a one-slot layer whose slot index is g_idx: place the slot at position g_idx of an otherwise empty table
    cfg = FoldedLayerConfig(hidden=hidden, inter=inter, n_experts=k * (g_idx + 1), group_size=k, rank=rank, top_k=1)
    groups = [g] * (g_idx + 1)
    layer = PackedLayer.from_groups(cfg, groups, device=device, include_tail=include_tail, keep_disk_order=True)
    rec = reconstruct_experts(layer, [g_idx * k + m for m in members])
    return [(a.to(dtype), b.to(dtype)) for a, b in rec]
