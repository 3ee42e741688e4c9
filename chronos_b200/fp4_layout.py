"""Operand images of the block-scaled FP4 tensor-core path (see csrc/bank_fp4.cu for the byte layout).

`tile_matrix_fp4` re-tiles a row-major NVFP4 matrix (packed nibbles [rows, K/2] + e4m3 scales [rows, K/16], the
on-disk layout of chronos_1t/converter/convert_glm53_flash_colab.py:77,62-65) into per-stage images: for every block
of `tile_rows` rows and every stage of 256 columns, the nibbles in K-major core-matrix order followed by four
512-byte scale blocks. It is a pure permutation of bytes (plus zero padding of scale blocks when tile_rows < 128).
"""
from __future__ import annotations

import torch

STAGE_K = 256


def tile_matrix_fp4(packed: torch.Tensor, scales: torch.Tensor, tile_rows: int) -> torch.Tensor:
    """packed u8 [..., rows, K/2], scales u8 [..., rows, K/16] -> u8 [..., rows/tile_rows, K/256, tile_rows*128 + 2048]."""
    *lead, rows, half = packed.shape
    k = half * 2
    if rows % tile_rows or k % STAGE_K or tile_rows % 32 or tile_rows > 128:
        raise ValueError("rows must be a multiple of tile_rows (32..128, multiple of 32) and K a multiple of 256")
    rb, ns = rows // tile_rows, k // STAGE_K
    nib = packed.reshape(*lead, rb, tile_rows, ns, 8, 16)                    # [.., rb, r, st, c, b]
    nd = len(lead)
    nib = nib.permute(*range(nd), nd, nd + 2, nd + 3, nd + 1, nd + 4)          # [.., rb, st, c, r, b]
    nib = nib.reshape(*lead, rb, ns, tile_rows * 128)
    sf = scales.reshape(*lead, rb, tile_rows // 32, 32, ns, 4, 4)             # [.., rb, r1, r0, st, j, s]
    sf = sf.permute(*range(nd), nd, nd + 3, nd + 4, nd + 2, nd + 1, nd + 5)   # [.., rb, st, j, r0, r1, s]
    if tile_rows < 128:
        pad = torch.zeros(*sf.shape[:-2], 4 - tile_rows // 32, 4, dtype=sf.dtype, device=sf.device)
        sf = torch.cat([sf, pad], dim=-2)
    sf = sf.reshape(*lead, rb, ns, 2048)
    return torch.cat([nib, sf], dim=-1).contiguous()
