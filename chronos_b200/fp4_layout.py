"""Operand images of the block-scaled FP4 tensor-core path (see csrc/bank_fp4.cu for the byte layout).

`tile_matrix_fp4` re-tiles a row-major NVFP4 matrix (packed nibbles [rows, K/2] + e4m3 scales [rows, K/16], the
on-disk layout of chronos_1t/converter/convert_glm53_flash_colab.py:77,62-65) into per-stage images: for every block
of `tile_rows` rows and every stage of 256 columns, the nibbles in K-major core-matrix order followed by the
512-byte scale blocks. It is a pure permutation of bytes (plus zero padding of scale blocks when tile_rows is not a
multiple of 128).
"""
from __future__ import annotations

import torch

STAGE_K = 256


def tile_matrix_fp4(packed: torch.Tensor, scales: torch.Tensor, tile_rows: int) -> torch.Tensor:
    """packed u8 [..., rows, K/2], scales u8 [..., rows, K/16] ->
    u8 [..., rows/tile_rows, K/256, tile_rows*128 + 2048*ceil(tile_rows/128)]: per stage the nibbles, then per MMA
    (64 columns) one 512-byte scale block per 128 rows."""
    *lead, rows, half = packed.shape
    k = half * 2
    if rows % tile_rows or k % STAGE_K or tile_rows % 32 or tile_rows > 256:
        raise ValueError("rows must be a multiple of tile_rows (32..256, multiple of 32) and K a multiple of 256")
    rb, ns = rows // tile_rows, k // STAGE_K
    nib = packed.reshape(*lead, rb, tile_rows, ns, 8, 16)                    # [.., rb, r, st, c, b]
    nd = len(lead)
    nib = nib.permute(*range(nd), nd, nd + 2, nd + 3, nd + 1, nd + 4)          # [.., rb, st, c, r, b]
    nib = nib.reshape(*lead, rb, ns, tile_rows * 128)
    nblk = (tile_rows + 127) // 128
    sf = scales.reshape(*lead, rb, tile_rows, ns, 4, 4)                       # [.., rb, r, st, j, s]
    if nblk * 128 != tile_rows:
        pad = torch.zeros(*lead, rb, nblk * 128 - tile_rows, ns, 4, 4, dtype=sf.dtype, device=sf.device)
        sf = torch.cat([sf, pad], dim=nd + 1)
    sf = sf.reshape(*lead, rb, nblk, 4, 32, ns, 4, 4)                         # [.., rb, blk, r1, r0, st, j, s]
    sf = sf.permute(*range(nd), nd, nd + 4, nd + 5, nd + 1, nd + 3, nd + 2, nd + 6)  # [.., rb, st, j, blk, r0, r1, s]
    sf = sf.reshape(*lead, rb, ns, 2048 * nblk)
    return torch.cat([nib, sf], dim=-1).contiguous()


def untile_matrix_fp4(image: torch.Tensor, tile_rows: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of `tile_matrix_fp4` for tile_rows a multiple of 128: u8 [..., rows/tile_rows, K/256, tile_rows*128 + 2048*nblk]
    -> (packed u8 [..., rows, K/2], scales u8 [..., rows, K/16]), the on-disk row-major bytes."""
    *lead, rb, ns, stage = image.shape
    nblk = tile_rows // 128
    if tile_rows % 128 or stage != tile_rows * 128 + 2048 * nblk:
        raise ValueError("not a stage image of tile_rows rows")
    nd = len(lead)
    nib = image[..., : tile_rows * 128].reshape(*lead, rb, ns, 8, tile_rows, 16)          # [.., rb, st, c, r, b]
    nib = nib.permute(*range(nd), nd, nd + 3, nd + 1, nd + 2, nd + 4)                      # [.., rb, r, st, c, b]
    packed = nib.reshape(*lead, rb * tile_rows, ns * 128).contiguous()
    sf = image[..., tile_rows * 128:].reshape(*lead, rb, ns, 4, nblk, 32, 4, 4)           # [.., rb, st, j, blk, r0, r1, s]
    sf = sf.permute(*range(nd), nd, nd + 3, nd + 5, nd + 4, nd + 1, nd + 2, nd + 6)        # [.., rb, blk, r1, r0, st, j, s]
    scales = sf.reshape(*lead, rb * tile_rows, ns * 16).contiguous()
    return packed, scales
