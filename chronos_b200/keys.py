"""Seeded sign / permutation keys of the folded experts and their compact device tables.

The draws follow `expert_keys` of the reference (chronos_1t/models/glm53_holo.py:66-86): a CPU `torch.Generator`
seeded with `seed_base + (member + 1) * 104729`, draw order r_s1, r_perm, r_s2, c_s1, c_perm, c_s2. The stream is
torch's own (`key_generator = "torch_cpu_v1"`), so torch is called rather than re-implemented.
"""
from __future__ import annotations

import numpy as np
import torch

KEY_SEED_MULT = 104729
SEED_GROUP_STRIDE = 8  # the reference keeps 8 in the seed formula whatever the fold factor is (glm53_chronos_spec.py:33,194-196)


def group_seed_bases(g_idx: int, stride: int = SEED_GROUP_STRIDE) -> tuple[int, int]:
    """(gate_up seed base, down seed base) of slot `g_idx` (chronos_1t/models/glm53_chronos_spec.py:194-196)."""
    return 101 + g_idx * stride, 303 + g_idx * stride


def expert_keys(rows: int, cols: int, local_m: int, seed_base: int) -> tuple[torch.Tensor, ...]:
    """(r_s1, r_perm, r_inv, r_s2, c_s1, c_perm, c_inv, c_s2) on the CPU; signs fp32 +-1, perms int64."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed_base + (local_m + 1) * KEY_SEED_MULT)
    r_s1 = torch.randint(0, 2, (rows,), generator=gen, dtype=torch.int8).float() * 2.0 - 1.0
    r_perm = torch.randperm(rows, generator=gen)
    r_s2 = torch.randint(0, 2, (rows,), generator=gen, dtype=torch.int8).float() * 2.0 - 1.0
    c_s1 = torch.randint(0, 2, (cols,), generator=gen, dtype=torch.int8).float() * 2.0 - 1.0
    c_perm = torch.randperm(cols, generator=gen)
    c_s2 = torch.randint(0, 2, (cols,), generator=gen, dtype=torch.int8).float() * 2.0 - 1.0
    return r_s1, r_perm, torch.argsort(r_perm), r_s2, c_s1, c_perm, torch.argsort(c_perm), c_s2


def _bitmask_u32(neg: np.ndarray) -> np.ndarray:
    """bit (j % 32) of word (j // 32) = neg[j]."""
    return np.packbits(neg.astype(np.uint8), bitorder="little").view("<u4").copy()


def compact_tables(rows: int, cols: int, local_m: int, seed_base: int) -> dict[str, np.ndarray]:
    """Device tables of one expert matrix:
      cin  u16 [cols]    bits 0-14 = c_perm[j], bit 15 = (c_s1[c_perm[j]] < 0)   (input gather + sign)
      cs2  u32 [cols/32] bit = (c_s2[j] < 0)
      rout u16 [rows]    bits 0-14 = r_inv[i],  bit 15 = (r_s1[i] < 0)           (output gather + sign)
      rs2  u32 [rows/32] bit = (r_s2[i] < 0)
    """
    if rows > 32768 or cols > 32768 or rows % 32 or cols % 32:
        raise ValueError("key tables need dimensions that are multiples of 32 and at most 32768")
    r_s1, _, r_inv, r_s2, c_s1, c_perm, _, c_s2 = (t.numpy() for t in expert_keys(rows, cols, local_m, seed_base))
    cin = c_perm.astype(np.uint16) | ((c_s1[c_perm] < 0).astype(np.uint16) << 15)
    rout = r_inv.astype(np.uint16) | ((r_s1 < 0).astype(np.uint16) << 15)
    return {"cin": cin, "cs2": _bitmask_u32(c_s2 < 0), "rout": rout, "rs2": _bitmask_u32(r_s2 < 0)}
