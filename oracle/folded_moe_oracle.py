"""CPU oracle for the folded-expert MoE forward (TEST INFRASTRUCTURE, not product code).

A numpy restatement of the reference's PyTorch algorithm for the path
  NVFP4 bank unpack -> permuted-Hadamard unbind -> + rank-r healer -> routed SwiGLU experts.
Only tests, the smoke check and the bench's CPU-baseline leg may import this module; the shipped
CUDA path never does.

Every function names the reference file:line it follows (paths relative to the Chronos project
root).  Pinned against the reference itself: `tests/golden/make_golden.py` runs the reference's
own converter and reconstruction code and stores their outputs; `tests/test_oracle_golden.py`
checks this module against those files (bit-exact where the arithmetic is integer/byte or a fixed
fp32 expression, tight fp32 tolerance where the reference uses BLAS matmuls).

fp8 (float8_e4m3fn) tensors are carried as uint8 bit patterns throughout.
"""
from __future__ import annotations

import ctypes
import math
import os
from pathlib import Path

import numpy as np

# chronos_1t/converter/convert_glm53_flash_colab.py:37 ; chronos_1t/models/chronos_moe_block.py:22
NVFP4_LUT = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32
)
# chronos_1t/converter/convert_glm53_flash_colab.py:38
LLOYD_MAX_2BIT_LUT = np.array([-1.510417, -0.452780, 0.452780, 1.510417], dtype=np.float32)
# chronos_1t/models/glm53_chronos_spec.py:33 (the reference hard-codes 8 in the seed formula, whatever K is)
SEED_GROUP_STRIDE = 8
KEY_SEED_MULT = 104729  # chronos_1t/models/glm53_holo.py:73


def _build_e4m3_table() -> np.ndarray:
    """All 256 float8_e4m3fn bit patterns as fp32 (bias 7, no inf, 0x7f/0xff = NaN)."""
    t = np.zeros(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0:
            v = (m / 8.0) * 2.0 ** -6
        elif e == 15 and m == 7:
            v = float("nan")
        else:
            v = (1.0 + m / 8.0) * 2.0 ** (e - 7)
        t[b] = s * v
    return t


E4M3_TABLE = _build_e4m3_table()
_E4M3_POS = E4M3_TABLE[:127].astype(np.float64)  # 0 .. 448, strictly increasing
_E4M3_MID = (_E4M3_POS[1:] + _E4M3_POS[:-1]) * 0.5


def e4m3_to_f32(u8: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[np.asarray(u8, dtype=np.uint8)]


def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> float8_e4m3fn bit pattern for |x| <= 448 (what `.to(torch.float8_e4m3fn)`
    does on already-clamped input, e.g. chronos_1t/converter/convert_glm53_flash_colab.py:64-65)."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64)
    idx = np.searchsorted(_E4M3_MID, a, side="left")  # a <= mid -> lower candidate
    # exact ties: choose the candidate with an even mantissa (even code)
    tie = (idx < 126) & (a == _E4M3_MID[np.minimum(idx, 125)])
    idx = np.where(tie & (idx % 2 == 1), idx + 1, idx)
    idx = np.minimum(idx, 126).astype(np.uint8)
    return np.where(np.signbit(x), idx | 0x80, idx).astype(np.uint8)


# ---------------------------------------------------------------------------------------------
# NVFP4 codec
# ---------------------------------------------------------------------------------------------
def unpack_nvfp4(packed: np.ndarray, scale_u8: np.ndarray, scale_2) -> np.ndarray:
    """chronos_1t/converter/convert_glm53_flash_colab.py:81-89.
    value = fl32( lut[nibble] * fl32( float(e4m3 scale) * scale_2 ) ); even column = low nibble (:77)."""
    packed = np.asarray(packed, dtype=np.uint8)
    rows = packed.shape[0]
    low = packed & 0x0F
    high = (packed >> 4) & 0x0F
    nib = np.stack([low, high], axis=-1).reshape(rows, -1)
    vals = NVFP4_LUT[nib].reshape(rows, -1, 16)
    scales = e4m3_to_f32(scale_u8).astype(np.float32)[..., None] * np.float32(scale_2)
    return (vals * scales.astype(np.float32)).astype(np.float32).reshape(rows, -1)


def pack_nvfp4(w: np.ndarray):
    """chronos_1t/converter/convert_glm53_flash_colab.py:56-78 (fp32 arithmetic, same operand order)."""
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    f32 = np.float32
    w_amax = np.maximum(np.abs(w).max(), f32(1e-12)).astype(f32)
    scale_2 = f32(w_amax / f32(6.0 * 448.0))
    w_blk = w.reshape(rows, cols // 16, 16)
    blk_max = np.abs(w_blk).max(axis=-1)
    raw_s = np.clip((blk_max / (f32(6.0) * scale_2)).astype(f32), f32(1e-6), f32(448.0))
    scale_u8 = f32_to_e4m3(raw_s)
    eff_s = np.maximum((e4m3_to_f32(scale_u8) * scale_2).astype(f32), f32(1e-12))[..., None]
    w_norm = (w_blk / eff_s).astype(f32)
    signs = (w_norm < 0).astype(np.uint8) << 3
    abs_v = np.abs(w_norm)
    idx = np.zeros(abs_v.shape, dtype=np.uint8)
    for ti, th in enumerate((0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0), start=1):
        idx = np.where(abs_v >= f32(th), np.uint8(ti), idx)
    nib = (signs | idx).reshape(rows, cols)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    return packed, scale_u8, scale_2


def dequant_fp8_block(w_u8: np.ndarray, scale_inv: np.ndarray, block: int = 128) -> np.ndarray:
    """chronos_1t/models/glm53_tiers.py:74-95 with dtype=float32: value = float(e4m3) * scale_inv[row // 128, col // 128]."""
    w = e4m3_to_f32(w_u8)
    n, k = w.shape
    s = np.asarray(scale_inv, dtype=np.float32)
    s_full = np.repeat(np.repeat(s, block, axis=0)[:n], block, axis=1)[:, :k]
    return (w * s_full).astype(np.float32)


def shared_fp8_weights(ex: dict):
    """fp32 (gate_up [2I, H], down [H, I]) of a block-FP8 shared expert given as sh8_gu_w / sh8_gu_s / sh8_dn_w / sh8_dn_s
    (gate rows, then up rows: chronos_1t/models/glm53_chronos_moe.py:176-181)."""
    return dequant_fp8_block(ex["sh8_gu_w"], ex["sh8_gu_s"]), dequant_fp8_block(ex["sh8_dn_w"], ex["sh8_dn_s"])


# ---------------------------------------------------------------------------------------------
# Tail lattices (carried by the on-disk format; excluded from the timed path)
# ---------------------------------------------------------------------------------------------
def unpack_tail_2bit(packed: np.ndarray, sigma_u8: np.ndarray, block: int = 32) -> np.ndarray:
    """chronos_1t/converter/convert_glm53_flash_colab.py:181-191, one expert: packed [rows, cols/4]."""
    rows, pc = packed.shape
    codes = np.stack([(packed >> s) & 3 for s in (0, 2, 4, 6)], axis=-1).reshape(rows, pc * 4)
    vals = LLOYD_MAX_2BIT_LUT[codes].reshape(rows, -1, block)
    return (vals * e4m3_to_f32(sigma_u8)[..., None]).astype(np.float32).reshape(rows, pc * 4)


def unpack_tail_1bit(packed: np.ndarray, sigma_u8: np.ndarray, block: int = 64) -> np.ndarray:
    """chronos_1t/converter/convert_glm53_flash_colab.py:206-211, one expert: packed [rows, cols/8]."""
    rows, pc = packed.shape
    bits = np.stack([(packed >> b) & 1 for b in range(8)], axis=-1).reshape(rows, pc * 8)
    signs = bits.astype(np.float32) * 2.0 - 1.0
    return (signs.reshape(rows, -1, block) * e4m3_to_f32(sigma_u8)[..., None]).astype(np.float32).reshape(rows, pc * 8)


# ---------------------------------------------------------------------------------------------
# Keys and the 128-block Hadamard
# ---------------------------------------------------------------------------------------------
def group_seed_bases(g_idx: int):
    """chronos_1t/models/glm53_chronos_spec.py:194-196."""
    return 101 + g_idx * SEED_GROUP_STRIDE, 303 + g_idx * SEED_GROUP_STRIDE


def expert_keys(rows: int, cols: int, local_m: int, seed_base: int):
    """chronos_1t/models/glm53_holo.py:66-86 — draws come from torch's CPU generator (the recorded
    `key_generator = "torch_cpu_v1"`); the stream is torch's, so torch is called rather than re-implemented.
    Returns (r_s1, r_perm, r_inv, r_s2, c_s1, c_perm, c_inv, c_s2): signs fp32 +-1, perms int64."""
    import torch

    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed_base + (local_m + 1) * KEY_SEED_MULT)
    r_s1 = torch.randint(0, 2, (rows,), generator=gen, dtype=torch.int8).float() * 2.0 - 1.0
    r_perm = torch.randperm(rows, generator=gen)
    r_s2 = torch.randint(0, 2, (rows,), generator=gen, dtype=torch.int8).float() * 2.0 - 1.0
    c_s1 = torch.randint(0, 2, (cols,), generator=gen, dtype=torch.int8).float() * 2.0 - 1.0
    c_perm = torch.randperm(cols, generator=gen)
    c_s2 = torch.randint(0, 2, (cols,), generator=gen, dtype=torch.int8).float() * 2.0 - 1.0
    out = (r_s1, r_perm, torch.argsort(r_perm), r_s2, c_s1, c_perm, torch.argsort(c_perm), c_s2)
    return tuple(t.numpy() for t in out)


def hadamard128() -> np.ndarray:
    """chronos_1t/converter/convert_glm53_flash_colab.py:41-45 — Sylvester H_128 / sqrt(128)."""
    h = np.array([[1.0]], dtype=np.float32)
    for _ in range(7):
        h = np.block([[h, h], [h, -h]])
    return (h / np.float32(math.sqrt(128.0))).astype(np.float32)


_H128 = hadamard128()


def _had_blocks(v: np.ndarray) -> np.ndarray:
    """Orthonormal H_128 on every contiguous 128-block of the last axis."""
    shp = v.shape
    return (v.reshape(*shp[:-1], shp[-1] // 128, 128) @ _H128).reshape(shp).astype(np.float32)


def fold_2d(w: np.ndarray, keys) -> np.ndarray:
    """chronos_1t/converter/convert_glm53_flash_colab.py:106-127 for one expert (w [rows, cols])."""
    r_s1, r_perm, _, r_s2, c_s1, c_perm, _, c_s2 = keys
    x = (w * c_s1[None, :])[:, c_perm]
    x = _had_blocks(x) * c_s2[None, :]
    xt = np.ascontiguousarray(x.T) * r_s1[None, :]
    xt = xt[:, r_perm]
    xt = _had_blocks(xt) * r_s2[None, :]
    return np.ascontiguousarray(xt.T).astype(np.float32)


def unbind_2d(s_mat: np.ndarray, keys) -> np.ndarray:
    """chronos_1t/converter/convert_glm53_flash_colab.py:130-151 for one expert."""
    r_s1, _, r_inv, r_s2, c_s1, _, c_inv, c_s2 = keys
    xt = np.ascontiguousarray(s_mat.T) * r_s2[None, :]
    xt = _had_blocks(xt)
    xt = xt[:, r_inv] * r_s1[None, :]
    x = np.ascontiguousarray(xt.T) * c_s2[None, :]
    x = _had_blocks(x)
    return (x[:, c_inv] * c_s1[None, :]).astype(np.float32)


# ---------------------------------------------------------------------------------------------
# Expert reconstruction (the "fp32 reconstruction" the layer tolerance refers to)
# ---------------------------------------------------------------------------------------------
def unpack_banks(g: dict):
    """Both banks of a slot dequantised once (chronos_1t/models/glm53_holo.py:350-351)."""
    return (unpack_nvfp4(g["s_gu.weight"], g["s_gu.weight_scale"], g["s_gu.weight_scale_2"]),
            unpack_nvfp4(g["s_down.weight"], g["s_down.weight_scale"], g["s_down.weight_scale_2"]))


def reconstruct_expert(g: dict, g_idx: int, m: int, hidden: int, inter: int, include_tail: bool = False, banks=None):
    """chronos_1t/models/glm53_holo.py:336-368 for one member `m` of group `g_idx`.
    `g` maps the on-disk suffixes (glm53_holo.py:45-51) to numpy arrays (fp8 as uint8). `banks` = `unpack_banks(g)`
    when the caller handles several members of a slot (the reference unpacks once per group call, :350-351).
    Returns (gu [2I,H], down [H,I])."""
    seed_gu, seed_dn = group_seed_bases(g_idx)
    s_gu, s_dn = banks if banks is not None else unpack_banks(g)
    kg = expert_keys(2 * inter, hidden, m, seed_gu)
    kd = expert_keys(hidden, inter, m, seed_dn)
    h_gu = unbind_2d(s_gu, kg)
    h_dn = unbind_2d(s_dn, kd)
    gu = np.float32(g["s_gu.beta"][m]) * h_gu + e4m3_to_f32(g["healer.u_gu"][m]) @ e4m3_to_f32(g["healer.v_gu"][m])
    dn = np.float32(g["s_down.beta"][m]) * h_dn + e4m3_to_f32(g["healer.u_down"][m]) @ e4m3_to_f32(g["healer.v_down"][m])
    if include_tail:
        gb = int(g["tail.gu_bits"]) if "tail.gu_bits" in g else 2
        db = int(g["tail.down_bits"]) if "tail.down_bits" in g else 2
        gu = gu + (unpack_tail_2bit if gb == 2 else unpack_tail_1bit)(g["tail.gu_packed"][m], g["tail.gu_scale"][m])
        dn = dn + (unpack_tail_2bit if db == 2 else unpack_tail_1bit)(g["tail.down_packed"][m], g["tail.down_scale"][m])
    return gu.astype(np.float32), dn.astype(np.float32)


def expert_forward_activation_space(x: np.ndarray, g: dict, g_idx: int, m: int, hidden: int, inter: int) -> np.ndarray:
    """chronos_1t/models/glm5_chronos_moe.py:149-195 with the hard-coded 4096/2048 dims made generic, fp32.
    The bank is used as stored; only activations are transformed. x [n, H] -> y [n, H]."""
    x = np.asarray(x, dtype=np.float32)
    return _expert_rows_activation_space(x, g, g_idx, m, hidden, inter, unpack_banks(g))


def silu(z: np.ndarray) -> np.ndarray:
    z = np.asarray(z, dtype=np.float32)
    return (z / (1.0 + np.exp(-z.astype(np.float64)))).astype(np.float32)


# ---------------------------------------------------------------------------------------------
# Router
# ---------------------------------------------------------------------------------------------
_CLIB = None


def _clib():
    """Loads the C part of the oracle (fixed-order fp32 reductions), building it on first use."""
    global _CLIB
    if _CLIB is None:
        here = Path(__file__).resolve().parent
        so = here / "liboracle_c.so"
        src = here / "oracle_kernels.c"
        if not so.exists() or so.stat().st_mtime < src.stat().st_mtime:
            import subprocess

            subprocess.check_call(["make", "-s", "-C", str(here), "liboracle_c.so"])
        lib = ctypes.CDLL(str(so))
        lib.oracle_router_logits_fixed.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 3
        lib.oracle_router_logits_fixed.restype = None
        lib.oracle_set_threads.argtypes = [ctypes.c_int]
        _CLIB = lib
    return _CLIB


def router_logits_fixed(x: np.ndarray, wr: np.ndarray) -> np.ndarray:
    """fp32 logits = x . Wr^T (chronos_1t/models/vllm_chronos_moe.py:311) in ONE stated summation order, so a
    device kernel can reproduce them bit for bit: lane l of 32 accumulates the products at k = 128 j + 4 l + i
    (j = 0, 1, ...; i = 0..3; j ascending, then i) with fused multiply-adds starting from +0, then lanes are combined by
    the xor butterfly 16, 8, 4, 2, 1."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    wr = np.ascontiguousarray(wr, dtype=np.float32)
    t, h = x.shape
    e = wr.shape[0]
    out = np.empty((t, e), dtype=np.float32)
    _clib().oracle_router_logits_fixed(x.ctypes.data, wr.ctypes.data, out.ctypes.data, t, e, h)
    return out


def topk_desc(vals: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest per row, descending; equal values -> lower index first. A candidate that is NaN or
    -inf can never be chosen: once only such candidates are left the remaining positions hold -1 (an entry every
    consumer skips). The reference's `torch.topk` has no defined answer for NaN rows; this is the stated rule of the
    device kernels."""
    v = np.asarray(vals, dtype=np.float64)
    v = np.where(np.isnan(v), -np.inf, v)
    order = np.lexsort((np.broadcast_to(np.arange(v.shape[1]), v.shape), -v), axis=1)
    ids = order[:, :k].astype(np.int64)
    chosen = np.take_along_axis(v, ids, axis=1)
    return np.where(np.isneginf(chosen), -1, ids)


def _gather_valid(src: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """src[t, ids[t, j]] with 0 where ids is -1."""
    return np.where(ids >= 0, np.take_along_axis(src, np.maximum(ids, 0), axis=1), np.float32(0.0)).astype(np.float32)


def router_softmax_topk(logits: np.ndarray, k: int):
    """chronos_1t/models/vllm_chronos_moe.py:310-314: topk(logits) then softmax over the k values (fp32)."""
    ids = topk_desc(logits, k)
    tv = _gather_valid(logits, ids)
    with np.errstate(invalid="ignore", divide="ignore"):
        ex = np.where(ids >= 0, np.exp((tv - tv[:, :1]).astype(np.float32)), np.float32(0.0)).astype(np.float32)
        w = (ex / ex.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return ids, np.where(ids >= 0, w, np.float32(0.0)).astype(np.float32)


def _noaux_topk(scores: np.ndarray, e_bias, k: int, routed_scaling: float, renorm: bool):
    """`noaux_tc` selection shared by the sigmoid and sqrt-softplus routers: choose by score + bias, weigh by the
    unbiased scores, optional renormalisation, times the routed scaling factor."""
    bias = np.zeros(scores.shape[1], dtype=np.float32) if e_bias is None else np.asarray(e_bias, dtype=np.float32)
    ids = topk_desc(scores + bias[None, :], k)
    w = _gather_valid(scores, ids)
    if renorm:
        w = w / (w.sum(axis=1, keepdims=True, dtype=np.float32) + np.float32(1e-20))
    return ids, np.where(ids >= 0, w * np.float32(routed_scaling), np.float32(0.0)).astype(np.float32)


def router_sigmoid_topk(logits: np.ndarray, e_bias: np.ndarray, k: int, routed_scaling: float = 2.5, renorm: bool = True):
    """chronos_1t/models/glm53_chronos_moe.py:392-399 (`noaux_tc`): choose by sigmoid+bias, weigh by unbiased scores."""
    scores = (1.0 / (1.0 + np.exp(-logits.astype(np.float32)))).astype(np.float32)
    return _noaux_topk(scores, e_bias, k, routed_scaling, renorm)


def softplus(x: np.ndarray) -> np.ndarray:
    """torch.nn.functional.softplus with beta 1, threshold 20 (fp32): x above the threshold passes through."""
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(over="ignore"):
        return np.where(x > np.float32(20.0), x, np.log1p(np.exp(x)).astype(np.float32)).astype(np.float32)


def router_sqrt_softplus_topk(logits: np.ndarray, e_bias, k: int, routed_scaling: float = 1.5, renorm: bool = True):
    """chronos_1t/models/dsv41_chronos_moe.py:3402-3410: scores = sqrt(softplus(logits)); topk(scores + bias); weights =
    unbiased scores, divided by their sum (+1e-20), times routed_scaling_factor."""
    scores = np.sqrt(softplus(logits)).astype(np.float32)
    return _noaux_topk(scores, e_bias, k, routed_scaling, renorm)


def router_coalesced(logits: np.ndarray, k: int, tokens_per_stream: int = 3, pool: int = 12, keep: int = 4, bonus: float = 1.0e4,
                     router: str = "softmax", e_bias=None, routed_scaling: float = 2.5, renorm: bool = True):
    """Batch-coalesced selection for speculative verify batches. PARITY UNPINNED: the reference only describes the policy
    (README.md:56, :208, :372; docs/CHRONOS_ARCHITECTURE_PAPER.md:270-277 - the kernel's source is not part of it), so
    this restates the clean-room rule of the device kernel, and the tests check the invariants the reference states:
    the anchor (token 0 of a stream) is untouched; a draft never leaves its natural top-`pool`; its `keep` best natural
    experts stay; the rest prefers experts the anchor selected (score + bonus), ties to the better natural rank."""
    lg = np.asarray(logits, dtype=np.float32)
    bias = np.zeros(lg.shape[1], dtype=np.float32) if e_bias is None else np.asarray(e_bias, dtype=np.float32)
    if router == "softmax":
        score = lg
        choice = lg
    else:
        score = (1.0 / (1.0 + np.exp(-lg))).astype(np.float32) if router == "sigmoid" else np.sqrt(softplus(lg)).astype(np.float32)
        choice = (score + bias[None, :]).astype(np.float32)
    n = lg.shape[0]
    nat = topk_desc(choice, pool)
    ids = np.full((n, k), -1, dtype=np.int64)
    for t in range(n):
        if t % tokens_per_stream == 0:
            ids[t] = nat[t, :k]
            continue
        anchor = set(int(e) for e in ids[t - t % tokens_per_stream] if e >= 0)
        cand = [(j, int(e)) for j, e in enumerate(nat[t]) if e >= 0]
        kept = [e for j, e in cand if j < keep]
        rest = [(j, e) for j, e in cand if j >= keep]
        key = lambda je: (-(np.float32(choice[t, je[1]]) + (np.float32(bonus) if je[1] in anchor else np.float32(0.0))), je[0])
        picked = kept + [e for _, e in sorted(rest, key=key)][: k - len(kept)]
        ids[t, : len(picked)] = picked
    w = _gather_valid(score, ids)
    if router == "softmax":
        with np.errstate(invalid="ignore", divide="ignore"):
            mx = np.where(ids >= 0, w, -np.inf).max(axis=1, keepdims=True)
            ex = np.where(ids >= 0, np.exp((w - mx).astype(np.float32)), np.float32(0.0)).astype(np.float32)
            w = (ex / ex.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    else:
        if renorm:
            w = w / (w.sum(axis=1, keepdims=True, dtype=np.float32) + np.float32(1e-20))
        w = (w * np.float32(routed_scaling)).astype(np.float32)
    return ids, np.where(ids >= 0, w, np.float32(0.0)).astype(np.float32)


# ---------------------------------------------------------------------------------------------
# Layer forward (grouped dense loop over distinct experts)
# ---------------------------------------------------------------------------------------------
def moe_layer_forward(x, groups, router_w, top_k, hidden, inter, group_size, router="softmax", e_bias=None,
                      routed_scaling=2.5, shared=None, logits=None, include_tail=False, return_routing=False):
    """Routed SwiGLU MoE in fp32 following chronos_1t/models/glm53_chronos_moe.py:452-472 (sort pairs by expert,
    handle each distinct expert once) with weights from `reconstruct_expert` (glm53_holo.py:336-368).
    `groups[g]` is the tensor dict of slot g; expert e = (slot e // group_size, member e % group_size).
    `shared` = optional (gu [2I_s,H], down [H,I_s]) fp32 always-on expert added with weight 1
    (chronos_1t/models/glm5_chronos_moe.py:457-458)."""
    x = np.asarray(x, dtype=np.float32)
    n_tok = x.shape[0]
    if logits is None:
        logits = router_logits_fixed(x, router_w)
    if router == "softmax":
        ids, w = router_softmax_topk(logits, top_k)
    elif router == "sqrt_softplus":
        ids, w = router_sqrt_softplus_topk(logits, e_bias, top_k, routed_scaling)
    else:
        ids, w = router_sigmoid_topk(logits, e_bias, top_k, routed_scaling)
    y = np.zeros((n_tok, hidden), dtype=np.float32)
    flat_ids = ids.reshape(-1)
    flat_w = w.reshape(-1)
    tok_of = np.repeat(np.arange(n_tok), top_k)
    bank_cache: tuple = (-1, None)  # each distinct slot is dequantised once (chronos_1t/models/glm5_chronos_moe.py:530-539)
    for eid in np.unique(flat_ids[flat_ids >= 0]):  # -1 = no expert chosen (see topk_desc)
        sel = np.nonzero(flat_ids == eid)[0]
        g_idx, m = int(eid) // group_size, int(eid) % group_size
        if bank_cache[0] != g_idx:
            bank_cache = (g_idx, unpack_banks(groups[g_idx]))
        gu_w, dn_w = reconstruct_expert(groups[g_idx], g_idx, m, hidden, inter, include_tail=include_tail, banks=bank_cache[1])
        xs = x[tok_of[sel]]
        gu = xs @ gu_w.T
        act = silu(gu[:, :inter]) * gu[:, inter:]
        np.add.at(y, tok_of[sel], (act @ dn_w.T) * flat_w[sel][:, None])
    if shared is not None:
        sgu, sdn = shared
        si = sdn.shape[1]
        z = x @ sgu.T
        y = y + (silu(z[:, :si]) * z[:, si:]) @ sdn.T
    if return_routing:
        return y.astype(np.float32), ids, w
    return y.astype(np.float32)


def routed_tokens_activation_space(x, ids, gates, groups, hidden, inter, group_size, shared=None, first_slot=0):
    """Layer output rows for explicit routing, evaluated in activation space: every (token, expert) pair goes through
    `expert_forward_activation_space` (chronos_1t/models/glm5_chronos_moe.py:149-195), pairs grouped by expert and the
    slot's banks dequantised once per slot (chronos_1t/models/glm5_chronos_moe.py:530-539). Algebraically the same as
    multiplying by the fp32 reconstruction (the two are pinned against each other by the golden tests) but without
    forming any [rows, cols] expert matrix, so a sample of tokens of a full-size layer takes seconds.
    x [n, H] fp32, ids [n, k] (global expert ids, < 0 skipped), gates [n, k]; `groups[g - first_slot]` is slot g.
    `shared` = optional (gu [2I, H], down [H, I]) fp32 always-on expert."""
    x = np.asarray(x, dtype=np.float32)
    ids = np.asarray(ids)
    gates = np.asarray(gates, dtype=np.float32)
    y = np.zeros((x.shape[0], hidden), dtype=np.float32)
    order = sorted({int(e) for e in ids.reshape(-1) if e >= 0})
    cache: tuple = (-1, None)
    for eid in order:
        g_idx, m = eid // group_size, eid % group_size
        g = groups[g_idx - first_slot]
        if cache[0] != g_idx:
            cache = (g_idx, unpack_banks(g))
        t_idx, j_idx = np.nonzero(ids == eid)
        out = _expert_rows_activation_space(x[t_idx], g, g_idx, m, hidden, inter, cache[1])
        np.add.at(y, t_idx, out * gates[t_idx, j_idx][:, None])
    if shared is not None:
        sgu, sdn = shared
        si = sdn.shape[1]
        z = x @ sgu.T
        y = y + (silu(z[:, :si]) * z[:, si:]) @ sdn.T
    return y.astype(np.float32)


def _expert_rows_activation_space(x, g, g_idx, m, hidden, inter, banks):
    """`expert_forward_activation_space` with the slot's dequantised banks supplied by the caller."""
    seed_gu, seed_dn = group_seed_bases(g_idx)
    s_gu, s_dn = banks
    r_s1, _, r_inv, r_s2, c_s1, c_perm, _, c_s2 = expert_keys(2 * inter, hidden, m, seed_gu)
    x_c = _had_blocks((x * c_s1[None, :])[:, c_perm]) * c_s2[None, :]
    z = _had_blocks((x_c @ s_gu.T) * r_s2[None, :])[:, r_inv] * r_s1[None, :]
    u, v = e4m3_to_f32(g["healer.u_gu"][m]), e4m3_to_f32(g["healer.v_gu"][m])
    z = np.float32(g["s_gu.beta"][m]) * z + (x @ v.T) @ u.T
    act = silu(z[:, :inter]) * z[:, inter:]
    r_s1, _, r_inv, r_s2, c_s1, c_perm, _, c_s2 = expert_keys(hidden, inter, m, seed_dn)
    a_c = _had_blocks((act * c_s1[None, :])[:, c_perm]) * c_s2[None, :]
    yv = _had_blocks((a_c @ s_dn.T) * r_s2[None, :])[:, r_inv] * r_s1[None, :]
    u, v = e4m3_to_f32(g["healer.u_down"][m]), e4m3_to_f32(g["healer.v_down"][m])
    return (np.float32(g["s_down.beta"][m]) * yv + (act @ v.T) @ u.T).astype(np.float32)


def rms_norm(x: np.ndarray, eps: float = 1e-6, weight=None) -> np.ndarray:
    """chronos_1t/models/glm53_engine.py:71-73 (fp32: w * x * rsqrt(mean(x^2) + eps))."""
    x = np.asarray(x, dtype=np.float32)
    y = x * (1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True, dtype=np.float32) + np.float32(eps))).astype(np.float32)
    return y if weight is None else (y * weight).astype(np.float32)


# ---------------------------------------------------------------------------------------------
# Synthetic slot builder (test / bench INPUT generator — not a parity object)
# ---------------------------------------------------------------------------------------------
def fold_group_synthetic(gate, up, down, g_idx: int, rank: int, seed: int = 0) -> dict:
    """Folds K experts into one slot with the reference's fold + NVFP4 pack + least-squares beta
    (chronos_1t/models/glm53_holo.py:179-203) and a plain randomised rank-`rank` SVD healer of the residual
    quantised to e4m3. The converter's router-importance weights, SMW weighting, tail and Woodbury steps are left
    out: they only change which bytes get written, not how bytes are read. Produces valid on-disk-format tensors
    with realistic value distributions for inputs the real converter would be too slow to produce."""
    k, inter, hid = gate.shape
    gu_b = np.concatenate([gate, up], axis=1).astype(np.float32)
    dn_b = np.asarray(down, dtype=np.float32)
    seed_gu, seed_dn = group_seed_bases(g_idx)
    rng = np.random.default_rng(seed * 7919 + g_idx)
    out: dict = {}
    for name, w_b, sb in (("gu", gu_b, seed_gu), ("down", dn_b, seed_dn)):
        rows, cols = w_b.shape[1:]
        keys = [expert_keys(rows, cols, m, sb) for m in range(k)]
        s = sum(fold_2d(w_b[m], keys[m]) for m in range(k)) / np.float32(math.sqrt(k))
        p, sc, s2 = pack_nvfp4(s.astype(np.float32))
        sq = unpack_nvfp4(p, sc, s2)
        betas, us, vs = [], [], []
        for m in range(k):
            h = unbind_2d(sq, keys[m])
            beta = float((w_b[m] * h).sum() / max(float((h * h).sum()), 1e-12))
            res = w_b[m] - np.float32(beta) * h
            q, _ = np.linalg.qr(res @ (res.T @ rng.standard_normal((rows, rank + 8)).astype(np.float32)))
            uu, ss, vv = np.linalg.svd(q.T @ res, full_matrices=False)
            sq_s = np.sqrt(ss[:rank]).astype(np.float32)
            us.append(f32_to_e4m3(np.clip((q @ uu[:, :rank]) * sq_s[None, :], -448, 448)))
            vs.append(f32_to_e4m3(np.clip(vv[:rank] * sq_s[:, None], -448, 448)))
            betas.append(beta)
        sfx = "s_gu" if name == "gu" else "s_down"
        out[f"{sfx}.weight"], out[f"{sfx}.weight_scale"] = p, sc
        out[f"{sfx}.weight_scale_2"] = np.float32(s2)
        out[f"{sfx}.beta"] = np.array(betas, dtype=np.float32)
        out[f"healer.u_{name}"], out[f"healer.v_{name}"] = np.stack(us), np.stack(vs)
    return out


def random_group(rng: np.random.Generator, k: int, hidden: int, inter: int, rank: int) -> dict:
    """Valid on-disk-format slot made of random bytes in the ranges the converter emits (fast; for big shapes)."""
    out: dict = {}
    for sfx, name, rows, cols in (("s_gu", "gu", 2 * inter, hidden), ("s_down", "down", hidden, inter)):
        out[f"{sfx}.weight"] = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
        # e4m3 codes 0x58..0x77 = 12 .. 240: block scales of a bank whose max block is ~4x its typical block
        out[f"{sfx}.weight_scale"] = rng.integers(0x58, 0x78, (rows, cols // 16), dtype=np.uint8)
        out[f"{sfx}.weight_scale_2"] = np.float32(0.08 / (6.0 * 448.0))
        out[f"{sfx}.beta"] = rng.uniform(0.3, 0.7, k).astype(np.float32)
        # healer factors ~ N(0, 0.05): e4m3 of small normals, both signs
        out[f"healer.u_{name}"] = f32_to_e4m3(rng.standard_normal((k, rows, rank)).astype(np.float32) * 0.05)
        out[f"healer.v_{name}"] = f32_to_e4m3(rng.standard_normal((k, rank, cols)).astype(np.float32) * 0.05)
    return out


def set_threads(n: int) -> None:
    _clib().oracle_set_threads(int(n))
    os.environ["OMP_NUM_THREADS"] = str(n)
