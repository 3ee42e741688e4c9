"""Device-resident packed layout of one folded MoE layer and its `chronos_layer_t` view.

The bank and healer bytes are the converter's on-disk bytes (chronos_1t/models/glm53_holo.py:291-302), stacked
over slots / experts; nothing is re-quantised. Two load-time rearrangements that do not touch the file format:
`healer.v_down` is stored transposed ([I, r] per expert) and the seeded keys are compacted into gather tables.
"""
from __future__ import annotations

import ctypes as C
import math
import re
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Iterable, Mapping

import numpy as np
import torch

from . import _lib, keys

GROUP_TENSOR_SUFFIXES = (  # chronos_1t/models/glm53_holo.py:45-51
    "s_gu.weight", "s_gu.weight_scale", "s_gu.weight_scale_2", "s_gu.beta",
    "s_down.weight", "s_down.weight_scale", "s_down.weight_scale_2", "s_down.beta",
    "healer.u_gu", "healer.v_gu", "healer.u_down", "healer.v_down",
    "tail.gu_bits", "tail.gu_packed", "tail.gu_scale",
    "tail.down_bits", "tail.down_packed", "tail.down_scale",
)
ROUTER_KINDS = {"softmax": _lib.ROUTER_SOFTMAX_TOPK, "sigmoid": _lib.ROUTER_SIGMOID_NOAUX, "sqrt_softplus": _lib.ROUTER_SQRT_SOFTPLUS}
_REQUIRED = GROUP_TENSOR_SUFFIXES[:12]  # the tail lattice tensors are optional (include_tail)


@dataclass
class FoldedLayerConfig:
    """Shape and router description of a folded layer (mirrors the `chronos_holographic_moe` block of config.json,
    chronos_1t/converter/convert_glm53_chronos.py:544-561, plus the router fields of the model config)."""

    hidden: int
    inter: int
    n_experts: int
    group_size: int
    rank: int
    top_k: int
    router: str = "softmax"        # "softmax" (top-k then softmax), "sigmoid" (noaux_tc) or "sqrt_softplus" (noaux_tc on sqrt(softplus))
    norm_topk_prob: bool = True
    routed_scaling_factor: float = 2.5
    seed_stride: int = keys.SEED_GROUP_STRIDE
    key_generator: str = "torch_cpu_v1"
    first_slot: int = 0                    # expert-parallel shard: global index of local slot 0 (keys are seeded by it)
    n_router_experts: int | None = None    # rows of the (replicated) router table when it is wider than the local experts

    @property
    def router_experts(self) -> int:
        return self.n_router_experts or self.n_experts

    @property
    def n_slots(self) -> int:
        return self.n_experts // self.group_size

    def validate(self) -> None:
        if self.hidden % 128 or self.inter % 128:
            raise ValueError("hidden and inter must be multiples of 128 (chronos_1t/models/glm53_chronos_spec.py:149-151)")
        if self.n_experts % self.group_size:
            raise ValueError("n_experts must be a multiple of group_size")
        if self.router not in ROUTER_KINDS:
            raise ValueError(f"unknown router flavour {self.router!r}")
        if self.key_generator != "torch_cpu_v1":
            raise ValueError("only key_generator = 'torch_cpu_v1' checkpoints can be read")

    def bank_bytes_per_slot(self) -> int:
        h, i = self.hidden, self.inter
        return 2 * i * h // 2 + 2 * i * h // 16 + h * i // 2 + h * i // 16

    def healer_bytes_per_expert(self) -> int:
        return self.rank * (2 * self.inter + self.hidden + self.hidden + self.inter)


def _norm_device(device: torch.device | str) -> torch.device:
    """'cuda' -> 'cuda:<current index>' so that device comparisons with tensors are exact."""
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return device


def _u8(t: Any) -> torch.Tensor:
    """Tensor or array -> CPU uint8 torch tensor holding the same bytes (fp8 is reinterpreted, not converted)."""
    if isinstance(t, np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(t))
    if t.dtype == torch.float8_e4m3fn:
        t = t.view(torch.uint8)
    if t.dtype != torch.uint8:
        raise TypeError(f"expected uint8 / float8_e4m3fn bytes, got {t.dtype}")
    return t.contiguous()


def _f32(t: Any) -> torch.Tensor:
    if isinstance(t, (np.ndarray, np.generic, float)):
        t = torch.from_numpy(np.ascontiguousarray(np.asarray(t, dtype=np.float32)))
    return t.detach().to(torch.float32).contiguous()


_KEY_TABLE_CACHE: dict[tuple, dict[str, torch.Tensor]] = {}


def key_tables(cfg: FoldedLayerConfig, device: torch.device) -> dict[str, torch.Tensor]:
    """Compact key tables of all experts of a layer shape. Keys depend on (slot, member, dims) only - not on the
    layer index - so one set per shape and device is shared by every layer (the reference caches them the same way,
    chronos_1t/models/glm53_holo.py:53,68-71)."""
    ck = (cfg.hidden, cfg.inter, cfg.n_experts, cfg.group_size, cfg.seed_stride, cfg.first_slot, str(device))
    hit = _KEY_TABLE_CACHE.get(ck)
    if hit is not None:
        return hit
    h, i, e, k = cfg.hidden, cfg.inter, cfg.n_experts, cfg.group_size
    acc: dict[str, list[np.ndarray]] = {n: [] for n in ("gu_cin", "gu_cs2", "gu_rout", "gu_rs2", "dn_cin", "dn_cs2", "dn_rout", "dn_rs2")}
    for eid in range(e):
        g, m = divmod(eid, k)
        sg, sd = keys.group_seed_bases(cfg.first_slot + g, cfg.seed_stride)
        for pre, rows, cols, sb in (("gu", 2 * i, h, sg), ("dn", h, i, sd)):
            t = keys.compact_tables(rows, cols, m, sb)
            for n in ("cin", "cs2", "rout", "rs2"):
                acc[f"{pre}_{n}"].append(t[n])
    out: dict[str, torch.Tensor] = {}
    for n, parts in acc.items():
        arr = np.stack(parts)
        view = arr.view(np.int16) if arr.dtype == np.uint16 else arr.view(np.int32)
        out[n] = torch.from_numpy(view.copy()).to(device)
    _KEY_TABLE_CACHE[ck] = out
    return out


def healer_tiles(u: torch.Tensor, beta: torch.Tensor, rout: torch.Tensor, rs2: torch.Tensor, s2: torch.Tensor,
                 group_size: int) -> tuple[torch.Tensor, float]:
    """The healer's output factor of every expert in the row order and basis of the bank-pass accumulators.

    u e4m3 bytes [E, rows, r], beta f32 [E], rout i16 [E, rows] (bits 0-14 r_inv, bit 15 r_s1 < 0), rs2 i32 [E, rows/32] sign
    bits, s2 f32 [n_slots]. Returns (tiles f16 [E, rows/128, r/8, 128, 8], scale): row j of block b of expert e holds
    r_s2[j] * WHT128(W)[j] / (scale_2 * scale) with W[r_inv[i]] = (r_s1[i] / beta) * U[i], laid out as K-major operand tiles
    (8 consecutive rank columns per 16-byte unit); `scale` is the power of two that puts the largest entry into (2048, 4096]."""
    dev = u.device
    n_e, rows, r = u.shape
    had = torch.ones(1, 1, device=dev)
    for _ in range(7):  # Sylvester construction, the matrix of build_hadamard_128 (convert_glm53_flash_colab.py:41-45)
        had = torch.cat([torch.cat([had, had], 1), torch.cat([had, -had], 1)], 0)
    had = had / math.sqrt(128.0)
    raw = torch.empty(n_e, rows // 128, r // 8, 128, 8, dtype=torch.float32, device=dev)
    shifts = torch.arange(32, device=dev, dtype=torch.int64)
    for e0 in range(0, n_e, 16):  # a few experts at a time: the fp32 transient stays small
        e1 = min(n_e, e0 + 16)
        n = e1 - e0
        uf = u[e0:e1].view(torch.float8_e4m3fn).to(torch.float32)
        ro = rout[e0:e1].to(torch.int32) & 0xffff
        r_inv = (ro & 0x7fff).to(torch.int64)
        s1 = 1.0 - 2.0 * ((ro >> 15) & 1).to(torch.float32)
        slot_s2 = s2[torch.arange(e0, e1, device=dev) // group_size]
        src = uf * (s1 / (beta[e0:e1, None] * slot_s2[:, None]))[..., None]
        w = torch.empty_like(src)
        w.scatter_(1, r_inv[..., None].expand(-1, -1, r), src)           # w[r_inv[i]] = src[i]
        w = torch.matmul(had, w.view(n, rows // 128, 128, r))            # 128-row blocks, orthonormal
        bits = ((rs2[e0:e1].to(torch.int64) & 0xffffffff)[..., None] >> shifts) & 1
        w = w * (1.0 - 2.0 * bits.to(torch.float32)).view(n, rows // 128, 128, 1)
        raw[e0:e1] = w.view(n, rows // 128, 128, r // 8, 8).permute(0, 1, 3, 2, 4)
    top = float(raw.abs().max())
    scale = 2.0 ** math.ceil(math.log2(top / 4096.0)) if top > 0.0 else 1.0
    return (raw / scale).to(torch.float16), scale


class PackedLayer:
    """Owns the device tensors of one layer and exposes them as a `chronos_layer_t`."""

    # Build the healer operand tiles of the FP4 tensor regime (`ut_gu` / `ut_dn`, + 2 * rank bytes per bank row) at load.
    # Instances read the class attribute at construction; set it to False for layers that only ever see decode-sized batches.
    fused_healer_default = True

    def __init__(self, cfg: FoldedLayerConfig, tensors: dict[str, torch.Tensor], device: torch.device,
                 fp4_images: bool = True, tail_bits: tuple[int, int] = (0, 0), keep_disk_order: bool = False):
        """`keep_disk_order`: keep the banks in their on-disk row-major order beside the re-tiled stage images. The FP4
        regimes read only the images, so by default the on-disk-order copy is released once the images exist (a layer is
        then resident once, not twice); the reconstruction probes and the forced "stream" / "tensor" regimes need it."""
        cfg.validate()
        self.cfg = cfg
        self.keep_disk_order = keep_disk_order
        self.tail_bits = tuple(tail_bits) if "tail_gu_p" in tensors else (0, 0)
        self.fp4_images = fp4_images
        self.device = _norm_device(device)
        self.t = tensors
        self.struct = _lib.LayerStruct()
        s = self.struct
        s.hidden, s.inter, s.n_experts, s.group_size, s.n_slots = cfg.hidden, cfg.inter, cfg.n_experts, cfg.group_size, cfg.n_slots
        s.rank, s.top_k = cfg.rank, cfg.top_k
        s.router_kind = ROUTER_KINDS[cfg.router]
        s.renorm = int(cfg.norm_topk_prob)
        s.routed_scaling = float(cfg.routed_scaling_factor)
        s.shared_inter = cfg.inter if ("sh_gu_w" in tensors or "sh_gu_t" in tensors or "sh8_gu_w" in tensors) else 0
        s.tail_bits = self.tail_bits[0] | (self.tail_bits[1] << 8)
        self._add_fp4_images()
        if self.fused_healer_default:
            self._add_healer_tiles()
        if "v_dn" not in tensors and "v_dn_t" in tensors and self.device.type == "cuda":
            # healer.v_down in its on-disk orientation [E, r, I] beside the transposed copy: the tensor-core healer
            # kernels of the large-batch regime contract over I
            tensors["v_dn"] = tensors["v_dn_t"].transpose(1, 2).contiguous()
        for name, _ in _lib.LayerStruct._fields_:
            if name in tensors:
                setattr(s, name, tensors[name].data_ptr())
        # the router may be wider than the local expert table (expert-parallel shards replicate the full router)
        self.router_struct = _lib.LayerStruct()
        rs = self.router_struct
        rs.hidden, rs.n_experts, rs.top_k = cfg.hidden, cfg.router_experts, cfg.top_k
        rs.router_kind, rs.renorm, rs.routed_scaling = s.router_kind, s.renorm, s.routed_scaling
        for name in ("router_w", "e_bias"):
            if name in tensors:
                setattr(rs, name, tensors[name].data_ptr())
        self._check_shapes()

    def _add_fp4_images(self) -> None:
        """Re-tiled bank copies for the block-scaled FP4 tensor-core pass (a byte permutation done once at load;
        needs hidden and inter to be multiples of 256; doubles the resident bank bytes)."""
        from .fp4_layout import tile_matrix_fp4

        c, t = self.cfg, self.t
        if c.hidden % 256 or c.inter % 256 or self.device.type != "cuda" or not self.fp4_images or "gu_t" in t:
            return
        # slot by slot, so that the transient of the byte permutation stays one slot large
        t["gu_t"] = torch.stack([tile_matrix_fp4(t["gu_w"][g], t["gu_s"][g], 128) for g in range(c.n_slots)])
        t["dn_t"] = torch.stack([tile_matrix_fp4(t["dn_w"][g], t["dn_s"][g], 128) for g in range(c.n_slots)])
        if "sh_gu_w" in t:
            t["sh_gu_t"] = tile_matrix_fp4(t["sh_gu_w"], t["sh_gu_s"], 128)
            t["sh_dn_t"] = tile_matrix_fp4(t["sh_dn_w"], t["sh_dn_s"], 128)
        if not self.keep_disk_order and self.fp4_only_ok():
            for name in ("gu_w", "gu_s", "dn_w", "dn_s", "sh_gu_w", "sh_gu_s", "sh_dn_w", "sh_dn_s"):
                t.pop(name, None)

    def _add_healer_tiles(self) -> None:
        """healer.u_gu / healer.u_down as fp16 operand tiles in the basis of the bank-pass accumulators (see `ut_gu` in
        include/chronos_b200.h). With z1 the bank-pass output after its epilogue (r_s2 sign, 128-row Walsh-Hadamard), the
        reference's z[i] = beta * r_s1[i] * z1[r_inv[i]] + (U h)[i] (chronos_1t/models/glm5_chronos_moe.py:149-195) equals
        beta * r_s1[i] * z1'[r_inv[i]] with z1' = z1 + W h, W[r_inv[i]] = (r_s1[i] / beta) U[i]; moving W h in front of
        the epilogue's orthonormal transform gives the tile rows r_s2 * WHT128(W)."""
        c, t = self.cfg, self.t
        if (self.device.type != "cuda" or "gu_t" not in t or "u_gu" not in t or "ut_gu" in t or c.rank % 16 or c.rank > 64
                or "gu_rout" not in t):
            return
        if any(bool((t[n].abs() < 1e-30).any()) for n in ("gu_beta", "dn_beta", "gu_s2", "dn_s2")):
            return  # a zero beta or scale_2 cannot be divided out: such a layer keeps the separate healer pass
        t["ut_gu"], k_gu = healer_tiles(t["u_gu"], t["gu_beta"], t["gu_rout"], t["gu_rs2"], t["gu_s2"], c.group_size)
        t["ut_dn"], k_dn = healer_tiles(t["u_dn"], t["dn_beta"], t["dn_rout"], t["dn_rs2"], t["dn_s2"], c.group_size)
        t["ut_scale"] = torch.tensor([k_gu, k_dn], dtype=torch.float32, device=self.device)

    def fp4_only_ok(self) -> bool:
        """True when every batch shape of this layer is served by an FP4 regime (the limits csrc/common.cuh states for
        them), so that nothing on the forward path ever reads the on-disk-order banks."""
        c = self.cfg
        return (c.hidden % 256 == 0 and c.inter % 256 == 0 and c.hidden <= 7168 and c.inter <= 7168
                and 8 * 3 * c.inter * 4 <= 220 * 1024 and 8 * c.hidden * 4 <= 220 * 1024 and self.tail_bits == (0, 0))

    @property
    def router_ptr(self):
        return C.byref(self.router_struct)

    # -- shape checks: wrong or short tensors are rejected here, before any launch ---------------------------------
    def _check_shapes(self) -> None:
        c, t = self.cfg, self.t
        h, i, e, ns, r = c.hidden, c.inter, c.n_experts, c.n_slots, c.rank
        want = {
            "gu_s2": (ns,), "gu_beta": (e,), "dn_s2": (ns,), "dn_beta": (e,),
            "u_gu": (e, 2 * i, r), "v_gu": (e, r, h), "u_dn": (e, h, r), "v_dn_t": (e, i, r),
            "gu_cin": (e, h), "gu_cs2": (e, h // 32), "gu_rout": (e, 2 * i), "gu_rs2": (e, 2 * i // 32),
            "dn_cin": (e, i), "dn_cs2": (e, i // 32), "dn_rout": (e, h), "dn_rs2": (e, h // 32),
        }
        if "gu_t" in t and "gu_w" not in t:  # resident as stage images only
            want.update({"gu_t": (ns, 2 * i // 128, h // 256, 18432), "dn_t": (ns, h // 128, i // 256, 18432)})
        else:
            want.update({"gu_w": (ns, 2 * i, h // 2), "gu_s": (ns, 2 * i, h // 16), "dn_w": (ns, h, i // 2), "dn_s": (ns, h, i // 16)})
        if "router_w" in t:
            want["router_w"] = (c.router_experts, h)
        if "e_bias" in t:
            want["e_bias"] = (c.router_experts,)
        if "sh_gu_w" in t:
            want.update({"sh_gu_w": (2 * i, h // 2), "sh_gu_s": (2 * i, h // 16), "sh_gu_s2": (2,),
                         "sh_dn_w": (h, i // 2), "sh_dn_s": (h, i // 16), "sh_dn_s2": (1,)})
        if "sh8_gu_w" in t:
            want.update({"sh8_gu_w": (2 * i, h), "sh8_gu_s": (2 * i // 128, h // 128), "sh8_dn_w": (h, i), "sh8_dn_s": (h // 128, i // 128)})
        elif "sh_gu_t" in t and "sh_gu_w" not in t:
            want.update({"sh_gu_t": (2 * i // 128, h // 256, 18432), "sh_dn_t": (h // 128, i // 256, 18432), "sh_gu_s2": (2,), "sh_dn_s2": (1,)})
        for name, shape in want.items():
            if name not in t:
                raise ValueError(f"packed layer is missing tensor {name!r}")
            if tuple(t[name].shape) != shape:
                raise ValueError(f"packed tensor {name!r} has shape {tuple(t[name].shape)}, expected {shape}")
            if not t[name].is_contiguous() or t[name].device != self.device:
                raise ValueError(f"packed tensor {name!r} must be contiguous on {self.device}")
        for name in ("gu_s2", "dn_s2", "gu_beta", "dn_beta"):
            if not bool(torch.isfinite(t[name]).all()):
                raise ValueError(f"packed tensor {name!r} holds a non-finite value")

    @property
    def ptr(self):
        return C.byref(self.struct)

    def resident_bytes(self) -> int:
        return sum(v.numel() * v.element_size() for v in self.t.values())

    # -- constructors ---------------------------------------------------------------------------------------------
    @classmethod
    def from_groups(cls, cfg: FoldedLayerConfig, groups: Iterable[Mapping[str, Any]], router_w: Any = None,
                    e_bias: Any = None, shared: Mapping[str, Any] | None = None,
                    device: torch.device | str = "cuda", include_tail: bool = False, keep_disk_order: bool = False) -> "PackedLayer":
        """`groups[g]` maps the on-disk suffixes to tensors/arrays (fp8 either as float8_e4m3fn or raw uint8).
        `shared` (optional) holds a plain-NVFP4 expert: `{gate,up,down}_proj.{weight,weight_scale,weight_scale_2}`.
        `include_tail` also loads the tail lattice tensors and makes every call on the layer add the tail term."""
        device = _norm_device(device)
        groups = list(groups)
        if len(groups) != cfg.n_slots:
            raise ValueError(f"{len(groups)} slot dicts for {cfg.n_slots} slots")
        for g, d in enumerate(groups):
            for sfx in _REQUIRED:
                if sfx not in d:
                    raise ValueError(f"slot {g} is missing tensor {sfx!r}")
            kk = int(np.asarray(_f32(d["s_gu.beta"])).shape[0])
            if kk != cfg.group_size:
                raise ValueError(f"slot {g} folds {kk} experts, config says {cfg.group_size}")

        def stack_u8(sfx: str) -> torch.Tensor:
            return torch.stack([_u8(d[sfx]) for d in groups])

        t: dict[str, torch.Tensor] = {
            "gu_w": stack_u8("s_gu.weight"), "gu_s": stack_u8("s_gu.weight_scale"),
            "dn_w": stack_u8("s_down.weight"), "dn_s": stack_u8("s_down.weight_scale"),
            "gu_s2": torch.stack([_f32(d["s_gu.weight_scale_2"]).reshape(()) for d in groups]),
            "dn_s2": torch.stack([_f32(d["s_down.weight_scale_2"]).reshape(()) for d in groups]),
            "gu_beta": torch.cat([_f32(d["s_gu.beta"]) for d in groups]),
            "dn_beta": torch.cat([_f32(d["s_down.beta"]) for d in groups]),
            "u_gu": torch.cat([_u8(d["healer.u_gu"]) for d in groups]),
            "v_gu": torch.cat([_u8(d["healer.v_gu"]) for d in groups]),
            "u_dn": torch.cat([_u8(d["healer.u_down"]) for d in groups]),
            "v_dn_t": torch.cat([_u8(d["healer.v_down"]) for d in groups]).transpose(1, 2).contiguous(),
        }
        if include_tail:
            # the tail lattice (chronos_1t/models/glm53_holo.py:362-366): per expert a 2-bit Lloyd-Max (block 32) or 1-bit
            # Rademacher (block 64) matrix with e4m3 block scales, added to the reconstruction in natural weight space
            for d in groups:
                for sfx in GROUP_TENSOR_SUFFIXES[12:]:
                    if sfx not in d:
                        raise ValueError(f"include_tail: a slot is missing tensor {sfx!r}")
            bits = {(int(np.asarray(d["tail.gu_bits"]).reshape(-1)[0]), int(np.asarray(d["tail.down_bits"]).reshape(-1)[0])) for d in groups}
            if len(bits) != 1 or not bits <= {(1, 1), (1, 2), (2, 1), (2, 2)}:
                raise ValueError(f"include_tail: slots disagree on the tail bit widths or use unsupported ones: {sorted(bits)}")
            t["tail_gu_p"] = torch.cat([_u8(d["tail.gu_packed"]) for d in groups])
            t["tail_gu_s"] = torch.cat([_u8(d["tail.gu_scale"]) for d in groups])
            t["tail_dn_p"] = torch.cat([_u8(d["tail.down_packed"]) for d in groups])
            t["tail_dn_s"] = torch.cat([_u8(d["tail.down_scale"]) for d in groups])
            tail_bits = next(iter(bits))
        if router_w is not None:
            t["router_w"] = _f32(router_w)
        if e_bias is not None:
            t["e_bias"] = _f32(e_bias)
        if shared is not None and "gate_proj.weight_scale_inv" in shared:
            # the stock block-FP8 format of the reference's shared expert (chronos_1t/models/glm53_chronos_moe.py:170-181):
            # e4m3 weights + one fp32 weight_scale_inv per 128 x 128 block; gate and up fused along the rows
            t["sh8_gu_w"] = torch.cat([_u8(shared["gate_proj.weight"]), _u8(shared["up_proj.weight"])])
            t["sh8_gu_s"] = torch.cat([_f32(shared["gate_proj.weight_scale_inv"]), _f32(shared["up_proj.weight_scale_inv"])])
            t["sh8_dn_w"], t["sh8_dn_s"] = _u8(shared["down_proj.weight"]), _f32(shared["down_proj.weight_scale_inv"])
        elif shared is not None:
            t["sh_gu_w"] = torch.cat([_u8(shared["gate_proj.weight"]), _u8(shared["up_proj.weight"])])
            t["sh_gu_s"] = torch.cat([_u8(shared["gate_proj.weight_scale"]), _u8(shared["up_proj.weight_scale"])])
            t["sh_gu_s2"] = torch.stack([_f32(shared["gate_proj.weight_scale_2"]).reshape(()), _f32(shared["up_proj.weight_scale_2"]).reshape(())])
            t["sh_dn_w"], t["sh_dn_s"] = _u8(shared["down_proj.weight"]), _u8(shared["down_proj.weight_scale"])
            t["sh_dn_s2"] = _f32(shared["down_proj.weight_scale_2"]).reshape(1)
        t = {n: v.to(device).contiguous() for n, v in t.items()}
        t.update(key_tables(cfg, device))
        return cls(cfg, t, device, tail_bits=tail_bits if include_tail else (0, 0), keep_disk_order=keep_disk_order)

    @classmethod
    def from_safetensors(cls, path: str | Path, cfg: FoldedLayerConfig, prefix: str, device: torch.device | str = "cuda",
                         shared_prefix: str | None = None, include_tail: bool = False, keep_disk_order: bool = False,
                         evict_page_cache: bool = True) -> "PackedLayer":
        """Reads `{prefix}.chronos_groups.{g}.{suffix}` (chronos_1t/models/glm53_chronos_spec.py:186-191) and
        `{prefix}.gate.weight` (+ `.gate.e_score_correction_bias`) from a converter shard.

        On a CUDA device the shard is streamed tensor by tensor from the memory-mapped file straight into the stacked
        device tensors (no CPU copy of the layer is ever assembled), the FP4 stage images are built on the device slot by
        slot, and the shard's pages are dropped from the page cache afterwards, as the reference's loader does
        (chronos_1t/models/glm53_chronos_moe.py:56-63) - a model of dozens of such shards would otherwise fill the host's
        page cache with bytes that are never read again."""
        from safetensors import safe_open

        device = _norm_device(device)
        if device.type == "cuda":
            layer = cls._from_safetensors_direct(path, cfg, prefix, device, shared_prefix, include_tail, keep_disk_order)
            if evict_page_cache:
                evict_from_page_cache(path)
            return layer
        with safe_open(str(path), framework="pt", device="cpu") as fh:
            names = set(fh.keys())
            groups = []
            for g in range(cfg.n_slots):
                gp = f"{prefix}.chronos_groups.{g}."
                missing = [s for s in _REQUIRED if gp + s not in names]
                if missing:
                    raise ValueError(f"{path}: slot {g} is missing {missing}")
                want = GROUP_TENSOR_SUFFIXES if include_tail else _REQUIRED
                groups.append({s: fh.get_tensor(gp + s) for s in want if gp + s in names})
            router_w = fh.get_tensor(f"{prefix}.gate.weight") if f"{prefix}.gate.weight" in names else None
            bias_key = f"{prefix}.gate.e_score_correction_bias"
            e_bias = fh.get_tensor(bias_key) if bias_key in names else None
            shared = None
            if shared_prefix is not None and f"{shared_prefix}.gate_proj.weight" in names:
                shared = _read_shared(fh, names, shared_prefix)
        return cls.from_groups(cfg, groups, router_w, e_bias, shared, device, include_tail=include_tail, keep_disk_order=keep_disk_order)

    @classmethod
    def _from_safetensors_direct(cls, path, cfg: FoldedLayerConfig, prefix: str, device: torch.device, shared_prefix, include_tail: bool,
                                 keep_disk_order: bool) -> "PackedLayer":
        from safetensors import safe_open

        h, i, ns, k, r, e = cfg.hidden, cfg.inter, cfg.n_slots, cfg.group_size, cfg.rank, cfg.n_experts
        u8 = dict(dtype=torch.uint8, device=device)
        t: dict[str, torch.Tensor] = {
            "gu_w": torch.empty((ns, 2 * i, h // 2), **u8), "gu_s": torch.empty((ns, 2 * i, h // 16), **u8),
            "dn_w": torch.empty((ns, h, i // 2), **u8), "dn_s": torch.empty((ns, h, i // 16), **u8),
            "gu_s2": torch.empty(ns, dtype=torch.float32, device=device), "dn_s2": torch.empty(ns, dtype=torch.float32, device=device),
            "gu_beta": torch.empty(e, dtype=torch.float32, device=device), "dn_beta": torch.empty(e, dtype=torch.float32, device=device),
            "u_gu": torch.empty((e, 2 * i, r), **u8), "v_gu": torch.empty((e, r, h), **u8),
            "u_dn": torch.empty((e, h, r), **u8), "v_dn": torch.empty((e, r, i), **u8),
        }
        dest = {"s_gu.weight": "gu_w", "s_gu.weight_scale": "gu_s", "s_down.weight": "dn_w", "s_down.weight_scale": "dn_s",
                "healer.u_gu": "u_gu", "healer.v_gu": "v_gu", "healer.u_down": "u_dn", "healer.v_down": "v_dn"}
        tail_bits = (0, 0)
        with safe_open(str(path), framework="pt", device="cpu") as fh:  # memory-mapped: a tensor's pages are touched when it is copied
            names = set(fh.keys())
            for g in range(ns):
                gp = f"{prefix}.chronos_groups.{g}."
                missing = [s for s in _REQUIRED if gp + s not in names]
                if missing:
                    raise ValueError(f"{path}: slot {g} is missing {missing}")
                beta = fh.get_tensor(gp + "s_gu.beta")
                if int(beta.shape[0]) != k:
                    raise ValueError(f"slot {g} folds {int(beta.shape[0])} experts, config says {k}")
                for sfx, name in dest.items():
                    src = _u8(fh.get_tensor(gp + sfx))
                    dst = t[name][g] if name in ("gu_w", "gu_s", "dn_w", "dn_s") else t[name][g * k:(g + 1) * k]
                    if tuple(src.shape) != tuple(dst.shape):
                        raise ValueError(f"{path}: {gp + sfx} has shape {tuple(src.shape)}, expected {tuple(dst.shape)}")
                    dst.copy_(src, non_blocking=True)
                t["gu_s2"][g].copy_(_f32(fh.get_tensor(gp + "s_gu.weight_scale_2")).reshape(()))
                t["dn_s2"][g].copy_(_f32(fh.get_tensor(gp + "s_down.weight_scale_2")).reshape(()))
                t["gu_beta"][g * k:(g + 1) * k].copy_(_f32(beta))
                t["dn_beta"][g * k:(g + 1) * k].copy_(_f32(fh.get_tensor(gp + "s_down.beta")))
            if include_tail:
                groups = [{s: fh.get_tensor(f"{prefix}.chronos_groups.{g}.{s}") for s in GROUP_TENSOR_SUFFIXES[12:]} for g in range(ns)]
                bits = {(int(d["tail.gu_bits"].reshape(-1)[0]), int(d["tail.down_bits"].reshape(-1)[0])) for d in groups}
                if len(bits) != 1 or not bits <= {(1, 1), (1, 2), (2, 1), (2, 2)}:
                    raise ValueError(f"include_tail: slots disagree on the tail bit widths or use unsupported ones: {sorted(bits)}")
                tail_bits = next(iter(bits))
                for name, sfx in (("tail_gu_p", "tail.gu_packed"), ("tail_gu_s", "tail.gu_scale"), ("tail_dn_p", "tail.down_packed"), ("tail_dn_s", "tail.down_scale")):
                    t[name] = torch.cat([_u8(d[sfx]).to(device) for d in groups])
            if f"{prefix}.gate.weight" in names:
                t["router_w"] = _f32(fh.get_tensor(f"{prefix}.gate.weight")).to(device)
            if f"{prefix}.gate.e_score_correction_bias" in names:
                t["e_bias"] = _f32(fh.get_tensor(f"{prefix}.gate.e_score_correction_bias")).to(device)
            sh = _read_shared(fh, names, shared_prefix) if (shared_prefix is not None and f"{shared_prefix}.gate_proj.weight" in names) else None
            if sh is not None and "gate_proj.weight_scale_inv" in sh:
                t["sh8_gu_w"] = torch.cat([_u8(sh["gate_proj.weight"]), _u8(sh["up_proj.weight"])]).to(device)
                t["sh8_gu_s"] = torch.cat([_f32(sh["gate_proj.weight_scale_inv"]), _f32(sh["up_proj.weight_scale_inv"])]).to(device)
                t["sh8_dn_w"], t["sh8_dn_s"] = _u8(sh["down_proj.weight"]).to(device), _f32(sh["down_proj.weight_scale_inv"]).to(device)
            elif sh is not None:
                t["sh_gu_w"] = torch.cat([_u8(sh["gate_proj.weight"]), _u8(sh["up_proj.weight"])]).to(device)
                t["sh_gu_s"] = torch.cat([_u8(sh["gate_proj.weight_scale"]), _u8(sh["up_proj.weight_scale"])]).to(device)
                t["sh_gu_s2"] = torch.stack([_f32(sh["gate_proj.weight_scale_2"]).reshape(()), _f32(sh["up_proj.weight_scale_2"]).reshape(())]).to(device)
                t["sh_dn_w"], t["sh_dn_s"] = _u8(sh["down_proj.weight"]).to(device), _u8(sh["down_proj.weight_scale"]).to(device)
                t["sh_dn_s2"] = _f32(sh["down_proj.weight_scale_2"]).reshape(1).to(device)
            torch.cuda.synchronize(device)  # the copies read the mapping: finish them before it is closed
        t["v_dn_t"] = t["v_dn"].transpose(1, 2).contiguous()
        t.update(key_tables(cfg, device))
        return cls(cfg, t, device, tail_bits=tail_bits, keep_disk_order=keep_disk_order)

    @classmethod
    def synthetic(cls, cfg: FoldedLayerConfig, seed: int, device: torch.device | str = "cuda",
                  with_shared: bool = False, tail_bits: tuple[int, int] = (0, 0), keep_disk_order: bool = False,
                  shared_format: str = "nvfp4") -> "PackedLayer":
        """Seeded random layer in the converter's byte format, generated on the device (for benchmarks: the real
        converter takes seconds per slot). Value ranges follow what the converter emits for N(0, 0.02) weights:
        uniform nibbles, e4m3 block-scale codes 0x58..0x77, scale_2 = amax / 2688, beta ~ 0.5, healer ~ N(0, 0.05)."""
        device = _norm_device(device)
        gen = torch.Generator(device=device).manual_seed(seed)
        t = cls._random_slot_tensors(cfg, gen, device)
        t["router_w"] = torch.randn(cfg.router_experts, cfg.hidden, generator=gen, device=device) * 0.02
        if cfg.router != "softmax":
            t["e_bias"] = torch.zeros(cfg.router_experts, device=device)
        if with_shared and shared_format == "fp8":
            t.update(cls._random_shared_fp8_tensors(cfg, gen, device))
        elif with_shared:
            t.update(cls._random_shared_tensors(cfg, gen, device))
        if tail_bits != (0, 0):  # random codes; block scales 0.004 .. 0.02, below the typical bank value
            h, i, e = cfg.hidden, cfg.inter, cfg.n_experts
            gb, db = tail_bits
            t["tail_gu_p"] = torch.randint(0, 256, (e, 2 * i, h * gb // 8), generator=gen, device=device, dtype=torch.uint8)
            t["tail_gu_s"] = torch.randint(0x02, 0x0C, (e, 2 * i, h // (32 if gb == 2 else 64)), generator=gen, device=device, dtype=torch.uint8)
            t["tail_dn_p"] = torch.randint(0, 256, (e, h, i * db // 8), generator=gen, device=device, dtype=torch.uint8)
            t["tail_dn_s"] = torch.randint(0x02, 0x0C, (e, h, i // (32 if db == 2 else 64)), generator=gen, device=device, dtype=torch.uint8)
        t.update(key_tables(cfg, device))
        return cls(cfg, t, device, tail_bits=tail_bits, keep_disk_order=keep_disk_order)

    @classmethod
    def synthetic_sharded(cls, cfg_global: FoldedLayerConfig, seed: int, slots: range, device: torch.device | str = "cuda",
                          with_shared: bool = False) -> "PackedLayer":
        """The slots `slots` of the seeded random layer `seed`, plus the replicated router (and shared expert).
        Every slot is drawn from its own generator seeded by (seed, slot), so a slot holds the same bytes whatever
        the number of ranks it is sharded over."""
        import dataclasses

        device = _norm_device(device)
        k = cfg_global.group_size
        cfg = dataclasses.replace(cfg_global, n_experts=len(slots) * k, first_slot=slots.start,
                                  n_router_experts=cfg_global.n_experts)
        one = dataclasses.replace(cfg_global, n_experts=k, first_slot=0, n_router_experts=None)
        parts: dict[str, list[torch.Tensor]] = {}
        for sl in slots:
            gen = torch.Generator(device=device).manual_seed(seed * 100003 + sl)
            for n, v in cls._random_slot_tensors(one, gen, device).items():
                parts.setdefault(n, []).append(v)
        t = {n: torch.cat(v) for n, v in parts.items()}
        gen = torch.Generator(device=device).manual_seed(seed * 100003 + 99991)
        t["router_w"] = torch.randn(cfg_global.n_experts, cfg.hidden, generator=gen, device=device) * 0.02
        if cfg.router != "softmax":
            t["e_bias"] = torch.zeros(cfg_global.n_experts, device=device)
        if with_shared:
            t.update(cls._random_shared_tensors(cfg, gen, device))
        t.update(key_tables(cfg, device))
        return cls(cfg, t, device)

    @staticmethod
    def _random_slot_tensors(cfg: FoldedLayerConfig, gen: torch.Generator, device: torch.device) -> dict[str, torch.Tensor]:
        h, i, e, ns, r = cfg.hidden, cfg.inter, cfg.n_experts, cfg.n_slots, cfg.rank

        def rnd_u8(shape, lo=0, hi=256):
            return torch.randint(lo, hi, shape, generator=gen, device=device, dtype=torch.uint8)

        def rnd_fp8(shape, std):
            return (torch.randn(shape, generator=gen, device=device) * std).to(torch.float8_e4m3fn).view(torch.uint8)

        return {
            "gu_w": rnd_u8((ns, 2 * i, h // 2)), "gu_s": rnd_u8((ns, 2 * i, h // 16), 0x58, 0x78),
            "dn_w": rnd_u8((ns, h, i // 2)), "dn_s": rnd_u8((ns, h, i // 16), 0x58, 0x78),
            "gu_s2": torch.full((ns,), 0.08 / 2688.0, device=device), "dn_s2": torch.full((ns,), 0.08 / 2688.0, device=device),
            "gu_beta": torch.rand(e, generator=gen, device=device) * 0.4 + 0.3,
            "dn_beta": torch.rand(e, generator=gen, device=device) * 0.4 + 0.3,
            "u_gu": rnd_fp8((e, 2 * i, r), 0.05), "v_gu": rnd_fp8((e, r, h), 0.05),
            "u_dn": rnd_fp8((e, h, r), 0.05), "v_dn_t": rnd_fp8((e, i, r), 0.05),
        }

    @staticmethod
    def _random_shared_tensors(cfg: FoldedLayerConfig, gen: torch.Generator, device: torch.device) -> dict[str, torch.Tensor]:
        h, i = cfg.hidden, cfg.inter

        def rnd_u8(shape, lo=0, hi=256):
            return torch.randint(lo, hi, shape, generator=gen, device=device, dtype=torch.uint8)

        return {
            "sh_gu_w": rnd_u8((2 * i, h // 2)), "sh_gu_s": rnd_u8((2 * i, h // 16), 0x58, 0x78),
            "sh_gu_s2": torch.full((2,), 0.08 / 2688.0, device=device),
            "sh_dn_w": rnd_u8((h, i // 2)), "sh_dn_s": rnd_u8((h, i // 16), 0x58, 0x78),
            "sh_dn_s2": torch.full((1,), 0.08 / 2688.0, device=device),
        }

    @staticmethod
    def _random_shared_fp8_tensors(cfg: FoldedLayerConfig, gen: torch.Generator, device: torch.device) -> dict[str, torch.Tensor]:
        """An N(0, 0.02) SwiGLU expert quantised to the stock 128 x 128 block-FP8 format (scale_inv = block max / 448)."""
        h, i = cfg.hidden, cfg.inter
        out = {}
        for name, rows, cols in (("sh8_gu", 2 * i, h), ("sh8_dn", h, i)):
            w = torch.randn((rows, cols), generator=gen, device=device) * 0.02
            blocks = w.view(rows // 128, 128, cols // 128, 128)
            s = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12) / 448.0
            q = (blocks / s[:, None, :, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
            out[f"{name}_w"] = q.view(torch.uint8).reshape(rows, cols).contiguous()
            out[f"{name}_s"] = s.float().contiguous()
        return out

    def to_groups_numpy(self) -> tuple[list[dict[str, np.ndarray]], dict[str, np.ndarray]]:
        """Back to per-slot dicts of on-disk suffixes (numpy, fp8 as uint8) + extras: what a checker needs."""
        c = self.cfg
        tt = dict(self.t)
        if "gu_w" not in tt and "gu_t" in tt:  # resident as stage images only: undo the byte permutation
            from .fp4_layout import untile_matrix_fp4

            tt["gu_w"], tt["gu_s"] = untile_matrix_fp4(tt["gu_t"])
            tt["dn_w"], tt["dn_s"] = untile_matrix_fp4(tt["dn_t"])
            if "sh_gu_t" in tt:
                tt["sh_gu_w"], tt["sh_gu_s"] = untile_matrix_fp4(tt["sh_gu_t"])
                tt["sh_dn_w"], tt["sh_dn_s"] = untile_matrix_fp4(tt["sh_dn_t"])
        t = {n: v.cpu().numpy() for n, v in tt.items() if not n.endswith("_t") or n == "v_dn_t"}
        k = c.group_size
        groups = []
        for g in range(c.n_slots):
            sl = slice(g * k, (g + 1) * k)
            groups.append({
                "s_gu.weight": t["gu_w"][g], "s_gu.weight_scale": t["gu_s"][g], "s_gu.weight_scale_2": t["gu_s2"][g],
                "s_gu.beta": t["gu_beta"][sl], "s_down.weight": t["dn_w"][g], "s_down.weight_scale": t["dn_s"][g],
                "s_down.weight_scale_2": t["dn_s2"][g], "s_down.beta": t["dn_beta"][sl],
                "healer.u_gu": t["u_gu"][sl], "healer.v_gu": t["v_gu"][sl], "healer.u_down": t["u_dn"][sl],
                "healer.v_down": np.ascontiguousarray(t["v_dn_t"][sl].transpose(0, 2, 1)),
            })
        if "tail_gu_p" in t:
            for g in range(c.n_slots):
                sl = slice(g * k, (g + 1) * k)
                groups[g].update({"tail.gu_bits": np.uint8(self.tail_bits[0]), "tail.gu_packed": t["tail_gu_p"][sl],
                                  "tail.gu_scale": t["tail_gu_s"][sl], "tail.down_bits": np.uint8(self.tail_bits[1]),
                                  "tail.down_packed": t["tail_dn_p"][sl], "tail.down_scale": t["tail_dn_s"][sl]})
        # (the re-tiled FP4 images are derived data and are not exported)
        extras = {n: t[n] for n in ("router_w", "e_bias", "sh_gu_w", "sh_gu_s", "sh_gu_s2", "sh_dn_w", "sh_dn_s", "sh_dn_s2",
                                    "sh8_gu_w", "sh8_gu_s", "sh8_dn_w", "sh8_dn_s") if n in t}
        return groups, extras


def _read_shared(fh, names: set, shared_prefix: str) -> dict:
    """The always-on expert's tensors under `shared_prefix`: plain NVFP4 (`weight`, `weight_scale`, `weight_scale_2`, the hub
    expert format of chronos_1t/models/vllm_chronos_moe.py:131-141) or stock block-FP8 (`weight`, `weight_scale_inv`,
    chronos_1t/models/glm53_chronos_moe.py:170-181), told apart by the scale tensor's name."""
    fp8 = f"{shared_prefix}.gate_proj.weight_scale_inv" in names
    sfx = ("weight", "weight_scale_inv") if fp8 else ("weight", "weight_scale", "weight_scale_2")
    return {f"{p}.{s}": fh.get_tensor(f"{shared_prefix}.{p}.{s}") for p in ("gate_proj", "up_proj", "down_proj") for s in sfx}


def evict_from_page_cache(path: str | Path) -> None:
    """Tells the kernel that the file's cached pages will not be needed again (chronos_1t/models/glm53_chronos_moe.py:56-63)."""
    import os

    if hasattr(os, "posix_fadvise") and hasattr(os, "POSIX_FADV_DONTNEED"):
        try:
            fd = os.open(os.path.realpath(str(path)), os.O_RDONLY)
            try:
                os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
            finally:
                os.close(fd)
        except OSError:
            pass


def layer_index_from_prefix(prefix: str) -> int | None:
    m = re.search(r"layers\.(\d+)", str(prefix))
    return int(m.group(1)) if m else None
