"""CPU-side checks: the C-ABI library loads and exports what the header declares, host logic (keys, layout
validation, plugin hook with stub vLLM modules) behaves, and nothing computes without a GPU."""
import re
import sys
import types
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import ROOT, golden_groups, load_golden
from oracle import folded_moe_oracle as O

import chronos_b200
from chronos_b200 import _lib, keys
from chronos_b200.layout import FoldedLayerConfig, PackedLayer


@pytest.fixture(scope="module", autouse=True)
def built_library():
    from chronos_b200 import build

    build.build()


def test_library_exports_every_declared_symbol():
    header = (ROOT / "include" / "chronos_b200.h").read_text()
    declared = set(re.findall(r"\b(chronos_b200_\w+)\s*\(", header))
    assert {"chronos_b200_dequant_nvfp4", "chronos_b200_unfold_expert_fp32", "chronos_b200_router_topk",
            "chronos_b200_workspace_bytes", "chronos_b200_folded_moe_decode", "chronos_b200_folded_moe_routed",
            "chronos_b200_last_error"} <= declared
    handle = _lib.lib()
    for name in declared:
        assert hasattr(handle, name), f"{name} is declared in the header but not exported"
    assert declared == set(_lib.EXPORTS), "ctypes table and header disagree"
    assert handle.chronos_b200_abi_version() == _lib.ABI_VERSION


def test_layer_struct_matches_header_layout():
    # 12 four-byte scalars then 41 pointers, no padding surprises
    import ctypes

    assert ctypes.sizeof(_lib.LayerStruct) == 12 * 4 + 44 * 8
    header = (ROOT / "include" / "chronos_b200.h").read_text()
    body = header[header.index("typedef struct chronos_layer {"):header.index("} chronos_layer_t;")]
    names = re.findall(r"(\w+)\s*[;,]", re.sub(r"/\*.*?\*/", "", body, flags=re.S))
    assert names == [n for n, _ in _lib.LayerStruct._fields_]


def test_host_rejects_bad_layer_without_a_gpu():
    s = _lib.LayerStruct()
    assert _lib.lib().chronos_b200_workspace_bytes(s, 4) == 0
    s.hidden, s.inter, s.n_experts, s.group_size, s.n_slots, s.rank, s.top_k = 256, 100, 8, 4, 2, 16, 2
    assert _lib.lib().chronos_b200_workspace_bytes(s, 4) == 0  # inter not a multiple of 128
    rc = _lib.lib().chronos_b200_dequant_nvfp4(None, None, None, None, 4, 30, None)
    assert rc == -1 and b"multiple of 16" in _lib.lib().chronos_b200_last_error()
    with pytest.raises(_lib.ChronosError):
        _lib.check(rc)


def _router_struct(hidden, n_experts, top_k, router_w_addr):
    s = _lib.LayerStruct()
    s.hidden, s.n_experts, s.top_k, s.router_kind, s.router_w = hidden, n_experts, top_k, 0, router_w_addr
    return s


def test_router_rejects_misaligned_table_on_the_host():
    """The router kernels fetch rows with 16-byte bulk copies and vector loads: a table that is not 16-byte aligned
    is refused with CHRONOS_E_ALIGN before any launch (no pointer is dereferenced on the host)."""
    lib = _lib.lib()
    s = _router_struct(256, 8, 2, 0x7F0000000008)  # 8-byte aligned only
    rc = lib.chronos_b200_router_topk(s, 0x7F0000001000, 0, 4, 0x7F0000002000, 0x7F0000003000, 0x7F0000004000, None)
    assert rc == -2 and b"router_w" in lib.chronos_b200_last_error()
    full = _lib.LayerStruct()
    full.hidden, full.inter, full.n_experts, full.group_size, full.n_slots, full.rank, full.top_k = 256, 128, 8, 4, 2, 16, 2
    for name, _ in _lib.LayerStruct._fields_[12:34]:
        setattr(full, name, 0x7F0000010000)
    full.router_w = 0x7F0000000004
    rc = lib.chronos_b200_folded_moe_forward(full, 0x7F0000001000, 0, 4, 0x7F0000002000, 0, 0x7F0000100000, 1 << 30, None)
    assert rc == -2 and b"router_w" in lib.chronos_b200_last_error()


@pytest.mark.skipif(torch.cuda.is_available(), reason="relies on launches being refused for lack of a device")
def test_router_with_rows_too_long_to_stage_takes_the_register_kernel():
    """hidden 16384 in fp32: four activation rows alone exceed the staging budget of the shared-memory router kernel, so
    the launcher must pick the register-tile kernel instead of asking for an impossible amount of shared memory.
    Without a device every launch is refused; which launch was attempted shows in the message."""
    lib = _lib.lib()
    s = _router_struct(16384, 8, 2, 0x7F0000000000)
    rc = lib.chronos_b200_router_topk(s, 0x7F0000100000, 0, 4, 0x7F0000200000, 0x7F0000300000, 0x7F0000400000, None)
    msg = lib.chronos_b200_last_error()
    assert rc == -4 and b"opt in" not in msg and b"router_logits" in msg, msg


def test_compact_key_tables_match_reference_keys(golden):
    h, i, e, k = (int(v) for v in golden["meta"][:4])
    g, m = e // k - 1, k - 1
    sg, sd = keys.group_seed_bases(g)
    for tag, rows, cols, sb in (("gu", 2 * i, h, sg), ("down", h, i, sd)):
        t = keys.compact_tables(rows, cols, m, sb)
        ref = {n: golden[f"ref.keys.{tag}.g{g}.m{m}.{n}"].astype(np.int64)
               for n in ("r_s1", "r_perm", "r_inv", "r_s2", "c_s1", "c_perm", "c_inv", "c_s2")}
        assert np.array_equal(t["cin"] & 0x7FFF, ref["c_perm"])
        assert np.array_equal(t["cin"] >> 15, (ref["c_s1"][ref["c_perm"]] < 0))
        assert np.array_equal(t["rout"] & 0x7FFF, ref["r_inv"])
        assert np.array_equal(t["rout"] >> 15, ref["r_s1"] < 0)
        for name, sign in (("cs2", ref["c_s2"]), ("rs2", ref["r_s2"])):
            bits = (t[name][np.arange(len(sign)) // 32] >> (np.arange(len(sign)) % 32)) & 1
            assert np.array_equal(bits, sign < 0)


def test_packed_layer_validation_on_cpu(golden):
    h, i, e, k, r, top_k, _ = (int(v) for v in golden["meta"])
    cfg = FoldedLayerConfig(hidden=h, inter=i, n_experts=e, group_size=k, rank=r, top_k=top_k)
    groups = golden_groups(golden)
    layer = PackedLayer.from_groups(cfg, groups, golden["router_w"], device="cpu")
    assert layer.struct.n_slots == e // k and layer.struct.shared_inter == 0
    # v_down is stored transposed; everything else byte-identical
    assert np.array_equal(layer.t["v_dn_t"][1].numpy(), groups[0]["healer.v_down"][1].T)
    back, _ = layer.to_groups_numpy()
    for sfx in ("s_gu.weight", "s_down.weight_scale", "healer.v_down", "healer.u_gu"):
        assert np.array_equal(back[1][sfx], groups[1][sfx])
    # failure injection on the host: missing tensor, short tensor, wrong fold factor, NaN scale
    bad = [dict(g) for g in groups]
    del bad[0]["healer.u_gu"]
    with pytest.raises(ValueError, match="missing"):
        PackedLayer.from_groups(cfg, bad, device="cpu")
    bad = [dict(g) for g in groups]
    bad[1]["s_gu.weight"] = bad[1]["s_gu.weight"][:-1]
    with pytest.raises((ValueError, RuntimeError)):
        PackedLayer.from_groups(cfg, bad, device="cpu")
    with pytest.raises(ValueError, match="folds"):
        PackedLayer.from_groups(FoldedLayerConfig(hidden=h, inter=i, n_experts=e, group_size=k // 2, rank=r, top_k=top_k),
                                groups + groups, device="cpu")
    bad = [dict(g) for g in groups]
    bad[0]["s_gu.weight_scale_2"] = np.float32("nan")
    with pytest.raises(ValueError, match="non-finite"):
        PackedLayer.from_groups(cfg, bad, device="cpu")


def test_tail_tensors_load_and_round_trip_on_cpu(tmp_path, golden):
    """include_tail stacks the tail lattice tensors per expert, records the bit widths in the struct, and the loader
    reads them from a converter shard; the oracle's view of the layer (to_groups_numpy) carries them back unchanged."""
    from safetensors.torch import save_file

    h, i, e, k, r, top_k, _ = (int(v) for v in golden["meta"])
    cfg = FoldedLayerConfig(hidden=h, inter=i, n_experts=e, group_size=k, rank=r, top_k=top_k)
    groups = golden_groups(golden)
    gb, db = int(np.asarray(groups[0]["tail.gu_bits"]).reshape(-1)[0]), int(np.asarray(groups[0]["tail.down_bits"]).reshape(-1)[0])
    layer = PackedLayer.from_groups(cfg, groups, golden["router_w"], device="cpu", include_tail=True)
    assert layer.tail_bits == (gb, db) and layer.struct.tail_bits == (gb | (db << 8))
    assert tuple(layer.t["tail_gu_p"].shape) == (e, 2 * i, h * gb // 8)
    assert tuple(layer.t["tail_dn_s"].shape) == (e, h, i // (32 if db == 2 else 64))
    back, _ = layer.to_groups_numpy()
    assert np.array_equal(back[1]["tail.gu_packed"], groups[1]["tail.gu_packed"])
    assert np.array_equal(back[1]["tail.down_scale"], groups[1]["tail.down_scale"])
    plain = PackedLayer.from_groups(cfg, groups, golden["router_w"], device="cpu")
    assert plain.tail_bits == (0, 0) and plain.struct.tail_bits == 0 and "tail_gu_p" not in plain.t
    bad = [dict(g) for g in groups]
    del bad[0]["tail.down_packed"]
    with pytest.raises(ValueError, match="include_tail"):
        PackedLayer.from_groups(cfg, bad, device="cpu", include_tail=True)
    prefix = "model.layers.0.mlp"
    tensors = {}
    for g, grp in enumerate(groups):
        for sfx, arr in grp.items():
            tensors[f"{prefix}.chronos_groups.{g}.{sfx}"] = torch.from_numpy(np.ascontiguousarray(arr)).reshape(np.asarray(arr).shape)
    tensors[f"{prefix}.gate.weight"] = torch.from_numpy(golden["router_w"])
    path = tmp_path / "chronos-glm53-layer-00000-of-00001.safetensors"
    save_file(tensors, str(path))
    loaded = PackedLayer.from_safetensors(path, cfg, prefix, device="cpu", include_tail=True)
    for n in layer.t:
        assert torch.equal(loaded.t[n], layer.t[n]), n


def test_fp4_stage_image_tiler_layout():
    """tile_matrix_fp4 is a pure byte permutation into the documented stage-image layout, for 32, 128 and 192 rows."""
    from chronos_b200.fp4_layout import tile_matrix_fp4

    g = torch.Generator().manual_seed(0)
    for rows in (32, 128, 192):
        p = torch.randint(0, 256, (rows, 256), dtype=torch.uint8, generator=g)   # K = 512: two stages
        s = torch.randint(0, 256, (rows, 32), dtype=torch.uint8, generator=g)
        img = tile_matrix_fp4(p, s, rows)
        nblk = (rows + 127) // 128
        assert tuple(img.shape) == (1, 2, rows * 128 + 2048 * nblk)
        for st in (0, 1):
            for r in (0, rows // 2 + 1, rows - 1):
                for c in (0, 3, 7):
                    for b in (0, 9, 15):
                        assert img[0, st, c * rows * 16 + r * 16 + b] == p[r, st * 128 + c * 16 + b]
                for j in range(4):
                    for si in range(4):
                        off = rows * 128 + j * 512 * nblk + (r // 128) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + si
                        assert img[0, st, off] == s[r, st * 16 + j * 4 + si]
        assert sorted(img[0, :, : rows * 128].reshape(-1).tolist()) == sorted(p.reshape(-1).tolist())


def test_no_cpu_compute_path(golden):
    h, i, e, k, r, top_k, _ = (int(v) for v in golden["meta"])
    cfg = FoldedLayerConfig(hidden=h, inter=i, n_experts=e, group_size=k, rank=r, top_k=top_k)
    if torch.cuda.is_available():
        pytest.skip("CPU-only behaviour")
    with pytest.raises(_lib.ChronosError):
        chronos_b200.FoldedMoELayer(packed=PackedLayer.from_groups(cfg, golden_groups(golden), golden["router_w"], device="cpu"))
    from chronos_b200 import codec

    with pytest.raises(_lib.ChronosError):
        codec.unpack_nvfp4(torch.zeros(4, 8, dtype=torch.uint8), torch.zeros(4, 1, dtype=torch.uint8), torch.tensor(1.0))


def test_safetensors_loader_reads_converter_layout(tmp_path, golden):
    from safetensors.torch import save_file

    h, i, e, k, r, top_k, _ = (int(v) for v in golden["meta"])
    cfg = FoldedLayerConfig(hidden=h, inter=i, n_experts=e, group_size=k, rank=r, top_k=top_k, router="sigmoid")
    prefix = "model.layers.3.mlp"
    tensors = {}
    for g, grp in enumerate(golden_groups(golden)):
        for sfx, arr in grp.items():
            t = torch.from_numpy(np.ascontiguousarray(arr))
            if sfx.split(".")[-1] in ("weight_scale", "u_gu", "v_gu", "u_down", "v_down", "gu_scale", "down_scale"):
                t = t.view(torch.float8_e4m3fn)
            tensors[f"{prefix}.chronos_groups.{g}.{sfx}"] = t
    tensors[f"{prefix}.gate.weight"] = torch.from_numpy(golden["router_w"])
    tensors[f"{prefix}.gate.e_score_correction_bias"] = torch.from_numpy(golden["e_bias"])
    path = tmp_path / "chronos-glm53-layer-00003-of-00005.safetensors"
    save_file(tensors, str(path))
    layer = PackedLayer.from_safetensors(path, cfg, prefix, device="cpu")
    ref = PackedLayer.from_groups(cfg, golden_groups(golden), golden["router_w"], golden["e_bias"], device="cpu")
    for n in ref.t:
        assert torch.equal(layer.t[n], ref.t[n]), n
    # a shard with a slot cut out is refused
    del tensors[f"{prefix}.chronos_groups.1.healer.v_down"]
    save_file(tensors, str(path))
    with pytest.raises(ValueError, match="missing"):
        PackedLayer.from_safetensors(path, cfg, prefix, device="cpu")


def test_vllm_hook_with_stub_modules(tmp_path, monkeypatch):
    """Stub `vllm.*` modules mirroring the import sites (the pattern of the reference's hook self-test,
    benchmarks/glm53_vllm_hook_selftest.py:21-63): class swap, fallback to the stock class, isinstance."""
    from chronos_b200 import vllm_plugin as VP

    class StockMoE(torch.nn.Module):
        def __init__(self, *a, **kw):
            super().__init__()
            self.kw = kw

    pkg = types.ModuleType("vllm")
    me = types.ModuleType("vllm.model_executor")
    models = types.ModuleType("vllm.model_executor.models")
    dsv2 = types.ModuleType("vllm.model_executor.models.deepseek_v2")
    dsv2.DeepseekV2MoE = StockMoE
    for name, mod in (("vllm", pkg), ("vllm.model_executor", me), ("vllm.model_executor.models", models),
                      ("vllm.model_executor.models.deepseek_v2", dsv2)):
        monkeypatch.setitem(sys.modules, name, mod)
    monkeypatch.setenv("CHRONOS_B200_CKPT", str(tmp_path))
    assert VP.enable_chronos_b200_vllm_hook() is True
    hooked = dsv2.DeepseekV2MoE
    assert isinstance(hooked, type) and hooked is not StockMoE and hooked._orig_moe_cls is StockMoE
    assert VP.enable_chronos_b200_vllm_hook() is True and dsv2.DeepseekV2MoE is hooked  # idempotent
    # no config.json / shard in the checkpoint dir -> stock class comes back
    obj = dsv2.DeepseekV2MoE(config=None, prefix="model.layers.7.mlp")
    assert type(obj) is StockMoE and obj.kw["prefix"] == "model.layers.7.mlp"
    # the operator exists and traces through its fake implementation
    assert hasattr(torch.ops.chronos_b200, "moe_forward")
    VP.register()  # never raises


def test_operator_traces_under_fullgraph_compile_and_answers_to_the_reference_name():
    """The operator is registered as `chronos_b200::moe_forward` and under the reference's own name
    `chronos_glm53::moe_forward` (chronos_1t/models/patch_glm53_vllm.py:79-93); a module that calls it compiles with
    `fullgraph=True` through the fake implementation (the check of benchmarks/glm53_vllm_hook_selftest.py:101-116).
    The live block is a stand-in here: this test is about the operator boundary, not the kernels."""
    from chronos_b200 import vllm_plugin as VP
    from chronos_b200.moe import LIVE_BLOCKS

    VP.register_custom_op()

    class Stand:
        def forward_impl(self, x):
            return x * 3.0

    LIVE_BLOCKS[901] = Stand()
    try:
        x = torch.randn(3, 16)
        for op in (torch.ops.chronos_b200.moe_forward, torch.ops.chronos_glm53.moe_forward):
            assert torch.equal(op(x, 901), x * 3.0)

        class Wrap(torch.nn.Module):
            def forward(self, h):
                return torch.ops.chronos_glm53.moe_forward(h, 901) * 2.0

        yc = torch.compile(Wrap(), fullgraph=True, backend="eager")(x)
        assert torch.allclose(yc, x * 6.0)
    finally:
        del LIVE_BLOCKS[901]


def test_packaging_declares_the_vllm_plugin_entry_point():
    import importlib
    import tomllib

    meta = tomllib.loads((ROOT / "pyproject.toml").read_text())
    eps = meta["project"]["entry-points"]["vllm.general_plugins"]
    assert eps == {"chronos_b200": "chronos_b200.vllm_plugin:register"}
    mod, fn = eps["chronos_b200"].split(":")
    assert callable(getattr(importlib.import_module(mod), fn))


def test_config_from_checkpoint(tmp_path):
    import json

    from chronos_b200 import vllm_plugin as VP

    assert VP.config_from_checkpoint(tmp_path) is None
    (tmp_path / "config.json").write_text(json.dumps({
        "hidden_size": 4096, "moe_intermediate_size": 1536, "n_routed_experts": 288, "num_experts_per_tok": 8,
        "scoring_func": "sigmoid", "routed_scaling_factor": 2.5, "norm_topk_prob": True,
        "chronos_holographic_moe": {"group_size": 4, "svd_rank": 64, "key_generator": "torch_cpu_v1"}}))
    cfg = VP.config_from_checkpoint(tmp_path)
    assert (cfg.hidden, cfg.inter, cfg.n_experts, cfg.group_size, cfg.rank, cfg.top_k, cfg.router) == (4096, 1536, 288, 4, 64, 8, "sigmoid")
    assert cfg.bank_bytes_per_slot() == 10_616_832 and cfg.healer_bytes_per_expert() == 819_200
    assert VP.find_layer_shard(tmp_path, 3) is None
    (tmp_path / "chronos-glm53-layer-00003-of-00046.safetensors").write_bytes(b"")
    assert VP.find_layer_shard(tmp_path, 3).name.endswith("00003-of-00046.safetensors")


def test_healer_tiles_carry_the_correction_into_the_accumulator_basis():
    """Load-time algebra of the fused healer: adding tiles . (h * scale) to the bank-pass accumulators BEFORE the epilogue
    (x pair scale x scale_2, r_s2 sign, 128-row Walsh-Hadamard) and gathering with r_inv / r_s1 / beta afterwards gives
    beta * r_s1 * z1[r_inv] + g * U h, the reference's healer term (chronos_1t/models/glm5_chronos_moe.py:149-195)."""
    import math

    import numpy as np
    import torch

    from chronos_b200 import keys
    from chronos_b200.layout import healer_tiles

    torch.manual_seed(0)
    rows, cols, r, n_e, fold = 256, 128, 16, 4, 4
    tabs = [keys.compact_tables(rows, cols, m, 101) for m in range(n_e)]
    rout = torch.from_numpy(np.stack([t["rout"] for t in tabs]).view(np.int16).copy())
    rs2 = torch.from_numpy(np.stack([t["rs2"] for t in tabs]).view(np.int32).copy())
    u8 = torch.randint(0, 256, (n_e, rows, r), dtype=torch.uint8)
    u8[(u8 & 0x7F) == 0x7F] = 0x30  # no NaN codes
    beta, s2 = torch.rand(n_e) + 0.5, torch.tensor([3e-5])
    tiles, scale = healer_tiles(u8, beta, rout, rs2, s2, fold)
    assert tiles.dtype == torch.float16 and tiles.shape == (n_e, rows // 128, r // 8, 128, 8)
    assert 2048.0 < float(tiles.abs().max()) <= 4096.0 and math.log2(scale) == round(math.log2(scale))
    had = torch.ones(1, 1)
    for _ in range(7):
        had = torch.cat([torch.cat([had, had], 1), torch.cat([had, -had], 1)], 0)
    had = had / math.sqrt(128.0)
    g = 2.0  # pair scale
    for e in range(n_e):
        bits = ((rs2[e].long() & 0xFFFFFFFF)[:, None] >> torch.arange(32)) & 1
        sign2 = (1.0 - 2.0 * bits.float()).view(rows)

        def epilogue(acc):
            return (had @ (acc * g * s2[0] * sign2).view(rows // 128, 128, 1)).view(rows)

        ro = rout[e].int() & 0xFFFF
        r_inv, s1 = (ro & 0x7FFF).long(), 1.0 - 2.0 * ((ro >> 15) & 1).float()
        u = u8[e].view(torch.float8_e4m3fn).float()
        h, acc = torch.randn(r), torch.randn(rows) * 1e4
        want = beta[e] * s1 * epilogue(acc)[r_inv] + g * (u @ h)
        tile_rows = tiles[e].float().permute(0, 2, 1, 3).reshape(rows, r)  # [block, unit, row, 8] -> [row, rank column]
        got = beta[e] * s1 * epilogue(acc + tile_rows @ (h * scale))[r_inv]
        assert float((got - want).norm() / want.norm()) < 2e-3
