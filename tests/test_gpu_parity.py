"""Parity of the CUDA path (through the C ABI) against the CPU oracle and the reference-generated golden files.

Bars: NVFP4 dequantisation bit-exact; router logits bit-exact against the oracle's stated summation order and
top-k ids exact (against the oracle everywhere, against the reference's own torch router on the golden cases);
weight-space reconstruction within fp32 round-off; layer output rel-L2 <= 1e-2 against the fp32 reconstruction.
"""
import numpy as np
import pytest
import torch

from conftest import golden_groups
from oracle import folded_moe_oracle as O

pytestmark = pytest.mark.gpu

LAYER_TOL = 1e-2  # relative L2 of the layer output, the tolerance stated for this path


def _rel_l2(a, b):
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _cfg(meta, router="softmax"):
    from chronos_b200 import FoldedLayerConfig

    h, i, e, k, r, top_k, _ = (int(v) for v in meta)
    return FoldedLayerConfig(hidden=h, inter=i, n_experts=e, group_size=k, rank=r, top_k=top_k, router=router)


def _golden_layer(golden, router="softmax", register=False):
    from chronos_b200 import FoldedMoELayer, PackedLayer

    packed = PackedLayer.from_groups(_cfg(golden["meta"], router), golden_groups(golden), golden["router_w"],
                                     golden["e_bias"] if router == "sigmoid" else None, device="cuda")
    return FoldedMoELayer(layer_idx=0, packed=packed, register=register)


# ---------------------------------------------------------------------------------------------------------------
def test_dequant_bit_exact_vs_reference(golden):
    from chronos_b200 import codec

    g0 = golden_groups(golden)[0]
    for tag, sfx in (("gu", "s_gu"), ("down", "s_down")):
        out = codec.unpack_nvfp4(torch.from_numpy(g0[f"{sfx}.weight"]).cuda(), torch.from_numpy(g0[f"{sfx}.weight_scale"]).cuda(),
                                 torch.tensor(float(g0[f"{sfx}.weight_scale_2"])))
        assert np.array_equal(out.cpu().numpy().view(np.uint32), golden[f"ref.dequant_{tag}_g0"].view(np.uint32))


def test_dequant_bit_exact_all_codes():
    from chronos_b200 import codec

    rng = np.random.default_rng(0)
    rows, cols = 64, 512
    packed = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    scale = rng.integers(0, 0x7F, (rows, cols // 16), dtype=np.uint8)  # every finite non-negative e4m3 code, incl. 0
    packed[0, :8] = 0xFF  # saturated nibbles under a zero scale: legal input, dequantises to signed zeros
    scale[0, 0] = 0
    s2 = np.float32(3.1e-5)
    ref = O.unpack_nvfp4(packed, scale, s2)
    out = codec.unpack_nvfp4(torch.from_numpy(packed).cuda(), torch.from_numpy(scale).cuda(), torch.tensor(float(s2)))
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    assert np.all(np.signbit(out.cpu().numpy()[0, :16]))  # -0.0 keeps its sign


def test_reconstruction_matches_reference(golden):
    from chronos_b200 import codec

    h, i, e, k = (int(v) for v in golden["meta"][:4])
    groups = golden_groups(golden)
    seen = 0
    for key in golden:
        if not key.startswith("ref.recon_notail.") or not key.endswith(".gu"):
            continue
        _, gs, ms, _ = key[len("ref.recon_"):].split(".")
        g, m = int(gs[1:]), int(ms[1:])
        gt = {s: torch.from_numpy(np.ascontiguousarray(v)) for s, v in groups[g].items()}
        gu, dn = codec.reconstruct_group_experts(gt, g, [m], h, i, include_tail=False)[0]
        for got, ref in ((gu, golden[key]), (dn, golden[key[:-3] + ".down"])):
            err = np.abs(got.cpu().numpy() - ref).max()
            assert err <= 4e-6 * max(1.0, np.abs(ref).max()), (key, err)
        seen += 1
    assert seen == 2


def test_reconstruction_with_tail_matches_reference(golden):
    """Weight-space probe with the tail lattice term (2-bit Lloyd-Max and 1-bit Rademacher cases) against the
    reference's reconstruct_group_experts(include_tail=True)."""
    from chronos_b200 import codec

    h, i, e, k = (int(v) for v in golden["meta"][:4])
    groups = golden_groups(golden)
    seen = 0
    for key in golden:
        if not key.startswith("ref.recon_tail.") or not key.endswith(".gu"):
            continue
        _, gs, ms, _ = key[len("ref.recon_"):].split(".")
        g, m = int(gs[1:]), int(ms[1:])
        gt = {s: torch.from_numpy(np.ascontiguousarray(v)) for s, v in groups[g].items()}
        gu, dn = codec.reconstruct_group_experts(gt, g, [m], h, i, include_tail=True)[0]
        for got, ref in ((gu, golden[key]), (dn, golden[key[:-3] + ".down"])):
            err = np.abs(got.cpu().numpy() - ref).max()
            assert err <= 4e-6 * max(1.0, np.abs(ref).max()), (key, err)
        seen += 1
    assert seen == 1


@pytest.mark.parametrize("regime,n_tok,tails", [("auto", 5, (2, 2)), ("auto", 5, (1, 2)), ("stream", 7, (2, 1)), ("tensor", 90, (2, 2)),
                                                ("tensor_fp4", 90, (1, 1)), ("tensor_fp4", 150, (2, 2))])
def test_layer_with_tail_matches_oracle(regime, n_tok, tails):
    """Whole layer with the tail lattice term in every regime against the fp32 oracle (include_tail=True)."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=512, inter=256, n_experts=8, group_size=4, rank=32, top_k=2)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=21, with_shared=True, tail_bits=tails, keep_disk_order=True), register=False)
    gen = torch.Generator(device="cuda").manual_seed(n_tok)
    x = torch.randn(n_tok, cfg.hidden, generator=gen, device="cuda").to(torch.bfloat16)
    y = layer.forward_impl(x, regime=regime)
    assert layer.device_status() == 0
    ref, _, _ = _oracle_layer(layer, x.float().cpu().numpy(), include_tail=True)
    ref0, _, _ = _oracle_layer(layer, x.float().cpu().numpy(), include_tail=False)
    assert _rel_l2(ref0, ref) > 5e-2, "the synthetic tail must matter, or the test proves nothing"
    assert _rel_l2(y.float().cpu().numpy(), ref) <= LAYER_TOL


def test_router_matches_reference_and_oracle(golden):
    top_k = int(golden["meta"][5])
    x = torch.from_numpy(golden["x"]).cuda()
    for flavour in ("softmax", "sigmoid"):
        layer = _golden_layer(golden, flavour)
        ids, w = layer.route(x)
        assert np.array_equal(ids.cpu().numpy(), golden[f"ref.router.{flavour}_ids"])
        assert np.allclose(w.cpu().numpy(), golden[f"ref.router.{flavour}_gates"], rtol=2e-5, atol=1e-7)
        fixed = O.router_logits_fixed(golden["x"], golden["router_w"])
        assert np.array_equal(layer.last_logits.cpu().numpy().view(np.uint32), fixed.view(np.uint32))


@pytest.mark.parametrize("n_tok,dtype", [(1, "f32"), (37, "bf16"), (100, "f32"), (256, "bf16"), (259, "f32")])
def test_router_bit_exact_large(n_tok, dtype):
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=1024, inter=128, n_experts=288, group_size=4, rank=16, top_k=8)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=5), register=False)
    gen = torch.Generator(device="cuda").manual_seed(n_tok)
    x = torch.randn(n_tok, cfg.hidden, generator=gen, device="cuda")
    if dtype == "bf16":
        x = x.to(torch.bfloat16)
    ids, w = layer.route(x)
    logits = O.router_logits_fixed(x.float().cpu().numpy(), layer.packed.t["router_w"].cpu().numpy())
    assert np.array_equal(layer.last_logits.cpu().numpy().view(np.uint32), logits.view(np.uint32))
    ref_ids, ref_w = O.router_softmax_topk(logits, cfg.top_k)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    assert np.allclose(w.cpu().numpy(), ref_w, rtol=2e-5, atol=1e-7)


@pytest.mark.parametrize("flavour", ["softmax", "sigmoid", "sqrt_softplus"])
def test_router_at_benchmark_shape_vs_reference(flavour):
    """288 experts x hidden 4096 x 512 bf16 tokens: device ids against the reference's own torch router (golden file).
    Logits are bit-equal to the oracle's stated order; tokens whose k / k+1 choice scores are closer than the fp32
    summation error are counted apart from true mismatches, of which there must be none."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer
    from conftest import compare_router_ids, router_case, router_choice_scores

    gold, x, router_w, e_bias, k = router_case()
    e, h = router_w.shape
    cfg = FoldedLayerConfig(hidden=h, inter=128, n_experts=e, group_size=4, rank=16, top_k=k, router=flavour,
                            routed_scaling_factor=1.5 if flavour == "sqrt_softplus" else 2.5)
    packed = PackedLayer.synthetic(cfg, seed=5)
    packed.t["router_w"].copy_(torch.from_numpy(router_w))
    if flavour != "softmax":
        packed.t["e_bias"].copy_(torch.from_numpy(e_bias))
    layer = FoldedMoELayer(packed=packed, register=False)
    ids, w = layer.route(torch.from_numpy(x).cuda().to(torch.bfloat16))
    fixed = O.router_logits_fixed(x, router_w)
    assert np.array_equal(layer.last_logits.cpu().numpy().view(np.uint32), fixed.view(np.uint32))
    ids, w = ids.cpu().numpy(), w.cpu().numpy()
    rep = compare_router_ids(ids, gold[f"{flavour}_ids"], router_choice_scores(gold["logits"], flavour, e_bias), k)
    print(flavour, rep)
    assert rep["true_mismatch_tokens"] == 0 and rep["near_tie_tokens"] <= rep["tokens"] // 50, rep
    same = (ids == gold[f"{flavour}_ids"]).all(axis=1)
    assert np.allclose(w[same], gold[f"{flavour}_gates"][same], rtol=3e-5, atol=1e-7)


@pytest.mark.parametrize("flavour", ["softmax", "sigmoid"])
def test_nan_activation_row_selects_no_expert(flavour):
    """A token whose hidden row is NaN has NaN logits: no candidate can win, the token gets ids -1 / gates 0 and its
    routed output is skipped; the other tokens of the batch are unaffected and no address is formed from a bad id."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=512, inter=256, n_experts=16, group_size=4, rank=16, top_k=4, router=flavour)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=31), register=False)
    gen = torch.Generator(device="cuda").manual_seed(2)
    for n_tok in (5, 70):  # top-k fused into the plan launch / the router's own top-k kernel
        x = torch.randn(n_tok, cfg.hidden, generator=gen, device="cuda")
        clean = layer(x).clone()
        xb = x.clone()
        xb[2] = float("nan")
        ids, w = layer.route(xb)
        assert ids[2].tolist() == [-1] * 4 and w[2].tolist() == [0.0] * 4
        ref_ids, ref_w = (O.router_softmax_topk if flavour == "softmax" else
                          (lambda lg, k: O.router_sigmoid_topk(lg, layer.packed.t["e_bias"].cpu().numpy(), k)))(layer.last_logits.cpu().numpy(), 4)
        assert np.array_equal(ids.cpu().numpy(), ref_ids)
        y = layer(xb)
        assert layer.device_status() == 0
        keep = [t for t in range(n_tok) if t != 2]
        assert torch.equal(y[keep], clean[keep])
        assert torch.count_nonzero(y[2]) == 0  # no shared expert in this layer: nothing was added for the token


def test_layer_output_matches_reference(golden):
    for flavour in ("softmax", "sigmoid"):
        layer = _golden_layer(golden, flavour)
        ref = golden[f"ref.layer_y.{flavour}"]
        y32 = layer(torch.from_numpy(golden["x"]).cuda())
        assert y32.dtype == torch.float32 and layer.device_status() == 0
        assert _rel_l2(y32.cpu().numpy(), ref) <= LAYER_TOL, flavour
        # bf16 activations: compare with the oracle fed the same rounded activations
        xb = torch.from_numpy(golden["x"]).cuda().to(torch.bfloat16)
        h, i, e, k, r, top_k, _ = (int(v) for v in golden["meta"])
        ref_b = O.moe_layer_forward(xb.float().cpu().numpy(), golden_groups(golden), golden["router_w"], top_k, h, i, k,
                                    router=flavour, e_bias=golden["e_bias"])
        yb = layer(xb)
        assert yb.dtype == torch.bfloat16
        assert _rel_l2(yb.float().cpu().numpy(), ref_b) <= LAYER_TOL, flavour


def _oracle_layer(layer, x_np, with_shared=True, include_tail=False):
    groups, extras = layer.packed.to_groups_numpy()
    c = layer.cfg
    shared = None
    if with_shared and "sh8_gu_w" in extras:
        shared = O.shared_fp8_weights(extras)
    elif with_shared and "sh_gu_w" in extras:
        i = c.inter
        gate = O.unpack_nvfp4(extras["sh_gu_w"][:i], extras["sh_gu_s"][:i], extras["sh_gu_s2"][0])
        up = O.unpack_nvfp4(extras["sh_gu_w"][i:], extras["sh_gu_s"][i:], extras["sh_gu_s2"][1])
        shared = (np.concatenate([gate, up]), O.unpack_nvfp4(extras["sh_dn_w"], extras["sh_dn_s"], extras["sh_dn_s2"][0]))
    return O.moe_layer_forward(x_np, groups, extras["router_w"], c.top_k, c.hidden, c.inter, c.group_size, router=c.router,
                               e_bias=extras.get("e_bias"), routed_scaling=c.routed_scaling_factor, shared=shared,
                               include_tail=include_tail, return_routing=True)


def test_config0_layer_with_folded_weights():
    """CPU-runnable case: hidden 2048, 64 experts, top-8 softmax router, inter 768, fold 4, rank 32, 3 tokens fp32."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=2048, inter=768, n_experts=64, group_size=4, rank=32, top_k=8)
    rng = np.random.default_rng(0)
    router_w = (rng.standard_normal((64, 2048)) * 0.02).astype(np.float32)
    x = rng.standard_normal((3, 2048)).astype(np.float32)
    logits = O.router_logits_fixed(x, router_w)
    ids, _ = O.router_softmax_topk(logits, 8)
    used = sorted({int(e) // 4 for e in ids.reshape(-1)})
    groups = []
    for g in range(16):
        if g in used:  # fold real N(0, 0.02) experts for the slots this batch touches; untouched slots get random bytes
            gate, up = (rng.standard_normal((4, 768, 2048)).astype(np.float32) * 0.02 for _ in range(2))
            down = rng.standard_normal((4, 2048, 768)).astype(np.float32) * 0.02
            groups.append(O.fold_group_synthetic(gate, up, down, g, 32))
        else:
            groups.append(O.random_group(rng, 4, 2048, 768, 32))
    layer = FoldedMoELayer(packed=PackedLayer.from_groups(cfg, groups, router_w, device="cuda"), register=False)
    y = layer(torch.from_numpy(x).cuda())
    ref, ref_ids, ref_w = _oracle_layer(layer, x)
    got_ids, got_w = layer.route(torch.from_numpy(x).cuda())
    assert np.array_equal(got_ids.cpu().numpy(), ref_ids)
    assert layer.device_status() == 0
    assert _rel_l2(y.cpu().numpy(), ref) <= LAYER_TOL


@pytest.mark.parametrize("streams", [1, 4])
def test_decode_shaped_layer(streams):
    """Decode-shaped layer: hidden 4096, 288 experts + shared, top-8, inter 1536, fold 4, rank 64, bf16, 3 tokens/stream."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=4096, inter=1536, n_experts=288, group_size=4, rank=64, top_k=8)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=1, with_shared=True), register=False)
    gen = torch.Generator(device="cuda").manual_seed(1)
    base = torch.randn(streams, 1, cfg.hidden, generator=gen, device="cuda")
    x = (0.55 * base + 0.84 * torch.randn(streams, 3, cfg.hidden, generator=gen, device="cuda")).reshape(-1, cfg.hidden).to(torch.bfloat16)
    y1 = layer(x)
    y2 = layer(x)
    assert torch.equal(y1, y2), "two runs on the same input must be bit-identical"
    assert layer.device_status() == 0
    ref, ref_ids, _ = _oracle_layer(layer, x.float().cpu().numpy())
    ids, _ = layer.route(x)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    assert _rel_l2(y1.float().cpu().numpy(), ref) <= LAYER_TOL


def test_fp4_streaming_regime_matches_oracle_and_cuda_core_regime():
    """The same decode-shaped batch through the block-scaled FP4 tensor-core pass and the CUDA-core conversion pass."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=1024, inter=512, n_experts=32, group_size=4, rank=32, top_k=4)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=4, with_shared=True, keep_disk_order=True), register=False)
    assert layer.packed.struct.gu_t and layer.packed.struct.dn_t
    gen = torch.Generator(device="cuda").manual_seed(8)
    for scale in (1.0, 37.0, 0.004):  # the per-pair power-of-two scale must absorb the activation magnitude
        x = (torch.randn(7, cfg.hidden, generator=gen, device="cuda") * scale).to(torch.bfloat16)
        y4 = layer.forward_impl(x, regime="stream_fp4")
        assert layer.device_status() == 0
        ys = layer.forward_impl(x, regime="stream")
        assert layer.device_status() == 0
        ref, _, _ = _oracle_layer(layer, x.float().cpu().numpy())
        assert _rel_l2(y4.float().cpu().numpy(), ref) <= LAYER_TOL, scale
        assert _rel_l2(ys.float().cpu().numpy(), ref) <= LAYER_TOL, scale
        assert torch.equal(y4, layer.forward_impl(x, regime="stream_fp4")), "FP4 pass must be reproducible"
        assert torch.equal(layer.forward_impl(x, regime="auto"), y4)  # 28 pairs on 8 slots: auto = FP4 streaming


@pytest.mark.parametrize("n_tok,top_k,rank", [(32, 8, 32), (40, 8, 32), (9, 6, 128), (2, 3, 16)])
def test_streaming_fp4_paths_at_their_batch_limits(n_tok, top_k, rank):
    """The FP4 streaming regime on both of its code paths: up to 32 tokens take the fused decode path (front kernel with
    the grid-wide hand-off, healer products inside the bank passes), larger batches the separate-kernel path; many
    slots, few pairs per slot, shared expert, every healer rank the side warps are instantiated for."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=512, inter=256, n_experts=288, group_size=4, rank=rank, top_k=top_k)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=41, with_shared=True), register=False)
    gen = torch.Generator(device="cuda").manual_seed(n_tok)
    x = torch.randn(n_tok, cfg.hidden, generator=gen, device="cuda").to(torch.bfloat16)
    y = layer.forward_impl(x, regime="stream_fp4")
    assert layer.device_status() == 0
    assert torch.equal(y, layer.forward_impl(x, regime="auto"))
    ref, ref_ids, _ = _oracle_layer(layer, x.float().cpu().numpy())
    ids, w = layer.route(x)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    assert _rel_l2(y.float().cpu().numpy(), ref) <= LAYER_TOL
    # the same batch with the routing handed in by the caller, fp32 activations at the boundary
    y_r = layer.routed_forward(x.float(), ids, w, with_shared=True, regime="stream_fp4")
    assert layer.device_status() == 0
    assert _rel_l2(y_r.cpu().numpy(), ref) <= LAYER_TOL


def test_many_tokens_on_one_slot_and_skipped_entries():
    """More than 8 pairs on a slot (several work items per slot), entries with id -1, routing supplied by the caller."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=512, inter=256, n_experts=16, group_size=4, rank=16, top_k=2)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=7, keep_disk_order=True), register=False)
    n = 21
    gen = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(n, cfg.hidden, generator=gen, device="cuda")
    ids = torch.zeros((n, 2), dtype=torch.int32, device="cuda")
    ids[:, 0] = 5                      # 21 pairs on expert 5 (slot 1)
    ids[:, 1] = torch.arange(n, device="cuda", dtype=torch.int32) % 4 + 4   # the other members of slot 1
    ids[::2, 1] = 6
    ids[3, 1] = -1                     # skipped entry
    w = torch.rand((n, 2), generator=gen, device="cuda")
    y = layer.routed_forward(x, ids, w)
    assert layer.device_status() == 0
    groups, _ = layer.packed.to_groups_numpy()
    ref = np.zeros((n, cfg.hidden), dtype=np.float32)
    xn, idn, wn = x.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy()
    for e in np.unique(idn[idn >= 0]):
        gu, dn = O.reconstruct_expert(groups[e // 4], int(e) // 4, int(e) % 4, cfg.hidden, cfg.inter)
        for t, j in zip(*np.nonzero(idn == e)):
            z = xn[t] @ gu.T
            ref[t] += wn[t, j] * ((O.silu(z[:cfg.inter]) * z[cfg.inter:]) @ dn.T)
    assert _rel_l2(y.cpu().numpy(), ref) <= LAYER_TOL
    # the tensor-core regime forced onto a batch below its usual threshold (its small-batch healer kernels)
    y_t = layer.routed_forward(x, ids, w, regime="tensor")
    assert layer.device_status() == 0
    assert _rel_l2(y_t.cpu().numpy(), ref) <= LAYER_TOL
    # all entries skipped -> exact zeros; zero tokens -> empty output
    y0 = layer.routed_forward(x, torch.full_like(ids, -1), w)
    assert torch.count_nonzero(y0) == 0
    assert layer(torch.empty(0, cfg.hidden, device="cuda")).shape == (0, cfg.hidden)


def _pairs_reference(layer, x, ids, w):
    """fp32 oracle of the routed experts for explicit routing (numpy arrays in, [T, H] out)."""
    c = layer.cfg
    groups, _ = layer.packed.to_groups_numpy()
    ref = np.zeros((x.shape[0], c.hidden), dtype=np.float32)
    for e in np.unique(ids[ids >= 0]):
        gu, dn = O.reconstruct_expert(groups[e // c.group_size], int(e) // c.group_size, int(e) % c.group_size, c.hidden, c.inter)
        for t, j in zip(*np.nonzero(ids == e)):
            z = x[t] @ gu.T
            ref[t] += w[t, j] * ((O.silu(z[:c.inter]) * z[c.inter:]) @ dn.T)
    return ref


def test_tensor_regime_matches_oracle_and_stream_regime():
    """The tcgen05 grouped-GEMM path against the fp32 oracle, and against the streaming path on the same batch
    (the decode-path vs prefill-path equivalence check of benchmarks/glm53_synthetic_e2e_test.py:194-204)."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=512, inter=256, n_experts=8, group_size=4, rank=16, top_k=2)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=11, with_shared=True, keep_disk_order=True), register=False)
    n = 300  # > 128 pairs on several experts: full tiles, ragged tiles and (expert 7 unused) empty ones
    gen = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(n, cfg.hidden, generator=gen, device="cuda").to(torch.bfloat16)
    ids = torch.randint(0, 7, (n, 2), generator=gen, device="cuda", dtype=torch.int32)
    ids[:, 1] = (ids[:, 0] + 1 + torch.randint(0, 5, (n,), generator=gen, device="cuda", dtype=torch.int32)) % 7
    ids[5, 0] = -1
    w = torch.rand((n, 2), generator=gen, device="cuda")
    y_t = layer.routed_forward(x, ids, w, regime="tensor", out_dtype=torch.float32)
    assert layer.device_status() == 0
    y_s = layer.routed_forward(x, ids, w, regime="stream", out_dtype=torch.float32)
    assert layer.device_status() == 0
    ref = _pairs_reference(layer, x.float().cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy())
    assert _rel_l2(y_t.cpu().numpy(), ref) <= LAYER_TOL
    assert _rel_l2(y_s.cpu().numpy(), ref) <= LAYER_TOL
    assert _rel_l2(y_t.cpu().numpy(), y_s.cpu().numpy()) <= 2e-3
    y_t2 = layer.routed_forward(x, ids, w, regime="tensor", out_dtype=torch.float32)
    assert torch.equal(y_t, y_t2), "two runs on the same input must be bit-identical"
    # fp32 activations at the boundary (same values): same result within the fp16 operand rounding
    y_f = layer.routed_forward(x.float(), ids, w, regime="tensor", out_dtype=torch.float32)
    assert _rel_l2(y_f.cpu().numpy(), ref) <= LAYER_TOL
    # the block-scaled FP4 grouped GEMM (work items of 64 pairs x 3 residual terms) on the same batch
    y_w = layer.routed_forward(x, ids, w, regime="tensor_fp4", out_dtype=torch.float32)
    assert layer.device_status() == 0
    assert _rel_l2(y_w.cpu().numpy(), ref) <= LAYER_TOL
    assert _rel_l2(y_w.cpu().numpy(), y_t.cpu().numpy()) <= 3e-3
    assert torch.equal(y_w, layer.routed_forward(x, ids, w, regime="tensor_fp4", out_dtype=torch.float32))
    assert torch.equal(y_w, layer.routed_forward(x, ids, w, regime="auto", out_dtype=torch.float32))


@pytest.mark.parametrize("rank", [32, 64, 128])
def test_tensor_regime_whole_layer_with_router_and_shared(rank):
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=1024, inter=384, n_experts=16, group_size=4, rank=rank, top_k=4)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=2, with_shared=True, keep_disk_order=True), register=False)
    gen = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(200, cfg.hidden, generator=gen, device="cuda").to(torch.bfloat16)
    y = layer.forward_impl(x, regime="tensor")
    assert layer.device_status() == 0
    ref, ref_ids, _ = _oracle_layer(layer, x.float().cpu().numpy())
    ids, _ = layer.route(x)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    assert _rel_l2(y.float().cpu().numpy(), ref) <= LAYER_TOL
    assert torch.equal(layer.forward_impl(x, regime="auto"), y)  # 800 pairs on 4 slots: auto picks the tensor regime


@pytest.mark.parametrize("scale", [1.0, 3e-3, 200.0])
def test_tensor_fp4_regime_whole_layer(scale):
    """Router + routed + shared expert through the FP4 grouped-GEMM regime, decode-like dimensions scaled down,
    activations of very different magnitudes (the per-pair scaling keeps the e2m1 images in range)."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=1024, inter=512, n_experts=16, group_size=4, rank=64, top_k=4)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=4, with_shared=True, keep_disk_order=True), register=False)
    gen = torch.Generator(device="cuda").manual_seed(13)
    x = (torch.randn(330, cfg.hidden, generator=gen, device="cuda") * scale).to(torch.bfloat16)
    y = layer.forward_impl(x, regime="tensor_fp4")
    assert layer.device_status() == 0
    ref, ref_ids, _ = _oracle_layer(layer, x.float().cpu().numpy())
    assert _rel_l2(y.float().cpu().numpy(), ref) <= LAYER_TOL
    assert torch.equal(layer.forward_impl(x, regime="auto"), y)  # 1320 pairs on 4 slots: auto = FP4 tensor regime
    y16 = layer.forward_impl(x, regime="tensor")
    assert _rel_l2(y16.float().cpu().numpy(), ref) <= LAYER_TOL


@pytest.mark.parametrize("rank", [16, 64])
def test_fused_healer_equals_separate_healer_pass(rank, monkeypatch):
    """FP4 tensor regime: the low-rank correction added inside the bank pass (healer tiles built at load) against the same
    layer without the tiles (a pass of its own after the bank pass), and both against the oracle."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=1024, inter=512, n_experts=16, group_size=4, rank=rank, top_k=4)
    fused = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=6, with_shared=True), register=False)
    assert "ut_gu" in fused.packed.t and fused.packed.struct.ut_gu
    monkeypatch.setattr(PackedLayer, "fused_healer_default", False)
    plain = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=6, with_shared=True), register=False)
    assert "ut_gu" not in plain.packed.t and not plain.packed.struct.ut_gu
    gen = torch.Generator(device="cuda").manual_seed(21)
    x = torch.randn(300, cfg.hidden, generator=gen, device="cuda").to(torch.bfloat16)
    y_f = fused.forward_impl(x, regime="tensor_fp4")
    y_p = plain.forward_impl(x, regime="tensor_fp4")
    assert fused.device_status() == 0 and plain.device_status() == 0
    ref, _, _ = _oracle_layer(plain, x.float().cpu().numpy())
    e_f, e_p = _rel_l2(y_f.float().cpu().numpy(), ref), _rel_l2(y_p.float().cpu().numpy(), ref)
    print(f"rank {rank}: fused {e_f:.3e}, separate pass {e_p:.3e}, fused vs separate {_rel_l2(y_f.float().cpu().numpy(), y_p.float().cpu().numpy()):.3e}")
    assert e_f <= LAYER_TOL and e_p <= LAYER_TOL
    assert _rel_l2(y_f.float().cpu().numpy(), y_p.float().cpu().numpy()) <= 3e-3  # both round to bf16 at the end


@pytest.mark.parametrize("n_tok,regime", [(6, "auto"), (200, "auto")])
def test_forward_is_cuda_graph_capturable(n_tok, regime):
    """The whole-layer call makes no host synchronisation and no allocation of its own: it can be captured into a CUDA graph
    (what a serving engine does with the decode step) and replayed on new inputs with the same result as an eager call."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=512, inter=256, n_experts=16, group_size=4, rank=32, top_k=4)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=23, with_shared=True), register=False)
    gen = torch.Generator(device="cuda").manual_seed(n_tok)
    x_static = torch.randn(n_tok, cfg.hidden, generator=gen, device="cuda").to(torch.bfloat16)
    x_new = torch.randn(n_tok, cfg.hidden, generator=gen, device="cuda").to(torch.bfloat16)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up: the workspace reaches its final size before capture
        layer.forward_impl(x_static, regime=regime)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y_static = layer.forward_impl(x_static, regime=regime)
    x_static.copy_(x_new)
    graph.replay()
    torch.cuda.synchronize()
    y_eager = layer.forward_impl(x_new, regime=regime)
    assert layer.device_status() == 0
    assert torch.equal(y_static, y_eager)


def test_large_batch_without_optional_copies_and_shared_expert_range():
    """A layer description without the optional load-time copies (FP4 stage images, healer.v_down as on disk) takes the
    fp16 tensor regime with the CUDA-core healer kernels; and the shared expert can be limited to a block of tokens
    (what an expert-parallel rank does for the tokens it is the home of)."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer

    cfg = FoldedLayerConfig(hidden=512, inter=256, n_experts=8, group_size=4, rank=32, top_k=2)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=17, with_shared=True, keep_disk_order=True), register=False)
    gen = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(120, cfg.hidden, generator=gen, device="cuda").to(torch.bfloat16)
    ids, w = layer.route(x)
    y_all = layer.routed_forward(x, ids, w, with_shared=True, out_dtype=torch.float32)
    y_none = layer.routed_forward(x, ids, w, with_shared=False, out_dtype=torch.float32)
    y_rng = layer.routed_forward(x, ids, w, out_dtype=torch.float32, shared_range=(40, 50))
    assert layer.device_status() == 0
    assert torch.equal(y_rng[:40], y_none[:40]) and torch.equal(y_rng[90:], y_none[90:])
    assert torch.equal(y_rng[40:90], y_all[40:90])
    with pytest.raises(Exception):
        layer.routed_forward(x, ids, w, shared_range=(100, 50))  # runs past the last token
    ref, _, _ = _oracle_layer(layer, x.float().cpu().numpy())
    assert _rel_l2(y_all.cpu().numpy(), ref) <= LAYER_TOL
    # strip the optional copies from the struct: same answer from the fallback kernels
    st = layer.packed.struct
    for name in ("gu_t", "dn_t", "sh_gu_t", "sh_dn_t", "v_dn"):
        setattr(st, name, None)
    y_fb = layer.routed_forward(x, ids, w, with_shared=True, out_dtype=torch.float32)
    assert layer.device_status() == 0
    assert _rel_l2(y_fb.cpu().numpy(), ref) <= LAYER_TOL
    assert _rel_l2(y_fb.cpu().numpy(), y_all.cpu().numpy()) <= 3e-3


@pytest.mark.parametrize("n_stages,b_rows", [(1, 32), (3, 32), (2, 192), (1, 256), (1, 64)])
def test_fp4_tensor_core_operand_format(n_stages, b_rows):
    """tcgen05 block-scaled FP4 MMA on re-tiled operand images == dequantise-and-multiply of the same bytes."""
    from chronos_b200 import _lib
    from chronos_b200.fp4_layout import tile_matrix_fp4

    rng = np.random.default_rng(n_stages)
    k = 256 * n_stages
    a_p = rng.integers(0, 256, (128, k // 2), dtype=np.uint8)
    b_p = rng.integers(0, 256, (b_rows, k // 2), dtype=np.uint8)
    a_s = rng.integers(0x28, 0x48, (128, k // 16), dtype=np.uint8)   # e4m3 2^-2 .. 2^1.9, non-negative
    b_s = rng.integers(0x28, 0x48, (b_rows, k // 16), dtype=np.uint8)
    ref = O.unpack_nvfp4(a_p, a_s, 1.0).astype(np.float64) @ O.unpack_nvfp4(b_p, b_s, 1.0).astype(np.float64).T
    a_img = tile_matrix_fp4(torch.from_numpy(a_p).cuda(), torch.from_numpy(a_s).cuda(), 128)
    b_img = tile_matrix_fp4(torch.from_numpy(b_p).cuda(), torch.from_numpy(b_s).cuda(), b_rows)
    assert a_img.shape == (1, n_stages, 18432)
    assert b_img.shape == (1, n_stages, b_rows * 128 + 2048 * ((b_rows + 127) // 128))
    d = torch.zeros((128, b_rows), dtype=torch.float32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check(_lib.lib().chronos_b200_fp4_mma_probe(a_img.data_ptr(), b_img.data_ptr(), n_stages, b_rows, d.data_ptr(),
                                                    status.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    got = d.cpu().numpy().astype(np.float64)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max(), np.abs(got - ref).max() / np.abs(ref).max()


def test_layer_resident_as_stage_images_only_and_direct_loader(golden, tmp_path):
    """By default a layer whose shapes the FP4 regimes serve keeps ONE copy of its banks (the stage images): half the
    resident bytes, same outputs; the regimes and probes that read the on-disk order refuse it with a clear message.
    And a converter-format shard written from reference-converted slots loads straight onto the device (tensor by tensor
    from the mapped file) and reproduces the reference's layer output."""
    from safetensors.torch import save_file

    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer, _lib

    cfg = FoldedLayerConfig(hidden=512, inter=256, n_experts=16, group_size=4, rank=16, top_k=4)
    both = PackedLayer.synthetic(cfg, seed=9, with_shared=True, keep_disk_order=True)
    lean = PackedLayer.synthetic(cfg, seed=9, with_shared=True)
    assert "gu_w" in both.t and "gu_w" not in lean.t and not lean.struct.gu_w and lean.struct.gu_t
    healer_tiles = sum(lean.t[n].numel() * lean.t[n].element_size() for n in ("ut_gu", "ut_dn"))  # in both layers alike
    assert lean.resident_bytes() - healer_tiles < 0.62 * (both.resident_bytes() - healer_tiles)
    ga, gb = both.to_groups_numpy(), lean.to_groups_numpy()  # the images invert to the very bytes that were dropped
    for da, db in zip(ga[0], gb[0]):
        assert all(np.array_equal(da[n], db[n]) for n in da)
    assert all(np.array_equal(ga[1][n], gb[1][n]) for n in ga[1])
    la, lb = FoldedMoELayer(packed=both, register=False), FoldedMoELayer(packed=lean, register=False)
    gen = torch.Generator(device="cuda").manual_seed(4)
    for n_tok in (5, 200):
        x = torch.randn(n_tok, cfg.hidden, generator=gen, device="cuda").to(torch.bfloat16)
        assert torch.equal(la(x), lb(x))
    with pytest.raises(_lib.ChronosError, match="on-disk order"):
        lb.forward_impl(x, regime="stream")
    # direct loader: golden slots (reference converter output) -> shard -> device
    h, i, e, k, r, top_k, _ = (int(v) for v in golden["meta"])
    gcfg = _cfg(golden["meta"], "sigmoid")
    prefix = "model.layers.3.mlp"
    tensors = {}
    for g, grp in enumerate(golden_groups(golden)):
        for sfx, arr in grp.items():
            t = torch.from_numpy(np.ascontiguousarray(arr))
            tensors[f"{prefix}.chronos_groups.{g}.{sfx}"] = t.view(torch.float8_e4m3fn) if (sfx.endswith("_scale") or sfx.startswith("healer.")) else t
    tensors[f"{prefix}.gate.weight"] = torch.from_numpy(golden["router_w"])
    tensors[f"{prefix}.gate.e_score_correction_bias"] = torch.from_numpy(golden["e_bias"])
    path = tmp_path / "chronos-glm53-layer-00003-of-00005.safetensors"
    save_file(tensors, str(path))
    direct = PackedLayer.from_safetensors(path, gcfg, prefix, device="cuda")
    staged = PackedLayer.from_groups(gcfg, golden_groups(golden), golden["router_w"], golden["e_bias"], device="cuda")
    for n in staged.t:
        assert torch.equal(direct.t[n], staged.t[n]), n
    y = FoldedMoELayer(packed=direct, register=False)(torch.from_numpy(golden["x"]).cuda())
    assert _rel_l2(y.cpu().numpy(), golden["ref.layer_y.sigmoid"]) <= LAYER_TOL
    with_tail = PackedLayer.from_safetensors(path, gcfg, prefix, device="cuda", include_tail=True)
    assert with_tail.tail_bits != (0, 0) and "tail_gu_p" in with_tail.t


@pytest.mark.parametrize("flavour", ["softmax", "sigmoid"])
def test_coalesced_routing_matches_its_oracle_and_runs_the_layer(flavour):
    """The batch-coalesced router on the device: ids identical to the oracle's restatement of the policy, gates equal,
    fewer distinct slots per step than natural routing, and the layer evaluated with that routing matches the oracle."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer
    from chronos_b200.workloads import decode_batches

    cfg = FoldedLayerConfig(hidden=512, inter=256, n_experts=288, group_size=4, rank=16, top_k=8, router=flavour)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=61, with_shared=True), register=False)
    if flavour != "softmax":
        layer.packed.t["e_bias"].copy_(torch.randn(cfg.n_experts, generator=torch.Generator().manual_seed(1)) * 0.05)
    x = decode_batches(cfg, 4, "cuda", seed=5, n_batches=1)[0]
    nat_ids, _ = layer.route(x)
    ids, w = layer.route_coalesced(x, tokens_per_stream=3, pool=12, keep=4)
    logits = layer.last_logits.cpu().numpy()
    bias = layer.packed.t["e_bias"].cpu().numpy() if flavour != "softmax" else None
    ref_ids, ref_w = O.router_coalesced(logits, cfg.top_k, 3, 12, 4, 1.0e4, router=flavour, e_bias=bias)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    assert np.allclose(w.cpu().numpy(), ref_w, rtol=3e-5, atol=1e-7)
    assert torch.equal(ids[0::3], nat_ids[0::3]), "anchors must be routed naturally"
    experts = lambda a: len(set(a.reshape(-1).tolist()))
    slots = lambda a: len({int(e) // cfg.group_size for e in a.reshape(-1).tolist()})
    assert experts(ids) < experts(nat_ids) and slots(ids) <= slots(nat_ids)
    same, _ = layer.route_coalesced(x, tokens_per_stream=3, pool=8, keep=4)
    assert torch.equal(torch.sort(same, dim=1).values, torch.sort(nat_ids, dim=1).values)
    y = layer.routed_forward(x, ids, w, with_shared=True)
    assert layer.device_status() == 0
    groups, ex = layer.packed.to_groups_numpy()
    shared = (np.concatenate([O.unpack_nvfp4(ex["sh_gu_w"][:cfg.inter], ex["sh_gu_s"][:cfg.inter], ex["sh_gu_s2"][0]),
                              O.unpack_nvfp4(ex["sh_gu_w"][cfg.inter:], ex["sh_gu_s"][cfg.inter:], ex["sh_gu_s2"][1])]),
              O.unpack_nvfp4(ex["sh_dn_w"], ex["sh_dn_s"], ex["sh_dn_s2"][0]))
    ref = O.routed_tokens_activation_space(x.float().cpu().numpy(), ref_ids, ref_w, groups, cfg.hidden, cfg.inter, cfg.group_size, shared=shared)
    assert _rel_l2(y.float().cpu().numpy(), ref) <= LAYER_TOL


def test_block_fp8_shared_expert(golden):
    """The always-on expert in the stock 128 x 128 block-FP8 format: the dequantisation probe is bit-exact against the
    reference's `dequant_fp8_block`, the shared expert alone reproduces the reference's output on the golden bytes, and
    layers that carry it match the oracle in every regime."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer, _lib
    from conftest import load_golden

    g8 = load_golden("fp8_block_shared")
    h, i, n_tok = (int(v) for v in g8["meta"])
    for name in ("gate_proj", "down_proj"):
        w, s_inv = torch.from_numpy(g8[f"{name}.weight"]).cuda(), torch.from_numpy(g8[f"{name}.weight_scale_inv"]).cuda()
        out = torch.empty(w.shape, dtype=torch.float32, device="cuda")
        _lib.check(_lib.lib().chronos_b200_dequant_fp8_block(w.data_ptr(), s_inv.data_ptr(), out.data_ptr(), w.shape[0], w.shape[1],
                                                            torch.cuda.current_stream().cuda_stream))
        assert np.array_equal(out.cpu().numpy().view(np.uint32), g8[f"ref.dequant.{name}"].view(np.uint32))
    if (int(golden["meta"][0]), int(golden["meta"][1])) == (h, i):  # the golden layer of the same dimensions hosts the shared expert
        shared = {f"{p}.{sfx}": g8[f"{p}.{sfx}"] for p in ("gate_proj", "up_proj", "down_proj") for sfx in ("weight", "weight_scale_inv")}
        packed = PackedLayer.from_groups(_cfg(golden["meta"]), golden_groups(golden), golden["router_w"], shared=shared, device="cuda")
        layer = FoldedMoELayer(packed=packed, register=False)
        x = torch.from_numpy(g8["x"]).cuda()
        none = torch.full((n_tok, layer.top_k), -1, dtype=torch.int32, device="cuda")
        y = layer.routed_forward(x, none, torch.zeros_like(none, dtype=torch.float32), with_shared=True)
        assert _rel_l2(y.cpu().numpy(), g8["ref.shared_y"]) <= 2e-3
    cfg = FoldedLayerConfig(hidden=512, inter=256, n_experts=16, group_size=4, rank=16, top_k=4)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=51, with_shared=True, shared_format="fp8", keep_disk_order=True), register=False)
    gen = torch.Generator(device="cuda").manual_seed(6)
    for n, regime in ((5, "auto"), (40, "stream"), (300, "auto"), (300, "tensor")):
        x = torch.randn(n, cfg.hidden, generator=gen, device="cuda").to(torch.bfloat16)
        y = layer.forward_impl(x, regime=regime)
        assert layer.device_status() == 0
        ref, _, _ = _oracle_layer(layer, x.float().cpu().numpy())
        ref0, _, _ = _oracle_layer(layer, x.float().cpu().numpy(), with_shared=False)
        assert _rel_l2(ref0, ref) > 5e-2, "the shared expert must matter"
        assert _rel_l2(y.float().cpu().numpy(), ref) <= LAYER_TOL, (n, regime)


def test_bounded_wait_gives_up_and_reports():
    """A wait that can never complete runs out after its poll limit, raises its status bit and lets the kernel return:
    no fault, no hang, and the context keeps working (the next launch below runs normally)."""
    from chronos_b200 import _lib

    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check(_lib.lib().chronos_b200_wait_probe(status.data_ptr(), 64, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(status.item()) == 0x200
    assert _lib.lib().chronos_b200_wait_probe(status.data_ptr(), 0, None) == -5
    assert float(torch.ones(8, device="cuda").sum().item()) == 8.0


def test_router_with_long_rows_matches_oracle():
    """hidden 16384 in fp32: the rows do not fit the shared-memory staging of the small-batch router kernel, the
    register-tile kernel takes over with the same bits."""
    from chronos_b200 import FoldedLayerConfig, _lib
    from chronos_b200.layout import ROUTER_KINDS

    h, e, k, n = 16384, 16, 4, 5
    gen = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(n, h, generator=gen, device="cuda")
    wr = torch.randn(e, h, generator=gen, device="cuda") * 0.02
    s = _lib.LayerStruct()
    s.hidden, s.n_experts, s.top_k, s.router_kind, s.router_w = h, e, k, ROUTER_KINDS["softmax"], wr.data_ptr()
    ids = torch.empty((n, k), dtype=torch.int32, device="cuda")
    gates = torch.empty((n, k), dtype=torch.float32, device="cuda")
    logits = torch.empty((n, e), dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib().chronos_b200_router_topk(s, x.data_ptr(), 0, n, ids.data_ptr(), gates.data_ptr(), logits.data_ptr(),
                                                  torch.cuda.current_stream().cuda_stream))
    fixed = O.router_logits_fixed(x.cpu().numpy(), wr.cpu().numpy())
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), fixed.view(np.uint32))
    assert np.array_equal(ids.cpu().numpy(), O.router_softmax_topk(fixed, k)[0])


def test_residual_rmsnorm_matches_oracle():
    from chronos_b200 import residual_rmsnorm

    gen = torch.Generator(device="cuda").manual_seed(0)
    h = torch.randn(5, 1024, generator=gen, device="cuda")
    y = torch.randn(5, 1024, generator=gen, device="cuda")
    ref_h = (h + y).cpu().numpy()
    out = residual_rmsnorm(h, y, None, 1e-6)
    assert np.allclose(h.cpu().numpy(), ref_h)
    assert np.allclose(out.cpu().numpy(), O.rms_norm(ref_h, 1e-6), rtol=2e-5, atol=1e-6)


def test_custom_op_equals_direct_call(golden):
    from chronos_b200 import vllm_plugin as VP

    layer = _golden_layer(golden, register=True)
    VP.register_custom_op()
    x = torch.from_numpy(golden["x"]).cuda()
    assert torch.equal(torch.ops.chronos_b200.moe_forward(x, 0), layer.forward_impl(x))


def test_hooked_vllm_class_with_a_shard_on_disk(golden, tmp_path, monkeypatch):
    """Stub `vllm` import site + a checkpoint folder holding config.json and one converter-format layer shard: the hooked
    class builds the folded layer from the shard, `forward` goes through the operator (both names), equals the direct
    call and the reference's layer output, and compiles with fullgraph=True."""
    import json
    import sys
    import types

    from safetensors.torch import save_file

    from chronos_b200 import vllm_plugin as VP

    h, i, e, k, r, top_k, _ = (int(v) for v in golden["meta"])
    l_idx = 4
    prefix = f"model.layers.{l_idx}.mlp"
    tensors = {}
    for g, grp in enumerate(golden_groups(golden)):
        for sfx, arr in grp.items():
            t = torch.from_numpy(np.ascontiguousarray(arr))
            if sfx.endswith("_scale") or sfx.startswith("healer."):
                t = t.view(torch.float8_e4m3fn)
            tensors[f"{prefix}.chronos_groups.{g}.{sfx}"] = t
    tensors[f"{prefix}.gate.weight"] = torch.from_numpy(golden["router_w"])
    tensors[f"{prefix}.gate.e_score_correction_bias"] = torch.from_numpy(golden["e_bias"])
    save_file(tensors, str(tmp_path / f"chronos-glm53-layer-{l_idx:05d}-of-00008.safetensors"))
    (tmp_path / "config.json").write_text(json.dumps({
        "hidden_size": h, "moe_intermediate_size": i, "n_routed_experts": e, "num_experts_per_tok": top_k, "scoring_func": "sigmoid",
        "routed_scaling_factor": 2.5, "norm_topk_prob": True,
        "chronos_holographic_moe": {"group_size": k, "svd_rank": r, "key_generator": "torch_cpu_v1"}}))

    class StockMoE(torch.nn.Module):
        def __init__(self, *a, **kw):
            super().__init__()

    dsv2 = types.ModuleType("vllm.model_executor.models.deepseek_v2")
    dsv2.DeepseekV2MoE = StockMoE
    for name, mod in (("vllm", types.ModuleType("vllm")), ("vllm.model_executor", types.ModuleType("vllm.model_executor")),
                      ("vllm.model_executor.models", types.ModuleType("vllm.model_executor.models")),
                      ("vllm.model_executor.models.deepseek_v2", dsv2)):
        monkeypatch.setitem(sys.modules, name, mod)
    monkeypatch.setenv("CHRONOS_B200_CKPT", str(tmp_path))
    assert VP.enable_chronos_b200_vllm_hook() is True
    cls = dsv2.DeepseekV2MoE
    moe = cls(config=None, parallel_config=None, quant_config=None, reduce_results=False, prefix=prefix, apply_routed_scale_to_output=False)
    stock = cls(config=None, prefix="model.layers.0.mlp")  # no shard for layer 0: the stock class comes back
    assert isinstance(moe, cls) and type(stock) is StockMoE
    assert moe.load_weights(iter([("x", torch.zeros(1))])) == set()
    x = torch.from_numpy(golden["x"]).cuda()
    y_direct = moe.forward_impl(x)
    assert torch.equal(moe(x), y_direct)
    assert torch.equal(torch.ops.chronos_glm53.moe_forward(x, l_idx), y_direct)
    assert _rel_l2(y_direct.cpu().numpy(), golden["ref.layer_y.sigmoid"]) <= LAYER_TOL

    class Wrap(torch.nn.Module):
        def __init__(self, m):
            super().__init__()
            self.m = m

        def forward(self, hs):
            return self.m(hs) * 2.0

    yc = torch.compile(Wrap(moe), fullgraph=True, backend="eager")(x)
    assert torch.allclose(yc, 2 * y_direct)


def test_bad_arguments_raise(golden):
    from chronos_b200 import _lib

    layer = _golden_layer(golden)
    with pytest.raises(_lib.ChronosError):
        layer(torch.from_numpy(golden["x"]))  # CPU tensor
    ws = torch.empty(16, dtype=torch.uint8, device="cuda")
    x = torch.from_numpy(golden["x"]).cuda()
    y = torch.empty_like(x)
    rc = _lib.lib().chronos_b200_folded_moe_decode(layer.packed.ptr, x.data_ptr(), 0, x.shape[0], y.data_ptr(), 0,
                                                   ws.data_ptr(), ws.numel(), None)
    assert rc == -3 and b"workspace" in _lib.lib().chronos_b200_last_error()


@pytest.fixture(scope="module")
def decode_shaped_layer():
    """The benchmark's layer (hidden 4096, 288 + 1 experts, top-8, inter 1536, fold 4, rank 64) with seeded synthetic bytes."""
    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer
    from chronos_b200.workloads import DECODE

    layer = FoldedMoELayer(packed=PackedLayer.synthetic(FoldedLayerConfig(**DECODE), seed=2, with_shared=True), register=False)
    yield layer
    del layer
    torch.cuda.empty_cache()


def _sampled_parity(layer, x, y, ids, w, sample):
    """rel-L2 of sampled output rows against the activation-space oracle (explicit routing + shared expert)."""
    c = layer.cfg
    groups, ex = layer.packed.to_groups_numpy()
    i = c.inter
    shared = (np.concatenate([O.unpack_nvfp4(ex["sh_gu_w"][:i], ex["sh_gu_s"][:i], ex["sh_gu_s2"][0]),
                              O.unpack_nvfp4(ex["sh_gu_w"][i:], ex["sh_gu_s"][i:], ex["sh_gu_s2"][1])]),
              O.unpack_nvfp4(ex["sh_dn_w"], ex["sh_dn_s"], ex["sh_dn_s2"][0]))
    sel = torch.as_tensor(sample, device=x.device)
    ref = O.routed_tokens_activation_space(x[sel].float().cpu().numpy(), ids[sel].cpu().numpy(), w[sel].cpu().numpy(), groups,
                                           c.hidden, c.inter, c.group_size, shared=shared)
    return _rel_l2(y[sel].float().cpu().numpy(), ref)


@pytest.mark.parametrize("n_tokens", [8192, 4096])
def test_prefill_shaped_layer_at_benchmark_size(decode_shaped_layer, n_tokens):
    """The prefill configuration at its own shape: 8192 (and 4096, the per-step batch of the 42-layer stack) bf16 tokens,
    router popularity Zipf(1.1) (one expert with thousands of pairs next to experts with one or none), through the
    auto regime and the forced FP4 tensor regime. A token's output depends only on its own routing, so a sample of
    tokens - including tokens of the most popular expert and of the least popular ones - is compared with the oracle."""
    from chronos_b200.workloads import zipf_prefill_batch

    layer = decode_shaped_layer
    cfg = layer.cfg
    x = zipf_prefill_batch(layer, n_tokens)
    ids, w = layer.route(x)
    ref_ids, _ = O.router_softmax_topk(O.router_logits_fixed(x[:64].float().cpu().numpy(), layer.packed.t["router_w"].cpu().numpy()), cfg.top_k)
    assert np.array_equal(ids[:64].cpu().numpy(), ref_ids)
    counts = torch.bincount(ids.reshape(-1).long(), minlength=cfg.n_experts)
    assert int(counts.max()) > n_tokens // 2 and int((counts <= 2).sum()) > 0, "the batch must be skewed, or the test proves nothing"
    hot, cold = int(counts.argmax()), [int(e) for e in torch.nonzero((counts > 0) & (counts <= 2)).flatten()[:6]]
    sample = torch.nonzero((ids == hot).any(dim=1)).flatten()[:10].tolist()
    for e in cold:
        sample += torch.nonzero((ids == e).any(dim=1)).flatten()[:1].tolist()
    gen = torch.Generator().manual_seed(n_tokens)
    sample += torch.randint(0, n_tokens, (32 - len(sample),), generator=gen).tolist()
    sample = sorted(set(sample))
    y_auto = layer.forward_impl(x, regime="auto")
    assert layer.device_status() == 0
    y_fp4 = layer.forward_impl(x, regime="tensor_fp4")
    assert layer.device_status() == 0
    assert torch.equal(y_auto, y_fp4), "the auto regime must pick the FP4 tensor regime for this batch"
    err = _sampled_parity(layer, x, y_fp4, ids, w, sample)
    print(f"prefill-shaped layer, {n_tokens} tokens: rel-L2 over {len(sample)} sampled tokens = {err:.3e}, hottest expert {int(counts.max())} pairs")
    assert err <= LAYER_TOL
