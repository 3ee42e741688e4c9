"""Pins the CPU oracle against outputs of the reference's own code (fixtures made by golden/make_golden.py)."""
import numpy as np
import pytest

from conftest import golden_groups
from oracle import folded_moe_oracle as O


def test_e4m3_table_roundtrip():
    codes = np.arange(256, dtype=np.uint8)
    vals = O.e4m3_to_f32(codes)
    ok = ~np.isnan(vals)
    back = O.f32_to_e4m3(vals[ok])
    # -0 and +0 keep their sign bit; every finite code round-trips
    assert np.array_equal(back, codes[ok])
    assert vals[0x7E] == 448.0 and vals[0x01] == 2.0 ** -9


def test_dequant_bit_exact(golden):
    g0 = golden_groups(golden)[0]
    for tag, sfx in (("gu", "s_gu"), ("down", "s_down")):
        got = O.unpack_nvfp4(g0[f"{sfx}.weight"], g0[f"{sfx}.weight_scale"], g0[f"{sfx}.weight_scale_2"])
        ref = golden[f"ref.dequant_{tag}_g0"]
        assert got.dtype == np.float32
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), f"{tag}: fp32 bit patterns differ"


def test_pack_known_answer(golden):
    p, s, s2 = O.pack_nvfp4(golden["ref.pack.in"])
    assert np.array_equal(p, golden["ref.pack.packed"])
    assert np.array_equal(s, golden["ref.pack.scale"])
    assert np.float32(s2) == golden["ref.pack.scale2"]
    dq = O.unpack_nvfp4(p, s, s2)
    assert np.array_equal(dq.view(np.uint32), golden["ref.pack.dequant"].view(np.uint32))
    # the tiny block quantises to a zero scale code with saturated nibbles: signed zeros are legal values
    assert np.all(golden["ref.pack.scale"][3, 1] == 0) and np.all(dq[3, 16:32] == 0.0)


def test_keys_match_reference(golden):
    names = ("r_s1", "r_perm", "r_inv", "r_s2", "c_s1", "c_perm", "c_inv", "c_s2")
    h, i, e, k = (int(v) for v in golden["meta"][:4])
    seen = 0
    for key in golden:
        if not key.startswith("ref.keys.") or not key.endswith(".r_s1"):
            continue
        _, _, tag, gs, ms, _ = key.split(".")
        g, m = int(gs[1:]), int(ms[1:])
        rows, cols = (2 * i, h) if tag == "gu" else (h, i)
        sb = O.group_seed_bases(g)[0 if tag == "gu" else 1]
        keys = O.expert_keys(rows, cols, m, sb)
        for nm, arr in zip(names, keys):
            assert np.array_equal(arr.astype(np.int64), golden[f"ref.keys.{tag}.g{g}.m{m}.{nm}"].astype(np.int64)), (key, nm)
        seen += 1
    assert seen == 4


def test_fold_unbind_roundtrip():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((256, 128)).astype(np.float32)
    keys = O.expert_keys(256, 128, 2, 101)
    back = O.unbind_2d(O.fold_2d(w, keys), keys)
    assert np.abs(back - w).max() < 1e-5


def test_reconstruction_matches_reference(golden):
    h, i, e, k = (int(v) for v in golden["meta"][:4])
    groups = golden_groups(golden)
    seen = 0
    for key in golden:
        if not key.startswith("ref.recon_") or not key.endswith(".gu"):
            continue
        tg, gs, ms, _ = key[len("ref.recon_"):].split(".")
        g, m = int(gs[1:]), int(ms[1:])
        gu, dn = O.reconstruct_expert(groups[g], g, m, h, i, include_tail=(tg == "tail"))
        for got, ref in ((gu, golden[key]), (dn, golden[key[:-3] + ".down"])):
            # same fp32 expression; only the BLAS summation order inside the H_128 / U.V matmuls may differ
            assert np.abs(got - ref).max() <= 2e-6 * max(1.0, np.abs(ref).max()) + 1e-7
        seen += 1
    assert seen == 3


def test_activation_space_equals_weight_space(golden):
    h, i, e, k = (int(v) for v in golden["meta"][:4])
    groups = golden_groups(golden)
    x = golden["x"]
    g, m = len(groups) - 1, k - 1
    gu, dn = O.reconstruct_expert(groups[g], g, m, h, i)
    z = x @ gu.T
    y_w = (O.silu(z[:, :i]) * z[:, i:]) @ dn.T
    y_a = O.expert_forward_activation_space(x, groups[g], g, m, h, i)
    assert np.linalg.norm(y_a - y_w) <= 1e-5 * np.linalg.norm(y_w)


def test_router_matches_reference(golden):
    top_k = int(golden["meta"][5])
    for logits in (golden["ref.router.logits"], O.router_logits_fixed(golden["x"], golden["router_w"])):
        ids, gates = O.router_softmax_topk(logits, top_k)
        assert np.array_equal(ids, golden["ref.router.softmax_ids"])
        assert np.allclose(gates, golden["ref.router.softmax_gates"], rtol=1e-5, atol=1e-7)
        ids, gates = O.router_sigmoid_topk(logits, golden["e_bias"], top_k)
        assert np.array_equal(ids, golden["ref.router.sigmoid_ids"])
        assert np.allclose(gates, golden["ref.router.sigmoid_gates"], rtol=1e-5, atol=1e-7)
    assert np.abs(O.router_logits_fixed(golden["x"], golden["router_w"]) - golden["ref.router.logits"]).max() < 1e-5


def test_router_at_benchmark_shape_matches_reference():
    """288 experts x hidden 4096 x 512 tokens: ids of the three router flavours from the oracle's fixed-order logits
    against the reference's torch routers. Tokens whose k / k+1 scores are closer than the fp32 summation error are
    counted and reported apart from true mismatches (there must be none of the latter)."""
    from conftest import compare_router_ids, router_case, router_choice_scores

    gold, x, router_w, e_bias, k = router_case()
    fixed = O.router_logits_fixed(x, router_w)
    assert np.abs(fixed - gold["logits"]).max() < 4e-6
    for flavour, fn in (("softmax", lambda lg: O.router_softmax_topk(lg, k)),
                        ("sigmoid", lambda lg: O.router_sigmoid_topk(lg, e_bias, k)),
                        ("sqrt_softplus", lambda lg: O.router_sqrt_softplus_topk(lg, e_bias, k))):
        # on the reference's own logits the selection rule itself must agree everywhere
        ids, gates = fn(gold["logits"])
        rep = compare_router_ids(ids, gold[f"{flavour}_ids"], router_choice_scores(gold["logits"], flavour, e_bias), k)
        assert rep["true_mismatch_tokens"] == 0, (flavour, rep)
        same = (ids == gold[f"{flavour}_ids"]).all(axis=1)
        assert np.allclose(gates[same], gold[f"{flavour}_gates"][same], rtol=2e-5, atol=1e-7), flavour
        # on the fixed-order logits only near-tie tokens may differ
        ids, _ = fn(fixed)
        rep = compare_router_ids(ids, gold[f"{flavour}_ids"], router_choice_scores(gold["logits"], flavour, e_bias), k)
        print(flavour, rep)
        assert rep["true_mismatch_tokens"] == 0 and rep["near_tie_tokens"] <= rep["tokens"] // 50, (flavour, rep)


def test_topk_never_selects_nan_or_minus_inf():
    """A NaN row (NaN activations) or -inf choice scores: the positions that cannot be filled hold id -1 and gate 0,
    and the layer loop skips them."""
    lg = np.array([[0.3, np.nan, 0.1, -np.inf], [np.nan] * 4, [1.0, 2.0, 3.0, 4.0]], dtype=np.float32)
    ids, w = O.router_softmax_topk(lg, 3)
    assert ids.tolist() == [[0, 2, -1], [-1, -1, -1], [3, 2, 1]]
    assert w[1].tolist() == [0.0, 0.0, 0.0] and w[0, 2] == 0.0 and abs(w[0, :2].sum() - 1.0) < 1e-6
    ids, w = O.router_sigmoid_topk(lg, np.array([0.0, 0.0, -np.inf, 0.0], dtype=np.float32), 2)
    assert ids.tolist() == [[0, 3], [-1, -1], [3, 1]] and w[1].tolist() == [0.0, 0.0]
    ids, w = O.router_sqrt_softplus_topk(lg, None, 2)
    assert ids[1].tolist() == [-1, -1] and np.isfinite(w).all()


def test_router_fixed_order_is_the_stated_order():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 96)).astype(np.float32)
    w = rng.standard_normal((3, 96)).astype(np.float32)
    got = O.router_logits_fixed(x, w)
    for t in range(2):
        for e in range(3):
            p = np.zeros(32, dtype=np.float32)
            for l in range(32):
                # fma = exact product + single rounding: emulate in fp64 (exact for fp32 inputs)
                a32 = np.float32(0)
                for kk in (j + 4 * l + i for j in range(0, 96, 128) for i in range(4)):
                    if kk < 96:
                        a32 = np.float32(np.float64(x[t, kk]) * np.float64(w[e, kk]) + np.float64(a32))
                p[l] = a32
            for off in (16, 8, 4, 2, 1):
                p = (p + p[np.arange(32) ^ off]).astype(np.float32)
            assert got[t, e] == p[0]


def test_layer_output_matches_reference(golden):
    h, i, e, k, r, top_k, n_tok = (int(v) for v in golden["meta"])
    groups = golden_groups(golden)
    for tag in ("softmax", "sigmoid"):
        y = O.moe_layer_forward(golden["x"], groups, golden["router_w"], top_k, h, i, k, router=tag,
                                e_bias=golden["e_bias"], logits=golden["ref.router.logits"])
        ref = golden[f"ref.layer_y.{tag}"]
        assert np.linalg.norm(y - ref) <= 1e-5 * np.linalg.norm(ref)


def test_sampled_activation_space_oracle_equals_layer_oracle(golden):
    """The sampled-token checker used at full-size shapes (activation space, explicit routing) against the grouped
    dense layer loop on the fp32 reconstruction."""
    h, i, e, k, r, top_k, n_tok = (int(v) for v in golden["meta"])
    groups = golden_groups(golden)
    ref, ids, w = O.moe_layer_forward(golden["x"], groups, golden["router_w"], top_k, h, i, k, return_routing=True)
    got = O.routed_tokens_activation_space(golden["x"], ids, w, groups, h, i, k)
    assert np.linalg.norm(got - ref) <= 1e-5 * np.linalg.norm(ref)
    sub = [3, 1]
    got = O.routed_tokens_activation_space(golden["x"][sub], ids[sub], w[sub], groups, h, i, k)
    assert np.linalg.norm(got - ref[sub]) <= 1e-5 * np.linalg.norm(ref[sub])


@pytest.mark.parametrize("flavour", ["softmax", "sigmoid"])
def test_coalesced_routing_keeps_the_stated_invariants(flavour):
    """The batch-coalesced policy (clean-room: the reference describes it in prose only, so there is nothing to compare
    bytes with): the anchor of every stream is routed naturally, a draft never leaves its natural top-`pool` and keeps its
    `keep` best natural experts, pool == k or bonus == 0 give natural routing, and the step touches fewer distinct experts."""
    rng = np.random.default_rng(7)
    e, k, tps, n_streams = 288, 8, 3, 40
    base = rng.standard_normal((n_streams, 1, e)).astype(np.float32)
    logits = (0.8 * base + 0.6 * rng.standard_normal((n_streams, tps, e)).astype(np.float32)).reshape(-1, e)
    bias = (rng.standard_normal(e) * 0.05).astype(np.float32)
    nat_fn = (lambda lg, kk: O.router_softmax_topk(lg, kk)) if flavour == "softmax" else (lambda lg, kk: O.router_sigmoid_topk(lg, bias, kk))
    nat_ids, nat_w = nat_fn(logits, k)
    kw = dict(router=flavour, e_bias=bias if flavour != "softmax" else None)
    pool, keep = 12, 4
    ids, w = O.router_coalesced(logits, k, tps, pool, keep, 1.0e4, **kw)
    nat_pool, _ = nat_fn(logits, pool)
    for t in range(logits.shape[0]):
        assert len(set(ids[t])) == k
        if t % tps == 0:
            assert np.array_equal(ids[t], nat_ids[t]) and np.allclose(w[t], nat_w[t], rtol=1e-6)
        else:
            assert set(ids[t]) <= set(nat_pool[t]), "a draft left its natural candidate pool"
            assert np.array_equal(ids[t, :keep], nat_ids[t, :keep]), "a draft lost one of its best natural experts"
    for args in ((k, keep, 1.0e4), (pool, keep, 0.0)):  # no pool beyond k, or no bonus: natural routing
        i2, w2 = O.router_coalesced(logits, k, tps, args[0], args[1], args[2], **kw)
        assert np.array_equal(np.sort(i2, axis=1), np.sort(nat_ids, axis=1))
    per_stream = lambda a: np.mean([len(set(a[s * tps:(s + 1) * tps].reshape(-1))) for s in range(n_streams)])
    assert per_stream(ids) < per_stream(nat_ids) - 0.5, (per_stream(ids), per_stream(nat_ids))
    tot = w.sum(axis=1)
    assert np.allclose(tot, 1.0 if flavour == "softmax" else 2.5, rtol=1e-5)


def test_block_fp8_dequant_and_shared_expert_match_reference():
    """Stock 128 x 128 block-FP8 (the reference's shared-expert format): dequantisation bit-exact against
    `dequant_fp8_block`, the SwiGLU expert built from it against the reference's fp32 evaluation."""
    from conftest import load_golden

    gold = load_golden("fp8_block_shared")
    h, i, n_tok = (int(v) for v in gold["meta"])
    for name in ("gate_proj", "up_proj", "down_proj"):
        got = O.dequant_fp8_block(gold[f"{name}.weight"], gold[f"{name}.weight_scale_inv"])
        assert np.array_equal(got.view(np.uint32), gold[f"ref.dequant.{name}"].view(np.uint32)), name
    ex = {"sh8_gu_w": np.concatenate([gold["gate_proj.weight"], gold["up_proj.weight"]]),
          "sh8_gu_s": np.concatenate([gold["gate_proj.weight_scale_inv"], gold["up_proj.weight_scale_inv"]]),
          "sh8_dn_w": gold["down_proj.weight"], "sh8_dn_s": gold["down_proj.weight_scale_inv"]}
    gu, dn = O.shared_fp8_weights(ex)
    z = gold["x"] @ gu.T
    y = (O.silu(z[:, :i]) * z[:, i:]) @ dn.T
    assert np.linalg.norm(y - gold["ref.shared_y"]) <= 1e-5 * np.linalg.norm(gold["ref.shared_y"])


def test_synthetic_fold_is_valid_format():
    rng = np.random.default_rng(1)
    k, i, h, r = 4, 128, 256, 8
    gate, up = (rng.standard_normal((k, i, h)).astype(np.float32) * 0.02 for _ in range(2))
    down = rng.standard_normal((k, h, i)).astype(np.float32) * 0.02
    g = O.fold_group_synthetic(gate, up, down, 1, r)
    assert g["s_gu.weight"].shape == (2 * i, h // 2) and g["s_gu.weight_scale"].shape == (2 * i, h // 16)
    assert g["healer.u_down"].shape == (k, h, r) and g["healer.v_down"].shape == (k, r, i)
    gu, dn = O.reconstruct_expert(g, 1, 2, h, i)
    ref = np.concatenate([gate[2], up[2]], 0)
    cos = float((gu * ref).sum() / (np.linalg.norm(gu) * np.linalg.norm(ref)))
    assert cos > 0.4  # a K=4 fold keeps ~1/sqrt(K) of each expert before healing
