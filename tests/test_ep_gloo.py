"""Expert-parallel host logic on CPU ranks (gloo, world size 2): deduplicated dispatch, ownership, combine and the
geometry check must reproduce the single-process oracle. The device work is replaced by callables written here with the
same contracts as the CUDA entry points - this file tests the exchange, not the kernels - and a rank that disagrees on
the batch size is detected on every rank before any data collective."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT, golden_groups, load_golden

CASE = "k4_h256_i128"


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_callables(world, n_local, top_k, groups, first_expert, k_fold, h, i):
    """CPU stand-ins for chronos_b200_ep_pack / the expert pass / chronos_b200_ep_combine."""
    from oracle import folded_moe_oracle as O

    def pack_fn(x, ids, gates, capacity):
        tl = x.shape[0]
        rows = torch.zeros((world, capacity, x.shape[1]), dtype=x.dtype)
        meta = torch.zeros((world, capacity + 1, 2 * top_k + 2), dtype=torch.int32)
        slot_of = torch.full((tl, world), -1, dtype=torch.int32)
        for d in range(world):
            n = 0
            for t in range(tl):
                loc = ids[t] - d * n_local
                mine = (loc >= 0) & (loc < n_local)
                if not bool(mine.any()):
                    continue
                assert n < capacity, "test batches never overflow a block"
                rows[d, n] = x[t]
                meta[d, n, 0] = t
                meta[d, n, 1:1 + top_k] = torch.where(mine, loc, torch.full_like(loc, -1)).to(torch.int32)
                meta[d, n, 1 + top_k:1 + 2 * top_k] = torch.where(mine, gates[t], torch.zeros_like(gates[t])).view(torch.int32)
                slot_of[t, d] = n
                n += 1
            meta[d, capacity, 0] = n
        return rows, meta, slot_of

    def compute_fn(recv_rows, recv_meta, x_local, capacity, recv_all=None):
        out = torch.zeros_like(recv_rows)
        for s in range(world):
            for p in range(int(recv_meta[s, capacity, 0])):
                xr = recv_rows[s, p].numpy()
                for j in range(top_k):
                    e = int(recv_meta[s, p, 1 + j])
                    if e < 0:
                        continue
                    ge = first_expert + e
                    gu, dn = O.reconstruct_expert(groups[ge // k_fold], ge // k_fold, ge % k_fold, h, i)
                    z = xr @ gu.T
                    g = float(recv_meta[s, p, 1 + top_k + j:2 + top_k + j].view(torch.float32))
                    out[s, p] += torch.from_numpy(g * ((O.silu(z[:i]) * z[i:]) @ dn.T))
        return out, None

    def combine_fn(back, slot_of, shared_rows, capacity):
        y = torch.zeros((slot_of.shape[0], back.shape[2]), dtype=torch.float32)
        for t in range(slot_of.shape[0]):
            for d in range(world):
                if slot_of[t, d] >= 0:
                    y[t] += back[d, slot_of[t, d]].float()
        return y

    return pack_fn, compute_fn, combine_fn


def _worker(rank: int, world: int, port: int, ret, mismatch: bool):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from chronos_b200 import FoldedLayerConfig
        from chronos_b200.ep import EpConfigMismatch, ExpertParallelMoE, block_capacity, localize_routing, slot_range
        from oracle import folded_moe_oracle as O

        gold = load_golden(CASE)
        h, i, e, k, r, top_k, n_tok = (int(v) for v in gold["meta"])
        groups = golden_groups(gold)
        cfg = FoldedLayerConfig(hidden=h, inter=i, n_experts=e, group_size=k, rank=r, top_k=top_k)
        x_all = np.concatenate([gold["x"], gold["x"][::-1] * 0.5])[: 2 * (n_tok - 1)]  # 8 tokens, 4 per rank
        tl = x_all.shape[0] // world
        x_local = torch.from_numpy(np.ascontiguousarray(x_all[rank * tl:(rank + 1) * tl]))
        slots = slot_range(cfg.n_slots, world, rank)
        first = slots.start * k

        def route_fn(x):
            ids, w = O.router_softmax_topk(O.router_logits_fixed(x.numpy(), gold["router_w"]), top_k)
            return torch.from_numpy(ids), torch.from_numpy(w)

        pack_fn, compute_fn, combine_fn = make_callables(world, len(slots) * k, top_k, groups, first, k, h, i)
        ep = ExpertParallelMoE(None, cfg, route_fn=route_fn, pack_fn=pack_fn, compute_fn=compute_fn, combine_fn=combine_fn)
        if mismatch:
            # rank 1 arrives with one token fewer: both ranks must raise before any all-to-all is issued
            calls = []
            orig = dist.all_to_all_single
            dist.all_to_all_single = lambda *a, **kw: calls.append(1) or orig(*a, **kw)
            try:
                ep(x_local[: tl - 1] if rank == 1 else x_local)
                ret[rank] = ("no error", len(calls))
            except EpConfigMismatch as exc:
                ret[rank] = ("mismatch", len(calls), "rank 1" in str(exc))
            finally:
                dist.all_to_all_single = orig
            return
        y_local = ep(x_local).numpy()
        ref = O.moe_layer_forward(x_all, groups, gold["router_w"], top_k, h, i, k)[rank * tl:(rank + 1) * tl]
        err = float(np.linalg.norm(y_local - ref) / np.linalg.norm(ref))
        # ownership masking
        ids = torch.tensor([[0, 3, 4, 7]])
        loc = localize_routing(ids, first, len(slots) * k)
        want = [[0, 3, -1, -1]] if rank == 0 else [[-1, -1, 0, 3]]
        ret[rank] = (err, loc.tolist() == want, block_capacity(tl, world, top_k))
    finally:
        dist.destroy_process_group()


def _run(mismatch: bool):
    world = 2
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, ret, mismatch)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    return [ret[r] for r in range(world)]


def test_expert_parallel_exchange_matches_single_rank_oracle():
    for r, (err, mask_ok, cap) in enumerate(_run(False)):
        assert err < 1e-5 and mask_ok and cap == 8, (r, err, mask_ok, cap)  # blocks never shrink below 8 rows


def test_rank_with_a_different_batch_size_is_detected_before_any_exchange():
    for r, res in enumerate(_run(True)):
        assert res[0] == "mismatch" and res[1] == 0 and res[2], (r, res)


def test_slot_range_never_splits_a_slot():
    from chronos_b200.ep import slot_range

    assert [list(slot_range(72, 8, r))[0] for r in range(8)] == [0, 9, 18, 27, 36, 45, 54, 63]
    assert len(slot_range(72, 4, 3)) == 18
    with pytest.raises(ValueError):
        slot_range(72, 5, 0)


def test_block_capacity_bounds():
    from chronos_b200.ep import block_capacity

    assert block_capacity(512, 8, 8) == 416          # 65.6 % expected (336) + six sigma (65) + 8, rounded up to a multiple of 8
    assert block_capacity(2048, 2, 8) == 2048        # two ranks: nearly every token goes to both
    assert block_capacity(512, 8, 8, capacity_factor=1.0) == 512
    assert 8 <= block_capacity(3, 8, 8) <= 8
