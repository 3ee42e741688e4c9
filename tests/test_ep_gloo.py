"""Expert-parallel host logic on CPU ranks (gloo, world size 2): dispatch, ownership masking and combine must
reproduce the single-process oracle. The device compute is replaced by oracle-backed callables - this file tests
the exchange, not the kernels - and a rank that disagrees on the batch size is detected before any collective."""
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


def _worker(rank: int, world: int, port: int, ret):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from chronos_b200 import FoldedLayerConfig
        from chronos_b200.ep import ExpertParallelMoE, localize_routing, slot_range
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

        def compute_routed(x, local_ids, gates):  # only this rank's slots exist here
            y = np.zeros((x.shape[0], h), dtype=np.float32)
            ids, w, xn = local_ids.numpy(), gates.numpy(), x.numpy()
            for t, j in zip(*np.nonzero(ids >= 0)):
                ge = first + int(ids[t, j])
                gu, dn = O.reconstruct_expert(groups[ge // k], ge // k, ge % k, h, i)
                z = xn[t] @ gu.T
                y[t] += w[t, j] * ((O.silu(z[:i]) * z[i:]) @ dn.T)
            return torch.from_numpy(y)

        ep = ExpertParallelMoE(None, cfg, route_fn=route_fn, compute_routed=compute_routed, compute_shared=lambda x: None)
        y_local = ep(x_local).numpy()
        ref = O.moe_layer_forward(x_all, groups, gold["router_w"], top_k, h, i, k)[rank * tl:(rank + 1) * tl]
        err = float(np.linalg.norm(y_local - ref) / np.linalg.norm(ref))
        # ownership masking
        ids = torch.tensor([[0, 3, 4, 7]])
        loc = localize_routing(ids, first, len(slots) * k)
        want = [[0, 3, -1, -1]] if rank == 0 else [[-1, -1, 0, 3]]
        ret[rank] = (err, loc.tolist() == want)
    finally:
        dist.destroy_process_group()


def test_expert_parallel_exchange_matches_single_rank_oracle():
    world = 2
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, ret)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    for r in range(world):
        err, mask_ok = ret[r]
        assert err < 1e-5 and mask_ok, (r, err, mask_ok)


def test_slot_range_never_splits_a_slot():
    from chronos_b200.ep import slot_range

    assert [list(slot_range(72, 8, r))[0] for r in range(8)] == [0, 9, 18, 27, 36, 45, 54, 63]
    assert len(slot_range(72, 4, 3)) == 18
    with pytest.raises(ValueError):
        slot_range(72, 5, 0)
