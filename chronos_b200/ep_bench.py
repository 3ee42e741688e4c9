"""Expert-parallel stack benchmark (driven by bench.py): 42 folded layers, experts sharded over the ranks,
4096 tokens per step split evenly over the ranks, residual + RMSNorm between layers."""
from __future__ import annotations

import os
import statistics

import torch
import torch.distributed as dist

from . import FoldedLayerConfig
from .ep import ExpertParallelMoE, ExpertParallelStack, block_capacity, build_local_layer
from .layout import PackedLayer


def layer_parity(cfg, lay, seed: int, x, y, ids, gates, dev, n_sample: int = 8) -> dict:
    """Layer output of the expert-parallel path against the CPU oracle for a sample of this rank's home tokens. The rank
    holds only its own slots, but every slot of the synthetic layer is drawn from a generator seeded by (layer seed,
    slot), so the slots the sampled tokens touch on OTHER ranks are regenerated here for the check."""
    import numpy as np

    from oracle import folded_moe_oracle as O  # checker only

    sel = torch.linspace(0, x.shape[0] - 1, n_sample).long().to(dev)
    ids_s, gates_s = ids[sel].cpu().numpy(), gates[sel].cpu().numpy()
    groups = {}
    for g in sorted({int(e) // cfg.group_size for e in ids_s.reshape(-1) if e >= 0}):
        one = PackedLayer.synthetic_sharded(cfg, seed, range(g, g + 1), dev, False)
        groups[g] = one.to_groups_numpy()[0][0]
        del one
    _, ex = lay.layer.packed.to_groups_numpy()
    i = cfg.inter
    shared = (np.concatenate([O.unpack_nvfp4(ex["sh_gu_w"][:i], ex["sh_gu_s"][:i], ex["sh_gu_s2"][0]),
                              O.unpack_nvfp4(ex["sh_gu_w"][i:], ex["sh_gu_s"][i:], ex["sh_gu_s2"][1])]),
              O.unpack_nvfp4(ex["sh_dn_w"], ex["sh_dn_s"], ex["sh_dn_s2"][0]))
    ref = O.routed_tokens_activation_space(x[sel].float().cpu().numpy(), ids_s, gates_s, groups, cfg.hidden, cfg.inter, cfg.group_size, shared=shared)
    got = y[sel].float().cpu().numpy()
    ref_ids, _ = O.router_softmax_topk(O.router_logits_fixed(x[sel].float().cpu().numpy(), ex["router_w"]), cfg.top_k)
    return {"rel_l2": float(np.linalg.norm(got - ref) / np.linalg.norm(ref)), "tokens": int(n_sample), "against": "oracle",
            "router_ids_equal": bool(np.array_equal(ids_s, ref_ids)), "layer": 0, "tolerance": 1e-2}


def run(args, n_layers: int, tokens: int, layer_kw: dict, sampler_cls=None) -> dict:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29531")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # NCCL's banner and warnings go to stderr: the bench prints exactly one JSON line on stdout
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        cfg = FoldedLayerConfig(**layer_kw)
        layers = [ExpertParallelMoE(build_local_layer(cfg, 3 + l, world, rank, dev, with_shared=True), cfg) for l in range(n_layers)]
        stack = ExpertParallelStack(layers)
        tl = tokens // world
        gen = torch.Generator(device=dev).manual_seed(3 + 1000 * rank)
        h0 = torch.randn(tl, cfg.hidden, generator=gen, device=dev).to(torch.bfloat16)
        K, W = args.steps, max(args.warmup, 3)
        sampler = sampler_cls(local) if (sampler_cls and rank == 0) else None
        st = torch.cuda.current_stream()
        h = h0.clone()
        for _ in range(W):
            h.copy_(h0)
            stack(h)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize()
        e0.record(st)
        for _ in range(K):
            h.copy_(h0)
            stack(h)
        e1.record(st)
        torch.cuda.synchronize()
        dist.barrier()
        ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        status = max(l.layer.device_status() for l in layers[-1:]) | layers[0].peer_status()  # incl. the exchange barriers' word
        overflow = stack.overflowed()  # a dispatch block too small for the routing would have dropped tokens: the run is void then
        from .ep import _PEER_EXCHANGES

        peer = any(ex is not None for ex in _PEER_EXCHANGES.values())
        # end to end: pinned host tokens -> device -> stack -> pinned host result
        host_in = h0.cpu().pin_memory()
        host_out = torch.empty_like(host_in).pin_memory()
        dist.barrier()
        torch.cuda.synchronize()
        e0.record(st)
        for _ in range(K):
            h.copy_(host_in, non_blocking=True)
            stack(h)
            host_out.copy_(h, non_blocking=True)
        e1.record(st)
        torch.cuda.synchronize()
        dist.barrier()
        ms_e2e = torch.tensor([e0.elapsed_time(e1)], device=dev)
        dist.all_reduce(ms_e2e, op=dist.ReduceOp.MAX)
        clocks = sampler.stop() if sampler else None
        # per-layer phase split on this rank (one extra untimed step with event pairs around the phases)
        for lay in layers:
            lay.phase_events = []
        h.copy_(h0)
        stack(h)
        torch.cuda.synchronize()
        phase_us: dict[str, float] = {}
        for lay in layers:
            for name, a, b in lay.phase_events:
                phase_us[name] = phase_us.get(name, 0.0) + 1e3 * a.elapsed_time(b) / n_layers
            lay.phase_events = None
        # bank passes of one layer on this rank (stage events inside the C ABI call) -> roofline of the dominant kernel
        import ctypes

        from . import _lib
        from .moe import residual_rmsnorm
        lay0 = layers[0]
        lay0.out_dtype = torch.float32  # the parity record compares the fp32 sums, not the stack's bf16 rounding of them
        x0 = residual_rmsnorm(h0.clone(), None, None, 1e-6)  # what layer 0 sees in the stack
        ids0, gates0 = lay0.route_fn(x0)
        ids_all = torch.empty((world * tl, cfg.top_k), dtype=ids0.dtype, device=dev)
        dist.all_gather_into_tensor(ids_all, ids0.contiguous())
        owned = int(((ids_all >= lay0.first_expert) & (ids_all < lay0.first_expert + lay0.n_local)).sum().item())
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
        for ev in evs:
            ev.record(st)
        torch.cuda.synchronize()
        arr = (ctypes.c_void_p * 8)(*[ev.cuda_event for ev in evs])
        _lib.check(_lib.lib().chronos_b200_set_stage_events(arr, 8))
        y0 = lay0(x0)
        _lib.check(_lib.lib().chronos_b200_set_stage_events(None, 0))
        torch.cuda.synchronize()
        gemm_ms = evs[3].elapsed_time(evs[4]) + evs[5].elapsed_time(evs[6])
        parity = layer_parity(cfg, lay0, 3, x0, y0, ids0, gates0, dev) if rank == 0 else None
        step_s = float(ms.item()) * 1e-3 / K
        pairs = tokens * cfg.top_k
        bank_flops = 2 * (2 * cfg.inter) * cfg.hidden + 2 * cfg.hidden * cfg.inter
        healer_flops = 2 * cfg.rank * (cfg.hidden + 2 * cfg.inter) + 2 * cfg.rank * (cfg.inter + cfg.hidden)
        useful = n_layers * (pairs * (bank_flops + healer_flops) + tokens * bank_flops)
        # this library's kernels per layer: rmsnorm; router (logits, token scales, top-k); dispatch (plan + rows, and the
        # barrier with peer stores), metadata unpack; one pass over the received rows + home tokens (token scales, plan +
        # scatter, fp16 rows, input transform, healer in + operand tile, bank pass, SwiGLU / transform, healer in + operand
        # tile, bank pass, gather-sum: 14); combine (send back + barrier with peer stores, sum)
        exchange = 0 if world == 1 else ((3 + 1 + 3) if peer else (2 + 1 + 1))
        launches_per_layer = 1 + 3 + exchange + 14
        return {
            "metric": "folded_moe_ep_stack_tokens_per_s", "value": tokens / step_s, "unit": "tokens/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": float(ms.item()) / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "e2m1 x ue4m3 block-scaled tensor-core operands (activations as 3 residual FP4 terms), fp32 accumulate", "data": "synthetic",
            "config": {"workload": "ep_stack", "layers": n_layers, "tokens_per_step": tokens, "hidden": cfg.hidden,
                       "routed_experts": cfg.n_experts, "experts_per_gpu": cfg.n_experts // world, "shared_experts": 1,
                       "top_k": cfg.top_k, "inter": cfg.inter, "fold_factor": cfg.group_size, "healer_rank": cfg.rank,
                       "parallelism": f"ep{world}", "activations": "bf16", "rmsnorm_eps": 1e-6,
                       "l2_policy": f"each rank streams {n_layers * (cfg.n_slots // world) * cfg.bank_bytes_per_slot() / 1e9:.1f} GB of banks per step (> 126 MB L2)"},
            "e2e": {"value": tokens / (float(ms_e2e.item()) * 1e-3 / K), "unit": "tokens/s",
                    "h2d_bytes_per_step": tokens * cfg.hidden * 2, "d2h_bytes_per_step": tokens * cfg.hidden * 2},
            "gpu_launches": launches_per_layer * n_layers * K,
            "clocks": clocks,
            "useful_tflops": useful / step_s / 1e12,
            "roofline": {"bound": "tensor", "kernel": "bank_fp4_wide_kernel (both passes of one layer, rank 0)",
                         "achieved": (owned + tl) * bank_flops / (gemm_ms * 1e-3) / 1e12, "peak": 9000.0,
                         "peak_kind": "nominal dense FP4 (datasheet; not in MEASURED_PEAKS.json); the pipe issues 3x the useful FLOPs",
                         "unit": "TFLOP/s", "frac": (owned + tl) * bank_flops / (gemm_ms * 1e-3) / 1e12 / 9000.0, "traffic": None,
                         "pairs_on_rank0": owned + tl, "bank_pass_ms": gemm_ms},
            "phase_us_per_layer_rank0": {k_: round(v, 1) for k_, v in phase_us.items()},
            "dispatch": {"kind": ("none (one rank)" if world == 1 else
                                  ("deduplicated exchange by peer stores over NVLink, fixed-capacity blocks, two bounded barriers per layer"
                                   if peer else "deduplicated all-to-all, fixed-capacity blocks")),
                         "block_capacity_rows": block_capacity(tl, world, cfg.top_k), "tokens_per_rank": tl, "overflowed": overflow},
            "parity": parity,
            "device_status": status,
        }
    finally:
        dist.destroy_process_group()
