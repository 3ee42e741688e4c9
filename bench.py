#!/usr/bin/env python3
"""Benchmark of the folded-expert MoE forward on B200.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload decode|ep_stack]

One JSON line on stdout (rank 0). A step = one forward of the workload over one batch of seeded synthetic input.

N = 1 (default) workload "decode": the decode-shaped layer (hidden 4096, 288 routed experts + 1 shared, top-8,
SwiGLU inter 1536, fold factor 4, healer rank 64, NVFP4 banks; 4 streams x 3 speculative tokens, bf16).
N > 1 workload "ep_stack": the same layer stacked 42 deep with experts sharded over the ranks (all-to-all
dispatch / combine over NCCL, residual + RMSNorm between layers), 4096 tokens per step.

`value`     device-resident throughput (tokens/s), CUDA events over exactly K steps, max over ranks.
`e2e`       the same metric through the public module call with pinned-host inputs and outputs (copies timed).
`roofline`  the dominant kernel (gate_up bank pass) against measured HBM bandwidth.
`cpu_baseline` / `--impl reference`: the CPU oracle (a numpy port of the reference's PyTorch path) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

DECODE = dict(hidden=4096, inter=1536, n_experts=288, group_size=4, rank=64, top_k=8)
DECODE_STREAMS, TOKENS_PER_STREAM = 4, 3
N_BATCHES = 8             # distinct routed batches the timed loop rotates through
STREAM_CORR = 0.67        # shared share of variance of a stream's tokens -> ~30 % top-8 overlap at 288 experts
EP_LAYERS, EP_TOKENS = 42, 4096
FALLBACK_HBM_GBS = 6650.0
# dram__bytes_read.sum + dram__bytes_write.sum of one gate_up launch of bank_fp4_kernel from the ncu capture summarised
# under profiles/ (bank_fp4_kernel, decode layer): 314.98 MB + 4.02 MB for a forward over 44 banks (311.43 MB algorithmic).
# Traffic grows in proportion to the banks a launch streams, so the line reports this ratio times the launch's bytes.
GU_PASS_TRAFFIC_OVER_ALGORITHMIC = (314.98 + 4.02) / 311.43


def _peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (OSError, ValueError, KeyError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """Samples SM clock and throttle reasons with nvidia-smi while the measurement loops run."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.rows: list[list[str]] = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=2)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm = [float(r[0]) for r in self.rows if len(r) >= 7 and r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if len(r) >= 7 and r[1].replace(".", "").isdigit()]
        reasons = []
        for i, name in ((3, "hw_slowdown"), (4, "hw_thermal_slowdown"), (5, "sw_thermal_slowdown"), (6, "sw_power_cap")):
            if any(len(r) >= 7 and r[i].lower().startswith("active") for r in self.rows):
                reasons.append(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


# ---------------------------------------------------------------------------------------------------------------
def decode_batches(cfg, streams: int, device, seed: int = 1):
    """N_BATCHES seeded activation batches [streams*3, H] bf16: the 3 tokens of a stream share a common component
    (correlation 0.67 of their router logits), which makes their top-8 sets overlap by about 30 % (the realised
    overlap is reported)."""
    import torch

    gen = torch.Generator(device=device).manual_seed(seed)
    out = []
    for _ in range(N_BATCHES):
        base = torch.randn(streams, 1, cfg.hidden, generator=gen, device=device)
        eps = torch.randn(streams, TOKENS_PER_STREAM, cfg.hidden, generator=gen, device=device)
        out.append((STREAM_CORR ** 0.5 * base + (1.0 - STREAM_CORR) ** 0.5 * eps).reshape(-1, cfg.hidden).to(torch.bfloat16).contiguous())
    return out


def routing_stats(layer, batches, streams: int):
    """Per batch: distinct slots / experts touched and the algorithmic HBM bytes of one forward."""
    cfg = layer.cfg
    stats = []
    for x in batches:
        ids = layer.route(x)[0].cpu().numpy()
        slots = {int(e) // cfg.group_size for e in ids.reshape(-1)}
        experts = {int(e) for e in ids.reshape(-1)}
        ov = []
        for s in range(streams):
            blk = ids[s * TOKENS_PER_STREAM:(s + 1) * TOKENS_PER_STREAM]
            for a in range(TOKENS_PER_STREAM):
                for b in range(a + 1, TOKENS_PER_STREAM):
                    ov.append(len(set(blk[a]) & set(blk[b])) / cfg.top_k)
        h, i = cfg.hidden, cfg.inter
        gu_bank = 2 * i * h // 2 + 2 * i * h // 16
        dn_bank = h * i // 2 + h * i // 16
        n_sh = 1 if layer.n_shared_experts else 0
        stats.append({
            "slots": len(slots), "experts": len(experts), "overlap": sum(ov) / max(len(ov), 1),
            "gu_pass_bytes": (len(slots) + n_sh) * gu_bank, "dn_pass_bytes": (len(slots) + n_sh) * dn_bank,
            "layer_bytes": (len(slots) + n_sh) * (gu_bank + dn_bank) + len(experts) * cfg.healer_bytes_per_expert()
                           + 2 * x.shape[0] * h * 2,
        })
    return stats


def cpu_oracle_tokens_per_s(layer, x_sample, threads: int) -> tuple[float, float]:
    """Times the CPU oracle (numpy port of the reference path) on a token sample; returns (tokens/s, seconds)."""
    import numpy as np

    from oracle import folded_moe_oracle as O  # CPU-baseline leg only

    O.set_threads(threads)
    groups, ex = layer.packed.to_groups_numpy()
    cfg = layer.cfg
    shared = None
    if "sh_gu_w" in ex:
        i = cfg.inter
        shared = (np.concatenate([O.unpack_nvfp4(ex["sh_gu_w"][:i], ex["sh_gu_s"][:i], ex["sh_gu_s2"][0]),
                                  O.unpack_nvfp4(ex["sh_gu_w"][i:], ex["sh_gu_s"][i:], ex["sh_gu_s2"][1])]),
                  O.unpack_nvfp4(ex["sh_dn_w"], ex["sh_dn_s"], ex["sh_dn_s2"][0]))
    xs = x_sample.float().cpu().numpy()
    t0 = time.perf_counter()
    O.moe_layer_forward(xs, groups, ex["router_w"], cfg.top_k, cfg.hidden, cfg.inter, cfg.group_size, router=cfg.router,
                        e_bias=ex.get("e_bias"), shared=shared)
    dt = time.perf_counter() - t0
    return xs.shape[0] / dt, dt


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------------------------------------------
def run_decode(args) -> dict:
    import ctypes

    import torch

    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer, _lib
    from chronos_b200 import build as cuda_build

    cuda_build.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = FoldedLayerConfig(**DECODE)
    tail = (args.tail, args.tail) if args.tail else (0, 0)  # optional tail lattice (next-row feature): same codes width for both products
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=1, device=dev, with_shared=True, tail_bits=tail), register=False)
    streams = args.streams
    batches = decode_batches(cfg, streams, dev)
    n_tok = batches[0].shape[0]
    stats = routing_stats(layer, batches, streams)
    K, W = args.steps, max(args.warmup, 3)
    st = torch.cuda.current_stream()

    sampler = ClockSampler(0)
    for i in range(W):
        layer(batches[i % N_BATCHES])
    torch.cuda.synchronize()
    # ---- device-resident throughput: exactly K steps between two events -----------------------------------------
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    for i in range(K):
        layer(batches[i % N_BATCHES])
    e1.record(st)
    torch.cuda.synchronize()
    ms_total = e0.elapsed_time(e1)
    assert layer.device_status() == 0, "device status word raised during the timed loop"

    # ---- per-stage durations (same steps, events at the stage boundaries inside the C ABI call) ------------------
    n_ev = 8
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n_ev)] for _ in range(K)]
    for row in evs:
        for ev in row:
            ev.record(st)  # forces creation of the underlying handle
    torch.cuda.synchronize()
    arr_t = ctypes.c_void_p * n_ev
    for i in range(K):
        arr = arr_t(*[ev.cuda_event for ev in evs[i]])
        _lib.check(_lib.lib().chronos_b200_set_stage_events(arr, n_ev))
        layer(batches[i % N_BATCHES])
    _lib.check(_lib.lib().chronos_b200_set_stage_events(None, 0))
    torch.cuda.synchronize()
    names = ("router", "plan", "gu_input", "gu_bank_pass", "swiglu_dn_input", "dn_bank_pass", "combine")
    fp4 = bool(layer.packed.struct.gu_t)  # the layer carries re-tiled banks: the auto regime streams them through FP4 MMA
    bank_kernel = "bank_fp4_kernel" if fp4 else "bank_stream_kernel"
    stage_us = {nm: 1e3 * statistics.mean(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(K)) for j, nm in enumerate(names)}
    gu_bytes = statistics.mean(stats[i % N_BATCHES]["gu_pass_bytes"] for i in range(K))
    dn_bytes = statistics.mean(stats[i % N_BATCHES]["dn_pass_bytes"] for i in range(K))
    layer_bytes = statistics.mean(stats[i % N_BATCHES]["layer_bytes"] for i in range(K))
    if args.tail:  # per distinct expert: codes + e4m3 block scales of the gate_up and down tail matrices
        blk = 32 if args.tail == 2 else 64
        tail_per_expert = 3 * cfg.hidden * cfg.inter * args.tail // 8 + 3 * cfg.hidden * cfg.inter // blk
        layer_bytes += statistics.mean(stats[i % N_BATCHES]["experts"] for i in range(K)) * tail_per_expert

    # ---- end to end: pinned host input -> device -> forward -> pinned host output, copies inside the timed region --
    host_in = [b.cpu().pin_memory() for b in batches]
    host_out = torch.empty_like(host_in[0]).pin_memory()
    dev_in = torch.empty_like(batches[0])
    for i in range(W):
        dev_in.copy_(host_in[i % N_BATCHES], non_blocking=True)
        host_out.copy_(layer(dev_in), non_blocking=True)
    torch.cuda.synchronize()
    e0.record(st)
    for i in range(K):
        dev_in.copy_(host_in[i % N_BATCHES], non_blocking=True)
        host_out.copy_(layer(dev_in), non_blocking=True)
    e1.record(st)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1)
    clocks = sampler.stop()

    peak, peak_kind = _peaks()
    gu_gbs = gu_bytes / (stage_us["gu_bank_pass"] * 1e-6) / 1e9
    dn_gbs = dn_bytes / (stage_us["dn_bank_pass"] * 1e-6) / 1e9
    step_s = ms_total * 1e-3 / K
    out = {
        "metric": "folded_moe_decode_tokens_per_s", "value": n_tok / step_s, "unit": "tokens/s", "n_gpus": 1,
        "steps": K, "warmup": W, "ms_per_step": ms_total / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": ("e2m1 x ue4m3 block-scaled FP4 MMA (banks as stored; activations as 3 residual e2m1 terms), fp32 accumulate" if fp4
                  else "f16 (NVFP4 e2m1 x e4m3 weights exact in f16; fp32 accumulate)"), "data": "synthetic",
        "config": {"workload": "decode_layer", "regime": "stream_fp4" if fp4 else "stream", "hidden": cfg.hidden, "routed_experts": cfg.n_experts, "shared_experts": 1,
                   "top_k": cfg.top_k, "inter": cfg.inter, "fold_factor": cfg.group_size, "healer_rank": cfg.rank,
                   "streams": streams, "tokens_per_stream": TOKENS_PER_STREAM, "activations": "bf16", "router": cfg.router,
                   "l2_policy": f"each step streams {layer_bytes / 1e6:.0f} MB of banks (> 126 MB L2) and batches rotate over {N_BATCHES} routings",
                   "tail_lattice_bits": args.tail,
                   "distinct_slots_per_step": statistics.mean(s["slots"] for s in stats),
                   "distinct_slots_by_routing": [s["slots"] for s in stats],
                   "distinct_experts_per_step": statistics.mean(s["experts"] for s in stats),
                   "top8_overlap_within_stream": round(statistics.mean(s["overlap"] for s in stats), 3)},
        "e2e": {"value": n_tok / (ms_e2e * 1e-3 / K), "unit": "tokens/s", "h2d_bytes_per_step": n_tok * cfg.hidden * 2,
                "d2h_bytes_per_step": n_tok * cfg.hidden * 2},
        "gpu_launches": (8 + (2 if args.tail else 0) + (1 if args.tail else 0)) * K,  # router, plan(+top-k), input transform, 2 bank passes, SwiGLU, down transform, combine (+ fp16 image, 2 tail passes)
        "clocks": clocks,
        "roofline": {"bound": "hbm", "kernel": f"{bank_kernel} (gate_up pass)", "achieved": gu_gbs, "peak": peak,
                     "peak_kind": f"of {peak_kind}", "unit": "GB/s", "frac": gu_gbs / peak,
                     "traffic": GU_PASS_TRAFFIC_OVER_ALGORITHMIC * gu_bytes, "algorithmic_bytes_per_launch": gu_bytes},
        "layer_hbm": {"algorithmic_bytes_per_step": layer_bytes, "achieved_gbs": layer_bytes / step_s / 1e9,
                      "frac_of_peak": layer_bytes / step_s / 1e9 / peak, "frac_of_8tbs": layer_bytes / step_s / 8e12},
        "stages_us": {k: round(v, 2) for k, v in stage_us.items()},
        "dn_bank_pass_gbs": dn_gbs,
    }
    if not args.no_cpu_baseline:
        threads = host_threads()
        tps, secs = cpu_oracle_tokens_per_s(layer, batches[0][:TOKENS_PER_STREAM], threads)
        out["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
                               "sample": f"one stream ({TOKENS_PER_STREAM} tokens) of batch 0, one pass, {secs:.1f} s"}
    return out


def run_prefill(args) -> dict:
    """Prefill-shaped layer (config index 3): the decode layer's shapes, 8192 tokens bf16, router biased so that
    expert popularity follows Zipf(1.1). Reports tokens/s and useful TFLOP/s of the tensor regime."""
    import numpy as np
    import torch

    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer
    from chronos_b200 import build as cuda_build

    cuda_build.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ceiling = args.workload == "fp4_ceiling"
    # fp4_ceiling: the same kernels on ONE slot (4 experts, every token routed to all 4): banks and activation images
    # stay in L2, work items are all full - an empirical ceiling for this tile shape, not a workload of the reference
    cfg = FoldedLayerConfig(**{**DECODE, **({"n_experts": 4, "top_k": 4} if ceiling else {})})
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=2, device=dev, with_shared=not ceiling), register=False)
    n_tok = args.tokens
    regime = args.regime or "tensor_fp4"
    gen = torch.Generator(device=dev).manual_seed(2)
    x = torch.randn(n_tok, cfg.hidden, generator=gen, device=dev).to(torch.bfloat16)
    # Zipf(1.1) popularity over a seeded permutation of experts: add c * log p_e to the logits by shifting the router
    # rows along the mean activation direction is not possible for N(0,1) inputs, so the bias is injected through one
    # extra input channel: x[:, 0] = 1 and router_w[:, 0] = c * log p_e.
    perm = torch.randperm(cfg.n_experts, generator=torch.Generator().manual_seed(2))
    p_e = (torch.arange(1, cfg.n_experts + 1, dtype=torch.float64) ** -1.1)
    p_e = (p_e / p_e.sum())[torch.argsort(perm)]
    if not ceiling:
        layer.packed.t["router_w"][:, 0] = (1.0 * torch.log(p_e)).to(torch.float32).to(dev)
        x[:, 0] = 1.0
    ids = layer.route(x)[0]
    counts = torch.bincount(ids.reshape(-1).long(), minlength=cfg.n_experts).cpu().numpy()
    K, W = max(args.steps // 20, 3), 3
    st = torch.cuda.current_stream()
    for _ in range(W):
        layer.forward_impl(x, regime=regime)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(K):
        layer.forward_impl(x, regime=regime)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / K
    assert layer.device_status() == 0
    import ctypes

    from chronos_b200 import _lib
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
    for ev in evs:
        ev.record(st)
    torch.cuda.synchronize()
    arr = (ctypes.c_void_p * 8)(*[ev.cuda_event for ev in evs])
    _lib.check(_lib.lib().chronos_b200_set_stage_events(arr, 8))
    layer.forward_impl(x, regime=regime)
    _lib.check(_lib.lib().chronos_b200_set_stage_events(None, 0))
    torch.cuda.synchronize()
    names = ("router", "plan", "gu_input", "gu_bank_pass", "swiglu_dn_input", "dn_bank_pass", "combine")
    stage_us = {nm: round(1e3 * evs[j].elapsed_time(evs[j + 1]), 1) for j, nm in enumerate(names)}
    pairs = n_tok * cfg.top_k
    bank_flops = 2 * (2 * cfg.inter) * cfg.hidden + 2 * cfg.hidden * cfg.inter
    healer_flops = 2 * cfg.rank * (cfg.hidden + 2 * cfg.inter) + 2 * cfg.rank * (cfg.inter + cfg.hidden)
    n_sh = 0 if ceiling else n_tok
    useful = pairs * (bank_flops + healer_flops) + n_sh * bank_flops
    gemm_flops = (pairs + n_sh) * bank_flops
    gemm_s = (stage_us["gu_bank_pass"] + stage_us["dn_bank_pass"]) * 1e-6
    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    bf16_peak = float(peaks.get("bf16_tflops", 1590.0))
    fp4 = regime == "tensor_fp4"
    achieved = gemm_flops / gemm_s / 1e12
    if fp4:
        # the block-scaled pass multiplies every bank tile by 3 residual FP4 terms of the activations: the pipe does 3x the
        # useful FLOPs; no FP4 figure is in MEASURED_PEAKS.json, so the denominator is the datasheet dense FP4 rate
        roof = {"bound": "tensor", "kernel": "bank_fp4_wide_kernel (both passes)", "achieved": achieved, "peak": 9000.0,
                "peak_kind": "nominal dense FP4 (datasheet; not in MEASURED_PEAKS.json)", "unit": "TFLOP/s", "frac": achieved / 9000.0,
                "mma_issue_tflops": 3 * achieved, "mma_issue_frac": 3 * achieved / 9000.0,
                "achieved_vs_measured_bf16": achieved / bf16_peak, "traffic": None}
        dtype = "e2m1 x ue4m3 block-scaled operands (banks as stored, activations as 3 residual FP4 terms), fp32 accumulate in TMEM"
    else:
        roof = {"bound": "tensor", "kernel": "bank_gemm_kernel (both passes)", "achieved": achieved, "peak": bf16_peak,
                "peak_kind": "of measured bf16 (operands are f16)", "unit": "TFLOP/s", "frac": achieved / bf16_peak, "traffic": None}
        dtype = "f16 operands (NVFP4 banks converted exactly), fp32 accumulate in TMEM"
    return {
        "metric": "folded_moe_prefill_tokens_per_s", "value": n_tok / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": K,
        "warmup": W, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": dtype, "data": "synthetic",
        "config": {"workload": "fp4_ceiling_one_slot" if ceiling else "prefill_layer", "regime": regime, "tokens": n_tok, "hidden": cfg.hidden, "routed_experts": cfg.n_experts,
                   "top_k": cfg.top_k, "inter": cfg.inter, "fold_factor": cfg.group_size, "healer_rank": cfg.rank,
                   "router_popularity": "all tokens to all 4 experts" if ceiling else "Zipf(1.1)", "pairs_per_expert_max": int(counts.max()), "pairs_per_expert_median": float(np.median(counts)),
                   "pairs_per_expert_min": int(counts.min())},
        "useful_tflops_layer": useful / (ms * 1e-3) / 1e12,
        "roofline": roof,
        "stages_us": stage_us,
    }


def run_sweep(args) -> dict:
    """Weight-reconstruction sweep (config index 1): 1..288 experts reconstructed-and-multiplied by a 1..16-token
    block, one pair per (token, expert); measures the streaming path's bytes/s against the HBM roofline."""
    import torch

    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer
    from chronos_b200 import build as cuda_build

    cuda_build.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = FoldedLayerConfig(**DECODE)
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=1, device=dev), register=False)
    peak, kind = _peaks()
    rows = []
    gen = torch.Generator(device=dev).manual_seed(1)
    st = torch.cuda.current_stream()
    for n_exp in (1, 4, 18, 72, 288):
        for n_tok in (1, 4, 16):
            # token t uses experts {(j * stride + t) % E}: n_exp distinct experts per token, spread over the slots
            per_tok = min(n_exp, cfg.top_k)
            if n_exp > cfg.top_k and n_tok * cfg.top_k < n_exp:
                continue  # cannot touch that many experts with this many (token, expert) pairs
            ids = torch.full((n_tok, cfg.top_k), -1, dtype=torch.int32, device=dev)
            e = 0
            for t in range(n_tok):
                for j in range(per_tok):
                    ids[t, j] = (e * (cfg.n_experts // n_exp)) % cfg.n_experts
                    e = (e + 1) % n_exp
            w = torch.rand((n_tok, cfg.top_k), generator=gen, device=dev)
            x = torch.randn(n_tok, cfg.hidden, generator=gen, device=dev).to(torch.bfloat16)
            used = ids[ids >= 0].unique().cpu().numpy()
            slots = len({int(v) // cfg.group_size for v in used})
            bytes_ = slots * cfg.bank_bytes_per_slot() + len(used) * cfg.healer_bytes_per_expert()
            for _ in range(5):
                layer.routed_forward(x, ids, w)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            reps = 30
            e0.record(st)
            for _ in range(reps):
                layer.routed_forward(x, ids, w)
            e1.record(st)
            torch.cuda.synchronize()
            us = 1e3 * e0.elapsed_time(e1) / reps
            rows.append({"experts": int(len(used)), "slots": slots, "tokens": n_tok, "pairs": int((ids >= 0).sum()), "us": round(us, 1),
                         "algorithmic_mb": round(bytes_ / 1e6, 1), "gbs": round(bytes_ / us / 1e3, 1), "frac_of_peak": round(bytes_ / us / 1e3 / peak, 3)})
    return {"metric": "folded_moe_reconstruction_sweep_gbs", "value": max(r["gbs"] for r in rows), "unit": "GB/s", "n_gpus": 1,
            "higher_is_better": True, "data": "synthetic", "config": {"workload": "reconstruction_sweep", "note": "banks of slots touched repeatedly stay in L2 for the small points"},
            "peak": peak, "peak_kind": f"of {kind}", "rows": rows}


def run_reference(args) -> dict:
    """The reference's algorithm on the host cores: the CPU oracle port, one token of the decode workload per step."""
    import torch

    from chronos_b200 import FoldedLayerConfig, PackedLayer

    cfg = FoldedLayerConfig(**DECODE)
    have_gpu = torch.cuda.is_available()
    dev = torch.device("cuda", 0) if have_gpu else torch.device("cpu")

    class _Holder:  # the packed bytes only; nothing of the CUDA path runs in this arm
        pass

    if have_gpu:
        packed = PackedLayer.synthetic(cfg, seed=1, device=dev, with_shared=True)
        batches = decode_batches(cfg, args.streams, dev)
    else:
        raise SystemExit(json.dumps({"impl": "reference", "unavailable": "needs the synthetic layer generator, which draws on a CUDA device"}))
    holder = _Holder()
    holder.packed, holder.cfg = packed, cfg
    threads = host_threads()
    K, W = args.steps, args.warmup
    times = []
    for i in range(W + K):
        x = batches[i % N_BATCHES][:1]
        tps, secs = cpu_oracle_tokens_per_s(holder, x, threads)
        if i >= W:
            times.append(secs)
        if sum(times) > 240:  # bounded: a few minutes at most
            break
    done = len(times)
    val = done / sum(times)
    return {
        "impl": "reference", "metric": "folded_moe_decode_tokens_per_s", "value": val, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": done, "warmup": W, "ms_per_step": 1e3 * sum(times) / done, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "decode_layer", "hidden": cfg.hidden, "routed_experts": cfg.n_experts, "shared_experts": 1,
                   "top_k": cfg.top_k, "inter": cfg.inter, "fold_factor": cfg.group_size, "healer_rank": cfg.rank,
                   "sample": "1 token per step (8 routed experts + shared), same packed bytes as the GPU arm"},
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{done} steps of 1 token each"},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


class _StdoutToStderr:
    """While active, file descriptor 1 points at stderr: libraries that print banners to stdout (NCCL does, depending on
    NCCL_DEBUG) cannot put a second line beside the one JSON line this program prints."""

    def __enter__(self):
        sys.stdout.flush()
        self._saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self._saved, 1)
        os.close(self._saved)
        return False


def ep_stack_single_gpu(args) -> dict:
    """The N > 1 workload (42-layer stack, 4096 tokens per step) on one GPU, 3 timed steps."""
    import argparse
    import gc

    import torch

    from chronos_b200 import ep_bench

    gc.collect()
    torch.cuda.empty_cache()
    small = argparse.Namespace(**{**vars(args), "steps": 3, "warmup": 3})
    res = ep_bench.run(small, args.layers, EP_TOKENS, DECODE, None)
    return {"metric": res["metric"], "value": res["value"], "unit": res["unit"], "ms_per_step": res["ms_per_step"],
            "steps": res["steps"], "config": {"workload": "ep_stack", "layers": args.layers, "tokens_per_step": EP_TOKENS}}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--workload", default=None, choices=(None, "decode", "ep_stack", "prefill", "sweep", "fp4_ceiling"))
    ap.add_argument("--tokens", type=int, default=8192, help="tokens of the prefill workload")
    ap.add_argument("--regime", default=None, choices=(None, "auto", "tensor", "tensor_fp4"), help="bank-pass regime of the prefill workload")
    ap.add_argument("--streams", type=int, default=DECODE_STREAMS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ep-base", action="store_true", help="skip the single-GPU run of the N > 1 workload appended to the default line")
    ap.add_argument("--tail", type=int, default=0, choices=(0, 1, 2), help="decode workload: add a tail lattice of this many bits per weight")
    ap.add_argument("--layers", type=int, default=EP_LAYERS, help="depth of the ep_stack workload")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return
    workload = args.workload or ("decode" if args.gpus == 1 and world == 1 else "ep_stack")
    if workload in ("decode", "prefill", "sweep", "fp4_ceiling"):
        if rank == 0:
            fn = {"decode": run_decode, "prefill": run_prefill, "sweep": run_sweep, "fp4_ceiling": run_prefill}[workload]
            out = fn(args)
            if workload == "decode" and args.workload is None and not args.no_ep_base:
                # the N > 1 lines run the expert-parallel stack (a different workload): give the N = 1 line the same
                # stack on one GPU, so that strong-scaling ratios can be formed from like quantities
                try:
                    with _StdoutToStderr():
                        out["ep_stack_1gpu"] = ep_stack_single_gpu(args)
                except Exception as exc:  # the headline line must not depend on this extra measurement
                    out["ep_stack_1gpu"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}
            print(json.dumps(out), flush=True)
        return
    from chronos_b200 import ep_bench

    with _StdoutToStderr():
        res = ep_bench.run(args, args.layers, EP_TOKENS, DECODE, ClockSampler)
    if rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
