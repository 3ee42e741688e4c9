#!/usr/bin/env python3
"""Benchmark of the folded-expert MoE forward on B200.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload decode|ep_stack|prefill|sweep]

One JSON line on stdout (rank 0). A step = one forward of the workload over one batch of seeded synthetic input.

Plain `python bench.py` (no launcher, N = 1), workload "decode": the decode-shaped layer (hidden 4096, 288 routed
experts + 1 shared, top-8, SwiGLU inter 1536, fold factor 4, healer rank 64, NVFP4 banks; 4 streams x 3 speculative
tokens, bf16). The line also carries a `prefill` sub-record (8192 tokens, Zipf(1.1) routing, FP4 tensor regime, with the
empirical FP4 ceiling of the same tile shapes measured in the same run) and an `ep_stack_1gpu` sub-record.
Under `torch.distributed.run` (any world size, 1 included), with `--gpus N > 1`, or with `--gpus 1` on a node that shows more
than one GPU (the first point of a 1-2-4-8 series; `--workload decode` overrides), workload "ep_stack": the same layer
stacked 42 deep with experts sharded over the ranks (all-to-all dispatch / combine over NCCL, residual + RMSNorm
between layers), 4096 tokens per step, strong scaling; at world size 1 the line carries the decode result as a
`decode_layer` sub-record, and every line carries `parity` (layer 0 of the stack against the CPU oracle on a sample of
rank 0's tokens; the run fails above 1e-2).

`value`     device-resident throughput (tokens/s), CUDA events over exactly K steps, max over ranks.
`e2e`       the same metric through the public module call with pinned-host inputs and outputs (copies timed).
`roofline`  the dominant kernel (gate_up bank pass) against measured HBM bandwidth.
`cpu_baseline` / `--impl reference`: the reference's own PyTorch code for this path (from oracle/_ref; the numpy port of it
when that folder is absent) on the host cores, same configuration, bounded number of steps.
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

from chronos_b200.workloads import DECODE, N_BATCHES, TOKENS_PER_STREAM, decode_batches  # noqa: E402  (no CUDA needed to import)

DECODE_STREAMS = 4
EP_LAYERS, EP_TOKENS = 42, 4096
PREFILL_TOKENS = 8192
FP4_NOMINAL_TFLOPS = 9000.0  # dense FP4 of a B200 (datasheet); MEASURED_PEAKS.json holds no FP4 figure
FALLBACK_HBM_GBS = 6650.0
REFERENCE_BUDGET_S = 150.0   # wall-clock bound of the reference arm's timed steps
# dram__bytes_read.sum + dram__bytes_write.sum of one gate_up launch of bank_fp4_kernel over its algorithmic bytes (bank
# images + the healer factors its side warps read), from the ncu capture summarised under profiles/ (bank_fp4_kernel,
# decode layer: 370.75 MB read + 5.23 MB written for 363.4 MB algorithmic). Traffic grows in proportion to the bytes a launch streams, so the line reports this ratio times them.
GU_PASS_TRAFFIC_OVER_ALGORITHMIC = 1.035


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
        h, i, r = cfg.hidden, cfg.inter, cfg.rank
        gu_bank = 2 * i * h // 2 + 2 * i * h // 16
        dn_bank = h * i // 2 + h * i // 16
        n_sh = 1 if layer.n_shared_experts else 0
        stats.append({
            "slots": len(slots), "experts": len(experts), "overlap": sum(ov) / max(len(ov), 1),
            # a bank pass streams the banks of the distinct slots (+ shared expert) and, in its side warps, the healer
            # factors of the distinct experts: V_gu [r, H] + U_gu [2I, r] (gate_up), V_down [r, I] + U_down [H, r] (down)
            "gu_pass_bytes": (len(slots) + n_sh) * gu_bank + len(experts) * r * (h + 2 * i),
            "dn_pass_bytes": (len(slots) + n_sh) * dn_bank + len(experts) * r * (i + h),
            "gu_bank_bytes": (len(slots) + n_sh) * gu_bank, "dn_bank_bytes": (len(slots) + n_sh) * dn_bank,
            "layer_bytes": (len(slots) + n_sh) * (gu_bank + dn_bank) + len(experts) * cfg.healer_bytes_per_expert()
                           + 2 * x.shape[0] * h * 2,
        })
    return stats


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def _shared_fp32(ex):
    """The plain-NVFP4 shared expert of a layer as fp32 (gate_up, down) via the numpy oracle."""
    import numpy as np

    from oracle import folded_moe_oracle as O  # checker / CPU-baseline leg only

    i = ex["sh_gu_w"].shape[0] // 2
    return (np.concatenate([O.unpack_nvfp4(ex["sh_gu_w"][:i], ex["sh_gu_s"][:i], ex["sh_gu_s2"][0]),
                            O.unpack_nvfp4(ex["sh_gu_w"][i:], ex["sh_gu_s"][i:], ex["sh_gu_s2"][1])]),
            O.unpack_nvfp4(ex["sh_dn_w"], ex["sh_dn_s"], ex["sh_dn_s2"][0]))


class CpuReference:
    """The reference's algorithm for one layer on the host cores: its own PyTorch code from oracle/_ref when present
    (kind "reference"), else the numpy port (kind "port"). Holds the layer's packed bytes, converts slots lazily."""

    def __init__(self, packed, threads: int):
        import torch

        from oracle import ref_torch  # CPU-baseline leg only

        self.cfg = packed.cfg
        self.threads = threads
        self.groups, self.ex = packed.to_groups_numpy()
        self.kind = "reference" if ref_torch.available() else "port"
        self._ref = ref_torch
        self._torch_groups: dict[int, dict] = {}
        torch.set_num_threads(threads)

    def _slots_of(self, x_f32):
        import numpy as np

        from oracle import folded_moe_oracle as O

        ids, _ = O.router_softmax_topk(O.router_logits_fixed(x_f32, self.ex["router_w"]), self.cfg.top_k)
        return sorted({int(e) // self.cfg.group_size for e in np.asarray(ids).reshape(-1)})

    def forward(self, x) -> tuple[float, int]:
        """Runs one forward over the token batch x (torch tensor, any device); returns (seconds, tokens)."""
        import torch

        c = self.cfg
        xs = x.float().cpu()
        if self.kind == "reference":
            for g in self._slots_of(xs.numpy()):  # conversion of the touched slots' bytes to tensors is not timed
                if g not in self._torch_groups:
                    self._torch_groups[g] = self._ref.group_to_torch(self.groups[g])
            shared = {k: torch.from_numpy(v) for k, v in self.ex.items() if k.startswith("sh_")} or None
            rw = torch.from_numpy(self.ex["router_w"])
            t0 = time.perf_counter()
            self._ref.layer_forward(xs, self._torch_groups, rw, c.top_k, c.hidden, c.inter, c.group_size, shared=shared)
            return time.perf_counter() - t0, xs.shape[0]
        from oracle import folded_moe_oracle as O

        O.set_threads(self.threads)
        shared = _shared_fp32(self.ex) if "sh_gu_w" in self.ex else None
        t0 = time.perf_counter()
        O.moe_layer_forward(xs.numpy(), self.groups, self.ex["router_w"], c.top_k, c.hidden, c.inter, c.group_size,
                            router=c.router, e_bias=self.ex.get("e_bias"), shared=shared)
        return time.perf_counter() - t0, xs.shape[0]


def _stage_events(layer, x, fn=None):
    """One forward with CUDA events at the stage boundaries inside the C ABI call; returns the 7 stage durations in us."""
    import ctypes

    import torch

    from chronos_b200 import _lib

    st = torch.cuda.current_stream()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
    for ev in evs:
        ev.record(st)  # forces creation of the underlying handle
    torch.cuda.synchronize()
    arr = (ctypes.c_void_p * 8)(*[ev.cuda_event for ev in evs])
    _lib.check(_lib.lib().chronos_b200_set_stage_events(arr, 8))
    (fn or layer)(x)
    _lib.check(_lib.lib().chronos_b200_set_stage_events(None, 0))
    torch.cuda.synchronize()
    return [1e3 * evs[j].elapsed_time(evs[j + 1]) for j in range(7)]


STAGE_NAMES = ("router", "plan", "gu_input", "gu_bank_pass", "swiglu_dn_input", "dn_bank_pass", "combine")


# ---------------------------------------------------------------------------------------------------------------
def run_decode(args, sampler=None, with_cpu_baseline=True) -> dict:
    import torch

    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer
    from chronos_b200 import build as cuda_build

    cuda_build.build()
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = FoldedLayerConfig(**DECODE)
    tail = (args.tail, args.tail) if args.tail else (0, 0)  # optional tail lattice: same code width for both products
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=1, device=dev, with_shared=True, tail_bits=tail), register=False)
    streams = args.streams
    batches = decode_batches(cfg, streams, dev)
    n_tok = batches[0].shape[0]
    stats = routing_stats(layer, batches, streams)
    K, W = args.steps, max(args.warmup, 3)
    st = torch.cuda.current_stream()

    own_sampler = sampler is None
    if own_sampler:
        sampler = ClockSampler(dev.index or 0)
    for i in range(W):
        layer(batches[i % N_BATCHES])
    torch.cuda.synchronize()
    # ---- device-resident throughput: exactly K steps between two events -----------------------------------------
    # The steps are replayed from CUDA graphs of N_BATCHES forward calls (the way a serving engine runs its decode steps), so
    # that the figure is the device's, not this host's launch rate; a shorter graph supplies the K % N_BATCHES steps left over.
    def capture_forwards(n_steps: int):
        g, keep = torch.cuda.CUDAGraph(), []
        with torch.cuda.graph(g):
            for i in range(n_steps):
                keep.append(layer(batches[i]))
        return g, keep

    g_full, keep_full = capture_forwards(N_BATCHES)
    g_tail, keep_tail = capture_forwards(K % N_BATCHES) if K % N_BATCHES else (None, None)
    g_full.replay()
    torch.cuda.synchronize()
    assert all(torch.equal(keep_full[i], layer(batches[i])) for i in range(N_BATCHES)), "graph replay differs from the eager forward"
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(K // N_BATCHES):
        g_full.replay()
    if g_tail is not None:
        g_tail.replay()
    e1.record(st)
    torch.cuda.synchronize()
    ms_total = e0.elapsed_time(e1)
    del g_full, g_tail, keep_full, keep_tail
    assert layer.device_status() == 0, "device status word raised during the timed loop"

    # ---- per-stage durations (same steps, events at the stage boundaries inside the C ABI call) ------------------
    n_ev_steps = min(K, 40)
    rows = [_stage_events(layer, batches[i % N_BATCHES]) for i in range(n_ev_steps)]
    fp4 = bool(layer.packed.struct.gu_t)  # the layer carries re-tiled banks: the auto regime streams them through FP4 MMA
    fused = fp4 and not args.tail
    bank_kernel = "bank_fp4_kernel" if fp4 else "bank_stream_kernel"
    stage_us = {nm: statistics.mean(r[j] for r in rows) for j, nm in enumerate(STAGE_NAMES)}
    key_gu, key_dn = ("gu_pass_bytes", "dn_pass_bytes") if fused else ("gu_bank_bytes", "dn_bank_bytes")
    gu_bytes = statistics.mean(stats[i % N_BATCHES][key_gu] for i in range(n_ev_steps))
    dn_bytes = statistics.mean(stats[i % N_BATCHES][key_dn] for i in range(n_ev_steps))
    layer_bytes = statistics.mean(stats[i % N_BATCHES]["layer_bytes"] for i in range(K))
    if args.tail:  # per distinct expert: codes + e4m3 block scales of the gate_up and down tail matrices
        blk = 32 if args.tail == 2 else 64
        tail_per_expert = 3 * cfg.hidden * cfg.inter * args.tail // 8 + 3 * cfg.hidden * cfg.inter // blk
        layer_bytes += statistics.mean(stats[i % N_BATCHES]["experts"] for i in range(K)) * tail_per_expert

    # ---- end to end: pinned host input -> device -> forward -> pinned host output, copies inside the timed region --
    # A CUDA graph holds a run of steps - per step the copy of its batch from pinned host memory, the public forward call, the
    # copy of the result to pinned host memory - with the copies on side streams of the capture, double-buffered: step i + 1's
    # input lands while step i computes, step i's output leaves while step i + 1 computes (the way a serving loop feeds a
    # layer). Graphs, so that the measurement does not depend on how fast this host's Python issues three operations per
    # 170 us step. Every step's copies are inside the timed region; exactly K steps are replayed.
    host_in = [b.cpu().pin_memory() for b in batches]
    host_out = [torch.empty_like(host_in[0]).pin_memory() for _ in range(N_BATCHES)]
    dev_in = [torch.empty_like(batches[0]) for _ in range(2)]
    for i in range(max(W, 3)):  # eager once: workspace and allocator pools exist before any capture
        dev_in[0].copy_(host_in[i % N_BATCHES], non_blocking=True)
        host_out[0].copy_(layer(dev_in[0]), non_blocking=True)
    torch.cuda.synchronize()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

    def capture(n_steps: int):
        g, keep = torch.cuda.CUDAGraph(), []
        with torch.cuda.graph(g):
            cur = torch.cuda.current_stream()
            s_in.wait_stream(cur)
            s_out.wait_stream(cur)
            landed, done = [None, None], [None] * n_steps
            with torch.cuda.stream(s_in):
                dev_in[0].copy_(host_in[0], non_blocking=True)
                landed[0] = torch.cuda.Event()
                landed[0].record(s_in)
            for i in range(n_steps):
                b = i & 1
                cur.wait_event(landed[b])
                y = layer(dev_in[b])
                keep.append(y)  # no block of the capture's pool is reused while a side stream may still read it
                done[i] = torch.cuda.Event()
                done[i].record(cur)
                s_out.wait_event(done[i])
                with torch.cuda.stream(s_out):
                    host_out[i].copy_(y, non_blocking=True)
                if i + 1 < n_steps:
                    if i >= 1:
                        s_in.wait_event(done[i - 1])  # the forward that read this input buffer has finished
                    with torch.cuda.stream(s_in):
                        dev_in[b ^ 1].copy_(host_in[i + 1], non_blocking=True)
                        landed[b ^ 1] = torch.cuda.Event()
                        landed[b ^ 1].record(s_in)
            cur.wait_stream(s_in)
            cur.wait_stream(s_out)
        return g, keep

    g_full, keep_full = capture(N_BATCHES)
    g_tail, keep_tail = capture(K % N_BATCHES) if K % N_BATCHES else (None, None)
    g_full.replay()
    torch.cuda.synchronize()
    for i in range(N_BATCHES):  # the replay left every step's result in its pinned host buffer
        assert torch.equal(host_out[i], layer(batches[i]).cpu()), "graph replay differs from the eager forward"
    e0.record(st)
    for _ in range(K // N_BATCHES):
        g_full.replay()
    if g_tail is not None:
        g_tail.replay()
    e1.record(st)
    torch.cuda.synchronize()
    del g_full, g_tail, keep_full, keep_tail
    ms_e2e = e0.elapsed_time(e1)
    clocks = sampler.stop() if own_sampler else None

    # ---- the same batches with the batch-coalesced routing policy (drafts prefer experts their stream's anchor selected) ----
    coalesced = None
    if not args.tail:
        pool, keep = 12, 4
        routed = [layer.route_coalesced(b, tokens_per_stream=TOKENS_PER_STREAM, pool=pool, keep=keep) for b in batches]
        c_slots = [len({int(e) // cfg.group_size for e in ids.reshape(-1).tolist()}) for ids, _ in routed]
        for i in range(W):
            layer.routed_forward(batches[i % N_BATCHES], *layer.route_coalesced(batches[i % N_BATCHES], TOKENS_PER_STREAM, pool, keep), with_shared=True)
        torch.cuda.synchronize()
        e0.record(st)
        for i in range(K):
            b = batches[i % N_BATCHES]
            layer.routed_forward(b, *layer.route_coalesced(b, TOKENS_PER_STREAM, pool, keep), with_shared=True)
        e1.record(st)
        torch.cuda.synchronize()
        coalesced = {"pool": pool, "keep": keep, "distinct_slots_per_step": statistics.mean(c_slots),
                     "distinct_slots_natural": statistics.mean(s["slots"] for s in stats),
                     "ms_per_step": e0.elapsed_time(e1) / K, "tokens_per_s": n_tok / (e0.elapsed_time(e1) * 1e-3 / K),
                     "note": "router + coalescing selection as separate launches, then the routed entry point"}

    peak, peak_kind = _peaks()
    gu_gbs = gu_bytes / (stage_us["gu_bank_pass"] * 1e-6) / 1e9
    dn_gbs = dn_bytes / (stage_us["dn_bank_pass"] * 1e-6) / 1e9
    step_s = ms_total * 1e-3 / K
    # kernels of this library per step: fused decode path = front, gate_up pass, mid, down pass, combine; the separate-kernel
    # path = router, plan (+ top-k), input transform, 2 bank passes, SwiGLU, down transform, combine (+ fp16 image, 2 tail passes)
    launches = 5 if fused else 8 + (3 if args.tail else 0)
    out = {
        "metric": "folded_moe_decode_tokens_per_s", "value": n_tok / step_s, "unit": "tokens/s", "n_gpus": 1,
        "steps": K, "warmup": W, "ms_per_step": ms_total / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": ("e2m1 x ue4m3 block-scaled FP4 MMA (banks as stored; activations as 3 residual e2m1 terms), fp32 accumulate" if fp4
                  else "f16 (NVFP4 e2m1 x e4m3 weights exact in f16; fp32 accumulate)"), "data": "synthetic",
        "config": {"workload": "decode_layer", "regime": "stream_fp4" if fp4 else "stream", "hidden": cfg.hidden, "routed_experts": cfg.n_experts, "shared_experts": 1,
                   "top_k": cfg.top_k, "inter": cfg.inter, "fold_factor": cfg.group_size, "healer_rank": cfg.rank,
                   "streams": streams, "tokens_per_stream": TOKENS_PER_STREAM, "activations": "bf16", "router": cfg.router,
                   "l2_policy": f"each step streams {layer_bytes / 1e6:.0f} MB of banks (> 126 MB L2) and batches rotate over {N_BATCHES} routings",
                   "launch": f"timed steps replayed from CUDA graphs of {N_BATCHES} forward calls (stage durations: eager calls with events)",
                   "tail_lattice_bits": args.tail,
                   "distinct_slots_per_step": statistics.mean(s["slots"] for s in stats),
                   "distinct_slots_by_routing": [s["slots"] for s in stats],
                   "distinct_experts_per_step": statistics.mean(s["experts"] for s in stats),
                   "top8_overlap_within_stream": round(statistics.mean(s["overlap"] for s in stats), 3)},
        "e2e": {"value": n_tok / (ms_e2e * 1e-3 / K), "unit": "tokens/s", "h2d_bytes_per_step": n_tok * cfg.hidden * 2,
                "d2h_bytes_per_step": n_tok * cfg.hidden * 2,
                "copies": "every step's input and output copy inside the timed region; CUDA graphs of 8 steps, copies on side streams, double-buffered"},
        "gpu_launches": launches * K,
        "clocks": clocks,
        "roofline": {"bound": "hbm", "kernel": f"{bank_kernel} (gate_up pass" + (", healer product in its side warps)" if fused else ")"),
                     "achieved": gu_gbs, "peak": peak, "peak_kind": f"of {peak_kind}", "unit": "GB/s", "frac": gu_gbs / peak,
                     "traffic": GU_PASS_TRAFFIC_OVER_ALGORITHMIC * gu_bytes, "algorithmic_bytes_per_launch": gu_bytes},
        "layer_hbm": {"algorithmic_bytes_per_step": layer_bytes, "achieved_gbs": layer_bytes / step_s / 1e9,
                      "frac_of_peak": layer_bytes / step_s / 1e9 / peak, "frac_of_8tbs": layer_bytes / step_s / 8e12},
        "stages_us": {k: round(v, 2) for k, v in stage_us.items()},
        "dn_bank_pass_gbs": dn_gbs,
        "coalesced_routing": coalesced,
    }
    if with_cpu_baseline and not args.no_cpu_baseline:
        threads = host_threads()
        ref = CpuReference(layer.packed, threads)
        ref.forward(batches[0][:1])  # untimed: thread pools, imports, first touch
        secs, n = ref.forward(batches[0])  # one full step of the workload (about ten seconds of host work)
        out["cpu_baseline"] = {"value": n / secs, "unit": "tokens/s", "cores": threads, "kind": ref.kind,
                               "sample": f"batch 0 of the workload ({n} tokens = one step), one pass, {secs:.1f} s"}
    del layer
    torch.cuda.empty_cache()
    return out


def run_prefill(args, steps: int | None = None, ceiling: bool | None = None) -> dict:
    """Prefill-shaped layer (config index 3): the decode layer's shapes, 8192 tokens bf16, router biased so that
    expert popularity follows Zipf(1.1). Reports tokens/s and useful TFLOP/s of the tensor regime."""
    import numpy as np
    import torch

    from chronos_b200 import FoldedLayerConfig, FoldedMoELayer, PackedLayer
    from chronos_b200 import build as cuda_build
    from chronos_b200.workloads import zipf_prefill_batch

    cuda_build.build()
    dev = torch.device("cuda", torch.cuda.current_device())
    ceiling = (args.workload == "fp4_ceiling") if ceiling is None else ceiling
    # fp4_ceiling: the same kernels on ONE slot (4 experts, every token routed to all 4): banks and activation images
    # stay in L2, work items are all full - an empirical ceiling for this tile shape, not a workload of the reference
    cfg = FoldedLayerConfig(**{**DECODE, **({"n_experts": 4, "top_k": 4} if ceiling else {})})
    layer = FoldedMoELayer(packed=PackedLayer.synthetic(cfg, seed=2, device=dev, with_shared=not ceiling), register=False)
    n_tok = args.tokens
    regime = args.regime or "tensor_fp4"
    if ceiling:
        x = torch.randn(n_tok, cfg.hidden, generator=torch.Generator(device=dev).manual_seed(2), device=dev).to(torch.bfloat16)
    else:
        x = zipf_prefill_batch(layer, n_tok, seed=2)
    ids = layer.route(x)[0]
    counts = torch.bincount(ids.reshape(-1).long(), minlength=cfg.n_experts).cpu().numpy()
    K, W = steps or max(args.steps // 20, 3), 3
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
    stage = _stage_events(layer, x, fn=lambda t: layer.forward_impl(t, regime=regime))
    stage_us = {nm: round(stage[j], 1) for j, nm in enumerate(STAGE_NAMES)}
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
    terms = layer.activation_terms if fp4 else 1
    if fp4:
        # the block-scaled pass multiplies every bank tile by `terms` residual FP4 terms of the activations: the pipe does
        # that many times the useful FLOPs; no FP4 figure is in MEASURED_PEAKS.json, so the denominator is the datasheet rate
        roof = {"bound": "tensor", "kernel": "bank_fp4_wide_kernel (both passes)", "achieved": achieved, "peak": FP4_NOMINAL_TFLOPS,
                "peak_kind": "nominal dense FP4 (datasheet; not in MEASURED_PEAKS.json)", "unit": "TFLOP/s", "frac": achieved / FP4_NOMINAL_TFLOPS,
                "activation_terms": terms, "mma_issue_tflops": terms * achieved, "mma_issue_frac": terms * achieved / FP4_NOMINAL_TFLOPS,
                "achieved_vs_measured_bf16": achieved / bf16_peak, "traffic": None}
        dtype = f"e2m1 x ue4m3 block-scaled operands (banks as stored, activations as {terms} residual FP4 terms), fp32 accumulate in TMEM"
    else:
        roof = {"bound": "tensor", "kernel": "bank_gemm_kernel (both passes)", "achieved": achieved, "peak": bf16_peak,
                "peak_kind": "of measured bf16 (operands are f16)", "unit": "TFLOP/s", "frac": achieved / bf16_peak, "traffic": None}
        dtype = "f16 operands (NVFP4 banks converted exactly), fp32 accumulate in TMEM"
    out = {
        "metric": "folded_moe_prefill_tokens_per_s", "value": n_tok / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": K,
        "warmup": W, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": dtype, "data": "synthetic",
        "config": {"workload": "fp4_ceiling_one_slot" if ceiling else "prefill_layer", "regime": regime, "tokens": n_tok, "hidden": cfg.hidden, "routed_experts": cfg.n_experts,
                   "top_k": cfg.top_k, "inter": cfg.inter, "fold_factor": cfg.group_size, "healer_rank": cfg.rank,
                   "router_popularity": "all tokens to all 4 experts" if ceiling else "Zipf(1.1)", "pairs_per_expert_max": int(counts.max()), "pairs_per_expert_median": float(np.median(counts)),
                   "pairs_per_expert_min": int(counts.min())},
        "useful_tflops_layer": useful / (ms * 1e-3) / 1e12,
        "non_gemm_share_of_layer": 1.0 - gemm_s / (sum(stage_us.values()) * 1e-6),
        "roofline": roof,
        "stages_us": stage_us,
    }
    del layer
    torch.cuda.empty_cache()
    return out


def prefill_subrecord(args) -> dict:
    """Config 3 (8192 tokens, Zipf(1.1)) with its roofline, plus the empirical FP4 ceiling of the same tile shapes."""
    import argparse as _ap

    a = _ap.Namespace(**{**vars(args), "tokens": PREFILL_TOKENS, "regime": "tensor_fp4", "workload": "prefill"})
    res = run_prefill(a, steps=5, ceiling=False)
    ceil = run_prefill(a, steps=5, ceiling=True)
    roof = res["roofline"]
    roof["empirical_ceiling_tflops"] = ceil["roofline"]["achieved"]
    roof["frac_of_empirical_ceiling"] = roof["achieved"] / ceil["roofline"]["achieved"]
    return {k: res[k] for k in ("metric", "value", "unit", "ms_per_step", "steps", "config", "useful_tflops_layer",
                                "non_gemm_share_of_layer", "roofline", "stages_us", "dtype")}


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


def run_reference(args, workload: str) -> dict:
    """The reference's algorithm for the same configuration on the host cores (its own PyTorch code from oracle/_ref;
    the numpy port when that folder is absent). decode: the GPU arm's 12-token batches, one batch per step, as many of
    the requested steps as fit the time bound. ep_stack: one layer of the stack on a token subsample, scaled to the
    42-layer step (the reference has no distributed path: the CPU arm is one process whatever N is)."""
    import torch

    from chronos_b200 import FoldedLayerConfig, PackedLayer

    cfg = FoldedLayerConfig(**DECODE)
    have_gpu = torch.cuda.is_available()
    dev = torch.device("cuda", 0) if have_gpu else torch.device("cpu")  # same seeded bytes as the GPU arm when it can draw them there
    threads = host_threads()
    K, W = args.steps, args.warmup
    if workload == "decode":
        packed = PackedLayer.synthetic(cfg, seed=1, device=dev, with_shared=True)
        batches = decode_batches(cfg, args.streams, dev)
        sample = f"{args.streams} streams x {TOKENS_PER_STREAM} tokens per step (the GPU arm's batches)"
        scale, metric, wl_cfg = 1.0, "folded_moe_decode_tokens_per_s", {"workload": "decode_layer", "streams": args.streams, "tokens_per_stream": TOKENS_PER_STREAM}
        scaling = "weak"
    else:
        packed = PackedLayer.synthetic_sharded(cfg, 3, range(cfg.n_slots), dev, True)
        gen = torch.Generator(device=dev).manual_seed(3)
        h0 = torch.randn(EP_TOKENS, cfg.hidden, generator=gen, device=dev).to(torch.bfloat16)
        n_sub = 12
        batches = [h0[i * n_sub:(i + 1) * n_sub] for i in range(N_BATCHES)]
        sample = f"layer 0 of the stack on {n_sub} of the {EP_TOKENS} tokens per step; tokens/s divided by the {args.layers} layers"
        scale, metric, wl_cfg = 1.0 / args.layers, "folded_moe_ep_stack_tokens_per_s", {"workload": "ep_stack", "layers": args.layers, "tokens_per_step": EP_TOKENS}
        scaling = "strong"
    ref = CpuReference(packed, threads)
    ref.forward(batches[0][:1])  # untimed: thread pools, imports, first-touch of one token's slots
    times, toks = [], 0
    for i in range(K):
        secs, n = ref.forward(batches[i % N_BATCHES])
        times.append(secs)
        toks += n
        if sum(times) + secs > REFERENCE_BUDGET_S:  # bounded: the next step would run past the budget
            break
    done = len(times)
    val = scale * toks / sum(times)
    out = {
        "impl": "reference", "metric": metric, "value": val, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": done, "warmup": 1, "ms_per_step": 1e3 * sum(times) / done, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {**wl_cfg, "hidden": cfg.hidden, "routed_experts": cfg.n_experts, "shared_experts": 1,
                   "top_k": cfg.top_k, "inter": cfg.inter, "fold_factor": cfg.group_size, "healer_rank": cfg.rank,
                   "sample": sample, "steps_requested": K, "time_bound_s": REFERENCE_BUDGET_S},
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": threads, "kind": ref.kind, "sample": f"{done} steps; {sample}"},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if have_gpu and ref.kind == "reference" and not args.no_reference_cuda:
        # the same reference code with its tensors on the GPU ("the reference on the same box"): one untimed + one timed step
        from oracle import ref_torch

        x = batches[0].float()
        groups = {g: ref_torch.group_to_torch(ref.groups[g], "cuda") for g in ref._slots_of(x.cpu().numpy())}
        shared = {k: torch.from_numpy(v).cuda() for k, v in ref.ex.items() if k.startswith("sh_")}
        rw = torch.from_numpy(ref.ex["router_w"]).cuda()
        for rep in range(2):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            ref_torch.layer_forward(x, groups, rw, cfg.top_k, cfg.hidden, cfg.inter, cfg.group_size, shared=shared)
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
        out["reference_on_gpu"] = {"value": scale * x.shape[0] / dt, "unit": "tokens/s", "ms_per_step": 1e3 * dt,
                                   "note": "the reference's PyTorch path with device=cuda, one step, wall clock around a synchronise"}
    return out


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
    """The expert-parallel workload (42-layer stack, 4096 tokens per step) on one GPU, as a sub-record of the decode line."""
    import argparse as _ap
    import gc

    import torch

    from chronos_b200 import ep_bench

    gc.collect()
    torch.cuda.empty_cache()
    small = _ap.Namespace(**{**vars(args), "steps": min(args.steps, 10), "warmup": 3})
    res = ep_bench.run(small, args.layers, EP_TOKENS, DECODE, None)
    return {k: res[k] for k in ("metric", "value", "unit", "ms_per_step", "steps", "parity", "phase_us_per_layer_rank0") if k in res} | {
        "config": {"workload": "ep_stack", "layers": args.layers, "tokens_per_step": EP_TOKENS}}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--workload", default=None, choices=(None, "decode", "ep_stack", "prefill", "sweep", "fp4_ceiling"))
    ap.add_argument("--tokens", type=int, default=PREFILL_TOKENS, help="tokens of the prefill workload")
    ap.add_argument("--regime", default=None, choices=(None, "auto", "tensor", "tensor_fp4"), help="bank-pass regime of the prefill workload")
    ap.add_argument("--streams", type=int, default=DECODE_STREAMS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub-records", action="store_true", help="skip the prefill / ep_stack (resp. decode) sub-records of the default lines")
    ap.add_argument("--no-reference-cuda", action="store_true", help="reference arm: skip the extra run of the reference code on the GPU")
    ap.add_argument("--tail", type=int, default=0, choices=(0, 1, 2), help="decode workload: add a tail lattice of this many bits per weight")
    ap.add_argument("--layers", type=int, default=EP_LAYERS, help="depth of the ep_stack workload")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    # under the distributed launcher (world size 1 included) and for N > 1 the line is the expert-parallel stack, so that the
    # lines of a 1-2-4-8 GPU series are the same metric; a plain `python bench.py` is the decode layer
    launched = "TORCHELASTIC_RUN_ID" in os.environ or "LOCAL_RANK" in os.environ
    # `--gpus 1` on a node that shows several GPUs is the first point of a 1-2-4-8 series: it runs the stack too, so that the
    # series is one metric (the decode layer rides along as a sub-record); on a one-GPU node it is the decode layer
    series_point = False
    if args.workload is None and args.gpus == 1 and not launched:
        try:
            import torch

            series_point = torch.cuda.device_count() > 1
        except Exception:
            series_point = False
    workload = args.workload or ("ep_stack" if (args.gpus > 1 or world > 1 or launched or series_point) else "decode")
    if args.impl == "reference":
        if rank == 0:
            with _StdoutToStderr():
                res = run_reference(args, "ep_stack" if workload == "ep_stack" else "decode")
            print(json.dumps(res), flush=True)
        return
    if workload in ("decode", "prefill", "sweep", "fp4_ceiling"):
        if rank == 0:
            import torch

            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
            with _StdoutToStderr():
                out = {"decode": run_decode, "prefill": run_prefill, "sweep": run_sweep, "fp4_ceiling": run_prefill}[workload](args)
                if workload == "decode" and args.workload is None and not args.no_sub_records:
                    # the other half of the metric (prefill FP4 TFLOP/s) and the N > 1 workload on one GPU, in the same line
                    for name, fn in (("prefill", prefill_subrecord), ("ep_stack_1gpu", ep_stack_single_gpu)):
                        try:
                            out[name] = fn(args)
                        except Exception as exc:  # the headline must not depend on the extra measurements
                            out[name] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
            print(json.dumps(out), flush=True)
        return
    from chronos_b200 import ep_bench

    with _StdoutToStderr():
        res = ep_bench.run(args, args.layers, EP_TOKENS, DECODE, ClockSampler)
        if rank == 0 and world == 1 and not args.no_sub_records:
            # world size 1: the decode layer (the configuration the headline metric is quoted on) rides along
            try:
                import argparse as _ap

                d = run_decode(_ap.Namespace(**{**vars(args), "steps": 100, "warmup": 10}), sampler=False, with_cpu_baseline=False)  # 175 us per step: cheap
                res["decode_layer"] = {k: d[k] for k in ("metric", "value", "unit", "ms_per_step", "steps", "roofline", "layer_hbm", "stages_us", "e2e")}
            except Exception as exc:
                res["decode_layer"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            # the reference's CPU path on a bounded sample of the same workload (one layer, 12 tokens, scaled by the depth)
            try:
                import argparse as _ap

                ref = run_reference(_ap.Namespace(**{**vars(args), "steps": 1, "no_reference_cuda": True}), "ep_stack")
                res["cpu_baseline"] = ref["cpu_baseline"]
            except Exception as exc:
                res["cpu_baseline"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    if rank == 0:
        print(json.dumps(res), flush=True)
        if res.get("parity", {}).get("rel_l2", 0.0) > 1e-2:
            sys.exit(3)


if __name__ == "__main__":
    main()
