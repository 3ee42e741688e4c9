"""Expert-parallel folded MoE: slots sharded over the ranks of one NVLink box.

The reference has no distributed path at all (single device, TP=1), so the partitioning below is new: a slot is
never split (its K experts share one bank), rank g owns slots [g*n_slots/G, (g+1)*n_slots/G); router weights,
RMSNorm and the shared expert are replicated; tokens are data-parallel.

Per layer, stream-ordered and free of host synchronisation:
  dispatch  every rank routes its own tokens, then the normed token rows and their (expert id, gate) lists are
            exchanged so that each rank sees all tokens (capacity-padded exchange: each peer gets a fixed-size
            block, so no split sizes ever travel through the host);
  compute   each rank evaluates only the routing entries whose expert it owns (the others are masked to -1 and
            skipped on the device) plus, in the same pass, the shared expert for the tokens it is the home of;
  combine   the per-rank partial sums are reduce-scattered back to the tokens' home ranks in fp32.
One process per GPU; `torch.distributed` (NCCL over NVLink, or gloo in CPU tests of the host logic).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib
from .layout import FoldedLayerConfig, PackedLayer
from .moe import FoldedMoELayer, residual_rmsnorm


def slot_range(n_slots: int, world: int, rank: int) -> range:
    """Slots owned by `rank`: contiguous, balanced, never splitting a slot."""
    if n_slots % world:
        raise ValueError(f"{n_slots} slots do not divide over {world} ranks")
    per = n_slots // world
    return range(rank * per, (rank + 1) * per)


def localize_routing(ids: torch.Tensor, first_expert: int, n_local: int) -> torch.Tensor:
    """Global expert ids -> ids local to the owning rank, -1 for experts another rank owns (skipped on the device)."""
    local = ids - first_expert
    return torch.where((local >= 0) & (local < n_local), local, torch.full_like(local, -1)).to(torch.int32)


class ExpertParallelMoE:
    """One expert-parallel layer. `local_layer` holds this rank's slots (its config describes the LOCAL expert table
    with `first_slot` set), `router` computes (global ids, gates) for local tokens.

    `compute_routed(x_all, local_ids, gates) -> fp32 [T, H]` and `compute_shared(x_local) -> fp32 [Tl, H]` default to
    the CUDA layer; tests of the host logic on CPU ranks substitute their own callables."""

    def __init__(self, local_layer: Optional[FoldedMoELayer], cfg_global: FoldedLayerConfig, group=None,
                 route_fn: Optional[Callable] = None, compute_routed: Optional[Callable] = None,
                 compute_shared: Optional[Callable] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.cfg = cfg_global
        slots = slot_range(cfg_global.n_slots, self.world, self.rank)
        self.first_expert = slots.start * cfg_global.group_size
        self.n_local = len(slots) * cfg_global.group_size
        self.layer = local_layer
        self.route_fn = route_fn or (lambda x: local_layer.route_global(x))
        # CUDA default: one pass over the gathered tokens evaluates the entries this rank owns AND the shared expert of
        # the tokens it is the home of (their block inside the gathered order); tests substitute CPU callables and a
        # separate shared-expert callable
        self.fused_shared = compute_routed is None and compute_shared is None
        self.compute_routed = compute_routed or self._routed_cuda
        self.compute_shared = compute_shared or self._shared_cuda
        self.phase_events = None   # set to [] to record (name, start, end) CUDA events of the next forward

    def _mark(self, name: str):
        """Context manager recording a CUDA event pair around a phase when `phase_events` is a list."""
        return _Phase(self.phase_events, name)

    def _routed_cuda(self, x_all: torch.Tensor, local_ids: torch.Tensor, gates_all: torch.Tensor) -> torch.Tensor:
        tl = x_all.shape[0] // self.world
        rng = (self.rank * tl, tl) if self.layer.n_shared_experts else None
        return self.layer.routed_forward(x_all, local_ids, gates_all, out_dtype=torch.float32, shared_range=rng)

    def _shared_cuda(self, x_local: torch.Tensor) -> Optional[torch.Tensor]:
        if self.layer.n_shared_experts == 0:
            return None
        none = torch.full((x_local.shape[0], self.cfg.top_k), -1, dtype=torch.int32, device=x_local.device)
        zero = torch.zeros((x_local.shape[0], self.cfg.top_k), dtype=torch.float32, device=x_local.device)
        return self.layer.routed_forward(x_local, none, zero, with_shared=True, out_dtype=torch.float32)

    @torch.no_grad()
    def forward(self, x_local: torch.Tensor) -> torch.Tensor:
        """x_local [Tl, H] (same Tl on every rank) -> y_local fp32 [Tl, H]."""
        tl, h = x_local.shape
        k = self.cfg.top_k
        # ---- dispatch: gather rows and routing lists of all ranks (fixed-size blocks, no host-side sizes). The token rows
        # do not depend on the routing, so their exchange is issued first and runs (on the collective's own stream) while
        # the router kernels run on this one; the current stream waits for it only before the expert pass. -----------------
        x_all = torch.empty((self.world * tl, h), dtype=x_local.dtype, device=x_local.device)
        with self._mark("dispatch_rows_issue"):
            rows = dist.all_gather_into_tensor(x_all, x_local.contiguous(), group=self.group, async_op=True)
        with self._mark("route"):
            ids, gates = self.route_fn(x_local)
        with self._mark("dispatch"):
            meta_local = torch.cat([ids.to(torch.float32), gates.to(torch.float32)], dim=1).contiguous()  # ids < 2^24: exact
            meta_all = torch.empty((self.world * tl, 2 * k), dtype=torch.float32, device=x_local.device)
            dist.all_gather_into_tensor(meta_all, meta_local, group=self.group)
            ids_all = meta_all[:, :k].to(torch.int64)
            gates_all = meta_all[:, k:].contiguous()
            local_ids = localize_routing(ids_all, self.first_expert, self.n_local)
            if rows is not None:
                rows.wait()  # stream-ordered: no host synchronisation
        # ---- compute: only entries this rank owns ---------------------------------------------------------------------
        with self._mark("routed_experts"):
            part = self.compute_routed(x_all, local_ids, gates_all)
        # ---- combine: partial sums back to the home ranks -------------------------------------------------------------
        with self._mark("combine"):
            y = torch.empty((tl, h), dtype=torch.float32, device=x_local.device)
            dist.reduce_scatter_tensor(y, part.contiguous(), op=dist.ReduceOp.SUM, group=self.group)
        if not self.fused_shared:
            with self._mark("shared_expert"):
                sh = self.compute_shared(x_local)
                if sh is not None:
                    y += sh
        return y

    __call__ = forward


class _Phase:
    def __init__(self, sink, name):
        self.sink, self.name = sink, name

    def __enter__(self):
        if self.sink is not None and torch.cuda.is_available():
            self.e0 = torch.cuda.Event(enable_timing=True)
            self.e0.record()
        return self

    def __exit__(self, *exc):
        if self.sink is not None and torch.cuda.is_available():
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
            self.sink.append((self.name, self.e0, e1))
        return False


def build_local_layer(cfg_global: FoldedLayerConfig, seed: int, world: int, rank: int, device, with_shared: bool,
                      shared_from: Optional[FoldedMoELayer] = None) -> FoldedMoELayer:
    """Synthetic layer holding only this rank's slots (seeded per slot so that every world size sees the same bytes
    for a given slot), with the full router table replicated."""
    slots = slot_range(cfg_global.n_slots, world, rank)
    packed = PackedLayer.synthetic_sharded(cfg_global, seed, slots, device, with_shared)
    return FoldedMoELayer(packed=packed, register=False)


class ExpertParallelStack:
    """`n_layers` expert-parallel layers with the residual + RMSNorm wiring of the reference's standalone engine
    (chronos_1t/models/glm53_engine.py:200-204): x = rms_norm(h); h = h + moe(x)."""

    def __init__(self, layers: list[ExpertParallelMoE], eps: float = 1e-6):
        self.layers = layers
        self.eps = eps

    @torch.no_grad()
    def forward(self, h_local: torch.Tensor) -> torch.Tensor:
        """h_local [Tl, H] bf16 or fp32, updated in place; returns it."""
        y = None
        for lay in self.layers:
            x = residual_rmsnorm(h_local, y, None, self.eps)   # h += y of the previous layer; x = norm(h)
            y = lay(x).to(h_local.dtype)
        residual_rmsnorm(h_local, y, None, self.eps)           # last residual add
        return h_local

    __call__ = forward
