"""Expert-parallel folded MoE: slots sharded over the ranks of one NVLink box.

The reference has no distributed path at all (single device, TP=1), so the partitioning below is new: a slot is
never split (its K experts share one bank), rank g owns slots [g*n_slots/G, (g+1)*n_slots/G); router weights,
RMSNorm and the shared expert are replicated; tokens are data-parallel.

Per layer, stream-ordered and free of host synchronisation:
  route     every rank routes its own tokens (global expert ids + gates);
  dispatch  a token's normed hidden row goes ONCE to every rank that owns at least one of its experts, with its expert
            ids local to that rank and their gates: device kernels fill fixed-capacity blocks per destination (rows, then
            the block's metadata). On CUDA ranks of one box the kernels store the blocks straight into the peers' receive
            buffers (symmetric memory over NVLink; `chronos_b200_ep_pack_peer`) and a barrier kernel with bounded waits
            (`chronos_b200_ep_barrier`) closes the phase; otherwise ONE all-to-all with equal splits moves them
            (`chronos_b200_ep_pack`) - no split sizes ever travel through the host;
  compute   each rank evaluates the received rows' entries (all of them are its own experts) and, in the same pass,
            the shared expert of the tokens it is the home of;
  combine   ONE bf16 partial-sum row per received token goes back the same way (`chronos_b200_ep_send_back_peer` + barrier,
            or the all-to-all), and the home rank adds the partial rows in rank order to the shared expert's row
            (`chronos_b200_ep_combine`).
A block's capacity covers the expected number of tokens per destination plus six standard deviations; a batch routed
so unevenly that a block overflows raises a device flag that `overflowed()` reads (the caller then repeats the step with
`capacity_factor = 1`, which always fits). One process per GPU; `torch.distributed` (NCCL over NVLink, or gloo in CPU
tests of the host logic, which substitute their own pack / compute / combine callables).
"""
from __future__ import annotations

import math
import os
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib
from .layout import FoldedLayerConfig, PackedLayer
from .moe import _DTYPES, FoldedMoELayer, residual_rmsnorm


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


def block_capacity(tokens_local: int, world: int, top_k: int, capacity_factor: Optional[float] = None) -> int:
    """Rows per (source, destination) block. A token routes >= 1 of its top_k experts to a given rank with probability
    p = 1 - (1 - 1/world)^top_k under balanced routing; the default leaves six standard deviations of head-room (and never
    exceeds the token count, which always fits). `capacity_factor` overrides it as a fraction of the local tokens."""
    if capacity_factor is not None:
        cap = math.ceil(capacity_factor * tokens_local)
    else:
        p = 1.0 - (1.0 - 1.0 / world) ** top_k
        cap = math.ceil(p * tokens_local + 6.0 * math.sqrt(tokens_local * p * (1.0 - p)) + 8.0)
    return max(8, min(tokens_local, (cap + 7) // 8 * 8))


_OVERFLOW_FLAGS: dict[torch.device, torch.Tensor] = {}  # one device flag per GPU, shared by all layers: one read per step


class _PeerExchange:
    """Receive and return buffers of one exchange shape in symmetric memory (every rank's buffers are mapped into every
    other rank's address space), shared by all layers of the process: a layer's two barriers order its use of them against
    the layers before and after. `recv` [world * block_rows + tokens, H]: block s = what rank s sent (rows, then metadata),
    the tail = this rank's own tokens; `back` [world, block_rows, H]: block s = the partial sums rank s returned."""

    def __init__(self, group, world: int, rank: int, tokens: int, block_rows: int, hidden: int, dtype: torch.dtype, device: torch.device):
        # plain peer loads and stores only: the buffers are not bound to an NVLink multicast object (a rank that dies while
        # its memory is bound to one can raise link faults on its peers)
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm_mem

        name = group.group_name if group is not None else dist.group.WORLD.group_name
        self.recv = symm_mem.empty((world * block_rows + tokens, hidden), dtype=dtype, device=device)
        self.back = symm_mem.empty((world, block_rows, hidden), dtype=dtype, device=device)
        self.recv.zero_()
        self.back.zero_()
        self._h_recv = symm_mem.rendezvous(self.recv, name)
        self._h_back = symm_mem.rendezvous(self.back, name)
        self.recv_bases = self._h_recv.buffer_ptrs_dev       # device array of world base pointers
        self.back_bases = self._h_back.buffer_ptrs_dev
        self.pads = self._h_recv.signal_pad_ptrs_dev         # device array of world pointers to peer-writable words
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.epoch = 0
        self.world, self.rank = world, rank

    def barrier(self) -> None:
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        _lib.check(_lib.lib().chronos_b200_ep_barrier(self.pads, self.rank, self.world, self.epoch, self.status.data_ptr(),
                                                    torch.cuda.current_stream().cuda_stream))


_PEER_EXCHANGES: dict[tuple, Optional[_PeerExchange]] = {}


class EpConfigMismatch(RuntimeError):
    """Raised on EVERY rank, before any data collective, when the ranks disagree on the exchange geometry."""


class ExpertParallelMoE:
    """One expert-parallel layer. `local_layer` holds this rank's slots (its config describes the LOCAL expert table
    with `first_slot` set); `route_fn(x) -> (global ids, gates)` for local tokens.

    The device work (pack, expert pass, combine) defaults to the CUDA library; tests of the host logic on CPU ranks pass
    their own `pack_fn`, `compute_fn` and `combine_fn` with the same contracts (see `_pack_cuda` & co.)."""

    def __init__(self, local_layer: Optional[FoldedMoELayer], cfg_global: FoldedLayerConfig, group=None,
                 route_fn: Optional[Callable] = None, pack_fn: Optional[Callable] = None, compute_fn: Optional[Callable] = None,
                 combine_fn: Optional[Callable] = None, capacity_factor: Optional[float] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.cfg = cfg_global
        slots = slot_range(cfg_global.n_slots, self.world, self.rank)
        self.first_expert = slots.start * cfg_global.group_size
        self.n_local = len(slots) * cfg_global.group_size
        self.layer = local_layer
        self.capacity_factor = capacity_factor
        self.route_fn = route_fn or (lambda x: local_layer.route_global(x))
        self.pack_fn = pack_fn or self._pack_cuda
        self.compute_fn = compute_fn or self._compute_cuda
        self.combine_fn = combine_fn or self._combine_cuda
        self.out_dtype = torch.float32  # dtype of forward()'s result (fp32 sums rounded once); a stack sets its activations' dtype
        self.phase_events = None   # set to [] to record (name, start, end) CUDA events of the next forward
        self._checked: set[tuple] = set()
        # peer stores over NVLink instead of the all-to-all (CUDA ranks of one box with symmetric memory; every rank must
        # succeed in setting it up, else all of them stay with the collective); CHRONOS_B200_EP_PEER=0 switches it off
        self.use_peer = pack_fn is None and compute_fn is None and combine_fn is None and os.environ.get("CHRONOS_B200_EP_PEER", "1") != "0"

    def _mark(self, name: str):
        """Context manager recording a CUDA event pair around a phase when `phase_events` is a list."""
        return _Phase(self.phase_events, name)

    # -- geometry agreement -----------------------------------------------------------------------------------------
    def check_geometry(self, tokens_local: int, hidden: int, capacity: int) -> None:
        """All ranks exchange (tokens, hidden, top_k, capacity, experts per rank) once per batch shape and compare: an
        all-to-all with equal splits would otherwise read or write past a peer's block. Raises `EpConfigMismatch` on
        every rank (they all see the same table), before any data collective of the layer runs."""
        key = (tokens_local, hidden, capacity)
        if key in self._checked:
            return
        mine = [tokens_local, hidden, self.cfg.top_k, capacity, self.n_local]
        table: list = [None] * self.world
        dist.all_gather_object(table, mine, group=self.group)
        if any(row != table[0] for row in table):
            raise EpConfigMismatch("expert-parallel ranks disagree on (tokens per rank, hidden, top_k, block capacity, experts per rank): "
                                   + "; ".join(f"rank {r}: {row}" for r, row in enumerate(table)))
        self._checked.add(key)

    # -- device work (CUDA library) -----------------------------------------------------------------------------------
    def _meta_rows(self, capacity: int, h: int, elem: int) -> int:
        """Rows of hidden-size elements that hold one block's metadata ((capacity + 1) x (2 k + 2) int32) behind its rows."""
        return -(-(capacity + 1) * (2 * self.cfg.top_k + 2) * 4 // (h * elem))

    def _pack_cuda(self, x, ids, gates, capacity):
        """One buffer [world, capacity + m, H]: per destination its rows, then m rows of bytes that hold the block's metadata,
        so that ONE collective moves both. Returns (buffer, None, slot_of)."""
        tl, h = x.shape
        k, w = self.cfg.top_k, self.world
        dev = x.device
        m = self._meta_rows(capacity, h, x.element_size())
        buf = torch.empty((w, capacity + m, h), dtype=x.dtype, device=dev)
        slot_of = torch.empty((tl, w), dtype=torch.int32, device=dev)
        flag = _OVERFLOW_FLAGS.get(dev)
        if flag is None:
            flag = _OVERFLOW_FLAGS[dev] = torch.zeros(1, dtype=torch.int32, device=dev)
        row_bytes = h * x.element_size()
        _lib.check(_lib.lib().chronos_b200_ep_pack(x.data_ptr(), _DTYPES[x.dtype], ids.data_ptr(), gates.data_ptr(), tl, k, h, w, self.n_local,
                                                 capacity, buf.data_ptr(), buf.data_ptr() + capacity * row_bytes, slot_of.data_ptr(),
                                                 flag.data_ptr(), capacity + m, (capacity + m) * row_bytes // 4,
                                                 torch.cuda.current_stream().cuda_stream))
        return buf, None, slot_of

    def _compute_cuda(self, recv_rows, recv_meta, x_local, capacity, recv_all=None):
        """Expert pass over the received blocks + the shared expert of the home tokens, one call. `recv_rows`
        [world, capacity + m, H] are the merged blocks (rows, then metadata bytes; `recv_meta` is None), `recv_all`
        [world * (capacity + m) + Tl, H] the buffer whose head they view and whose tail already holds the home tokens' rows.
        The metadata rows ride through the pass as rows without experts. Returns (partial rows in the same block shape,
        shared rows [Tl, H] or None), both in the activation dtype."""
        w, k = self.world, self.cfg.top_k
        tl, h = x_local.shape
        block_rows = recv_rows.shape[1]
        n_recv = w * block_rows
        has_shared = self.layer.n_shared_experts > 0
        dev = x_local.device
        tail = tl if has_shared else 0
        ids = torch.empty((n_recv + tail, k), dtype=torch.int32, device=dev)
        gates = torch.empty((n_recv + tail, k), dtype=torch.float32, device=dev)
        row_bytes = h * x_local.element_size()
        _lib.check(_lib.lib().chronos_b200_ep_unpack_meta(recv_rows.data_ptr() + capacity * row_bytes, w, capacity, k, ids.data_ptr(),
                                                        gates.data_ptr(), block_rows, block_rows * row_bytes // 4, tail,
                                                        torch.cuda.current_stream().cuda_stream))
        if has_shared:  # the home tokens ride along as extra rows that take the shared expert only
            x_all = recv_all if recv_all is not None else torch.cat([recv_rows.reshape(n_recv, h), x_local])
            out = self.layer.routed_forward(x_all, ids, gates, out_dtype=x_local.dtype, shared_range=(n_recv, tl))
            return out[:n_recv].view(w, block_rows, h), out[n_recv:]
        out = self.layer.routed_forward(recv_rows.view(n_recv, h), ids, gates, out_dtype=x_local.dtype)
        return out.view(w, block_rows, h), None

    def _combine_cuda(self, back_rows, slot_of, shared_rows, capacity):
        w, block_rows, h = back_rows.shape
        tl = slot_of.shape[0]
        y = torch.empty((tl, h), dtype=self.out_dtype, device=back_rows.device)
        _lib.check(_lib.lib().chronos_b200_ep_combine(back_rows.data_ptr(), _DTYPES[back_rows.dtype], slot_of.data_ptr(),
                                                    shared_rows.data_ptr() if shared_rows is not None else None, tl, h, w, capacity,
                                                    y.data_ptr(), _DTYPES[self.out_dtype], block_rows, torch.cuda.current_stream().cuda_stream))
        return y

    def _peer_exchange(self, x: torch.Tensor, capacity: int) -> Optional[_PeerExchange]:
        """The symmetric buffers of this exchange shape, or None when any rank could not set them up (decided together,
        once per shape and process; the layers of a stack share the result)."""
        if not self.use_peer or x.device.type != "cuda":
            return None
        tl, h = x.shape
        block_rows = capacity + self._meta_rows(capacity, h, x.element_size())
        key = (id(self.group), self.world, tl, block_rows, h, x.dtype, x.device)
        if key not in _PEER_EXCHANGES:
            ex, why = None, ""
            try:
                ex = _PeerExchange(self.group, self.world, self.rank, tl, block_rows, h, x.dtype, x.device)
            except Exception as exc:  # no symmetric memory on this system / for this group: the collective path serves
                why = f"{type(exc).__name__}: {exc}"[:200]
            table: list = [None] * self.world
            dist.all_gather_object(table, ex is not None, group=self.group)
            if not all(table):
                ex = None
                if self.rank == 0 and why:
                    print(f"chronos_b200: expert-parallel exchange stays on the all-to-all ({why})", flush=True)
            _PEER_EXCHANGES[key] = ex
        return _PEER_EXCHANGES[key]

    def _forward_peer(self, ex: _PeerExchange, x_local: torch.Tensor, ids, gates, capacity: int) -> torch.Tensor:
        """dispatch / compute / combine with peer stores: the pack kernel writes block `rank` of every peer's receive buffer,
        a barrier, the expert pass over the receive buffer, the partial rows go into block `rank` of every peer's return
        buffer, a barrier, the sum."""
        tl, h = x_local.shape
        k, w = self.cfg.top_k, self.world
        dev = x_local.device
        block_rows = ex.back.shape[1]
        stream = torch.cuda.current_stream().cuda_stream
        with self._mark("dispatch"):
            slot_of = torch.empty((tl, w), dtype=torch.int32, device=dev)
            flag = _OVERFLOW_FLAGS.get(dev)
            if flag is None:
                flag = _OVERFLOW_FLAGS[dev] = torch.zeros(1, dtype=torch.int32, device=dev)
            _lib.check(_lib.lib().chronos_b200_ep_pack_peer(x_local.data_ptr(), _DTYPES[x_local.dtype], ids.data_ptr(), gates.data_ptr(), tl, k, h,
                                                          w, self.n_local, capacity, ex.recv_bases, self.rank, block_rows,
                                                          slot_of.data_ptr(), flag.data_ptr(), stream))
            ex.barrier()  # (the pack kernels also put x_local behind the blocks of the local buffer)
        with self._mark("routed_experts"):
            recv_rows = ex.recv[:w * block_rows].view(w, block_rows, h)
            part, shared_rows = self._compute_cuda(recv_rows, None, x_local, capacity, recv_all=ex.recv)
        with self._mark("combine"):
            _lib.check(_lib.lib().chronos_b200_ep_send_back_peer(part.data_ptr(), _DTYPES[part.dtype], h, w, block_rows, capacity, k,
                                                               ex.recv.data_ptr(), ex.back_bases, self.rank, stream))
            ex.barrier()
            y = self._combine_cuda(ex.back, slot_of, shared_rows, capacity)
        return y

    def peer_status(self) -> int:
        """Status words of the peer-exchange barriers of this process OR-ed together (0 = every barrier completed);
        reading them synchronises, so call it once per step."""
        word = 0
        for ex in _PEER_EXCHANGES.values():
            if ex is not None:
                word |= int(ex.status.item())
        return word

    def overflowed(self) -> bool:
        """True when a dispatch block of ANY layer on this rank's device overflowed since the last call (the layers share
        one device flag; reading it synchronises, so call it once per step, not per layer)."""
        hit = False
        for flag in _OVERFLOW_FLAGS.values():
            if int(flag.item()):
                hit = True
                flag.zero_()
        return hit

    # -- the layer ------------------------------------------------------------------------------------------------------
    @torch.no_grad()
    def forward(self, x_local: torch.Tensor) -> torch.Tensor:
        """x_local [Tl, H] (same Tl on every rank) -> y_local [Tl, H] in `out_dtype` (fp32 unless a stack set its own)."""
        tl, h = x_local.shape
        x_local = x_local.contiguous()
        capacity = block_capacity(tl, self.world, self.cfg.top_k, self.capacity_factor)
        self.check_geometry(tl, h, capacity)
        with self._mark("route"):
            ids, gates = self.route_fn(x_local)
        if self.world == 1 and self.layer is not None:  # every expert is local: nothing to exchange
            with self._mark("routed_experts"):
                return self.layer.routed_forward(x_local, ids, gates, with_shared=self.layer.n_shared_experts > 0, out_dtype=self.out_dtype)
        ex = self._peer_exchange(x_local, capacity)
        if ex is not None:
            return self._forward_peer(ex, x_local, ids, gates, capacity)
        with self._mark("dispatch"):
            send_rows, send_meta, slot_of = self.pack_fn(x_local, ids, gates, capacity)
            # received blocks and, behind them, the home tokens' own rows (they take the shared expert in the same pass)
            block_rows = send_rows.shape[1]  # capacity, plus the metadata rows when the pack function merged them in
            recv_all = torch.empty((self.world * block_rows + tl, h), dtype=x_local.dtype, device=x_local.device)
            recv_rows = recv_all[:self.world * block_rows].view(self.world, block_rows, h)
            recv_all[self.world * block_rows:].copy_(x_local)
            recv_meta = None
            if send_meta is not None:  # a pack function that keeps the metadata apart: a collective of its own
                recv_meta = torch.empty_like(send_meta)
                dist.all_to_all_single(recv_meta, send_meta, group=self.group)
            dist.all_to_all_single(recv_rows, send_rows, group=self.group)
        with self._mark("routed_experts"):
            part, shared_rows = self.compute_fn(recv_rows, recv_meta, x_local, capacity, recv_all=recv_all)
        with self._mark("combine"):
            back = torch.empty_like(part)
            dist.all_to_all_single(back, part.contiguous(), group=self.group)
            y = self.combine_fn(back, slot_of, shared_rows, capacity)
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


def build_local_layer(cfg_global: FoldedLayerConfig, seed: int, world: int, rank: int, device, with_shared: bool) -> FoldedMoELayer:
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
            if h_local.dtype in (torch.bfloat16, torch.float32) and h_local.device.type == "cuda":
                lay.out_dtype = h_local.dtype                   # the layer's last kernel rounds to the stack's dtype itself
            y = lay(x).to(h_local.dtype)
        residual_rmsnorm(h_local, y, None, self.eps)           # last residual add
        return h_local

    def overflowed(self) -> bool:
        """True when any layer's dispatch overflowed since the last call (synchronises once)."""
        return bool(self.layers) and self.layers[0].overflowed()

    __call__ = forward
