"""Host-side mirror of the reference's folded MoE block, executing through libchronos_b200.so.

`FoldedMoELayer` keeps the module surface of `ChronosGlm53SparseMoeBlock`
(chronos_1t/models/glm53_chronos_moe.py:109-162, :386-399, :441-486): constructor keywords, `forward`,
`forward_impl`, `route`, `routed_forward`, `load_weights`, and the attributes vLLM's `DeepseekV2MoE` bookkeeping
reads. The arithmetic happens in hand-written CUDA reached through the C ABI; a missing library or a non-CUDA
input raises - nothing here computes on the CPU.
"""
from __future__ import annotations

import os
from pathlib import Path
from typing import Any, Iterable

import torch
from torch import nn

from . import _lib
from .layout import FoldedLayerConfig, PackedLayer, _norm_device, layer_index_from_prefix

LIVE_BLOCKS: dict[int, "FoldedMoELayer"] = {}  # layer index -> block, read by the custom op (glm53_chronos_moe.py:273)


def moe_prefix(layer_idx: int) -> str:
    """chronos_1t/models/glm53_chronos_spec.py:186-187."""
    return f"model.layers.{layer_idx}.mlp"


class _DummyExperts(nn.Module):
    """Satisfies vLLM's `moe_layers.append(layer.mlp.experts)` (chronos_1t/models/glm53_chronos_moe.py:102-106)."""

    def update_expert_map(self) -> None:
        return None


_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}
_REGIMES = {"auto": _lib.REGIME_AUTO, "stream": _lib.REGIME_STREAM, "tensor": _lib.REGIME_TENSOR,
            "stream_fp4": _lib.REGIME_STREAM_FP4, "tensor_fp4": _lib.REGIME_TENSOR_FP4}

# One scratch buffer per device, shared by every layer on it: layers of a model run one after another on the
# worker's stream (the reference's blocks are used the same way), so they never need scratch at the same time.
# Two forwards that overlap on the SAME device from different streams would race on it.
_WORKSPACE_POOL: dict[torch.device, torch.Tensor] = {}
# Buffers the pool outgrew stay allocated: a CUDA graph captured while one of them was current replays with that
# pointer baked in, and it is still large enough for the batch the graph was captured for.
_WORKSPACE_RETIRED: list[torch.Tensor] = []


class FoldedMoELayer(nn.Module):
    def __init__(self, layer_idx: int = 3, shard_path: str | Path | None = None, config: FoldedLayerConfig | None = None,
                 device: torch.device | str | None = None, packed: PackedLayer | None = None, vllm_config: Any = None,
                 prefix: str = "", register: bool = True, check_status: bool | None = None, **_: Any) -> None:
        super().__init__()
        # opt-in: read the device status word after every forward (a synchronisation per call) and raise when a kernel
        # reported an expired wait; off by default because it breaks stream-ordered / graph-captured use
        self.check_status = bool(int(os.environ.get("CHRONOS_B200_CHECK_STATUS", "0"))) if check_status is None else check_status
        if vllm_config is not None:
            idx = layer_index_from_prefix(prefix)
            if idx is not None:
                layer_idx = idx
        if device is None:
            if not torch.cuda.is_available():
                raise _lib.ChronosError("FoldedMoELayer needs a CUDA device: chronos_b200 has no CPU path")
            device = torch.device(f"cuda:{torch.cuda.current_device()}")
        self.device = _norm_device(device)
        if packed is None:
            if shard_path is None or config is None:
                raise ValueError("either `packed` or (`shard_path` and `config`) is required")
            packed = PackedLayer.from_safetensors(shard_path, config, prefix or moe_prefix(layer_idx), self.device)
        _lib.lib()  # fail now, not at the first forward, if the CUDA library is absent
        self.packed = packed
        self.cfg = packed.cfg
        self.layer_idx = layer_idx
        self.hidden, self.inter = self.cfg.hidden, self.cfg.inter
        self.n_experts, self.top_k = self.cfg.n_experts, self.cfg.top_k
        self.routed_scaling_factor = self.cfg.routed_scaling_factor
        # vLLM `DeepseekV2MoE` compatibility surface (chronos_1t/models/glm53_chronos_moe.py:154-162)
        self.n_routed_experts = self.n_experts
        self.n_shared_experts = 1 if packed.struct.shared_inter > 0 else 0
        self.n_logical_experts = self.n_experts
        self.n_physical_experts = self.n_experts
        self.n_local_physical_experts = self.n_experts
        self.n_redundant_experts = 0
        self.experts = _DummyExperts()
        self.is_sequence_parallel = False
        self.activation_terms = 3  # residual FP4 terms per activation in the block-scaled tensor-core regimes
        self._ws: torch.Tensor | None = None
        self._ws_need: dict[int, int] = {}
        self._last_n = 0
        if register:
            LIVE_BLOCKS[layer_idx] = self

    # -- plumbing ---------------------------------------------------------------------------------------------------
    def _workspace(self, n_tokens: int) -> torch.Tensor:
        """Scratch from the per-device pool. The pool only grows, and a buffer it outgrows is kept alive, so a graph
        captured earlier keeps replaying on valid memory. Growing inside a stream capture is refused (an allocation there
        would belong to the graph's private pool): run the largest batch once, or call `reserve_workspace`, before capture."""
        need = self._ws_need.get(n_tokens)
        if need is None:
            need = _lib.lib().chronos_b200_workspace_bytes(self.packed.ptr, n_tokens)
            if need == 0:
                raise _lib.ChronosError("workspace_bytes rejected the layer description")
            self._ws_need[n_tokens] = need
        buf = _WORKSPACE_POOL.get(self.device)
        if buf is None or buf.numel() < need:
            if torch.cuda.is_current_stream_capturing():
                raise _lib.ChronosError(f"the workspace would have to grow to {need} bytes inside a stream capture: run this "
                                        "batch size once (or call reserve_workspace) before capturing")
            if buf is not None:
                _WORKSPACE_RETIRED.append(buf)
            buf = torch.empty(need, dtype=torch.uint8, device=self.device)
            _WORKSPACE_POOL[self.device] = buf
        self._ws = buf
        return buf

    def reserve_workspace(self, max_tokens: int) -> None:
        """Sizes the device's scratch pool for batches of up to `max_tokens` tokens ahead of time."""
        self._workspace(max_tokens)

    def _prep(self, hidden_states: torch.Tensor) -> torch.Tensor:
        if not hidden_states.is_cuda:
            raise _lib.ChronosError("hidden_states must be a CUDA tensor: chronos_b200 has no CPU path")
        x = hidden_states.reshape(-1, self.hidden)
        if x.dtype not in _DTYPES:
            x = x.to(torch.bfloat16)
        return x.contiguous()

    @staticmethod
    def _stream() -> int:
        return torch.cuda.current_stream().cuda_stream

    def device_status(self) -> int:
        """Status word of the last forward (synchronises). 0 = no device-side anomaly; see the C header for bits."""
        if self._ws is None or self._last_n == 0:
            return 0
        off = _lib.lib().chronos_b200_workspace_status_offset(self.packed.ptr, self._last_n)
        if off < 0:
            raise _lib.ChronosError("workspace_status_offset rejected the layer description")
        return int(self._ws[off:off + 4].view(torch.int32).item())

    def _after_call(self) -> None:
        if self.check_status:
            st = self.device_status()
            if st != 0:
                raise _lib.ChronosError(f"device status word 0x{st:x} after the forward: a kernel gave up a bounded wait "
                                        "(bits are listed in include/chronos_b200.h); the output of this call is invalid")

    def load_weights(self, weights: Iterable[tuple[str, torch.Tensor]]) -> set[str]:
        """Drains and ignores vLLM's weight stream (chronos_1t/models/glm53_chronos_moe.py:386-389)."""
        for _ in weights:
            pass
        return set()

    # -- reference-shaped API -----------------------------------------------------------------------------------------
    @torch.no_grad()
    def route(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """ids int32 [T, top_k], weights f32 [T, top_k] (chronos_1t/models/glm53_chronos_moe.py:392-399 /
        chronos_1t/models/vllm_chronos_moe.py:310-314, per the layer's router flavour)."""
        x = self._prep(x)
        n = x.shape[0]
        ids = torch.empty((n, self.top_k), dtype=torch.int32, device=self.device)
        w = torch.empty((n, self.top_k), dtype=torch.float32, device=self.device)
        logits = torch.empty((n, self.cfg.router_experts), dtype=torch.float32, device=self.device)
        _lib.check(_lib.lib().chronos_b200_router_topk(self.packed.router_ptr, x.data_ptr(), _DTYPES[x.dtype], n, ids.data_ptr(),
                                                     w.data_ptr(), logits.data_ptr(), self._stream()))
        self.last_logits = logits
        return ids, w

    @torch.no_grad()
    def route_coalesced(self, x: torch.Tensor, tokens_per_stream: int = 3, pool: int = 12, keep: int = 4,
                        bonus: float = 1.0e4) -> tuple[torch.Tensor, torch.Tensor]:
        """Batch-coalesced routing for speculative verify batches (streams of `tokens_per_stream` tokens, token 0 of each
        the anchor): the anchor keeps its natural top-k; a draft keeps its `keep` best natural experts and fills the rest from
        its own natural top-`pool`, preferring experts the anchor selected. Fewer distinct banks per step, no token ever
        routed outside its natural top-`pool`. A clean-room stand-in for the policy the reference describes in prose only
        (README.md:56, :208, :372). Returns (ids, weights) for `routed_forward`."""
        x = self._prep(x)
        n = x.shape[0]
        ids = torch.empty((n, self.top_k), dtype=torch.int32, device=self.device)
        w = torch.empty((n, self.top_k), dtype=torch.float32, device=self.device)
        logits = torch.empty((n, self.cfg.router_experts), dtype=torch.float32, device=self.device)
        _lib.check(_lib.lib().chronos_b200_router_topk_coalesced(self.packed.router_ptr, x.data_ptr(), _DTYPES[x.dtype], n, int(tokens_per_stream),
                                                               int(pool), int(keep), float(bonus), ids.data_ptr(), w.data_ptr(),
                                                               logits.data_ptr(), self._stream()))
        self.last_logits = logits
        return ids, w

    route_global = route  # expert-parallel shards: ids index the full (replicated) router table

    @torch.no_grad()
    def routed_forward(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, with_shared: bool = False,
                       out_dtype: torch.dtype | None = None, regime: str = "auto",
                       shared_range: tuple[int, int] | None = None) -> torch.Tensor:
        """Routed experts for caller-supplied routing (chronos_1t/models/glm53_chronos_moe.py:441-472). Entries with
        ids < 0 are skipped. `with_shared` adds the shared expert for every token; `shared_range = (first, count)`
        only for that block of tokens (an expert-parallel rank: the tokens it is the home of)."""
        x = self._prep(x)
        n = x.shape[0]
        out_dtype = out_dtype or x.dtype
        y = torch.empty((n, self.hidden), dtype=out_dtype, device=self.device)
        if n == 0:
            return y
        ids = ids.to(device=self.device, dtype=torch.int32).contiguous()
        w = w.to(device=self.device, dtype=torch.float32).contiguous()
        ws = self._workspace(n)
        self._last_n = n
        sh_first, sh_count = shared_range if shared_range is not None else ((0, n) if with_shared else (0, 0))
        _lib.check(_lib.lib().chronos_b200_folded_moe_routed(self.packed.ptr, x.data_ptr(), _DTYPES[x.dtype], n, ids.data_ptr(),
                                                           w.data_ptr(), int(sh_first), int(sh_count), _REGIMES[regime], y.data_ptr(), _DTYPES[out_dtype],
                                                           ws.data_ptr(), ws.numel(), self._stream()))
        self._after_call()
        return y

    @torch.no_grad()
    def forward_impl(self, hidden_states: torch.Tensor, regime: str = "auto") -> torch.Tensor:
        """Router + routed experts + shared expert (chronos_1t/models/glm53_chronos_moe.py:474-483). fp32 inputs stay
        fp32 end to end; anything else is computed from bf16 activations. `regime`: "auto" (by batch shape),
        "stream_fp4" (HBM-bound pass on the block-scaled FP4 tensor cores), "stream" (HBM-bound pass with CUDA-core
        conversion), "tensor_fp4" (block-scaled FP4 grouped GEMM, both operands streamed) or "tensor" (fp16 tcgen05
        grouped GEMM with the bank converted on the fly)."""
        orig_shape, orig_dtype = hidden_states.shape, hidden_states.dtype
        x = self._prep(hidden_states)
        n = x.shape[0]
        if regime in ("stream", "tensor") and n:  # regimes without a whole-layer entry point of their own
            ids, w = self.route(x)
            y = self.routed_forward(x, ids, w, with_shared=True, out_dtype=x.dtype, regime=regime)
            return y.to(orig_dtype).view(orig_shape)
        y = torch.empty_like(x)
        if n:
            ws = self._workspace(n)
            self._last_n = n
            fn = {"auto": _lib.lib().chronos_b200_folded_moe_forward, "stream_fp4": _lib.lib().chronos_b200_folded_moe_decode,
                  "tensor_fp4": _lib.lib().chronos_b200_folded_moe_prefill}[regime]
            _lib.check(fn(self.packed.ptr, x.data_ptr(), _DTYPES[x.dtype], n, y.data_ptr(),
                          _DTYPES[x.dtype], ws.data_ptr(), ws.numel(), self._stream()))
            self._after_call()
        return y.to(orig_dtype).view(orig_shape)

    def forward(self, hidden_states: torch.Tensor, *args: Any, **kwargs: Any) -> torch.Tensor:
        return self.forward_impl(hidden_states)

    def extra_repr(self) -> str:
        c = self.cfg
        return (f"layer={self.layer_idx}, hidden={c.hidden}, inter={c.inter}, experts={c.n_experts}, fold={c.group_size}, "
                f"rank={c.rank}, top_k={c.top_k}, router={c.router}, shared={self.n_shared_experts}")

    def resident_bytes(self) -> dict[str, int]:
        return {"gpu": self.packed.resident_bytes(), "host": 0}


def residual_rmsnorm(h: torch.Tensor, y: torch.Tensor | None, weight: torch.Tensor | None = None, eps: float = 1e-6) -> torch.Tensor:
    """In place h += y, returns RMSNorm(h) (chronos_1t/models/glm53_engine.py:71-73, :203), fp32 math on the device."""
    if not h.is_cuda:
        raise _lib.ChronosError("residual_rmsnorm needs CUDA tensors")
    n, hidden = h.shape
    out = torch.empty_like(h)
    _lib.check(_lib.lib().chronos_b200_residual_rmsnorm(h.data_ptr(), y.data_ptr() if y is not None else None,
                                                      weight.data_ptr() if weight is not None else None, out.data_ptr(),
                                                      _DTYPES[h.dtype], n, hidden, float(eps), torch.cuda.current_stream().cuda_stream))
    return out
