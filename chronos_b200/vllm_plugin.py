"""vLLM plugin / operator boundary of the folded MoE layer.

Same shape as the reference's boundary: a `vllm.general_plugins` entry point `register()`
(chronos_1t/vllm_plugin.py:15-38), a `torch.library` operator `moe_forward(hidden_states, layer_idx) -> Tensor` with
an `empty_like` fake implementation (chronos_1t/models/patch_glm53_vllm.py:79-93), and a class swap that keeps
`isinstance(layer.mlp, DeepseekV2MoE)` true and falls back to the stock class when a layer has no folded shard
(chronos_1t/models/patch_glm53_vllm.py:134-168).
"""
from __future__ import annotations

import json
import os
from pathlib import Path
from typing import Any, Callable

import torch

from .layout import FoldedLayerConfig, layer_index_from_prefix
from .moe import LIVE_BLOCKS, FoldedMoELayer

OP_NAME = "chronos_b200::moe_forward"
REFERENCE_OP_NAME = "chronos_glm53::moe_forward"  # the name the reference registers (chronos_1t/models/patch_glm53_vllm.py:79-93)
_OP_REGISTERED = False
MODEL_SITES = (
    "vllm.models.deepseek_v32.nvidia.model",
    "vllm.models.deepseek_v32.nvidia.mtp",
    "vllm.model_executor.models.deepseek_v2",
)


def _reference_op_taken() -> bool:
    """True when `torch.ops.chronos_glm53.moe_forward` already exists (the reference package registered it first)."""
    try:
        return hasattr(torch.ops.chronos_glm53, "moe_forward")
    except (AttributeError, RuntimeError):
        return False


def register_custom_op() -> None:
    """Registers `torch.ops.chronos_b200.moe_forward(hidden_states, layer_idx) -> Tensor` once, traceable by torch.compile
    through its `empty_like` fake impl, and the same operator under the reference's own name
    `torch.ops.chronos_glm53.moe_forward` (chronos_1t/models/patch_glm53_vllm.py:79-93) so that an unchanged caller of
    the reference resolves it - unless the reference package already registered that name in this process."""
    global _OP_REGISTERED
    if _OP_REGISTERED:
        return
    names = [OP_NAME] + ([] if _reference_op_taken() else [REFERENCE_OP_NAME])
    for name in names:
        @torch.library.custom_op(name, mutates_args=())
        def _moe_forward(hidden_states: torch.Tensor, layer_idx: int) -> torch.Tensor:
            return LIVE_BLOCKS[layer_idx].forward_impl(hidden_states)

        @_moe_forward.register_fake
        def _(hidden_states: torch.Tensor, layer_idx: int) -> torch.Tensor:
            return torch.empty_like(hidden_states)

    _OP_REGISTERED = True


def config_from_checkpoint(model_dir: Path) -> FoldedLayerConfig | None:
    """Builds the layer description from `config.json` (`chronos_holographic_moe` block written by
    chronos_1t/converter/convert_glm53_chronos.py:544-561 + the model's MoE fields)."""
    cfg_path = Path(model_dir) / "config.json"
    if not cfg_path.exists():
        return None
    try:
        cfg = json.loads(cfg_path.read_text())
    except (OSError, ValueError):
        return None
    holo = cfg.get("chronos_holographic_moe")
    if not isinstance(holo, dict):
        return None
    text = cfg.get("text_config", cfg)
    try:
        return FoldedLayerConfig(
            hidden=int(text["hidden_size"]), inter=int(text["moe_intermediate_size"]),
            n_experts=int(text["n_routed_experts"]), group_size=int(holo.get("group_size", 8)),
            rank=int(holo.get("svd_rank", 64)), top_k=int(text["num_experts_per_tok"]),
            router={"sigmoid": "sigmoid", "sqrtsoftplus": "sqrt_softplus", "sqrt_softplus": "sqrt_softplus"}.get(
                str(text.get("scoring_func", "sigmoid")), "softmax"),
            norm_topk_prob=bool(text.get("norm_topk_prob", True)),
            routed_scaling_factor=float(text.get("routed_scaling_factor", 2.5)),
            key_generator=str(holo.get("key_generator", "torch_cpu_v1")),
        )
    except (KeyError, TypeError, ValueError):
        return None


def find_layer_shard(model_dir: Path, layer_idx: int) -> Path | None:
    """`chronos-*-layer-XXXXX-of-NNNNN.safetensors` of a layer, if present."""
    hits = sorted(Path(model_dir).glob(f"chronos-*-layer-{layer_idx:05d}-of-*.safetensors"))
    hits = [h for h in hits if "-hot" not in h.name and "-tiers-" not in h.name]
    return hits[0] if hits else None


def make_hooked_class(orig_cls: type, model_dir_of: Callable[[], Path | None]) -> type:
    """A type (not a factory function) to put in place of the module-global `DeepseekV2MoE`, so `isinstance` checks
    against that global keep working: `__new__` hands back the stock class when the layer has no folded shard,
    otherwise a `FoldedMoELayer` whose `forward` goes through the custom op."""

    class ChronosB200VllmMoE(FoldedMoELayer):
        _chronos_b200 = True
        _orig_moe_cls = orig_cls

        def __new__(cls, *args: Any, **kwargs: Any) -> Any:
            l_idx = layer_index_from_prefix(kwargs.get("prefix", ""))
            mdir = model_dir_of()
            if l_idx is not None and mdir is not None and config_from_checkpoint(mdir) is not None \
                    and find_layer_shard(mdir, l_idx) is not None:
                return super().__new__(cls)
            return cls._orig_moe_cls(*args, **kwargs)

        def __init__(self, config: Any = None, parallel_config: Any = None, quant_config: Any = None,
                     reduce_results: bool = True, prefix: str = "", apply_routed_scale_to_output: bool = False,
                     **kwargs: Any) -> None:
            mdir = model_dir_of()
            l_idx = layer_index_from_prefix(prefix)
            super().__init__(layer_idx=l_idx, shard_path=find_layer_shard(mdir, l_idx), config=config_from_checkpoint(mdir),
                             prefix="")

        def forward(self, hidden_states: torch.Tensor, *args: Any, **kwargs: Any) -> torch.Tensor:
            return torch.ops.chronos_b200.moe_forward(hidden_states, self.layer_idx)

    return ChronosB200VllmMoE


def _model_dir(default_ckpt_dir: str | Path | None) -> Path | None:
    for env in ("CHRONOS_B200_CKPT", "CHRONOS_GLM53_CKPT"):
        if os.environ.get(env):
            return Path(os.environ[env])
    try:
        from vllm.config import get_current_vllm_config

        return Path(get_current_vllm_config().model_config.model)
    except Exception:
        return Path(default_ckpt_dir) if default_ckpt_dir else None


def enable_chronos_b200_vllm_hook(default_ckpt_dir: str | Path | None = None) -> bool:
    """Replaces `DeepseekV2MoE` in every vLLM model module that defines it. Returns True if any site was patched."""
    sites = []
    for mod_name in MODEL_SITES:
        try:
            mod = __import__(mod_name, fromlist=["DeepseekV2MoE"])
        except Exception:
            continue
        if getattr(mod, "DeepseekV2MoE", None) is not None:
            sites.append(mod)
    if not sites:
        return False
    if any(getattr(getattr(mod, "DeepseekV2MoE"), "_chronos_b200", False) for mod in sites):
        return True  # already hooked
    orig_cls = next((getattr(mod, "DeepseekV2MoE") for mod in sites if isinstance(getattr(mod, "DeepseekV2MoE"), type)), None)
    if orig_cls is None:
        return False
    register_custom_op()
    hooked = make_hooked_class(orig_cls, lambda: _model_dir(default_ckpt_dir))
    for mod in sites:
        setattr(mod, "_ChronosB200OrigDeepseekV2MoE", orig_cls)
        setattr(mod, "DeepseekV2MoE", hooked)
    return True


def register() -> None:
    """`vllm.general_plugins` entry point: every stage is allowed to fail without taking the worker down
    (chronos_1t/vllm_plugin.py:17-38)."""
    try:
        enable_chronos_b200_vllm_hook()
    except Exception:
        pass
