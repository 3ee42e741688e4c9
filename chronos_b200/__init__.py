"""chronos_b200: B200 (sm_100a) native folded-expert MoE forward behind the Chronos plugin / operator boundary."""
from .layout import FoldedLayerConfig, PackedLayer  # noqa: F401
from .moe import LIVE_BLOCKS, FoldedMoELayer, residual_rmsnorm  # noqa: F401

__all__ = ["FoldedLayerConfig", "PackedLayer", "FoldedMoELayer", "LIVE_BLOCKS", "residual_rmsnorm"]
