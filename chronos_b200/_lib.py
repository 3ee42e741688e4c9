"""ctypes binding of libchronos_b200.so (the C ABI declared in include/chronos_b200.h).

There is deliberately no fallback: if the shared library is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libchronos_b200.so"

DTYPE_F32, DTYPE_BF16 = 0, 1
ROUTER_SOFTMAX_TOPK, ROUTER_SIGMOID_NOAUX, ROUTER_SQRT_SOFTPLUS = 0, 1, 2
ABI_VERSION = 11
REGIME_AUTO, REGIME_STREAM, REGIME_TENSOR, REGIME_STREAM_FP4, REGIME_TENSOR_FP4 = 0, 1, 2, 3, 4


class ChronosError(RuntimeError):
    """A non-zero status from the C ABI."""


class LayerStruct(C.Structure):
    """Mirror of `chronos_layer_t`."""

    _fields_ = (
        [(n, C.c_int32) for n in ("hidden", "inter", "n_experts", "group_size", "n_slots", "rank", "top_k",
                                  "router_kind", "renorm")]
        + [("routed_scaling", C.c_float), ("shared_inter", C.c_int32), ("tail_bits", C.c_int32)]
        + [(n, C.c_void_p) for n in (
            "router_w", "e_bias",
            "gu_w", "gu_s", "gu_s2", "gu_beta", "dn_w", "dn_s", "dn_s2", "dn_beta",
            "u_gu", "v_gu", "u_dn", "v_dn_t",
            "gu_cin", "gu_cs2", "gu_rout", "gu_rs2", "dn_cin", "dn_cs2", "dn_rout", "dn_rs2",
            "sh_gu_w", "sh_gu_s", "sh_gu_s2", "sh_dn_w", "sh_dn_s", "sh_dn_s2",
            "gu_t", "dn_t", "sh_gu_t", "sh_dn_t", "v_dn",
            "tail_gu_p", "tail_gu_s", "tail_dn_p", "tail_dn_s",
            "sh8_gu_w", "sh8_gu_s", "sh8_dn_w", "sh8_dn_s", "ut_gu", "ut_dn", "ut_scale")]
    )


EXPORTS = {
    "chronos_b200_abi_version": (C.c_int, []),
    "chronos_b200_last_error": (C.c_char_p, []),
    "chronos_b200_dequant_nvfp4": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "chronos_b200_dequant_fp8_block": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "chronos_b200_unfold_expert_fp32": (C.c_int, [C.POINTER(LayerStruct), C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "chronos_b200_unfold_expert_fp32_static": (C.c_int, [C.POINTER(LayerStruct), C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "chronos_b200_router_topk": (C.c_int, [C.POINTER(LayerStruct), C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "chronos_b200_router_topk_coalesced": (C.c_int, [C.POINTER(LayerStruct), C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "chronos_b200_workspace_bytes": (C.c_size_t, [C.POINTER(LayerStruct), C.c_int]),
    "chronos_b200_fp4_mma_probe": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "chronos_b200_ep_pack": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                      C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_long, C.c_void_p]),
    "chronos_b200_ep_pack_peer": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                           C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "chronos_b200_ep_send_back_peer": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                                C.c_int, C.c_void_p]),
    "chronos_b200_ep_barrier": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_uint32, C.c_void_p, C.c_void_p]),
    "chronos_b200_ep_unpack_meta": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_long, C.c_int,
                                             C.c_void_p]),
    "chronos_b200_ep_combine": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                         C.c_int, C.c_void_p]),
    "chronos_b200_wait_probe": (C.c_int, [C.c_void_p, C.c_uint, C.c_void_p]),
    "chronos_b200_set_stage_events": (C.c_int, [C.POINTER(C.c_void_p), C.c_int]),
    "chronos_b200_workspace_status_offset": (C.c_long, [C.POINTER(LayerStruct), C.c_int]),
    "chronos_b200_folded_moe_decode": (C.c_int, [C.POINTER(LayerStruct), C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]),
    "chronos_b200_folded_moe_prefill": (C.c_int, [C.POINTER(LayerStruct), C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]),
    "chronos_b200_folded_moe_forward": (C.c_int, [C.POINTER(LayerStruct), C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]),
    "chronos_b200_folded_moe_routed": (C.c_int, [C.POINTER(LayerStruct), C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]),
    "chronos_b200_residual_rmsnorm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float, C.c_void_p]),
}

_LIB = None


def lib() -> C.CDLL:
    """Loads the shared library (once). Raises if it has not been built: there is no CPU path."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise ChronosError(
                f"{LIB_PATH} is missing: build it with `python -m chronos_b200.build` (needs nvcc, sm_100a). "
                "chronos_b200 has no CPU or PyTorch fallback."
            )
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in EXPORTS.items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = res, args
        if handle.chronos_b200_abi_version() != ABI_VERSION:
            raise ChronosError("libchronos_b200.so was built from a different ABI version: rebuild it")
        _LIB = handle
    return _LIB


def check(status: int) -> None:
    if status != 0:
        msg = lib().chronos_b200_last_error().decode("utf-8", "replace")
        raise ChronosError(f"chronos_b200 status {status}: {msg}")
