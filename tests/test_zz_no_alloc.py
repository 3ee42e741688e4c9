"""The allocation-free reconstruction entry point, for callers that are not allowed to allocate device memory
(a serving process whose framework owns the whole GPU memory pool, or a step where allocator calls are forbidden).

It must give exactly what the caller-scratch entry point gives, on two calls in a row (the built-in scratch is shared
by all calls and keeps the previous call's contents), and refuse matrices beyond its stated limit.
Collected last on purpose: a run that stops at the first failure has then already run every other test."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_static_scratch_entry_matches_caller_scratch_entry():
    from chronos_b200 import FoldedLayerConfig, PackedLayer, _lib

    lib = _lib.lib()
    cfg = FoldedLayerConfig(hidden=512, inter=256, n_experts=8, group_size=4, rank=16, top_k=2)
    layer = PackedLayer.synthetic(cfg, seed=21, keep_disk_order=True)  # the probe reads the banks in their on-disk order
    stream = torch.cuda.current_stream().cuda_stream
    for which, (rows, cols) in enumerate(((2 * cfg.inter, cfg.hidden), (cfg.hidden, cfg.inter))):
        scratch = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
        # two calls in a row, different experts: the second must not be disturbed by what the first left behind
        for expert in (5, 2):
            ref = torch.empty((rows, cols), dtype=torch.float32, device="cuda")
            got = torch.full((rows, cols), float("nan"), dtype=torch.float32, device="cuda")
            _lib.check(lib.chronos_b200_unfold_expert_fp32(layer.ptr, expert, which, ref.data_ptr(), scratch.data_ptr(), stream))
            _lib.check(lib.chronos_b200_unfold_expert_fp32_static(layer.ptr, expert, which, got.data_ptr(), stream))
            torch.cuda.synchronize()
            assert torch.equal(got, ref), (which, expert)  # same kernels, same order of operations: bit-identical


def test_static_scratch_entry_rejects_oversized_matrices():
    from chronos_b200 import FoldedLayerConfig, PackedLayer, _lib

    lib = _lib.lib()
    cfg = FoldedLayerConfig(hidden=4096, inter=1536, n_experts=4, group_size=4, rank=16, top_k=2)  # 3072 x 4096 > limit
    layer = PackedLayer.synthetic(cfg, seed=22, keep_disk_order=True)
    out = torch.empty((2 * cfg.inter, cfg.hidden), dtype=torch.float32, device="cuda")
    rc = lib.chronos_b200_unfold_expert_fp32_static(layer.ptr, 0, 0, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == -1
    msg = lib.chronos_b200_last_error().decode()
    assert "4194304" in msg and "scratch" in msg
    with pytest.raises(_lib.ChronosError):
        _lib.check(rc)
