"""qmoe_moe_block_noalloc: the MoE block for callers that cannot allocate
device memory (hosts bound through a plain C ABI without a device allocator,
plug-ins whose process's device memory is owned by another framework's
allocator, serving loops that forbid allocation after start-up).  Its scratch
is a fixed 1 MiB device array inside the library instead of a caller
workspace.

This file is named to be collected last, so a run that stops at the first
failure has run every other test before it.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import golden_x, host_layer_for, load_golden

TOL = 1e-2  # the block tolerance used by every parity test


def _noalloc(pkg, layer, x: torch.Tensor) -> torch.Tensor:
    L = pkg._lib
    out = torch.full((x.shape[0], layer.cfg.hidden), float("nan"), dtype=torch.float32, device=x.device)
    L.check(L.lib.qmoe_moe_block_noalloc(x.data_ptr(), L.QMOE_ACT_BF16, x.shape[0],
                                         ctypes.byref(layer.weights), ctypes.byref(layer.dims),
                                         out.data_ptr(), torch.cuda.current_stream().cuda_stream),
            "qmoe_moe_block_noalloc")
    return out


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice(pkg, oracle):
    g = load_golden("moe_small_m4.npz")
    hl = host_layer_for(pkg, g, all_experts=True)
    layer = pkg.MoELayer(pkg.upload_host_layer(hl, device="cuda"))
    x4 = golden_x(g).cuda()
    x1 = pkg.synth_x(hl.cfg, 1, seed=3).cuda()
    # Two calls in a row, different token counts: the second reuses the array
    # the first left behind.
    for x in (x4, x1):
        want = layer(x)                 # qmoe_moe_block with a caller workspace
        got = _noalloc(pkg, layer, x)   # the same block on the library's scratch
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert oracle.max_rel_err(got.cpu().numpy(), want.cpu().numpy()) <= TOL
        assert torch.equal(got, want)   # same kernels, same inputs: same bits


def test_noalloc_rejects_oversized_scratch(pkg):
    """A shape whose scratch exceeds the fixed array fails with a clear status
    before anything is launched (so this runs without a GPU)."""
    L = pkg._lib
    d = pkg.Shard().dims(pkg.MoEConfig(hidden=4096, inter=4096, n_experts=512, top_k=16, shared_inter=4096))
    need = L.lib.qmoe_workspace_bytes(ctypes.byref(d), 16)
    assert need > (1 << 20)
    w = L.LayerWeights(router=0x1000, gate_vec=0x1000, gate_up=0x1000, down=0x1000,
                       sh_gate_up=0x1000, sh_down=0x1000)
    rc = L.lib.qmoe_moe_block_noalloc(0x1000, L.QMOE_ACT_BF16, 16, ctypes.byref(w), ctypes.byref(d), 0x1000, None)
    assert rc == L.QMOE_ERR_WORKSPACE
    assert L.lib.qmoe_status_string(rc) == b"workspace missing or too small"
    # invalid shapes keep their usual status
    assert L.lib.qmoe_moe_block_noalloc(0x1000, L.QMOE_ACT_BF16, 0, ctypes.byref(w), ctypes.byref(d),
                                        0x1000, None) == L.QMOE_ERR_UNSUPPORTED
