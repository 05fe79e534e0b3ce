"""qmoe_moe_block_noalloc: the MoE block for callers that cannot allocate
device memory (hosts bound through a plain C ABI without a device allocator,
plug-ins whose process's device memory is owned by another framework's
allocator, serving loops that forbid allocation after start-up).  Its scratch
is a fixed 1 MiB device array inside the library instead of a caller
workspace; qmoe_noalloc_read_status reads back the status word that array
holds.

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


def _noalloc_status(pkg) -> int:
    L = pkg._lib
    st = ctypes.c_int(-1)
    L.check(L.lib.qmoe_noalloc_read_status(ctypes.byref(st), torch.cuda.current_stream().cuda_stream),
            "qmoe_noalloc_read_status")
    return st.value


@pytest.mark.gpu
def test_noalloc_at_the_config1_shape(pkg):
    """BASELINE config 1's block (hidden 2048, 512 experts, top-10 + shared) with 16 tokens, the
    most the decode entry points take, fits the fixed array; two calls in a row equal the
    workspace entry point bit for bit."""
    L = pkg._lib
    cfg = pkg.C1
    d = pkg.Shard().dims(cfg)
    assert L.lib.qmoe_workspace_bytes(ctypes.byref(d), 16) <= (1 << 20)
    layer = pkg.MoELayer(pkg.synth_device_layer(cfg, 0, seed=11))
    _noalloc_status(pkg)  # start from a clear status word
    for seed in (1, 2):
        x = pkg.synth_x(cfg, 16, seed=seed).cuda()
        want = layer(x)
        got = _noalloc(pkg, layer, x)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert oracle_free_rel_err(got, want) <= TOL
        assert torch.equal(got, want)
    assert _noalloc_status(pkg) == L.QMOE_OK


@pytest.mark.gpu
def test_noalloc_reports_a_non_finite_router_logit(pkg):
    """The status the kernels record on the library's array is not lost: a non-finite input
    makes the router flag QMOE_ERR_NOT_FINITE, which qmoe_noalloc_read_status returns once."""
    L = pkg._lib
    g = load_golden("moe_small_m1.npz")
    hl = host_layer_for(pkg, g, all_experts=True)
    layer = pkg.MoELayer(pkg.upload_host_layer(hl, device="cuda"))
    _noalloc_status(pkg)
    x = golden_x(g).cuda().clone()
    x[0, 5] = float("inf")
    _noalloc(pkg, layer, x)
    torch.cuda.synchronize()
    assert _noalloc_status(pkg) == L.QMOE_ERR_NOT_FINITE
    assert _noalloc_status(pkg) == L.QMOE_OK  # the read cleared it
    out = _noalloc(pkg, layer, golden_x(g).cuda())  # and the next call is clean
    torch.cuda.synchronize()
    assert torch.isfinite(out).all() and _noalloc_status(pkg) == L.QMOE_OK


def oracle_free_rel_err(got: torch.Tensor, want: torch.Tensor) -> float:
    denom = want.abs().max().item()
    return (got.double() - want.double()).abs().max().item() / denom if denom else 0.0


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
