"""The C-ABI library loads, exports every declared entry point, and rejects
bad arguments on the host (no GPU needed: each check returns before any CUDA
call)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> list[str]:
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"\b(qmoe_\w+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ("qmoe_moe_block", "qmoe_route", "qmoe_gateup_swiglu", "qmoe_down_combine",
              "qmoe_stack_decode", "qmoe_dequant_iq4xs_f32", "qmoe_shared_expert"):
        assert n in names


def test_library_exports_every_declared_symbol(pkg):
    lib = ctypes.CDLL(str(pkg._lib.LIB_PATH))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_covers_every_declared_symbol(pkg):
    assert set(declared_symbols()) <= set(pkg._lib.EXPORTED)


def test_status_strings(pkg):
    lib = pkg._lib.lib
    assert lib.qmoe_status_string(0) == b"ok"
    assert lib.qmoe_status_string(6) == b"expert id out of range"
    assert lib.qmoe_status_string(99) == b"unknown status"
    assert lib.qmoe_version() >= 1
    assert lib.qmoe_max_tokens() == 16


def test_workspace_bytes_and_shape_checks(pkg):
    lib = pkg._lib.lib
    d = pkg.Shard().dims(pkg.C1)
    n = lib.qmoe_workspace_bytes(ctypes.byref(d), 1)
    assert n > 0 and n % 256 == 0
    assert lib.qmoe_workspace_bytes(ctypes.byref(d), 8) > n
    assert lib.qmoe_workspace_bytes(ctypes.byref(d), 17) == 0          # too many tokens
    bad = pkg.Shard().dims(pkg.C1)
    bad.hidden = 2000                                                    # not a multiple of 256
    assert lib.qmoe_workspace_bytes(ctypes.byref(bad), 1) == 0
    bad = pkg.Shard().dims(pkg.C1)
    bad.top_k = 0
    assert lib.qmoe_workspace_bytes(ctypes.byref(bad), 1) == 0
    bad = pkg.Shard().dims(pkg.C1)
    bad.down_nsub = 3                                                    # 2 x 3 x 32 != 512
    assert lib.qmoe_workspace_bytes(ctypes.byref(bad), 1) == 0


def test_entry_points_reject_bad_arguments(pkg):
    L = pkg._lib
    lib = L.lib
    d = pkg.Shard().dims(pkg.C1)
    w = L.LayerWeights()
    fake = 0x1000  # never dereferenced: every call below fails validation first
    # null activations / weights / workspace
    assert lib.qmoe_moe_block(None, 0, 1, ctypes.byref(w), ctypes.byref(d), fake, fake, 1 << 20, None) == L.QMOE_ERR_INVALID_ARG
    w.router = fake
    w.gate_up = fake
    w.down = fake
    w.sh_gate_up = fake
    w.sh_down = fake
    assert lib.qmoe_moe_block(fake, 0, 1, ctypes.byref(w), ctypes.byref(d), fake, None, 0, None) == L.QMOE_ERR_WORKSPACE
    assert lib.qmoe_moe_block(fake, 0, 1, ctypes.byref(w), ctypes.byref(d), fake, fake, 16, None) == L.QMOE_ERR_WORKSPACE
    assert lib.qmoe_moe_block(fake, 0, 0, ctypes.byref(w), ctypes.byref(d), fake, fake, 1 << 20, None) == L.QMOE_ERR_UNSUPPORTED
    assert lib.qmoe_moe_block(fake, 0, 17, ctypes.byref(w), ctypes.byref(d), fake, fake, 1 << 20, None) == L.QMOE_ERR_UNSUPPORTED
    assert lib.qmoe_moe_block(fake, 7, 1, ctypes.byref(w), ctypes.byref(d), fake, fake, 1 << 20, None) == L.QMOE_ERR_INVALID_ARG
    # misaligned router / workspace
    w.router = fake + 4
    assert lib.qmoe_moe_block(fake, 0, 1, ctypes.byref(w), ctypes.byref(d), fake, fake, 1 << 20, None) == L.QMOE_ERR_ALIGNMENT
    w.router = fake
    assert lib.qmoe_moe_block(fake, 0, 1, ctypes.byref(w), ctypes.byref(d), fake, fake + 8, 1 << 20, None) == L.QMOE_ERR_ALIGNMENT
    # a shard that expects a shared expert but has none
    w.sh_gate_up = None
    assert lib.qmoe_moe_block(fake, 0, 1, ctypes.byref(w), ctypes.byref(d), fake, fake, 1 << 20, None) == L.QMOE_ERR_INVALID_ARG
    # dequant / quantise arguments
    assert lib.qmoe_dequant_iq4xs_f32(None, 4, fake, None) == L.QMOE_ERR_INVALID_ARG
    assert lib.qmoe_dequant_iq4xs_f32(fake, -1, fake, None) == L.QMOE_ERR_INVALID_ARG
    assert lib.qmoe_dequant_iq4xs_f32(fake + 4, 4, fake, None) == L.QMOE_ERR_ALIGNMENT
    assert lib.qmoe_dequant_iq4xs_f32(None, 0, None, None) == L.QMOE_OK
    assert lib.qmoe_quantize_iq4xs(fake, 100, fake, None) == L.QMOE_ERR_INVALID_ARG
    # stack: no layers
    assert lib.qmoe_stack_decode(fake, 1, None, 48, ctypes.byref(d), fake, fake, 1 << 20, None) == L.QMOE_ERR_INVALID_ARG


def test_host_quantiser_round_trip(pkg, oracle):
    rng = np.random.default_rng(5)
    vals = (rng.standard_normal((64, 512)) * 0.02).astype(np.float32)
    q = pkg.weights.quantize_host(vals)
    assert q.shape == (64, 2 * 136)
    deq = oracle.dequant_iq4xs(q)
    rel = np.linalg.norm(deq - vals) / np.linalg.norm(vals)
    assert rel < 0.12, rel  # 4.25-bit non-linear code on Gaussian data
    assert np.array_equal(q, pkg.weights.quantize_host(vals, n_threads=1))  # deterministic, thread-independent


def test_host_quantiser_edge_values(pkg, oracle):
    vals = np.zeros((4, 256), np.float32)
    vals[1, 7] = 3.0                           # one spike
    vals[2] = np.linspace(-1, 1, 256)          # both signs
    vals[3] = 1e-30                            # tiny: the fp16 scale underflows
    q = pkg.weights.quantize_host(vals)
    deq = oracle.dequant_iq4xs(q)
    assert np.all(deq[0] == 0) or np.all(np.abs(deq[0]) < 1e-30)
    assert abs(deq[1, 7] - 3.0) < 0.05
    assert np.all(np.isfinite(deq))
    assert np.max(np.abs(deq[2] - vals[2])) < 0.1


def test_quantiser_rejects_partial_blocks(pkg):
    with pytest.raises(ValueError):
        pkg.weights.quantize_host(np.zeros((3, 100), np.float32))


def test_prefill_small_group_threshold(pkg):
    """The grouped-GEMV threshold: query, set, clamp to 8, restore (host state only)."""
    lib = pkg._lib.lib
    prev = lib.qmoe_prefill_small_group_max(-1)
    assert prev == 8
    assert lib.qmoe_prefill_small_group_max(3) == 8
    assert lib.qmoe_prefill_small_group_max(-1) == 3
    assert lib.qmoe_prefill_small_group_max(100) == 3
    assert lib.qmoe_prefill_small_group_max(-1) == 8
    lib.qmoe_prefill_small_group_max(prev)


def test_prefill_workspace_grows_with_the_chunk(pkg):
    """The prefill workspace covers the chunk's buffers (router split partials at small T, the
    small-group list and block-floating-point x) and grows with T."""
    import ctypes

    lib = pkg._lib.lib
    d = pkg.Shard().dims(pkg.C1)
    sizes = [lib.qmoe_prefill_workspace_bytes(ctypes.byref(d), t) for t in (1, 5, 64, 128, 300, 2048, 8192)]
    assert all(b > 0 for b in sizes)
    assert sizes == sorted(sizes)
    D, E, k = 2048, 512, 10
    for t, b in zip((128, 2048), (sizes[3], sizes[5])):
        rows = t * (k + 1)
        floor = t * D * 2 + t * (E + 1) * 4 + rows * 512 * 2 + rows * D * 2 + t * (D // 32) * 68
        assert b >= floor, (t, b, floor)
    # at T = 128 the router splits K eight ways: eight more logit planes than at T = 2048's share
    assert sizes[3] >= 128 * (E + 1) * 4 * 9


def test_single_launch_covers_rank_slices(pkg):
    """The stack's single launch runs the whole layer and every variant-B rank slice of the
    config-2 shape (one rank's chain, no exchange), not variant A or sliced-off shared experts."""
    import ctypes

    lib = pkg._lib.lib
    for world in (1, 2, 4, 8):
        for rank in range(world):
            shard = pkg.Shard("B", rank, world) if world > 1 else pkg.Shard()
            d = shard.dims(pkg.C2)
            assert lib.qmoe_stack_single_launch(ctypes.byref(d), 1, 48) == 1, (world, rank)
            assert lib.qmoe_stack_single_launch(ctypes.byref(d), 2, 48) == 0
    da = pkg.Shard("A", 1, 2).dims(pkg.C2)
    assert lib.qmoe_stack_single_launch(ctypes.byref(da), 1, 48) == 0
