"""Shard descriptions (variants A and B), the row-slice byte format, and the
N>1 host logic: per-rank partial sums all-reduced over gloo ranks on CPU equal
the unsharded block."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import golden_x, host_layer_for, load_golden


def decode_row_slices(raw: np.ndarray, nseg: int, nsub: int, ib0: int) -> np.ndarray:
    """Decode rows stored as segments of (8-byte super-block header + nsub
    16-byte qs groups of sub-blocks ib0..ib0+nsub-1) -- the layout the device
    kernels read -- by re-assembling each segment into a full super-block."""
    rows = raw.reshape(-1, raw.shape[-1])
    seg_bytes = 8 + 16 * nsub
    full = np.zeros((rows.shape[0], nseg, 136), np.uint8)
    for s in range(nseg):
        seg = rows[:, s * seg_bytes:(s + 1) * seg_bytes]
        full[:, s, :8] = seg[:, :8]
        full[:, s, 8 + 16 * ib0:8 + 16 * (ib0 + nsub)] = seg[:, 8:]
    from oracle import moe_ref

    vals = moe_ref.dequant_iq4xs(full.reshape(rows.shape[0], -1)).reshape(rows.shape[0], nseg, 256)
    return vals[:, :, 32 * ib0:32 * (ib0 + nsub)].reshape(rows.shape[0], -1)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_variant_b_dims_and_slices(pkg, oracle, world):
    cfg = pkg.C1
    rng = np.random.default_rng(0)
    down = pkg.weights.quantize_host((rng.standard_normal((16, cfg.inter)) * 0.02).astype(np.float32))
    full = oracle.dequant_iq4xs(down)
    for r in range(world):
        sh = pkg.Shard("B", r, world)
        d = sh.dims(cfg)
        lo, hi = sh.inter_window(cfg.inter)
        assert d.inter_local == hi - lo == cfg.inter // world
        assert d.down_nseg * d.down_nsub * 32 == d.inter_local
        sl = pkg.weights.slice_down(down, lo, hi)
        assert sl.shape[-1] == d.down_nseg * (8 + 16 * d.down_nsub)
        got = decode_row_slices(sl, d.down_nseg, d.down_nsub, d.down_ib0)
        assert np.array_equal(got, full[:, lo:hi])
        assert d.sh_inter_local == cfg.shared_inter // world


def test_variant_b_bytes_per_rank(pkg):
    cfg = pkg.C1
    for world, per_row in [(1, 272), (2, 136), (4, 72), (8, 40)]:
        lo, hi = pkg.Shard("B", 0, world).inter_window(cfg.inter)
        assert pkg.weights.slice_down(np.zeros((1, 272), np.uint8), lo, hi).shape[-1] == per_row


@pytest.mark.parametrize("world", [2, 4, 8])
def test_variant_a_windows(pkg, world):
    cfg = pkg.C1
    wins = [pkg.Shard("A", r, world).expert_window(cfg) for r in range(world)]
    assert wins[0][0] == 0 and wins[-1][1] == cfg.n_experts
    assert all(a[1] == b[0] for a, b in zip(wins, wins[1:]))
    dims = [pkg.Shard("A", r, world).dims(cfg) for r in range(world)]
    assert dims[0].sh_inter_local == cfg.shared_inter
    assert all(d.sh_inter_local == 0 for d in dims[1:])   # shared expert on rank 0 only
    assert all(d.inter_local == cfg.inter for d in dims)


def test_bad_shards_raise(pkg):
    with pytest.raises(ValueError):
        pkg.Shard("C", 0, 1)
    with pytest.raises(ValueError):
        pkg.Shard("A", 2, 2)
    with pytest.raises(ValueError):
        pkg.Shard("B", 0, 3).inter_window(512)      # 512 / 3 is not a whole number of blocks
    with pytest.raises(ValueError):
        pkg.Shard.row_slice(16, 272)


def test_gate_up_slice_keeps_gate_and_up_rows(pkg):
    gu = np.arange(8 * 4).reshape(8, 4)            # 2*inter rows, inter = 4
    sl = pkg.weights.slice_gate_up(gu, 4, 1, 3)
    assert sl[:, 0].tolist() == [4, 8, 20, 24]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, variant: str, q) -> None:
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        import __graft_entry__
        from conftest import golden_x as gx, host_layer_for as hlf, load_golden as lg
        from oracle import moe_ref

        pkg = __graft_entry__.load_package()
        g = lg("moe_small_m4.npz")
        hl = hlf(pkg, g, all_experts=True)
        shard = pkg.Shard(variant, rank, world)
        x = gx(g).float().numpy()
        part = moe_ref.moe_forward(
            x, moe_ref.ExpertSource.from_host_layer(hl), hl.cfg.top_k, with_shared=shard.has_shared(),
            expert_window=shard.expert_window(hl.cfg) if variant == "A" else None,
            inter_window=shard.inter_window(hl.cfg.inter) if variant == "B" else None)["out"]
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        if rank == 0:
            q.put(t.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("variant", ["A", "B"])
def test_gloo_ranks_allreduce_partials(pkg, oracle, variant):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, variant, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    g = load_golden("moe_small_m4.npz")
    assert oracle.max_rel_err(got, g["out"]) < 1e-5


def test_rank_failure_surfaces_as_error():
    """A rank that never joins: the other rank's collective ends with an
    error inside the process-group timeout instead of hanging."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    p = ctx.Process(target=_lonely_rank, args=(port,))
    p.start()
    p.join(timeout=120)
    assert p.exitcode == 3, "the waiting rank should fail with a timeout error"


def _lonely_rank(port: int) -> None:
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=3))
        dist.all_reduce(torch.zeros(4))
    except Exception:  # noqa: BLE001 -- any error is the expected outcome
        os._exit(3)
    os._exit(0)


def test_exchange_host_logic(pkg):
    """In-kernel exchange: buffer sizes, and which dims it runs (host-side checks, no GPU)."""
    import ctypes

    lib = pkg._lib.lib
    assert lib.qmoe_xchg_bytes(2, 2048) == 128 + 2 * 2 * 2048 * 8
    assert lib.qmoe_xchg_bytes(8, 2048) == 128 + 2 * 8 * 2048 * 8
    assert lib.qmoe_xchg_bytes(9, 2048) == 0 and lib.qmoe_xchg_bytes(0, 2048) == 0
    cfg = pkg.C2
    for world in (2, 4, 8):
        for rank in (0, world - 1):
            d = pkg.Shard("B", rank, world).dims(cfg)
            assert lib.qmoe_stack_xchg_supported(ctypes.byref(d), world, 1, 48) == 1
            assert lib.qmoe_stack_xchg_supported(ctypes.byref(d), world, 2, 48) == 0  # one token only
            assert lib.qmoe_stack_xchg_supported(ctypes.byref(d), world, 1, 65) == 0
            other = 2 if world != 2 else 4
            assert lib.qmoe_stack_xchg_supported(ctypes.byref(d), other, 1, 48) == 0  # slice width != inter / R
    da = pkg.Shard("A", 0, 2).dims(cfg)
    assert lib.qmoe_stack_xchg_supported(ctypes.byref(da), 2, 1, 48) == 0
    dn = pkg.Shard().dims(cfg)
    assert lib.qmoe_stack_xchg_supported(ctypes.byref(dn), 1, 1, 48) == 0
    x = pkg._lib.Xchg(rank=0, n_ranks=2)
    dims = pkg.Shard("B", 0, 2).dims(cfg)
    # argument checks come before any device work
    assert lib.qmoe_stack_decode_xchg(None, 1, None, 1, ctypes.byref(dims), ctypes.byref(x), None, None, 0,
                                      None) == pkg._lib.QMOE_ERR_INVALID_ARG


def _gather_main(rank: int, world: int, port: int, q) -> None:
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        import __graft_entry__
        from importlib import import_module

        pkg = __graft_entry__.load_package()
        gather = import_module(pkg.__name__ + ".dist").gather_handles
        got = gather(bytes([rank]) * 64)
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_exchange_handles_gathered_in_rank_order(pkg):
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    want = [bytes([r]) * 64 for r in range(world)]
    assert all(res[r] == want for r in range(world))
