"""The stack sharded over ranks with the per-layer sum inside the kernel.

On one GPU: the single launch on one rank's variant-B slice (I / R local
rows; down rows cut inside super-blocks at 4 and 8 ranks) against the
per-layer launches on the same slice.  On two GPUs (skipped with fewer): two
processes (and 4 and 8 where the box has them) exchange partial rows over
NVLink inside `qmoe_stack_decode_xchg`; all end with bitwise the same output, equal to the unsharded stack within
the block tolerance, and a rank that never launches makes the other's
bounded wait end with QMOE_ERR_TIMEOUT (no hang, no fault).
"""

from __future__ import annotations

import os
import socket
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

TOL = 1e-2


def max_rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def well_conditioned(x: torch.Tensor, router: torch.Tensor, k: int, rel_gap: float = 1e-5) -> bool:
    p = torch.softmax(x.float() @ router.T, -1).sort(-1, descending=True).values
    return bool(((p[:, k - 1] - p[:, k]) > rel_gap * p[:, k - 1]).all())


@pytest.mark.parametrize("world,rank", [(2, 1), (4, 2), (8, 5)])
def test_stack_kernel_on_a_rank_slice(pkg, world, rank):
    """The chain of one rank's partials (each layer's partial output feeding
    the next, no exchange): single launch vs per-layer launches."""
    cfg = pkg.MoEConfig(n_layers=2)
    shard = pkg.Shard("B", rank, world)
    dls = [pkg.synth_device_layer(cfg, l, seed=7, shard=shard) for l in range(cfg.n_layers)]
    x = pkg.synth_x(cfg, 1, seed=7).cuda()
    act, checked = x, 0
    for n in range(1, cfg.n_layers + 1):
        st = pkg.MoEStack(dls[:n], max_tokens=1)
        assert st.single_launch(1)
        got = st.decode(x).clone()
        torch.cuda.synchronize()
        st.ws.raise_if_error("stack kernel on a rank slice")
        inp = act if n == 1 else act.to(torch.bfloat16)
        want = pkg.MoELayer(dls[n - 1])(inp)
        if well_conditioned(inp, dls[n - 1].router, cfg.top_k):
            assert max_rel_err(got, want) <= 2e-3, f"layers {n}"
            checked += 1
        act = want
    assert checked >= 1


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, n_layers: int, mode: str, out_dir: str) -> None:
    import datetime
    import sys

    import torch.distributed as dist

    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import __graft_entry__

        pkg = __graft_entry__.load_package()
        from importlib import import_module

        ShardedMoEStack = import_module(pkg.__name__ + ".dist").ShardedMoEStack
        cfg = pkg.MoEConfig(n_layers=n_layers)
        shard = pkg.Shard("B", rank, world)
        dls = [pkg.synth_device_layer(cfg, l, seed=3, shard=shard, device=dev) for l in range(n_layers)]
        x = pkg.synth_x(cfg, 1, seed=3).to(dev)
        if mode == "ok":
            stack = ShardedMoEStack(dls, max_tokens=1, exchange="kernel")
            outs, sts = [], []
            for _ in range(3):  # graph replays: the launch counter makes every exchange new
                outs.append(stack.decode(x).clone().cpu().numpy())
                torch.cuda.synchronize(dev)
                sts.append(stack.read_status())
            np.savez(Path(out_dir) / f"rank{rank}.npz", out=np.stack(outs), status=np.array(sts))
        else:  # "peer_absent": rank 0 launches once, rank 1 never does
            stack = ShardedMoEStack(dls, max_tokens=1, exchange="kernel", use_graph=False)
            st = -1
            if rank == 0:
                stack.x_in[:1].copy_(x)
                stack.run(1)
                torch.cuda.synchronize(dev)
                st = stack.read_status()
                assert torch.ones(4, device=dev).sum().item() == 4.0  # the context is still usable
            np.savez(Path(out_dir) / f"rank{rank}.npz", status=np.array([st]))
        stack.release()
    finally:
        dist.destroy_process_group()


def _spawn(world: int, n_layers: int, mode: str, out_dir: str) -> None:
    mp.start_processes(_rank_main, args=(world, _free_port(), n_layers, mode, out_dir), nprocs=world,
                       start_method="spawn", join=True)


@pytest.mark.timeout(900)
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("n_layers", [1, 2])
def test_ranks_exchange_inside_the_kernel(pkg, n_layers, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        _spawn(world, n_layers, "ok", d)
        rs = [np.load(Path(d) / f"rank{r}.npz") for r in range(world)]
        for r in rs:
            assert (r["status"] == 0).all()
            assert np.array_equal(r["out"], rs[0]["out"]), "ranks must hold the same bits"
        r0 = rs[0]
        assert np.array_equal(r0["out"][0], r0["out"][1]) and np.array_equal(r0["out"][1], r0["out"][2])
        got = torch.from_numpy(r0["out"][0])
    cfg = pkg.MoEConfig(n_layers=n_layers)
    dls = [pkg.synth_device_layer(cfg, l, seed=3) for l in range(n_layers)]
    x = pkg.synth_x(cfg, 1, seed=3).cuda()
    want = pkg.MoEStack(dls, max_tokens=1).decode(x).clone()
    torch.cuda.synchronize()
    assert max_rel_err(got, want) <= TOL


@pytest.mark.timeout(600)
def test_absent_peer_times_out_with_status():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from importlib import import_module

    lib = import_module("ttrunner_qwen38_flash_next_b200._lib")
    with tempfile.TemporaryDirectory() as d:
        _spawn(2, 1, "peer_absent", d)
        st = int(np.load(Path(d) / "rank0.npz")["status"][0])
    assert st == lib.QMOE_ERR_TIMEOUT
