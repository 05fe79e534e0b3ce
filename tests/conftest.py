from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402

__graft_entry__._load_build_module().build()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run with -m gpu on a B200)")


@pytest.fixture(scope="session")
def pkg():
    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def oracle():
    from oracle import moe_ref

    moe_ref.build()
    return moe_ref


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / name, allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def golden_cfg(pkg, g: dict):
    return pkg.MoEConfig(hidden=int(g["hidden"]), inter=int(g["inter"]), n_experts=int(g["n_experts"]),
                         top_k=int(g["top_k"]), shared_inter=int(g["shared_inter"]),
                         weight_std=float(g["weight_std"]))


def golden_x(g: dict):
    import torch

    return torch.from_numpy(g["x_bf16"]).view(torch.bfloat16)


_HOST_LAYERS: dict = {}


def host_layer_for(pkg, g: dict, all_experts: bool = False):
    """The seeded host-family layer a golden case was made from (cached)."""
    cfg = golden_cfg(pkg, g)
    key = (cfg, int(g["seed"]))
    hl = _HOST_LAYERS.get(key)
    if hl is None:
        hl = _HOST_LAYERS[key] = pkg.synth_host_layer(cfg, layer=0, seed=int(g["seed"]))
    if "router_row0" in g:  # the tie case replaces the router
        import copy

        hl = copy.copy(hl)
        hl.router = np.repeat(g["router_row0"][None, :], cfg.n_experts, axis=0).astype(np.float32)
    if all_experts:
        hl.ensure_all()
    return hl


def needs_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
