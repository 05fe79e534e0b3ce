"""The hyper-connection mixer kernels (csrc/hc.cu) against the reference's own
outputs (tests/golden/hc_*.npz, from Qwen4ExpModel._gated_residual /
_reinject, reference/model.py:53-81) and against the oracle at a wider
shape, bf16 and fp32 streams.  fp32 arithmetic with another summation
order: 1e-5 relative."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu

TOL = 1e-5


def rel(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / np.abs(b).max())


def _weights(hc_ref, seed, D, hc, r):
    return {k: torch.from_numpy(v).cuda() for k, v in hc_ref.synth_weights(seed, D, hc, r).items()}


@pytest.mark.parametrize("name", ["small", "c1"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_hc_mix_matches_reference(pkg, name, dtype):
    from oracle import hc_ref

    g = load_golden(f"hc_{name}.npz")
    D, hc, r, m, seed = (int(g[k]) for k in ("hidden", "hc", "rank", "n_tokens", "seed"))
    w = _weights(hc_ref, seed, D, hc, r)
    hyper, branch = hc_ref.synth_inputs(seed, D, hc, m)
    h = torch.from_numpy(hyper).cuda().to(dtype).reshape(1, 1, m, hc * D)  # bf16-exact values
    mixed, inject = pkg.gated_residual_mix(h, w["norm_w"], w["down_w"], w["up_w"], w["inject_w"],
                                           float(g["eps"]), hc, D)
    out = pkg.reinject(h, torch.from_numpy(branch).cuda().to(dtype).reshape(1, 1, m, D), inject, hc)
    torch.cuda.synchronize()
    assert mixed.shape == (1, 1, m, D) and inject.shape == (1, 1, m, hc) and out.shape == (1, 1, m, hc * D)
    assert rel(mixed.cpu().numpy().reshape(m, D), g["mixed"]) < TOL
    assert rel(inject.cpu().numpy().reshape(m, hc), g["inject"]) < TOL
    assert rel(out.cpu().numpy().reshape(m, hc * D), g["reinjected"]) < TOL


@pytest.mark.parametrize("m", [1, 5, 16])
def test_hc_mix_matches_oracle_wide(pkg, m):
    """A 4 x 2048 stream set with a 256-wide gate, 1..16 tokens (several staged groups)."""
    from oracle import hc_ref

    D, hc, r, seed = 2048, 4, 256, 31
    w = _weights(hc_ref, seed, D, hc, r)
    wn = hc_ref.synth_weights(seed, D, hc, r)
    hyper, branch = hc_ref.synth_inputs(seed, D, hc, m)
    h = torch.from_numpy(hyper).cuda()
    mixed, inject = pkg.gated_residual_mix(h, w["norm_w"], w["down_w"], w["up_w"], w["inject_w"], 1e-6, hc, D)
    out = pkg.reinject(h, torch.from_numpy(branch).cuda(), inject, hc)
    torch.cuda.synchronize()
    ref = hc_ref.gated_residual(hyper, wn, 1e-6, hc, D)
    assert rel(mixed.cpu().numpy(), ref["mixed"]) < TOL
    assert rel(inject.cpu().numpy(), ref["inject"]) < TOL
    assert rel(out.cpu().numpy(), hc_ref.reinject(hyper, branch, ref["inject"])) < TOL


def test_hc_around_the_block(pkg, oracle):
    """mix -> MoE block -> reinject, the model's order (reference/model.py:454-455), against the
    oracle chain on the same weights."""
    from oracle import hc_ref

    cfg = pkg.MoEConfig(hidden=512, inter=256, n_experts=64, top_k=10, shared_inter=256)
    hl = pkg.synth_host_layer(cfg, layer=0, seed=5, all_experts=True)
    dl = pkg.upload_host_layer(hl, device="cuda")
    hc, r, m = 4, 64, 3
    wn = hc_ref.synth_weights(9, cfg.hidden, hc, r)
    w = {k: torch.from_numpy(v).cuda() for k, v in wn.items()}
    hyper, _ = hc_ref.synth_inputs(9, cfg.hidden, hc, m)
    h = torch.from_numpy(hyper).cuda()
    mixed, inject = pkg.gated_residual_mix(h, w["norm_w"], w["down_w"], w["up_w"], w["inject_w"], 1e-6, hc,
                                           cfg.hidden)
    branch = pkg.MoELayer(dl)(mixed.to(torch.bfloat16))
    out = pkg.reinject(h, branch, inject, hc)
    torch.cuda.synchronize()
    ref = hc_ref.gated_residual(hyper, wn, 1e-6, hc, cfg.hidden)
    xb = ref["mixed"].astype(np.float32)
    xb = torch.from_numpy(xb).to(torch.bfloat16).float().numpy()
    blk = oracle.moe_forward(xb, oracle.ExpertSource.from_host_layer(hl), cfg.top_k)
    want = hc_ref.reinject(hyper, blk["out"], ref["inject"])
    assert rel(out.cpu().numpy(), want) < 1e-2
