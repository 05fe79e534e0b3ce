"""Chunked prefill (grouped tcgen05 GEMMs, and the grouped GEMV for experts
with at most 8 tokens) vs the CPU oracle.

one layer of the config-1 shape (hidden 2048, inter 512,
512 experts, top-10 + shared), chunks of T = 128 and 2048 tokens, x ~ N(0,1)
bf16; plus ragged chunk sizes (a partial tile, a shared group of three
n-tiles), fp32 input, and externally supplied routing.  Bars: routed ids
exact (rows whose 10th/11th probabilities are well separated: the router is
an fp32 GEMM whose summation order differs from numpy's), output max relative
error <= 1e-2 (bf16 weights and activations into fp32 tensor-core
accumulation).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from test_gpu_parity import TOL, device_layer

pytestmark = pytest.mark.gpu


def _x(T: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(T, 2048, generator=g).to(torch.bfloat16)


def _oracle(oracle, hl, x_bf16: torch.Tensor, k: int) -> dict:
    src = oracle.ExpertSource.from_host_layer(hl)
    return oracle.moe_forward(x_bf16.float().numpy(), src, k)


def _rows_ok(probs: np.ndarray, k: int) -> np.ndarray:
    p = -np.sort(-probs, axis=-1)
    return (p[:, k - 1] - p[:, k]) > 1e-5 * p[:, k - 1]


@pytest.fixture(scope="module")
def c1(pkg):
    g = load_golden("moe_c1_m1.npz")
    hl, dl = device_layer(pkg, g)
    return hl, dl, pkg.MoELayer(dl)


@pytest.mark.parametrize("T", [128, 2048, 37, 300])
def test_prefill_matches_oracle(pkg, oracle, c1, T):
    hl, dl, layer = c1
    x = _x(T, seed=100 + T)
    ref = _oracle(oracle, hl, x, hl.cfg.top_k)
    ids, w, sl = layer.prefill_route(x.cuda())
    ok = _rows_ok(ref["probs"], hl.cfg.top_k)
    assert ok.mean() > 0.9
    got_ids = ids.cpu().numpy()
    assert np.array_equal(got_ids[ok], ref["ids"][ok]), "routed ids differ on well-separated rows"
    np.testing.assert_allclose(w.cpu().numpy()[ok], ref["weights"][ok], rtol=1e-4, atol=1e-6)
    out = layer.prefill(x.cuda())
    torch.cuda.synchronize()
    pkg.moe.prefill_workspace_for(layer.dims, T, out.device).raise_if_error("prefill")
    err = oracle.max_rel_err(out.cpu().numpy(), ref["out"])
    assert err <= TOL, f"T={T}: max rel err {err:.3e}"
    # per token too: every row within the bar relative to its own scale
    got = out.cpu().numpy().astype(np.float64)
    r = ref["out"].astype(np.float64)
    row_err = np.max(np.abs(got - r), axis=1) / np.max(np.abs(r), axis=1)
    assert float(np.max(row_err)) <= 5 * TOL


def test_prefill_fp32_input_and_repeat(pkg, oracle, c1):
    hl, dl, layer = c1
    x = _x(64, seed=5)
    ref = _oracle(oracle, hl, x, hl.cfg.top_k)
    out32 = layer.prefill(x.float().cuda())
    out16 = layer.prefill(x.cuda())
    torch.cuda.synchronize()
    assert oracle.max_rel_err(out32.cpu().numpy(), ref["out"]) <= TOL
    # fp32 input is rounded to bf16 first, so both are the same computation
    assert oracle.max_rel_err(out32.cpu().numpy(), out16.cpu().numpy()) <= 1e-5


def test_prefill_experts_given_routing(pkg, oracle, c1):
    """apply_experts with the oracle's routing (tt/moe.py:330-368) + shared expert; an
    out-of-range id is skipped and reported."""
    hl, dl, layer = c1
    T, k = 96, hl.cfg.top_k
    x = _x(T, seed=9)
    ref = _oracle(oracle, hl, x, k)
    ids = torch.from_numpy(ref["ids"].astype(np.int32)).cuda()
    w = torch.from_numpy(ref["weights"]).cuda()
    sl = torch.from_numpy((x.float().numpy() @ hl.gate_vec.reshape(-1, 1)).reshape(-1).astype(np.float32)).cuda()
    out = layer.prefill_experts(x.cuda(), ids, w, sl)
    torch.cuda.synchronize()
    pws = pkg.moe.prefill_workspace_for(layer.dims, T, out.device)
    pws.raise_if_error("prefill_experts")
    assert oracle.max_rel_err(out.cpu().numpy(), ref["out"]) <= TOL

    bad = ids.clone()
    bad[3, 0] = hl.cfg.n_experts + 5
    w_bad = w.clone()
    out_bad = layer.prefill_experts(x.cuda(), bad, w_bad, sl)
    torch.cuda.synchronize()
    assert pws.read_status() == pkg._lib.QMOE_ERR_DEVICE_RANGE
    # the other tokens are untouched by the skipped pair
    keep = np.ones(T, dtype=bool)
    keep[3] = False
    assert oracle.max_rel_err(out_bad.cpu().numpy()[keep], ref["out"][keep]) <= TOL


def test_prefill_operator_api(pkg, oracle, c1):
    """route / apply_experts on raw tensors take the chunked path above 16 tokens."""
    hl, dl, layer = c1
    T, k = 48, hl.cfg.top_k
    x = _x(T, seed=21).cuda()
    dense_w, keep = pkg.route(x, dl.router, k)
    ref = _oracle(oracle, hl, x.cpu(), k)
    ok = _rows_ok(ref["probs"], k)
    ids = torch.topk(keep, k, dim=-1).indices.sort(dim=-1).values.cpu().numpy()
    assert np.array_equal(ids[ok], np.sort(ref["ids"], axis=-1)[ok])
    routed = pkg.apply_experts(x, dense_w, keep, dl.gate_up, None, dl.down, hl.cfg.n_experts,
                               hl.cfg.hidden, hl.cfg.inter)
    torch.cuda.synchronize()
    assert oracle.max_rel_err(routed.cpu().numpy(), ref["routed"]) <= TOL


def test_prefill_matches_decode_path(pkg, c1):
    """At 16 tokens the prefill path and the decode kernels compute the same block."""
    hl, dl, layer = c1
    x = _x(16, seed=33).cuda()
    a = layer.prefill(x)
    b = layer(x)
    torch.cuda.synchronize()
    d = (a - b).abs().max().item() / b.abs().max().item()
    assert d <= TOL


@pytest.mark.parametrize("T", [5, 128, 300])
def test_prefill_small_groups_both_paths(pkg, oracle, c1, T):
    """The same chunk with every group on the tensor cores and with the small
    groups (<= 8 tokens; at T = 5 the shared group too) on the grouped GEMV:
    both within the bar of the oracle and of each other."""
    hl, dl, layer = c1
    x = _x(T, seed=200 + T)
    ref = _oracle(oracle, hl, x, hl.cfg.top_k)
    lib = pkg._lib.lib
    prev = lib.qmoe_prefill_small_group_max(0)
    try:
        tc = layer.prefill(x.cuda()).clone()
        lib.qmoe_prefill_small_group_max(8)
        gv = layer.prefill(x.cuda()).clone()
    finally:
        lib.qmoe_prefill_small_group_max(prev)
    torch.cuda.synchronize()
    pkg.moe.prefill_workspace_for(layer.dims, T, gv.device).raise_if_error("prefill")
    assert oracle.max_rel_err(tc.cpu().numpy(), ref["out"]) <= TOL
    assert oracle.max_rel_err(gv.cpu().numpy(), ref["out"]) <= TOL
    assert oracle.max_rel_err(gv.cpu().numpy(), tc.cpu().numpy()) <= TOL


def test_prefill_pipeline_trace_opt_in(pkg, c1):
    """qmoe_prefill_trace: off by default; when on, CTA 0 of the grouped GEMM stamps its
    pipeline clock per A slot into workspace bytes 256 .. 4351 (the MMA thread's waits and
    issues of the first slots non-zero and ordered); the output is the same either way, up to the
    order of the scatter-adds."""
    hl, dl, layer = c1
    lib = pkg._lib.lib
    x = _x(256, seed=77).cuda()
    prev_small = lib.qmoe_prefill_small_group_max(0)
    try:
        assert lib.qmoe_prefill_trace(-1) == 0
        ws = pkg.moe.prefill_workspace_for(layer.dims, 256, x.device)
        ws.buf[256:256 + 64 * 64].zero_()
        plain = layer.prefill(x).clone()
        torch.cuda.synchronize()
        assert int(ws.buf[256:256 + 64 * 64].count_nonzero()) == 0
        assert lib.qmoe_prefill_trace(1) == 0
        traced = layer.prefill(x).clone()
        torch.cuda.synchronize()
        tr = ws.buf[256:256 + 64 * 64].view(torch.int64).view(64, 8).cpu().numpy()
    finally:
        lib.qmoe_prefill_trace(0)
        lib.qmoe_prefill_small_group_max(prev_small)
    assert lib.qmoe_prefill_trace(-1) == 0
    ws.raise_if_error("prefill")
    # slot 0: MMA thread past its wait (event 1), MMAs issued (event 3)
    assert tr[0, 1] > 0 and tr[0, 3] >= tr[0, 1]
    # the same result up to the order of the scatter-adds (float atomics from several CTAs)
    assert float((plain - traced).abs().max()) <= 1e-5 * float(plain.abs().max())
