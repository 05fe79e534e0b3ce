"""The tie-admitting threshold routing mode (the reference device select with
EXACT_TOPK off, scripts/kernels/router_select.cpp:223-255, and the ttnn chain
tt/moe.py:308-327) against the oracle's restatement, on the golden layers,
on a layer whose router rows tie at the k-th place, and through the block.

Selection compares probabilities; the device's logits and the oracle's come
from different summation orders (last-bit differences), so a row is compared
for its selected set only when no probability sits within 1e-5 (relative) of
the threshold without being exactly tied with it -- and, in the bf16 mode,
none within 1e-5 of a bf16 rounding boundary.  Exact ties (identical router
rows give bitwise identical logits on both sides) are compared always.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from conftest import golden_x, host_layer_for, load_golden

pytestmark = pytest.mark.gpu

TOL = 1e-2
CASES = ["small_m1", "small_m4", "tie_m2", "c1_m1", "c1_m4", "c1_m8"]
K_SEL = 16


def _probs(oracle, logits):
    return oracle.softmax(np.asarray(logits, dtype=np.float32))


def robust_rows(oracle, logits, k, probs_bf16):
    """Rows whose selection and weights cannot hinge on last-bit differences (module docstring):
    no probability within 1e-5 of the threshold unless exactly tied with it, and in the bf16 mode
    no kept or nearly kept probability within 64 fp32 ulps of a bf16 rounding midpoint."""
    p = _probs(oracle, logits)
    ok = []
    for row in p:
        good = True
        if probs_bf16:
            low = row.view(np.uint32).astype(np.int64) & 0xFFFF
            near_mid = np.abs(low - 0x8000) <= 64
            row = oracle.bf16_round(row)
            thr = np.sort(row)[::-1][k - 1]
            good = not np.any(near_mid & (row >= thr * (1 - 2.0 ** -7)))
        thr = np.sort(row)[::-1][k - 1]
        near = (row != thr) & (np.abs(row - thr) <= 1e-5 * thr)
        ok.append(good and not near.any())
    return np.array(ok)


def oracle_logits(hl, x):
    return (np.asarray(x, dtype=np.float64) @ hl.router.astype(np.float64).T).astype(np.float32)


def _layer(pkg, g):
    hl = host_layer_for(pkg, g, all_experts=True)
    dl = pkg.upload_host_layer(hl, device="cuda")
    return hl, dl


@pytest.mark.parametrize("probs_bf16", [False, True])
@pytest.mark.parametrize("case", CASES)
def test_threshold_route_matches_oracle(pkg, oracle, case, probs_bf16):
    g = load_golden(f"moe_{case}.npz")
    hl, dl = _layer(pkg, g)
    k = hl.cfg.top_k
    mode = "threshold_bf16" if probs_bf16 else "threshold"
    layer = pkg.MoELayer(dl, route_mode=mode)
    x = golden_x(g)
    ids, w, _ = layer.route(x.cuda())
    torch.cuda.synchronize()
    layer.ws.raise_if_error(case)
    ids, w = ids.cpu().numpy(), w.cpu().numpy()
    lg = oracle_logits(hl, x.float().numpy())
    rids, rw = oracle.route_threshold(lg, k, K_SEL, probs_bf16=probs_bf16)
    rob = robust_rows(oracle, lg, k, probs_bf16)
    assert rob.sum() >= 1, "no row is far enough from the threshold to compare"
    for m in np.nonzero(rob)[0]:
        assert np.array_equal(ids[m], rids[m]), f"{case} row {m}: {ids[m]} vs {rids[m]}"
        np.testing.assert_allclose(w[m], rw[m], rtol=1e-5, atol=1e-7)
    # at least k kept, weights of the kept sum to 1 when all fit in the slots
    kept = (w > 0).sum(-1)
    assert np.all(kept >= min(k, K_SEL))
    full = kept < K_SEL
    np.testing.assert_allclose(w[full].sum(-1), 1.0, rtol=1e-5)


def test_threshold_admits_exact_ties(pkg, oracle):
    """Router rows copied so that four experts tie exactly at the k-th place for token 0: the
    threshold mode keeps all of them (k + 3), the exact mode keeps the k lowest ids."""
    g = load_golden("moe_c1_m4.npz")
    hl, dl = _layer(pkg, g)
    k = hl.cfg.top_k
    x = golden_x(g)
    lg = oracle_logits(hl, x.float().numpy())
    order = np.argsort(-lg[0], kind="stable")
    src = int(order[k - 1])
    router = hl.router.copy()
    for e in order[k:k + 3]:
        router[int(e)] = router[src]
    dl2 = dataclasses.replace(dl, router=torch.from_numpy(router).cuda())
    lg2 = (x.float().numpy().astype(np.float64) @ router.astype(np.float64).T).astype(np.float32)
    assert len(set(lg2[0][[src] + [int(e) for e in order[k:k + 3]]].tolist())) == 1
    thr = pkg.MoELayer(dl2, route_mode="threshold")
    ids, w, _ = thr.route(x.cuda())
    exact = pkg.MoELayer(dl2)
    eids, _, _ = exact.route(x.cuda())
    torch.cuda.synchronize()
    ids, w, eids = ids.cpu().numpy(), w.cpu().numpy(), eids.cpu().numpy()
    assert (w[0] > 0).sum() == k + 3
    tied = sorted([src] + [int(e) for e in order[k:k + 3]])
    assert set(tied) <= set(ids[0][w[0] > 0].tolist())
    rids, rw = oracle.route_threshold(lg2, k, K_SEL)
    assert np.array_equal(ids[0], rids[0])
    np.testing.assert_allclose(w[0], rw[0], rtol=1e-5, atol=1e-7)
    # the exact select keeps k: the k - 1 above the tie, then the lowest tied id
    assert sorted(eids[0].tolist()) == sorted([int(e) for e in order[:k - 1]] + [tied[0]])


@pytest.mark.parametrize("mode", ["threshold", "threshold_bf16"])
def test_threshold_block_matches_oracle(pkg, oracle, mode):
    """The whole block in a threshold mode against the oracle's _moe fed the same selection."""
    g = load_golden("moe_c1_m4.npz")
    hl, dl = _layer(pkg, g)
    layer = pkg.MoELayer(dl, route_mode=mode)
    x = golden_x(g)
    out = layer(x.cuda())
    ids, w, _ = layer.route(x.cuda())
    torch.cuda.synchronize()
    layer.ws.raise_if_error(mode)
    ref = oracle.moe_forward(x.float().numpy(), oracle.ExpertSource.from_host_layer(hl), hl.cfg.top_k,
                             routing=(ids.cpu().numpy().astype(np.int64), w.cpu().numpy()))
    err = oracle.max_rel_err(out.cpu().numpy(), ref["out"])
    assert err <= TOL, err


def test_threshold_operator_and_prefill(pkg, oracle):
    """pkg.route(mode="threshold_bf16") is the ttnn chain's dense (weights, keep) wherever the kept
    set fits the 16 slots; a 40-token chunk takes the prefill router with the same select."""
    g = load_golden("moe_c1_m8.npz")
    hl, dl = _layer(pkg, g)
    k = hl.cfg.top_k
    x = golden_x(g)
    wd, keep = pkg.route(x.cuda(), dl.router, k, mode="threshold_bf16")
    torch.cuda.synchronize()
    lg = oracle_logits(hl, x.float().numpy())
    dense = oracle.route_threshold_dense(lg, k, probs_bf16=True)
    rob = robust_rows(oracle, lg, k, True)
    for m in np.nonzero(rob)[0]:
        if (dense[m] > 0).sum() <= K_SEL:
            assert np.array_equal(keep[m].cpu().numpy() > 0, dense[m] > 0)
            np.testing.assert_allclose(wd[m].cpu().numpy(), dense[m], rtol=1e-5, atol=1e-7)
    xt = pkg.synth_x(hl.cfg, 40, seed=5)
    pids, pw = pkg.route_threshold(xt.cuda(), dl.router, k, K_SEL, probs_bf16=False)
    torch.cuda.synchronize()
    lgt = oracle_logits(hl, xt.float().numpy())
    rids, rw = oracle.route_threshold(lgt, k, K_SEL)
    rob = robust_rows(oracle, lgt, k, False)
    assert rob.sum() >= 30
    for m in np.nonzero(rob)[0]:
        assert np.array_equal(pids[m].cpu().numpy(), rids[m])
        np.testing.assert_allclose(pw[m].cpu().numpy(), rw[m], rtol=1e-5, atol=1e-7)
