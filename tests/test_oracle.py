"""The CPU oracle pinned against the reference's own outputs (tests/golden/)."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from conftest import golden_x, host_layer_for, load_golden

MOE_CASES = ["small_m1", "small_m4", "tie_m2", "c1_m1", "c1_m4", "c1_m8"]


def test_dequant_random_bytes_match_reference(oracle):
    g = load_golden("iq4xs_dequant.npz")
    mine = oracle.dequant_iq4xs(g["raw_random"])
    fin = g["finite_random"]
    assert np.array_equal(mine[fin], g["out_random"][fin])
    # non-finite scales decode to the same non-finite class
    assert np.array_equal(np.isnan(mine), np.isnan(g["out_random"]))
    assert np.array_equal(np.isinf(mine), np.isinf(g["out_random"]))


def test_dequant_quantiser_blocks_match_reference(oracle):
    g = load_golden("iq4xs_dequant.npz")
    assert np.array_equal(oracle.dequant_iq4xs(g["raw_quant"]), g["out_quant"])
    assert np.array_equal(oracle.dequant_iq4xs_numpy(g["raw_quant"]), g["out_quant"])


def test_numpy_restatement_matches_c(oracle):
    g = load_golden("iq4xs_dequant.npz")
    a = oracle.dequant_iq4xs(g["raw_random"])
    b = oracle.dequant_iq4xs_numpy(g["raw_random"])
    fin = np.isfinite(a)
    assert np.array_equal(a[fin], b[fin])


def test_dequant_empty(oracle):
    assert oracle.dequant_iq4xs(np.zeros((0, 136), np.uint8)).shape == (0, 256)


def test_golden_weights_regenerate_identically(pkg):
    """The host generator + quantiser still produce the bytes the goldens were made from."""
    g = load_golden("moe_small_m1.npz")
    hl = host_layer_for(pkg, g)
    digests = dict(s.split("=") for s in g["digest"])
    assert hashlib.sha256(hl.router.tobytes()).hexdigest() == digests["blk.0.ffn_gate_inp.weight"]
    assert hashlib.sha256(hl.sh_down.tobytes()).hexdigest() == digests["blk.0.ffn_down_shexp.weight"]
    assert hashlib.sha256(hl.sh_gate_up[: hl.cfg.shared_inter].tobytes()).hexdigest() == \
        digests["blk.0.ffn_gate_shexp.weight"]


@pytest.mark.parametrize("case", MOE_CASES)
def test_oracle_matches_reference_moe(pkg, oracle, case):
    g = load_golden(f"moe_{case}.npz")
    hl = host_layer_for(pkg, g)
    x = golden_x(g).float().numpy()
    r = oracle.moe_forward(x, oracle.ExpertSource.from_host_layer(hl), int(g["top_k"]))
    assert np.array_equal(r["ids"], g["ids"]), "expert ids differ from the reference"
    np.testing.assert_allclose(r["weights"], g["weights"], rtol=1e-5, atol=1e-7)
    assert oracle.max_rel_err(r["out"], g["out"]) < 1e-5


def test_tie_case_is_lower_index(pkg, oracle):
    g = load_golden("moe_tie_m2.npz")
    k = int(g["top_k"])
    assert np.array_equal(g["ids"], np.tile(np.arange(k), (g["ids"].shape[0], 1)))
    # the reference's raw CPU topk does not pick the lower ids: canonicalisation matters
    assert not np.array_equal(np.sort(g["raw_ids"], 1), g["ids"])
    np.testing.assert_allclose(g["weights"], 1.0 / k, rtol=1e-6)


def test_topk_canonical_orders_ties_by_index(oracle):
    p = np.array([[0.1, 0.3, 0.3, 0.2, 0.3]], dtype=np.float32)
    v, i = oracle.topk_canonical(p, 3)
    assert i.tolist() == [[1, 2, 4]]


def test_max_rel_err_definition(oracle):
    ref = np.array([1.0, -4.0, 2.0])
    assert oracle.max_rel_err(ref + np.array([0, 0.04, 0]), ref) == pytest.approx(0.01)
    assert oracle.max_rel_err(np.zeros(3), np.zeros(3)) == 0.0


def test_warm_cache_is_the_same_computation(pkg, oracle):
    """moe_forward with the dequantised experts cached (the warm CPU baseline) equals the cold
    call bit for bit, on a first and a repeated call."""
    g = load_golden("moe_small_m4.npz")
    hl = host_layer_for(pkg, g, all_experts=True)
    src = oracle.ExpertSource.from_host_layer(hl)
    x = golden_x(g).float().numpy()
    cold = oracle.moe_forward(x, src, hl.cfg.top_k)["out"]
    cache: dict = {}
    first = oracle.moe_forward(x, src, hl.cfg.top_k, cache=cache)["out"]
    again = oracle.moe_forward(x, src, hl.cfg.top_k, cache=cache)["out"]
    assert "shared" in cache and len(cache) > 1
    assert np.array_equal(cold, first) and np.array_equal(cold, again)
