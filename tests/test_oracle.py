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


# ---- the synthetic-weight generator: the oracle's C restatement vs the product ----------------

GEN_CASES = [(0, (3 << 40) | (4 << 32) | 17, 2 * 512 * 2048, 0.02), (7, 12345, 256 * 64, 1.0),
             (2**40 + 5, 2**63 + 9, 256 * 8, 0.5), (0, (47 << 40) | (5 << 32) | 511, 2048 * 512, 0.02)]


@pytest.mark.parametrize("seed,sid,n,std", GEN_CASES)
def test_generator_restatement_is_byte_exact(pkg, oracle, seed, sid, n, std):
    """The oracle's own generator (synth_ref.c) gives the product host generator's bytes, both the
    fp32 stream and its IQ4_XS form; the oracle's quantiser matches the product's on that stream."""
    L = pkg._lib
    want_q = np.empty(n // 256 * 136, np.uint8)
    want_f = np.empty(n, np.float32)
    L.check(L.lib.qmoe_synth_iq4xs_host(seed, sid, n, std, want_q.ctypes.data, 4), "synth_iq4xs_host")
    L.check(L.lib.qmoe_synth_f32_host(seed, sid, n, std, want_f.ctypes.data, 4), "synth_f32_host")
    got_f = oracle.synth_f32(seed, sid, n, std)
    got_q = oracle.synth_iq4xs(seed, sid, n, std)
    assert np.array_equal(got_f.view(np.uint32), want_f.view(np.uint32))
    assert np.array_equal(got_q, want_q)
    assert np.array_equal(oracle.quantize_iq4xs(got_f.reshape(-1, 256)).reshape(-1), want_q)
    assert np.array_equal(pkg.weights.quantize_host(got_f.reshape(-1, 256)).reshape(-1), want_q)


def test_generator_is_standard_normal(oracle):
    z = oracle.synth_f32(1, 1, 1 << 22, 1.0).astype(np.float64)
    assert abs(z.mean()) < 3e-3 and abs(z.std() - 1.0) < 3e-3
    assert abs((np.abs(z) > 2).mean() - 0.0455) < 2e-3
    assert abs((np.abs(z) > 3).mean() - 0.0027) < 4e-4
    # odd sizes: the tail of the last counter group is cut, the rest is the same stream
    assert np.array_equal(oracle.synth_f32(1, 1, 7, 1.0), z[:7].astype(np.float32))


def test_family_layer_matches_product_device_family_layout(pkg):
    """oracle.synth_family numbers the streams as the product's generator does (layer << 40 |
    tag << 32 | expert, with the product's tag values)."""
    from oracle import synth_family

    assert synth_family.sid(3, synth_family.TAG_DOWN, 9) == pkg.weights._sid(3, pkg.weights.TAG_DOWN, 9)
    for name in ("TAG_ROUTER", "TAG_GATE_VEC", "TAG_SH_GATE_UP", "TAG_SH_DOWN", "TAG_GATE_UP", "TAG_DOWN",
                 "TAG_X"):
        assert getattr(synth_family, name) == getattr(pkg.weights, name)
    x = synth_family.synth_x(512, 3, seed=5)
    assert np.array_equal(x, pkg.synth_x(pkg.MoEConfig(hidden=512), 3, seed=5).float().numpy())


def test_row_cache_is_lru_by_bytes():
    from oracle import synth_family

    c = synth_family.RowCache(limit_bytes=3 * 400)
    v0, v1 = c.view(0), c.view(1)
    row = (np.zeros(50, np.float64), np.zeros(50, np.float32))  # 600 bytes
    v0[1] = row
    v1[1] = row
    assert v0.get(1) is row                  # hit: (0, 1) becomes the most recent
    v1[2] = row                              # over the limit: evicts the least recent, (1, 1)
    assert v1.get(1) is None and v0.get(1) is row and v1.get(2) is row
    assert c.hits == 3 and c.misses == 1


def test_threshold_oracle_is_the_dense_chain_and_exact_without_ties(oracle):
    """route_threshold (the device select's tie-admitting mode) keeps what the ttnn chain keeps
    (tt/moe.py:318-327) and, with no tie at the k-th place, selects the exact top-k."""
    rng = np.random.default_rng(3)
    lg = rng.standard_normal((6, 512)).astype(np.float32)
    tenth = int(np.argsort(-lg[2], kind="stable")[9])
    others = [e for e in (40, 41, 42) if e != tenth]
    lg[2, others] = lg[2, tenth]  # a tie at the 10th place
    for bf16 in (False, True):
        ids, w = oracle.route_threshold(lg, 10, 16, probs_bf16=bf16)
        dense = oracle.route_threshold_dense(lg, 10, probs_bf16=bf16)
        for m in range(lg.shape[0]):
            kept = np.nonzero(dense[m] > 0)[0]
            assert set(ids[m][w[m] > 0].tolist()) == set(kept.tolist())
            np.testing.assert_allclose(w[m][w[m] > 0], dense[m][ids[m][w[m] > 0]], rtol=1e-6)
    ids, w = oracle.route_threshold(lg, 10, 16)
    assert (w[2] > 0).sum() == 10 + len(others)  # the tie admitted
    for m in (0, 1, 3):
        probs = oracle.softmax(lg[m:m + 1])
        _, top = oracle.topk_canonical(probs, 10)
        assert np.array_equal(ids[m][:10], top[0])
        assert np.all(w[m][10:] == 0) and np.all(ids[m][10:] == 0)
    # a window keeps only its experts, normalised over all that pass
    wi, ww = oracle.route_threshold(lg, 10, 16, e_lo=256, e_hi=512)
    for m in range(lg.shape[0]):
        sel = wi[m][ww[m] > 0]
        assert np.all((sel >= 256) & (sel < 512))
        assert set(sel.tolist()) == set(e for e in ids[m][w[m] > 0].tolist() if e >= 256)


@pytest.mark.parametrize("name", ["small", "c1"])
def test_hc_oracle_matches_reference_fixture(name):
    """oracle/hc_ref.py against the reference's own _gated_residual / _reinject outputs."""
    from oracle import hc_ref

    g = load_golden(f"hc_{name}.npz")
    D, hc, r, m, seed = (int(g[k]) for k in ("hidden", "hc", "rank", "n_tokens", "seed"))
    w = hc_ref.synth_weights(seed, D, hc, r)
    hyper, branch = hc_ref.synth_inputs(seed, D, hc, m)
    o = hc_ref.gated_residual(hyper, w, float(g["eps"]), hc, D)
    for got, ref in ((o["mixed"], g["mixed"]), (o["inject"], g["inject"]),
                     (hc_ref.reinject(hyper, branch, o["inject"]), g["reinjected"])):
        assert float(np.abs(got - ref).max() / np.abs(ref).max()) < 1e-6


def test_format_oracles_match_reference_dequant(oracle):
    """oracle/formats_ref.c (Q8_0, IQ4_NL, IQ3_S) bit for bit against the reference's dequantize,
    non-finite and zero scales included."""
    g = load_golden("formats_dequant.npz")
    for name, fmt in (("Q8_0", oracle.Q8_0), ("IQ4_NL", oracle.IQ4_NL), ("IQ3_S", oracle.IQ3_S)):
        got = oracle.dequant(fmt, g[f"{name}_raw"].reshape(1, -1))[0]
        ref = g[f"{name}_out"]
        assert np.array_equal(got.view(np.uint32)[np.isfinite(ref)], ref.view(np.uint32)[np.isfinite(ref)]), name
        assert np.array_equal(np.isnan(got), np.isnan(ref)) and np.array_equal(np.isinf(got), np.isinf(ref)), name


@pytest.mark.parametrize("m", [1, 4])
def test_format_moe_oracle_matches_reference(oracle, m):
    """The oracle's _moe on a layer of IQ3_S gate|up, IQ4_NL down and a Q8_0 shared down against
    the reference's own _moe on the same bytes."""
    import torch

    g = load_golden(f"formats_moe_m{m}.npz")
    lay = oracle.synth_formats_layer(int(g["seed"]), 64, 512, 256, 256)
    src = oracle.ExpertSource(lambda e: (lay["gate_up"][e], lay["down"][e]), lay["sh_gate_up"], lay["sh_down"],
                              lay["router"], lay["gate_vec"], 256, 256, formats=lay["formats"])
    x = torch.from_numpy(g["x_bf16"]).view(torch.bfloat16).float().numpy()
    got = oracle.moe_forward(x, src, 10)["out"]
    assert oracle.max_rel_err(got, g["out"]) < 1e-5
