"""The real checkpoint's expert formats on the GPU (Q8_0, IQ4_NL, IQ3_S next to IQ4_XS):
the device decode against the reference's `gguf.quants.dequantize` outputs (fixtures made by
importing the reference, bitwise) and against the oracle's C restatement on every byte pattern
(random bytes, non-finite scales included), and the MoE block in the format mix the reference
loads (IQ3_S gate|up, IQ4_NL down, IQ3_S / Q8_0 shared expert; tt/plan.py:90-103) against the
reference's `_moe` (reference/model.py:387-417) and the oracle at the checkpoint's dimensions.

Tolerance of the block: relative max error 1e-2 of max |out| (the block runs on the integer core:
int8 weight words against x and h in block floating point, int16 mantissas per 32 values, then
fp32 accumulation, against the reference's fp32 matmuls)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu

TOL = 1e-2
FMTS = {"Q8_0": 8, "IQ4_NL": 20, "IQ3_S": 21, "IQ4_XS": 23}
BLOCK = {8: (32, 34), 20: (32, 18), 21: (256, 110), 23: (256, 136)}


def _same_bits(a: np.ndarray, b: np.ndarray) -> None:
    """Bitwise equality, any NaN matching any NaN (payloads are not part of the format)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    assert a.shape == b.shape
    both_nan = np.isnan(a) & np.isnan(b)
    diff = (a.view(np.uint32) != b.view(np.uint32)) & ~both_nan
    assert not diff.any(), f"{int(diff.sum())} values differ, first at {np.argwhere(diff)[:3].ravel()}"


def _dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("name", ["Q8_0", "IQ4_NL", "IQ3_S"])
def test_dequant_matches_reference_fixture(pkg, name):
    g = load_golden("formats_dequant.npz")
    out = pkg.dequant(FMTS[name], _dev(g[name + "_raw"])).cpu().numpy()
    _same_bits(out, g[name + "_out"])


@pytest.mark.parametrize("name", list(FMTS))
def test_dequant_random_bytes_match_oracle(pkg, oracle, name):
    fmt = FMTS[name]
    bv, bb = BLOCK[fmt]
    rng = np.random.default_rng(fmt)
    for n_blocks in (1, 7, 4099):
        raw = rng.integers(0, 256, size=(n_blocks * bb,), dtype=np.uint8)
        out = pkg.dequant(fmt, _dev(raw)).cpu().numpy()
        _same_bits(out, oracle.dequant(fmt, raw))
    rows = rng.integers(0, 256, size=(3, 5, 2 * bb), dtype=np.uint8)
    out = pkg.dequant(fmt, _dev(rows)).cpu().numpy()
    assert out.shape == (3, 5, 2 * bv)
    _same_bits(out, oracle.dequant(fmt, rows.reshape(-1)).reshape(3, 5, 2 * bv))


def _layer_dev(lay: dict) -> dict:
    return {k: (_dev(v) if isinstance(v, np.ndarray) else v) for k, v in lay.items()}


def _run(pkg, d: dict, x: torch.Tensor, top_k: int) -> np.ndarray:
    return pkg.moe_block_formats(x.cuda(), d["router"], d["gate_vec"], d["gate_up"], d["down"],
                                 d["sh_gate_up"], d["sh_down"], d["formats"], top_k).cpu().numpy()


def _rel(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.abs(a - b).max() / max(float(np.abs(b).max()), 1e-30))


@pytest.fixture(scope="module")
def small_layer(oracle):
    g = load_golden("formats_moe_m1.npz")
    return oracle.synth_formats_layer(int(g["seed"]), 64, 512, 256, 256)


@pytest.mark.parametrize("m", [1, 4])
def test_block_matches_reference_fixture(pkg, small_layer, m):
    g = load_golden(f"formats_moe_m{m}.npz")
    x = torch.from_numpy(g["x_bf16"]).view(torch.bfloat16)
    out = _run(pkg, _layer_dev(small_layer), x, 10)
    assert out.shape == g["out"].shape
    assert _rel(out, g["out"]) < TOL


def _oracle_block(oracle, lay: dict, x: torch.Tensor, k: int) -> np.ndarray:
    E, D = lay["router"].shape
    I = lay["gate_up"].shape[1] // 2
    Ish = lay["sh_gate_up"].shape[0] // 2
    src = oracle.ExpertSource(lambda e: (lay["gate_up"][e], lay["down"][e]), lay["sh_gate_up"], lay["sh_down"],
                              lay["router"], lay["gate_vec"], I, Ish, formats=lay["formats"])
    return oracle.moe_forward(x.float().numpy(), src, k)["out"]


@pytest.mark.parametrize("m", [2, 8, 16])
def test_block_small_matches_oracle(pkg, oracle, small_layer, m):
    x = (torch.randn(m, 512, generator=torch.Generator().manual_seed(m)) * 0.5).to(torch.bfloat16)
    out = _run(pkg, _layer_dev(small_layer), x, 10)
    assert _rel(out, _oracle_block(oracle, small_layer, x, 10)) < TOL


def test_block_checkpoint_dims_matches_oracle(pkg, oracle):
    """hidden 2048, 512 experts, top-10, inter 512, shared inter 512: the checkpoint's shapes."""
    lay = oracle.synth_formats_layer(43, 512, 2048, 512, 512)
    d = _layer_dev(lay)
    for m in (1, 4):
        x = (torch.randn(m, 2048, generator=torch.Generator().manual_seed(100 + m)) * 0.5).to(torch.bfloat16)
        out = _run(pkg, d, x, 10)
        assert np.isfinite(out).all()
        assert _rel(out, _oracle_block(oracle, lay, x, 10)) < TOL


def test_block_iq4xs_formats_match_block(pkg):
    """All four tensors IQ4_XS: the formats entry point and the IQ4_XS block agree."""
    cfg = pkg.MoEConfig(hidden=512, inter=256, n_experts=64, top_k=10, shared_inter=256)
    hl = pkg.synth_host_layer(cfg, layer=0, seed=5, all_experts=True)
    dl = pkg.upload_host_layer(hl, device="cuda")
    x = (torch.randn(3, 512, generator=torch.Generator().manual_seed(9)) * 0.5).to(torch.bfloat16).cuda()
    ref = pkg.MoELayer(dl)(x).float().cpu().numpy()
    out = pkg.moe_block_formats(x, dl.router, dl.gate_vec, dl.gate_up, dl.down, dl.sh_gate_up, dl.sh_down,
                                (23, 23, 23, 23), 10).cpu().numpy()
    assert _rel(out, ref.reshape(out.shape)) < 1e-4


def test_formats_rejects_bad_arguments(pkg, small_layer):
    d = _layer_dev(small_layer)
    x = torch.zeros(1, 512, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        pkg.moe_block_formats(x.cuda(), d["router"], d["gate_vec"], d["gate_up"], d["down"], d["sh_gate_up"],
                              d["sh_down"], (21, 20, 21, 99), 10)
    with pytest.raises(ValueError):
        pkg.dequant(99, torch.zeros(34, dtype=torch.uint8, device="cuda"))
    raw = torch.zeros(64, dtype=torch.uint8, device="cuda")
    out = torch.empty(64, dtype=torch.float32, device="cuda")
    assert pkg._lib.lib.qmoe_dequant_f32(99, raw.data_ptr(), 32, out.data_ptr(), None) != 0
    assert pkg._lib.lib.qmoe_dequant_f32(8, raw.data_ptr(), 33, out.data_ptr(), None) != 0


@pytest.mark.parametrize("formats", [(21, 8, 21, 8), (20, 20, 20, 20), (8, 8, 8, 8), (23, 21, 8, 20)],
                         ids=["iq3s-q8_0", "iq4nl", "q8_0", "mixed"])
def test_block_other_format_mixes_match_oracle(pkg, oracle, formats):
    """Other mixes the block accepts: the checkpoint's first layers (Q8_0 down), all IQ4_NL, all
    Q8_0, and a mix with IQ3_S down rows; seeded bytes, the oracle decoding the same bytes."""
    E, D, I, Ish = 64, 512, 256, 256
    fg, fd, fsg, fsd = formats
    seed = 50 + fg + fd
    lay = {
        "formats": formats,
        "gate_up": oracle.synth_format_bytes(fg, seed, 1, E * 2 * I, D, 2e-4).reshape(E, 2 * I, -1),
        "down": oracle.synth_format_bytes(fd, seed, 2, E * D, I, 2e-4).reshape(E, D, -1),
        "sh_gate_up": oracle.synth_format_bytes(fsg, seed, 3, 2 * Ish, D, 2e-4),
        "sh_down": oracle.synth_format_bytes(fsd, seed, 4, D, Ish, 2e-4),
        "router": oracle.synth_f32(seed, 5, E * D, 0.02).reshape(E, D),
        "gate_vec": oracle.synth_f32(seed, 6, D, 0.02),
    }
    d = _layer_dev(lay)
    for m in (1, 5):
        x = (torch.randn(m, D, generator=torch.Generator().manual_seed(seed + m)) * 0.5).to(torch.bfloat16)
        out = _run(pkg, d, x, 10)
        assert np.isfinite(out).all()
        assert _rel(out, _oracle_block(oracle, lay, x, 10)) < TOL


def test_formats_rejects_misaligned_weights(pkg, small_layer):
    """Weight tensors must start 16-byte aligned: an offset view is refused before any launch."""
    d = _layer_dev(small_layer)
    x = torch.zeros(1, 512, dtype=torch.bfloat16, device="cuda")
    flat = torch.zeros(d["down"].numel() + 2, dtype=torch.uint8, device="cuda")
    shifted = flat[2:].view(d["down"].shape)   # 2 bytes off a 256-byte boundary
    shifted.copy_(d["down"])
    with pytest.raises(RuntimeError) as e:
        pkg.moe_block_formats(x, d["router"], d["gate_vec"], d["gate_up"], shifted, d["sh_gate_up"], d["sh_down"],
                              d["formats"], 10)
    assert e.value.status == pkg._lib.QMOE_ERR_ALIGNMENT
