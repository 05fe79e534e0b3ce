"""Generate the golden fixtures of this directory from the reference itself.

Run where the reference checkout is available (read-only is enough), with
the environment variable REFERENCE_SRC naming its `src` directory, and its
`gguf` 0.19 dependency installed:

    REFERENCE_SRC=<checkout>/src python tests/golden/make_golden.py

What it records (all small, committed as .npz):

* iq4xs_dequant.npz -- IQ4_XS decode pins.  64 super-blocks of random bytes
  drawn exactly as the reference's tests/test_quants.py:19-42 draws them
  (rng seed 1234 + 23), plus 32 super-blocks of this project's quantiser
  output; each decoded by the reference's `dequantize`
  (gguf/quants.py:214 -> _dequant_iq4_xs :112-129) and, as a cross-check, by
  gguf 0.19.0 (the reference's pinned dependency, uv.lock:150-152).
* moe_*.npz -- outputs of the reference's CPU MoE, `Qwen4ExpModel._moe`
  (reference/model.py:387-417), run through its own `WeightStore`
  (reference/weights.py) over a duck-typed in-memory GGUF holding this
  project's seeded IQ4_XS weights (host family of weights.py).  A sha256 of
  every weight tensor is stored so a test can tell generator drift from a
  parity failure.  Cases:
    small_m1, small_m4  hidden 512, inter 256, 64 experts, top-10, shared 256
    c1_m1               BASELINE config 1: hidden 2048, inter 512, 512 experts
    c1_m4, c1_m8        the config-3 token counts through one config-1 layer
    tie_m2              a router whose 64 rows are identical: every logit ties.
    formats_*           the real checkpoint's other expert formats (`make_golden.py
                        formats`): the reference's dequantize of Q8_0, IQ4_NL
                        and IQ3_S bytes, and its _moe on a layer of IQ3_S
                        gate|up, IQ4_NL down and a Q8_0 shared down.
    hc_small, hc_c1     the hyper-connection mixer around the block
                        (reference/model.py:53-81; `make_golden.py hc` makes
                        these alone): 4 streams of hidden 512 / 2048, low rank
                        64 / 32, seeded by oracle/hc_ref.py.
                        torch.topk's CPU tie order is not lower-index, so this
                        case runs the reference with torch.topk replaced by a
                        stable lower-index selection (the rule of the
                        reference's device kernel, router_select.cpp:163-164)
                        and also records the unpatched selection.
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
if not os.environ.get("REFERENCE_SRC"):
    sys.exit("set REFERENCE_SRC to the reference checkout's src directory")
REF = Path(os.environ["REFERENCE_SRC"])
sys.path.insert(0, str(REF))
sys.path.insert(0, str(ROOT))

from ttrunner_qwen38_flash_next.gguf.quants import dequantize  # noqa: E402
from ttrunner_qwen38_flash_next.gguf.reader import GGMLType, TensorInfo  # noqa: E402
from ttrunner_qwen38_flash_next.reference.config import Qwen4ExpConfig  # noqa: E402
from ttrunner_qwen38_flash_next.reference.model import Qwen4ExpModel  # noqa: E402
from ttrunner_qwen38_flash_next.reference.weights import WeightStore  # noqa: E402

import __graft_entry__  # noqa: E402

pkg = __graft_entry__.load_package()


class FakeGGUF:
    """The two members WeightStore uses: `.tensors[name]` and `.raw(name)`."""

    def __init__(self) -> None:
        self.tensors: dict[str, TensorInfo] = {}
        self._raw: dict[str, np.ndarray] = {}

    def add(self, name: str, torch_shape: tuple[int, ...], ggml_type: GGMLType, raw: np.ndarray) -> None:
        self.tensors[name] = TensorInfo(name=name, shape=tuple(reversed(torch_shape)), ggml_type=ggml_type,
                                        offset=0, file=Path("synthetic"), data_start=0)
        self._raw[name] = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)

    def raw(self, name: str) -> memoryview:
        return memoryview(self._raw[name])


def make_config(cfg) -> Qwen4ExpConfig:
    # Only the MoE fields are read by _moe; the rest must merely construct.
    return Qwen4ExpConfig(
        hidden_size=cfg.hidden, num_layers=1, vocab_size=16, rms_norm_eps=1e-6, context_length=16,
        num_attention_heads=1, num_kv_heads=1, head_dim=64, rope_theta=10000.0, rope_dim=16,
        mrope_section=[4, 2, 2], full_attention_interval=4, indexer_heads=1, indexer_head_dim=16,
        indexer_budget=16, indexer_compress_ratio=4, linear_num_v_heads=1, linear_num_k_heads=1,
        linear_head_dim=16, conv_kernel=4, num_experts=cfg.n_experts, num_experts_per_tok=cfg.top_k,
        expert_intermediate=cfg.inter, shared_expert_intermediate=cfg.shared_inter, hc_count=1,
        hc_lowrank=1, ple_layers=[], ngram_size=2, heads_per_ngram=1, ple_conv_kernel=1, ple_head_dim=16,
        ple_eos_token_id=0, ngram_layer_multipliers=[], ngram_head_offsets=[], ngram_head_vocab_sizes=[],
    )


def gguf_from_host_layer(hl, layer: int = 0) -> tuple[FakeGGUF, dict[str, str]]:
    cfg = hl.cfg
    E, D, I, Ish = cfg.n_experts, cfg.hidden, cfg.inter, cfg.shared_inter
    g = FakeGGUF()
    p = f"blk.{layer}."
    hl.ensure_all()
    gu = np.stack([hl.expert(e)[0] for e in range(E)])   # [E, 2I, rb]
    dn = np.stack([hl.expert(e)[1] for e in range(E)])   # [E, D, rb_dn]
    tensors = {
        p + "ffn_gate_inp.weight": ((E, D), GGMLType.F32, hl.router),
        p + "ffn_gate_inp_shexp.weight": ((D,), GGMLType.F32, hl.gate_vec),
        p + "ffn_gate_shexp.weight": ((Ish, D), GGMLType.IQ4_XS, hl.sh_gate_up[:Ish]),
        p + "ffn_up_shexp.weight": ((Ish, D), GGMLType.IQ4_XS, hl.sh_gate_up[Ish:]),
        p + "ffn_down_shexp.weight": ((D, Ish), GGMLType.IQ4_XS, hl.sh_down),
        p + "ffn_gate_exps.weight": ((E, I, D), GGMLType.IQ4_XS, gu[:, :I]),
        p + "ffn_up_exps.weight": ((E, I, D), GGMLType.IQ4_XS, gu[:, I:]),
        p + "ffn_down_exps.weight": ((E, D, I), GGMLType.IQ4_XS, dn),
    }
    digests = {}
    for name, (shape, t, raw) in tensors.items():
        g.add(name, shape, t, raw)
        digests[name] = hashlib.sha256(np.ascontiguousarray(raw).tobytes()).hexdigest()
    return g, digests


def stable_topk(probs, k, dim=-1, largest=True, sorted=True):
    """Lower-index tie rule, for the tie case only."""
    order = torch.argsort(-probs, dim=dim, stable=True).narrow(dim, 0, k)
    return torch.gather(probs, dim, order), order


def run_reference(hl, x_bf16: torch.Tensor, patch_topk: bool = False) -> dict:
    g, digests = gguf_from_host_layer(hl)
    model = Qwen4ExpModel(make_config(hl.cfg), WeightStore(g))
    x = x_bf16.float().reshape(1, -1, hl.cfg.hidden)   # bf16 -> fp32 is exact
    captured = {}
    real_topk = torch.topk

    def spy_topk(t, k, dim=-1, largest=True, sorted=True):
        fn = stable_topk if patch_topk else real_topk
        v, i = fn(t, k, dim=dim, largest=largest, sorted=sorted)
        captured["probs"] = t.clone()
        captured["ids"] = i.clone()
        captured["raw_ids"] = real_topk(t, k, dim=dim).indices.clone()
        return v, i

    torch.topk = spy_topk
    try:
        with torch.no_grad():
            out = model._moe(x, 0)
    finally:
        torch.topk = real_topk
    probs = captured["probs"].numpy()
    ids = captured["ids"].numpy()
    w = np.take_along_axis(probs, ids, -1)
    w = w / w.sum(-1, keepdims=True)
    return {
        "out": out.reshape(-1, hl.cfg.hidden).numpy().astype(np.float32),
        "ids": ids.astype(np.int64),
        "raw_ids": captured["raw_ids"].numpy().astype(np.int64),
        "weights": w.astype(np.float32),
        "probs": probs.astype(np.float32),
        "digest": np.array(sorted(f"{k}={v}" for k, v in digests.items())),
    }


def save_case(name: str, cfg, seed: int, m: int, x: torch.Tensor, res: dict, **extra) -> None:
    np.savez_compressed(
        HERE / f"moe_{name}.npz",
        hidden=cfg.hidden, inter=cfg.inter, n_experts=cfg.n_experts, top_k=cfg.top_k,
        shared_inter=cfg.shared_inter, weight_std=cfg.weight_std, seed=seed, n_tokens=m,
        x_bf16=x.view(torch.int16).numpy(), **{k: v for k, v in res.items() if k != "probs"},
        probs_top=np.take_along_axis(res["probs"], res["ids"], -1), **extra,
    )
    print(f"moe_{name}: ids {res['ids'][0][:10].tolist()} out[0,:3] {res['out'][0, :3]}")


def dequant_fixture() -> None:
    import gguf
    from gguf.quants import dequantize as gguf_dequantize

    n_blocks = 64
    rng = np.random.default_rng(1234 + int(GGMLType.IQ4_XS))
    raw_random = rng.integers(0, 256, size=n_blocks * 136, dtype=np.uint8)
    out_random = dequantize(memoryview(raw_random.tobytes()), GGMLType.IQ4_XS, n_blocks * 256)
    theirs = gguf_dequantize(raw_random, gguf.GGMLQuantizationType.IQ4_XS).reshape(-1)
    finite = np.isfinite(theirs)
    assert np.array_equal(out_random[finite], theirs[finite]), "reference and gguf disagree"

    vals = np.random.default_rng([99, 1]).standard_normal(32 * 256, dtype=np.float32) * np.float32(0.02)
    raw_quant = pkg.weights.quantize_host(vals.reshape(32, 256)).reshape(-1)
    out_quant = dequantize(memoryview(raw_quant.tobytes()), GGMLType.IQ4_XS, 32 * 256)
    np.savez_compressed(HERE / "iq4xs_dequant.npz", raw_random=raw_random, out_random=out_random,
                        finite_random=finite, raw_quant=raw_quant, out_quant=out_quant,
                        quant_input=vals)
    print("iq4xs_dequant: random", int(finite.sum()), "finite of", finite.size, "| quantiser blocks 32")


def hc_fixture(name: str, hidden: int, hc: int, rank: int, m: int, seed: int) -> None:
    """The reference's hyper-connection mixer (reference/model.py:53-81) on seeded weights and
    inputs: the fixture keeps the seeds and the reference's outputs (the weights regenerate from
    oracle/hc_ref.synth_weights)."""
    from oracle import hc_ref

    w = hc_ref.synth_weights(seed, hidden, hc, rank)
    hyper, branch = hc_ref.synth_inputs(seed, hidden, hc, m)
    g = FakeGGUF()
    n = hc * hidden
    for tag, shape in (("norm", (n,)), ("down", (rank, n)), ("up", (n, rank)), ("inject", (hc, n))):
        g.add(f"blk.0.hc_ffn_{tag}.weight", shape, GGMLType.F32, w[f"{tag}_w"])
    cfg = make_config(pkg.MoEConfig(hidden=hidden))
    cfg.hc_count, cfg.hc_lowrank = hc, rank
    model = Qwen4ExpModel(cfg, WeightStore(g))
    h = torch.from_numpy(hyper).reshape(1, m, n)
    mixed, _, inject = model._gated_residual(h, 0, "ffn")
    out = model._reinject(h, torch.from_numpy(branch).reshape(1, m, hidden), inject)
    np.savez_compressed(HERE / f"hc_{name}.npz", hidden=hidden, hc=hc, rank=rank, n_tokens=m, seed=seed,
                        eps=cfg.rms_norm_eps, mixed=mixed.reshape(m, hidden).numpy(),
                        inject=inject.reshape(m, hc).numpy(), reinjected=out.reshape(m, n).numpy())
    print(f"hc_{name}: mixed[0,:3] {mixed.reshape(m, hidden)[0, :3].tolist()} inject[0] {inject.reshape(m, hc)[0].tolist()}")


# The real checkpoint's other expert formats (gguf/quants.py): GGML type ids.
FORMATS = {"Q8_0": GGMLType.Q8_0, "IQ4_NL": GGMLType.IQ4_NL, "IQ3_S": GGMLType.IQ3_S}
# The formats' MoE fixture: IQ3_S gate|up, IQ4_NL down (tt/plan.py:90-103), Q8_0 shared down.
FMT_SEED = 41


def formats_dequant_fixture() -> None:
    """The reference's dequantize on seeded bytes of Q8_0, IQ4_NL and IQ3_S (a few blocks with
    non-finite or zero scales)."""
    from oracle import moe_ref

    out = {}
    for i, (name, t) in enumerate(FORMATS.items()):
        bv, bb = moe_ref.BLOCK[int(t)]
        nblk = 48
        raw = moe_ref.synth_format_bytes(int(t), 90 + i, 1, 1, nblk * bv, 0.01)[0].copy()
        for b, h in ((3, 0x7C00), (7, 0xFE00), (11, 0x0000), (13, 0x8001)):  # inf, nan, zero, -subnormal
            raw[b * bb:b * bb + 2] = np.array([h & 0xFF, h >> 8], dtype=np.uint8)
        ref = dequantize(memoryview(raw.tobytes()), t, nblk * bv)
        out[f"{name}_raw"], out[f"{name}_out"] = raw, ref
    np.savez_compressed(HERE / "formats_dequant.npz", **out)
    print("formats_dequant:", {k: v.shape for k, v in out.items()})


def formats_moe_fixture() -> None:
    """One small layer with the real checkpoint's format mix through the reference's _moe."""
    from oracle import moe_ref

    small = pkg.MoEConfig(hidden=512, inter=256, n_experts=64, top_k=10, shared_inter=256)
    E, D, I, Ish = small.n_experts, small.hidden, small.inter, small.shared_inter
    lay = moe_ref.synth_formats_layer(FMT_SEED, E, D, I, Ish)
    gu, dn, sgu, sdn = lay["gate_up"], lay["down"], lay["sh_gate_up"], lay["sh_down"]
    router, gate_vec = lay["router"], lay["gate_vec"]
    g = FakeGGUF()
    p = "blk.0."
    for name, shape, t, raw in (
        ("ffn_gate_inp.weight", (E, D), GGMLType.F32, router),
        ("ffn_gate_inp_shexp.weight", (D,), GGMLType.F32, gate_vec),
        ("ffn_gate_shexp.weight", (Ish, D), GGMLType.IQ3_S, sgu[:Ish]),
        ("ffn_up_shexp.weight", (Ish, D), GGMLType.IQ3_S, sgu[Ish:]),
        ("ffn_down_shexp.weight", (D, Ish), GGMLType.Q8_0, sdn),
        ("ffn_gate_exps.weight", (E, I, D), GGMLType.IQ3_S, gu[:, :I]),
        ("ffn_up_exps.weight", (E, I, D), GGMLType.IQ3_S, gu[:, I:]),
        ("ffn_down_exps.weight", (E, D, I), GGMLType.IQ4_NL, dn),
    ):
        g.add(p + name, shape, t, raw)
    model = Qwen4ExpModel(make_config(small), WeightStore(g))
    for m in (1, 4):
        x = pkg.synth_x(small, m, seed=FMT_SEED)
        out = model._moe(x.float().reshape(1, m, D), 0).reshape(m, D).numpy()
        np.savez_compressed(HERE / f"formats_moe_m{m}.npz", seed=FMT_SEED, n_tokens=m,
                            x_bf16=x.view(torch.int16).numpy(), out=out)
        print(f"formats_moe_m{m}: out[0,:3] {out[0, :3]}")


def main() -> None:
    if len(sys.argv) > 1 and sys.argv[1] == "formats":
        formats_dequant_fixture()
        formats_moe_fixture()
        return
    if len(sys.argv) > 1 and sys.argv[1] == "hc":
        hc_fixture("small", 512, 4, 64, 2, 21)
        hc_fixture("c1", 2048, 4, 32, 1, 22)
        return
    dequant_fixture()
    small = pkg.MoEConfig(hidden=512, inter=256, n_experts=64, top_k=10, shared_inter=256)
    hl = pkg.synth_host_layer(small, layer=0, seed=7, all_experts=True)
    for m in (1, 4):
        x = pkg.synth_x(small, m, seed=7)
        save_case(f"small_m{m}", small, 7, m, x, run_reference(hl, x))

    # Ties: all router rows equal -> all logits equal for any x.
    tie = pkg.synth_host_layer(small, layer=0, seed=8, all_experts=True)
    tie.router = np.repeat(tie.router[:1], small.n_experts, axis=0)
    x = pkg.synth_x(small, 2, seed=8)
    res = run_reference(tie, x, patch_topk=True)
    save_case("tie_m2", small, 8, 2, x, res, router_row0=tie.router[0])

    c1 = pkg.C1
    hl1 = pkg.synth_host_layer(c1, layer=0, seed=0, all_experts=True)
    for m in (1, 4, 8):
        x = pkg.synth_x(c1, m, seed=0)
        save_case(f"c1_m{m}", c1, 0, m, x, run_reference(hl1, x))


if __name__ == "__main__":
    main()
