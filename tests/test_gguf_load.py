"""The GGUF loader (gguf_load.py): a GGUF v3 checkpoint written by the `gguf` package's own writer
(an independent implementation of the format), read back by this loader and by the package's
reader; one layer's MoE tensors assembled into the block's layout; and (on a GPU) the block run
on that layer against the oracle decoding the same bytes.

The layer has the checkpoint's format mix (IQ3_S gate|up, IQ4_NL down, IQ3_S shared gate|up, Q8_0
shared down; tt/plan.py:90-103) at a small shape, split over two files as a sharded checkpoint is.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

gguf = pytest.importorskip("gguf")

E, D, I, ISH = 32, 512, 256, 256
SEED = 61


@pytest.fixture(scope="module")
def layer_bytes(oracle):
    lay = oracle.synth_formats_layer(SEED, E, D, I, ISH)
    return lay


@pytest.fixture(scope="module")
def ckpt_files(tmp_path_factory, layer_bytes):
    lay = layer_bytes
    qt = gguf.GGMLQuantizationType
    d = tmp_path_factory.mktemp("ckpt")
    paths = [d / "m-00001-of-00002.gguf", d / "m-00002-of-00002.gguf"]
    w = gguf.GGUFWriter(str(paths[0]), "qwen4exp")
    w.add_uint32("qwen4exp.expert_used_count", 10)
    w.add_uint32("qwen4exp.expert_count", E)
    w.add_array("tokenizer.ggml.tokens", ["a", "bc", "def"])
    w.add_float32("qwen4exp.rope.freq_base", 1.0e6)
    p = "blk.0."
    w.add_tensor(p + "ffn_gate_inp.weight", np.ascontiguousarray(lay["router"]))
    w.add_tensor(p + "ffn_gate_inp_shexp.weight", np.ascontiguousarray(lay["gate_vec"]))
    w.add_tensor(p + "ffn_gate_exps.weight", np.ascontiguousarray(lay["gate_up"][:, :I]), raw_dtype=qt.IQ3_S)
    w.add_tensor(p + "ffn_up_exps.weight", np.ascontiguousarray(lay["gate_up"][:, I:]), raw_dtype=qt.IQ3_S)
    w.add_tensor(p + "ffn_down_exps.weight", np.ascontiguousarray(lay["down"]), raw_dtype=qt.IQ4_NL)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    w = gguf.GGUFWriter(str(paths[1]), "qwen4exp")
    w.add_tensor(p + "ffn_gate_shexp.weight", np.ascontiguousarray(lay["sh_gate_up"][:ISH]), raw_dtype=qt.IQ3_S)
    w.add_tensor(p + "ffn_up_shexp.weight", np.ascontiguousarray(lay["sh_gate_up"][ISH:]), raw_dtype=qt.IQ3_S)
    w.add_tensor(p + "ffn_down_shexp.weight", np.ascontiguousarray(lay["sh_down"]), raw_dtype=qt.Q8_0)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return paths


def test_reader_matches_the_gguf_package(pkg, ckpt_files):
    ck = pkg.GGUFCheckpoint(ckpt_files)
    try:
        assert ck.meta_int(".expert_used_count") == 10
        assert ck.metadata["tokenizer.ggml.tokens"] == ["a", "bc", "def"]
        assert abs(ck.metadata["qwen4exp.rope.freq_base"] - 1.0e6) < 1.0
        assert len(ck.tensors) == 8
        for path in ckpt_files:
            r = gguf.GGUFReader(str(path))
            for t in r.tensors:
                mine = ck.tensors[t.name]
                assert mine.ggml_type == int(t.tensor_type)
                assert mine.dims == tuple(int(v) for v in t.shape)
                assert mine.nbytes == int(t.n_bytes)
                ref = np.asarray(t.data).view(np.uint8).reshape(-1)
                assert np.array_equal(ck.raw(t.name), ref), t.name
        assert ck.tensors["blk.0.ffn_gate_exps.weight"].shape == (E, I, D)
        assert ck.tensors["blk.0.ffn_down_exps.weight"].shape == (E, D, I)
    finally:
        ck.close()


def test_layer_assembly(pkg, ckpt_files, layer_bytes):
    with pkg.GGUFCheckpoint(ckpt_files) as ck:
        lb = pkg.moe_layer_bytes(ck, 0)
        assert lb.formats == (21, 20, 21, 8)
        assert (lb.hidden, lb.inter, lb.n_experts, lb.shared_inter, lb.top_k) == (D, I, E, ISH, 10)
        for key in ("router", "gate_vec", "gate_up", "down", "sh_gate_up", "sh_down"):
            assert np.array_equal(getattr(lb, key), layer_bytes[key]), key


def test_loader_rejects_formats_it_cannot_run(pkg, tmp_path):
    qt = gguf.GGMLQuantizationType
    path = tmp_path / "bad.gguf"
    w = gguf.GGUFWriter(str(path), "qwen4exp")
    w.add_tensor("blk.0.ffn_gate_inp.weight", np.zeros((E, D), dtype=np.float32))
    w.add_tensor("blk.0.ffn_gate_exps.weight", np.zeros((E, I, D // 256 * 144), dtype=np.uint8), raw_dtype=qt.Q4_K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(ValueError):
        with pkg.GGUFCheckpoint(path) as ck:
            pkg.moe_layer_bytes(ck, 0)


@pytest.mark.gpu
def test_checkpoint_layer_on_gpu_matches_oracle(pkg, oracle, ckpt_files, layer_bytes):
    lay = layer_bytes
    with pkg.GGUFCheckpoint(ckpt_files) as ck:
        moe = pkg.load_moe_layer(ck, 0, device="cuda")
    src = oracle.ExpertSource(lambda e: (lay["gate_up"][e], lay["down"][e]), lay["sh_gate_up"], lay["sh_down"],
                              lay["router"], lay["gate_vec"], I, ISH, formats=lay["formats"])
    for m in (1, 4):
        x = (torch.randn(m, D, generator=torch.Generator().manual_seed(m)) * 0.5).to(torch.bfloat16)
        out = moe(x.cuda().reshape(1, 1, m, D)).float().cpu().numpy().reshape(m, D)
        ref = oracle.moe_forward(x.float().numpy(), src, 10)["out"]
        assert np.abs(out - ref).max() / np.abs(ref).max() < 1e-2


def test_reader_metadata_types_and_alignment(pkg, tmp_path):
    """Every scalar type, strings, arrays and a non-default `general.alignment` (the tensor-data
    section starts at the next multiple of it), against the gguf package's reader."""
    path = tmp_path / "meta.gguf"
    w = gguf.GGUFWriter(str(path), "qwen4exp")
    w.add_custom_alignment(64)
    w.add_uint8("k.u8", 200)
    w.add_int8("k.i8", -5)
    w.add_uint16("k.u16", 60000)
    w.add_int16("k.i16", -30000)
    w.add_uint32("k.u32", 4000000000)
    w.add_int32("k.i32", -2000000000)
    w.add_float32("k.f32", 0.5)
    w.add_bool("k.bool", True)
    w.add_uint64("k.u64", 2 ** 40)
    w.add_int64("k.i64", -(2 ** 40))
    w.add_float64("k.f64", 0.25)
    w.add_string("k.str", "héllo")
    w.add_array("k.arr_i32", [1, -2, 3])
    w.add_array("k.arr_f32", [0.5, 1.5])
    w.add_tensor("t.a", np.arange(12, dtype=np.float32).reshape(3, 4))
    w.add_tensor("t.b", np.arange(8, dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pkg.GGUFCheckpoint(path) as ck:
        m = ck.metadata
        assert (m["k.u8"], m["k.i8"], m["k.u16"], m["k.i16"]) == (200, -5, 60000, -30000)
        assert (m["k.u32"], m["k.i32"], m["k.u64"], m["k.i64"]) == (4000000000, -2000000000, 2 ** 40, -(2 ** 40))
        assert (m["k.f32"], m["k.f64"], m["k.bool"], m["k.str"]) == (0.5, 0.25, True, "héllo")
        assert m["k.arr_i32"] == [1, -2, 3] and m["k.arr_f32"] == [0.5, 1.5]
        assert m["general.alignment"] == 64
        assert ck._data[0] % 64 == 0
        assert np.array_equal(ck.raw("t.a").view(np.float32).reshape(3, 4), np.arange(12, dtype=np.float32).reshape(3, 4))
        assert np.array_equal(ck.raw("t.b").view(np.float32), np.arange(8, dtype=np.float32))
        r = gguf.GGUFReader(str(path))
        for t in r.tensors:
            assert ck._data[0] + ck.tensors[t.name].offset == int(t.data_offset)


def _write_iq4xs_layers(path, pkg, cfg, n_layers, seed):
    qt = gguf.GGMLQuantizationType
    w = gguf.GGUFWriter(str(path), "qwen4exp")
    w.add_uint32("qwen4exp.expert_used_count", cfg.top_k)
    hls = []
    for L in range(n_layers):
        hl = pkg.synth_host_layer(cfg, layer=L, seed=seed, all_experts=True)
        hls.append(hl)
        gu = np.stack([hl.expert(e)[0] for e in range(cfg.n_experts)])
        dn = np.stack([hl.expert(e)[1] for e in range(cfg.n_experts)])
        p = f"blk.{L}."
        w.add_tensor(p + "ffn_gate_inp.weight", np.ascontiguousarray(hl.router))
        w.add_tensor(p + "ffn_gate_inp_shexp.weight", np.ascontiguousarray(hl.gate_vec))
        w.add_tensor(p + "ffn_gate_exps.weight", np.ascontiguousarray(gu[:, :cfg.inter]), raw_dtype=qt.IQ4_XS)
        w.add_tensor(p + "ffn_up_exps.weight", np.ascontiguousarray(gu[:, cfg.inter:]), raw_dtype=qt.IQ4_XS)
        w.add_tensor(p + "ffn_down_exps.weight", np.ascontiguousarray(dn), raw_dtype=qt.IQ4_XS)
        w.add_tensor(p + "ffn_gate_shexp.weight", np.ascontiguousarray(hl.sh_gate_up[:cfg.shared_inter]),
                     raw_dtype=qt.IQ4_XS)
        w.add_tensor(p + "ffn_up_shexp.weight", np.ascontiguousarray(hl.sh_gate_up[cfg.shared_inter:]),
                     raw_dtype=qt.IQ4_XS)
        w.add_tensor(p + "ffn_down_shexp.weight", np.ascontiguousarray(hl.sh_down), raw_dtype=qt.IQ4_XS)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return hls


@pytest.mark.gpu
def test_iq4xs_checkpoint_runs_the_stack(pkg, tmp_path):
    """An all-IQ4_XS checkpoint: its layers as DeviceLayers (bytes equal to the generator's), the
    stack over two of them equal to the layer-by-layer chain of MoELayer calls."""
    cfg = pkg.MoEConfig(hidden=512, inter=256, n_experts=64, top_k=10, shared_inter=256)
    path = tmp_path / "iq4xs.gguf"
    hls = _write_iq4xs_layers(path, pkg, cfg, 2, seed=17)
    with pkg.GGUFCheckpoint(path) as ck:
        stack = pkg.load_moe_stack(ck, [0, 1], max_tokens=4)
        dls = [pkg.gguf_load.device_layer(pkg.moe_layer_bytes(ck, L)) for L in range(2)]
    ref_dls = [pkg.upload_host_layer(h) for h in hls]
    for a, b in zip(dls, ref_dls):
        for key in ("router", "gate_vec", "gate_up", "down", "sh_gate_up", "sh_down"):
            assert torch.equal(getattr(a, key), getattr(b, key)), key
    x = (torch.randn(3, 512, generator=torch.Generator().manual_seed(4)) * 0.5).to(torch.bfloat16).cuda()
    out = stack.decode(x).clone()
    y = x
    for dl in ref_dls:
        y = pkg.MoELayer(dl)(y, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert float((out - y).abs().max()) <= 1e-5 * float(y.abs().max())
