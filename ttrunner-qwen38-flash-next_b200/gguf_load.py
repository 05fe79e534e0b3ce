"""GGUF checkpoints onto the GPU in the MoE block's layout.

The reference opens its checkpoint with its own GGUF v3 reader (gguf/reader.py: header, typed
metadata, tensor infos, the tensor-data section at `general.alignment`, memory-mapped shards) and
hands the MoE tensors of a layer to its kernels (reference/weights.py:118-179, tt/weights.py:38-61).
This module does the same for this library: it reads GGUF v3 files (split checkpoints as one
namespace), and assembles one layer's MoE tensors, bytes unchanged, into the layout the C ABI takes:
router fp32 [E, D], shared gate vector fp32 [D], gate|up [E, 2I, row bytes] (each expert's gate rows
then its up rows), down [E, D, row bytes], the shared expert as [2 Ish, row bytes] and [D, row bytes],
with the GGML type of each expert tensor (IQ4_XS, IQ3_S, IQ4_NL or Q8_0; tt/plan.py:90-103 lists the
checkpoint's mix).  `CheckpointMoE` runs the block on such a layer.
"""

from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np
import torch

GGUF_MAGIC = b"GGUF"
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q",
           12: "<d"}
_STRING, _ARRAY = 8, 9
F32, F16, Q8_0, IQ4_NL, IQ3_S, IQ4_XS, BF16 = 0, 1, 8, 20, 21, 23, 30
# (values per block, bytes per block) of the types a MoE layer's tensors may have
TYPE_BLOCKS = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q8_0: (32, 34), IQ4_NL: (32, 18), IQ3_S: (256, 110),
               IQ4_XS: (256, 136)}
EXPERT_TYPES = (Q8_0, IQ4_NL, IQ3_S, IQ4_XS)


@dataclass(frozen=True)
class GGUFTensor:
    name: str
    dims: tuple[int, ...]  # GGUF order: fastest-varying first
    ggml_type: int
    offset: int            # from the file's tensor-data section
    file: int              # index into GGUFCheckpoint.files

    @property
    def shape(self) -> tuple[int, ...]:
        """Row-major (numpy / torch) shape."""
        return tuple(reversed(self.dims))

    @property
    def nbytes(self) -> int:
        if self.ggml_type not in TYPE_BLOCKS:
            raise ValueError(f"{self.name}: GGML type {self.ggml_type} is not one this loader handles")
        bv, bb = TYPE_BLOCKS[self.ggml_type]
        n = int(np.prod(self.dims, dtype=np.int64))
        if n % bv:
            raise ValueError(f"{self.name}: {n} values is not a whole number of blocks")
        return n // bv * bb


class _Cursor:
    def __init__(self, buf: memoryview) -> None:
        self.buf, self.pos = buf, 0

    def scalar(self, fmt: str) -> Any:
        (v,) = struct.unpack_from(fmt, self.buf, self.pos)
        self.pos += struct.calcsize(fmt)
        return v

    def string(self) -> str:
        n = self.scalar("<Q")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8", errors="replace")
        self.pos += n
        return s

    def value(self, vtype: int) -> Any:
        if vtype == _STRING:
            return self.string()
        if vtype == _ARRAY:
            etype, count = self.scalar("<I"), self.scalar("<Q")
            if etype == _STRING:
                return [self.string() for _ in range(count)]
            if etype == _ARRAY:
                return [self.value(_ARRAY) for _ in range(count)]
            fmt = _SCALAR[etype]
            vals = list(struct.unpack_from(f"<{count}{fmt[1:]}", self.buf, self.pos))
            self.pos += struct.calcsize(fmt) * count
            return vals
        if vtype not in _SCALAR:
            raise ValueError(f"unknown GGUF value type {vtype}")
        return self.scalar(_SCALAR[vtype])


class GGUFCheckpoint:
    """One or more GGUF v3 files (a split checkpoint) as one tensor namespace, memory-mapped."""

    def __init__(self, paths: str | Path | list[str | Path]) -> None:
        if isinstance(paths, (str, Path)):
            paths = [paths]
        if not paths:
            raise ValueError("no GGUF files given")
        self.files: list[Path] = sorted((Path(p) for p in paths), key=str)
        self._fds, self._maps, self._views, self._data = [], [], [], []
        self.metadata: dict[str, Any] = {}
        self.tensors: dict[str, GGUFTensor] = {}
        for i, path in enumerate(self.files):
            meta, infos, data_start, fd, mm = self._open(path)
            self._fds.append(fd)
            self._maps.append(mm)
            self._views.append(memoryview(mm))
            self._data.append(data_start)
            if i == 0:
                self.metadata = meta
            for name, dims, gtype, off in infos:
                if name in self.tensors:
                    raise ValueError(f"tensor {name!r} appears in two files")
                self.tensors[name] = GGUFTensor(name, dims, gtype, off, i)

    @staticmethod
    def _open(path: Path):
        fd = open(path, "rb")
        mm = mmap.mmap(fd.fileno(), 0, access=mmap.ACCESS_READ)
        cur = _Cursor(memoryview(mm))
        if bytes(cur.buf[:4]) != GGUF_MAGIC:
            raise ValueError(f"{path.name}: not a GGUF file")
        cur.pos = 4
        version = cur.scalar("<I")
        if version != 3:
            raise ValueError(f"{path.name}: GGUF version {version}, only 3 is read")
        n_tensors, n_kv = cur.scalar("<Q"), cur.scalar("<Q")
        meta: dict[str, Any] = {}
        for _ in range(n_kv):
            key = cur.string()
            meta[key] = cur.value(cur.scalar("<I"))
        infos = []
        for _ in range(n_tensors):
            name = cur.string()
            nd = cur.scalar("<I")
            dims = tuple(cur.scalar("<Q") for _ in range(nd))
            infos.append((name, dims, cur.scalar("<I"), cur.scalar("<Q")))
        align = int(meta.get("general.alignment", 32))
        data_start = (cur.pos + align - 1) // align * align
        cur.buf.release()
        return meta, infos, data_start, fd, mm

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes (uint8, no copy) in row-major order of its rows."""
        t = self.tensors[name]
        start = self._data[t.file] + t.offset
        return np.frombuffer(self._views[t.file], dtype=np.uint8, count=t.nbytes, offset=start)

    def meta_int(self, suffix: str) -> int | None:
        """The integer metadata value whose key ends with `suffix` (e.g. `.expert_used_count`)."""
        for k, v in self.metadata.items():
            if k.endswith(suffix) and isinstance(v, int):
                return v
        return None

    def close(self) -> None:
        """Unmap the files; arrays still viewing them keep their mapping alive until they go."""
        for v, m in zip(self._views, self._maps):
            try:
                v.release()
                m.close()
            except BufferError:
                pass
        for f in self._fds:
            f.close()
        self._views, self._maps, self._fds = [], [], []

    def __enter__(self) -> "GGUFCheckpoint":
        return self

    def __exit__(self, *exc: object) -> None:
        self.close()


# ---- one layer's MoE tensors -------------------------------------------------------------------


def _float_rows(ckpt: GGUFCheckpoint, name: str) -> np.ndarray:
    """An F32 / F16 / BF16 tensor as fp32 in its row-major shape."""
    t = ckpt.tensors[name]
    raw = ckpt.raw(name)
    if t.ggml_type == F32:
        a = raw.view(np.float32)
    elif t.ggml_type == F16:
        a = raw.view(np.float16).astype(np.float32)
    elif t.ggml_type == BF16:
        a = (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    else:
        raise ValueError(f"{name}: expected F32, F16 or BF16, found GGML type {t.ggml_type}")
    return a.reshape(t.shape)


def _expert_rows(ckpt: GGUFCheckpoint, name: str) -> tuple[np.ndarray, int]:
    """A quantised tensor as bytes [leading dims..., row bytes] and its GGML type."""
    t = ckpt.tensors[name]
    if t.ggml_type not in EXPERT_TYPES:
        raise ValueError(f"{name}: GGML type {t.ggml_type} is not one the block decodes "
                         f"(Q8_0, IQ4_NL, IQ3_S, IQ4_XS)")
    return ckpt.raw(name).reshape(t.shape[:-1] + (-1,)), t.ggml_type


@dataclass
class MoELayerBytes:
    """One layer's MoE tensors in the block's layout (host arrays)."""

    router: np.ndarray              # fp32 [E, D]
    gate_vec: np.ndarray | None     # fp32 [D]
    gate_up: np.ndarray             # uint8 [E, 2I, row bytes]
    down: np.ndarray                # uint8 [E, D, row bytes]
    sh_gate_up: np.ndarray | None   # uint8 [2 Ish, row bytes]
    sh_down: np.ndarray | None      # uint8 [D, row bytes]
    formats: tuple[int, int, int, int]  # GGML types of gate|up, down, shared gate|up, shared down
    hidden: int
    inter: int
    n_experts: int
    shared_inter: int
    top_k: int | None               # from the checkpoint's `*.expert_used_count`, if present


def moe_layer_bytes(ckpt: GGUFCheckpoint, layer: int, prefix: str = "blk.{layer}.") -> MoELayerBytes:
    """Assemble layer `layer`'s MoE tensors (GGUF names as the reference loads them,
    reference/weights.py:5-6 and tt/plan.py:90-103): ffn_gate_inp (router), ffn_gate_inp_shexp
    (shared gate vector, optional), ffn_gate_exps + ffn_up_exps (concatenated per expert),
    ffn_down_exps, and ffn_{gate,up,down}_shexp (optional)."""
    p = prefix.format(layer=layer)
    router = np.ascontiguousarray(_float_rows(ckpt, p + "ffn_gate_inp.weight"))
    E, D = router.shape
    gate, fg = _expert_rows(ckpt, p + "ffn_gate_exps.weight")
    up, fu = _expert_rows(ckpt, p + "ffn_up_exps.weight")
    if fg != fu or gate.shape != up.shape:
        raise ValueError(f"layer {layer}: gate and up expert tensors differ in type or shape")
    down, fd = _expert_rows(ckpt, p + "ffn_down_exps.weight")
    I = ckpt.tensors[p + "ffn_gate_exps.weight"].shape[1]
    if gate.shape[0] != E or down.shape[:2] != (E, D):
        raise ValueError(f"layer {layer}: expert tensors do not match the router's [E, D] = [{E}, {D}]")
    gate_up = np.concatenate([gate, up], axis=1)
    gv = sgu = sdn = None
    fsg = fsd = fg
    Ish = 0
    if p + "ffn_gate_shexp.weight" in ckpt.tensors:
        sg, fsg = _expert_rows(ckpt, p + "ffn_gate_shexp.weight")
        su, fsu = _expert_rows(ckpt, p + "ffn_up_shexp.weight")
        if fsg != fsu or sg.shape != su.shape:
            raise ValueError(f"layer {layer}: shared gate and up differ in type or shape")
        sdn, fsd = _expert_rows(ckpt, p + "ffn_down_shexp.weight")
        sgu = np.concatenate([sg, su], axis=0)
        Ish = sg.shape[0]
        if p + "ffn_gate_inp_shexp.weight" in ckpt.tensors:
            gv = np.ascontiguousarray(_float_rows(ckpt, p + "ffn_gate_inp_shexp.weight").reshape(-1))
    return MoELayerBytes(router=router, gate_vec=gv, gate_up=gate_up, down=np.ascontiguousarray(down),
                         sh_gate_up=sgu, sh_down=None if sdn is None else np.ascontiguousarray(sdn),
                         formats=(fg, fd, fsg, fsd), hidden=D, inter=I, n_experts=E, shared_inter=Ish,
                         top_k=ckpt.meta_int(".expert_used_count"))


class CheckpointMoE:
    """A checkpoint layer resident in HBM, called like the reference's per-layer MoE forward:
    x [.., M, D] -> out with x's leading shape (routed experts + gated shared expert)."""

    def __init__(self, lb: MoELayerBytes, device: str | torch.device = "cuda", top_k: int | None = None):
        dev = torch.device(device)

        def up(a):
            return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)

        self.formats = lb.formats
        self.top_k = top_k if top_k is not None else lb.top_k
        if self.top_k is None:
            raise ValueError("top_k: not in the checkpoint's metadata, pass it")
        self.router, self.gate_vec = up(lb.router), up(lb.gate_vec)
        self.gate_up, self.down = up(lb.gate_up), up(lb.down)
        self.sh_gate_up, self.sh_down = up(lb.sh_gate_up), up(lb.sh_down)

    def __call__(self, x: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        from .moe import moe_block_formats

        return moe_block_formats(x, self.router, self.gate_vec, self.gate_up, self.down, self.sh_gate_up,
                                 self.sh_down, self.formats, self.top_k, out_dtype=out_dtype)


def load_moe_layer(ckpt: GGUFCheckpoint, layer: int, device: str | torch.device = "cuda",
                   top_k: int | None = None) -> CheckpointMoE:
    """Layer `layer`'s MoE block from a checkpoint, on `device`."""
    return CheckpointMoE(moe_layer_bytes(ckpt, layer), device, top_k)


def device_layer(lb: MoELayerBytes, device: str | torch.device = "cuda", top_k: int | None = None):
    """An all-IQ4_XS checkpoint layer as the library's DeviceLayer (unsharded), so the IQ4_XS paths
    (MoELayer, and MoEStack's single launch over many layers) run it."""
    from .config import MoEConfig, Shard
    from .weights import DeviceLayer

    if lb.formats != (IQ4_XS,) * 4:
        raise ValueError(f"formats {lb.formats}: the IQ4_XS paths need every expert tensor IQ4_XS")
    k = top_k if top_k is not None else lb.top_k
    if k is None:
        raise ValueError("top_k: not in the checkpoint's metadata, pass it")
    dev = torch.device(device)

    def up(a):
        return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    cfg = MoEConfig(hidden=lb.hidden, inter=lb.inter, n_experts=lb.n_experts, top_k=k, shared_inter=lb.shared_inter)
    return DeviceLayer(cfg=cfg, shard=Shard(), router=up(lb.router), gate_vec=up(lb.gate_vec),
                       gate_up=up(lb.gate_up), down=up(lb.down), sh_gate_up=up(lb.sh_gate_up),
                       sh_down=up(lb.sh_down))


def load_moe_stack(ckpt: GGUFCheckpoint, layers: list[int], device: str | torch.device = "cuda",
                   top_k: int | None = None, max_tokens: int = 16):
    """Consecutive checkpoint layers whose experts are all IQ4_XS as one MoEStack (the 48-layer
    decode as one launch per step, `qmoe_stack_decode`)."""
    from .stack import MoEStack

    return MoEStack([device_layer(moe_layer_bytes(ckpt, L), device, top_k) for L in layers], max_tokens=max_tokens)
