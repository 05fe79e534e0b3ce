"""Synthetic qwen4exp MoE weights: generation, IQ4_XS quantisation, sharding.

The reference loads a GGUF checkpoint (gguf/reader.py:247) and converts it for
its device (tt/convert.py:151); this project generates seeded weights with the
BASELINE shapes and distributions instead: every tensor is N(0, std^2) fp32,
the experts and the shared expert quantised to IQ4_XS.

Two generator families, each deterministic:
  * host  -- numpy `default_rng([seed, layer, tag, expert])`, quantised by the
             library's host quantiser.  Used by the golden fixtures and parity
             tests, which need the same bytes on the CPU oracle side.
  * device -- the library's Philox generator + device quantiser, one stream per
             (layer, tag, expert).  Used for the 48-layer stack (~41 GB), with
             the oracle reading back only the experts it needs.
Both give every expert its own stream, so a shard holds exactly the bytes of
the same experts in the unsharded model.

Device layout (per layer):
  router     fp32 [E, D]
  gate_vec   fp32 [D]
  gate_up    uint8 [E_loc, 2*I_loc, D/256*136]   gate rows, then up rows
  down       uint8 [E_loc, D, row_slice_bytes]
  sh_gate_up uint8 [2*I_sh_loc, D/256*136]
  sh_down    uint8 [D, sh_row_slice_bytes]
"""

from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Callable

import numpy as np
import torch

from . import _lib
from .config import SB_BYTES, MoEConfig, Shard, iq4xs_bytes

# Stream tags of the generators.
TAG_ROUTER, TAG_GATE_VEC, TAG_SH_GATE_UP, TAG_SH_DOWN, TAG_GATE_UP, TAG_DOWN, TAG_X = range(7)

_THREADS = max(1, min(16, os.cpu_count() or 1))


def quantize_host(values: np.ndarray, n_threads: int = _THREADS) -> np.ndarray:
    """fp32 values (last dim a multiple of 256) -> IQ4_XS bytes, shape [..., n/256*136]."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    if v.shape[-1] % 256:
        raise ValueError("last dimension must be a multiple of 256")
    out = np.empty(v.shape[:-1] + (v.shape[-1] // 256 * SB_BYTES,), dtype=np.uint8)
    _lib.check(_lib.lib.qmoe_quantize_iq4xs_host(v.ctypes.data, v.size, out.ctypes.data, n_threads),
               "qmoe_quantize_iq4xs_host")
    return out


def _normal(key: list[int], n: int, std: float) -> np.ndarray:
    x = np.random.default_rng(key).standard_normal(n, dtype=np.float32)
    x *= np.float32(std)
    return x


# ---------------------------------------------------------------------------
# host family

@dataclass
class HostLayer:
    """One layer's weights in host memory (full, unsharded)."""

    cfg: MoEConfig
    layer: int
    seed: int
    router: np.ndarray                 # fp32 [E, D]
    gate_vec: np.ndarray               # fp32 [D]
    sh_gate_up: np.ndarray             # uint8 [2*I_sh, rb]
    sh_down: np.ndarray                # uint8 [D, rb_sh]
    gate_up: dict[int, np.ndarray] = field(default_factory=dict)   # e -> uint8 [2I, rb]
    down: dict[int, np.ndarray] = field(default_factory=dict)      # e -> uint8 [D, rb_dn]
    # Source of expert bytes not yet held: None generates them (host family).
    fetch: Callable[[int], tuple[np.ndarray, np.ndarray]] | None = None

    def expert(self, e: int) -> tuple[np.ndarray, np.ndarray]:
        if e not in self.gate_up:
            src = self.fetch or (lambda i: _host_expert(self.cfg, self.layer, self.seed, i))
            self.gate_up[e], self.down[e] = src(e)
        return self.gate_up[e], self.down[e]

    def ensure_all(self) -> None:
        missing = [e for e in range(self.cfg.n_experts) if e not in self.gate_up]
        with ThreadPoolExecutor(_THREADS) as ex:
            for e, (gu, dn) in zip(missing, ex.map(lambda e: _host_expert(self.cfg, self.layer, self.seed, e, 1), missing)):
                self.gate_up[e], self.down[e] = gu, dn


def _host_expert(cfg: MoEConfig, layer: int, seed: int, e: int, threads: int = _THREADS):
    D, I = cfg.hidden, cfg.inter
    gu = quantize_host(_normal([seed, layer, TAG_GATE_UP, e], 2 * I * D, cfg.weight_std).reshape(2 * I, D), threads)
    dn = quantize_host(_normal([seed, layer, TAG_DOWN, e], D * I, cfg.dn_std).reshape(D, I), threads)
    return gu, dn


def synth_host_layer(cfg: MoEConfig, layer: int = 0, seed: int = 0, all_experts: bool = False) -> HostLayer:
    """Seeded host weights; experts are generated lazily unless all_experts."""
    D, Ish = cfg.hidden, cfg.shared_inter
    hl = HostLayer(
        cfg=cfg, layer=layer, seed=seed,
        router=_normal([seed, layer, TAG_ROUTER], cfg.n_experts * D, cfg.weight_std).reshape(cfg.n_experts, D),
        gate_vec=_normal([seed, layer, TAG_GATE_VEC], D, cfg.weight_std),
        sh_gate_up=quantize_host(_normal([seed, layer, TAG_SH_GATE_UP], 2 * Ish * D, cfg.weight_std).reshape(2 * Ish, D)),
        sh_down=quantize_host(_normal([seed, layer, TAG_SH_DOWN], D * Ish, cfg.dn_std).reshape(D, Ish)),
    )
    if all_experts:
        hl.ensure_all()
    return hl


def synth_x(cfg: MoEConfig, n_tokens: int, seed: int = 0) -> torch.Tensor:
    """Activations x ~ N(0, 1) as bf16 [M, D] (host)."""
    x = np.random.default_rng([seed, TAG_X, n_tokens]).standard_normal((n_tokens, cfg.hidden), dtype=np.float32)
    return torch.from_numpy(x).to(torch.bfloat16)


# ---------------------------------------------------------------------------
# shard slicing (works on uint8 IQ4_XS row arrays)

def slice_gate_up(gu: np.ndarray | torch.Tensor, inter: int, lo: int, hi: int):
    """Rows [lo, hi) of gate and of up from a fused [.., 2*inter, rb] array."""
    if lo == 0 and hi == inter:
        return gu
    cat = np.concatenate if isinstance(gu, np.ndarray) else torch.cat
    return cat([gu[..., lo:hi, :], gu[..., inter + lo:inter + hi, :]], -2)


def slice_down(dn: np.ndarray | torch.Tensor, lo: int, hi: int):
    """Columns [lo, hi) of IQ4_XS down rows [.., D, inter/256*136] as row slices."""
    nseg, nsub, ib0 = Shard.row_slice(lo, hi)
    if nsub == 8:
        return dn[..., lo // 256 * SB_BYTES:(lo // 256 + nseg) * SB_BYTES]
    sb = lo // 256
    cat = np.concatenate if isinstance(dn, np.ndarray) else torch.cat
    hdr = dn[..., sb * SB_BYTES:sb * SB_BYTES + 8]
    qs = dn[..., sb * SB_BYTES + 8 + 16 * ib0:sb * SB_BYTES + 8 + 16 * (ib0 + nsub)]
    return cat([hdr, qs], -1)


# ---------------------------------------------------------------------------
# device layers

@dataclass
class DeviceLayer:
    """One layer resident in HBM, for one shard."""

    cfg: MoEConfig
    shard: Shard
    router: torch.Tensor
    gate_vec: torch.Tensor | None
    gate_up: torch.Tensor
    down: torch.Tensor
    sh_gate_up: torch.Tensor | None
    sh_down: torch.Tensor | None

    def c_struct(self) -> _lib.LayerWeights:
        def p(t):
            return None if t is None else t.data_ptr()
        has_sh = self.shard.has_shared() and self.sh_gate_up is not None
        return _lib.LayerWeights(
            router=p(self.router), gate_vec=p(self.gate_vec) if has_sh else None,
            gate_up=p(self.gate_up), down=p(self.down),
            sh_gate_up=p(self.sh_gate_up) if has_sh else None,
            sh_down=p(self.sh_down) if has_sh else None,
        )

    def nbytes(self) -> int:
        ts = [self.router, self.gate_vec, self.gate_up, self.down, self.sh_gate_up, self.sh_down]
        return sum(t.numel() * t.element_size() for t in ts if t is not None)

    def expert_bytes_host(self, e: int) -> tuple[np.ndarray, np.ndarray]:
        """Read back local expert e's gate|up and down bytes (for the oracle)."""
        lo, _ = self.shard.expert_window(self.cfg)
        return self.gate_up[e - lo].cpu().numpy(), self.down[e - lo].cpu().numpy()


def upload_host_layer(hl: HostLayer, shard: Shard = Shard(), device: str | torch.device = "cuda") -> DeviceLayer:
    cfg = hl.cfg
    e_lo, e_hi = shard.expert_window(cfg)
    i_lo, i_hi = shard.inter_window(cfg.inter)
    hl_experts = range(e_lo, e_hi)
    gu = np.stack([slice_gate_up(hl.expert(e)[0], cfg.inter, i_lo, i_hi) for e in hl_experts])
    dn = np.stack([slice_down(hl.expert(e)[1], i_lo, i_hi) for e in hl_experts])
    sh_gu = sh_dn = gv = None
    if shard.has_shared():
        s_lo, s_hi = shard.inter_window(cfg.shared_inter)
        sh_gu = torch.from_numpy(np.ascontiguousarray(slice_gate_up(hl.sh_gate_up, cfg.shared_inter, s_lo, s_hi))).to(device)
        sh_dn = torch.from_numpy(np.ascontiguousarray(slice_down(hl.sh_down, s_lo, s_hi))).to(device)
        gv = torch.from_numpy(hl.gate_vec).to(device)
    return DeviceLayer(
        cfg=cfg, shard=shard,
        router=torch.from_numpy(hl.router).to(device),
        gate_vec=gv,
        gate_up=torch.from_numpy(np.ascontiguousarray(gu)).to(device),
        down=torch.from_numpy(np.ascontiguousarray(dn)).to(device),
        sh_gate_up=sh_gu, sh_down=sh_dn,
    )


def _sid(layer: int, tag: int, expert: int = 0) -> int:
    return (layer << 40) | (tag << 32) | expert


def _dev_iq4(seed: int, sid: int, n: int, std: float, out: torch.Tensor, stream: int) -> None:
    _lib.check(_lib.lib.qmoe_synth_iq4xs(seed, sid, n, std, out.data_ptr(), stream), "qmoe_synth_iq4xs")


def _dev_f32(seed: int, sid: int, n: int, std: float, out: torch.Tensor, stream: int) -> None:
    _lib.check(_lib.lib.qmoe_synth_f32(seed, sid, n, std, out.data_ptr(), stream), "qmoe_synth_f32")


def synth_device_layer(cfg: MoEConfig, layer: int, seed: int = 0, shard: Shard = Shard(),
                       device: str | torch.device = "cuda") -> DeviceLayer:
    """Generate one layer's shard directly in HBM with the device family."""
    dev = torch.device(device)
    stream = torch.cuda.current_stream(dev).cuda_stream
    D, I, E = cfg.hidden, cfg.inter, cfg.n_experts
    std = cfg.weight_std
    e_lo, e_hi = shard.expert_window(cfg)
    i_lo, i_hi = shard.inter_window(I)
    n_loc = e_hi - e_lo
    rb = iq4xs_bytes(D)
    router = torch.empty(E, D, dtype=torch.float32, device=dev)
    _dev_f32(seed, _sid(layer, TAG_ROUTER), E * D, std, router, stream)
    sliced = (i_lo, i_hi) != (0, I)
    gu_full = torch.empty(2 * I, rb, dtype=torch.uint8, device=dev) if sliced else None
    dn_full = torch.empty(D, iq4xs_bytes(I), dtype=torch.uint8, device=dev) if sliced else None
    nseg, nsub, _ = Shard.row_slice(i_lo, i_hi)
    gate_up = torch.empty(n_loc, 2 * (i_hi - i_lo), rb, dtype=torch.uint8, device=dev)
    down = torch.empty(n_loc, D, nseg * (8 + 16 * nsub), dtype=torch.uint8, device=dev)
    for j, e in enumerate(range(e_lo, e_hi)):
        if sliced:
            _dev_iq4(seed, _sid(layer, TAG_GATE_UP, e), 2 * I * D, std, gu_full, stream)
            _dev_iq4(seed, _sid(layer, TAG_DOWN, e), D * I, cfg.dn_std, dn_full, stream)
            gate_up[j].copy_(slice_gate_up(gu_full, I, i_lo, i_hi))
            down[j].copy_(slice_down(dn_full, i_lo, i_hi))
        else:
            _dev_iq4(seed, _sid(layer, TAG_GATE_UP, e), 2 * I * D, std, gate_up[j], stream)
            _dev_iq4(seed, _sid(layer, TAG_DOWN, e), D * I, cfg.dn_std, down[j], stream)
    gv = sh_gu = sh_dn = None
    if shard.has_shared():
        Ish = cfg.shared_inter
        s_lo, s_hi = shard.inter_window(Ish)
        gv = torch.empty(D, dtype=torch.float32, device=dev)
        _dev_f32(seed, _sid(layer, TAG_GATE_VEC), D, std, gv, stream)
        full_gu = torch.empty(2 * Ish, rb, dtype=torch.uint8, device=dev)
        full_dn = torch.empty(D, iq4xs_bytes(Ish), dtype=torch.uint8, device=dev)
        _dev_iq4(seed, _sid(layer, TAG_SH_GATE_UP), 2 * Ish * D, std, full_gu, stream)
        _dev_iq4(seed, _sid(layer, TAG_SH_DOWN), D * Ish, cfg.dn_std, full_dn, stream)
        sh_gu = slice_gate_up(full_gu, Ish, s_lo, s_hi).contiguous()
        sh_dn = slice_down(full_dn, s_lo, s_hi).contiguous()
    return DeviceLayer(cfg=cfg, shard=shard, router=router, gate_vec=gv, gate_up=gate_up, down=down,
                       sh_gate_up=sh_gu, sh_down=sh_dn)


def device_layer_host_view(dl: DeviceLayer) -> HostLayer:
    """Host copies of an unsharded device layer's router, gate vector and shared
    expert; routed experts are read back on demand."""
    if dl.shard.variant != "none":
        raise ValueError("host view needs the unsharded layer")
    hl = HostLayer(cfg=dl.cfg, layer=-1, seed=-1, router=dl.router.cpu().numpy(),
                   gate_vec=dl.gate_vec.cpu().numpy(), sh_gate_up=dl.sh_gate_up.cpu().numpy(),
                   sh_down=dl.sh_down.cpu().numpy(), fetch=dl.expert_bytes_host)
    return hl
