"""The hyper-connection mixer around the MoE block, behind the reference's
operators (tt/ops.py:2627 `gated_residual_mix`, :2825 `reinject`; the CPU
model's `_gated_residual` / `_reinject`, reference/model.py:53-81).

The model keeps `hc` residual streams, hyper [.., M, hc * hidden].  Before
the block, `gated_residual_mix` RMS-normalises each stream, gates it through
a low-rank projection and averages the streams into the block's input
`mixed` [.., M, hidden]; after it, `reinject` adds the block's output back
into every stream, stream s weighted by inject[.., s].  On the device: three
launches for the mix, one for the reinjection (csrc/hc.cu).
"""

from __future__ import annotations

import ctypes

import torch

from ._lib import QMOE_ACT_BF16, QMOE_ACT_F32, HcDims, HcWeights, check, lib


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dt(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return QMOE_ACT_BF16
    if t.dtype == torch.float32:
        return QMOE_ACT_F32
    raise TypeError(f"activations must be bf16 or fp32, got {t.dtype}")


_WS: dict = {}


def _workspace(dims: HcDims, m: int, device) -> torch.Tensor:
    n = lib.qmoe_hc_workspace_bytes(ctypes.byref(dims), m)
    if n == 0:
        raise ValueError("hyper-connection shapes outside what the kernels are built for")
    key = (device, n)
    ws = _WS.get(key)
    if ws is None:
        ws = _WS[key] = torch.empty(n + 256, dtype=torch.uint8, device=device)
    off = (-ws.data_ptr()) % 256
    return ws[off:off + n]


def gated_residual_mix(hyper: torch.Tensor, norm_w: torch.Tensor, down_w: torch.Tensor, up_w: torch.Tensor,
                       inject_w: torch.Tensor | None, eps: float, hc_count: int,
                       hidden_size: int) -> tuple[torch.Tensor, torch.Tensor | None]:
    """(mixed [.., M, hidden] fp32, inject [.., M, hc] fp32 or None without inject_w) for hyper
    [.., M, hc * hidden] (bf16 or fp32): the reference's read gate (tt/ops.py:2627-2711)."""
    lead = hyper.shape[:-1]
    n = hc_count * hidden_size
    if hyper.shape[-1] != n:
        raise ValueError(f"hyper's last axis is {hyper.shape[-1]}, expected hc * hidden = {n}")
    h2 = hyper.reshape(-1, n).contiguous()
    m = h2.shape[0]
    rank = down_w.shape[0]
    nw = norm_w.float().contiguous()
    dw = down_w.float().contiguous()
    uw = up_w.float().contiguous()
    iw = (inject_w.float() if inject_w is not None else torch.zeros(hc_count, n, device=hyper.device)).contiguous()
    dims = HcDims(hidden=hidden_size, hc=hc_count, rank=rank, eps=float(eps))
    w = HcWeights(norm_w=nw.data_ptr(), down_w=dw.data_ptr(), up_w=uw.data_ptr(), inject_w=iw.data_ptr())
    mixed = torch.empty(m, hidden_size, dtype=torch.float32, device=hyper.device)
    inject = torch.empty(m, hc_count, dtype=torch.float32, device=hyper.device)
    ws = _workspace(dims, m, hyper.device)
    check(lib.qmoe_hc_mix(h2.data_ptr(), _dt(h2), m, ctypes.byref(w), ctypes.byref(dims), mixed.data_ptr(),
                          inject.data_ptr(), ws.data_ptr(), ws.numel(), _stream()), "qmoe_hc_mix")
    return mixed.view(*lead, hidden_size), (inject.view(*lead, hc_count) if inject_w is not None else None)


def reinject(hyper: torch.Tensor, branch: torch.Tensor, inject: torch.Tensor, hc_count: int) -> torch.Tensor:
    """hyper + branch (outer) inject, flattened back to [.., M, hc * hidden] fp32 (tt/ops.py:2825;
    model.py:80-81).  branch [.., M, hidden] bf16 / fp32; inject [.., M, hc]."""
    n = hyper.shape[-1]
    hidden = n // hc_count
    lead = hyper.shape[:-1]
    h2 = hyper.reshape(-1, n).contiguous()
    b2 = branch.reshape(-1, hidden).contiguous()
    i2 = inject.reshape(-1, hc_count).float().contiguous()
    m = h2.shape[0]
    dims = HcDims(hidden=hidden, hc=hc_count, rank=1, eps=0.0)
    out = torch.empty(m, n, dtype=torch.float32, device=hyper.device)
    check(lib.qmoe_hc_reinject(h2.data_ptr(), _dt(h2), b2.data_ptr(), _dt(b2), i2.data_ptr(), m, ctypes.byref(dims),
                               out.data_ptr(), _stream()), "qmoe_hc_reinject")
    return out.view(*lead, n)
