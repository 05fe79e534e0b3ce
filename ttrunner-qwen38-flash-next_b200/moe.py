"""The MoE block on the device, behind the reference's operator interface.

`MoELayer` is the drop-in for `TTModel._moe_block(mixed, layer)`
(tt/model.py:2010-2052): routed experts plus the sigmoid-gated shared
expert, x [M, hidden] -> [M, hidden] fp32 (a partial sum when sharded; the
caller all-reduces).  Its stages are exposed as the reference's operators:

  route(x, router_w, top_k)                 tt/moe.py:308   -> (weights, keep) [M, E]
  apply_experts(x, weights, keep, ...)      tt/moe.py:330   -> routed output
  moe_block(x, router_w, gate_w, up_w, ...) tt/moe.py:159   -> routed output
  shared_expert(x, gate_w, up_w, down_w, g) tt/moe.py:983   -> shared output

Routing is exact top-k with ties to the lower expert id by default (the
reference's device kernel in EXACT_TOPK mode, scripts/kernels/router_select.cpp
:198-222, and its CPU model); `route_mode="threshold"` / `"threshold_bf16"`
selects the tie-admitting mode of the same kernel (:223-255) and of the ttnn
chain (tt/moe.py:308-327), with up to 16 experts per token.  Errors raise
`QMoEError` instead of warning and falling back (tt/moe.py:264-271) -- there is
no fallback path.

IQ4_XS operands are uint8 tensors of GGUF bytes: gate_w [E, I, D/256*136]
(or the fused gate|up [E, 2I, D/256*136] with up_w None, as
`TTWeights.fused_gate_up`, tt/weights.py:66-99), down_w [E, D, I/256*136].
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import Dims, LayerWeights, QMoEError, check, lib
from .config import MoEConfig, Shard
from .weights import DeviceLayer


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dims_key(d: Dims) -> tuple:
    return tuple(getattr(d, f) for f, _ in Dims._fields_)


class Workspace:
    """Device scratch for one shape family: router logits, routing table, h."""

    def __init__(self, dims: Dims, max_tokens: int, device: torch.device):
        self.dims = dims
        self.max_tokens = max_tokens
        nbytes = lib.qmoe_workspace_bytes(ctypes.byref(dims), max_tokens)
        if nbytes == 0:
            raise QMoEError(_lib.QMOE_ERR_UNSUPPORTED, "qmoe_workspace_bytes")
        self.buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        check(lib.qmoe_workspace_init(self.buf.data_ptr(), nbytes, _stream()), "qmoe_workspace_init")

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()

    @property
    def nbytes(self) -> int:
        return self.buf.numel()

    def read_status(self) -> int:
        st = ctypes.c_int(0)
        check(lib.qmoe_read_status(self.ptr, ctypes.byref(st), _stream()), "qmoe_read_status")
        return st.value

    def raise_if_error(self, where: str = "device") -> None:
        st = self.read_status()
        if st != _lib.QMOE_OK:
            raise QMoEError(st, where)


_WS: dict[tuple, Workspace] = {}


def workspace_for(dims: Dims, max_tokens: int, device: torch.device) -> Workspace:
    key = (_dims_key(dims), max_tokens, str(device))
    ws = _WS.get(key)
    if ws is None:
        ws = _WS[key] = Workspace(dims, max_tokens, device)
    return ws


class PrefillWorkspace(Workspace):
    """Device scratch of the chunked-prefill path for chunks of up to `max_tokens` tokens: bf16 copy
    of x, router logits, routing table, per-expert groups, h [T * (k + 1), inter] bf16."""

    def __init__(self, dims: Dims, max_tokens: int, device: torch.device):
        self.dims = dims
        self.max_tokens = max_tokens
        nbytes = lib.qmoe_prefill_workspace_bytes(ctypes.byref(dims), max_tokens)
        if nbytes == 0:
            raise QMoEError(_lib.QMOE_ERR_UNSUPPORTED, "qmoe_prefill_workspace_bytes")
        self.buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        check(lib.qmoe_workspace_init(self.buf.data_ptr(), nbytes, _stream()), "qmoe_workspace_init")


_PWS: dict[tuple, PrefillWorkspace] = {}


def prefill_workspace_for(dims: Dims, n_tokens: int, device: torch.device) -> PrefillWorkspace:
    """A prefill workspace covering n_tokens (grown in powers of two, kept per shape and device)."""
    key = (_dims_key(dims), str(device))
    ws = _PWS.get(key)
    if ws is None or ws.max_tokens < n_tokens:
        cap = min(max(128, 1 << (n_tokens - 1).bit_length()), lib.qmoe_prefill_max_tokens())
        ws = _PWS[key] = PrefillWorkspace(dims, max(cap, n_tokens), device)
    return ws


def _shaped(out: torch.Tensor, x: torch.Tensor, out_dtype: torch.dtype | None) -> torch.Tensor:
    """[M, K] fp32 -> x's leading shape ([1, 1, M, K] for the reference's operators) and dtype
    `out_dtype` (None: fp32, the accumulation type; torch.bfloat16: the reference's device dtype)."""
    out = out.view(*x.shape[:-1], out.shape[-1])
    return out if out_dtype is None or out_dtype == torch.float32 else out.to(out_dtype)


def _act(x: torch.Tensor) -> tuple[torch.Tensor, int]:
    """[.., M, D] bf16/fp32 -> contiguous [M, D] and its act dtype code."""
    if not x.is_cuda:
        raise ValueError("x must be a CUDA tensor")
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    if x2.dtype == torch.bfloat16:
        return x2, _lib.QMOE_ACT_BF16
    if x2.dtype == torch.float32:
        return x2, _lib.QMOE_ACT_F32
    raise TypeError(f"activations must be bf16 or fp32, got {x.dtype}")


class MoELayer:
    """One MoE block resident in HBM (one shard of it)."""

    ROUTE_MODES = ("exact", "threshold", "threshold_bf16")

    def __init__(self, layer: DeviceLayer, max_tokens: int | None = None, route_mode: str = "exact",
                 k_sel: int = 16):
        """route_mode: "exact" top-k, or the tie-admitting threshold select at the top_k-th
        probability in fp32 ("threshold") or bf16 ("threshold_bf16") with k_sel slots."""
        if route_mode not in self.ROUTE_MODES:
            raise ValueError(f"route_mode {route_mode!r} not in {self.ROUTE_MODES}")
        self.layer = layer
        self.cfg: MoEConfig = layer.cfg
        self.shard: Shard = layer.shard
        self.route_mode = route_mode
        self.dims = layer.shard.dims(layer.cfg)
        if route_mode != "exact":
            if not layer.cfg.top_k <= k_sel <= 16:
                raise ValueError(f"k_sel {k_sel} outside [top_k, 16]")
            self.dims.top_k = k_sel  # the slots the experts see
        self.max_tokens = max_tokens or lib.qmoe_max_tokens()
        self.weights = layer.c_struct()
        self.ws = workspace_for(self.dims, self.max_tokens, layer.router.device)

    @property
    def slots(self) -> int:
        """Routed slots per token: top_k, or k_sel in a threshold mode."""
        return self.dims.top_k

    def _m(self, x: torch.Tensor) -> int:
        m = x.shape[0]
        if not 1 <= m <= self.max_tokens:
            raise ValueError(f"{m} tokens outside [1, {self.max_tokens}]")
        return m

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None,
                 out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """x [.., M, hidden] (e.g. the reference's [1, 1, M, K]) -> the same leading shape, fp32 (or
        `out_dtype`).  `out`: an fp32 buffer of M x hidden values to write into (kept as given)."""
        x2, dt = _act(x)
        m = self._m(x2)
        given = out is not None
        if self.route_mode != "exact":
            ids, w, sl = self.route(x2)
            y = self.down(self.gate_up(x2, ids), ids, w, sl)
            if given:
                out.view(m, self.cfg.hidden).copy_(y)
                return out
            return _shaped(y, x, out_dtype)
        if out is None:
            out = torch.empty(m, self.cfg.hidden, dtype=torch.float32, device=x2.device)
        check(lib.qmoe_moe_block(x2.data_ptr(), dt, m, ctypes.byref(self.weights), ctypes.byref(self.dims),
                                 out.data_ptr(), self.ws.ptr, self.ws.nbytes, _stream()), "qmoe_moe_block")
        return out if given else _shaped(out, x, out_dtype)

    # ---- chunked prefill (tt/model.py:2812-2907 _prefill_ffn_half) ------------
    def prefill(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """x [T, hidden] bf16/fp32 -> [T, hidden] fp32: route, group tokens per expert, tcgen05
        grouped GEMMs (gate|up + SwiGLU, down + weighted scatter-add), shared expert."""
        x2, dt = _act(x)
        t = x2.shape[0]
        ws = prefill_workspace_for(self.dims, t, x2.device)
        if out is None:
            out = torch.empty(t, self.cfg.hidden, dtype=torch.float32, device=x2.device)
        check(lib.qmoe_prefill(x2.data_ptr(), dt, t, ctypes.byref(self.weights), ctypes.byref(self.dims),
                               out.data_ptr(), ws.ptr, ws.nbytes, _stream()), "qmoe_prefill")
        return out

    def prefill_route(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(ids [T, k] int32, weights [T, k] fp32, shared_logit [T] fp32) for a chunk of T tokens."""
        x2, dt = _act(x)
        t = x2.shape[0]
        k = self.cfg.top_k
        ws = prefill_workspace_for(self.dims, t, x2.device)
        ids = torch.empty(t, k, dtype=torch.int32, device=x2.device)
        w = torch.empty(t, k, dtype=torch.float32, device=x2.device)
        sl = torch.empty(t, dtype=torch.float32, device=x2.device)
        check(lib.qmoe_prefill_route(x2.data_ptr(), dt, t, ctypes.byref(self.weights), ctypes.byref(self.dims),
                                     ids.data_ptr(), w.data_ptr(), sl.data_ptr(), ws.ptr, ws.nbytes, _stream()),
              "qmoe_prefill_route")
        return ids, w, sl

    def prefill_experts(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                        shared_logit: torch.Tensor | None) -> torch.Tensor:
        """Routed experts (+ the shared expert) of a chunk for a given routing table."""
        x2, dt = _act(x)
        t = x2.shape[0]
        ws = prefill_workspace_for(self.dims, t, x2.device)
        ids = ids.to(torch.int32).contiguous()
        weights = weights.to(torch.float32).contiguous()
        sl = None if shared_logit is None else shared_logit.to(torch.float32).contiguous()
        out = torch.empty(t, self.cfg.hidden, dtype=torch.float32, device=x2.device)
        check(lib.qmoe_prefill_experts(x2.data_ptr(), dt, t, ids.data_ptr(), weights.data_ptr(),
                                       None if sl is None else sl.data_ptr(), ctypes.byref(self.weights),
                                       ctypes.byref(self.dims), out.data_ptr(), ws.ptr, ws.nbytes, _stream()),
              "qmoe_prefill_experts")
        return out

    def route(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(ids [M, slots] int32, weights [M, slots] fp32, shared_logit [M] fp32)."""
        x2, dt = _act(x)
        m = self._m(x2)
        k = self.slots
        ids = torch.empty(m, k, dtype=torch.int32, device=x2.device)
        w = torch.empty(m, k, dtype=torch.float32, device=x2.device)
        sl = torch.empty(m, dtype=torch.float32, device=x2.device)
        if self.route_mode == "exact":
            check(lib.qmoe_route(x2.data_ptr(), dt, m, ctypes.byref(self.weights), ctypes.byref(self.dims),
                                 ids.data_ptr(), w.data_ptr(), sl.data_ptr(), self.ws.ptr, self.ws.nbytes,
                                 _stream()), "qmoe_route")
        else:
            check(lib.qmoe_route_threshold(x2.data_ptr(), dt, m, ctypes.byref(self.weights), ctypes.byref(self.dims),
                                           self.cfg.top_k, int(self.route_mode == "threshold_bf16"), ids.data_ptr(),
                                           w.data_ptr(), sl.data_ptr(), self.ws.ptr, self.ws.nbytes, _stream()),
                  "qmoe_route_threshold")
        return ids, w, sl

    def gate_up(self, x: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        """h [M, k+1, I_loc] fp32; slot k is the shared expert."""
        x2, dt = _act(x)
        m = self._m(x2)
        hs = max(self.dims.inter_local, self.dims.sh_inter_local)
        h = torch.zeros(m, self.slots + 1, hs, dtype=torch.float32, device=x2.device)
        ids = ids.to(torch.int32).contiguous()
        check(lib.qmoe_gateup_swiglu(x2.data_ptr(), dt, m, ids.data_ptr(), ctypes.byref(self.weights),
                                     ctypes.byref(self.dims), h.data_ptr(), hs, self.ws.ptr,
                                     self.ws.nbytes, _stream()), "qmoe_gateup_swiglu")
        return h

    def down(self, h: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
             shared_logit: torch.Tensor | None) -> torch.Tensor:
        m = h.shape[0]
        out = torch.empty(m, self.cfg.hidden, dtype=torch.float32, device=h.device)
        ids = ids.to(torch.int32).contiguous()
        weights = weights.to(torch.float32).contiguous()
        check(lib.qmoe_down_combine(h.data_ptr(), h.shape[-1], m, ids.data_ptr(), weights.data_ptr(),
                                    None if shared_logit is None else shared_logit.data_ptr(),
                                    ctypes.byref(self.weights), ctypes.byref(self.dims), out.data_ptr(),
                                    self.ws.ptr, self.ws.nbytes, _stream()), "qmoe_down_combine")
        return out


# ---------------------------------------------------------------------------
# the reference's operator interface on raw tensors

_FUSED: dict[tuple, torch.Tensor] = {}


def _fused_gate_up(gate_w: torch.Tensor, up_w: torch.Tensor | None) -> torch.Tensor:
    if up_w is None:
        return gate_w.contiguous()
    key = (gate_w.data_ptr(), up_w.data_ptr(), tuple(gate_w.shape))
    t = _FUSED.get(key)
    if t is None:
        t = _FUSED[key] = torch.cat([gate_w, up_w], dim=-2).contiguous()
    return t


def _raw_dims(hidden: int, inter: int, n_experts: int, top_k: int, shared_inter: int = 0) -> Dims:
    nseg, nsub, ib0 = Shard.row_slice(0, inter)
    d = Dims(hidden=hidden, inter=inter, n_experts=n_experts, top_k=top_k, expert_lo=0,
             expert_hi=n_experts, inter_local=inter, down_nseg=nseg, down_nsub=nsub, down_ib0=ib0)
    if shared_inter:
        s = Shard.row_slice(0, shared_inter)
        d.sh_inter_local = shared_inter
        d.sh_down_nseg, d.sh_down_nsub, d.sh_down_ib0 = s
    return d


def _check_u8(t: torch.Tensor, name: str) -> None:
    if t.dtype != torch.uint8 or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA uint8 tensor of IQ4_XS bytes")


def moe_block(x: torch.Tensor, router_w: torch.Tensor, gate_w: torch.Tensor, up_w: torch.Tensor | None,
              down_w: torch.Tensor, top_k: int, num_experts: int, hidden_size: int,
              intermediate_size: int, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Routed experts only (tt/moe.py:159-295): x [1, 1, M, K] (or any [.., M, K]) -> the same
    leading shape, fp32, or `out_dtype` (torch.bfloat16 for the reference's device dtype)."""
    _check_u8(gate_w, "gate_w")
    _check_u8(down_w, "down_w")
    x2, dt = _act(x)
    m = x2.shape[0]
    gu = _fused_gate_up(gate_w, up_w)
    dims = _raw_dims(hidden_size, intermediate_size, num_experts, top_k)
    # Keep every operand referenced until the launches are enqueued.
    r_w, d_w = router_w.float().contiguous(), down_w.contiguous()
    w = LayerWeights(router=r_w.data_ptr(), gate_vec=None, gate_up=gu.data_ptr(),
                     down=d_w.data_ptr(), sh_gate_up=None, sh_down=None)
    ws = workspace_for(dims, max(m, 1), x2.device)
    out = torch.empty(m, hidden_size, dtype=torch.float32, device=x2.device)
    check(lib.qmoe_moe_block(x2.data_ptr(), dt, m, ctypes.byref(w), ctypes.byref(dims), out.data_ptr(),
                             ws.ptr, ws.nbytes, _stream()), "moe_block")
    return _shaped(out, x, out_dtype)


def shared_expert(x: torch.Tensor, gate_w: torch.Tensor, up_w: torch.Tensor, down_w: torch.Tensor,
                  gate_vec: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """sigmoid(x . gate_vec) * down(silu(gate x) * up x) (tt/moe.py:983-1044): x [1, 1, M, K] (or
    any [.., M, K]) -> the same leading shape, fp32 or `out_dtype`."""
    _check_u8(gate_w, "gate_w")
    _check_u8(up_w, "up_w")
    _check_u8(down_w, "down_w")
    x2, dt = _act(x)
    m = x2.shape[0]
    inter = gate_w.shape[-2]
    hidden = down_w.shape[-2]
    gu = _fused_gate_up(gate_w, up_w)
    dims = _raw_dims(hidden, inter, 32, 1, shared_inter=inter)
    g_v, d_w = gate_vec.float().contiguous(), down_w.contiguous()
    w = LayerWeights(router=None, gate_vec=g_v.data_ptr(), gate_up=None,
                     down=None, sh_gate_up=gu.data_ptr(), sh_down=d_w.data_ptr())
    ws = workspace_for(dims, max(m, 1), x2.device)
    out = torch.empty(m, hidden, dtype=torch.float32, device=x2.device)
    check(lib.qmoe_shared_expert(x2.data_ptr(), dt, m, ctypes.byref(w), ctypes.byref(dims), out.data_ptr(),
                                 ws.ptr, ws.nbytes, _stream()), "shared_expert")
    return _shaped(out, x, out_dtype)


def route_topk(x: torch.Tensor, router_w: torch.Tensor, top_k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(ids [M, k] int32, weights [M, k] fp32), descending, ties to the lower id."""
    x2, dt = _act(x)
    m = x2.shape[0]
    E, D = router_w.shape
    dims = _raw_dims(D, 256, E, top_k)
    r_w = router_w.float().contiguous()
    w = LayerWeights(router=r_w.data_ptr())
    ids = torch.empty(m, top_k, dtype=torch.int32, device=x2.device)
    wt = torch.empty(m, top_k, dtype=torch.float32, device=x2.device)
    if m > lib.qmoe_max_tokens():  # a prefill chunk
        pws = prefill_workspace_for(dims, m, x2.device)
        check(lib.qmoe_prefill_route(x2.data_ptr(), dt, m, ctypes.byref(w), ctypes.byref(dims), ids.data_ptr(),
                                     wt.data_ptr(), None, pws.ptr, pws.nbytes, _stream()), "route")
        return ids, wt
    ws = workspace_for(dims, max(m, 1), x2.device)
    check(lib.qmoe_route(x2.data_ptr(), dt, m, ctypes.byref(w), ctypes.byref(dims), ids.data_ptr(),
                         wt.data_ptr(), None, ws.ptr, ws.nbytes, _stream()), "route")
    return ids, wt


def dequant(fmt: int, raw: torch.Tensor) -> torch.Tensor:
    """GGML blocks of `fmt` (Q8_0, IQ4_NL, IQ3_S, IQ4_XS; uint8 CUDA tensor [..., row bytes]) -> fp32
    [..., values], bitwise the reference's `gguf.quants.dequantize`."""
    if raw.dtype != torch.uint8 or not raw.is_cuda:
        raise TypeError("raw must be a CUDA uint8 tensor of GGML blocks")
    blk = {8: (32, 34), 20: (32, 18), 21: (256, 110), 23: (256, 136)}.get(fmt)
    if blk is None:
        raise ValueError(f"unsupported GGML type {fmt}")
    bv, bb = blk
    raw = raw.contiguous()
    n = raw.numel() // bb * bv
    out = torch.empty(*raw.shape[:-1], raw.shape[-1] // bb * bv, dtype=torch.float32, device=raw.device)
    check(lib.qmoe_dequant_f32(fmt, raw.data_ptr(), n, out.data_ptr(), _stream()), "qmoe_dequant_f32")
    return out


def moe_block_formats(x: torch.Tensor, router_w: torch.Tensor, gate_vec: torch.Tensor | None,
                      gate_up: torch.Tensor, down: torch.Tensor, sh_gate_up: torch.Tensor | None,
                      sh_down: torch.Tensor | None, formats: tuple[int, int, int, int], top_k: int,
                      out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """The MoE block (routed experts + sigmoid-gated shared expert, reference/model.py:387-417) on the
    real checkpoint's formats: `formats` = GGML types of (gate|up, down, shared gate|up, shared down),
    e.g. (IQ3_S, IQ4_NL, IQ3_S, Q8_0) as tt/plan.py:90-103 loads them.  gate_up [E, 2I, row bytes],
    down [E, D, row bytes] uint8 CUDA tensors; x [.., M, D] -> the same leading shape."""
    x2, dt = _act(x)
    m = x2.shape[0]
    E, D = router_w.shape
    I = gate_up.shape[1] // 2
    Ish = sh_gate_up.shape[0] // 2 if sh_gate_up is not None else 0
    def segs(n):  # the IQ4_XS row-slice fields, consistent with a whole row (unused by other formats)
        return (n // 256, 8) if n % 256 == 0 else (n // 32, 1)

    (dseg, dsub), (sseg, ssub) = segs(I), segs(max(Ish, 32))
    dims = Dims(hidden=D, inter=I, n_experts=E, top_k=top_k, expert_lo=0, expert_hi=E, inter_local=I,
                down_nseg=dseg, down_nsub=dsub, down_ib0=0, sh_inter_local=Ish, sh_down_nseg=sseg,
                sh_down_nsub=ssub, sh_down_ib0=0)
    r_w = router_w.float().contiguous()
    g_v = gate_vec.float().contiguous() if gate_vec is not None else None
    gu, dn = gate_up.contiguous(), down.contiguous()
    sgu = sh_gate_up.contiguous() if sh_gate_up is not None else None
    sdn = sh_down.contiguous() if sh_down is not None else None
    w = LayerWeights(router=r_w.data_ptr(), gate_vec=None if g_v is None else g_v.data_ptr(),
                     gate_up=gu.data_ptr(), down=dn.data_ptr(),
                     sh_gate_up=None if sgu is None else sgu.data_ptr(), sh_down=None if sdn is None else sdn.data_ptr())
    f = _lib.Formats(*formats)
    ws = workspace_for(dims, max(m, 1), x2.device)
    out = torch.empty(m, D, dtype=torch.float32, device=x2.device)
    check(lib.qmoe_moe_block_formats(x2.data_ptr(), dt, m, ctypes.byref(w), ctypes.byref(dims), ctypes.byref(f),
                                     out.data_ptr(), ws.ptr, ws.nbytes, _stream()), "qmoe_moe_block_formats")
    return _shaped(out, x, out_dtype)


def route_threshold(x: torch.Tensor, router_w: torch.Tensor, top_k: int, k_sel: int = 16,
                    probs_bf16: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """The tie-admitting select (router_select.cpp:223-255, TT_ROUTER_EXACT_TOPK=0): (ids [M, k_sel]
    int32, weights [M, k_sel] fp32), every expert at or above the top_k-th probability (bf16 when
    probs_bf16, as the ttnn chain compares them), largest first, ties to the lower id, renormalised
    over all of them; unused slots are (0, 0)."""
    x2, dt = _act(x)
    m = x2.shape[0]
    E, D = router_w.shape
    dims = _raw_dims(D, 256, E, k_sel)
    r_w = router_w.float().contiguous()
    w = LayerWeights(router=r_w.data_ptr())
    ids = torch.empty(m, k_sel, dtype=torch.int32, device=x2.device)
    wt = torch.empty(m, k_sel, dtype=torch.float32, device=x2.device)
    if m > lib.qmoe_max_tokens():  # a prefill chunk
        pws = prefill_workspace_for(dims, m, x2.device)
        check(lib.qmoe_prefill_route_threshold(x2.data_ptr(), dt, m, ctypes.byref(w), ctypes.byref(dims), top_k,
                                               int(probs_bf16), ids.data_ptr(), wt.data_ptr(), None, pws.ptr,
                                               pws.nbytes, _stream()), "route_threshold")
        return ids, wt
    ws = workspace_for(dims, max(m, 1), x2.device)
    check(lib.qmoe_route_threshold(x2.data_ptr(), dt, m, ctypes.byref(w), ctypes.byref(dims), top_k,
                                   int(probs_bf16), ids.data_ptr(), wt.data_ptr(), None, ws.ptr, ws.nbytes,
                                   _stream()), "route_threshold")
    return ids, wt


def route(x: torch.Tensor, router_w: torch.Tensor, top_k: int,
          mode: str = "exact") -> tuple[torch.Tensor, torch.Tensor]:
    """Dense routing as tt/moe.py:308-327 returns it: (weights, keep), both with x's leading shape
    and E last ([1, 1, M, E] for the reference's [1, 1, M, K] activations).  mode "exact": the top_k
    (the reference's default device select); "threshold_bf16": the ttnn chain's own rule, every
    probability >= the top_k-th in bf16 kept (up to 16); "threshold": the same on fp32 probabilities."""
    if mode == "exact":
        ids, wt = route_topk(x, router_w, top_k)
    elif mode in ("threshold", "threshold_bf16"):
        ids, wt = route_threshold(x, router_w, top_k, 16, mode == "threshold_bf16")
    else:
        raise ValueError(f"route mode {mode!r}")
    E = router_w.shape[0]
    dense = torch.zeros(ids.shape[0], E, dtype=torch.float32, device=ids.device)
    dense.scatter_add_(1, ids.long(), wt)
    if mode == "exact":
        keep = torch.zeros_like(dense).scatter_(1, ids.long(), 1.0)
    else:  # the padding slots (id 0, weight 0) keep nothing
        keep = (dense > 0).float()
    lead = x.shape[:-1]
    return dense.view(*lead, E), keep.view(*lead, E)


def apply_experts(x: torch.Tensor, weights: torch.Tensor, keep: torch.Tensor, gate_w: torch.Tensor,
                  up_w: torch.Tensor | None, down_w: torch.Tensor, num_experts: int, hidden_size: int,
                  intermediate_size: int, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Routed output for dense routing (tt/moe.py:330-368): the experts kept per row.  x [1, 1, M, K]
    (or any [.., M, K]) with weights / keep [.., M, E] -> x's leading shape, fp32 or `out_dtype`."""
    _check_u8(gate_w, "gate_w")
    _check_u8(down_w, "down_w")
    x2, dt = _act(x)
    m = x2.shape[0]
    weights = weights.reshape(m, -1)
    keep = keep.reshape(m, -1)
    k = int(keep.sum(dim=-1).max().item())
    if k < 1:
        return _shaped(torch.zeros(m, hidden_size, dtype=torch.float32, device=x2.device), x, out_dtype)
    kv, ids = torch.topk(keep.float() * 2.0 + weights.float(), k, dim=-1)
    wt = torch.gather(weights.float(), 1, ids)
    wt = torch.where(torch.gather(keep.float(), 1, ids) > 0, wt, torch.zeros_like(wt))
    gu = _fused_gate_up(gate_w, up_w)
    dims = _raw_dims(hidden_size, intermediate_size, num_experts, k)
    d_w = down_w.contiguous()
    lw = LayerWeights(gate_up=gu.data_ptr(), down=d_w.data_ptr())
    if m > lib.qmoe_max_tokens():  # a prefill chunk: grouped tensor-core path
        pws = prefill_workspace_for(dims, m, x2.device)
        ids32 = ids.to(torch.int32).contiguous()
        wt = wt.contiguous()
        out = torch.empty(m, hidden_size, dtype=torch.float32, device=x2.device)
        check(lib.qmoe_prefill_experts(x2.data_ptr(), dt, m, ids32.data_ptr(), wt.data_ptr(), None, ctypes.byref(lw),
                                       ctypes.byref(dims), out.data_ptr(), pws.ptr, pws.nbytes, _stream()),
              "apply_experts")
        return _shaped(out, x, out_dtype)
    ws = workspace_for(dims, max(m, 1), x2.device)
    hs = intermediate_size
    h = torch.empty(m, k + 1, hs, dtype=torch.float32, device=x2.device)
    ids32 = ids.to(torch.int32).contiguous()
    check(lib.qmoe_gateup_swiglu(x2.data_ptr(), dt, m, ids32.data_ptr(), ctypes.byref(lw), ctypes.byref(dims),
                                 h.data_ptr(), hs, ws.ptr, ws.nbytes, _stream()), "apply_experts gate|up")
    out = torch.empty(m, hidden_size, dtype=torch.float32, device=x2.device)
    wt = wt.contiguous()
    check(lib.qmoe_down_combine(h.data_ptr(), hs, m, ids32.data_ptr(), wt.data_ptr(), None, ctypes.byref(lw),
                                ctypes.byref(dims), out.data_ptr(), ws.ptr, ws.nbytes, _stream()),
          "apply_experts down")
    return _shaped(out, x, out_dtype)
