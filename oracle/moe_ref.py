"""TEST INFRASTRUCTURE ONLY -- the CPU oracle of the qwen4exp MoE block.

Only tests/, `__graft_entry__.smoke()` and bench.py's CPU-baseline leg may
import this module, and only as the checker (or the timed CPU baseline); the
product path never calls it.

A numpy restatement of the reference's plain-PyTorch CPU MoE,
`Qwen4ExpModel._moe` (ttrunner_qwen38_flash_next/reference/model.py:387-417),
on weights served by a `WeightStore`-like source that dequantises one
expert at a time (reference/weights.py:118-179).  IQ4_XS decoding is the C
restatement in iq4xs_ref.c (gguf/quants.py:112-129).

Pinning: tests/golden/ holds outputs of the reference itself (imported in the
development container and run on the same seeded IQ4_XS bytes) and of its
dequantiser; tests/test_oracle.py checks this module against them.

The one deliberate difference from the reference is the tie rule of top-k:
the reference's `torch.topk` (model.py:401) does not break ties by lower
index on CPU, so the oracle canonicalises to a stable (-p, index) order -- the
rule of the reference's own device kernel (scripts/kernels/router_select.cpp
:163-164).  `raw_topk_differs` reports when that changes the selected set.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_SO = HERE / "liboracle_iq4xs.so"


def build() -> Path:
    """Compile the C restatements (make in this directory)."""
    srcs = [HERE / "iq4xs_ref.c", HERE / "synth_ref.c", HERE / "formats_ref.c", HERE / "iq3s_grid.inc",
            HERE / "Makefile"]
    if not _SO.exists() or any(_SO.stat().st_mtime < s.stat().st_mtime for s in srcs):
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return _SO


_lib = None


def _c() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        _lib.oracle_dequant_iq4xs.restype = None
        _lib.oracle_dequant_iq4xs.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        for name in ("oracle_synth_f32", "oracle_synth_iq4xs"):
            fn = getattr(_lib, name)
            fn.restype = None
            fn.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p]
        _lib.oracle_quantize_iq4xs.restype = None
        _lib.oracle_quantize_iq4xs.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        _lib.oracle_dequant.restype = ctypes.c_int
        _lib.oracle_dequant.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    return _lib


def synth_f32(seed: int, sid: int, n: int, std: float) -> np.ndarray:
    """n values of the synthetic generator's stream (seed, sid), fp32 (synth_ref.c)."""
    out = np.empty(n, dtype=np.float32)
    _c().oracle_synth_f32(seed, sid, n, std, out.ctypes.data)
    return out


def synth_iq4xs(seed: int, sid: int, n_values: int, std: float) -> np.ndarray:
    """The same stream quantised to IQ4_XS: n_values / 256 * 136 bytes (synth_ref.c)."""
    if n_values % 256:
        raise ValueError("n_values must be a multiple of 256")
    out = np.empty(n_values // 256 * 136, dtype=np.uint8)
    _c().oracle_synth_iq4xs(seed, sid, n_values, std, out.ctypes.data)
    return out


def quantize_iq4xs(values: np.ndarray) -> np.ndarray:
    """fp32 [..., n] (n % 256 == 0) -> IQ4_XS bytes [..., n / 256 * 136] (synth_ref.c)."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(v.shape[:-1] + (v.shape[-1] // 256 * 136,), dtype=np.uint8)
    _c().oracle_quantize_iq4xs(v.ctypes.data, v.size, out.ctypes.data)
    return out


def dequant_iq4xs(raw: np.ndarray) -> np.ndarray:
    """IQ4_XS bytes [..., n_sb*136] -> fp32 [..., n_sb*256] (quants.py:112-129)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    if raw.shape[-1] % 136:
        raise ValueError("last dimension is not a whole number of 136-byte super-blocks")
    nb = raw.size // 136
    out = np.empty(raw.shape[:-1] + (raw.shape[-1] // 136 * 256,), dtype=np.float32)
    _c().oracle_dequant_iq4xs(raw.ctypes.data, nb, out.ctypes.data)
    return out


# GGML type ids and block traits (gguf/reader.py:53-74, 85-108): (values, bytes) per block.
Q8_0, IQ4_NL, IQ3_S, IQ4_XS = 8, 20, 21, 23
BLOCK = {Q8_0: (32, 34), IQ4_NL: (32, 18), IQ3_S: (256, 110), IQ4_XS: (256, 136)}


def row_bytes(fmt: int, n_values: int) -> int:
    bv, bb = BLOCK[fmt]
    if n_values % bv:
        raise ValueError(f"{n_values} values is not a whole number of blocks of format {fmt}")
    return n_values // bv * bb


def dequant(fmt: int, raw: np.ndarray) -> np.ndarray:
    """Bytes [..., row bytes] of `fmt` -> fp32 [..., values] (quants.py; formats_ref.c)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    bv, bb = BLOCK[fmt]
    if raw.shape[-1] % bb:
        raise ValueError("last dimension is not a whole number of blocks")
    n = raw.size // bb * bv
    out = np.empty(raw.shape[:-1] + (raw.shape[-1] // bb * bv,), dtype=np.float32)
    if _c().oracle_dequant(fmt, raw.ctypes.data, ctypes.c_int64(n), out.ctypes.data) != 0:
        raise ValueError(f"format {fmt}")
    return out


def synth_format_bytes(fmt: int, seed: int, sid: int, n_rows: int, row_values: int,
                       d_scale: float) -> np.ndarray:
    """Seeded bytes of `fmt` [n_rows, row bytes]: every byte from the exact-arithmetic generator's
    stream, then each block's fp16 scale set to d_scale * (1 + |z| / 2) so the decoded weights have
    the magnitude of N(0, 0.02) weights (no quantiser exists here for these formats; the
    reference decodes whatever bytes it is given)."""
    rb = row_bytes(fmt, row_values)
    n = n_rows * rb
    u = np.abs(synth_f32(seed, sid, n, 1.0)).astype(np.float64)
    raw = (np.floor(u * 1e6).astype(np.int64) % 256).astype(np.uint8).reshape(n_rows, rb)
    bv, bb = BLOCK[fmt]
    z = np.abs(synth_f32(seed, sid + 1000, n_rows * (rb // bb), 1.0)).reshape(n_rows, rb // bb)
    d = (np.float32(d_scale) * (np.float32(1.0) + z / np.float32(2.0))).astype(np.float16)
    blocks = raw.reshape(n_rows, rb // bb, bb)
    blocks[:, :, 0:2] = d.view(np.uint8).reshape(n_rows, rb // bb, 2)
    return blocks.reshape(n_rows, rb)


def synth_formats_layer(seed: int, E: int, D: int, I: int, Ish: int) -> dict:
    """A seeded layer in the real checkpoint's format mix: IQ3_S gate|up [E, 2I, ...], IQ4_NL down
    [E, D, ...], IQ3_S shared gate|up, Q8_0 shared down, fp32 router and gate vector."""
    return {
        "formats": (IQ3_S, IQ4_NL, IQ3_S, Q8_0),
        "gate_up": synth_format_bytes(IQ3_S, seed, 1, E * 2 * I, D, 2e-4).reshape(E, 2 * I, -1),
        "down": synth_format_bytes(IQ4_NL, seed, 2, E * D, I, 2e-4).reshape(E, D, -1),
        "sh_gate_up": synth_format_bytes(IQ3_S, seed, 3, 2 * Ish, D, 2e-4),
        "sh_down": synth_format_bytes(Q8_0, seed, 4, D, Ish, 2e-4),
        "router": synth_f32(seed, 5, E * D, 0.02).reshape(E, D),
        "gate_vec": synth_f32(seed, 6, D, 0.02),
    }


def dequant_iq4xs_numpy(raw: np.ndarray) -> np.ndarray:
    """The same decode written with numpy array operations (a second restatement)."""
    kv = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], dtype=np.int8)
    b = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1, 136)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    sh = b[:, 2:4].copy().view(np.uint16).astype(np.uint32)[:, 0]
    sl = b[:, 4:8].astype(np.uint32)
    qs = b[:, 8:136]
    out = np.empty((b.shape[0], 256), dtype=np.float32)
    for ib in range(8):
        ls = ((sl[:, ib // 2] >> (4 * (ib % 2))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4)
        dl = d * (ls.astype(np.float32) - np.float32(32.0))
        q = qs[:, ib * 16:(ib + 1) * 16]
        out[:, ib * 32:ib * 32 + 16] = kv[q & 0xF] * dl[:, None]
        out[:, ib * 32 + 16:ib * 32 + 32] = kv[q >> 4] * dl[:, None]
    return out.reshape(raw.shape[:-1] + (raw.shape[-1] // 136 * 256,))


def _silu(v: np.ndarray) -> np.ndarray:
    return v / (np.float32(1.0) + np.exp(-v))


def _sigmoid(v: np.ndarray) -> np.ndarray:
    return np.float32(1.0) / (np.float32(1.0) + np.exp(-v))


def softmax(logits: np.ndarray) -> np.ndarray:
    """fp32 softmax over the last axis (model.py:400)."""
    z = logits - logits.max(axis=-1, keepdims=True)
    e = np.exp(z, dtype=np.float32)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def topk_canonical(probs: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """The k largest per row, ties to the lower index, in descending order."""
    order = np.argsort(-probs, axis=-1, kind="stable")[..., :k]
    return np.take_along_axis(probs, order, -1), order.astype(np.int64)


def route(x: np.ndarray, router: np.ndarray, k: int) -> dict:
    """model.py:399-403: logits, probabilities, top-k and renormalised weights."""
    logits = (x @ router.T).astype(np.float32)
    probs = softmax(logits)
    w, ids = topk_canonical(probs, k)
    w = (w / w.sum(axis=-1, keepdims=True)).astype(np.float32)
    return {"logits": logits, "probs": probs, "ids": ids, "weights": w}


def bf16_round(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 -> fp32, round to nearest even (finite values)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def _lane_sum(v: np.ndarray) -> np.float32:
    """Sum of E values (E % 32 == 0) in the device warp's order: lane t adds
    ids t, t + 32, ... in turn, then a butterfly over the 32 lanes."""
    lanes = np.zeros(32, np.float32)
    for j in range(v.shape[0] // 32):
        lanes = (lanes + v[32 * j:32 * (j + 1)]).astype(np.float32)
    for o in (16, 8, 4, 2, 1):
        lanes = (lanes + lanes[np.arange(32) ^ o]).astype(np.float32)
    return lanes[0]


def route_threshold(logits: np.ndarray, k: int, k_sel: int, e_lo: int = 0, e_hi: int | None = None,
                    probs_bf16: bool = False) -> tuple[np.ndarray, np.ndarray]:
    """The reference device select's tie-admitting mode, EXACT_TOPK off
    (scripts/kernels/router_select.cpp:223-255): on the softmax probabilities
    (rounded to bf16 when probs_bf16, as the ttnn chain compares them,
    tt/moe.py:318-327) the threshold is the k-th largest counting equal values
    separately (:176-193); `total` sums every probability >= the threshold
    (:226-235); the k_sel largest positive ones >= the threshold inside
    [e_lo, e_hi) are selected, ties to the lower id (:237-254), with weight
    p * (1 / total) (:256-260); empty slots are (e_lo, 0).  The softmax sum and
    `total` are taken in the device warp's order (_lane_sum) -- the reference
    sums in id order -- so the oracle matches the kernel to the last bit of
    its own arithmetic.  logits [M, E] fp32 -> ids [M, k_sel] int32, weights
    [M, k_sel] fp32."""
    logits = np.asarray(logits, dtype=np.float32)
    M, E = logits.shape
    e_hi = E if e_hi is None else e_hi
    ids = np.full((M, k_sel), e_lo, dtype=np.int32)
    wts = np.zeros((M, k_sel), dtype=np.float32)
    for m in range(M):
        l = logits[m].copy()
        l[np.isnan(l)] = -np.inf
        p = np.exp((l - l.max()).astype(np.float32)).astype(np.float32)
        probs = (p / _lane_sum(p)).astype(np.float32)
        if probs_bf16:
            probs = bf16_round(probs)
        thr = np.sort(probs)[::-1][k - 1]
        total = _lane_sum(np.where(probs >= thr, probs, np.float32(0.0)).astype(np.float32))
        inv = np.float32(1.0) / total if total > 0 else np.float32(0.0)
        cand = [e for e in range(e_lo, e_hi) if probs[e] > 0 and probs[e] >= thr]
        cand.sort(key=lambda e: (-probs[e], e))
        for i, e in enumerate(cand[:k_sel]):
            ids[m, i] = e
            wts[m, i] = np.float32(probs[e] * inv)
    return ids, wts


def route_threshold_dense(logits: np.ndarray, k: int, probs_bf16: bool = True) -> np.ndarray:
    """The ttnn chain of tt/moe.py:318-327 on CPU: probabilities, their k-th
    largest as the threshold, keep = probs >= threshold, the kept ones
    renormalised -> dense weights [M, E] (every kept expert, no slot cap)."""
    probs = softmax(np.asarray(logits, dtype=np.float32))
    if probs_bf16:
        probs = bf16_round(probs)
    thr = -np.sort(-probs, axis=-1)[:, k - 1:k]
    kept = np.where(probs >= thr, probs, np.float32(0.0)).astype(np.float32)
    return (kept / kept.sum(axis=-1, keepdims=True)).astype(np.float32)


def raw_topk_differs(probs: np.ndarray, ids: np.ndarray, k: int) -> np.ndarray:
    """Rows whose `torch.topk` selection differs as a set from the canonical one."""
    import torch

    raw = torch.topk(torch.from_numpy(probs), k, dim=-1).indices.numpy()
    return np.array([set(a) != set(b) for a, b in zip(raw.tolist(), ids.tolist())])


class ExpertSource:
    """Dequantising weight source in the role of WeightStore.get_rows
    (reference/weights.py:118-179): experts come from `expert(e)` as IQ4_XS
    bytes (gate|up [2I, rb], down [D, rb_dn]) and are decoded on each use."""

    def __init__(self, expert, sh_gate_up: np.ndarray | None, sh_down: np.ndarray | None,
                 router: np.ndarray, gate_vec: np.ndarray | None, inter: int, shared_inter: int,
                 formats: tuple[int, int, int, int] = (23, 23, 23, 23)):
        """formats: GGML types of (gate|up, down, shared gate|up, shared down); IQ4_XS by default."""
        self.formats = formats
        self.expert = expert
        self.sh_gate_up = sh_gate_up
        self.sh_down = sh_down
        self.router = router
        self.gate_vec = gate_vec
        self.inter = inter
        self.shared_inter = shared_inter

    @classmethod
    def from_host_layer(cls, hl) -> "ExpertSource":
        return cls(hl.expert, hl.sh_gate_up, hl.sh_down, hl.router, hl.gate_vec,
                   hl.cfg.inter, hl.cfg.shared_inter)


def moe_forward(x: np.ndarray, src: ExpertSource, k: int, with_shared: bool = True,
                expert_window: tuple[int, int] | None = None,
                inter_window: tuple[int, int] | None = None, cache: dict | None = None,
                routing: tuple[np.ndarray, np.ndarray] | None = None) -> dict:
    """Qwen4ExpModel._moe (model.py:387-417) on flat fp32 x [M, D].

    expert_window / inter_window restrict the routed experts to a variant-A
    window or every expert (and the shared one) to a variant-B slice of the
    intermediate axis: the partial sum a rank produces before the all-reduce.
    cache: dequantised experts kept across calls (keys: expert id, "shared"),
    the role of WeightStore's row cache (reference/weights.py:48-53) when it
    is warm; None decodes every expert on each use (cold).
    routing: (ids [M, n], weights [M, n]) to use instead of the top-k of
    model.py:399-403 (e.g. route_threshold's selection; weight-0 slots add 0).
    """

    def dq(key, gu_b, dn_b):
        fg, fd = src.formats[2:4] if key == "shared" else src.formats[0:2]
        if cache is None:
            return dequant(fg, gu_b), dequant(fd, dn_b)
        got = cache.get(key)
        if got is None:
            got = cache[key] = (dequant(fg, gu_b), dequant(fd, dn_b))
        return got

    x = np.ascontiguousarray(x, dtype=np.float32)
    M = x.shape[0]
    I, Ish = src.inter, src.shared_inter
    lo, hi = inter_window if inter_window is not None else (0, I)
    slo, shi = (lo * Ish // I, hi * Ish // I) if inter_window is not None else (0, Ish)

    shared = np.zeros_like(x)
    if with_shared and src.sh_gate_up is not None:                                   # :392-397
        gu, dn = dq("shared", src.sh_gate_up, src.sh_down)
        h = _silu(x @ gu[slo:shi].T) * (x @ gu[Ish + slo:Ish + shi].T)
        s = h @ dn[:, slo:shi].T
        gate = _sigmoid(x @ src.gate_vec.reshape(-1, 1))
        shared = (s * gate).astype(np.float32)

    r = route(x, src.router, k)                                                      # :399-403
    if routing is not None:
        r["ids"], r["weights"] = routing
    ids, weights = r["ids"], r["weights"]
    out = np.zeros_like(x)
    for e in np.unique(ids):                                                          # :407
        e = int(e)
        if expert_window is not None and not expert_window[0] <= e < expert_window[1]:
            continue
        slot, tok = np.nonzero(ids == e)                                             # :409
        gu_b, dn_b = src.expert(e)
        gu, dn = dq(e, gu_b, dn_b)                                                    # :411-413
        xs = x[slot]
        h = _silu(xs @ gu[lo:hi].T) * (xs @ gu[I + lo:I + hi].T)                      # :414
        np.add.at(out, slot, (h @ dn[:, lo:hi].T) * weights[slot, tok, None])        # :415
    r.update(out=(out + shared).astype(np.float32), routed=out, shared=shared)       # :417
    return r


def max_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max|got - ref| / max|ref|, the reference harnesses' error metric
    (scripts/stage3_swiglu_fusion.py:128-133)."""
    denom = float(np.max(np.abs(ref)))
    diff = float(np.max(np.abs(np.asarray(got, dtype=np.float64) - np.asarray(ref, dtype=np.float64))))
    if denom == 0.0:
        return 0.0 if diff == 0.0 else float("inf")
    return diff / denom


def threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
