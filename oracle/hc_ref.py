"""TEST INFRASTRUCTURE ONLY -- the CPU oracle of the hyper-connection mixer
around the MoE block.

Only tests/ and tests/golden/make_golden.py import this module, as the
checker; the product path never calls it.

A numpy restatement of the reference's gated residual (its "hyper
connections"), reference/model.py:53-81:

  normed  = rms_norm(hyper, norm_w, eps, group_size=hidden)      (layers.py:31-43)
  mix     = sigmoid(silu(normed @ down_w.T / hc) @ up_w.T)        (model.py:68-69)
  mixed   = mean over the hc streams of mix * normed              (model.py:70-71)
  inject  = 2 * sigmoid(normed @ inject_w.T / hc)                 (model.py:75-77)
  reinject: hyper + branch (outer) inject, flattened              (model.py:80-81)

hyper [M, hc * hidden] fp32; the MoE block consumes `mixed` and its output is
the `branch` that `reinject` adds back into every stream, weighted per stream.
Pinned by tests/golden/hc_*.npz, outputs of the reference's own
Qwen4ExpModel._gated_residual / _reinject on the same inputs.
"""

from __future__ import annotations

import numpy as np

from . import moe_ref


def synth_weights(seed: int, hidden: int, hc: int, rank: int) -> dict:
    """Seeded fp32 mixer weights (the exact-arithmetic generator of moe_ref)."""
    n = hc * hidden
    return {
        "norm_w": (np.float32(1.0) + moe_ref.synth_f32(seed, 11, n, 0.1)).astype(np.float32),
        "down_w": moe_ref.synth_f32(seed, 12, rank * n, 0.02).reshape(rank, n),
        "up_w": moe_ref.synth_f32(seed, 13, n * rank, 0.05).reshape(n, rank),
        "inject_w": moe_ref.synth_f32(seed, 14, hc * n, 0.02).reshape(hc, n),
    }


def synth_inputs(seed: int, hidden: int, hc: int, m: int) -> tuple[np.ndarray, np.ndarray]:
    """bf16-representable hyper [m, hc * hidden] (each stream its own scale) and branch [m, hidden]."""
    h = moe_ref.synth_f32(seed, 15, m * hc * hidden, 1.0).reshape(m, hc, hidden)
    h = h * (np.float32(0.5) + np.arange(hc, dtype=np.float32)).reshape(1, hc, 1)
    b = moe_ref.synth_f32(seed, 16, m * hidden, 1.0).reshape(m, hidden)
    return moe_ref.bf16_round(h.reshape(m, hc * hidden)), moe_ref.bf16_round(b)


def rms_norm_groups(x: np.ndarray, w: np.ndarray, eps: float, group: int) -> np.ndarray:
    """layers.py:31-43 with group_size: each `group` values normalised on their own."""
    shp = x.shape
    g = x.reshape(*shp[:-1], -1, group).astype(np.float32)
    g = g * (np.float32(1.0) / np.sqrt((g * g).mean(-1, keepdims=True) + np.float32(eps)))
    return (g.reshape(shp) * w).astype(np.float32)


def gated_residual(hyper: np.ndarray, wts: dict, eps: float, hc: int, hidden: int) -> dict:
    """model.py:53-78 for a layer's mixer: (mixed [M, hidden], normed, inject [M, hc])."""
    x = np.asarray(hyper, dtype=np.float32)
    normed = rms_norm_groups(x, wts["norm_w"], eps, hidden)
    t = (normed.astype(np.float64) @ wts["down_w"].astype(np.float64).T).astype(np.float32) / np.float32(hc)
    mix = (t / (np.float32(1.0) + np.exp(-t))).astype(np.float32)
    u = (mix.astype(np.float64) @ wts["up_w"].astype(np.float64).T).astype(np.float32)
    mix = (np.float32(1.0) / (np.float32(1.0) + np.exp(-u))).astype(np.float32)
    m = x.shape[0]
    mixed = (mix.reshape(m, hc, hidden) * normed.reshape(m, hc, hidden)).mean(axis=1).astype(np.float32)
    z = (normed.astype(np.float64) @ wts["inject_w"].astype(np.float64).T).astype(np.float32) / np.float32(hc)
    inject = (np.float32(2.0) / (np.float32(1.0) + np.exp(-z))).astype(np.float32)
    return {"mixed": mixed, "normed": normed, "inject": inject}


def reinject(hyper: np.ndarray, branch: np.ndarray, inject: np.ndarray) -> np.ndarray:
    """model.py:80-81: hyper + (branch[:, None, :] * inject[:, :, None]).flatten."""
    m, hc = inject.shape
    add = branch[:, None, :].astype(np.float32) * inject[:, :, None].astype(np.float32)
    return (np.asarray(hyper, dtype=np.float32) + add.reshape(m, -1)).astype(np.float32)
