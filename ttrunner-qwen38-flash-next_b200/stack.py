"""The 48-layer MoE decode stack as one CUDA graph.

`MoEStack.decode(x)` runs n_layers MoE blocks back to back, the fp32 output of
layer L (rounded to bf16 on load, the activation dtype) feeding layer L+1 --
the per-layer MoE calls of `TTModel.step` (tt/model.py:2056) with nothing in
between.  The reference replays the step as a ttnn trace
(`TracedDecoder.step`, tt/traced.py:261-277); here the whole stack is one
`qmoe_stack_decode` call captured once per token count into a CUDA graph, and
a step is a graph replay.  Buffers are allocated once and reused by every
layer and every replay (the reference's persistent-output rule,
tt/moe.py:392-409).
"""

from __future__ import annotations

import ctypes

import torch

from ._lib import LayerWeights, check, lib
from .moe import Workspace, _stream
from .weights import DeviceLayer


# The single-launch kernel's phase stamps per layer (qmoe_read_stack_trace).
TRACE_SLOTS = 24
TRACE_POINTS = ("layer start", "x gathered", "x checked", "ranked, gate|up copies issued", "shared pairs done",
                "gate|up pairs done", "h words written", "h round complete", "h converted", "down rows landed",
                "down done", "output rows written", "arrived", "", "", "",
                "gate|up chunk 0 landed", "chunk 1 landed", "chunk 2 landed", "chunk 3 landed", "chunk 4 landed",
                "chunk 5 landed", "exchange: partial rows sent", "exchange: peers' rows summed")


class MoEStack:
    def __init__(self, layers: list[DeviceLayer], max_tokens: int = 16, use_graph: bool = True):
        if not layers:
            raise ValueError("empty stack")
        self.layers = layers
        self.cfg = layers[0].cfg
        self.shard = layers[0].shard
        self.dims = self.shard.dims(self.cfg)
        self.max_tokens = max_tokens
        self.device = layers[0].router.device
        self.c_layers = (LayerWeights * len(layers))(*[l.c_struct() for l in layers])
        self.ws = Workspace(self.dims, max_tokens, self.device)
        self.x_in = torch.zeros(max_tokens, self.cfg.hidden, dtype=torch.bfloat16, device=self.device)
        self.out = torch.zeros(max_tokens, self.cfg.hidden, dtype=torch.float32, device=self.device)
        self.use_graph = use_graph
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}

    @property
    def n_layers(self) -> int:
        return len(self.layers)

    TRACE_POINTS = TRACE_POINTS

    def phase_trace(self, m: int = 1):
        """Raw SM cycle-counter stamps of the last single-launch step,
        [2, n_layers, TRACE_SLOTS]: CTA 0 then the last CTA, in the order of
        TRACE_POINTS (unnamed slots unused)."""
        import numpy as np

        buf = np.zeros((2, self.n_layers, TRACE_SLOTS), dtype=np.uint64)
        check(lib.qmoe_read_stack_trace(self.ws.ptr, ctypes.byref(self.dims), m, self.n_layers,
                                        buf.ctypes.data, _stream()), "qmoe_read_stack_trace")
        return buf

    def route_trace(self, n_layers: int | None = None):
        """The single launch's per-layer record of its last one-token call: (act [L, hidden] fp32
        holding each layer's bf16 output, ids [L, k] int32, weights [L, k] fp32)."""
        import numpy as np

        n = self.n_layers if n_layers is None else n_layers
        k, D = self.cfg.top_k, self.cfg.hidden
        act = np.zeros((n, D), dtype=np.uint16)
        ids = np.zeros((n, k), dtype=np.int32)
        w = np.zeros((n, k), dtype=np.float32)
        check(lib.qmoe_read_stack_route_trace(self.ws.ptr, ctypes.byref(self.dims), 1, n, act.ctypes.data,
                                              ids.ctypes.data, w.ctypes.data, _stream()), "qmoe_read_stack_route_trace")
        return (act.astype(np.uint32) << 16).view(np.float32), ids, w

    def decode_teacher(self, x_layers: torch.Tensor) -> torch.Tensor:
        """The single launch with layer L's input taken from x_layers[L] (bf16 [n_layers, hidden])
        instead of layer L-1's output; returns the last layer's fp32 output.  Per-layer outputs,
        ids and weights: route_trace()."""
        xl = x_layers.to(device=self.device, dtype=torch.bfloat16).contiguous()
        if xl.shape != (self.n_layers, self.cfg.hidden):
            raise ValueError(f"x_layers must be [{self.n_layers}, {self.cfg.hidden}]")
        check(lib.qmoe_stack_decode_teacher(xl.data_ptr(), self.c_layers, self.n_layers, ctypes.byref(self.dims),
                                            self.out.data_ptr(), self.ws.ptr, self.ws.nbytes, _stream()),
              "qmoe_stack_decode_teacher")
        return self.out[:1]

    def single_launch(self, m: int = 1) -> bool:
        """True when a step of m tokens is one persistent kernel launch."""
        return bool(lib.qmoe_stack_single_launch(ctypes.byref(self.dims), m, self.n_layers))

    def _launch(self, m: int) -> None:
        check(lib.qmoe_stack_decode(self.x_in.data_ptr(), m, self.c_layers, self.n_layers,
                                    ctypes.byref(self.dims), self.out.data_ptr(), self.ws.ptr,
                                    self.ws.nbytes, _stream()), "qmoe_stack_decode")

    def graph(self, m: int) -> torch.cuda.CUDAGraph:
        g = self._graphs.get(m)
        if g is None:
            self._launch(m)  # warm-up outside capture (sets kernel attributes)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._launch(m)
            self._graphs[m] = g
        return g

    def run(self, m: int) -> torch.Tensor:
        """One step on the tokens already in `x_in[:m]`; returns out[:m] (a view)."""
        if self.use_graph:
            self.graph(m).replay()
        else:
            self._launch(m)
        return self.out[:m]

    def decode(self, x: torch.Tensor) -> torch.Tensor:
        """x [M, hidden] (any device, bf16 or castable) -> out [M, hidden] fp32 on the device."""
        m = x.shape[0]
        if not 1 <= m <= self.max_tokens:
            raise ValueError(f"{m} tokens outside [1, {self.max_tokens}]")
        self.x_in[:m].copy_(x.reshape(m, -1), non_blocking=True)
        return self.run(m)
