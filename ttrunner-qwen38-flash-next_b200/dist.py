"""The MoE stack sharded over the GPUs of one node (one process per GPU).

Each rank holds one shard of every layer (config.Shard: variant "A" by expert
id, variant "B" by intermediate rows) and produces a partial sum; the single
exchange per layer is a sum over ranks, as in the reference
(`TTModel._moe_block` -> `all_reduce`, tt/model.py:2041-2052, over tt-fabric,
tt/ops.py:97-111).  Here it is an NCCL all-reduce of the fp32 [M, hidden]
partial over NVLink/NVSwitch, captured with the MoE launches of all layers in
one CUDA graph; the next layer reads the reduced sum (rounded to bf16 on
load).  `torch.distributed` is the plumbing: process group, communicator and
the graph-capturable collective.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from ._lib import check, lib
from .moe import Workspace, _stream
from .weights import DeviceLayer


class ShardedMoEStack:
    def __init__(self, layers: list[DeviceLayer], group=None, max_tokens: int = 16, use_graph: bool = True):
        if not layers:
            raise ValueError("empty stack")
        self.layers = layers
        self.cfg = layers[0].cfg
        self.shard = layers[0].shard
        self.group = group
        self.dims = self.shard.dims(self.cfg)
        self.device = layers[0].router.device
        self.max_tokens = max_tokens
        self.c_layers = [l.c_struct() for l in layers]
        self.ws = Workspace(self.dims, max_tokens, self.device)
        self.x_in = torch.zeros(max_tokens, self.cfg.hidden, dtype=torch.bfloat16, device=self.device)
        self.act = torch.zeros(max_tokens, self.cfg.hidden, dtype=torch.float32, device=self.device)
        self.use_graph = use_graph
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}

    def _launch(self, m: int) -> None:
        part = self.act[:m]
        for l, w in enumerate(self.c_layers):
            x, dt = (self.x_in, 0) if l == 0 else (self.act, 1)
            check(lib.qmoe_moe_block(x.data_ptr(), dt, m, ctypes.byref(w), ctypes.byref(self.dims),
                                     self.act.data_ptr(), self.ws.ptr, self.ws.nbytes, _stream()),
                  f"qmoe_moe_block layer {l}")
            if self.shard.world > 1:
                dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)

    def graph(self, m: int) -> torch.cuda.CUDAGraph:
        g = self._graphs.get(m)
        if g is None:
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                self._launch(m)  # warm-up: kernel attributes, NCCL communicator
            torch.cuda.current_stream(self.device).wait_stream(s)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._launch(m)
            self._graphs[m] = g
        return g

    def run(self, m: int) -> torch.Tensor:
        if self.use_graph:
            self.graph(m).replay()
        else:
            self._launch(m)
        return self.act[:m]

    def decode(self, x: torch.Tensor) -> torch.Tensor:
        m = x.shape[0]
        self.x_in[:m].copy_(x.reshape(m, -1), non_blocking=True)
        return self.run(m)

    def release(self) -> None:
        """Drop captured graphs (they hold NCCL work) before destroy_process_group."""
        self._graphs.clear()
