"""The MoE stack sharded over the GPUs of one node (one process per GPU).

Each rank holds one shard of every layer (config.Shard: variant "A" by expert
id, variant "B" by intermediate rows) and produces a partial sum; the single
exchange per layer is a sum over ranks, as in the reference
(`TTModel._moe_block` -> `all_reduce`, tt/model.py:2041-2052, over tt-fabric,
tt/ops.py:97-111).  Two ways to run it:

* exchange="kernel" (variant B, 2/4/8 ranks, one token): every rank runs the
  whole stack as one persistent launch (`qmoe_stack_decode_xchg`), and the
  kernel itself stores each layer's partial rows into the peers' exchange
  buffers over NVLink and sums the ranks' partials of its rows in rank order:
  no collective, every rank ends with the same bits.  The buffers are plain
  cudaMalloc allocations shared through CUDA IPC handles that the ranks
  all-gather over the process group.
* exchange="nccl": three launches per layer and an NCCL all-reduce of the
  fp32 [M, hidden] partial, all captured in one CUDA graph (any variant, any
  token count); the next layer reads the reduced sum (rounded to bf16 on
  load).

`torch.distributed` is the plumbing: process group, handle exchange,
barriers, and the graph-capturable collective of the NCCL mode.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from ._lib import XCHG_HANDLE_BYTES, LayerWeights, Xchg, check, lib
from .moe import Workspace, _stream
from .weights import DeviceLayer


def gather_handles(handle: bytes, group=None) -> list[bytes]:
    """Every rank's exchange-buffer handle, in rank order."""
    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    return [bytes(h) for h in out]


def kernel_exchange_supported(layers: list[DeviceLayer], m: int = 1) -> bool:
    """True when the in-kernel exchange runs this shard (variant B, 2-8 ranks, one token)."""
    shard = layers[0].shard
    if shard.variant != "B" or shard.world < 2:
        return False
    dims = shard.dims(layers[0].cfg)
    return bool(lib.qmoe_stack_xchg_supported(ctypes.byref(dims), shard.world, m, len(layers)))


class ShardedMoEStack:
    def __init__(self, layers: list[DeviceLayer], group=None, max_tokens: int = 16, use_graph: bool = True,
                 exchange: str = "auto"):
        if not layers:
            raise ValueError("empty stack")
        self.layers = layers
        self.cfg = layers[0].cfg
        self.shard = layers[0].shard
        self.group = group
        self.dims = self.shard.dims(self.cfg)
        self.device = layers[0].router.device
        self.max_tokens = max_tokens
        if exchange == "auto":
            exchange = "kernel" if max_tokens == 1 and kernel_exchange_supported(layers) else "nccl"
        if exchange not in ("kernel", "nccl"):
            raise ValueError(f"unknown exchange {exchange!r}")
        if exchange == "kernel" and not kernel_exchange_supported(layers):
            raise ValueError("the in-kernel exchange needs variant B on 2, 4 or 8 ranks of the compiled shapes")
        self.exchange = exchange
        self.c_layers = [l.c_struct() for l in layers]
        self.c_layer_array = (LayerWeights * len(layers))(*self.c_layers)
        self.ws = Workspace(self.dims, max_tokens, self.device)
        self.x_in = torch.zeros(max_tokens, self.cfg.hidden, dtype=torch.bfloat16, device=self.device)
        self.act = torch.zeros(max_tokens, self.cfg.hidden, dtype=torch.float32, device=self.device)
        self.use_graph = use_graph
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self._xchg = None
        self._own_buf = None
        self._peer_bufs: list[int] = []
        self._needs_reset = False
        if exchange == "kernel":
            self._open_exchange()

    # ---- in-kernel exchange --------------------------------------------------
    def _open_exchange(self) -> None:
        world, rank = self.shard.world, self.shard.rank
        buf = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(XCHG_HANDLE_BYTES)
        with torch.cuda.device(self.device):
            check(lib.qmoe_xchg_alloc(world, self.cfg.hidden, ctypes.byref(buf), handle), "qmoe_xchg_alloc")
            self._own_buf = buf.value
            try:
                handles = gather_handles(handle.raw, self.group)
                xc = Xchg(rank=rank, n_ranks=world)
                for q, h in enumerate(handles):
                    if q == rank:
                        xc.buf[q] = self._own_buf
                        continue
                    peer = ctypes.c_void_p()
                    check(lib.qmoe_xchg_open(h, ctypes.byref(peer)), f"qmoe_xchg_open rank {q}")
                    self._peer_bufs.append(peer.value)
                    xc.buf[q] = peer.value
            except BaseException:
                # no kernel has used the buffers yet: unmap and free this rank's share at once
                for p in self._peer_bufs:
                    lib.qmoe_xchg_close(p)
                self._peer_bufs = []
                lib.qmoe_xchg_free(self._own_buf)
                self._own_buf = None
                raise
        self._xchg = xc
        dist.barrier(group=self.group)

    def reset_exchange(self) -> None:
        """Every rank zeroes its own exchange buffer (launch counter and receive words), with no
        launch in flight and a barrier before and after: the in-kernel exchange starts again from
        launch 0.  Collective: every rank calls it (check_and_recover does, when any rank failed)."""
        if self._xchg is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            check(lib.qmoe_xchg_reset(self._own_buf, self.shard.world, self.cfg.hidden, _stream()), "qmoe_xchg_reset")
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._needs_reset = False

    def check_and_recover(self) -> int:
        """Collective status check after a step: every rank reads its workspace status word; if
        any rank saw an error (or failed to launch), every rank resets the exchange so that the
        launch counters agree again.  Returns this rank's status (0 when all went well)."""
        st = self.ws.read_status()
        bad = torch.tensor([float(st != 0 or self._needs_reset)], device=self.device)
        dist.all_reduce(bad, op=dist.ReduceOp.MAX, group=self.group)
        if bad.item() > 0:
            self.reset_exchange()
        return st

    # ---- launches ------------------------------------------------------------
    def _launch(self, m: int) -> None:
        if self.exchange == "kernel":
            if m != 1:
                raise ValueError("the in-kernel exchange runs one token per step")
            try:
                check(lib.qmoe_stack_decode_xchg(self.x_in.data_ptr(), m, self.c_layer_array, len(self.c_layers),
                                                 ctypes.byref(self.dims), ctypes.byref(self._xchg),
                                                 self.act.data_ptr(), self.ws.ptr, self.ws.nbytes, _stream()),
                      "qmoe_stack_decode_xchg")
            except BaseException:
                # this rank's launch counter did not advance: the peers' next launches would wait
                # for flags it never writes until every rank resets (check_and_recover)
                self._needs_reset = True
                raise
            return
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
            if self.exchange == "kernel":
                # the ranks' warm-up launches wait on one another: start them together
                torch.cuda.synchronize(self.device)
                dist.barrier(group=self.group)
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

    def read_status(self) -> int:
        """The workspace status word (0, or the first QMOE_ERR_* a kernel recorded)."""
        return self.ws.read_status()

    def phase_trace(self, m: int = 1):
        """Stamps of the last in-kernel-exchange launch ([2, n_layers, TRACE_SLOTS], as MoEStack.phase_trace)."""
        import numpy as np

        from .stack import TRACE_SLOTS

        n = len(self.c_layers)
        buf = np.zeros((2, n, TRACE_SLOTS), dtype=np.uint64)
        check(lib.qmoe_read_stack_trace(self.ws.ptr, ctypes.byref(self.dims), m, n, buf.ctypes.data, _stream()),
              "qmoe_read_stack_trace")
        return buf

    def release(self) -> None:
        """Drop captured graphs (they hold NCCL work) before destroy_process_group,
        and unmap and free the exchange buffers once no rank has a launch in flight."""
        self._graphs.clear()
        if self._xchg is not None:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            for p in self._peer_bufs:
                check(lib.qmoe_xchg_close(p), "qmoe_xchg_close")
            self._peer_bufs = []
            dist.barrier(group=self.group)
            check(lib.qmoe_xchg_free(self._own_buf), "qmoe_xchg_free")
            self._own_buf = None
            self._xchg = None
