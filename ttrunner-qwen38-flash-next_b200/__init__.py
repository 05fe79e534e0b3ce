"""B200-native qwen4exp MoE block (decode, verify, multi-GPU), a drop-in for
the per-layer MoE forward of ttrunner-qwen38-flash-next.

The compute is the C-ABI library `libqmoe_b200.so` (hand-written sm_100a
kernels, include/qmoe_b200.h); this package is its host-side mirror of the
reference's operator interface.  Importing it without the built library
raises: there is no fallback.
"""

from . import _lib
from ._lib import QMoEError
from .config import C1, C2, MoEConfig, Shard
from .moe import (
    MoELayer,
    PrefillWorkspace,
    Workspace,
    apply_experts,
    moe_block,
    route,
    dequant,
    moe_block_formats,
    route_threshold,
    route_topk,
    shared_expert,
)
from .gguf_load import CheckpointMoE, GGUFCheckpoint, load_moe_layer, load_moe_stack, moe_layer_bytes
from .hc import gated_residual_mix, reinject
from .stack import MoEStack
from .weights import (
    DeviceLayer,
    HostLayer,
    synth_device_layer,
    synth_host_layer,
    synth_x,
    upload_host_layer,
)

__all__ = [
    "C1", "C2", "MoEConfig", "Shard", "QMoEError", "MoELayer", "MoEStack", "Workspace", "PrefillWorkspace",
    "DeviceLayer", "HostLayer", "apply_experts", "moe_block", "route", "route_topk", "shared_expert",
    "synth_device_layer", "synth_host_layer", "synth_x", "upload_host_layer",
    "route_threshold",
    "gated_residual_mix",
    "reinject",
    "dequant",
    "moe_block_formats",
    "GGUFCheckpoint",
    "CheckpointMoE",
    "load_moe_layer",
    "moe_layer_bytes",
    "load_moe_stack",
]
