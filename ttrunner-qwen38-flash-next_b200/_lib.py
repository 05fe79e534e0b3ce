"""ctypes binding of `libqmoe_b200.so` (declared in include/qmoe_b200.h).

The library is the product: there is no Python or PyTorch fallback.  If it is
missing, importing this module raises; build it with `build.py`.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqmoe_b200.so"

QMOE_OK = 0
QMOE_ERR_INVALID_ARG = 1
QMOE_ERR_UNSUPPORTED = 2
QMOE_ERR_ALIGNMENT = 3
QMOE_ERR_WORKSPACE = 4
QMOE_ERR_CUDA = 5
QMOE_ERR_DEVICE_RANGE = 6
QMOE_ERR_NOT_FINITE = 7
QMOE_ERR_TIMEOUT = 8

QMOE_ACT_BF16 = 0
QMOE_ACT_F32 = 1


class QMoEError(RuntimeError):
    """A libqmoe_b200 entry point returned a non-zero status."""

    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {lib.qmoe_status_string(status).decode()} (status {status})")


class LayerWeights(ctypes.Structure):
    _fields_ = [
        ("router", c_void_p),
        ("gate_vec", c_void_p),
        ("gate_up", c_void_p),
        ("down", c_void_p),
        ("sh_gate_up", c_void_p),
        ("sh_down", c_void_p),
    ]


class Dims(ctypes.Structure):
    _fields_ = [
        ("hidden", c_int),
        ("inter", c_int),
        ("n_experts", c_int),
        ("top_k", c_int),
        ("expert_lo", c_int),
        ("expert_hi", c_int),
        ("inter_local", c_int),
        ("down_nseg", c_int),
        ("down_nsub", c_int),
        ("down_ib0", c_int),
        ("sh_inter_local", c_int),
        ("sh_down_nseg", c_int),
        ("sh_down_nsub", c_int),
        ("sh_down_ib0", c_int),
    ]


class Xchg(ctypes.Structure):
    """qmoe_xchg: this rank, the rank count and every rank's exchange buffer as mapped here."""

    _fields_ = [
        ("rank", c_int),
        ("n_ranks", c_int),
        ("buf", c_void_p * 8),
    ]


class Formats(ctypes.Structure):
    """qmoe_formats: GGML type ids of a layer's expert tensors."""

    _fields_ = [("gate_up", c_int), ("down", c_int), ("sh_gate_up", c_int), ("sh_down", c_int)]


QMOE_FMT_Q8_0, QMOE_FMT_IQ4_NL, QMOE_FMT_IQ3_S, QMOE_FMT_IQ4_XS = 8, 20, 21, 23


class HcWeights(ctypes.Structure):
    """qmoe_hc_weights: the hyper-connection mixer's fp32 weights."""

    _fields_ = [("norm_w", c_void_p), ("down_w", c_void_p), ("up_w", c_void_p), ("inject_w", c_void_p)]


class HcDims(ctypes.Structure):
    """qmoe_hc_dims."""

    _fields_ = [("hidden", c_int), ("hc", c_int), ("rank", c_int), ("eps", c_float)]


XCHG_HANDLE_BYTES = 64


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH.name} is not built: run `python {LIB_PATH.parent / 'build.py'}` "
            "(the MoE path has no fallback)"
        )
    return ctypes.CDLL(str(LIB_PATH))


lib = _load()

_P = c_void_p
_SIGS = {
    "qmoe_status_string": (ctypes.c_char_p, [c_int]),
    "qmoe_version": (c_int, []),
    "qmoe_max_tokens": (c_int, []),
    "qmoe_workspace_bytes": (c_size_t, [POINTER(Dims), c_int]),
    "qmoe_workspace_init": (c_int, [_P, c_size_t, _P]),
    "qmoe_read_status": (c_int, [_P, POINTER(c_int), _P]),
    "qmoe_dequant_iq4xs_f32": (c_int, [_P, c_int64, _P, _P]),
    "qmoe_quantize_iq4xs_host": (c_int, [_P, c_int64, _P, c_int]),
    "qmoe_quantize_iq4xs": (c_int, [_P, c_int64, _P, _P]),
    "qmoe_synth_iq4xs": (c_int, [c_uint64, c_uint64, c_int64, c_float, _P, _P]),
    "qmoe_synth_f32": (c_int, [c_uint64, c_uint64, c_int64, c_float, _P, _P]),
    "qmoe_synth_iq4xs_host": (c_int, [c_uint64, c_uint64, c_int64, c_float, _P, c_int]),
    "qmoe_synth_f32_host": (c_int, [c_uint64, c_uint64, c_int64, c_float, _P, c_int]),
    "qmoe_route": (c_int, [_P, c_int, c_int, POINTER(LayerWeights), POINTER(Dims), _P, _P, _P, _P,
                           c_size_t, _P]),
    "qmoe_route_threshold": (c_int, [_P, c_int, c_int, POINTER(LayerWeights), POINTER(Dims), c_int, c_int, _P,
                                     _P, _P, _P, c_size_t, _P]),
    "qmoe_gateup_swiglu": (c_int, [_P, c_int, c_int, _P, POINTER(LayerWeights), POINTER(Dims), _P,
                                   c_int, _P, c_size_t, _P]),
    "qmoe_down_combine": (c_int, [_P, c_int, c_int, _P, _P, _P, POINTER(LayerWeights),
                                  POINTER(Dims), _P, _P, c_size_t, _P]),
    "qmoe_moe_block": (c_int, [_P, c_int, c_int, POINTER(LayerWeights), POINTER(Dims), _P, _P,
                               c_size_t, _P]),
    "qmoe_shared_expert": (c_int, [_P, c_int, c_int, POINTER(LayerWeights), POINTER(Dims), _P, _P,
                                   c_size_t, _P]),
    "qmoe_stack_decode": (c_int, [_P, c_int, POINTER(LayerWeights), c_int, POINTER(Dims), _P, _P,
                                  c_size_t, _P]),
    "qmoe_read_stack_trace": (c_int, [_P, POINTER(Dims), c_int, c_int, _P, _P]),
    "qmoe_stack_single_launch": (c_int, [POINTER(Dims), c_int, c_int]),
    "qmoe_read_stack_route_trace": (c_int, [_P, POINTER(Dims), c_int, c_int, _P, _P, _P, _P]),
    "qmoe_stack_decode_teacher": (c_int, [_P, POINTER(LayerWeights), c_int, POINTER(Dims), _P, _P, c_size_t, _P]),
    "qmoe_xchg_bytes": (c_size_t, [c_int, c_int]),
    "qmoe_xchg_alloc": (c_int, [c_int, c_int, POINTER(c_void_p), _P]),
    "qmoe_xchg_open": (c_int, [_P, POINTER(c_void_p)]),
    "qmoe_xchg_close": (c_int, [_P]),
    "qmoe_xchg_free": (c_int, [_P]),
    "qmoe_xchg_reset": (c_int, [_P, c_int, c_int, _P]),
    "qmoe_stack_xchg_supported": (c_int, [POINTER(Dims), c_int, c_int, c_int]),
    "qmoe_stack_decode_xchg": (c_int, [_P, c_int, POINTER(LayerWeights), c_int, POINTER(Dims), POINTER(Xchg), _P,
                                       _P, c_size_t, _P]),
    "qmoe_moe_block_noalloc": (c_int, [_P, c_int, c_int, POINTER(LayerWeights), POINTER(Dims), _P, _P]),
    "qmoe_noalloc_read_status": (c_int, [POINTER(c_int), _P]),
    "qmoe_format_row_bytes": (c_size_t, [c_int, c_int64]),
    "qmoe_dequant_f32": (c_int, [c_int, _P, c_int64, _P, _P]),
    "qmoe_moe_block_formats": (c_int, [_P, c_int, c_int, POINTER(LayerWeights), POINTER(Dims), POINTER(Formats), _P,
                                       _P, c_size_t, _P]),
    "qmoe_hc_workspace_bytes": (c_size_t, [POINTER(HcDims), c_int]),
    "qmoe_hc_mix": (c_int, [_P, c_int, c_int, POINTER(HcWeights), POINTER(HcDims), _P, _P, _P, c_size_t, _P]),
    "qmoe_hc_reinject": (c_int, [_P, c_int, _P, c_int, _P, c_int, POINTER(HcDims), _P, _P]),
    "qmoe_prefill_max_tokens": (c_int, []),
    "qmoe_prefill_small_group_max": (c_int, [c_int]),
    "qmoe_prefill_trace": (c_int, [c_int]),
    "qmoe_prefill_workspace_bytes": (c_size_t, [POINTER(Dims), c_int]),
    "qmoe_prefill_route": (c_int, [_P, c_int, c_int, POINTER(LayerWeights), POINTER(Dims), _P, _P, _P, _P,
                                   c_size_t, _P]),
    "qmoe_prefill_route_threshold": (c_int, [_P, c_int, c_int, POINTER(LayerWeights), POINTER(Dims), c_int, c_int,
                                             _P, _P, _P, _P, c_size_t, _P]),
    "qmoe_prefill_experts": (c_int, [_P, c_int, c_int, _P, _P, _P, POINTER(LayerWeights), POINTER(Dims), _P,
                                     _P, c_size_t, _P]),
    "qmoe_prefill": (c_int, [_P, c_int, c_int, POINTER(LayerWeights), POINTER(Dims), _P, _P, c_size_t, _P]),
}

for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args

EXPORTED = tuple(_SIGS)


def check(status: int, where: str) -> None:
    if status != QMOE_OK:
        raise QMoEError(status, where)
