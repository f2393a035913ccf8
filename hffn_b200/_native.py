"""ctypes binding of ``libhffn_b200.so`` (the C ABI of ``include/hffn_b200.h``).

The library is built in-tree by ``hffn_b200.build`` (nvcc, sm_100a). There is no fallback: importing the runtime
without the library raises, so no HFFN call can run anywhere but in these kernels.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libhffn_b200.so"

HFFN_OK, HFFN_ERR_ARGUMENT, HFFN_ERR_CUDA, HFFN_ERR_LAYOUT = 0, 1, 2, 3
F32, BF16 = 0, 1
MODE_AUTO = -1
UP_CODES = {"coop": 0, "lane": 1, "tile": 2}
DOWN_CODES = {"coop": 0, "tiled": 1, "blocked": 2}

_P = ctypes.c_void_p
_I32, _I64 = ctypes.c_int32, ctypes.c_int64


class Layer(ctypes.Structure):
    _fields_ = [("d_model", _I32), ("d_ff", _I32), ("nnz_up", _I64), ("nnz_down", _I64),
                ("b_up", _P), ("up_offsets", _P), ("up_idx", _P), ("up_val", _P),
                ("b_down", _P), ("out_offsets", _P), ("out_hidden", _P), ("out_val", _P)]


class PeerConfig(ctypes.Structure):
    _fields_ = [("world", _I32), ("rank", _I32), ("tokens", _I64), ("dtype", _I32),
                ("gather", _P * 2), ("gather_peer", (ctypes.c_uint64 * 8) * 2),
                ("slots", _P * 3), ("slot_peer", (ctypes.c_uint64 * 8) * 3),
                ("partial", _P * 2), ("signal", _P), ("signal_peer", ctypes.c_uint64 * 8), ("work", _P)]


class Supports(ctypes.Structure):
    _fields_ = [("in_offsets", _P), ("in_pos", _P), ("in_hidden", _P),
                ("hid_offsets", _P), ("hid_pos", _P), ("hid_output", _P)]


class Param(ctypes.Structure):
    _fields_ = [("value", _P), ("grad", _P), ("m", _P), ("v", _P), ("count", _I64)]


class TrainParams(ctypes.Structure):
    _fields_ = [("up_val", Param), ("b_up", Param), ("out_val", Param), ("b_down", Param)]


class Dense(ctypes.Structure):
    _fields_ = [("up_hi", _P), ("up_lo", _P), ("down_hi", _P), ("down_lo", _P)]


class DenseF16x3(ctypes.Structure):
    _fields_ = [("up_hi", _P), ("up_lo", _P), ("up_scale", _P), ("down_hi", _P), ("down_lo", _P), ("down_scale", _P),
                ("up_bound", _P)]


class AdamWStep(ctypes.Structure):
    _fields_ = [(name, ctypes.c_float) for name in
                ("lr_decay", "beta1", "one_minus_beta1", "beta2", "one_minus_beta2", "step_size", "bias2_sqrt", "eps")]


# name: (restype, argtypes) of every entry declared in include/hffn_b200.h
SIGNATURES = {
    "hffn_version": (ctypes.c_char_p, []),
    "hffn_last_error": (ctypes.c_char_p, []),
    "hffn_up_mode": (ctypes.c_int, [_I64, _I32]),
    "hffn_down_mode": (ctypes.c_int, [_I64, _I32]),
    "hffn_up": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I64, _P]),
    "hffn_down": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, _P, _P, _P, _P, _P, _P, _I32, _I32, _I64, _P]),
    "hffn_forward": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(Layer), _P, _P, _P, _P, _I64, ctypes.c_int,
                                    ctypes.c_int, _P]),
    "hffn_backward_workspace": (_I64, [ctypes.POINTER(Layer), _I64]),
    "hffn_backward": (ctypes.c_int, [ctypes.POINTER(Layer), ctypes.POINTER(Supports), _P, _P, _P, _P, _P, _P,
                                     ctypes.POINTER(TrainParams), ctypes.POINTER(AdamWStep), _P, _I64, _P]),
    "hffn_adamw": (ctypes.c_int, [ctypes.POINTER(Param), ctypes.POINTER(AdamWStep), _P]),
    "hffn_mse": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I32, _P, _P]),
    "hffn_validate_layout": (ctypes.c_int, [ctypes.POINTER(Layer), _P, _P]),
    "hffn_decode_error": (ctypes.c_int, [ctypes.POINTER(_I32), ctypes.c_int]),
    "hffn_build_layout_workspace": (_I64, [_I32, _I32, _I64, _I64]),
    "hffn_build_out_major": (ctypes.c_int, [ctypes.c_int, _I32, _I32, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _P]),
    "hffn_build_supports": (ctypes.c_int, [_I32, _I32, _P, _P, _I64, _P, _P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "hffn_densify": (ctypes.c_int, [ctypes.c_int, _P, _P, _P, _I32, _I32, _P, _P, _P]),
    "hffn_up_tc": (ctypes.c_int, [ctypes.c_int, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I64, _P]),
    "hffn_down_tc": (ctypes.c_int, [ctypes.c_int, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I64, _P]),
    "hffn_set_tc_max_ctas": (ctypes.c_int, [_I32]),
    "hffn_set_tc_tile_tokens": (ctypes.c_int, [_I32]),
    "hffn_down_tc_peer": (ctypes.c_int, [ctypes.c_int, _P, _P, _P, _P, _P, ctypes.POINTER(ctypes.c_uint64), _I32, _I64,
                                         _P, _I32, _I32, _I64, _P]),
    "hffn_sum_slots": (ctypes.c_int, [ctypes.c_int, _P, _I32, _I64, _P, _P]),
    "hffn_peer_pipeline_create": (ctypes.c_int, [ctypes.POINTER(PeerConfig), ctypes.POINTER(Layer),
                                                  ctypes.POINTER(Dense), _P, ctypes.POINTER(_P)]),
    "hffn_peer_pipeline_run": (ctypes.c_int, [_P, ctypes.POINTER(_P), ctypes.POINTER(_P), _I32, _P]),
    "hffn_peer_pipeline_destroy": (ctypes.c_int, [_P]),
    "hffn_peer_barrier": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_uint64), _I32, _I32, ctypes.c_uint32, _I64, _P,
                                         _P]),
    "hffn_gemm_tc_f32": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I64,
                                        _P, _P]),
    "hffn_train_step_tc_workspace": (_I64, [ctypes.POINTER(Layer), _I64]),
    "hffn_train_step_tc": (ctypes.c_int, [ctypes.POINTER(Layer), ctypes.POINTER(Dense), ctypes.POINTER(DenseF16x3), _P,
                                          _P, _P, _P,
                                          ctypes.POINTER(TrainParams), ctypes.POINTER(AdamWStep), _P, _P, _P, _I64,
                                          _I64, _P]),
    "hffn_forward_noalloc_max_bytes": (_I64, []),
    "hffn_forward_noalloc": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(Layer), _P, _P, _I64, _P]),
    "hffn_densify_f16x3": (ctypes.c_int, [_P, _P, _P, _P, _I32, _I32, _P, _P, _P, _P, _P]),
    "hffn_forward_f16x3_workspace": (_I64, [ctypes.POINTER(Layer), _I64]),
    "hffn_forward_f16x3": (ctypes.c_int, [ctypes.POINTER(Layer), ctypes.POINTER(DenseF16x3), _P, _P, _P, _P, _P, _I64,
                                          _P]),
    "hffn_f16x3_packet_bytes": (_I64, [_I32]),
    "hffn_split_f16x3": (ctypes.c_int, [_P, ctypes.POINTER(DenseF16x3), _P, _I32, _I32, _I64, _P]),
    "hffn_forward_f16x3_packets": (ctypes.c_int, [ctypes.POINTER(Layer), ctypes.POINTER(DenseF16x3), _P, _P, _P, _P,
                                                  _P, _I64, _P]),
    "hffn_up_f16x3": (ctypes.c_int, [_P, ctypes.POINTER(DenseF16x3), _P, _P, _P, _P, _I32, _I32, _I64, _P]),
    "hffn_down_f16x3": (ctypes.c_int, [_P, ctypes.POINTER(DenseF16x3), _P, _P, _P, _I32, _I32, _I64, _P]),
    "hffn_forward_tc_workspace": (_I64, [ctypes.c_int, ctypes.POINTER(Layer), _I64]),
    "hffn_forward_tc": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(Layer), ctypes.POINTER(Dense), _P, _P, _P, _P, _P,
                                       _I64, _P]),
}


class NativeError(RuntimeError):
    pass


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -c 'import hffn_b200.build as b; b.build()'` "
                          "(nvcc, sm_100a); the HFFN path has no CPU or library fallback")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        function = getattr(lib, name)
        function.restype, function.argtypes = restype, argtypes
    return lib


lib = _load()


def check(status: int, what: str) -> None:
    """Raise on a non-zero status: ValueError for argument errors (as the reference runtime), else NativeError."""
    if status == HFFN_OK:
        return
    message = f"{what}: {lib.hffn_last_error().decode()}"
    if status == HFFN_ERR_ARGUMENT:
        raise ValueError(message)
    raise NativeError(message)


def stream_handle(device) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream
