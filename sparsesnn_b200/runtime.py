"""ctypes binding of libsnnb200.so (C ABI declared in include/snn_b200.h).

This is the only place Python touches the native library.  If the library
is missing, ``load()`` raises: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libsnnb200.so"

SNN_OK = 0
SNN_E_INVALID = -1
SNN_E_NOT_24 = -2
SNN_E_CUDA = -3
SNN_E_NO_DEVICE = -4
SNN_E_DEVICE = -5

SNN_NEURON_LIF = 0
SNN_NEURON_IF = 1
SNN_NEURON_NONE = 2
SNN_NEURON_NONE_F16 = 3
SNN_FLAG_READ_STATE = 1
SNN_FLAG_WRITE_STATE = 2
SNN_FLAG_FORCE_GENERIC = 4
SNN_FLAG_CTA_PAIR = 8
SNN_FLAG_DENSE = 16
SNN_FLAG_QKV_PACKED = 32
SNN_FLAG_SPIKE_BITS = 64
SNN_VARIANT_GENERIC = 0
SNN_VARIANT_HALO_RESIDENT = 1
SNN_VARIANT_HALO_STREAM = 2
SNN_RES_ADD_AFTER = 0
SNN_RES_ADD_BEFORE = 1
SNN_RES_TWO_NEURON = 2

NEURONS = {"lif": SNN_NEURON_LIF, "if": SNN_NEURON_IF, "none": SNN_NEURON_NONE,
           "none_f16": SNN_NEURON_NONE_F16}

# Every symbol include/snn_b200.h declares.
EXPORTED = (
    "snn_abi_version", "snn_init", "snn_conv_variant", "snn_conv_out_shape", "snn_conv_weight_bytes",
    "snn_pack_weight_24", "snn_conv_forward", "snn_conv_forward_res", "snn_conv_forward_res2",
    "snn_stem_forward", "snn_stem_forward_dual", "snn_spikformer_attn_forward", "snn_add_lif_forward",
    "snn_maxpool_lif_forward", "snn_lif_forward", "snn_conv_tsplit_workspace_bytes",
    "snn_conv_forward_tsplit", "snn_conv_forward_tsplit_static",
    "snn_head_forward", "snn_get_device_error", "snn_last_error_message",
    "snn_engine_check_file", "snn_engine_load", "snn_engine_io", "snn_engine_capture",
    "snn_engine_run", "snn_engine_destroy",
)


class SnnConvDesc(ctypes.Structure):
    _fields_ = [
        ("T", ctypes.c_int32), ("B", ctypes.c_int32), ("Cin", ctypes.c_int32),
        ("H", ctypes.c_int32), ("W", ctypes.c_int32), ("Cout", ctypes.c_int32),
        ("KH", ctypes.c_int32), ("KW", ctypes.c_int32), ("stride", ctypes.c_int32),
        ("pad", ctypes.c_int32), ("neuron", ctypes.c_int32), ("flags", ctypes.c_int32),
        ("tau", ctypes.c_float), ("v_threshold", ctypes.c_float), ("v_reset", ctypes.c_float),
        ("res_mode", ctypes.c_int32), ("neuron2", ctypes.c_int32),
        ("tau2", ctypes.c_float), ("v_threshold2", ctypes.c_float), ("v_reset2", ctypes.c_float),
    ]


class SnnError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"libsnnb200 error {code}: {message}")
        self.code = code


_lib = None
_lock = threading.Lock()


def _declare(lib):
    P = ctypes.c_void_p
    D = ctypes.POINTER(SnnConvDesc)
    i32 = ctypes.c_int32
    sig = {
        "snn_abi_version": ([], ctypes.c_int),
        "snn_init": ([], ctypes.c_int),
        "snn_conv_variant": ([D], ctypes.c_int),
        "snn_conv_out_shape": ([D, ctypes.POINTER(i32), ctypes.POINTER(i32)], ctypes.c_int),
        "snn_conv_weight_bytes": ([D, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
        "snn_pack_weight_24": ([D, P, P], ctypes.c_int),
        "snn_conv_forward": ([D, P, P, P, P, P, P, P], ctypes.c_int),
        "snn_conv_forward_res": ([D, P, P, P, P, P, P, P, P], ctypes.c_int),
        "snn_conv_forward_res2": ([D, P, P, P, P, P, P, P, P, P], ctypes.c_int),
        "snn_stem_forward": ([D, i32, P, P, P, P, P, P], ctypes.c_int),
        "snn_stem_forward_dual": ([D, i32, P, P, P, P, P, P, P], ctypes.c_int),
        "snn_head_forward": ([i32, i32, i32, i32, i32, P, P, P, P, P], ctypes.c_int),
        "snn_add_lif_forward": ([D, P, P, P, P, P], ctypes.c_int),
        "snn_maxpool_lif_forward": ([D, P, P, P, P], ctypes.c_int),
        "snn_lif_forward": ([D, P, P, P, P], ctypes.c_int),
        "snn_conv_tsplit_workspace_bytes": ([D, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
        "snn_conv_forward_tsplit": ([D, P, P, P, P, P, P, P, P, ctypes.c_size_t, P], ctypes.c_int),
        "snn_conv_forward_tsplit_static": ([D, P, P, P, P, P, P, P, P], ctypes.c_int),
        "snn_spikformer_attn_forward": ([i32, i32, i32, i32, i32, ctypes.c_float, ctypes.c_float,
                                         ctypes.c_float, ctypes.c_float, i32, P, P, P, P, P, P],
                                        ctypes.c_int),
        "snn_get_device_error": ([ctypes.POINTER(ctypes.c_uint32), ctypes.c_int], ctypes.c_int),
        "snn_last_error_message": ([], ctypes.c_char_p),
        "snn_engine_check_file": ([ctypes.c_char_p, ctypes.POINTER(i32), ctypes.POINTER(i32)],
                                  ctypes.c_int),
        "snn_engine_load": ([ctypes.c_char_p, ctypes.POINTER(P)], ctypes.c_int),
        "snn_engine_io": ([P, ctypes.POINTER(i32), ctypes.POINTER(i32), ctypes.POINTER(ctypes.c_size_t),
                           ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
        "snn_engine_capture": ([P, P], ctypes.c_int),
        "snn_engine_run": ([P, P, P, P], ctypes.c_int),
        "snn_engine_destroy": ([P], None),
    }
    for name, (args, res) in sig.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = res


def load(path: str | Path | None = None):
    """Load (once) and return the library handle.  Raises if it is absent."""
    global _lib
    with _lock:
        if _lib is None:
            p = Path(path) if path else LIB_PATH
            if not p.exists():
                raise RuntimeError(
                    f"{p} is missing: build it with `python -m sparsesnn_b200.build` "
                    "(there is no CPU or eager fallback)")
            lib = ctypes.CDLL(str(p))
            _declare(lib)
            _lib = lib
        return _lib


def check(rc: int) -> None:
    if rc != SNN_OK:
        msg = load().snn_last_error_message()
        raise SnnError(rc, msg.decode() if msg else "")


RES_MODES = {"add_after": SNN_RES_ADD_AFTER, "add_before": SNN_RES_ADD_BEFORE,
             "two_neuron": SNN_RES_TWO_NEURON}


def make_desc(*, T, B, Cin, H, W, Cout, KH, KW, stride=1, pad=None, neuron="lif",
              flags=0, tau=2.0, v_threshold=1.0, v_reset=0.0, res_mode="add_after",
              neuron2="lif", tau2=2.0, v_threshold2=1.0, v_reset2=0.0) -> SnnConvDesc:
    if pad is None:
        pad = KH // 2
    return SnnConvDesc(T, B, Cin, H, W, Cout, KH, KW, stride, pad, NEURONS[neuron], flags,
                       tau, v_threshold, v_reset, RES_MODES[res_mode], NEURONS[neuron2],
                       tau2, v_threshold2, v_reset2)


def variant(desc: SnnConvDesc) -> int:
    """Kernel variant the library picks for ``desc`` (SNN_VARIANT_*)."""
    v = load().snn_conv_variant(ctypes.byref(desc))
    if v < 0:
        check(v)
    return v


def out_shape(desc: SnnConvDesc):
    oh, ow = ctypes.c_int32(), ctypes.c_int32()
    check(load().snn_conv_out_shape(ctypes.byref(desc), ctypes.byref(oh), ctypes.byref(ow)))
    return oh.value, ow.value


def weight_bytes(desc: SnnConvDesc) -> int:
    n = ctypes.c_size_t()
    check(load().snn_conv_weight_bytes(ctypes.byref(desc), ctypes.byref(n)))
    return n.value


def pack_weight_24(desc: SnnConvDesc, w_fchw):
    """Pack a pruned fp32 ``[Cout, Cin, KH, KW]`` numpy array; returns uint8 numpy blob."""
    import numpy as np
    w = np.ascontiguousarray(w_fchw, dtype=np.float32)
    if w.shape != (desc.Cout, desc.Cin, desc.KH, desc.KW):
        raise ValueError(f"weight shape {w.shape} does not match descriptor")
    blob = np.zeros(weight_bytes(desc), np.uint8)
    check(load().snn_pack_weight_24(ctypes.byref(desc), w.ctypes.data, blob.ctypes.data))
    return blob


def device_error(reset: bool = True) -> int:
    code = ctypes.c_uint32()
    check(load().snn_get_device_error(ctypes.byref(code), 1 if reset else 0))
    return code.value
