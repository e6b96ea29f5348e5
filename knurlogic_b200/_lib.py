"""ctypes binding of libvqmoe.so (the C ABI in include/vqmoe.h).

The library is the only compute path: there is no CPU or PyTorch fallback.
`lib()` raises if the shared object is missing or cannot be loaded, and the
modules refuse to run on anything but a CUDA tensor.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import (POINTER, Structure, c_char_p, c_float, c_int32, c_int64, c_size_t,
                    c_uint32, c_uint8, c_void_p)
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libvqmoe.so"

FMT_DENSE_BF16 = 0
FMT_VQ_U8 = 1
FMT_VQ_REF = 2          # reference-layout codes (uint8 / uint16), dim 2, 4 or 8
FMT_AFFINE = 3          # affine-quantized (QuantizedSwitchLinear): packed q, scales, biases
OUT_BF16 = 0
OUT_F32 = 1
ACT_SWIGLU = 0          # vqmoe_linear.activation of a SwitchGLU's gate linear
ACT_GEGLU = 1
ROUTER_SOFTMAX_TOPK_RENORM = 0   # Qwen3.5 (qwen3_5.py:174-179)
ROUTER_TOPK_SOFTMAX = 1          # Qwen4-exp, norm_topk_prob (qwen4_exp.py:806-810)
ROUTER_SOFTMAX_TOPK = 2          # Qwen4-exp, not renormalised (qwen4_exp.py:811-814)

STATUS = {0: "OK", 1: "BAD_SHAPE", 2: "BAD_FORMAT", 3: "BAD_POINTER",
          4: "WORKSPACE_TOO_SMALL", 5: "BAD_CODE", 6: "LAUNCH_FAILED",
          7: "TIMEOUT", 8: "NOT_SUPPORTED"}


class Linear(Structure):
    """vqmoe_linear"""
    _fields_ = [("format", c_int32), ("num_experts", c_int32),
                ("out_features", c_int32), ("in_features", c_int32),
                ("weight", c_void_p), ("codes", c_void_p),
                ("codebook", c_void_p), ("scales", c_void_p),
                ("codebook_size", c_int32), ("dim", c_int32),
                ("group_size", c_int32), ("activation", c_int32),
                ("biases", c_void_p), ("bits", c_int32), ("reserved", c_int32)]


class Tp(Structure):
    """vqmoe_tp"""
    _fields_ = [("rank", c_int32), ("world", c_int32), ("buffers", c_void_p * 8),
                ("buffer_bytes", c_int64), ("wait_polls", c_int32), ("reserved", c_int32)]


class Block(Structure):
    """vqmoe_block"""
    _fields_ = [("hidden", c_int32), ("num_experts", c_int32),
                ("top_k", c_int32), ("shared_inter", c_int32),
                ("router_w", c_void_p), ("gate", Linear), ("up", Linear),
                ("down", Linear), ("shared_gate_w", c_void_p),
                ("shared_up_w", c_void_p), ("shared_down_w", c_void_p),
                ("shared_expert_gate_w", c_void_p),
                ("router_mode", c_int32), ("wait_polls", c_int32)]


#: every symbol include/vqmoe.h declares: (name, restype, argtypes)
SIGNATURES = [
    ("vqmoe_abi_version", c_int32, []),
    ("vqmoe_workspace_status", c_int32, [c_void_p, c_void_p]),
    ("vqmoe_tp_buffer_bytes", c_size_t, [c_int32, c_int32]),
    ("vqmoe_sparse_moe_block_tp", c_int32,
     [POINTER(Block), POINTER(Tp), c_void_p, c_int32, c_void_p, c_void_p, c_size_t, c_void_p]),
    ("vqmoe_ep_buffer_bytes", c_size_t, [c_int32, c_int32, c_int32]),
    ("vqmoe_sparse_moe_block_ep", c_int32,
     [POINTER(Block), POINTER(Tp), c_void_p, c_int32, c_void_p, c_void_p, c_size_t, c_void_p]),
    ("vqmoe_sparse_moe_block_tp_timed", c_int32,
     [POINTER(Block), POINTER(Tp), c_void_p, c_int32, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p, c_int32]),
    ("vqmoe_last_error", c_char_p, []),
    ("vqmoe_block_workspace_size", c_size_t, [POINTER(Block), c_int32]),
    ("vqmoe_switch_glu_workspace_size", c_size_t,
     [POINTER(Linear), POINTER(Linear), c_int32, c_int32]),
    ("vqmoe_switch_linear_workspace_size", c_size_t,
     [POINTER(Linear), c_int32, c_int32, c_int32]),
    ("vqmoe_router_workspace_size", c_size_t, [c_int32, c_int32]),
    ("vqmoe_sparse_moe_block", c_int32,
     [POINTER(Block), c_void_p, c_int32, c_void_p, c_int32, c_void_p,
      c_size_t, c_void_p]),
    ("vqmoe_sparse_moe_block_timed", c_int32,
     [POINTER(Block), c_void_p, c_int32, c_void_p, c_int32, c_void_p,
      c_size_t, c_void_p, POINTER(c_void_p), c_int32]),
    ("vqmoe_switch_glu", c_int32,
     [POINTER(Linear), POINTER(Linear), POINTER(Linear), c_void_p, c_void_p,
      c_int32, c_int32, c_void_p, c_void_p, c_size_t, c_void_p]),
    ("vqmoe_switch_glu_noalloc", c_int32,
     [POINTER(Linear), POINTER(Linear), POINTER(Linear), c_void_p, c_void_p,
      c_int32, c_int32, c_void_p, c_void_p]),
    ("vqmoe_switch_linear", c_int32,
     [POINTER(Linear), c_void_p, c_int32, c_void_p, c_int32, c_int32,
      c_void_p, c_void_p, c_size_t, c_void_p]),
    ("vqmoe_router", c_int32,
     [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
      c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    ("vqmoe_router_ex", c_int32,
     [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32,
      c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    ("vqmoe_rms_norm", c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_float, c_void_p, c_void_p]),
    ("vqmoe_add_rms_norm", c_int32,
     [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_float, c_void_p, c_void_p, c_void_p]),
    ("vqmoe_moe_experts_workspace_size", c_size_t, [POINTER(Linear), POINTER(Linear), c_int32, c_int32]),
    ("vqmoe_moe_experts", c_int32,
     [POINTER(Linear), POINTER(Linear), POINTER(Linear), c_void_p, c_void_p, c_void_p, c_int32, c_int32,
      c_void_p, c_void_p, c_size_t, c_void_p]),
    ("vqmoe_dequant", c_int32,
     [POINTER(Linear), c_int32, c_int32, c_void_p, c_void_p]),
    ("vqmoe_vq_layout_bytes", c_int32,
     [c_int32, c_int32, c_int32, POINTER(c_int64), POINTER(c_int64)]),
    ("vqmoe_prepare_vq", c_int32,
     [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p]),
    ("vqmoe_count_bad_codes", c_int32,
     [c_void_p, c_int64, c_int32, c_void_p, c_void_p]),
    ("vqmoe_count_bad_codes_u16", c_int32,
     [c_void_p, c_int64, c_int32, c_void_p, c_void_p]),
    ("vqmoe_unprepare_codes", c_int32,
     [c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p]),
]

_lock = threading.Lock()
_lib = None


class VQMoEError(RuntimeError):
    """A non-OK vqmoe_status, with the library's message."""

    def __init__(self, func: str, status: int, msg: str):
        super().__init__(f"{func}: {STATUS.get(status, status)}: {msg}")
        self.status = status


def lib():
    """The loaded library (loads once). Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with "
                    "`python -m knurlogic_b200.build` (nvcc, sm_100a)")
            h = ctypes.CDLL(str(LIB_PATH))
            for name, res, args in SIGNATURES:
                f = getattr(h, name)
                f.restype = res
                f.argtypes = args
            _lib = h
    return _lib


def vq_layout_bytes(E: int, OUT: int, IN: int):
    """(code bytes, scale bytes) of the device layout of one VQ linear."""
    cb, sb = c_int64(), c_int64()
    call("vqmoe_vq_layout_bytes", E, OUT, IN, ctypes.byref(cb), ctypes.byref(sb))
    return cb.value, sb.value


def call(name: str, *args) -> None:
    """Call a status-returning entry point; raise VQMoEError unless OK."""
    h = lib()
    st = getattr(h, name)(*args)
    if st != 0:
        raise VQMoEError(name, st, (h.vqmoe_last_error() or b"").decode())
