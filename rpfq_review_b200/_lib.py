"""ctypes binding of ``librpfq_b200.so`` (the C ABI in ``include/rpfq_b200.h``).

The library is built in-tree by :func:`rpfq_review_b200.build.build` with nvcc
for sm_100a. There is no fallback: if the library is missing, :func:`lib`
raises ``RuntimeError`` telling how to build it.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librpfq_b200.so")

RPFQ_OK = 0
RPFQ_ERR_INVALID = 1
RPFQ_ERR_UNSUPPORTED = 2
RPFQ_ERR_CUDA = 3
RPFQ_ERR_DEVICE = 4

ACT_NONE = 0
ACT_GELU = 1
GEMM_OUT_F32 = 1
GEMM_RESIDUAL_F32 = 2
GEMM_BIAS_F32 = 4
ROUND_NEAREST_EVEN = 0
ROUND_TIES_AWAY = 1

# Every symbol include/rpfq_b200.h declares; tests check the library exports them.
EXPORTED_SYMBOLS = (
    "rpfq_prepack_sm100",
    "rpfq_gemm_sm100",
    "rpfq_gemm_workspace_bytes",
    "rpfq_gemm_plan_sm100",
    "rpfq_act_quant_sm100",
    "rpfq_patch_unfold_sm100",
    "rpfq_layernorm_sm100",
    "rpfq_layernorm_rows_sm100",
    "rpfq_layernorm_ex_sm100",
    "rpfq_wide_linear_sm100",
    "rpfq_wide_linear_noalloc_sm100",
    "rpfq_attention_sm100",
    "rpfq_window_attention_sm100",
    "rpfq_vision_workspace_bytes",
    "rpfq_vision_act_quant_sm100",
    "rpfq_pack_workspace_bytes",
    "rpfq_pack_linear_sm100",
    "rpfq_last_error",
    "rpfq_device_error",
    "rpfq_version",
)


class RpfqGemmPlan(ctypes.Structure):
    _fields_ = [("block_n", ctypes.c_int32), ("cta_pair", ctypes.c_int32), ("split_k", ctypes.c_int32),
                ("stream_k_tiles", ctypes.c_int32), ("units", ctypes.c_int32), ("tiles", ctypes.c_int32),
                ("tail_tiles", ctypes.c_int32), ("pieces", ctypes.c_int32)]


class RpfqPhasePlane(ctypes.Structure):
    _fields_ = [("codes", ctypes.c_void_p), ("gamma_real", ctypes.c_void_p), ("gamma_imag", ctypes.c_void_p)]


class RpfqPhasePlaneOut(ctypes.Structure):
    _fields_ = [("codes", ctypes.c_void_p), ("gamma_real", ctypes.c_void_p), ("gamma_imag", ctypes.c_void_p)]


class RpfqPackedLinear(ctypes.Structure):
    _fields_ = [
        ("n_c", ctypes.c_int32), ("k_c", ctypes.c_int32),
        ("n_cp", ctypes.c_int32), ("k_cp", ctypes.c_int32),
        ("stages", ctypes.c_int32), ("code_bits", ctypes.c_int32),
        ("u", RpfqPhasePlane * 4), ("w", RpfqPhasePlane * 4),
    ]


class RpfqGemmArgs(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64),
        ("w", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("residual", ctypes.c_void_p), ("ldr", ctypes.c_int64),
        ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64),
        ("m", ctypes.c_int64), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
        ("activation", ctypes.c_int32), ("block_n", ctypes.c_int32),
        ("flags", ctypes.c_int32), ("cta_pair", ctypes.c_int32),
        ("split_k", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64),
    ]


class RpfqLayerNormArgs(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64), ("x_rows", ctypes.c_int64),
        ("rows", ctypes.c_void_p),
        ("add", ctypes.c_void_p), ("ld_add", ctypes.c_int64), ("add_bound", ctypes.c_int64),
        ("add_rows", ctypes.c_void_p),
        ("weight", ctypes.c_void_p), ("bias", ctypes.c_void_p),
        ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64),
        ("y32", ctypes.c_void_p), ("ldy32", ctypes.c_int64),
        ("m", ctypes.c_int64), ("d", ctypes.c_int32), ("eps", ctypes.c_float),
        ("act_bits", ctypes.c_int32), ("merge_side", ctypes.c_int32),
        ("y32_prenorm", ctypes.c_int32), ("reserved", ctypes.c_int32),
    ]


class RpfqWideLinearArgs(ctypes.Structure):
    _fields_ = [
        ("layer", ctypes.POINTER(RpfqPackedLinear)),
        ("dense", ctypes.c_void_p),
        ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64),
        ("bias", ctypes.c_void_p),
        ("residual", ctypes.c_void_p), ("ldr", ctypes.c_int64),
        ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64),
        ("m", ctypes.c_int64),
        ("act_bits", ctypes.c_int32), ("activation", ctypes.c_int32),
        ("scratch", ctypes.c_void_p),
        ("flags", ctypes.c_int32), ("split_k", ctypes.c_int32),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64),
    ]


_lock = threading.Lock()
_lib = None


def lib() -> ctypes.CDLL:
    """Load the CUDA library (once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "or `python -m rpfq_review_b200.build` (nvcc, sm_100a). There is no CPU fallback.")
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        I32 = ctypes.c_int32
        I64 = ctypes.c_int64
        L.rpfq_prepack_sm100.argtypes = [ctypes.POINTER(RpfqPackedLinear), P, I32, P]
        L.rpfq_gemm_sm100.argtypes = [ctypes.POINTER(RpfqGemmArgs), P]
        L.rpfq_gemm_workspace_bytes.argtypes = [I64, I32, I32]
        L.rpfq_gemm_workspace_bytes.restype = ctypes.c_uint64
        L.rpfq_gemm_plan_sm100.argtypes = [ctypes.POINTER(RpfqGemmArgs), ctypes.POINTER(RpfqGemmPlan)]
        L.rpfq_act_quant_sm100.argtypes = [P, I64, P, I64, I64, I32, I32, P]
        L.rpfq_patch_unfold_sm100.argtypes = [P, I32, I64, I32, I32, I32, I32, P, I64, P]
        L.rpfq_layernorm_sm100.argtypes = [P, I64, P, P, P, I64, I64, I32, ctypes.c_float, I32, P]
        L.rpfq_layernorm_rows_sm100.argtypes = [P, I64, I64, P, P, P, P, I64, I64, I32, ctypes.c_float, I32, P]
        L.rpfq_layernorm_ex_sm100.argtypes = [ctypes.POINTER(RpfqLayerNormArgs), P]
        L.rpfq_wide_linear_sm100.argtypes = [ctypes.POINTER(RpfqWideLinearArgs), P]
        L.rpfq_wide_linear_noalloc_sm100.argtypes = [ctypes.POINTER(RpfqWideLinearArgs), P]
        L.rpfq_attention_sm100.argtypes = [P, I64, I32, I32, I32, P, I64, P]
        L.rpfq_window_attention_sm100.argtypes = [P, I64, I32, I32, I32, P, I32, P, I64, P]
        L.rpfq_vision_workspace_bytes.argtypes = [I64, I32]
        L.rpfq_vision_workspace_bytes.restype = ctypes.c_uint64
        L.rpfq_vision_act_quant_sm100.argtypes = [P, I64, P, I64, I64, I32, I32, ctypes.c_double, ctypes.c_double,
                                                  ctypes.c_double, I32, P, P, ctypes.c_uint64, P]
        L.rpfq_pack_workspace_bytes.argtypes = [I32, I32]
        L.rpfq_pack_workspace_bytes.restype = ctypes.c_uint64
        L.rpfq_pack_linear_sm100.argtypes = [P, I64, I32, I32, I32, ctypes.POINTER(RpfqPhasePlaneOut),
                                             ctypes.POINTER(RpfqPhasePlaneOut), P, ctypes.c_uint64, P]
        L.rpfq_last_error.restype = ctypes.c_char_p
        L.rpfq_device_error.argtypes = [ctypes.POINTER(I32)]
        for name in ("rpfq_prepack_sm100", "rpfq_gemm_sm100", "rpfq_gemm_plan_sm100", "rpfq_act_quant_sm100",
                     "rpfq_layernorm_sm100",
                     "rpfq_layernorm_rows_sm100", "rpfq_layernorm_ex_sm100",
                     "rpfq_wide_linear_sm100", "rpfq_wide_linear_noalloc_sm100", "rpfq_pack_linear_sm100",
                     "rpfq_vision_act_quant_sm100", "rpfq_attention_sm100", "rpfq_window_attention_sm100",
                     "rpfq_device_error",
                     "rpfq_version"):
            getattr(L, name).restype = ctypes.c_int
        _lib = L
        return L


def check(rc: int, what: str) -> None:
    """Turn a nonzero status into an exception with the library's message."""
    if rc == RPFQ_OK:
        return
    msg = lib().rpfq_last_error().decode(errors="replace")
    if rc == RPFQ_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    if rc == RPFQ_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg} (status {rc})")


def device_error() -> int:
    """Read and clear the device-side error word (synchronises the device)."""
    code = ctypes.c_int32(0)
    check(lib().rpfq_device_error(ctypes.byref(code)), "rpfq_device_error")
    return int(code.value)
