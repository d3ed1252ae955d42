"""ctypes binding to ``oracle/_ref/librpfq_ref.so`` (TEST INFRASTRUCTURE ONLY).

The library is the reference's own C++ CPU runtime for the packed
phase-linear layer (RPFQ-ViTAndroid/app/src/main/cpp/ops/phase_linear.cpp and
kernels/*.cpp), compiled from its sources by ``oracle/Makefile`` with the shim
``oracle/ref_shim.cpp``. Used by the tests as a second oracle and by
``bench.py`` as the "reference" CPU baseline. Returns ``None`` from
:func:`load` when the library has not been built.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

from .packed_ref import PLANE_NAMES

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "librpfq_ref.so")
_lib = None


def load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        return None
    lib = ctypes.CDLL(LIB_PATH)
    P = ctypes.c_void_p
    I = ctypes.c_int
    lib.rpfq_ref_last_error.restype = ctypes.c_char_p
    lib.rpfq_ref_wide_linear.argtypes = [P, I, I, I, I, I, P, P, P, P, I, I, P]
    lib.rpfq_ref_wide_linear.restype = I
    lib.rpfq_ref_coefficient_planes.argtypes = [I, I, I, I, P, P, P, P, P, P, P]
    lib.rpfq_ref_coefficient_planes.restype = I
    lib.rpfq_ref_prepare.argtypes = [I, I, I, I, P, P, P, P]
    lib.rpfq_ref_prepare.restype = P
    lib.rpfq_ref_run_prepared.argtypes = [P, P, I, I, P]
    lib.rpfq_ref_run_prepared.restype = I
    lib.rpfq_ref_release.argtypes = [P]
    _lib = lib
    return lib


class _Planes:
    """Keeps contiguous copies alive and exposes pointer arrays for the C ABI."""

    def __init__(self, packed: dict):
        self.codes = [np.ascontiguousarray(packed[f"{p}.codes"]) for p in PLANE_NAMES]
        self.g_re = [np.ascontiguousarray(packed[f"{p}.gamma_real"]).view(np.uint16) for p in PLANE_NAMES]
        self.g_im = [np.ascontiguousarray(packed[f"{p}.gamma_imag"]).view(np.uint16) for p in PLANE_NAMES]
        self.bias = np.ascontiguousarray(packed["bias"]).view(np.uint16)
        arr = ctypes.c_void_p * 4
        self.p_codes = arr(*[a.ctypes.data for a in self.codes])
        self.p_re = arr(*[a.ctypes.data for a in self.g_re])
        self.p_im = arr(*[a.ctypes.data for a in self.g_im])
        self.n_cp = self.codes[0].shape[0]
        self.k_cp = self.codes[0].shape[1] * 4


def _check(lib, rc):
    if rc != 0:
        raise RuntimeError(lib.rpfq_ref_last_error().decode())


def wide_linear(packed: dict, x: np.ndarray, n_c: int, k_c: int, mode: int = 0, threads: int = 1):
    """Run the reference C++ layer forward. mode 0 = wideLinearReference,
    1 = wideLinearOptimized, 2 = fp16 coefficient cache."""
    lib = load()
    pl = _Planes(packed)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty((x.shape[0], 2 * n_c), np.float32)
    _check(lib, lib.rpfq_ref_wide_linear(x.ctypes.data, x.shape[0], n_c, k_c, pl.n_cp, pl.k_cp,
                                         pl.p_codes, pl.p_re, pl.p_im, pl.bias.ctypes.data,
                                         mode, threads, y.ctypes.data))
    return y


def coefficient_planes(packed: dict, n_c: int, k_c: int) -> dict[str, np.ndarray]:
    """fp16 planes from the reference's buildFusedWideLinearCache."""
    lib = load()
    pl = _Planes(packed)
    out = {k: np.empty((n_c, k_c), np.uint16) for k in ("rr", "ir", "ri", "ii")}
    _check(lib, lib.rpfq_ref_coefficient_planes(n_c, k_c, pl.n_cp, pl.k_cp, pl.p_codes, pl.p_re, pl.p_im,
                                                out["rr"].ctypes.data, out["ir"].ctypes.data,
                                                out["ri"].ctypes.data, out["ii"].ctypes.data))
    return {k: v.view(np.float16) for k, v in out.items()}


class PreparedLayer:
    """A layer with its fp16 cache built once; :meth:`run` times only the GEMM."""

    def __init__(self, packed: dict, n_c: int, k_c: int):
        self.lib = load()
        pl = _Planes(packed)
        self.n_c, self.k_c = n_c, k_c
        self.handle = self.lib.rpfq_ref_prepare(n_c, k_c, pl.n_cp, pl.k_cp, pl.p_codes, pl.p_re, pl.p_im,
                                                pl.bias.ctypes.data)
        if not self.handle:
            raise RuntimeError(self.lib.rpfq_ref_last_error().decode())

    def run(self, x: np.ndarray, threads: int) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty((x.shape[0], 2 * self.n_c), np.float32)
        _check(self.lib, self.lib.rpfq_ref_run_prepared(self.handle, x.ctypes.data, x.shape[0], threads,
                                                        y.ctypes.data))
        return y

    def __del__(self):
        if getattr(self, "handle", None):
            self.lib.rpfq_ref_release(self.handle)
            self.handle = None
