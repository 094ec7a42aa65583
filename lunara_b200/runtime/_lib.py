"""ctypes binding of the sm_100a kernel library (``include/lunara_b200.h``).

This is the binding a reference-side runtime would add: plain pointers, sizes
and a ``cudaStream_t``; no torch types cross the boundary. The library is the
in-tree ``lunara_b200/liblunara_b200.so`` built by ``lunara_b200.build``.
Loading fails loudly when it is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent.parent / "liblunara_b200.so"

# lunara_status
OK, ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_LAUNCH, ERR_DEVICE = range(5)
# lunara_dtype
F16, BF16, F32 = 0, 1, 2
# lunara_activation
ACT_NONE, ACT_RELU, ACT_GELU_ERF, ACT_GELU_TANH, ACT_SIGMOID, ACT_TANH = range(6)
# lunara_binary_op
BIN_ADD, BIN_MUL = 0, 1
# lunara_b_layout
B_KN, B_NK = 0, 1

# Every exported symbol with its ctypes signature; the header declares exactly these.
_p, _i, _i64, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
_pi64 = ctypes.POINTER(ctypes.c_int64)


class GemmConfig(ctypes.Structure):
    """``lunara_gemm_config``: block_n, stages, num_ctas, cta_pair (0 = automatic)."""

    _fields_ = [("block_n", ctypes.c_int32), ("stages", ctypes.c_int32),
                ("num_ctas", ctypes.c_int32), ("cta_pair", ctypes.c_int32)]


SIGNATURES = {
    "lunara_gemm": ([_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i, _i, _i,
                     ctypes.POINTER(GemmConfig), _p], _i),
    "lunara_gemm_layernorm": ([_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i, _i, _f,
                               ctypes.POINTER(GemmConfig), _p], _i),
    "lunara_attention": ([_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _pi64, _pi64, _pi64, _pi64,
                          _f, _i, _i, _p], _i),
    "lunara_layernorm": ([_p, _p, _p, _p, _i64, _i64, _f, _i, _p], _i),
    "lunara_softmax": ([_p, _p, _i64, _i64, _i, _p], _i),
    "lunara_eltwise_unary": ([_i, _p, _p, _i64, _i, _p], _i),
    "lunara_eltwise_binary": ([_i, _p, _p, _p, _i64, _i, _p], _i),
    "lunara_bias_act": ([_p, _p, _p, _i64, _i64, _i, _i, _p], _i),
    "lunara_gather": ([_p, _p, _p, _i64, _i64, _i64, _p], _i),
    "lunara_copy_strided": ([_p, _p, _i, _pi64, _pi64, _i64, _p], _i),
    "lunara_slice": ([_p, _p, _i, _pi64, _pi64, _pi64, _pi64, _i64, _p], _i),
    "lunara_qkv_split": ([_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p], _i),
    "lunara_last_error_string": ([], ctypes.c_char_p),
    "lunara_device_error": ([_p, _i], _i),
    "lunara_num_sms": ([], _i),
    "lunara_version": ([], _i),
}

# Internal self-test entry points, declared in include/lunara_b200_selftest.h
# (not part of the kernel ABI; used by the tests only).
SELFTEST_SIGNATURES = {
    "lunara_selftest_ex2_poly": ([_p, _p, _i64, _i, _p], _i),
    "lunara_selftest_bounded_wait": ([ctypes.c_uint64, ctypes.c_uint, _p], _i),
}


class LunaraError(RuntimeError):
    """A kernel-library call returned a non-zero lunara_status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[lunara status {status}] {message}")
        self.status = status


_lib = None


def load(path: os.PathLike | str | None = None) -> ctypes.CDLL:
    """Load (once) and return the kernel library with typed entry points."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"lunara_b200 kernel library not found at {p}; build it with `python -m lunara_b200.build`")
    lib = ctypes.CDLL(str(p))
    for name, (argtypes, restype) in {**SIGNATURES, **SELFTEST_SIGNATURES}.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    _lib = lib
    return lib


def check(rc: int) -> None:
    """Raise LunaraError for a non-zero status, with the library's message."""
    if rc != OK:
        msg = load().lunara_last_error_string().decode(errors="replace")
        if rc == ERR_INVALID_ARG:
            raise ValueError(f"[lunara status {rc}] {msg}")
        raise LunaraError(rc, msg)


def i64_array(values) -> ctypes.Array:
    vals = [int(v) for v in values]
    return (ctypes.c_int64 * max(1, len(vals)))(*vals)
