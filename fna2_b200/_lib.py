"""ctypes binding of ``libfna2_b200.so`` (the C ABI declared in include/fna2.h).

The structures below mirror the C structs field for field.  Loading fails
loudly when the shared library is missing: there is no fallback path.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("FNA2_LIB", os.path.join(HERE, "libfna2_b200.so"))

FNA2_ABI_VERSION = 5
FNA2_OK = 0
FNA2_ERR_INVALID = -1
FNA2_ERR_CUDA = -2
FNA2_ERR_WORKSPACE = -3

EXPORTED = ["fna2_fwd", "fna2_bwd", "fna2_bwd_workspace_size", "fna2_last_error", "fna2_device_status",
            "fna2_abi_version", "fna2_bwd_noalloc", "fna2_qk_prep_fwd", "fna2_qk_prep_bwd", "fna2_decode", "fna2_decode_workspace_size",
            "fna2_debug_watchdog", "fna2_fwd_workspace_size", "fna2_gemm"]
FNA2_DTYPE_F32 = 0
FNA2_DTYPE_BF16 = 1
NOALLOC_SCRATCH_BYTES = 32 * 1024 * 1024  # FNA2_NOALLOC_SCRATCH_BYTES


class Fna2Tensor(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("stride", ctypes.c_int64 * 4)]


class Fna2Problem(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("seqlen_q", ctypes.c_int32),
        ("seqlen_k", ctypes.c_int32),
        ("total_q", ctypes.c_int32),
        ("total_k", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("heads_kv", ctypes.c_int32),
        ("heads_graph", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("softmax_scale", ctypes.c_float),
        ("causal", ctypes.c_int32),
        ("cu_seqlens_q", ctypes.c_void_p),
        ("cu_seqlens_k", ctypes.c_void_p),
    ]


class Fna2FwdArgs(ctypes.Structure):
    _fields_ = [
        ("prob", Fna2Problem),
        ("q", Fna2Tensor),
        ("k", Fna2Tensor),
        ("v", Fna2Tensor),
        ("r_q", Fna2Tensor),
        ("r_k", Fna2Tensor),
        ("graph_scale", ctypes.c_void_p),
        ("out", Fna2Tensor),
        ("lse", ctypes.c_void_p),
        ("launch_events", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


class Fna2BwdArgs(ctypes.Structure):
    _fields_ = [
        ("prob", Fna2Problem),
        ("q", Fna2Tensor),
        ("k", Fna2Tensor),
        ("v", Fna2Tensor),
        ("r_q", Fna2Tensor),
        ("r_k", Fna2Tensor),
        ("graph_scale", ctypes.c_void_p),
        ("out", Fna2Tensor),
        ("dout", Fna2Tensor),
        ("lse", ctypes.c_void_p),
        ("dq", Fna2Tensor),
        ("dk", Fna2Tensor),
        ("dv", Fna2Tensor),
        ("dr_q", Fna2Tensor),
        ("dr_k", Fna2Tensor),
        ("d_graph_scale", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("launch_events", ctypes.c_void_p),
    ]


class Fna2Rows(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("token_stride", ctypes.c_int64), ("head_stride", ctypes.c_int64)]


class Fna2QkPrepArgs(ctypes.Structure):
    _fields_ = [
        ("total_tokens", ctypes.c_int64),
        ("num_seqs", ctypes.c_int32),
        ("cu_seqlens", ctypes.c_void_p),
        ("heads_q", ctypes.c_int32),
        ("heads_k", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("in_dtype", ctypes.c_int32),
        ("weight_dtype", ctypes.c_int32),
        ("rope_dtype", ctypes.c_int32),
        ("q_in", Fna2Rows),
        ("k_in", Fna2Rows),
        ("q_out", Fna2Rows),
        ("k_out", Fna2Rows),
        ("q_weight", ctypes.c_void_p),
        ("k_weight", ctypes.c_void_p),
        ("eps", ctypes.c_float),
        ("inv_freq", ctypes.c_void_p),
    ]


class Fna2QkPrepBwdArgs(ctypes.Structure):
    _fields_ = [
        ("fwd", Fna2QkPrepArgs),
        ("dq_out", Fna2Rows),
        ("dk_out", Fna2Rows),
        ("dq_in", Fna2Rows),
        ("dk_in", Fna2Rows),
        ("dq_weight", ctypes.c_void_p),
        ("dk_weight", ctypes.c_void_p),
    ]


_I64 = ctypes.c_int64


class Fna2DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int), ("heads", ctypes.c_int), ("kv_heads", ctypes.c_int),
        ("graph_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("rank", ctypes.c_int),
        ("capacity", ctypes.c_int), ("softmax_scale", ctypes.c_float),
        ("q", ctypes.c_void_p), ("q_batch_stride", _I64), ("q_head_stride", _I64),
        ("r_q", ctypes.c_void_p), ("rq_batch_stride", _I64), ("rq_head_stride", _I64),
        ("k_cache", ctypes.c_void_p), ("k_batch_stride", _I64), ("k_token_stride", _I64), ("k_head_stride", _I64),
        ("v_cache", ctypes.c_void_p), ("v_batch_stride", _I64), ("v_token_stride", _I64), ("v_head_stride", _I64),
        ("rk_cache", ctypes.c_void_p), ("rk_batch_stride", _I64), ("rk_token_stride", _I64),
        ("rk_head_stride", _I64),
        ("graph_scale", ctypes.c_void_p), ("cache_seqlens", ctypes.c_void_p), ("cache_offsets", ctypes.c_void_p),
        ("k_new", ctypes.c_void_p), ("kn_batch_stride", _I64), ("kn_head_stride", _I64),
        ("v_new", ctypes.c_void_p), ("vn_batch_stride", _I64), ("vn_head_stride", _I64),
        ("rk_new", ctypes.c_void_p), ("rkn_batch_stride", _I64), ("rkn_head_stride", _I64),
        ("out", ctypes.c_void_p), ("out_batch_stride", _I64), ("out_head_stride", _I64),
        ("lse", ctypes.c_void_p), ("num_splits", ctypes.c_int),
    ]


class Fna2GemmArgs(ctypes.Structure):
    _fields_ = [
        ("m", _I64), ("n", _I64), ("k", _I64),
        ("a", ctypes.c_void_p), ("lda", _I64), ("a_mn_major", ctypes.c_int32),
        ("b", ctypes.c_void_p), ("ldb", _I64), ("b_mn_major", ctypes.c_int32),
        ("c", ctypes.c_void_p), ("ldc", _I64), ("c_dtype", ctypes.c_int32),
        ("split_k", ctypes.c_int32),
    ]


_lib: Optional[ctypes.CDLL] = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library once; raise if it is missing or of another ABI."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"libfna2_b200.so not found at {path}; build it with `python -m fna2_b200.build` "
            "(there is no CPU or fallback implementation)")
    lib = ctypes.CDLL(path)
    lib.fna2_fwd.argtypes = [ctypes.POINTER(Fna2FwdArgs), ctypes.c_void_p]
    lib.fna2_fwd.restype = ctypes.c_int
    lib.fna2_bwd.argtypes = [ctypes.POINTER(Fna2BwdArgs), ctypes.c_void_p]
    lib.fna2_bwd.restype = ctypes.c_int
    lib.fna2_bwd_noalloc.argtypes = [ctypes.POINTER(Fna2BwdArgs), ctypes.c_void_p]
    lib.fna2_bwd_noalloc.restype = ctypes.c_int
    lib.fna2_qk_prep_fwd.argtypes = [ctypes.POINTER(Fna2QkPrepArgs), ctypes.c_void_p]
    lib.fna2_qk_prep_fwd.restype = ctypes.c_int
    lib.fna2_qk_prep_bwd.argtypes = [ctypes.POINTER(Fna2QkPrepBwdArgs), ctypes.c_void_p]
    lib.fna2_qk_prep_bwd.restype = ctypes.c_int
    lib.fna2_decode.argtypes = [ctypes.POINTER(Fna2DecodeArgs), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.fna2_decode.restype = ctypes.c_int
    lib.fna2_decode_workspace_size.argtypes = [ctypes.POINTER(Fna2DecodeArgs)]
    lib.fna2_decode_workspace_size.restype = ctypes.c_size_t
    lib.fna2_fwd_workspace_size.argtypes = [ctypes.POINTER(Fna2Problem)]
    lib.fna2_fwd_workspace_size.restype = ctypes.c_size_t
    lib.fna2_bwd_workspace_size.argtypes = [ctypes.POINTER(Fna2Problem)]
    lib.fna2_bwd_workspace_size.restype = ctypes.c_size_t
    lib.fna2_last_error.argtypes = []
    lib.fna2_last_error.restype = ctypes.c_char_p
    lib.fna2_device_status.argtypes = [ctypes.c_int]
    lib.fna2_device_status.restype = ctypes.c_int
    lib.fna2_debug_watchdog.argtypes = [ctypes.c_int, ctypes.c_ulonglong]
    lib.fna2_debug_watchdog.restype = ctypes.c_int
    lib.fna2_gemm.argtypes = [ctypes.POINTER(Fna2GemmArgs), ctypes.c_void_p]
    lib.fna2_gemm.restype = ctypes.c_int
    lib.fna2_abi_version.argtypes = []
    lib.fna2_abi_version.restype = ctypes.c_int
    v = lib.fna2_abi_version()
    if v != FNA2_ABI_VERSION:
        raise RuntimeError(f"libfna2_b200.so ABI {v} != expected {FNA2_ABI_VERSION}; rebuild it")
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != FNA2_OK:
        msg = load().fna2_last_error().decode(errors="replace")
        kind = {FNA2_ERR_INVALID: "invalid argument", FNA2_ERR_CUDA: "CUDA error",
                FNA2_ERR_WORKSPACE: "workspace too small"}.get(rc, f"error {rc}")
        raise RuntimeError(f"{what}: {kind}: {msg}")
