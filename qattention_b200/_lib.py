"""ctypes binding of ``libqattn_b200.so`` (the C ABI declared in include/qattn_b200.h).

The library is loaded from this package directory only. There is no fallback:
if it is missing or fails to load, :func:`lib` raises, so a GPU box without the
built extension fails loudly instead of silently computing elsewhere.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, Structure, c_char_p, c_float, c_int, c_int32, c_int64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqattn_b200.so"

QA_OK = 0
QA_DTYPE_F16 = 0
QA_DTYPE_BF16 = 1

# Every symbol the header declares; tests check the library exports all of them.
EXPORTED = (
    "qa_add_rmsnorm",
    "qa_rope_qkv",
    "qa_silu_mul",
    "qa_ancestor_attn",
    "qa_lse_merge",
    "qa_prefix_attn",
    "qa_check_device_error",
    "qa_ancestor_diagnostics",
    "qa_ancestor_workspace_bytes",
    "qa_ancestor_plan",
    "qa_set_pipeline_wait_limit",
    "qa_w4a16_gemm",
    "qa_w4a16_plan",
    "qa_w4a16_dequant",
    "qa_w4a16_gemm_noalloc",
    "qa_status_string",
    "qa_version",
)


class AncestorArgs(Structure):
    """Mirror of ``qa_ancestor_args`` (field order and types must match the header)."""

    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("o", c_void_p),
        ("lse", c_void_p),
        ("cu_seqlens_q", c_void_p), ("cu_seqlens_kv", c_void_p), ("parents", c_void_p),
        ("prefix_o", c_void_p), ("prefix_lse", c_void_p),
        ("q_stride_t", c_int64), ("q_stride_h", c_int64),
        ("k_stride_t", c_int64), ("k_stride_h", c_int64),
        ("v_stride_t", c_int64), ("v_stride_h", c_int64),
        ("o_stride_t", c_int64), ("o_stride_h", c_int64),
        ("lse_stride_t", c_int64), ("lse_stride_h", c_int64),
        ("prefix_o_stride_t", c_int64), ("prefix_o_stride_h", c_int64),
        ("prefix_lse_stride_t", c_int64), ("prefix_lse_stride_h", c_int64),
        ("batch", c_int32), ("num_q_heads", c_int32), ("num_kv_heads", c_int32),
        ("head_dim", c_int32), ("kv_offset", c_int32), ("branching", c_int32),
        ("max_depth", c_int32), ("max_seqlen", c_int32),
        ("scale", c_float), ("dtype", c_int32),
        ("page_table", c_void_p), ("page_table_stride", c_int64),
        ("k_stride_page", c_int64), ("v_stride_page", c_int64), ("page_size", c_int32),
        ("q_stride_b", c_int64),
        ("workspace", c_void_p), ("workspace_bytes", c_int64), ("workspace_planned", c_int32),
    ]


class PrefixArgs(Structure):
    """Mirror of ``qa_prefix_args``."""

    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("o", c_void_p), ("lse", c_void_p),
        ("q_stride_b", c_int64), ("q_stride_t", c_int64), ("q_stride_h", c_int64),
        ("k_stride_b", c_int64), ("k_stride_t", c_int64), ("k_stride_h", c_int64),
        ("v_stride_b", c_int64), ("v_stride_t", c_int64), ("v_stride_h", c_int64),
        ("o_stride_b", c_int64), ("o_stride_t", c_int64), ("o_stride_h", c_int64),
        ("lse_stride_b", c_int64), ("lse_stride_t", c_int64), ("lse_stride_h", c_int64),
        ("batch", c_int32), ("num_queries", c_int32), ("prefix_len", c_int32),
        ("num_q_heads", c_int32), ("num_kv_heads", c_int32), ("head_dim", c_int32),
        ("scale", c_float), ("dtype", c_int32),
    ]


class W4A16Args(Structure):
    """Mirror of ``qa_w4a16_args``."""

    _fields_ = [
        ("x", c_void_p), ("qweight", c_void_p), ("scales", c_void_p), ("y", c_void_p),
        ("workspace", c_void_p), ("x_stride", c_int64), ("y_stride", c_int64),
        ("M", c_int32), ("N", c_int32), ("K", c_int32), ("splits", c_int32),
        ("counters", c_void_p),
    ]


_LIB = None


class QAError(RuntimeError):
    """A non-zero status returned by the C ABI."""


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH.name} is not built; run `python -m qattention_b200.build` "
                "(nvcc, sm_100a) before using the CUDA path")
        L = ctypes.CDLL(str(LIB_PATH))
        L.qa_ancestor_attn.argtypes = [POINTER(AncestorArgs), c_void_p]
        L.qa_ancestor_attn.restype = c_int
        i64p = POINTER(c_int64)
        L.qa_lse_merge.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                   c_int32, c_int32, c_int32, c_int32,
                                   i64p, i64p, i64p, i64p, i64p, c_int32, c_void_p]
        L.qa_lse_merge.restype = c_int
        L.qa_prefix_attn.argtypes = [POINTER(PrefixArgs), c_void_p]
        L.qa_prefix_attn.restype = c_int
        L.qa_check_device_error.argtypes = [POINTER(c_int)]
        L.qa_check_device_error.restype = c_int
        L.qa_ancestor_diagnostics.argtypes = [POINTER(c_int32)]
        L.qa_ancestor_diagnostics.restype = c_int
        L.qa_ancestor_workspace_bytes.argtypes = [POINTER(AncestorArgs), POINTER(c_int64)]
        L.qa_ancestor_workspace_bytes.restype = c_int
        L.qa_ancestor_plan.argtypes = [POINTER(AncestorArgs), c_void_p]
        L.qa_ancestor_plan.restype = c_int
        L.qa_set_pipeline_wait_limit.argtypes = [ctypes.c_uint32]
        L.qa_set_pipeline_wait_limit.restype = c_int
        L.qa_w4a16_gemm.argtypes = [POINTER(W4A16Args), c_void_p]
        L.qa_w4a16_gemm.restype = c_int
        L.qa_w4a16_gemm_noalloc.argtypes = [POINTER(W4A16Args), c_void_p]
        L.qa_w4a16_gemm_noalloc.restype = c_int
        L.qa_w4a16_plan.argtypes = [c_int32, c_int32, c_int32, POINTER(c_int32), POINTER(c_int64)]
        L.qa_w4a16_plan.restype = c_int
        L.qa_w4a16_dequant.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_void_p]
        L.qa_w4a16_dequant.restype = c_int
        L.qa_add_rmsnorm.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_float, c_void_p]
        L.qa_add_rmsnorm.restype = c_int
        L.qa_rope_qkv.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                  c_int32, c_int32, c_int64, c_int64, c_int32, c_void_p]
        L.qa_rope_qkv.restype = c_int
        L.qa_silu_mul.argtypes = [c_void_p, c_void_p, c_int32, c_int32, c_void_p]
        L.qa_silu_mul.restype = c_int
        L.qa_status_string.argtypes = [c_int]
        L.qa_status_string.restype = c_char_p
        L.qa_version.argtypes = []
        L.qa_version.restype = c_char_p
        _LIB = L
    return _LIB


def device_error() -> int:
    """Read and clear the device error flag of the pipelined kernels (synchronising)."""
    flag = c_int(0)
    check(lib().qa_check_device_error(ctypes.byref(flag)), "qa_check_device_error")
    return flag.value


def check(status: int, what: str) -> None:
    if status != QA_OK:
        msg = lib().qa_status_string(status).decode()
        raise QAError(f"{what} failed: {msg} (status {status})")


def i64_array(vals) -> ctypes.Array:
    return (c_int64 * len(vals))(*[int(v) for v in vals])


def ancestor_diagnostics() -> list:
    """Read and clear the ancestor kernel's first failed plan check (8 ints; [0] == 0: none)."""
    out = (c_int32 * 8)()
    check(lib().qa_ancestor_diagnostics(out), "qa_ancestor_diagnostics")
    return list(out)
