"""ctypes binding of the C-ABI kernel library (include/llama_int4_b200.h).

The library is lib/libllama_int4_b200.so next to this package, built by
build.py.  There is no fallback: if it is missing or fails to load, every
entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libllama_int4_b200.so")

LI4_OK = 0
LI4_ERR_INVALID_ARG = 1
LI4_ERR_ALIGNMENT = 2
LI4_ERR_WORKSPACE = 3
LI4_ERR_UNSUPPORTED = 4
LI4_ERR_CUDA = 5

LI4_F16, LI4_BF16, LI4_F32 = 0, 1, 2
WORKSPACE_COUNTER_BYTES = 65536  # LI4_WORKSPACE_COUNTER_BYTES
KERNEL_AUTO, KERNEL_CUDA_CORE, KERNEL_MMA, KERNEL_STREAM, KERNEL_TILE, KERNEL_BULK, KERNEL_SLAB, KERNEL_ROWS, \
    KERNEL_RING = 0, 1, 2, 3, 4, 5, 6, 7, 8

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_INT = ctypes.c_int

LI4_EPI_STORE, LI4_EPI_RESIDUAL, LI4_EPI_SWIGLU, LI4_EPI_QKV_ROPE, LI4_EPI_STORE_F32 = 0, 1, 2, 3, 4
LI4_EPI_ALLREDUCE_RESIDUAL = 5


class GemvProblem(ctypes.Structure):
    """struct li4_gemv_problem (include/llama_int4_b200.h): one GEMV of a grouped launch."""

    _fields_ = [("x", ctypes.c_void_p), ("packed", ctypes.c_void_p), ("scale", ctypes.c_void_p),
                ("zero", ctypes.c_void_p), ("y", ctypes.c_void_p), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
                ("stride_xm", ctypes.c_int64), ("stride_pn", ctypes.c_int64), ("stride_sn", ctypes.c_int64),
                ("stride_ym", ctypes.c_int64)]


class Fusion(ctypes.Structure):
    """struct li4_fusion (include/llama_int4_b200.h): fused prologue / epilogue of one GEMV."""

    _fields_ = [
        ("norm_weight", ctypes.c_void_p),
        ("norm_eps", ctypes.c_float),
        ("epilogue", ctypes.c_int),
        ("residual", ctypes.c_void_p),
        ("stride_rm", ctypes.c_int64),
        ("q_rows", ctypes.c_int64),
        ("k_rows", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("pos", ctypes.c_void_p),
        ("rope_cos", ctypes.c_void_p),
        ("rope_sin", ctypes.c_void_p),
        ("rope_stride", ctypes.c_int64),
        ("q_out", ctypes.c_void_p),
        ("stride_qm", ctypes.c_int64),
        ("cache_k", ctypes.c_void_p),
        ("cache_v", ctypes.c_void_p),
        ("cache_stride_b", ctypes.c_int64),
        ("cache_stride_s", ctypes.c_int64),
        ("sumsq_out", ctypes.c_void_p),
        ("sumsq_in", ctypes.c_void_p),
        ("sumsq_tiles", ctypes.c_int64),
        ("argmax_out", ctypes.c_void_p),
        ("argmax_stride", ctypes.c_int64),
        ("argmax_scratch", ctypes.c_void_p),
        ("ar_recv", ctypes.c_void_p),
        ("ar_recv_bytes", ctypes.c_size_t),
        ("ar_epochs", ctypes.c_void_p),
        ("ar_world", ctypes.c_int),
        ("ar_rank", ctypes.c_int),
    ]


# name -> (restype, argtypes); mirrors include/llama_int4_b200.h
SIGNATURES = {
    "li4_version": (_INT, []),
    "li4_last_error": (ctypes.c_char_p, []),
    "li4_int4_linear_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I64, _INT]),
    "li4_int4_linear_plan": (_INT, [_I64, _I64, _I64, _I64, _INT, ctypes.POINTER(_INT), ctypes.POINTER(_INT),
                                    ctypes.POINTER(_INT), ctypes.POINTER(_SZ)]),
    "li4_int4_linear": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _SZ, _P]),
    "li4_int4_linear_ex": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _SZ, _P,
                                  _INT, _INT, _INT, _INT]),
    "li4_argmax_rows_allreduce": (_INT, [_P, _INT, _I64, _I64, _I64, _I64, _P, _SZ, _P, _INT, _INT, _P, _I64, _P]),
    "li4_int4_linear_grouped_table_bytes": (_SZ, [_P, _INT, _I64, ctypes.POINTER(_INT)]),
    "li4_int4_linear_grouped_build": (_INT, [_P, _INT, _I64, _I64, _P, _SZ]),
    "li4_int4_linear_grouped": (_INT, [_P, _INT, _INT, _I64, _P]),
    "li4_int4_linear_noalloc": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "li4_int4_gemm": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "li4_int4_linear_fused": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                     ctypes.POINTER(Fusion), _P, _SZ, _P]),
    "li4_decode_attention": (_INT, [_P, _I64, _P, _P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I64, _P, _I64, _P]),
    "li4_argmax_rows": (_INT, [_P, _INT, _I64, _I64, _I64, _P, _I64, _P]),
    "li4_argmax_rows_keys": (_INT, [_P, _INT, _I64, _I64, _I64, _I64, _P, _I64, _P]),
    "li4_device_errors": (_INT, [ctypes.POINTER(ctypes.c_uint), _INT]),
    "li4_debug_set_wait_limits": (_INT, [ctypes.c_uint, ctypes.c_uint, ctypes.c_uint]),
    "li4_comm_alloc": (_INT, [_SZ, ctypes.POINTER(_P)]),
    "li4_comm_free": (_INT, [_P]),
    "li4_ipc_get_handle": (_INT, [_P, _P]),
    "li4_ipc_open_handle": (_INT, [_P, ctypes.POINTER(_P)]),
    "li4_ipc_close": (_INT, [_P]),
    "li4_allreduce_add": (_INT, [ctypes.POINTER(_P), ctypes.POINTER(_P), _P, _INT, _INT, _INT, _I64, _P, _P, _P]),
    "li4_gather_rows": (_INT, [_P, _I64, _I64, _I64, _P, _I64, _P, _I64, _P]),
    "li4_program_create": (_INT, [ctypes.POINTER(_P)]),
    "li4_program_destroy": (_INT, [_P]),
    "li4_program_add_linear": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                      ctypes.POINTER(Fusion), _INT, ctypes.POINTER(_INT)]),
    "li4_program_add_attention": (_INT, [_P, _P, _I64, _P, _P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I64, _P,
                                         _I64, _INT, ctypes.POINTER(_INT)]),
    "li4_program_add_gather": (_INT, [_P, _P, _I64, _I64, _I64, _P, _I64, _P, _I64, _INT, ctypes.POINTER(_INT)]),
    "li4_program_add_argmax": (_INT, [_P, _P, _I64, _I64, _I64, _P, _I64, _INT, ctypes.POINTER(_INT)]),
    "li4_program_add_increment": (_INT, [_P, _P]),
    "li4_program_finalize": (_INT, [_P]),
    "li4_program_launch": (_INT, [_P, _P]),
    "li4_program_set_trace": (_INT, [_P, _P, _I64]),
    "li4_program_info": (_INT, [_P, ctypes.POINTER(_INT), ctypes.POINTER(_INT), ctypes.POINTER(_SZ)]),
    "li4_dequantize": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "li4_quantize": (_INT, [_P, _INT, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
}

_lock = threading.Lock()
_lib = None


class Li4Error(RuntimeError):
    """A C-ABI call returned a non-zero li4_status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (li4_status {status})")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load the kernel library (once)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is missing: build it with "
                                  f"`python {os.path.join(PKG_DIR, 'build.py')}` (nvcc, sm_100a)")
            l = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(l, name)
                fn.restype = res
                fn.argtypes = args
            _lib = l
    return _lib


def last_error() -> str:
    return lib().li4_last_error().decode(errors="replace")


def check(status: int, what: str = "") -> None:
    if status != LI4_OK:
        msg = last_error()
        raise Li4Error(status, f"{what}: {msg}" if what else msg)


def device_errors(reset: bool = True) -> int:
    """Device-side error flags (li4_device_errors); synchronises the device."""
    flags = ctypes.c_uint(0)
    check(lib().li4_device_errors(ctypes.byref(flags), int(reset)), "device_errors")
    return flags.value


KERNEL_NAMES = {KERNEL_CUDA_CORE: "cuda_core", KERNEL_MMA: "mma", KERNEL_STREAM: "stream", KERNEL_TILE: "tile",
                KERNEL_BULK: "bulk", KERNEL_SLAB: "slab", KERNEL_ROWS: "rows", KERNEL_RING: "ring"}
KERNEL_SYMBOLS = {KERNEL_CUDA_CORE: "gemv_cc_kernel", KERNEL_MMA: "gemv_mma_kernel", KERNEL_STREAM: "gemv_stream_kernel",
                  KERNEL_TILE: "gemv_tile_kernel", KERNEL_BULK: "gemv_bulk_kernel", KERNEL_SLAB: "gemv_slab_kernel",
                  KERNEL_ROWS: "gemv_rows_kernel", KERNEL_RING: "gemv_ring_kernel"}


def plan(M: int, N: int, K: int, group_size: int = 128, sm_count: int = 0) -> dict:
    """The launch plan li4_int4_linear picks for a contiguous problem (li4_int4_linear_plan)."""
    k, sp, gx, sm = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
    check(lib().li4_int4_linear_plan(M, N, K, group_size, sm_count, ctypes.byref(k), ctypes.byref(sp),
                                     ctypes.byref(gx), ctypes.byref(sm)), "int4_linear_plan")
    return {"kernel": KERNEL_NAMES.get(k.value, str(k.value)), "symbol": KERNEL_SYMBOLS.get(k.value, ""),
            "split": sp.value, "grid_x": gx.value, "smem": sm.value}


def stream_ptr(device: torch.device) -> int:
    """The current CUDA stream of `device` as a raw handle (cheap: no Stream object is built)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return torch._C._cuda_getCurrentRawStream(idx)


def ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


# ---------------------------------------------------------------------------
# Split-K workspace: one zero-initialised buffer per device, grown outside
# CUDA-graph capture.  Kernels leave its counters at zero, so launches that
# follow each other on a stream (eager or replayed) can share it; launches that
# may overlap on the GPU (different streams) must not.
# ---------------------------------------------------------------------------
_ws: dict[int, torch.Tensor] = {}
_WS_MIN = 8 << 20


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _ws.get(idx)
    if buf is None or buf.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(f"int4_linear needs a {nbytes}-byte split-K workspace on cuda:{idx} but a CUDA graph "
                               f"is being captured; run the same call once eagerly (warm-up) before capture, or "
                               f"call llama.int4_gemv.reserve_workspace() first")
        size = max(nbytes, _WS_MIN, 2 * (buf.numel() if buf is not None else 0))
        buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
        _ws[idx] = buf
    return buf
