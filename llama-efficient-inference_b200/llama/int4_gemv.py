"""Fused INT4 dequant + GEMV / small-M GEMM on B200 (sm_100a): drop-in for the
reference's llama/int4_gemv.py.

    y[M, N] = x[M, K] @ W[N, K]^T,   W stored as QuantizedLinear buffers:
        packed [N, K/2] uint8 (low nibble = even k, high nibble = odd k)
        scale, zp [N, K/group] fp16,  W = (q - zp) * scale

Same entry point and contract as the reference's int4_linear
(llama/int4_gemv.py:105-140): x fp16 with any leading dims (made contiguous
when needed), prod(leading dims) <= MAX_M, K % group_size == 0, a new fp16
tensor [..., N] on the current stream.  The Triton tuning knobs (block_n,
split_k, num_warps) are accepted and ignored: the launch shape is chosen in
C++ from (M, N, K, SM count).  The work runs in one CUDA kernel from
libllama_int4_b200.so (no Triton, no CPU path): split-K partial sums are
reduced inside the same launch, so there is no zero-fill or cast kernel.

This module may be loaded by file path (llama/quantize.py int4_linear_fn does,
like the reference), so it locates its sibling _native.py by path too.
"""
from __future__ import annotations

import ctypes
import importlib.util
import os
import sys

import torch


def _load_native():
    mod = sys.modules.get("li4_native")
    if mod is None:
        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_native.py")
        spec = importlib.util.spec_from_file_location("li4_native", path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules["li4_native"] = mod
        spec.loader.exec_module(mod)
    return mod


_native = _load_native()

MAX_M = 16
_ws_bytes: dict = {}  # (M, N, K, group_size, device) -> split-K workspace bytes


def _check_operands(x2: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, zp: torch.Tensor):
    if not x2.is_cuda:
        raise RuntimeError("int4_linear runs on CUDA tensors only (x is on %s)" % x2.device)
    dev = x2.device
    for name, t in (("packed", packed), ("scale", scale), ("zp", zp)):
        if t.device != dev:
            raise RuntimeError(f"int4_linear: {name} is on {t.device}, x is on {dev}")
    if packed.dtype != torch.uint8:
        raise RuntimeError(f"int4_linear: packed must be uint8, got {packed.dtype}")
    if scale.dtype != torch.float16 or zp.dtype != torch.float16:
        raise RuntimeError(f"int4_linear: scale / zp must be float16, got {scale.dtype} / {zp.dtype}")
    if packed.stride(1) != 1:
        packed = packed.contiguous()
    if scale.stride(1) != 1 or zp.stride(1) != 1 or scale.stride(0) != zp.stride(0):
        scale, zp = scale.contiguous(), zp.contiguous()
    return packed, scale, zp


def int4_linear_out(x2: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, zp: torch.Tensor,
                    y: torch.Tensor, group_size: int = 128, kernel: int = 0, rows_per_cta: int = 0,
                    split: int = 0, max_ctas: int = 0, workspace: torch.Tensor = None) -> torch.Tensor:
    """y[M, N] = x2[M, K] @ W^T into a caller-owned fp16 y (row stride y.stride(0)).

    For CUDA-graph capture with static buffers.  kernel / rows_per_cta /
    split / max_ctas force a launch shape (0 = automatic), for tuning sweeps.
    workspace: a caller-owned zero-initialised uint8 split-K workspace (for
    launches that may overlap on the GPU, e.g. on several streams); default:
    the device's shared one.
    """
    M, K = x2.shape
    N = packed.shape[0]
    if y.shape != (M, N) or y.dtype != torch.float16 or y.stride(1) != 1 or y.device != x2.device:
        raise RuntimeError(f"int4_linear_out: y must be a float16 [{M}, {N}] row-major tensor on {x2.device}")
    if x2.stride(1) != 1:
        raise RuntimeError("int4_linear_out: x rows must be contiguous")
    packed, scale, zp = _check_operands(x2, packed, scale, zp)
    if M == 0 or N == 0:
        return y
    lib = _native.lib()
    dev = x2.device
    key = (M, N, K, group_size, dev.index)
    nbytes = _ws_bytes.get(key)
    if nbytes is None:  # the plan depends only on the shape and the device: ask the library once
        nbytes = _ws_bytes[key] = lib.li4_int4_linear_workspace_bytes(M, N, K, group_size, 0)
    if workspace is not None:
        if workspace.dtype != torch.uint8 or workspace.device != dev or workspace.numel() < nbytes:
            raise RuntimeError(f"int4_linear_out: the workspace must be a uint8 tensor of >= {nbytes} bytes on {dev}")
        ws = workspace
    else:
        ws = _native.workspace(dev, nbytes) if nbytes else None
    ws_ptr, ws_len = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    stream = _native.stream_ptr(dev)
    if kernel or rows_per_cta or split or max_ctas:
        if split > 1:  # the fixed counter region + split fp32 partials of [M, N]
            need = _native.WORKSPACE_COUNTER_BYTES + split * M * N * 4
            ws = _native.workspace(dev, max(need, nbytes))
            ws_ptr, ws_len = ws.data_ptr(), ws.numel()
        rc = lib.li4_int4_linear_ex(x2.data_ptr(), packed.data_ptr(), scale.data_ptr(), zp.data_ptr(), y.data_ptr(),
                                    M, N, K, group_size, x2.stride(0), packed.stride(0), scale.stride(0),
                                    y.stride(0), ws_ptr, ws_len, stream, kernel, rows_per_cta, split, max_ctas)
    else:
        rc = lib.li4_int4_linear(x2.data_ptr(), packed.data_ptr(), scale.data_ptr(), zp.data_ptr(), y.data_ptr(),
                                 M, N, K, group_size, x2.stride(0), packed.stride(0), scale.stride(0), y.stride(0),
                                 ws_ptr, ws_len, stream)
    _native.check(rc, "int4_linear")
    return y


def int4_linear(x, packed, scale, zp, group_size=128, block_n=128, split_k=None, num_warps=8):
    """x [..., K] fp16 with prod(...) <= 16  ->  [..., N] fp16."""
    N, half_k = packed.shape
    K = half_k * 2
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    M = x2.shape[0]
    assert M <= MAX_M and x.dtype == torch.float16 and K % group_size == 0
    y = torch.empty(M, N, dtype=torch.float16, device=x.device)
    int4_linear_out(x2, packed, scale, zp, y, group_size)
    return y.reshape(*lead, N)


class GroupedGemv:
    """Many independent INT4 GEMVs in one persistent launch (li4_int4_linear_grouped).

    problems: (x [M, K] fp16, packed, scale, zp, y [M, N] fp16) tuples on one device, every x with
    the same M (1..8).  The device table (the problems and their tiles cut into per-CTA ranges of
    about equal weight bytes) is built once here; each call launches on the current stream with no
    host data (capturable in a CUDA graph).  Results are li4_int4_linear's up to the order of the
    fp32 sums."""

    def __init__(self, problems, group_size: int = 128):
        lib = _native.lib()
        if not problems:
            raise ValueError("GroupedGemv: no problems")
        M = problems[0][0].shape[0]
        self.device = problems[0][0].device
        arr = (_native.GemvProblem * len(problems))()
        for i, (x, p, s, z, y) in enumerate(problems):
            if x.shape[0] != M or y.shape != (M, p.shape[0]) or x.dtype != torch.float16 or y.dtype != torch.float16:
                raise RuntimeError(f"GroupedGemv: problem {i}: x [{M}, K] and y [{M}, N] fp16 expected")
            p, s, z = _check_operands(x, p, s, z)
            arr[i] = _native.GemvProblem(x.data_ptr(), p.data_ptr(), s.data_ptr(), z.data_ptr(), y.data_ptr(),
                                         p.shape[0], x.shape[1], x.stride(0), p.stride(0), s.stride(0), y.stride(0))
        units = ctypes.c_int()
        nbytes = lib.li4_int4_linear_grouped_table_bytes(arr, len(problems), M, ctypes.byref(units))
        if nbytes == 0:
            _native.check(_native.LI4_ERR_INVALID_ARG, "int4_linear_grouped_table_bytes")
        self.table = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        _native.check(lib.li4_int4_linear_grouped_build(arr, len(problems), M, group_size, self.table.data_ptr(),
                                                        nbytes), "int4_linear_grouped_build")
        self.n, self.units, self.M = len(problems), units.value, M
        self._keep = problems  # the tensors the table points at

    def __call__(self) -> None:
        _native.check(_native.lib().li4_int4_linear_grouped(self.table.data_ptr(), self.n, self.units, self.M,
                                                            _native.stream_ptr(self.device)), "int4_linear_grouped")


def int4_gemm(x, packed, scale, zp, group_size=128):
    """x [..., K] fp16 (any number of rows)  ->  [..., N] fp16 on the tensor cores (li4_int4_gemm):
    the prefill path, the reference's dequantize + F.linear (llama/quantize.py:143-146) in one kernel."""
    N, half_k = packed.shape
    K = half_k * 2
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous() or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    assert x.dtype == torch.float16 and K % group_size == 0
    packed, scale, zp = _check_operands(x2, packed, scale, zp)
    M = x2.shape[0]
    y = torch.empty(M, N, dtype=torch.float16, device=x.device)
    if M and N:
        rc = _native.lib().li4_int4_gemm(x2.data_ptr(), packed.data_ptr(), scale.data_ptr(), zp.data_ptr(),
                                         y.data_ptr(), M, N, K, group_size, x2.stride(0), packed.stride(0),
                                         scale.stride(0), y.stride(0), _native.stream_ptr(x.device))
        _native.check(rc, "int4_gemm")
    return y.reshape(*lead, N)


# ---------------------------------------------------------------------------
# The kernel as a PyTorch operator (li4::int4_linear), with a shape-only fake kernel, so that
# torch.compile / fake-tensor tracing pass through QuantizedLinear.forward without a graph break.
# Eager callers keep the direct path above (no dispatcher overhead per call).
# ---------------------------------------------------------------------------
def _registered(name: str) -> bool:
    try:
        getattr(torch.ops.li4, name)
        return True
    except (AttributeError, RuntimeError):
        return False


# This file may be loaded twice (imported as llama.int4_gemv and by file path from quantize.py):
# the operators are registered by whichever load comes first.
if not _registered("int4_linear"):
    @torch.library.custom_op("li4::int4_linear", mutates_args=())
    def int4_linear_op(x: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, zp: torch.Tensor,
                       group_size: int) -> torch.Tensor:
        """int4_linear as an operator (decode sizes, prod(x.shape[:-1]) <= MAX_M)."""
        return int4_linear(x, packed, scale, zp, group_size)

    @int4_linear_op.register_fake
    def _(x, packed, scale, zp, group_size):
        torch._check(x.shape[-1] == packed.shape[1] * 2, lambda: "int4_linear: x's last dim must be 2 * packed.shape[1]")
        return x.new_empty(*x.shape[:-1], packed.shape[0])

if not _registered("int4_gemm"):
    @torch.library.custom_op("li4::int4_gemm", mutates_args=())
    def int4_gemm_op(x: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, zp: torch.Tensor,
                     group_size: int) -> torch.Tensor:
        """int4_gemm as an operator (any number of rows)."""
        return int4_gemm(x, packed, scale, zp, group_size)

    @int4_gemm_op.register_fake
    def _(x, packed, scale, zp, group_size):
        torch._check(x.shape[-1] == packed.shape[1] * 2, lambda: "int4_gemm: x's last dim must be 2 * packed.shape[1]")
        return x.new_empty(*x.shape[:-1], packed.shape[0])


def reserve_workspace(device=None, nbytes: int = 16 << 20) -> None:
    """Allocate the per-device split-K workspace ahead of CUDA-graph capture."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    _native.workspace(dev, nbytes)
