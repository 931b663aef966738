"""INT4 weight-only quantization for Llama 3.2-1B, B200 edition: drop-in for the
reference's llama/quantize.py.

Same module surface, buffers and state-dict keys (packed_weight, scale,
zero_point), so converted packs and checkpoints stay loadable:

    QuantizedLinear                 llama/quantize.py:14-173
    QuantizedLinear.quantize_tensor llama/quantize.py:44-75   -> li4_quantize (CUDA)
    QuantizedLinear.dequantize_packed / _v2  :78-126          -> li4_dequantize (CUDA)
    DEQUANT_IMPL / set_dequant_impl / dequant_fn  :176-203
    int4_linear_fn                           :206-216          -> int4_gemv.py, loaded by path
    quantize_model                           :219-240

Every computation runs in the CUDA kernels of libllama_int4_b200.so and is
bit-identical to the reference (quantize: packed bytes, scale and zero bits;
dequantize: fp16 weights).  CPU tensors are moved to the current CUDA device
for the computation and the results moved back; without a CUDA device these
functions raise.  DEQUANT_IMPL keeps the reference's meaning:
  v1, v2, v3  dequantize to fp16 (one CUDA kernel) + F.linear (cuBLAS)
  v4          fused INT4 GEMV kernel for M <= 16 tokens; above, as v3, or with
              set_prefill_gemm(True) the tensor-core INT4 GEMM (li4_int4_gemm, group 128)
"""
from __future__ import annotations

import importlib.util
import os
import sys

import torch
import torch.nn as nn
import torch.nn.functional as F


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

_DTYPE_CODES = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def _cuda_target(t: torch.Tensor) -> torch.device:
    if t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("the INT4 kernels need a CUDA device (none available)")
    return torch.device("cuda", torch.cuda.current_device())


class QuantizedLinear(nn.Module):
    """A linear layer that stores its weight in INT4 (two values per uint8,
    fp16 scale and zero point per group of `group_size` along in_features).
    Replaces nn.Linear."""

    def __init__(self, in_features: int, out_features: int, group_size: int = 128, bias: bool = False):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size
        self.n_groups = in_features // group_size
        self.register_buffer("packed_weight", torch.zeros(out_features, in_features // 2, dtype=torch.uint8))
        self.register_buffer("scale", torch.zeros(out_features, self.n_groups, dtype=torch.float16))
        self.register_buffer("zero_point", torch.zeros(out_features, self.n_groups, dtype=torch.float16))
        if bias:
            self.register_buffer("bias", torch.zeros(out_features, dtype=torch.float16))
        else:
            self.bias = None
        _int4_gemv()  # registers the li4:: operators that traced forwards call

    @staticmethod
    def quantize_tensor(weight: torch.Tensor, group_size: int = 128):
        """weight [out, in] (fp16 / bf16 / fp32) -> (packed uint8 [out, in/2],
        scale fp16 [out, in/group], zero_point fp16 [out, in/group])."""
        out_features, in_features = weight.shape
        assert in_features % group_size == 0, \
            f"in_features ({in_features}) must be divisible by group_size ({group_size})"
        home = weight.device
        dev = _cuda_target(weight)
        w = weight.detach()
        if w.dtype not in _DTYPE_CODES:
            w = w.float()
        w = w.to(dev)
        if w.stride(-1) != 1:
            w = w.contiguous()
        n_groups = in_features // group_size
        packed = torch.empty(out_features, in_features // 2, dtype=torch.uint8, device=dev)
        scale = torch.empty(out_features, n_groups, dtype=torch.float16, device=dev)
        zero = torch.empty(out_features, n_groups, dtype=torch.float16, device=dev)
        lib = _native.lib()
        with torch.cuda.device(dev):
            rc = lib.li4_quantize(w.data_ptr(), _DTYPE_CODES[w.dtype], packed.data_ptr(), scale.data_ptr(),
                                  zero.data_ptr(), out_features, in_features, group_size, w.stride(0),
                                  _native.stream_ptr(dev))
        _native.check(rc, "quantize_tensor")
        return packed.to(home), scale.to(home), zero.to(home)

    @staticmethod
    def dequantize_packed(packed_weight, scale, zero_point, group_size):
        """-> fp16 weight [out, in] = fp16((q - zero_point) * scale), fp32 math."""
        home = packed_weight.device
        dev = _cuda_target(packed_weight)
        out_features, half_in = packed_weight.shape
        in_features = half_in * 2
        p = packed_weight.to(dev)
        s = scale.to(dev, torch.float16)
        z = zero_point.to(dev, torch.float16)
        if p.stride(-1) != 1:
            p = p.contiguous()
        if s.stride(-1) != 1 or z.stride(-1) != 1 or s.stride(0) != z.stride(0):
            s, z = s.contiguous(), z.contiguous()
        w16 = torch.empty(out_features, in_features, dtype=torch.float16, device=dev)
        lib = _native.lib()
        with torch.cuda.device(dev):
            rc = lib.li4_dequantize(p.data_ptr(), s.data_ptr(), z.data_ptr(), w16.data_ptr(), out_features,
                                    in_features, group_size, p.stride(0), s.stride(0), w16.stride(0),
                                    _native.stream_ptr(dev))
        _native.check(rc, "dequantize_packed")
        return w16.to(home)

    # The reference's v2 is bit-identical to v1 by construction (llama/quantize.py:107-115);
    # both map to the same exact CUDA kernel here.
    dequantize_packed_v2 = dequantize_packed

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if DEQUANT_IMPL == "v4" and self.bias is None:
            compiling = torch.compiler.is_compiling()  # traced: the registered operators (li4::...)
            if x.numel() // x.shape[-1] <= 16:  # decode: the fused INT4 GEMV
                fn = torch.ops.li4.int4_linear if compiling else int4_linear_fn()
                return fn(x, self.packed_weight, self.scale, self.zero_point, self.group_size)
            if (PREFILL_GEMM and self.group_size == 128 and x.is_cuda and x.dtype == torch.float16):
                fn = torch.ops.li4.int4_gemm if compiling else int4_gemm_fn()
                return fn(x, self.packed_weight, self.scale, self.zero_point, self.group_size)
        weight = dequant_fn(DEQUANT_IMPL)(self.packed_weight, self.scale, self.zero_point, self.group_size)
        return F.linear(x, weight, self.bias)

    @classmethod
    def from_linear(cls, linear: nn.Linear, group_size: int = 128):
        has_bias = linear.bias is not None
        ql = cls(linear.in_features, linear.out_features, group_size=group_size, bias=has_bias)
        packed, scale, zp = cls.quantize_tensor(linear.weight.data, group_size)
        ql.packed_weight.copy_(packed)
        ql.scale.copy_(scale.half())
        ql.zero_point.copy_(zp.half())
        if has_bias:
            ql.bias.copy_(linear.bias.data.half())
        return ql


# Which path every QuantizedLinear uses (same names and default as the reference):
#   v1 / v2 / v3  exact CUDA dequantize kernel + F.linear
#   v4            fused INT4 GEMV kernel for M <= 16; above, as v3 or (PREFILL_GEMM) the tensor-core INT4 GEMM
DEQUANT_IMPL = "v1"
# v4 prefill (M > 16) on the tensor-core INT4 GEMM (li4_int4_gemm) instead of dequantize + F.linear;
# off by default while the GEMM measures slower than dequantize + cuBLAS (set_prefill_gemm).
PREFILL_GEMM = False
_int4_linear = None


def set_prefill_gemm(enabled: bool) -> None:
    """Route v4 prefill (M > 16, group 128, fp16 CUDA inputs) to the tensor-core INT4 GEMM."""
    global PREFILL_GEMM
    PREFILL_GEMM = bool(enabled)


def set_dequant_impl(impl: str):
    global DEQUANT_IMPL
    assert impl in ("v1", "v2", "v3", "v4"), impl
    DEQUANT_IMPL = impl


def dequant_fn(impl: str):
    if impl in ("v1", "v2", "v3", "v4"):
        return QuantizedLinear.dequantize_packed
    raise ValueError(impl)


_int4_gemv_module = None


def _int4_gemv():
    """int4_gemv.py, loaded by file path (so this also works when quantize.py itself was loaded by path)."""
    global _int4_gemv_module
    if _int4_gemv_module is None:
        spec = importlib.util.spec_from_file_location(
            "llama_int4_gemv", os.path.join(os.path.dirname(os.path.abspath(__file__)), "int4_gemv.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _int4_gemv_module = mod
    return _int4_gemv_module


def int4_linear_fn():
    """The decode kernel's entry point (cached in _int4_linear, which callers may replace)."""
    global _int4_linear
    if _int4_linear is None:
        _int4_linear = _int4_gemv().int4_linear
    return _int4_linear


def int4_gemm_fn():
    """The prefill (M > 16) tensor-core GEMM's entry point."""
    return _int4_gemv().int4_gemm


def quantize_model(model, group_size=128):
    """Replace all nn.Linear layers in the model with QuantizedLinear (in place)."""
    linear_layers = [(name, module) for name, module in model.named_modules() if isinstance(module, nn.Linear)]
    for name, module in linear_layers:
        if name == "":
            return QuantizedLinear.from_linear(module, group_size).to(module.weight.device)
        parent_name, child_name = name.rsplit(".", 1) if "." in name else ("", name)
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, child_name, QuantizedLinear.from_linear(module, group_size).to(module.weight.device))
    return model
