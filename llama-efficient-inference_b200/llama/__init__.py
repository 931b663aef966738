"""B200 (sm_100a) INT4 weight-only decode path for Llama 3.2-1B.

Mirrors the reference's `llama` package layout: llama.quantize (QuantizedLinear
and the quantize / dequantize functions), llama.int4_gemv (int4_linear), and
the decode model (llama.model, llama.generation).  Submodules are imported on
use.  The ctypes binding (_native.py) is one module instance whether it is
reached as llama._native or, from a file-path load of int4_gemv.py /
quantize.py, as li4_native; the kernel library itself loads on first call.
"""
import importlib.util as _ilu
import os as _os
import sys as _sys


def _native_module():
    mod = _sys.modules.get("li4_native")
    if mod is None:
        path = _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "_native.py")
        spec = _ilu.spec_from_file_location("li4_native", path)
        mod = _ilu.module_from_spec(spec)
        _sys.modules["li4_native"] = mod
        spec.loader.exec_module(mod)
    return mod


_sys.modules[__name__ + "._native"] = _native_module()
