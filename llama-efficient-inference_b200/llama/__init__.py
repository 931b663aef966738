"""B200 (sm_100a) INT4 weight-only decode path for Llama 3.2-1B.

Mirrors the reference's `llama` package layout: llama.quantize (QuantizedLinear
and the quantize / dequantize functions), llama.int4_gemv (int4_linear), and
the decode model (llama.model, llama.generation).  Submodules are imported on
use; importing the package itself loads nothing.
"""
