"""The tensor-core INT4 GEMM (li4_int4_gemm, the prefill path for M > 16) against the reference's
dequantize + F.linear.

The kernel rebuilds the reference's fp16 weights fp16((q - zero) * scale) bit for bit in shared memory and
accumulates in fp32 on the tensor cores, so y differs from the exact sums over those weights only by the
fp32 accumulation and the fp16 output rounding.  Checked against the oracle (the reference's v1 dequantize
restated in C, exact sums) at the small sizes, and against a plain PyTorch fp32 product of the exact fp16
weights (li4_dequantize, bit-exact against the golden fixtures) at prefill sizes, under the parity
acceptance bound max|y - y_ref| <= 2e-3 * max|y_ref| and a per-output bound
    |y - y_ref| <= 2^-11 |y_ref| + 2^-14 sum|W16||x|.
"""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def g(cuda_device):
    from llama import _native, int4_gemv
    from llama.quantize import QuantizedLinear

    return int4_gemv, _native, QuantizedLinear


def quantized(N, K, seed, device):
    gen = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, K, generator=gen) * 0.02).half()
    packed, scale, zero = oracle.quantize(w.numpy(), 128)
    return (torch.from_numpy(packed).to(device), torch.from_numpy(scale).to(device), torch.from_numpy(zero).to(device),
            (packed, scale, zero))


def check(y, y_ref, w16_abs, x_abs):
    y = y.float()
    err = (y - y_ref).abs()
    assert float(err.max()) <= 2e-3 * float(y_ref.abs().max()), f"max err {float(err.max()):.3e}"
    bound = 2.0 ** -11 * y_ref.abs() + 2.0 ** -14 * (x_abs @ w16_abs.T)
    excess = float((err - bound).max())
    assert excess <= 0, f"per-output bound exceeded by {excess:.3e}"


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (17, 512, 2048), (33, 300, 1024), (100, 2048, 2048),
                                   (5, 1000, 256), (16, 2048, 8192)])
def test_gemm_matches_oracle(M, N, K, g, cuda_device):
    int4_gemv, native, _ = g
    p, s, z, host = quantized(N, K, M + N + K, cuda_device)
    gen = torch.Generator().manual_seed(M * 7 + 1)
    xh = torch.randn(M, K, generator=gen).half()
    y = int4_gemv.int4_gemm(xh.to(cuda_device), p, s, z, 128)
    torch.cuda.synchronize()
    y_ref, y32 = oracle.linear(xh.numpy(), *host)
    w16 = torch.from_numpy(oracle.dequantize(*host, 128).astype(np.float32)).abs()
    check(y.cpu(), torch.from_numpy(y32.astype(np.float32)), w16, xh.float().abs())
    assert native.device_errors() == 0


@pytest.mark.parametrize("M", [512, 4096, 8192])
@pytest.mark.parametrize("N,K", [(2048, 2048), (512, 2048), (8192, 2048), (2048, 8192)])
def test_gemm_prefill_sizes(M, N, K, g, cuda_device):
    """Prefill sizes of Llama-3.2-1B at batch 1 / 8 / 16 (512-token prompts), against torch fp32 on the exact
    fp16 weights; deterministic."""
    int4_gemv, native, QL = g
    gen = torch.Generator(device=cuda_device).manual_seed(N + K + M)
    w = (torch.randn(N, K, generator=gen, device=cuda_device) * 0.02).half()
    p, s, z = QL.quantize_tensor(w, 128)
    x = torch.randn(M, K, generator=gen, device=cuda_device).half()
    y = int4_gemv.int4_gemm(x, p, s, z, 128)
    w16 = QL.dequantize_packed(p, s, z, 128).float()
    y_ref = x.float() @ w16.T
    check(y, y_ref, w16.abs(), x.float().abs())
    y2 = int4_gemv.int4_gemm(x, p, s, z, 128)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))
    assert native.device_errors() == 0


def test_gemm_strided_and_lm_head_tile(g, cuda_device):
    """Row strides above the row length on every operand, and the lm_head's N (1002 feature tiles)."""
    int4_gemv, native, QL = g
    M, N, K = 40, 128256, 2048
    gen = torch.Generator(device=cuda_device).manual_seed(5)
    w = (torch.randn(N, K, generator=gen, device=cuda_device) * 0.02).half()
    p, s, z = QL.quantize_tensor(w, 128)
    xbig = torch.randn(M, K + 64, generator=gen, device=cuda_device).half()
    x = xbig[:, :K]
    y = torch.empty(M, N + 8, dtype=torch.float16, device=cuda_device)
    rc = native.lib().li4_int4_gemm(x.data_ptr(), p.data_ptr(), s.data_ptr(), z.data_ptr(), y.data_ptr(), M, N, K,
                                    128, x.stride(0), p.stride(0), s.stride(0), y.stride(0),
                                    native.stream_ptr(cuda_device))
    native.check(rc, "int4_gemm")
    w16 = QL.dequantize_packed(p, s, z, 128).float()
    y_ref = x.float() @ w16.T
    check(y[:, :N], y_ref, w16.abs(), x.float().abs())
    assert native.device_errors() == 0


def test_quantized_linear_prefill_routes_to_gemm(g, cuda_device):
    """QuantizedLinear.forward with the v4 implementation and set_prefill_gemm(True): M > 16 on the
    tensor-core GEMM, in agreement with the reference's dequantize + F.linear (the v1 path)."""
    _, _, QL = g
    from llama import quantize

    lin = torch.nn.Linear(2048, 1024, bias=False).to(cuda_device).half()
    with torch.no_grad():
        lin.weight.normal_(0, 0.02)
    ql = QL.from_linear(lin, 128).to(cuda_device)
    x = torch.randn(2, 300, 2048, device=cuda_device).half()
    old, old_gemm = quantize.DEQUANT_IMPL, quantize.PREFILL_GEMM
    try:
        quantize.set_dequant_impl("v1")
        y1 = ql(x)
        quantize.set_dequant_impl("v4")
        quantize.set_prefill_gemm(True)
        y4 = ql(x)
    finally:
        quantize.set_dequant_impl(old)
        quantize.set_prefill_gemm(old_gemm)
    assert y4.shape == y1.shape
    assert float((y4.float() - y1.float()).abs().max()) <= 2e-3 * float(y1.float().abs().max())


def test_compiled_forward_runs_the_operators(g, cuda_device):
    """torch.compile(fullgraph=True) of QuantizedLinear.forward traces through li4::int4_linear (decode) and
    li4::int4_gemm (prefill) with no graph break, and gives the eager results."""
    _, _, QL = g
    from llama import quantize

    lin = torch.nn.Linear(2048, 512, bias=False).to(cuda_device).half()
    with torch.no_grad():
        lin.weight.normal_(0, 0.02)
    ql = QL.from_linear(lin, 128).to(cuda_device)
    old, old_gemm = quantize.DEQUANT_IMPL, quantize.PREFILL_GEMM
    try:
        quantize.set_dequant_impl("v4")
        quantize.set_prefill_gemm(True)
        compiled = torch.compile(ql.forward, fullgraph=True, backend="aot_eager")
        for rows in (3, 100):
            x = torch.randn(rows, 2048, device=cuda_device).half()
            assert torch.equal(compiled(x), ql(x))
    finally:
        quantize.set_dequant_impl(old)
        quantize.set_prefill_gemm(old_gemm)
