"""CUDA quantize / dequantize against the reference's outputs, bit for bit.

quantize_tensor (llama/quantize.py:44-75) and dequantize_packed (:78-104)
run as CUDA kernels through the C-ABI; the golden fixtures are the
reference's own outputs on the same seeded inputs.
"""
import numpy as np
import pytest
import torch

import cases
from oracle import oracle

pytestmark = pytest.mark.gpu


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy()


@pytest.fixture(scope="module")
def QL(cuda_device):
    from llama.quantize import QuantizedLinear

    return QuantizedLinear


@pytest.mark.parametrize("case", cases.QUANT_CASES, ids=[c[0] for c in cases.QUANT_CASES])
def test_quantize_bits_match_reference(case, golden, QL, cuda_device):
    meta, arr = golden
    name, N, K, group = case[:4]
    w = cases.make_quant_input(case).to(cuda_device)
    p, s, z = QL.quantize_tensor(w, group)
    assert p.is_cuda and p.dtype == torch.uint8 and s.dtype == torch.float16
    assert np.array_equal(p.cpu().numpy(), arr[f"quant/{name}/packed"])
    assert np.array_equal(bits16(s), arr[f"quant/{name}/scale"].view(np.int16))
    assert np.array_equal(bits16(z), arr[f"quant/{name}/zero"].view(np.int16))
    w16 = QL.dequantize_packed(p, s, z, group)
    assert np.array_equal(bits16(w16), arr[f"quant/{name}/w16"].view(np.int16))


@pytest.mark.parametrize("case", cases.GEMV_CASES, ids=[c[0] for c in cases.GEMV_CASES])
def test_quantize_and_dequantize_hashes(case, golden, QL, cuda_device):
    meta, arr = golden
    name, N, K, M, group = case[:5]
    info = meta["gemv"][name]
    w, _ = cases.make_gemv_inputs(case)
    p, s, z = QL.quantize_tensor(w.to(cuda_device), group)
    assert cases.sha256(p.cpu().numpy()) == info["sha256"]["packed"]
    assert cases.sha256(s.cpu().numpy()) == info["sha256"]["scale"]
    assert cases.sha256(z.cpu().numpy()) == info["sha256"]["zero"]
    w16 = QL.dequantize_packed(p, s, z, group)
    assert cases.sha256(w16.cpu().numpy()) == info["sha256"]["w16"]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_quantize_other_input_dtypes(dtype, QL, cuda_device):
    w = (torch.randn(64, 512, generator=torch.Generator().manual_seed(5)) * 0.05).to(dtype)
    p, s, z = QL.quantize_tensor(w.to(cuda_device), 128)
    # the oracle restates weight.float() for any input dtype
    po, so, zo = oracle.quantize(w.float().numpy(), 128)
    assert np.array_equal(p.cpu().numpy(), po)
    assert np.array_equal(bits16(s), so.view(np.int16))
    assert np.array_equal(bits16(z), zo.view(np.int16))


def test_quantize_cpu_tensor_round_trips_through_gpu(QL, cuda_device):
    w = (torch.randn(32, 256, generator=torch.Generator().manual_seed(6)) * 0.02).half()
    p, s, z = QL.quantize_tensor(w, 128)
    assert p.device.type == "cpu"
    po, so, zo = oracle.quantize(w.numpy(), 128)
    assert np.array_equal(p.numpy(), po) and np.array_equal(s.numpy().view(np.int16), so.view(np.int16))


@pytest.mark.parametrize("N,K,group", [(7, 100, 10), (5, 96, 32), (3, 64, 2)])
def test_dequantize_scalar_path(N, K, group, QL, cuda_device):
    """Shapes the vectorised kernel does not take (K % 32 != 0, tiny groups)."""
    gen = torch.Generator().manual_seed(N * K)
    w = (torch.randn(N, K, generator=gen) * 0.02).half()
    po, so, zo = oracle.quantize(w.numpy(), group)
    w16 = QL.dequantize_packed(torch.from_numpy(po).to(cuda_device), torch.from_numpy(so).to(cuda_device),
                               torch.from_numpy(zo).to(cuda_device), group)
    ref = oracle.dequantize(po, so, zo, group)
    assert np.array_equal(bits16(w16), ref.view(np.int16))


def test_dequantize_strided_views(QL, cuda_device):
    """Row-strided views of wider buffers (column shards of a row-parallel layer)."""
    gen = torch.Generator().manual_seed(8)
    w = (torch.randn(64, 1024, generator=gen) * 0.02).half()
    po, so, zo = oracle.quantize(w.numpy(), 128)
    p = torch.from_numpy(po).to(cuda_device)[:, 128:384]  # k in [256, 768)
    s = torch.from_numpy(so).to(cuda_device)[:, 2:6]
    z = torch.from_numpy(zo).to(cuda_device)[:, 2:6]
    w16 = QL.dequantize_packed(p, s, z, 128)
    ref = oracle.dequantize(po, so, zo, 128)[:, 256:768]
    assert np.array_equal(bits16(w16), np.ascontiguousarray(ref).view(np.int16))
