"""The allocation-free decode GEMV, li4_int4_linear_noalloc, against li4_int4_linear.

Callers that cannot allocate device memory at call time -- code running while a CUDA
graph is captured, allocators that refuse new allocations after warm-up, hosts that
bind only the C ABI -- use li4_int4_linear_noalloc, whose split-K scratch is a static
device array inside the library instead of a caller-provided workspace.  These tests
call it through the C ABI on shapes that do and do not need the scratch, twice in a
row (the second call sees the array as the first left it), and compare each result
with the workspace entry point within the acceptance bound of the parity tests,
2e-3 * max|y|.  The file is named to run last.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [  # (M, N, K): split-K (scratch used) unless noted
    (1, 512, 2048),  # k_proj / v_proj
    (8, 2048, 2048),  # q_proj / o_proj at M=8
    (16, 2048, 8192),  # down_proj at M=16 (K ranges of <= 2048)
    (2, 16384, 2048),  # enough row tiles: no scratch needed
]


@pytest.fixture(scope="module")
def native(cuda_device):
    from llama import _native

    return _native


def quantized(N, K, device, seed):
    from llama.quantize import QuantizedLinear

    gen = torch.Generator(device=device).manual_seed(seed)
    w = (torch.randn(N, K, generator=gen, device=device) * 0.02).half()
    return QuantizedLinear.quantize_tensor(w, 128)


def call_noalloc(native, x, p, s, z, y):
    M, K = x.shape
    N = p.shape[0]
    rc = native.lib().li4_int4_linear_noalloc(x.data_ptr(), p.data_ptr(), s.data_ptr(), z.data_ptr(), y.data_ptr(),
                                              M, N, K, 128, x.stride(0), p.stride(0), s.stride(0), y.stride(0),
                                              native.stream_ptr(x.device))
    native.check(rc, "li4_int4_linear_noalloc")


def call_workspace(native, x, p, s, z, y):
    M, K = x.shape
    N = p.shape[0]
    lib = native.lib()
    need = lib.li4_int4_linear_workspace_bytes(M, N, K, 128, 0)
    ws = native.workspace(x.device, need) if need else None
    rc = lib.li4_int4_linear(x.data_ptr(), p.data_ptr(), s.data_ptr(), z.data_ptr(), y.data_ptr(), M, N, K, 128,
                             x.stride(0), p.stride(0), s.stride(0), y.stride(0),
                             ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
                             native.stream_ptr(x.device))
    native.check(rc, "li4_int4_linear")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_noalloc_matches_workspace_entry_point(native, cuda_device, M, N, K):
    p, s, z = quantized(N, K, cuda_device, seed=N + K + M)
    uses_scratch = native.lib().li4_int4_linear_workspace_bytes(M, N, K, 128, 0) > 0
    assert uses_scratch == (N < 16384)
    for call in range(2):  # two calls in a row share the static scratch
        gen = torch.Generator(device=cuda_device).manual_seed(100 * call + M)
        x = torch.randn(M, K, generator=gen, device=cuda_device).half()
        y_na = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda_device)
        y_ws = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
        call_noalloc(native, x, p, s, z, y_na)
        call_workspace(native, x, p, s, z, y_ws)
        torch.cuda.synchronize()
        a, b = y_na.float().cpu().numpy(), y_ws.float().cpu().numpy()
        assert np.isfinite(a).all()
        assert np.abs(a - b).max() <= 2e-3 * np.abs(b).max()


def test_noalloc_rejects_problems_beyond_the_scratch(native, cuda_device):
    M, N, K = 16, 32768, 8192  # 4 K ranges x 16 x 32768 fp32 partials = 8 MiB > 4 MiB
    lib = native.lib()
    assert lib.li4_int4_linear_workspace_bytes(M, N, K, 128, 0) > (4 << 20)
    x = torch.zeros(M, K, dtype=torch.float16, device=cuda_device)
    p = torch.zeros(N, K // 2, dtype=torch.uint8, device=cuda_device)
    s = torch.zeros(N, K // 128, dtype=torch.float16, device=cuda_device)
    y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    rc = lib.li4_int4_linear_noalloc(x.data_ptr(), p.data_ptr(), s.data_ptr(), s.data_ptr(), y.data_ptr(), M, N, K,
                                     128, K, K // 2, K // 128, N, native.stream_ptr(cuda_device))
    assert rc == native.LI4_ERR_WORKSPACE
    assert "static scratch" in native.last_error()
