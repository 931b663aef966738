"""The allocation-free decode GEMV, li4_int4_linear_noalloc, against li4_int4_linear.

Callers that cannot allocate device memory at call time -- code running while a CUDA
graph is captured, allocators that refuse new allocations after warm-up, hosts that
bind only the C ABI -- use li4_int4_linear_noalloc, whose split-K scratch is a static
device array inside the library instead of a caller-provided workspace.  These tests
call it through the C ABI on shapes that do and do not need the scratch, twice in a
row (the second call sees the array as the first left it), compare each result bit
for bit with the workspace entry point (same plan, same fixed reduction order) and
with the oracle within the acceptance bound of the parity tests, 2e-3 * max|y|.
The file is named to run last.
"""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

SHAPES = [  # (M, N, K, uses the scratch)
    (4, 3000, 8192, True),    # a ragged K = 8192 linear at batch 4: two K ranges reduced by the last-arriving CTA
    (4, 2048, 8192, False),   # down_proj at batch 4: the shared-memory ring, one K range, no scratch
    (8, 2048, 8192, True),    # down_proj at batch 8: four K ranges
    (16, 2048, 8192, True),   # down_proj at batch 16
    (1, 512, 2048, False),    # k_proj / v_proj at batch 1: one K range, no scratch
]


@pytest.fixture(scope="module")
def native(cuda_device):
    from llama import _native

    return _native


def quantized(N, K, device, seed):
    """INT4 weights from the oracle's quantizer (host copies kept for the oracle's product)."""
    gen = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, K, generator=gen) * 0.02).half()
    packed, scale, zero = oracle.quantize(w.numpy(), 128)
    dev = torch.device(device)
    return (torch.from_numpy(packed).to(dev), torch.from_numpy(scale).to(dev), torch.from_numpy(zero).to(dev),
            (packed, scale, zero))


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


@pytest.mark.parametrize("M,N,K,scratch", SHAPES)
def test_noalloc_matches_workspace_entry_point(native, cuda_device, M, N, K, scratch):
    """Same launch plan, same kernels, same fixed reduction order: the allocation-free call gives the
    workspace call's output bit for bit, and both meet the parity bound against the oracle."""
    p, s, z, host = quantized(N, K, cuda_device, seed=N + K + M)
    assert (native.plan(M, N, K)["split"] > 1) == scratch  # split-K: the scratch holds partials and counters
    for call in range(2):  # two calls in a row share the static scratch
        gen = torch.Generator().manual_seed(100 * call + M)
        xh = torch.randn(M, K, generator=gen).half()
        x = xh.to(cuda_device)
        y_na = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda_device)
        y_ws = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
        call_noalloc(native, x, p, s, z, y_na)
        call_workspace(native, x, p, s, z, y_ws)
        torch.cuda.synchronize()
        assert torch.equal(y_na.view(torch.int16), y_ws.view(torch.int16)), f"call {call}: outputs differ"
        y_ref, _ = oracle.linear(xh.numpy(), *host)
        err = np.abs(y_na.float().cpu().numpy() - y_ref.astype(np.float32)).max()
        assert err <= oracle.tolerance(y_ref), f"call {call}: max|y - y_ref| = {err:.3e}"


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
