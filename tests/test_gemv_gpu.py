"""Fused INT4 GEMV on the GPU against the oracle and the reference's outputs.

The acceptance bound is the one the reference's kernel is held to:
    max|y - y_ref| <= 2e-3 * max|y_ref|
where y_ref is the reference's dequantize-to-fp16 + matmul (golden
fixtures) or the oracle's restatement of it.  Every call goes through the
C-ABI (li4_int4_linear / li4_int4_linear_ex) from the int4_linear mirror.
"""
import ctypes

import numpy as np
import pytest
import torch

import cases
from oracle import oracle

pytestmark = pytest.mark.gpu

LLAMA_SHAPES = [  # (name, N = out_features, K = in_features)
    ("q_proj", 2048, 2048), ("k_proj", 512, 2048), ("v_proj", 512, 2048), ("o_proj", 2048, 2048),
    ("gate_proj", 8192, 2048), ("up_proj", 8192, 2048), ("down_proj", 2048, 8192), ("lm_head", 128256, 2048),
]
KERNELS = {"auto": 0, "cuda_core": 1, "mma": 2, "stream": 3, "tile": 4, "bulk": 5, "slab": 6, "rows": 7, "ring": 8}


def sm_count() -> int:
    return torch.cuda.get_device_properties(0).multi_processor_count


def slab_fits(M: int, N: int, K: int, group: int = 128, split: int = 0, max_ctas: int = 0) -> bool:
    """The slab kernel's planning rule (li4_gemv.cu slab_shape): the staged x within 32 KiB (64 KiB at M > 8)
    per K range, at most one CTA per SM per K range, <= 16 resident row tiles and <= 200 KiB per CTA."""
    if group != 128 or K <= 0 or K % 128:
        return False
    n_ks, nt = K // 128, (1 if M <= 8 else 2)
    m8 = M if nt == 1 else 8
    x_cap = 32768 if nt == 1 else 65536
    if split > 0:
        if n_ks % split:
            return False
    else:
        split = 1
        while (n_ks // split) * nt * m8 * 256 > x_cap and n_ks % (2 * split) == 0:
            split *= 2
        if (n_ks // split) * nt * m8 * 256 > x_cap:
            return False
    ks = n_ks // split
    n_tiles = (N + 15) // 16
    gx = max(1, sm_count() // split)
    if max_ctas > 0:
        gx = max(1, min(gx, max_ctas // split))
    gx = min(gx, n_tiles)
    tiles = -(-n_tiles // gx)
    slots = 1
    while slots < 8 and ks % (2 * slots) == 0:
        slots *= 2
    pitch = ks * 64 + 64
    stage = (16 * pitch + 64 * ks + 127) & ~127
    smem = 128 + tiles * stage + ks * nt * m8 * 256 + tiles * slots * 16 * M * 4
    return tiles <= 16 and smem <= 200 * 1024


def ring_fits(M: int, K: int, rows: int = 0) -> bool:
    """The ring kernel's planning rule (li4_gemv.cu ring_shape): group 128, M <= 8, K a multiple of 1024
    with M x K fp16 within 64 KiB, 16 / 32 / 64-row stages whose ksteps split over the 16 consumer warps,
    and two stages beside the staged x, the warp partials and the mbarriers within 227 KiB."""
    if M > 8 or K <= 0 or K % 1024 or M * K * 2 > 65536 or rows % 16:
        return False
    ks = K // 128

    def fits(T):
        if T not in (1, 2, 4) or (ks * T) % 16:
            return False
        pitch = ks * 64 + 64
        stage = (16 * T * pitch + 64 * T * ks + 127) & ~127
        fixed = ((ks * M * 256 + 127) & ~127) + 2 * 16 * 16 * M * 4 + 2 * 8 * 8
        return fixed + 2 * stage <= 227 * 1024

    return fits(rows // 16) if rows else any(fits(t) for t in (4, 2, 1))


def supported(kernel: str, M: int, group: int = 128, K: int = 2048, N: int = 300) -> bool:
    """Which forced kernel families take the problem."""
    if kernel == "slab":
        return slab_fits(M, N, K, group)
    if kernel == "rows":
        return M == 1 and group == 128 and K in (1024, 2048)
    if kernel == "cuda_core":
        return M <= 8
    if kernel == "stream":
        return group >= 128 and K > 0
    if kernel == "tile":
        return group == 128 and K > 0 and K % 2048 == 0
    if kernel == "bulk":
        return group == 128 and K > 0 and K % 1024 == 0
    if kernel == "ring":
        return group == 128 and ring_fits(M, K)
    return True


@pytest.fixture(scope="module")
def g(cuda_device):
    from llama import int4_gemv, _native

    return int4_gemv, _native


def make_problem(N, K, M, group=128, seed=0, device="cuda", x_scale=1.0):
    gen = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, K, generator=gen) * 0.02).half()
    x = (torch.randn(M, K, generator=gen) * x_scale).half()
    packed, scale, zero = oracle.quantize(w.numpy(), group)
    dev = torch.device(device)
    return (x.to(dev), torch.from_numpy(packed).to(dev), torch.from_numpy(scale).to(dev),
            torch.from_numpy(zero).to(dev), (x.numpy(), packed, scale, zero))


def check_close(y_gpu: torch.Tensor, y_ref: np.ndarray, y32: np.ndarray = None, host=None, group: int = 128):
    """Acceptance bound against y_ref; with the operands (`host`) also a per-output bound against
    the exact sums y32 = sum_k W16 x (W16 = the reference's fp16 weights):
      |y - y32| <= 2^-11 |y32|              fp16 output rounding
                 + (2^-11 + 2^-14) sum|W16||x|  weights not rounded to fp16 + fp32 accumulation
                 + 2^-24 (1 + sum|x|)          fp16-subnormal weights
    """
    y = y_gpu.float().cpu().numpy()
    ref = y_ref.astype(np.float32)
    err = np.abs(y - ref).max()
    tol = oracle.tolerance(y_ref)
    assert err <= tol, f"max|y - y_ref| = {err:.3e} > {tol:.3e}"
    if y32 is not None and host is not None:
        x, packed, scale, zero = host
        w16 = np.abs(oracle.dequantize(packed, scale, zero, group).astype(np.float32))
        ax = np.abs(x.astype(np.float32))
        mag = (ax @ w16.T).astype(np.float64)
        bound = 2.0 ** -11 * np.abs(y32) + (2.0 ** -11 + 2.0 ** -14) * mag + 2.0 ** -24 * (1 + ax.sum(1, keepdims=True))
        excess = np.abs(y.astype(np.float64) - y32) - bound
        assert excess.max() <= 0, f"per-output bound exceeded by {excess.max():.3e} at {np.unravel_index(excess.argmax(), excess.shape)}"


@pytest.mark.parametrize("kernel", list(KERNELS))
@pytest.mark.parametrize("case", cases.GEMV_CASES, ids=[c[0] for c in cases.GEMV_CASES])
def test_golden_cases(case, kernel, golden, g, cuda_device):
    int4_gemv, _ = g
    meta, arr = golden
    name, N, K, M, group = case[:5]
    if not supported(kernel, M, group, K, N):
        pytest.skip(f"{kernel} does not take M={M} N={N} group={group} K={K}")
    w, x = cases.make_gemv_inputs(case)
    packed, scale, zero = oracle.quantize(w.numpy(), group)
    dev = cuda_device
    xg = x.to(dev)
    y = torch.empty(M, N, dtype=torch.float16, device=dev)
    int4_gemv.int4_linear_out(xg, torch.from_numpy(packed).to(dev), torch.from_numpy(scale).to(dev),
                              torch.from_numpy(zero).to(dev), y, group, kernel=KERNELS[kernel])
    check_close(y, arr[f"gemv/{name}/y"], arr[f"gemv/{name}/y32"].astype(np.float64),
                (x.numpy(), packed, scale, zero), group)


@pytest.mark.parametrize("M", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("shape", LLAMA_SHAPES, ids=[s[0] for s in LLAMA_SHAPES])
def test_llama_shapes(shape, M, g, cuda_device):
    int4_gemv, _ = g
    name, N, K = shape
    x, p, s, z, host = make_problem(N, K, M, seed=sum(map(ord, name)) + M)
    y_ref, y32 = oracle.linear(*host)
    for kernel in KERNELS:
        if not supported(kernel, M, 128, K, N):
            continue
        y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
        int4_gemv.int4_linear_out(x, p, s, z, y, 128, kernel=KERNELS[kernel])
        check_close(y, y_ref, y32, host)


@pytest.mark.parametrize("M", [1, 3, 8, 11, 16])
@pytest.mark.parametrize("N,K", [(1, 128), (7, 256), (16, 128), (31, 1152), (100, 2048), (1000, 512), (5000, 4096),
                                 (257, 8192)])
def test_shape_sweep(N, K, M, g, cuda_device):
    int4_gemv, _ = g
    x, p, s, z, host = make_problem(N, K, M, seed=N * 31 + K + M)
    y_ref, y32 = oracle.linear(*host)
    y = int4_gemv.int4_linear(x, p, s, z, 128)
    check_close(y, y_ref, y32, host)


@pytest.mark.parametrize("group", [32, 64, 256, 512])
@pytest.mark.parametrize("M", [1, 5, 16])
def test_group_sizes(group, M, g, cuda_device):
    int4_gemv, _ = g
    x, p, s, z, host = make_problem(300, 2048, M, group=group, seed=group + M)
    y_ref, y32 = oracle.linear(*host, group_size=group)
    for kernel in KERNELS:
        if not supported(kernel, M, group):
            continue
        y = torch.empty(M, 300, dtype=torch.float16, device=cuda_device)
        int4_gemv.int4_linear_out(x, p, s, z, y, group, kernel=KERNELS[kernel])
        check_close(y, y_ref, y32, host, group)


@pytest.mark.parametrize("kernel", ["cuda_core", "mma"])
@pytest.mark.parametrize("rows", [16, 32])
@pytest.mark.parametrize("split", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("max_ctas", [0, 1, 5])
def test_forced_launch_shapes(kernel, rows, split, max_ctas, g, cuda_device):
    """Every split-K / tile / persistent-grid combination gives the same answer, deterministically."""
    int4_gemv, _ = g
    M, N, K = 3, 700, 2048
    x, p, s, z, host = make_problem(N, K, M, seed=99)
    y_ref, y32 = oracle.linear(*host)
    y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    int4_gemv.int4_linear_out(x, p, s, z, y, 128, kernel=KERNELS[kernel], rows_per_cta=rows, split=split,
                              max_ctas=max_ctas)
    check_close(y, y_ref, y32, host)
    y2 = torch.empty_like(y)
    int4_gemv.int4_linear_out(x, p, s, z, y2, 128, kernel=KERNELS[kernel], rows_per_cta=rows, split=split,
                              max_ctas=max_ctas)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16)), "split-K result is not deterministic"


@pytest.mark.parametrize("M", [1, 3, 9, 16])
@pytest.mark.parametrize("split", [0, 1, 2, 4, 8, 16])
@pytest.mark.parametrize("max_ctas", [0, 1, 5])
@pytest.mark.parametrize("N", [700, 4100, 20000])
def test_stream_launch_shapes(M, split, max_ctas, N, g, cuda_device):
    """Streaming-warp kernel: rows mode (many tiles) and K-split mode (few), split-K, short grids (each warp
    walks many tiles, the register ring runs across tile boundaries), a partial last tile; deterministic."""
    int4_gemv, _ = g
    K = 2048
    x, p, s, z, host = make_problem(N, K, M, seed=N + M + split + max_ctas)
    y_ref, y32 = oracle.linear(*host)
    y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    int4_gemv.int4_linear_out(x, p, s, z, y, 128, kernel=KERNELS["stream"], split=split, max_ctas=max_ctas)
    check_close(y, y_ref, y32, host)
    y2 = torch.empty_like(y)
    int4_gemv.int4_linear_out(x, p, s, z, y2, 128, kernel=KERNELS["stream"], split=split, max_ctas=max_ctas)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))


@pytest.mark.parametrize("M", [1, 2, 4])
@pytest.mark.parametrize("split", [0, 1, 2])
@pytest.mark.parametrize("N", [700, 2048])
def test_stream_long_k_ranges(M, split, N, g, cuda_device):
    """Streaming warps with K ranges above 2048 (x staged for up to 8192 k when M is small): down_proj's
    K=8192 in one or two ranges, in K-split mode."""
    int4_gemv, _ = g
    K = 8192
    if split == 1 and M > 2:
        pytest.skip("x for M > 2 over 8192 k exceeds the 32 KiB staging limit")
    x, p, s, z, host = make_problem(N, K, M, seed=7 * N + M + split)
    y_ref, y32 = oracle.linear(*host)
    y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    int4_gemv.int4_linear_out(x, p, s, z, y, 128, kernel=KERNELS["stream"], split=split)
    check_close(y, y_ref, y32, host)


@pytest.mark.parametrize("M", [1, 5, 9, 16])
@pytest.mark.parametrize("rows", [16, 32])
@pytest.mark.parametrize("max_ctas", [0, 1, 3])
@pytest.mark.parametrize("N,K", [(17, 2048), (300, 4096), (4100, 2048), (20000, 2048), (2049, 8192)])
def test_tile_launch_shapes(M, rows, max_ctas, N, K, g, cuda_device):
    """Tile-streaming kernel: 16- and 32-row warp tiles, K ranges of 2048 (split-K above), short grids (each
    warp walks many tiles and prefetches the next one), partial last tiles; deterministic.  N >= 17: with a
    single output the 2e-3 * max|y_ref| bound is a bound on one near-cancelling sum, which fp32 sums of the
    unrounded weights need not meet (the per-output bound holds there; the shape sweep checks N=1)."""
    int4_gemv, _ = g
    x, p, s, z, host = make_problem(N, K, M, seed=N + K + M + rows + max_ctas)
    y_ref, y32 = oracle.linear(*host)
    y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    int4_gemv.int4_linear_out(x, p, s, z, y, 128, kernel=KERNELS["tile"], rows_per_cta=rows, max_ctas=max_ctas)
    check_close(y, y_ref, y32, host)
    y2 = torch.empty_like(y)
    int4_gemv.int4_linear_out(x, p, s, z, y2, 128, kernel=KERNELS["tile"], rows_per_cta=rows, max_ctas=max_ctas)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))


@pytest.mark.parametrize("M", [1, 5, 9, 16])
@pytest.mark.parametrize("split", [0, 1, 2, 4, 8])
@pytest.mark.parametrize("max_ctas", [0, 1, 7])
@pytest.mark.parametrize("N,K", [(17, 2048), (300, 4096), (4100, 2048), (20000, 2048), (2049, 8192), (512, 1024)])
def test_bulk_launch_shapes(M, split, max_ctas, N, K, g, cuda_device):
    """Bulk-copy ring kernel: K ranges of 8 and 16 ksteps (split-K above), one to many tiles per CTA (the
    ring wraps around its stages), partial last tiles; deterministic, and no device-side wait ran out."""
    int4_gemv, native = g
    n_ks = K // 128
    if split and (n_ks % split or n_ks // split not in (8, 16)):
        pytest.skip("the bulk kernel takes K ranges of 8 or 16 ksteps")
    x, p, s, z, host = make_problem(N, K, M, seed=N + K + M + split + max_ctas)
    y_ref, y32 = oracle.linear(*host)
    y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    int4_gemv.int4_linear_out(x, p, s, z, y, 128, kernel=KERNELS["bulk"], split=split, max_ctas=max_ctas)
    check_close(y, y_ref, y32, host)
    y2 = torch.empty_like(y)
    int4_gemv.int4_linear_out(x, p, s, z, y2, 128, kernel=KERNELS["bulk"], split=split, max_ctas=max_ctas)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))
    assert native.device_errors() == 0


@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("rows", [0, 16, 32, 64])
@pytest.mark.parametrize("max_ctas", [0, 1, 5])
@pytest.mark.parametrize("N,K", [(17, 2048), (300, 1024), (4100, 2048), (20000, 2048), (2049, 8192), (40, 4096)])
def test_ring_launch_shapes(M, rows, max_ctas, N, K, g, cuda_device):
    """Ring kernel: 16-, 32- and 64-row stages (consumer warps sharing a tile's ksteps 16, 8 or 4 ways),
    one to many stage units per CTA (short grids wrap the ring around its stages many times), partial last
    tiles and stage units, K from 1024 to 8192; deterministic, and no device-side wait ran out."""
    int4_gemv, native = g
    if not ring_fits(M, K, rows):
        pytest.skip("x above the 64 KiB staging, a consumer warp without a kstep, or two stages beyond 227 KiB")
    x, p, s, z, host = make_problem(N, K, M, seed=N + K + M + rows + max_ctas)
    y_ref, y32 = oracle.linear(*host)
    y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    int4_gemv.int4_linear_out(x, p, s, z, y, 128, kernel=KERNELS["ring"], rows_per_cta=rows, max_ctas=max_ctas)
    check_close(y, y_ref, y32, host)
    y2 = torch.empty_like(y)
    int4_gemv.int4_linear_out(x, p, s, z, y2, 128, kernel=KERNELS["ring"], rows_per_cta=rows, max_ctas=max_ctas)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))
    assert native.device_errors() == 0


@pytest.mark.parametrize("M", [1, 4])
@pytest.mark.parametrize("rows", [16, 64])
@pytest.mark.parametrize("N,K", [(300, 2048), (2049, 8192)])
def test_ring_strided_rows(M, rows, N, K, g, cuda_device):
    """Ring kernel on packed / scale / zero rows with padded row strides: the per-row copies into padded
    shared-memory rows instead of the three block copies of contiguous tensors."""
    int4_gemv, native = g
    if not ring_fits(M, K, rows):
        pytest.skip("does not fit the ring kernel")
    x, p, s, z, host = make_problem(N, K, M, seed=N + K + M + rows)
    pw = torch.zeros(N, K // 2 + 48, dtype=torch.uint8, device=cuda_device)[:, :K // 2]
    sw = torch.zeros(N, K // 128 + 8, dtype=torch.float16, device=cuda_device)[:, :K // 128]
    zw = torch.zeros_like(sw)
    pw.copy_(p), sw.copy_(s), zw.copy_(z)
    y_ref, y32 = oracle.linear(*host)
    y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    int4_gemv.int4_linear_out(x, pw, sw, zw, y, 128, kernel=KERNELS["ring"], rows_per_cta=rows)
    check_close(y, y_ref, y32, host)
    y2 = torch.empty_like(y)
    int4_gemv.int4_linear_out(x, p, s, z, y2, 128, kernel=KERNELS["ring"], rows_per_cta=rows)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16)), "strided and contiguous rows differ"
    assert native.device_errors() == 0


def test_ring_rejects_what_does_not_fit(g, cuda_device):
    """A forced ring launch outside its range (M > 8, K not a multiple of 1024, x above 64 KiB, a K split)
    fails with a clear error and launches nothing."""
    int4_gemv, native = g
    for M, N, K, kw in ((16, 512, 2048, {}), (1, 512, 1536, {}), (8, 512, 8192, {}), (1, 512, 2048, {"split": 2})):
        x, p, s, z, _ = make_problem(N, K, M, seed=M + K)
        y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
        with pytest.raises(native.Li4Error, match="ring kernel"):
            int4_gemv.int4_linear_out(x, p, s, z, y, 128, kernel=KERNELS["ring"], **kw)


@pytest.mark.parametrize("M", [1, 5, 9, 16])
@pytest.mark.parametrize("split", [0, 1, 2, 4])
@pytest.mark.parametrize("max_ctas", [0, 1, 7])
@pytest.mark.parametrize("N,K", [(17, 2048), (300, 4096), (4100, 2048), (2049, 8192), (512, 1024), (100, 640),
                                 (16384, 2048)])
def test_slab_launch_shapes(M, split, max_ctas, N, K, g, cuda_device):
    """Slab kernel: one to 16 resident row tiles per CTA, K split across 1-8 warps (K = 640: five ksteps,
    one warp per tile, scale / zero rows by plain loads), split-K across CTAs with the last range reducing,
    partial last tiles; deterministic, and no device-side wait ran out."""
    int4_gemv, native = g
    if not slab_fits(M, N, K, 128, split, max_ctas):
        pytest.skip("more resident tiles or shared memory than one slab CTA takes")
    x, p, s, z, host = make_problem(N, K, M, seed=N + K + M + split + max_ctas)
    y_ref, y32 = oracle.linear(*host)
    y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    int4_gemv.int4_linear_out(x, p, s, z, y, 128, kernel=KERNELS["slab"], split=split, max_ctas=max_ctas)
    check_close(y, y_ref, y32, host)
    y2 = torch.empty_like(y)
    int4_gemv.int4_linear_out(x, p, s, z, y2, 128, kernel=KERNELS["slab"], split=split, max_ctas=max_ctas)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))
    assert native.device_errors() == 0


@pytest.mark.parametrize("N,K", [(1, 2048), (17, 1024), (512, 2048), (2048, 2048), (3000, 1024), (4100, 2048)])
def test_rows_launch_shapes(N, K, g, cuda_device):
    """Register-rows kernel (M = 1): one partial tile, every row count modulo 16, K = 1024 / 2048;
    deterministic."""
    int4_gemv, _ = g
    x, p, s, z, host = make_problem(N, K, 1, seed=N + K)
    y_ref, y32 = oracle.linear(*host)
    y = torch.empty(1, N, dtype=torch.float16, device=cuda_device)
    int4_gemv.int4_linear_out(x, p, s, z, y, 128, kernel=KERNELS["rows"])
    check_close(y, y_ref, y32, host)
    y2 = torch.empty_like(y)
    int4_gemv.int4_linear_out(x, p, s, z, y2, 128, kernel=KERNELS["rows"])
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))


def test_rows_rejects_misaligned_x(g, cuda_device):
    """A forced register-rows launch refuses an x that is not 16-byte aligned; the dispatcher re-plans it."""
    int4_gemv, native = g
    N, K = 512, 2048
    x, p, s, z, host = make_problem(N, K, 1, seed=5)
    buf = torch.zeros(K + 8, dtype=torch.float16, device=cuda_device)
    buf[1:K + 1] = x[0]
    xm = buf[1:K + 1].view(1, K)  # 2 bytes past a 16-byte boundary
    y = torch.empty(1, N, dtype=torch.float16, device=cuda_device)
    with pytest.raises(native.Li4Error, match="register-rows"):
        int4_gemv.int4_linear_out(xm, p, s, z, y, 128, kernel=KERNELS["rows"])
    int4_gemv.int4_linear_out(xm, p, s, z, y, 128)
    y_ref, y32 = oracle.linear(*host)
    check_close(y, y_ref, y32, host)


def test_slab_rejects_what_does_not_fit(g, cuda_device):
    """A forced slab launch beyond its resident tiles (lm_head at M=1) fails with a clear error, no launch."""
    int4_gemv, native = g
    N, K, M = 128256, 2048, 1
    assert not slab_fits(M, N, K)
    x = torch.zeros(M, K, dtype=torch.float16, device=cuda_device)
    p = torch.zeros(N, K // 2, dtype=torch.uint8, device=cuda_device)
    s = torch.zeros(N, K // 128, dtype=torch.float16, device=cuda_device)
    y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    with pytest.raises(native.Li4Error, match="does not fit the slab"):
        int4_gemv.int4_linear_out(x, p, s, s, y, 128, kernel=KERNELS["slab"])


def test_slab_fits_every_layer_shape(g, cuda_device):
    """The slab kernel takes every Llama-3.2-1B layer shape at M <= 16 (not lm_head)."""
    for name, N, K in LLAMA_SHAPES:
        for M in (1, 2, 4, 8, 16):
            assert slab_fits(M, N, K) == (name != "lm_head"), (name, M)


def test_auto_dispatch_plans(g, cuda_device):
    """The dispatcher's measured choices at M = 1: streaming warps for the layer shapes, the shared-memory
    ring for down_proj, the tile kernel for lm_head (li4_int4_linear_plan reports what li4_int4_linear
    launches)."""
    from llama import _native

    want = {"lm_head": "tile", "down_proj": "ring"}
    for name, N, K in LLAMA_SHAPES:
        k = _native.plan(1, N, K)["kernel"]
        assert k == want.get(name, "stream"), (name, k)


def test_split_counters_reset_across_launches(g, cuda_device):
    """The arrival counters are left at zero: 40 back-to-back split-K launches all reduce correctly."""
    int4_gemv, _ = g
    M, N, K = 1, 512, 2048  # k/v shape: split-K on the streaming-warp kernel
    x, p, s, z, host = make_problem(N, K, M, seed=3)
    xs = [(torch.randn(M, K, generator=torch.Generator().manual_seed(i))).half() for i in range(40)]
    outs = []
    for xi in xs:
        yi = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
        int4_gemv.int4_linear_out(xi.to(cuda_device), p, s, z, yi, 128, kernel=KERNELS["stream"])
        outs.append(yi)
    torch.cuda.synchronize()
    for xi, yi in zip(xs, outs):
        y_ref, y32 = oracle.linear(xi.numpy(), *host[1:])
        check_close(yi, y_ref, y32, (xi.numpy(),) + tuple(host[1:]))


def test_workspace_shared_by_shapes_of_different_tile_counts(g, cuda_device):
    """Split-K launches of different shapes share one workspace: a launch with few row tiles
    writes partial sums where a launch with many tiles keeps arrival counters unless the
    counters have a region of their own."""
    int4_gemv, _ = g
    problems = [make_problem(N, K, M, seed=40 + i) for i, (N, K, M) in
                enumerate([(64, 8192, 4), (2048, 2048, 8), (40, 4096, 16), (2048, 2048, 8), (512, 8192, 1)])]
    for _ in range(2):
        for x, p, s, z, host in problems:
            y = int4_gemv.int4_linear(x, p, s, z, 128)
            y_ref, y32 = oracle.linear(*host)
            check_close(y, y_ref, y32, host)


def test_leading_dims_and_noncontiguous_x(g, cuda_device):
    int4_gemv, _ = g
    N, K = 96, 512
    x, p, s, z, host = make_problem(N, K, 6, seed=4)
    x3 = x.reshape(2, 3, K)
    y = int4_gemv.int4_linear(x3, p, s, z, 128)
    assert y.shape == (2, 3, N)
    y_ref, _ = oracle.linear(*host)
    check_close(y.reshape(6, N), y_ref)
    wide = torch.zeros(6, 2 * K, dtype=torch.float16, device=cuda_device)
    wide[:, :K] = x
    y2 = int4_gemv.int4_linear(wide[:, :K], p, s, z, 128)  # row stride 2K, made contiguous by the wrapper
    check_close(y2, y_ref)


def test_strided_operands_through_c_abi(g, cuda_device):
    """x, packed, scale/zero and y with row strides wider than their rows (no copies)."""
    int4_gemv, native = g
    M, N, K = 4, 200, 1024
    x, p, s, z, host = make_problem(N, K, M, seed=5)
    y_ref, y32 = oracle.linear(*host)
    dev = cuda_device
    xw = torch.zeros(M, K + 64, dtype=torch.float16, device=dev)
    xw[:, :K] = x
    pw = torch.zeros(N, K // 2 + 48, dtype=torch.uint8, device=dev)
    pw[:, :K // 2] = p
    sw = torch.zeros(N, K // 128 + 3, dtype=torch.float16, device=dev)
    zw = torch.zeros_like(sw)
    sw[:, :K // 128] = s
    zw[:, :K // 128] = z
    yw = torch.full((M, N + 40), 7.0, dtype=torch.float16, device=dev)
    lib = native.lib()
    ws = native.workspace(dev, lib.li4_int4_linear_workspace_bytes(M, N, K, 128, 0))
    for kernel in (1, 2):
        rc = lib.li4_int4_linear_ex(xw.data_ptr(), pw.data_ptr(), sw.data_ptr(), zw.data_ptr(), yw.data_ptr(),
                                    M, N, K, 128, xw.stride(0), pw.stride(0), sw.stride(0), yw.stride(0),
                                    ws.data_ptr(), ws.numel(), native.stream_ptr(dev), kernel, 0, 0, 0)
        native.check(rc)
        check_close(yw[:, :N], y_ref, y32, host)
        assert torch.all(yw[:, N:] == 7.0), "wrote past the row"


def test_misaligned_packed_is_rejected(g, cuda_device):
    int4_gemv, native = g
    x, p, s, z, _ = make_problem(64, 256, 1, seed=6)
    buf = torch.zeros(p.numel() + 16, dtype=torch.uint8, device=cuda_device)
    pv = buf[1:1 + p.numel()].view(p.shape)
    pv.copy_(p)
    with pytest.raises(native.Li4Error) as e:
        int4_gemv.int4_linear(x, pv, s, z, 128)
    assert e.value.status == native.LI4_ERR_ALIGNMENT


def test_reference_asserts(g, cuda_device):
    int4_gemv, _ = g
    x, p, s, z, _ = make_problem(64, 256, 17, seed=7)
    with pytest.raises(AssertionError):
        int4_gemv.int4_linear(x, p, s, z, 128)  # M > MAX_M
    with pytest.raises(AssertionError):
        int4_gemv.int4_linear(x[:1].float(), p, s, z, 128)  # not fp16
    with pytest.raises(AssertionError):
        int4_gemv.int4_linear(x[:1], p, s, z, 96)  # K % group_size


def test_empty_m(g, cuda_device):
    int4_gemv, _ = g
    x, p, s, z, _ = make_problem(64, 256, 1, seed=8)
    y = int4_gemv.int4_linear(x[:0], p, s, z, 128)
    assert y.shape == (0, 64)


def test_cuda_graph_capture_and_replay(g, cuda_device):
    """Static-buffer capture of several launches (one split-K) replays like eager."""
    int4_gemv, _ = g
    probs = [make_problem(N, K, M, seed=10 + i) for i, (N, K, M) in enumerate([(512, 2048, 1), (2048, 8192, 2),
                                                                               (8192, 2048, 16)])]
    xs = [pr[0].clone() for pr in probs]
    ys = [torch.empty(pr[0].shape[0], pr[1].shape[0], dtype=torch.float16, device=cuda_device) for pr in probs]
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for xi, (_, p, s, z, _), yi in zip(xs, probs, ys):  # warm-up sizes the workspace
            int4_gemv.int4_linear_out(xi, p, s, z, yi, 128)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for xi, (_, p, s, z, _), yi in zip(xs, probs, ys):
            int4_gemv.int4_linear_out(xi, p, s, z, yi, 128)
    for rep in range(3):
        for i, xi in enumerate(xs):
            xi.copy_(torch.randn(xi.shape, generator=torch.Generator().manual_seed(100 * rep + i)).half())
        graph.replay()
        torch.cuda.synchronize()
        for xi, (_, p, s, z, host), yi in zip(xs, probs, ys):
            y_ref, y32 = oracle.linear(xi.cpu().numpy(), *host[1:])
            check_close(yi, y_ref, y32, (xi.cpu().numpy(),) + tuple(host[1:]))


def test_quantized_linear_module(cuda_device):
    from llama import quantize

    lin = torch.nn.Linear(1024, 384, bias=False).half().to(cuda_device)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(384, 1024, generator=torch.Generator().manual_seed(9)).half() * 0.02)
    ql = quantize.QuantizedLinear.from_linear(lin, 128).to(cuda_device)
    assert set(ql.state_dict()) == {"packed_weight", "scale", "zero_point"}
    x = torch.randn(1, 3, 1024, generator=torch.Generator().manual_seed(10)).half().to(cuda_device)
    old = quantize.DEQUANT_IMPL
    try:
        quantize.set_dequant_impl("v4")
        y4 = ql(x)
        quantize.set_dequant_impl("v1")
        y1 = ql(x)
    finally:
        quantize.set_dequant_impl(old)
    packed, scale, zero = (t.cpu().numpy() for t in (ql.packed_weight, ql.scale, ql.zero_point))
    y_ref, y32 = oracle.linear(x.reshape(3, 1024).cpu().numpy(), packed, scale, zero)
    check_close(y4.reshape(3, 384), y_ref, y32, (x.reshape(3, 1024).cpu().numpy(), packed, scale, zero))
    check_close(y1.reshape(3, 384), y_ref)


def test_int4_linear_fn_is_path_loaded_and_patchable(cuda_device):
    from llama import quantize

    fn = quantize.int4_linear_fn()
    assert callable(fn) and fn.__name__ == "int4_linear"
    assert quantize.int4_linear_fn() is fn
