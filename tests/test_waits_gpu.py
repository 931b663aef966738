"""The bounded device waits run out without a fault, report it, and leave the context usable.

Four kernels here spin on memory that another agent writes: li4_allreduce_add waits for
every peer's flag, a row-parallel GEMV with the all-reduce epilogue waits for every peer's
words, li4_argmax_rows_allreduce waits for every peer's key, and a decode program's op waits
for the completion counter of the op it depends on.  Each wait gives up after a poll limit, sets its bit in li4_device_errors and
returns.  li4_debug_set_wait_limits shortens the limits so a test can make the waits run out
on one GPU, with nothing faulting or hanging: the peer is a local buffer that nobody writes,
and the program's counter target is one no op can meet.  Every test restores the defaults.
"""
import ctypes

import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

SHORT = 1 << 12  # polls: microseconds of spinning


@pytest.fixture()
def native(cuda_device):
    from llama import _native

    _native.device_errors(reset=True)
    yield _native
    _native.check(_native.lib().li4_debug_set_wait_limits(0, 0, 0), "debug_set_wait_limits")
    _native.device_errors(reset=True)


def test_allreduce_peer_wait_runs_out(native, cuda_device):
    """Rank 0 of a 2-rank all-reduce whose peer never raises its flag: the kernel gives up after the
    short limit, sets bit 1, and still writes fp16(residual + sum of the slots it read)."""
    lib = native.lib()
    native.check(lib.li4_debug_set_wait_limits(SHORT, 0, 0), "debug_set_wait_limits")
    n, ctas, world = 4096, 4, 2
    slots = [torch.full((n,), 0.5, dtype=torch.float16, device=cuda_device),
             torch.zeros(n, dtype=torch.float16, device=cuda_device)]  # the silent peer's slot
    flags = [torch.zeros(ctas * world, dtype=torch.int32, device=cuda_device) for _ in range(world)]
    counts = torch.zeros(ctas, dtype=torch.int32, device=cuda_device)
    residual = torch.full((n,), 1.0, dtype=torch.float16, device=cuda_device)
    out = torch.empty(n, dtype=torch.float16, device=cuda_device)
    sp = (ctypes.c_void_p * world)(*[s.data_ptr() for s in slots])
    fp = (ctypes.c_void_p * world)(*[f.data_ptr() for f in flags])
    rc = lib.li4_allreduce_add(sp, fp, counts.data_ptr(), ctas, world, 0, n, residual.data_ptr(), out.data_ptr(),
                               native.stream_ptr(cuda_device))
    native.check(rc, "allreduce_add")
    torch.cuda.synchronize()
    assert native.device_errors(reset=True) & 2, "the peer-flag wait did not report running out"
    assert torch.equal(out, torch.full_like(out, 1.5))
    assert int(counts.min()) == 1 and int(counts.max()) == 1  # every CTA finished its call
    # our own flag went up in both arrays; the peer's never did
    assert int(flags[0].view(ctas, world)[:, 0].min()) == 1 and int(flags[0].view(ctas, world)[:, 1].max()) == 0
    # a 1-rank call afterwards needs no peer and reports nothing
    native.check(lib.li4_debug_set_wait_limits(0, 0, 0), "debug_set_wait_limits")
    rc = lib.li4_allreduce_add(sp, fp, counts.data_ptr(), ctas, 1, 0, n, residual.data_ptr(), out.data_ptr(),
                               native.stream_ptr(cuda_device))
    native.check(rc, "allreduce_add")
    torch.cuda.synchronize()
    assert native.device_errors(reset=True) == 0
    assert torch.equal(out, torch.full_like(out, 1.5))


def test_fused_allreduce_wait_runs_out(native, cuda_device):
    """Rank 0 of a 2-rank row-parallel GEMV that finishes its own all-reduce (LI4_EPI_ALLREDUCE_RESIDUAL),
    with a "peer" whose words never arrive: every wait gives up after the short limit, sets bit 5, and
    the launch still writes fp16(residual + fp16(own partial + the zeros it read)), which is the
    residual epilogue's output; with the defaults back, a 1-rank call reports nothing."""
    from llama import fused

    lib = native.lib()
    native.check(lib.li4_debug_set_wait_limits(SHORT, 0, 0), "debug_set_wait_limits")
    M, N, K, world = 1, 2048, 1024, 2
    gen = torch.Generator().manual_seed(5)
    w = (torch.randn(N, K, generator=gen) * 0.02).half()
    packed, scale, zero = oracle.quantize(w.numpy(), 128)
    p, s, z = (torch.from_numpy(a).to(cuda_device) for a in (packed, scale, zero))
    x = torch.randn(M, K, generator=gen).half().to(cuda_device)
    res = torch.randn(M, N, generator=gen).half().to(cuda_device)
    words = N // 16 * M * 8
    recv = [torch.zeros(world * words, dtype=torch.int64, device=cuda_device) for _ in range(world)]
    epochs = torch.zeros(N // 16, dtype=torch.int32, device=cuda_device)
    ptrs = (ctypes.c_void_p * world)(*[r.data_ptr() for r in recv])
    f = native.Fusion(epilogue=native.LI4_EPI_ALLREDUCE_RESIDUAL, residual=res.data_ptr(), stride_rm=N,
                      ar_recv=ctypes.cast(ptrs, ctypes.c_void_p), ar_recv_bytes=world * words * 8,
                      ar_epochs=epochs.data_ptr(), ar_world=world, ar_rank=0)
    out = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    fused.int4_linear_fused(x, p, s, z, out, f)
    torch.cuda.synchronize()
    assert native.device_errors(reset=True) & 32, "the fused all-reduce wait did not report running out"
    want = torch.empty_like(out)
    fused.int4_linear_fused(x, p, s, z, want, native.Fusion(epilogue=native.LI4_EPI_RESIDUAL, residual=res.data_ptr(),
                                                            stride_rm=N))
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    assert int(epochs.min()) == 1 and int(epochs.max()) == 1  # one call counted on every tile
    # our words went into the "peer's" buffer with epoch 1; nothing arrived in ours
    assert int((recv[1][:words] >> 32).min()) == 1 and int(recv[0].abs().max()) == 0
    native.check(lib.li4_debug_set_wait_limits(0, 0, 0), "debug_set_wait_limits")
    f.ar_world, f.ar_rank = 1, 0
    fused.int4_linear_fused(x, p, s, z, out, f)
    torch.cuda.synchronize()
    assert native.device_errors(reset=True) == 0
    assert torch.equal(out, want)


def test_argmax_exchange_wait_runs_out(native, cuda_device):
    """Rank 0 of a 2-rank greedy step over vocabulary shards (li4_argmax_rows_allreduce) whose peer never
    sends its keys: the wait gives up after the short limit, sets bit 6, and the launch still writes a
    token -- this shard's winner, since the zero words it read make a key below any positive maximum."""
    lib = native.lib()
    native.check(lib.li4_debug_set_wait_limits(SHORT, 0, 0), "debug_set_wait_limits")
    rows, cols, world = 4, 3000, 2
    logits = torch.randn(rows, cols, generator=torch.Generator().manual_seed(9)).abs().to(cuda_device)
    recv = [torch.zeros(2 * world * rows * 2, dtype=torch.int64, device=cuda_device) for _ in range(world)]
    epochs = torch.zeros(rows, dtype=torch.int32, device=cuda_device)
    ptrs = (ctypes.c_void_p * world)(*[r.data_ptr() for r in recv])
    out = torch.full((rows, 1), -1, dtype=torch.long, device=cuda_device)
    rc = lib.li4_argmax_rows_allreduce(logits.data_ptr(), native.LI4_F32, rows, cols, cols, 0,
                                       ctypes.cast(ptrs, ctypes.c_void_p), recv[0].numel() * 8, epochs.data_ptr(),
                                       world, 0, out.data_ptr(), 1, native.stream_ptr(cuda_device))
    native.check(rc, "argmax_rows_allreduce")
    torch.cuda.synchronize()
    assert native.device_errors(reset=True) & 64, "the key exchange wait did not report running out"
    assert torch.equal(out.view(-1), logits.argmax(-1))
    assert torch.equal(epochs, torch.ones_like(epochs))
    native.check(lib.li4_debug_set_wait_limits(0, 0, 0), "debug_set_wait_limits")
    rc = lib.li4_argmax_rows_allreduce(logits.data_ptr(), native.LI4_F32, rows, cols, cols, 0,
                                       ctypes.cast(ptrs, ctypes.c_void_p), recv[0].numel() * 8, epochs.data_ptr(),
                                       1, 0, out.data_ptr(), 1, native.stream_ptr(cuda_device))
    native.check(rc, "argmax_rows_allreduce")
    torch.cuda.synchronize()
    assert native.device_errors(reset=True) == 0
    assert torch.equal(out.view(-1), logits.argmax(-1))


def test_program_counter_wait_runs_out(native, cuda_device):
    """A two-op program whose second op waits for the first: with a target no counter can meet the wait
    gives up after the short limit, sets bit 2 and the launch returns; with the defaults restored the same
    program runs clean and its outputs match the oracle."""
    from llama.program import Program

    M, N, K = 1, 512, 2048
    gen = torch.Generator().manual_seed(11)
    w = (torch.randn(N, K, generator=gen) * 0.02).half()
    packed, scale, zero = oracle.quantize(w.numpy(), 128)
    p, s, z = (torch.from_numpy(a).to(cuda_device) for a in (packed, scale, zero))
    xh = torch.randn(M, K, generator=gen).half()
    x = xh.to(cuda_device)
    y0 = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    y1 = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    prog = Program()
    op0 = prog.linear(x, p, s, z, y0)
    prog.linear(x, p, s, z, y1, wait=op0)
    prog.finalize()
    lib = native.lib()
    native.check(lib.li4_debug_set_wait_limits(0, SHORT, 1), "debug_set_wait_limits")
    prog.launch()
    torch.cuda.synchronize()
    assert native.device_errors(reset=True) & 4, "the op-counter wait did not report running out"
    native.check(lib.li4_debug_set_wait_limits(0, 0, 0), "debug_set_wait_limits")
    prog.launch()
    torch.cuda.synchronize()
    assert native.device_errors(reset=True) == 0
    y_ref, _ = oracle.linear(xh.numpy(), packed, scale, zero)
    for y in (y0, y1):
        err = (y.float().cpu().numpy() - y_ref.astype("float32")).__abs__().max()
        assert err <= oracle.tolerance(y_ref)
