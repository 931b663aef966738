"""Row layouts of the fused decode step (llama.fused), on the CPU: the paired-row
permutation used by the RoPE epilogue and the gate/up interleave used by the
SwiGLU epilogue keep every INT4 row intact and put each pair in one 16-row tile."""
import pytest
import torch


def test_pair_permutation_puts_pairs_in_tile_rows():
    from llama.fused import pair_permutation

    n = 64
    perm = pair_permutation(n)
    assert sorted(perm.tolist()) == list(range(n))
    for p in range(n // 2):
        t, j = divmod(p, 8)
        assert perm[16 * t + j].item() == 2 * p
        assert perm[16 * t + 8 + j].item() == 2 * p + 1


def test_pair_permutation_rejects_partial_tiles():
    from llama.fused import pair_permutation

    with pytest.raises(ValueError):
        pair_permutation(24)


def test_swiglu_rows_interleave_blocks_of_eight():
    from llama.fused import swiglu_rows

    a = torch.arange(32 * 3).view(32, 3)
    b = -torch.arange(32 * 3).view(32, 3) - 1
    out = swiglu_rows(a, b)
    assert out.shape == (64, 3)
    for p in range(32):
        t, j = divmod(p, 8)
        assert torch.equal(out[16 * t + j], a[p])
        assert torch.equal(out[16 * t + 8 + j], b[p])


class _Q:
    """The buffers of a QuantizedLinear (llama/quantize.py:29-36)."""

    def __init__(self, n, k, base):
        self.packed_weight = (torch.arange(n * k // 2) % 251 + base).to(torch.uint8).view(n, k // 2)
        self.scale = (torch.arange(n * k // 128) + base).half().view(n, k // 128)
        self.zero_point = (torch.arange(n * k // 128) % 16).half().view(n, k // 128)


def test_fuse_qkv_is_a_row_permutation_of_the_concatenation():
    from llama.fused import fuse_qkv, pair_permutation

    wq, wk, wv = _Q(64, 256, 0), _Q(16, 256, 1), _Q(16, 256, 2)
    p, s, z = fuse_qkv(wq, wk, wv)
    cat = torch.cat([wq.packed_weight, wk.packed_weight, wv.packed_weight])
    assert torch.equal(p, cat[pair_permutation(96)])
    assert torch.equal(s, torch.cat([wq.scale, wk.scale, wv.scale])[pair_permutation(96)])
    assert p.is_contiguous() and s.is_contiguous() and z.is_contiguous()


def test_fuse_gate_up_keeps_rows():
    from llama.fused import fuse_gate_up

    w1, w3 = _Q(32, 256, 3), _Q(32, 256, 4)
    p, s, z = fuse_gate_up(w1, w3)
    assert torch.equal(p[0:8], w1.packed_weight[0:8]) and torch.equal(p[8:16], w3.packed_weight[0:8])
    assert torch.equal(z[16:24], w1.zero_point[8:16]) and torch.equal(s[24:32], w3.scale[8:16])
