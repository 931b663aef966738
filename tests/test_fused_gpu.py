"""Fused decode-step kernels (li4_int4_linear_fused, li4_decode_attention) on the GPU.

Each fused operation is checked against the reference's own composition of
the same operation in torch on the GPU: RMSNorm as llama/model.py:61-75,
F.linear on the reference's dequantized fp16 weights (the v1 forward,
llama/quantize.py:143-146), RoPE through complex views (:126-152), SwiGLU
(:315), residual adds (:358-362) and the decode attention (:262-275).  The
bound is the GEMV's acceptance bound, max|d| <= 2e-3 * max|ref|, per output
tensor.  The whole fused step is checked against the reference model's golden
logits and tokens (tests/golden) and against the unfused decode step.
"""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import cases

pytestmark = pytest.mark.gpu
TOL = 2e-3


@pytest.fixture(scope="module")
def fz(cuda_device):
    from llama import _native, fused

    return fused, _native


def quantized(N, K, dev, seed):
    from llama.quantize import QuantizedLinear

    gen = torch.Generator(device=dev).manual_seed(seed)
    w = (torch.randn(N, K, generator=gen, device=dev) * 0.02).half()
    p, s, z = QuantizedLinear.quantize_tensor(w, 128)
    return p, s, z, QuantizedLinear.dequantize_packed(p, s, z, 128)


def rmsnorm_ref(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).type_as(x) * w


def close(got, ref, tol=TOL, what=""):
    err = (got.float() - ref.float()).abs().max().item()
    bound = tol * ref.float().abs().max().item()
    assert err <= bound, f"{what} max|d| = {err:.3e} > {bound:.3e}"


def randn(shape, dev, seed, scale=1.0):
    gen = torch.Generator(device=dev).manual_seed(seed)
    return (torch.randn(*shape, generator=gen, device=dev) * scale).half()


@pytest.mark.parametrize("M", [1, 5, 16])
@pytest.mark.parametrize("N,K", [(512, 2048), (2048, 2048), (1000, 256), (2048, 8192)])
def test_norm_prologue(M, N, K, fz, cuda_device):
    fused, nat = fz
    p, s, z, w16 = quantized(N, K, cuda_device, N + K)
    x = randn((M, K), cuda_device, M + 1, 3.0)
    nw = (1 + 0.1 * randn((K,), cuda_device, 7).float()).half()
    y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    f = nat.Fusion(norm_weight=nw.data_ptr(), norm_eps=1e-5, epilogue=nat.LI4_EPI_STORE)
    fused.int4_linear_fused(x, p, s, z, y, f)
    close(y, F.linear(rmsnorm_ref(x, nw, 1e-5), w16), what="norm+gemv")


@pytest.mark.parametrize("M", [1, 3, 16])
@pytest.mark.parametrize("N,K", [(2048, 2048), (2048, 8192), (256, 1024), (2048, 256)])
def test_residual_epilogue(M, N, K, fz, cuda_device):
    fused, nat = fz
    p, s, z, w16 = quantized(N, K, cuda_device, N * 3 + K)
    x = randn((M, K), cuda_device, 11 + M)
    res = randn((M, N), cuda_device, 12 + M)
    y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    f = nat.Fusion(epilogue=nat.LI4_EPI_RESIDUAL, residual=res.data_ptr(), stride_rm=res.stride(0))
    fused.int4_linear_fused(x, p, s, z, y, f)
    close(y, res + F.linear(x, w16), what="residual")
    # in place: the output overwrites the residual it reads
    res2 = res.clone()
    f = nat.Fusion(epilogue=nat.LI4_EPI_RESIDUAL, residual=res2.data_ptr(), stride_rm=res2.stride(0))
    fused.int4_linear_fused(x, p, s, z, res2, f)
    assert torch.equal(res2, y)


@pytest.mark.parametrize("M", [1, 4, 16])
@pytest.mark.parametrize("hidden,K", [(8192, 2048), (512, 2048), (1024, 2048), (1024, 256)])
def test_swiglu_epilogue(M, hidden, K, fz, cuda_device):
    fused, nat = fz
    from llama.quantize import QuantizedLinear

    w1 = QuantizedLinear(K, hidden).to(cuda_device)
    w3 = QuantizedLinear(K, hidden).to(cuda_device)
    p1, s1, z1, d1 = quantized(hidden, K, cuda_device, 21 + hidden)
    p3, s3, z3, d3 = quantized(hidden, K, cuda_device, 22 + hidden)
    for lin, (p, s, z) in ((w1, (p1, s1, z1)), (w3, (p3, s3, z3))):
        lin.packed_weight.copy_(p)
        lin.scale.copy_(s)
        lin.zero_point.copy_(z)
    gp, gs, gz = fused.fuse_gate_up(w1, w3)
    x = randn((M, K), cuda_device, 23 + M, 2.0)
    nw = (1 + 0.1 * randn((K,), cuda_device, 24).float()).half()
    y = torch.empty(M, hidden, dtype=torch.float16, device=cuda_device)
    f = nat.Fusion(norm_weight=nw.data_ptr(), norm_eps=1e-5, epilogue=nat.LI4_EPI_SWIGLU)
    fused.int4_linear_fused(x, gp, gs, gz, y, f)
    xn = rmsnorm_ref(x, nw, 1e-5)
    close(y, F.silu(F.linear(xn, d1)) * F.linear(xn, d3), what="swiglu")


def rope_ref(t, cos, sin, pos, head_dim):
    """apply_rotary_emb of llama/model.py:126-152 on rows t [M, n * head_dim] at one position."""
    M = t.shape[0]
    tc = torch.view_as_complex(t.float().reshape(M, -1, head_dim // 2, 2))
    fc = torch.complex(cos[pos], sin[pos])
    return torch.view_as_real(tc * fc).reshape(M, -1).type_as(t)


@pytest.mark.parametrize("M", [1, 2, 16])
@pytest.mark.parametrize("q_rows,k_rows,head_dim,K", [(2048, 512, 64, 2048), (256, 64, 64, 2048), (256, 64, 32, 256),
                                                      (512, 128, 128, 2048)])
def test_qkv_rope_epilogue(M, q_rows, k_rows, head_dim, K, fz, cuda_device):
    fused, nat = fz
    from llama.model import precompute_freqs_cis
    from llama.quantize import QuantizedLinear

    lins = []
    dq = []
    for i, n in enumerate((q_rows, k_rows, k_rows)):
        lin = QuantizedLinear(K, n).to(cuda_device)
        p, s, z, d = quantized(n, K, cuda_device, 31 + i + n)
        lin.packed_weight.copy_(p)
        lin.scale.copy_(s)
        lin.zero_point.copy_(z)
        lins.append(lin)
        dq.append(d)
    qp, qs, qz = fused.fuse_qkv(*lins)
    S, pos = 24, 13
    freqs = precompute_freqs_cis(head_dim, 2 * S, 500000.0).to(cuda_device)
    cos, sin = freqs.real.float().contiguous(), freqs.imag.float().contiguous()
    x = randn((M, K), cuda_device, 41 + M, 2.0)
    nw = (1 + 0.1 * randn((K,), cuda_device, 42).float()).half()
    kvh = k_rows // head_dim
    cache_k = randn((M + 1, S, kvh, head_dim), cuda_device, 43)
    cache_v = randn((M + 1, S, kvh, head_dim), cuda_device, 44)
    ck0, cv0 = cache_k.clone(), cache_v.clone()
    q_out = torch.empty(M, q_rows, dtype=torch.float16, device=cuda_device)
    pos_t = torch.tensor([pos], dtype=torch.long, device=cuda_device)
    f = nat.Fusion(norm_weight=nw.data_ptr(), norm_eps=1e-5, epilogue=nat.LI4_EPI_QKV_ROPE, q_rows=q_rows,
                   k_rows=k_rows, head_dim=head_dim, pos=pos_t.data_ptr(), rope_cos=cos.data_ptr(),
                   rope_sin=sin.data_ptr(), rope_stride=cos.stride(0), q_out=q_out.data_ptr(),
                   stride_qm=q_out.stride(0), cache_k=cache_k.data_ptr(), cache_v=cache_v.data_ptr(),
                   cache_stride_b=cache_k.stride(0), cache_stride_s=cache_k.stride(1))
    fused.int4_linear_fused(x, qp, qs, qz, None, f)
    xn = rmsnorm_ref(x, nw, 1e-5)
    q_ref = rope_ref(F.linear(xn, dq[0]), cos, sin, pos, head_dim)
    k_ref = rope_ref(F.linear(xn, dq[1]), cos, sin, pos, head_dim)
    v_ref = F.linear(xn, dq[2])
    close(q_out, q_ref, what="q")
    close(cache_k[:M, pos].reshape(M, -1), k_ref, what="k")
    close(cache_v[:M, pos].reshape(M, -1), v_ref, what="v")
    # nothing else of the caches is touched
    mask = torch.ones(M + 1, S, dtype=torch.bool, device=cuda_device)
    mask[:M, pos] = False
    assert torch.equal(cache_k[mask], ck0[mask]) and torch.equal(cache_v[mask], cv0[mask])


def attention_ref(q, ck, cv, pos, n_heads, n_kv_heads, head_dim):
    """llama/model.py:262-275 at seqlen 1 over cache rows 0..pos (repeat_kv expanded)."""
    B = q.shape[0]
    rep = n_heads // n_kv_heads
    keys = ck[:B, :pos + 1].repeat_interleave(rep, dim=2).transpose(1, 2)  # [B, H, L, d]
    values = cv[:B, :pos + 1].repeat_interleave(rep, dim=2).transpose(1, 2)
    xq = q.view(B, n_heads, 1, head_dim)
    scores = torch.matmul(xq, keys.transpose(2, 3)) / math.sqrt(head_dim)
    scores = F.softmax(scores.float(), dim=-1).type_as(xq)
    return torch.matmul(scores, values).reshape(B, n_heads * head_dim)


@pytest.mark.parametrize("B", [1, 3])
@pytest.mark.parametrize("n_heads,n_kv_heads,head_dim", [(32, 8, 64), (4, 1, 64), (8, 2, 32), (16, 2, 128),
                                                         (8, 8, 64)])
@pytest.mark.parametrize("pos", [0, 17, 299])
def test_decode_attention(B, n_heads, n_kv_heads, head_dim, pos, fz, cuda_device):
    fused, _ = fz
    S = 300
    q = randn((B, n_heads * head_dim), cuda_device, 51 + B)
    ck = randn((B + 1, S, n_kv_heads, head_dim), cuda_device, 52)
    cv = randn((B + 1, S, n_kv_heads, head_dim), cuda_device, 53)
    out = torch.empty_like(q)
    pos_t = torch.tensor([pos], dtype=torch.long, device=cuda_device)
    fused.decode_attention(q, ck, cv, pos_t, out, n_heads, n_kv_heads)
    close(out, attention_ref(q, ck, cv, pos, n_heads, n_kv_heads, head_dim), what="attention")


def build_tiny(device):
    from llama import quantize
    from llama.model import Llama, ModelArgs

    torch.set_default_dtype(torch.float16)
    try:
        m = Llama(ModelArgs(**cases.TINY_MODEL))
    finally:
        torch.set_default_dtype(torch.float32)
    m.load_state_dict(cases.tiny_state_dict(cases.TINY_MODEL), strict=True)
    m = m.to(device).eval()
    quantize.quantize_model(m, 128)
    quantize.set_dequant_impl("v4")
    return m


@torch.inference_mode()
def test_fused_decode_matches_reference_model(golden, cuda_device):
    """Prefill through forward, then fused decode steps: the reference's INT4 logits and greedy tokens."""
    meta, arr = golden
    from llama import quantize

    try:
        m = build_tiny(cuda_device).enable_fused_decode()
        prompt = torch.from_numpy(arr["model/prompt"]).to(cuda_device)
        nxt = m(prompt, 0)[:, -1].argmax(-1, keepdim=True)
        pos = torch.tensor([prompt.shape[1]], dtype=torch.long, device=cuda_device)
        ref = arr["model/int4/decode_logits"]
        toks = [nxt]
        for i in range(cases.TINY_DECODE_STEPS):
            lg = m.decode_step(nxt, pos)
            got = lg.float().cpu().numpy()
            err = np.abs(got - ref[:, i:i + 1]).max()
            assert err <= 1e-2 * np.abs(ref).max(), f"step {i}: max|d logits| = {err:.3e}"
            nxt = lg[:, -1].argmax(-1, keepdim=True)
            toks.append(nxt)
            pos += 1
        assert np.array_equal(torch.cat(toks, 1).cpu().numpy(), arr["model/int4/tokens"])
    finally:
        quantize.set_dequant_impl("v1")


@torch.inference_mode()
def test_fused_graph_tokens(golden, cuda_device):
    """One captured graph of the fused step replayed per position gives the reference's tokens."""
    meta, arr = golden
    from llama import quantize
    from llama.generation import DecodeGraph

    try:
        m = build_tiny(cuda_device).enable_fused_decode()
        prompt = torch.from_numpy(arr["model/prompt"]).to(cuda_device)
        graph = DecodeGraph(m, prompt.shape[0])
        toks = graph.tokens(prompt, cases.TINY_DECODE_STEPS)
        assert np.array_equal(toks.cpu().numpy(), arr["model/int4/tokens"])
        assert torch.equal(graph.tokens(prompt, cases.TINY_DECODE_STEPS), toks)
    finally:
        quantize.set_dequant_impl("v1")


@pytest.mark.parametrize("bs", [1, 16])
@torch.inference_mode()
def test_fused_step_matches_unfused_llama_block(bs, cuda_device):
    """Llama-3.2-1B dimensions (2 blocks, random N(0, 0.02) weights): fused vs unfused decode logits."""
    from llama import quantize
    from llama.model import Llama, ModelArgs

    args = ModelArgs(n_layers=2, max_batch_size=bs, max_seq_len=64)
    torch.manual_seed(0)
    torch.set_default_dtype(torch.float16)
    try:
        with torch.device(cuda_device):
            m = Llama(args)
    finally:
        torch.set_default_dtype(torch.float32)
    try:
        with torch.no_grad():
            for name, prm in m.named_parameters():
                if name.endswith("norm.weight"):
                    prm.fill_(1.0)
                else:
                    prm.normal_(0.0, 0.02)
        m.eval()
        quantize.quantize_model(m, 128)
        quantize.set_dequant_impl("v4")
        tokens = torch.randint(0, args.vocab_size, (bs, 20), device=cuda_device)
        m(tokens, 0)
        nxt = torch.randint(0, args.vocab_size, (bs, 1), device=cuda_device)
        pos = torch.tensor([20], dtype=torch.long, device=cuda_device)
        ck = [l.attention.cache_k.clone() for l in m.layers]
        cv = [l.attention.cache_v.clone() for l in m.layers]
        ref = m.decode_step(nxt, pos).float()
        for l, a, b in zip(m.layers, ck, cv):  # same cache state for the fused step
            l.attention.cache_k.copy_(a)
            l.attention.cache_v.copy_(b)
        m.enable_fused_decode()
        got = m.decode_step(nxt, pos).float()
        err = (got - ref).abs().max().item()
        assert err <= 1e-2 * ref.abs().max().item(), f"max|d logits| = {err:.3e}, max|ref| = {ref.abs().max():.3e}"
    finally:
        quantize.set_dequant_impl("v1")


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("rows,cols", [(1, 128256), (16, 128256), (3, 1000), (2, 7)])
def test_argmax_rows_matches_torch(dtype, rows, cols, fz, cuda_device):
    fused, _ = fz
    gen = torch.Generator(device=cuda_device).manual_seed(rows * cols)
    x = torch.randn(rows, cols, generator=gen, device=cuda_device).to(dtype)
    if cols > 10:
        x[0, 5] = x[0, cols - 3] = x[0].max() + 1  # a tie: the first index wins
    out = torch.full((rows, 1), -1, dtype=torch.long, device=cuda_device)
    fused.argmax_rows(x, out)
    assert torch.equal(out.view(-1), x.argmax(-1))
    if rows > 1:
        x[1, cols // 2] = float("nan")  # NaN counts as the maximum
        fused.argmax_rows(x, out)
        assert out[1, 0].item() == cols // 2 == x[1].argmax().item()


@pytest.mark.parametrize("B,max_seq,pos", [(2, 8192, 8191), (16, 640, 600), (1, 640, 1)])
def test_decode_attention_cluster_shapes(B, max_seq, pos, fz, cuda_device):
    """Long caches (several CTAs per head, shared memory above 48 KiB) and batch 16 (one CTA per head)."""
    fused, _ = fz
    n_heads, n_kv_heads, head_dim = 32, 8, 64
    q = randn((B, n_heads * head_dim), cuda_device, 61 + B)
    ck = randn((B, max_seq, n_kv_heads, head_dim), cuda_device, 62)
    cv = randn((B, max_seq, n_kv_heads, head_dim), cuda_device, 63)
    out = torch.empty_like(q)
    pos_t = torch.tensor([pos], dtype=torch.long, device=cuda_device)
    fused.decode_attention(q, ck, cv, pos_t, out, n_heads, n_kv_heads)
    close(out, attention_ref(q, ck, cv, pos, n_heads, n_kv_heads, head_dim), what="attention")


@pytest.mark.parametrize("B,max_seq,old,new", [(1, 640, 100, 517), (4, 640, 517, 30), (16, 576, 200, 575)])
def test_decode_attention_position_written_by_preceding_kernel(B, max_seq, old, new, fz, cuda_device):
    """The position is written by the kernel right before the attention (li4_argmax_rows storing its
    index into *pos): the attention reads the position before its dependency wait to start copying
    cache rows, so it may see the old value and must then copy again (the "moved" path).  Whichever
    way each launch goes, the result attends rows 0..new."""
    fused, _ = fz
    n_heads, n_kv_heads, head_dim = 32, 8, 64
    q = randn((B, n_heads * head_dim), cuda_device, 71 + B)
    ck = randn((B, max_seq, n_kv_heads, head_dim), cuda_device, 72)
    cv = randn((B, max_seq, n_kv_heads, head_dim), cuda_device, 73)
    logits = torch.zeros(1, max_seq, device=cuda_device)
    logits[0, new] = 1.0
    want = attention_ref(q, ck, cv, new, n_heads, n_kv_heads, head_dim)
    out = torch.empty_like(q)
    for _ in range(20):
        pos_t = torch.tensor([old], dtype=torch.long, device=cuda_device)
        out.zero_()
        fused.argmax_rows(logits, pos_t.view(1, 1))  # *pos = new, written by the preceding kernel
        fused.decode_attention(q, ck, cv, pos_t, out, n_heads, n_kv_heads)
        torch.cuda.synchronize()
        assert pos_t.item() == new
        close(out, want, what="attention")


@pytest.mark.parametrize("M", [1, 16])
@pytest.mark.parametrize("N,K", [(128256, 2048), (1000, 256), (2048, 8192)])
def test_store_f32_epilogue(M, N, K, fz, cuda_device):
    """fp32 output of the fp16-rounded GEMV (the lm_head's output(h).float()), with the final RMSNorm."""
    fused, nat = fz
    p, s, z, w16 = quantized(N, K, cuda_device, N + 3 * K)
    x = randn((M, K), cuda_device, 5 + M, 2.0)
    nw = (1 + 0.1 * randn((K,), cuda_device, 6).float()).half()
    y = torch.empty(M, N, dtype=torch.float32, device=cuda_device)
    f = nat.Fusion(norm_weight=nw.data_ptr(), norm_eps=1e-5, epilogue=nat.LI4_EPI_STORE_F32)
    fused.int4_linear_fused(x, p, s, z, None, f, y_ptr=y.data_ptr(), y_stride=y.stride(0))
    assert torch.equal(y, y.half().float()), "fp32 outputs are not widened fp16 values"
    close(y, F.linear(rmsnorm_ref(x, nw, 1e-5), w16).float(), what="store_f32")


@pytest.mark.parametrize("M", [1, 3, 16])
@pytest.mark.parametrize("N,K", [(2048, 2048), (2048, 8192), (2048, 256)])
def test_sumsq_handoff(M, N, K, fz, cuda_device):
    """A residual epilogue leaves per-16-row-tile sums of squares of what it wrote; an RMSNorm
    prologue reading them gives the same result as the prologue that reads x itself."""
    fused, nat = fz
    p, s, z, w16 = quantized(N, K, cuda_device, 9 * N + K)
    x = randn((M, K), cuda_device, 70 + M)
    res = randn((M, N), cuda_device, 71 + M)
    h = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    ssq = torch.full(((N + 15) // 16, M), float("nan"), dtype=torch.float32, device=cuda_device)
    f = nat.Fusion(epilogue=nat.LI4_EPI_RESIDUAL, residual=res.data_ptr(), stride_rm=N, sumsq_out=ssq.data_ptr())
    fused.int4_linear_fused(x, p, s, z, h, f)
    want = h.float().view(M, -1, 16).pow(2).sum(-1).t()  # [tiles, M]
    torch.testing.assert_close(ssq, want, rtol=1e-5, atol=0)
    # the next launch's RMSNorm over h: from the sums of squares vs from h itself
    p2, s2, z2, _ = quantized(3072, N, cuda_device, 5 * N + 1)
    nw = (1 + 0.1 * randn((N,), cuda_device, 72).float()).half()
    y_a = torch.empty(M, 3072, dtype=torch.float16, device=cuda_device)
    y_b = torch.empty_like(y_a)
    fused.int4_linear_fused(h, p2, s2, z2, y_a, nat.Fusion(norm_weight=nw.data_ptr(), norm_eps=1e-5,
                                                          epilogue=nat.LI4_EPI_STORE))
    fused.int4_linear_fused(h, p2, s2, z2, y_b, nat.Fusion(norm_weight=nw.data_ptr(), norm_eps=1e-5,
                                                          epilogue=nat.LI4_EPI_STORE, sumsq_in=ssq.data_ptr(),
                                                          sumsq_tiles=ssq.shape[0]))
    close(y_b, y_a, what="norm from handed-over sums of squares")


def test_gather_rows_matches_index_select(fz, cuda_device):
    """li4_gather_rows: the embedding lookup, bit-exact against torch.index_select; an id outside the
    table is clamped and flagged (bit 3 of li4_device_errors)."""
    fused, nat = fz
    table = randn((5000, 2048), cuda_device, 91)
    for ids in ([7], [4999, 0, 3, 3, 1234] * 3 + [17]):
        idx = torch.tensor(ids, dtype=torch.long, device=cuda_device)
        out = torch.empty(len(ids), 2048, dtype=torch.float16, device=cuda_device)
        fused.gather_rows(table, idx, out)
        torch.cuda.synchronize()
        assert torch.equal(out, torch.index_select(table, 0, idx))
    assert nat.device_errors(reset=True) == 0
    bad = torch.tensor([2, 5000], dtype=torch.long, device=cuda_device)
    out = torch.empty(2, 2048, dtype=torch.float16, device=cuda_device)
    fused.gather_rows(table, bad, out)
    torch.cuda.synchronize()
    assert nat.device_errors(reset=True) & 8
    assert torch.equal(out[1], table[4999])


@pytest.mark.parametrize("M", [1, 3, 8])
def test_fused_argmax_epilogue(M, fz, cuda_device):
    """The lm_head's fused greedy argmax (li4_fusion.argmax_*): torch.argmax of the fp32 logits the same
    launch writes, on two launches in a row (the scratch is left zero); M > 8 is refused."""
    fused, nat = fz
    N, K = 128256, 2048
    p, s, z, _ = quantized(N, K, cuda_device, 1234)
    scratch = torch.zeros(8 * 16 + 8, dtype=torch.uint8, device=cuda_device)
    lg = torch.empty(M, N, dtype=torch.float32, device=cuda_device)
    out = torch.full((M, 1), -1, dtype=torch.long, device=cuda_device)
    for seed in (1, 2):
        x = randn((M, K), cuda_device, 300 + seed + M)
        f = nat.Fusion(epilogue=nat.LI4_EPI_STORE_F32, argmax_out=out.data_ptr(), argmax_stride=out.stride(0),
                       argmax_scratch=scratch.data_ptr())
        fused.int4_linear_fused(x, p, s, z, None, f, y_ptr=lg.data_ptr(), y_stride=lg.stride(0))
        torch.cuda.synchronize()
        assert torch.equal(out.view(-1), torch.argmax(lg, dim=-1))
        assert int(scratch.count_nonzero()) == 0
    x16 = randn((16, K), cuda_device, 399)
    lg16 = torch.empty(16, N, dtype=torch.float32, device=cuda_device)
    with pytest.raises(nat.Li4Error) as err:
        fused.int4_linear_fused(x16, p, s, z, None, f, y_ptr=lg16.data_ptr(), y_stride=lg16.stride(0))
    assert err.value.status == nat.LI4_ERR_UNSUPPORTED
    assert nat.device_errors(reset=True) == 0
