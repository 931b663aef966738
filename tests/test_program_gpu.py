"""Decode programs (li4_program_*): many ops in one persistent launch, on the GPU.

Every op kind is checked against the same torch compositions as the per-launch
fused kernels (tests/test_fused_gpu.py): F.linear on the reference's dequantized
fp16 weights with RMSNorm / RoPE / SwiGLU / residual around it, the reference's
decode attention, index_select and torch.argmax, with the GEMV's acceptance
bound max|d| <= 2e-3 * max|ref|.  Programs of several ops check the waits
between ops (a chain) and ops without waits (a GEMV list); the whole decode step
as one program is checked against the per-launch fused step and against the
reference model's golden logits and tokens.  Every test also checks that no
bounded wait ran out.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import cases
from test_fused_gpu import attention_ref, close, quantized, randn, rmsnorm_ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pg(cuda_device):
    from llama import _native, fused, program

    return program, fused, _native


def no_device_errors(nat):
    torch.cuda.synchronize()
    assert nat.device_errors(reset=True) == 0


def run(prog):
    prog.finalize()
    prog.launch()
    torch.cuda.synchronize()


@pytest.mark.parametrize("M", [1, 4, 9, 16])
@pytest.mark.parametrize("N,K", [(2048, 2048), (512, 2048), (2048, 8192), (1000, 256), (4096, 1024), (16032, 2048),
                                 (96, 6144)])
def test_program_linear(M, N, K, pg, cuda_device):
    program, fused, nat = pg
    p, s, z, w16 = quantized(N, K, cuda_device, 3 * N + K)
    x = randn((M, K), cuda_device, M + 2)
    y = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    prog = program.Program()
    prog.linear(x, p, s, z, y)
    run(prog)
    close(y, F.linear(x, w16), what="program linear")
    no_device_errors(nat)


@pytest.mark.parametrize("M", [1, 5, 16])
@pytest.mark.parametrize("N,K", [(2048, 2048), (2048, 8192), (1000, 256)])
def test_program_norm_and_residual(M, N, K, pg, cuda_device):
    program, fused, nat = pg
    p, s, z, w16 = quantized(N, K, cuda_device, N + 7 * K)
    x = randn((M, K), cuda_device, M + 11, 3.0)
    nw = (1 + 0.1 * randn((K,), cuda_device, 7).float()).half()
    res = randn((M, N), cuda_device, 12 + M)
    y1 = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    y2 = torch.empty(M, N, dtype=torch.float16, device=cuda_device)
    lg = torch.empty(M, N, dtype=torch.float32, device=cuda_device)
    prog = program.Program()
    prog.linear(x, p, s, z, y1, nat.Fusion(norm_weight=nw.data_ptr(), norm_eps=1e-5, epilogue=nat.LI4_EPI_STORE),
                keep=(nw,))
    prog.linear(x, p, s, z, y2, nat.Fusion(epilogue=nat.LI4_EPI_RESIDUAL, residual=res.data_ptr(),
                                           stride_rm=res.stride(0)), keep=(res,))
    prog.linear(x, p, s, z, None, nat.Fusion(norm_weight=nw.data_ptr(), norm_eps=1e-5,
                                             epilogue=nat.LI4_EPI_STORE_F32),
                y_ptr=lg.data_ptr(), y_stride=lg.stride(0), keep=(nw, lg))
    run(prog)
    ref_norm = F.linear(rmsnorm_ref(x, nw, 1e-5), w16)
    close(y1, ref_norm, what="norm prologue")
    close(y2, res + F.linear(x, w16), what="residual epilogue")
    close(lg, ref_norm.float(), what="fp32 logits")
    no_device_errors(nat)


@pytest.mark.parametrize("M", [1, 3, 16])
def test_program_swiglu_and_qkv(M, pg, cuda_device):
    """The paired epilogues: norm + SwiGLU, and norm + RoPE + KV-cache write, in one program."""
    program, fused, nat = pg
    from llama.model import precompute_freqs_cis
    from llama.quantize import QuantizedLinear
    from test_fused_gpu import rope_ref

    def qlin(n, k, seed):
        lin = QuantizedLinear(k, n).to(cuda_device)
        p, s, z, d = quantized(n, k, cuda_device, seed)
        lin.packed_weight.copy_(p)
        lin.scale.copy_(s)
        lin.zero_point.copy_(z)
        return lin, d

    K, hidden = 2048, 1024
    (w1, d1), (w3, d3) = qlin(hidden, K, 21), qlin(hidden, K, 22)
    gp, gs, gz = fused.fuse_gate_up(w1, w3)
    q_rows, k_rows, hd, S, pos = 2048, 512, 64, 24, 13
    (wq, dq), (wk, dk), (wv, dv) = qlin(q_rows, K, 31), qlin(k_rows, K, 32), qlin(k_rows, K, 33)
    qp, qs, qz = fused.fuse_qkv(wq, wk, wv)
    freqs = precompute_freqs_cis(hd, 2 * S, 500000.0).to(cuda_device)
    cos, sin = freqs.real.float().contiguous(), freqs.imag.float().contiguous()
    x = randn((M, K), cuda_device, 23 + M, 2.0)
    nw = (1 + 0.1 * randn((K,), cuda_device, 24).float()).half()
    ffn = torch.empty(M, hidden, dtype=torch.float16, device=cuda_device)
    kvh = k_rows // hd
    cache_k = randn((M + 1, S, kvh, hd), cuda_device, 43)
    cache_v = randn((M + 1, S, kvh, hd), cuda_device, 44)
    ck0, cv0 = cache_k.clone(), cache_v.clone()
    q_out = torch.empty(M, q_rows, dtype=torch.float16, device=cuda_device)
    pos_t = torch.tensor([pos], dtype=torch.long, device=cuda_device)
    prog = program.Program()
    prog.linear(x, gp, gs, gz, ffn, nat.Fusion(norm_weight=nw.data_ptr(), norm_eps=1e-5,
                                               epilogue=nat.LI4_EPI_SWIGLU), keep=(nw,))
    f = nat.Fusion(norm_weight=nw.data_ptr(), norm_eps=1e-5, epilogue=nat.LI4_EPI_QKV_ROPE, q_rows=q_rows,
                   k_rows=k_rows, head_dim=hd, pos=pos_t.data_ptr(), rope_cos=cos.data_ptr(),
                   rope_sin=sin.data_ptr(), rope_stride=cos.stride(0), q_out=q_out.data_ptr(),
                   stride_qm=q_out.stride(0), cache_k=cache_k.data_ptr(), cache_v=cache_v.data_ptr(),
                   cache_stride_b=cache_k.stride(0), cache_stride_s=cache_k.stride(1))
    prog.linear(x, qp, qs, qz, None, f, keep=(nw, pos_t, cos, sin, q_out, cache_k, cache_v))
    run(prog)
    xn = rmsnorm_ref(x, nw, 1e-5)
    close(ffn, F.silu(F.linear(xn, d1)) * F.linear(xn, d3), what="swiglu")
    close(q_out, rope_ref(F.linear(xn, dq), cos, sin, pos, hd), what="q")
    close(cache_k[:M, pos].reshape(M, -1), rope_ref(F.linear(xn, dk), cos, sin, pos, hd), what="k")
    close(cache_v[:M, pos].reshape(M, -1), F.linear(xn, dv), what="v")
    mask = torch.ones(M + 1, S, dtype=torch.bool, device=cuda_device)
    mask[:M, pos] = False
    assert torch.equal(cache_k[mask], ck0[mask]) and torch.equal(cache_v[mask], cv0[mask])
    no_device_errors(nat)


@pytest.mark.parametrize("B", [1, 3, 16])
@pytest.mark.parametrize("n_heads,n_kv_heads,head_dim", [(32, 8, 64), (8, 2, 32), (16, 4, 128), (8, 8, 64),
                                                         (16, 2, 64)])
@pytest.mark.parametrize("pos", [0, 17, 639])
def test_program_attention(B, n_heads, n_kv_heads, head_dim, pos, pg, cuda_device):
    program, fused, nat = pg
    S = 640
    q = randn((B, n_heads * head_dim), cuda_device, 51 + B)
    ck = randn((B, S, n_kv_heads, head_dim), cuda_device, 52)
    cv = randn((B, S, n_kv_heads, head_dim), cuda_device, 53)
    out = torch.empty_like(q)
    pos_t = torch.tensor([pos], dtype=torch.long, device=cuda_device)
    prog = program.Program()
    prog.attention(q, ck, cv, pos_t, out, n_heads, n_kv_heads)
    run(prog)
    close(out, attention_ref(q, ck, cv, pos, n_heads, n_kv_heads, head_dim), what="program attention")
    no_device_errors(nat)


def test_program_gather_and_argmax(pg, cuda_device):
    program, fused, nat = pg
    table = randn((5000, 2048), cuda_device, 71)
    ids = torch.tensor([3, 4999, 0, 3, 1234], dtype=torch.long, device=cuda_device)
    rows = torch.empty(5, 2048, dtype=torch.float16, device=cuda_device)
    logits = torch.randn(6, 128256, device=cuda_device)
    logits[1, 7] = logits[1].max() + 1  # a tie: the first index wins
    logits[1, 90000] = logits[1, 7]
    logits[2, 100] = float("nan")       # NaN is the maximum
    logits[3] = 0.0                     # all equal
    logits[4, 128255] = 1e30            # the last column
    logits[5, :] = -0.0
    logits[5, 3] = 0.0                  # -0 and +0 are equal: the first index
    out = torch.full((6, 1), -1, dtype=torch.long, device=cuda_device)
    prog = program.Program()
    prog.gather(table, ids, rows)
    prog.argmax(logits, out)
    prog.finalize()
    for _ in range(3):  # the argmax keys reset themselves between launches
        out.fill_(-1)
        prog.launch()
        torch.cuda.synchronize()
        assert torch.equal(rows, table[ids])
        assert torch.equal(out.view(-1), torch.argmax(logits, dim=-1)), (out.view(-1), torch.argmax(logits, -1))
    no_device_errors(nat)


def test_program_chain_and_increment(pg, cuda_device):
    """A chain of dependent linears (each waits for the previous) replayed with a changing input and
    a position counter, eagerly and from a CUDA graph, against the same chain composed in torch."""
    program, fused, nat = pg
    M, D, Hd = 4, 2048, 8192
    w = [quantized(Hd, D, cuda_device, 81), quantized(D, Hd, cuda_device, 82), quantized(D, D, cuda_device, 83)]
    x = torch.empty(M, D, dtype=torch.float16, device=cuda_device)
    a = torch.empty(M, Hd, dtype=torch.float16, device=cuda_device)
    b = torch.empty(M, D, dtype=torch.float16, device=cuda_device)
    c = torch.empty(M, D, dtype=torch.float16, device=cuda_device)
    ctr = torch.zeros(1, dtype=torch.long, device=cuda_device)
    prog = program.Program()
    o0 = prog.linear(x, *w[0][:3], a)
    o1 = prog.linear(a, *w[1][:3], b, nat.Fusion(epilogue=nat.LI4_EPI_RESIDUAL, residual=x.data_ptr(),
                                                  stride_rm=x.stride(0)), wait=o0)
    prog.linear(b, *w[2][:3], c, wait=o1)
    prog.increment(ctr)
    prog.finalize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        prog.launch()
    for step in range(4):
        x.copy_(randn((M, D), cuda_device, 90 + step))
        if step % 2:
            g.replay()
        else:
            prog.launch()
        torch.cuda.synchronize()
        ra = F.linear(x, w[0][3])
        rb = x + F.linear(ra, w[1][3])
        close(a, ra, what="chain 0")
        close(b, rb, what="chain 1")
        close(c, F.linear(b, w[2][3]), what="chain 2")
        assert ctr.item() == step + 1
    no_device_errors(nat)


def test_program_independent_gemv_list(pg, cuda_device):
    """The decode step's linear shapes as independent ops (no waits), twice over."""
    program, fused, nat = pg
    shapes = [(2048, 2048), (512, 2048), (512, 2048), (2048, 2048), (8192, 2048), (8192, 2048), (2048, 8192)] * 2
    prog = program.Program()
    outs = []
    for i, (N, K) in enumerate(shapes):
        p, s, z, w16 = quantized(N, K, cuda_device, 100 + i)
        x = randn((1, K), cuda_device, 200 + i)
        y = torch.empty(1, N, dtype=torch.float16, device=cuda_device)
        prog.linear(x, p, s, z, y)
        outs.append((x, w16, y))
    run(prog)
    for x, w16, y in outs:
        close(y, F.linear(x, w16), what="gemv list")
    no_device_errors(nat)


def one_b_model(bs, cuda_device, n_layers=2, max_seq_len=64):
    from llama import quantize
    from llama.model import Llama, ModelArgs

    args = ModelArgs(n_layers=n_layers, max_batch_size=bs, max_seq_len=max_seq_len)
    torch.manual_seed(0)
    torch.set_default_dtype(torch.float16)
    try:
        with torch.device(cuda_device):
            m = Llama(args)
    finally:
        torch.set_default_dtype(torch.float32)
    with torch.no_grad():
        for name, prm in m.named_parameters():
            if name.endswith("norm.weight"):
                prm.fill_(1.0)
            else:
                prm.normal_(0.0, 0.02)
    m.eval()
    quantize.quantize_model(m, 128)
    return m, args


def same_argmax_or_tie(tp, tr, lr, tol):
    """Greedy tokens of the program (tp) and of the reference step (tr): equal, or the program's pick is
    within the logit bound of the reference's maximum (a near-tie that summation order decides)."""
    rows = (tp.view(-1) != tr.view(-1)).nonzero().view(-1)
    for r in rows.tolist():
        gap = (lr[r, 0, tr.view(-1)[r]] - lr[r, 0, tp.view(-1)[r]]).item()
        assert gap <= tol, f"row {r}: token {tp.view(-1)[r].item()} vs {tr.view(-1)[r].item()}, logit gap {gap:.3e}"


@pytest.mark.parametrize("bs", [1, 4, 16])
@torch.inference_mode()
def test_program_decode_step_matches_launches(bs, pg, cuda_device):
    """Llama-3.2-1B dimensions (2 blocks): the one-launch step against the per-launch fused step over
    several positions, both fed the same tokens -- logits within the bound, the same greedy tokens
    (up to near-ties of random weights)."""
    program, fused, nat = pg
    from llama import quantize

    try:
        quantize.set_dequant_impl("v4")
        m, args = one_b_model(bs, cuda_device)
        tokens = torch.randint(0, args.vocab_size, (bs, 20), device=cuda_device)
        m(tokens, 0)
        ck = [l.attention.cache_k.clone() for l in m.layers]
        cv = [l.attention.cache_v.clone() for l in m.layers]
        inputs, ref = [], []
        tok = torch.randint(0, args.vocab_size, (bs, 1), device=cuda_device,
                            generator=torch.Generator(device=cuda_device).manual_seed(5))
        for use_program in (False, True):
            for l, a, b in zip(m.layers, ck, cv):
                l.attention.cache_k.copy_(a)
                l.attention.cache_v.copy_(b)
            dec = fused.FusedDecoder(m, program=use_program)
            pos = torch.tensor([20], dtype=torch.long, device=cuda_device)
            for i in range(4):
                if use_program:
                    tok.copy_(inputs[i])
                else:
                    inputs.append(tok.clone())
                lg = dec.decode_step(tok, pos, next_tokens=tok, advance_pos=True).float().clone()
                if not use_program:
                    ref.append((lg, tok.clone()))
                    continue
                lr, tr = ref[i]
                tol = 1e-2 * lr.abs().max().item()
                err = (lg - lr).abs().max().item()
                assert err <= tol, f"step {i}: max|d logits| = {err:.3e}"
                same_argmax_or_tie(tok, tr, lr, tol)
            assert dec.last_path == ("program" if use_program else "launches")
            assert pos.item() == 24
        no_device_errors(nat)
    finally:
        quantize.set_dequant_impl("v1")


@torch.inference_mode()
def test_program_decode_graph(golden, pg, cuda_device):
    """DecodeGraph over the one-launch step: the reference model's golden greedy tokens."""
    program, fused, nat = pg
    meta, arr = golden
    from llama import quantize
    from llama.generation import DecodeGraph
    from test_fused_gpu import build_tiny

    try:
        m = build_tiny(cuda_device).enable_fused_decode(program=True)
        prompt = torch.from_numpy(arr["model/prompt"]).to(cuda_device)
        graph = DecodeGraph(m, prompt.shape[0])
        assert m._fused.last_path == "program"
        toks = graph.tokens(prompt, cases.TINY_DECODE_STEPS)
        assert np.array_equal(toks.cpu().numpy(), arr["model/int4/tokens"])
        assert torch.equal(graph.tokens(prompt, cases.TINY_DECODE_STEPS), toks)
        no_device_errors(nat)
    finally:
        quantize.set_dequant_impl("v1")


@torch.inference_mode()
def test_program_golden_model(golden, pg, cuda_device):
    """The reference model's golden INT4 logits and tokens through the one-launch step (tiny model:
    head_dim 32, a 1000-row lm_head with a ragged last tile)."""
    program, fused, nat = pg
    meta, arr = golden
    from llama import quantize
    from test_fused_gpu import build_tiny

    try:
        m = build_tiny(cuda_device).enable_fused_decode(program=True)
        prompt = torch.from_numpy(arr["model/prompt"]).to(cuda_device)
        nxt = m(prompt, 0)[:, -1].argmax(-1, keepdim=True)
        pos = torch.tensor([prompt.shape[1]], dtype=torch.long, device=cuda_device)
        ref = arr["model/int4/decode_logits"]
        toks = [nxt]
        for i in range(cases.TINY_DECODE_STEPS):
            lg = m.decode_step(nxt, pos)
            assert m._fused.last_path == "program"
            err = np.abs(lg.float().cpu().numpy() - ref[:, i:i + 1]).max()
            assert err <= 1e-2 * np.abs(ref).max(), f"step {i}: max|d logits| = {err:.3e}"
            nxt = lg[:, -1].argmax(-1, keepdim=True)
            toks.append(nxt)
            pos += 1
        assert np.array_equal(torch.cat(toks, 1).cpu().numpy(), arr["model/int4/tokens"])
        no_device_errors(nat)
    finally:
        quantize.set_dequant_impl("v1")
