"""Fused INT4 decode step: five kernel launches per transformer block.

The reference's decode step runs every block as ~45 ATen kernels around its
seven INT4 linears (llama/model.py:222-277, 310-315, 358-362): two RMSNorms of
five or six kernels each, RoPE through complex views, the cache writes,
repeat_kv copies, two matmuls, the softmax, SiLU, the product and two residual
adds.  Here a block is:

  1. QKV GEMV   RMSNorm(attention_norm) while staging x; RoPE on q and k; q to a
                buffer, k and v into the KV cache at row *pos  (li4_int4_linear_fused)
                (at batch <= 4 the mean of squares comes from the previous block's w2
                epilogue, which leaves per-tile sums of squares of h beside h)
  2. attention  grouped-query decode attention over cache rows 0..*pos
                                                                (li4_decode_attention)
  3. wo GEMV    h1 = h + wo(attn)                               (residual epilogue)
  4. w1/w3 GEMV RMSNorm(ffn_norm) while staging h1; fp16(silu(g)) * u
                                                                (SwiGLU epilogue)
  5. w2 GEMV    h = h1 + w2(ffn)                                (residual epilogue)

and the step ends with lm_head with the final RMSNorm fused into its staging.  The embedding rows
come from li4_gather_rows and the greedy tokens from li4_argmax_rows.
Under tensor parallelism the wo / w2 outputs are partial sums.  By default the
row-parallel GEMV finishes them itself: it stores its fp16 partial into every
rank's receive buffer over NVLink and sums the ranks' partials with the residual
in the same launch (LI4_EPI_ALLREDUCE_RESIDUAL, llama.comm.push_fusion).  With
fused_allreduce=False the GEMV writes its partial into a buffer every rank has
mapped and a second kernel sums the partials (li4_allreduce_add); with
nvlink_allreduce=False NCCL all-reduces and torch adds the residual.  The
greedy step over the vocabulary-sharded lm_head likewise exchanges each rank's
winner over NVLink inside the argmax launch (li4_argmax_rows_allreduce), or
through an NCCL MAX all-reduce of ordered keys.

The fused epilogues pair two GEMV outputs in one thread.  They take weights
whose rows are rearranged once, at construction (pair_permutation,
swiglu_rows): the INT4 bytes, scales and zero points are the model's own,
only their row order changes.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _native as native


def pair_permutation(n: int) -> torch.Tensor:
    """Row order that puts rows (2p, 2p + 1) at tile rows (16t + j, 16t + 8 + j), p = 8t + j.

    new_rows = old_rows[pair_permutation(n)]; n must be a multiple of 16."""
    if n % 16:
        raise ValueError(f"paired rows need a multiple of 16 rows, got {n}")
    return torch.arange(n).view(n // 16, 8, 2).permute(0, 2, 1).reshape(n)


def swiglu_rows(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Interleave the rows of w1 (a) and w3 (b) in blocks of 8: tile t holds a[8t:8t+8] then b[8t:8t+8]."""
    n = a.shape[0]
    if b.shape != a.shape or n % 8:
        raise ValueError(f"w1 / w3 rows must match and be a multiple of 8, got {tuple(a.shape)} {tuple(b.shape)}")
    return torch.stack([a.reshape(n // 8, 8, -1), b.reshape(n // 8, 8, -1)], dim=1).reshape(2 * n, *a.shape[1:])


def _qparams(lin):
    return lin.packed_weight, lin.scale, lin.zero_point


def fuse_qkv(wq, wk, wv):
    """Packed / scale / zero of [wq; wk; wv] in paired-row order (LI4_EPI_QKV_ROPE)."""
    parts = [_qparams(w) for w in (wq, wk, wv)]
    perm = pair_permutation(sum(p[0].shape[0] for p in parts)).to(parts[0][0].device)
    return tuple(torch.cat([p[i] for p in parts]).index_select(0, perm).contiguous() for i in range(3))


def fuse_gate_up(w1, w3):
    """Packed / scale / zero of w1 and w3 interleaved for the SwiGLU epilogue."""
    a, b = _qparams(w1), _qparams(w3)
    return tuple(swiglu_rows(a[i], b[i]).contiguous() for i in range(3))


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def int4_linear_fused(x: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, zp: torch.Tensor,
                      y: Optional[torch.Tensor], fusion: native.Fusion, group_size: int = 128,
                      y_ptr: Optional[int] = None, y_stride: int = 0) -> None:
    """One li4_int4_linear_fused launch on the current stream: x [M, K] fp16 (row-contiguous).
    y_ptr / y_stride give the output as a raw device address instead of a tensor (a communication slot)."""
    M, K = x.shape
    N = packed.shape[0]
    lib = native.lib()
    dev = x.device
    nbytes = lib.li4_int4_linear_workspace_bytes(M, N, K, group_size, 0)
    ws = native.workspace(dev, nbytes) if nbytes else None
    if y_ptr is None:
        y_ptr, y_stride = _ptr(y), (y.stride(0) if y is not None else 0)
    rc = lib.li4_int4_linear_fused(x.data_ptr(), packed.data_ptr(), scale.data_ptr(), zp.data_ptr(), y_ptr,
                                   M, N, K, group_size, x.stride(0), packed.stride(0), scale.stride(0), y_stride,
                                   ctypes.byref(fusion), _ptr(ws), ws.numel() if ws is not None else 0,
                                   native.stream_ptr(dev))
    native.check(rc, "int4_linear_fused")


def decode_attention(q: torch.Tensor, cache_k: torch.Tensor, cache_v: torch.Tensor, pos: torch.Tensor,
                     out: torch.Tensor, n_heads: int, n_kv_heads: int, max_seq: Optional[int] = None) -> None:
    """out[b] = attention of q[b] (fp16 [B, n_heads * 64]) over cache rows 0..pos (cache [B', S, n_kv_heads, 64])."""
    B = q.shape[0]
    S = cache_k.shape[1]
    if cache_k.stride(3) != 1 or cache_k.stride(2) != cache_k.shape[3] or cache_v.stride() != cache_k.stride():
        raise RuntimeError("decode_attention: cache rows [n_kv_heads, head_dim] must be contiguous, K and V alike")
    rc = native.lib().li4_decode_attention(q.data_ptr(), q.stride(0), cache_k.data_ptr(), cache_v.data_ptr(),
                                           cache_k.stride(0), cache_k.stride(1), out.data_ptr(), out.stride(0),
                                           B, n_heads, n_kv_heads, cache_k.shape[3], pos.data_ptr(),
                                           S if max_seq is None else max_seq, native.stream_ptr(q.device))
    native.check(rc, "decode_attention")


def gather_rows(table: torch.Tensor, ids: torch.Tensor, out: torch.Tensor) -> None:
    """out[r] = table[ids[r]] (li4_gather_rows): fp16 rows, ids int64, on the current stream."""
    rc = native.lib().li4_gather_rows(table.data_ptr(), table.shape[0], table.shape[1], table.stride(0),
                                      ids.data_ptr(), ids.numel(), out.data_ptr(), out.stride(0),
                                      native.stream_ptr(out.device))
    native.check(rc, "gather_rows")


def argmax_rows(logits: torch.Tensor, out: torch.Tensor) -> None:
    """out[r, 0] = torch.argmax(logits[r]) for fp16 / fp32 logits [rows, cols] (li4_argmax_rows)."""
    codes = {torch.float16: native.LI4_F16, torch.float32: native.LI4_F32}
    if logits.dtype not in codes or logits.stride(-1) != 1 or out.dtype != torch.long:
        raise RuntimeError("argmax_rows: fp16 / fp32 logits with contiguous rows and an int64 output")
    rows, cols = logits.shape
    rc = native.lib().li4_argmax_rows(logits.data_ptr(), codes[logits.dtype], rows, cols, logits.stride(0),
                                      out.data_ptr(), out.stride(0), native.stream_ptr(logits.device))
    native.check(rc, "argmax_rows")


def argmax_rows_keys(logits: torch.Tensor, index_offset: int, keys: torch.Tensor) -> None:
    """keys[r] = the signed 64-bit key of the winner of logits[r] at global index index_offset + column
    (li4_argmax_rows_keys): the largest key over every vocabulary shard is the row's argmax."""
    codes = {torch.float16: native.LI4_F16, torch.float32: native.LI4_F32}
    if logits.dtype not in codes or logits.stride(-1) != 1 or keys.dtype != torch.long:
        raise RuntimeError("argmax_rows_keys: fp16 / fp32 logits with contiguous rows and an int64 output")
    rows, cols = logits.shape
    rc = native.lib().li4_argmax_rows_keys(logits.data_ptr(), codes[logits.dtype], rows, cols, logits.stride(0),
                                           index_offset, keys.data_ptr(), keys.stride(0),
                                           native.stream_ptr(logits.device))
    native.check(rc, "argmax_rows_keys")


def key_index(keys: torch.Tensor) -> torch.Tensor:
    """The global index a key of argmax_rows_keys carries: 0xFFFFFFFF - (key & 0xFFFFFFFF)."""
    return 0xFFFFFFFF - torch.bitwise_and(keys, 0xFFFFFFFF)


class _Block:
    """Fused weights and fusion descriptors of one transformer block."""

    def __init__(self, layer, cos: torch.Tensor, sin: torch.Tensor):
        att, ff = layer.attention, layer.feed_forward
        for lin in (att.wq, att.wk, att.wv, att.wo, ff.w1, ff.w2, ff.w3):
            if not hasattr(lin, "packed_weight") or lin.group_size != 128 or lin.bias is not None:
                raise TypeError("the fused decode step needs INT4 group-128 QuantizedLinear layers without bias "
                                "(run quantize_model first)")
        self.att, self.ff = att, ff
        self.qkv = fuse_qkv(att.wq, att.wk, att.wv)
        self.gate_up = fuse_gate_up(ff.w1, ff.w3)
        self.wo = _qparams(att.wo)
        self.w2 = _qparams(ff.w2)
        self.attn_norm = layer.attention_norm.weight.detach().contiguous()
        self.attn_eps = float(layer.attention_norm.eps)
        self.ffn_norm = layer.ffn_norm.weight.detach().contiguous()
        self.ffn_eps = float(layer.ffn_norm.eps)
        self.q_rows = att.wq.out_features
        self.k_rows = att.wk.out_features
        self.cos, self.sin = cos, sin


class FusedDecoder:
    """The decode step of a quantized Llama (llama.model.Llama) as fused kernels.

    decode_step(tokens [bs, 1], pos int64 [1]) has the semantics of
    Llama.decode_step and shares the model's KV caches, so a prefill through
    Llama.forward followed by fused decode steps is the reference's generation
    loop.  Every launch reads the position from `pos`: one CUDA graph of the
    step serves every position.
    """

    # Batches up to this hand sums of squares from the residual epilogues to the next RMSNorm
    # (li4_fusion.sumsq_*); larger ones let the norm's GEMV read x once more instead.  Measured
    # (A/B on one B200): at batch 16 the hand-over costs 6% of the step (1.023 vs 0.966 ms); at
    # batch 4 it is even (0.7372 vs 0.7363 ms).
    sumsq_handoff_max_batch = 4

    def __init__(self, model, nvlink_allreduce: bool = True, program: bool = False, fused_allreduce: bool = True):
        self.model = model
        self.nvlink_allreduce = nvlink_allreduce
        self.fused_allreduce = fused_allreduce
        # single GPU: the whole step as one persistent launch (llama.program) where it applies
        self.use_program = program
        self._programs = {}
        self._fused_argmax = {}  # batch size -> whether the lm_head launch runs the greedy argmax
        self.last_path = None  # "program" or "launches": how the last decode_step ran
        self._ar = None  # NvlinkAllReduce of the model's TP group, built on first use
        p = model.params
        emb = model.tok_embeddings.weight
        self.device = emb.device
        if emb.dtype != torch.float16:
            raise TypeError("the fused decode step runs an fp16 model")
        freqs = model.freqs_cis.to(self.device)
        self.cos = freqs.real.float().contiguous()
        self.sin = freqs.imag.float().contiguous()
        self.blocks = [_Block(layer, self.cos, self.sin) for layer in model.layers]
        self.out = _qparams(model.output)
        self.final_norm = model.norm.weight.detach().contiguous()
        self.final_eps = float(model.norm.eps)
        self.dim = p.dim
        self.head_dim = p.dim // p.n_heads
        att0 = model.layers[0].attention
        self.n_heads = att0.n_local_heads
        self.n_kv_heads = att0.n_local_kv_heads
        self.ffn = model.layers[0].feed_forward.w1.out_features
        self.vocab_local = model.output.out_features
        self._bufs = {}

    def _buffers(self, bs: int):
        b = self._bufs.get(bs)
        if b is None:
            f16 = dict(dtype=torch.float16, device=self.device)
            b = {"h": torch.empty(bs, self.dim, **f16), "h1": torch.empty(bs, self.dim, **f16),
                 "q": torch.empty(bs, self.n_heads * self.head_dim, **f16),
                 "attn": torch.empty(bs, self.n_heads * self.head_dim, **f16),
                 "ffn": torch.empty(bs, self.ffn, **f16), "part": torch.empty(bs, self.dim, **f16),
                 # sums of squares of h / h1 per 16-row tile, from the residual epilogues to the next RMSNorm
                 "ssq_h": torch.zeros((self.dim + 15) // 16, bs, dtype=torch.float32, device=self.device),
                 "ssq_h1": torch.zeros((self.dim + 15) // 16, bs, dtype=torch.float32, device=self.device),
                 "logits": torch.empty(bs, self.vocab_local, dtype=torch.float32, device=self.device)}
            self._bufs[bs] = b
        return b

    def _allreduce_add(self, part: torch.Tensor, residual: torch.Tensor, out: torch.Tensor, group) -> None:
        import torch.distributed as dist

        dist.all_reduce(part, group=group)
        torch.add(residual, part, out=out)

    def _row_parallel(self, x: torch.Tensor, w, residual: torch.Tensor, out: torch.Tensor, part: torch.Tensor,
                      group, slot: int) -> None:
        """out = residual + allreduce(x @ w^T) for a row-parallel INT4 linear: in the GEMV's own launch
        (fused_allreduce), or the partial goes straight into this rank's NVLink communication slot and
        one kernel sums the ranks' slots (or NCCL)."""
        E = native
        if self.nvlink_allreduce:
            if self._ar is None:
                from .comm import NvlinkAllReduce

                self._ar = NvlinkAllReduce(group, max_elems=self.model.params.max_batch_size * self.dim,
                                           device=self.device, key_rows=max(64, self.model.params.max_batch_size))
            if self.fused_allreduce:
                int4_linear_fused(x, *w, out, self._ar.push_fusion(slot, residual))
                return
            int4_linear_fused(x, *w, None, E.Fusion(epilogue=E.LI4_EPI_STORE),
                              y_ptr=self._ar.slot_ptr(slot), y_stride=out.stride(0))
            self._ar.all_reduce_add(slot, residual, out)
        else:
            int4_linear_fused(x, *w, part, E.Fusion(epilogue=E.LI4_EPI_STORE))
            self._allreduce_add(part, residual, out, group)

    def _staging(self, bs: int):
        """Decoder-owned token / position buffers of the staged program (see _program)."""
        key = ("staging", bs)
        b = self._bufs.get(key)
        if b is None:
            i64 = dict(dtype=torch.long, device=self.device)
            b = {"tok": torch.zeros(bs, 1, **i64), "pos": torch.zeros(1, **i64), "out": torch.zeros(bs, 1, **i64)}
            self._bufs[key] = b
        return b

    def _program(self, tokens: torch.Tensor, pos: torch.Tensor, next_tokens: Optional[torch.Tensor],
                 advance_pos: bool):
        """(program, direct): the cached one-launch program of this step, built on first use (outside
        graph capture), or None where it does not apply (tensor parallelism, shapes it does not take).

        direct: the caller feeds the greedy tokens back in place (next_tokens is tokens, as
        DecodeGraph does), so the program reads tokens and pos and writes the next tokens and
        pos + 1 itself.  Otherwise (fresh tensors each step) one program per batch size reads
        decoder-owned buffers that decode_step fills with two small copies."""
        if not self.use_program or self.model.tp_group is not None:
            return None, False
        bs = tokens.shape[0]
        for blk in self.blocks:
            blk.att._ensure_cache(self._buffers(bs)["h"])
        caches = tuple(b.att.cache_k.data_ptr() for b in self.blocks)
        direct = next_tokens is not None and next_tokens.data_ptr() == tokens.data_ptr()
        key = ("direct", bs, tokens.data_ptr(), pos.data_ptr(), advance_pos, caches) if direct \
            else ("staged", bs, caches)
        if key in self._programs:
            return self._programs[key], direct
        from .program import decode_step_program

        try:
            if direct:
                prog = decode_step_program(self, tokens, pos, next_tokens, advance_pos)
            else:
                st = self._staging(bs)
                prog = decode_step_program(self, st["tok"], st["pos"], st["out"], False)
        except native.Li4Error as e:
            if e.status != native.LI4_ERR_UNSUPPORTED:
                raise
            prog = None  # e.g. a context longer than the program's attention holds: per-launch kernels
        self._programs[key] = prog
        return prog, direct

    @torch.no_grad()
    def decode_step(self, tokens: torch.Tensor, pos: torch.Tensor,
                    next_tokens: Optional[torch.Tensor] = None, advance_pos: bool = False) -> torch.Tensor:
        """fp32 logits [bs, 1, vocab]; with next_tokens (int64 [bs, 1], may be `tokens`) also
        the greedy argmax of each row, written on the GPU; with advance_pos, pos += 1 after the step."""
        bs = tokens.shape[0]
        prog, direct = self._program(tokens, pos, next_tokens, advance_pos)
        if prog is not None:
            if not direct:
                st = self._staging(bs)
                st["tok"].copy_(tokens.view(bs, 1))
                st["pos"].copy_(pos.view(1))
            prog.launch(native.stream_ptr(self.device))
            if not direct:
                if next_tokens is not None:
                    next_tokens.view(bs, 1).copy_(st["out"])
                if advance_pos:
                    pos.add_(1)
            self.last_path = "program"
            return self._buffers(bs)["logits"].view(bs, 1, -1)
        self.last_path = "launches"
        logits = self._decode_launches(tokens, pos, next_tokens)
        if advance_pos:
            pos.add_(1)
        return logits

    def _decode_launches(self, tokens: torch.Tensor, pos: torch.Tensor,
                         next_tokens: Optional[torch.Tensor]) -> torch.Tensor:
        """The step as five launches per block (and the tensor-parallel path)."""
        bs = tokens.shape[0]
        buf = self._buffers(bs)
        h, h1, q, attn, ffn, part = buf["h"], buf["h1"], buf["q"], buf["attn"], buf["ffn"], buf["part"]
        gather_rows(self.model.tok_embeddings.weight, tokens.view(-1), h)
        E = native
        ssq_h, ssq_h1 = buf["ssq_h"], buf["ssq_h1"]
        tiles = ssq_h.shape[0]
        handoff = bs <= self.sumsq_handoff_max_batch
        h_ssq = None  # the embedding rows carry no sums of squares: the first block's norm reads x
        for blk in self.blocks:
            att = blk.att
            att._ensure_cache(h)
            ck, cv = att.cache_k, att.cache_v
            f = E.Fusion(norm_weight=blk.attn_norm.data_ptr(), norm_eps=blk.attn_eps, epilogue=E.LI4_EPI_QKV_ROPE,
                         sumsq_in=h_ssq, sumsq_tiles=tiles if h_ssq else 0,
                         q_rows=blk.q_rows, k_rows=blk.k_rows, head_dim=self.head_dim, pos=pos.data_ptr(),
                         rope_cos=blk.cos.data_ptr(), rope_sin=blk.sin.data_ptr(), rope_stride=blk.cos.stride(0),
                         q_out=q.data_ptr(), stride_qm=q.stride(0), cache_k=ck.data_ptr(), cache_v=cv.data_ptr(),
                         cache_stride_b=ck.stride(0), cache_stride_s=ck.stride(1))
            int4_linear_fused(h, *blk.qkv, None, f)
            decode_attention(q, ck, cv, pos, attn, self.n_heads, self.n_kv_heads)
            if att.tp_group is None:
                f = E.Fusion(epilogue=E.LI4_EPI_RESIDUAL, residual=h.data_ptr(), stride_rm=h.stride(0),
                             sumsq_out=ssq_h1.data_ptr() if handoff else None)
                int4_linear_fused(attn, *blk.wo, h1, f)
                h1_ssq = ssq_h1.data_ptr() if handoff else None
            else:
                self._row_parallel(attn, blk.wo, h, h1, part, att.tp_group, slot=0)
                h1_ssq = None
            f = E.Fusion(norm_weight=blk.ffn_norm.data_ptr(), norm_eps=blk.ffn_eps, epilogue=E.LI4_EPI_SWIGLU,
                         sumsq_in=h1_ssq, sumsq_tiles=tiles if h1_ssq else 0)
            int4_linear_fused(h1, *blk.gate_up, ffn, f)
            if blk.ff.tp_group is None:
                f = E.Fusion(epilogue=E.LI4_EPI_RESIDUAL, residual=h1.data_ptr(), stride_rm=h1.stride(0),
                             sumsq_out=ssq_h.data_ptr() if handoff else None)
                int4_linear_fused(ffn, *blk.w2, h, f)
                h_ssq = ssq_h.data_ptr() if handoff else None
            else:
                self._row_parallel(ffn, blk.w2, h1, h, part, blk.ff.tp_group, slot=1)
                h_ssq = None
        logits = buf["logits"]  # fp32: the lm_head writes its fp16 outputs widened (output(h).float())
        f = E.Fusion(norm_weight=self.final_norm.data_ptr(), norm_eps=self.final_eps, epilogue=E.LI4_EPI_STORE_F32,
                     sumsq_in=h_ssq, sumsq_tiles=tiles if h_ssq else 0)
        # the greedy argmax in the lm_head's own launch where its plan takes it (single GPU)
        fuse_argmax = next_tokens is not None and self.model.tp_group is None and self._fused_argmax.get(bs, True)
        if fuse_argmax:
            scratch = self._bufs.get(("argmax", bs))
            if scratch is None:
                scratch = self._bufs[("argmax", bs)] = torch.zeros(8 * bs + 8, dtype=torch.uint8, device=self.device)
            nt = next_tokens.view(bs, 1)
            f.argmax_out, f.argmax_stride, f.argmax_scratch = nt.data_ptr(), nt.stride(0), scratch.data_ptr()
            try:
                int4_linear_fused(h, *self.out, None, f, y_ptr=logits.data_ptr(), y_stride=logits.stride(0))
                self._fused_argmax[bs] = True
                return logits.view(bs, 1, -1)
            except native.Li4Error as e:
                if e.status != native.LI4_ERR_UNSUPPORTED:
                    raise
                self._fused_argmax[bs] = False  # e.g. M > 8 runs the lm_head off the tile kernel
                f.argmax_out, f.argmax_stride, f.argmax_scratch = None, 0, None
        int4_linear_fused(h, *self.out, None, f, y_ptr=logits.data_ptr(), y_stride=logits.stride(0))
        if self.model.tp_group is not None:
            # vocabulary-sharded logits: each rank's winner as an ordered key, one int64 MAX all-reduce,
            # the winning global index -- instead of all-gathering bs x vocab fp32 logits
            import torch.distributed as dist

            if next_tokens is not None:
                shard = logits.shape[-1]
                offset = dist.get_rank(self.model.tp_group) * shard
                if self._ar is not None and self.fused_allreduce:
                    # the keys cross NVLink inside the argmax launch (li4_argmax_rows_allreduce)
                    self._ar.argmax_allreduce(logits, offset, next_tokens.view(bs, 1))
                else:
                    keys = self._bufs.get(("keys", bs))
                    if keys is None:
                        keys = self._bufs[("keys", bs)] = torch.empty(bs, 1, dtype=torch.long, device=self.device)
                    argmax_rows_keys(logits, offset, keys)
                    dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=self.model.tp_group)
                    next_tokens.view(bs, 1).copy_(key_index(keys))
            return logits.view(bs, 1, -1)  # this rank's vocabulary shard
        if next_tokens is not None:
            argmax_rows(logits, next_tokens.view(bs, 1))
        return logits.view(bs, 1, -1)
