"""Decode programs: a list of ops run by one persistent launch (li4_program_*).

`Program` wraps the C-ABI builder: add ops (INT4 linears with their fusion,
decode attention, the embedding gather, the greedy argmax), finalize once
outside CUDA-graph capture, then `launch()` on the current stream as often as
needed -- a launch is capturable.  Every op reads the pointers it was given at
each launch; an op with `wait=j` reads its inputs only after every CTA has
finished op j.

`decode_step_program` builds the fused decode step of `llama.fused.FusedDecoder`
as one program: embedding gather, then per block QKV (RMSNorm prologue, RoPE and
KV-cache epilogue), attention, wo (+ residual), gate/up (RMSNorm prologue,
SwiGLU epilogue), w2 (+ residual), and the lm_head (final RMSNorm, fp32 logits)
followed by the greedy argmax -- the same ops and arithmetic as the per-launch
step, in one launch instead of 5 per block + 4.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _native as native

NO_WAIT = -1


class Program:
    """One decode program on the current CUDA device."""

    def __init__(self):
        self._lib = native.lib()
        h = ctypes.c_void_p()
        native.check(self._lib.li4_program_create(ctypes.byref(h)), "program_create")
        self._h = h
        self._keep = []  # tensors whose addresses the ops hold
        self.n_ops = 0
        self.finalized = False

    def _added(self, rc: int, what: str, idx: ctypes.c_int, *tensors) -> int:
        native.check(rc, what)
        self._keep.extend(t for t in tensors if isinstance(t, torch.Tensor))
        self.n_ops += 1
        return idx.value

    def linear(self, x: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor,
               y: Optional[torch.Tensor], fusion: Optional[native.Fusion] = None, wait: int = NO_WAIT,
               group_size: int = 128, y_ptr: Optional[int] = None, y_stride: int = 0, keep=()) -> int:
        """y = x @ W^T (+ fusion) for x [M, K] fp16 row-contiguous; returns the op index."""
        M, K = x.shape
        N = packed.shape[0]
        if y_ptr is None:
            y_ptr = y.data_ptr() if y is not None else None
            y_stride = y.stride(0) if y is not None else 0
        idx = ctypes.c_int(-1)
        rc = self._lib.li4_program_add_linear(self._h, x.data_ptr(), packed.data_ptr(), scale.data_ptr(),
                                              zero.data_ptr(), y_ptr, M, N, K, group_size, x.stride(0),
                                              packed.stride(0), scale.stride(0), y_stride,
                                              ctypes.byref(fusion) if fusion is not None else None, wait,
                                              ctypes.byref(idx))
        return self._added(rc, "program_add_linear", idx, x, packed, scale, zero, y, *keep)

    def attention(self, q: torch.Tensor, cache_k: torch.Tensor, cache_v: torch.Tensor, pos: torch.Tensor,
                  out: torch.Tensor, n_heads: int, n_kv_heads: int, wait: int = NO_WAIT) -> int:
        """Decode attention as llama.fused.decode_attention: q / out [bs, n_heads * head_dim],
        caches [bs, max_seq, n_kv_heads, head_dim]."""
        max_seq = cache_k.shape[1]
        head_dim = q.shape[-1] // n_heads
        idx = ctypes.c_int(-1)
        rc = self._lib.li4_program_add_attention(self._h, q.data_ptr(), q.stride(0), cache_k.data_ptr(),
                                                 cache_v.data_ptr(), cache_k.stride(0), cache_k.stride(1),
                                                 out.data_ptr(), out.stride(0), q.shape[0], n_heads, n_kv_heads,
                                                 head_dim, pos.data_ptr(), max_seq, wait, ctypes.byref(idx))
        return self._added(rc, "program_add_attention", idx, q, cache_k, cache_v, pos, out)

    def gather(self, table: torch.Tensor, ids: torch.Tensor, out: torch.Tensor, wait: int = NO_WAIT) -> int:
        """out[r] = table[ids[r]] (the embedding lookup)."""
        idx = ctypes.c_int(-1)
        rc = self._lib.li4_program_add_gather(self._h, table.data_ptr(), table.shape[0], table.shape[1],
                                              table.stride(0), ids.data_ptr(), ids.numel(), out.data_ptr(),
                                              out.stride(0), wait, ctypes.byref(idx))
        return self._added(rc, "program_add_gather", idx, table, ids, out)

    def argmax(self, logits: torch.Tensor, out: torch.Tensor, wait: int = NO_WAIT) -> int:
        """out[r] = argmax(logits[r]) for fp32 logits [rows, cols]; out int64 with one index per row."""
        rows, cols = logits.shape
        idx = ctypes.c_int(-1)
        rc = self._lib.li4_program_add_argmax(self._h, logits.data_ptr(), rows, cols, logits.stride(0),
                                              out.data_ptr(), out.stride(0) if out.dim() > 1 else 1, wait,
                                              ctypes.byref(idx))
        return self._added(rc, "program_add_argmax", idx, logits, out)

    def increment(self, value: torch.Tensor) -> None:
        """value (int64, one element) += 1 after every op of a launch."""
        native.check(self._lib.li4_program_add_increment(self._h, value.data_ptr()), "program_add_increment")
        self._keep.append(value)

    def finalize(self) -> "Program":
        native.check(self._lib.li4_program_finalize(self._h), "program_finalize")
        self.finalized = True
        return self

    def info(self) -> dict:
        ctas, stages, smem = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_size_t(0)
        native.check(self._lib.li4_program_info(self._h, ctypes.byref(ctas), ctypes.byref(stages),
                                                ctypes.byref(smem)), "program_info")
        return {"ctas": ctas.value, "stages": stages.value, "smem_bytes": smem.value, "ops": self.n_ops}

    def set_trace(self, stamps: Optional[torch.Tensor]) -> None:
        """Record per-op globaltimer stamps of later launches into stamps (int64 [ops, ctas, 4]; None: off)."""
        cap = stamps.numel() if stamps is not None else 0
        native.check(self._lib.li4_program_set_trace(self._h, stamps.data_ptr() if stamps is not None else None, cap),
                     "program_set_trace")
        if stamps is not None:
            self._keep.append(stamps)

    def launch(self, stream: Optional[int] = None) -> None:
        if stream is None:
            stream = torch.cuda.current_stream().cuda_stream
        native.check(self._lib.li4_program_launch(self._h, stream), "program_launch")

    def close(self) -> None:
        if self._h is not None and self._h.value:
            self._lib.li4_program_destroy(self._h)
        self._h = None
        self._keep = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def decode_step_program(dec, tokens: torch.Tensor, pos: torch.Tensor, next_tokens: Optional[torch.Tensor],
                        advance_pos: bool = False) -> Program:
    """The fused decode step of FusedDecoder `dec` at batch tokens.shape[0] as one program:
    tokens [bs, 1] in, fp32 logits in dec's buffer, greedy tokens into next_tokens (may be tokens),
    pos += 1 at the end with advance_pos.  Single GPU (no tensor parallelism)."""
    E = native
    bs = tokens.shape[0]
    buf = dec._buffers(bs)
    h, h1, q, attn, ffn = buf["h"], buf["h1"], buf["q"], buf["attn"], buf["ffn"]
    logits = buf["logits"]
    prog = Program()
    last = prog.gather(dec.model.tok_embeddings.weight, tokens.view(-1), h)
    for blk in dec.blocks:
        att = blk.att
        att._ensure_cache(h)
        ck, cv = att.cache_k, att.cache_v
        f = E.Fusion(norm_weight=blk.attn_norm.data_ptr(), norm_eps=blk.attn_eps, epilogue=E.LI4_EPI_QKV_ROPE,
                     q_rows=blk.q_rows, k_rows=blk.k_rows, head_dim=dec.head_dim, pos=pos.data_ptr(),
                     rope_cos=blk.cos.data_ptr(), rope_sin=blk.sin.data_ptr(), rope_stride=blk.cos.stride(0),
                     q_out=q.data_ptr(), stride_qm=q.stride(0), cache_k=ck.data_ptr(), cache_v=cv.data_ptr(),
                     cache_stride_b=ck.stride(0), cache_stride_s=ck.stride(1))
        last = prog.linear(h, *blk.qkv, None, f, wait=last, keep=(blk.attn_norm, blk.cos, blk.sin, pos, q, ck, cv))
        last = prog.attention(q, ck, cv, pos, attn, dec.n_heads, dec.n_kv_heads, wait=last)
        f = E.Fusion(epilogue=E.LI4_EPI_RESIDUAL, residual=h.data_ptr(), stride_rm=h.stride(0))
        last = prog.linear(attn, *blk.wo, h1, f, wait=last, keep=(h,))
        f = E.Fusion(norm_weight=blk.ffn_norm.data_ptr(), norm_eps=blk.ffn_eps, epilogue=E.LI4_EPI_SWIGLU)
        last = prog.linear(h1, *blk.gate_up, ffn, f, wait=last, keep=(blk.ffn_norm,))
        f = E.Fusion(epilogue=E.LI4_EPI_RESIDUAL, residual=h1.data_ptr(), stride_rm=h1.stride(0))
        last = prog.linear(ffn, *blk.w2, h, f, wait=last, keep=(h1,))
    f = E.Fusion(norm_weight=dec.final_norm.data_ptr(), norm_eps=dec.final_eps, epilogue=E.LI4_EPI_STORE_F32)
    last = prog.linear(h, *dec.out, None, f, wait=last, y_ptr=logits.data_ptr(), y_stride=logits.stride(0),
                       keep=(dec.final_norm, logits))
    if next_tokens is not None:
        prog.argmax(logits, next_tokens.view(bs, 1), wait=last)
    if advance_pos:
        prog.increment(pos)
    return prog.finalize()
