"""Llama-3.2-1B for INT4 decode on B200: same modules, parameter names and math as the
reference's llama/model.py, plus a decode step that takes its position from a device
tensor so one CUDA graph serves every position.

Module tree and state-dict keys match llama/model.py:167-456 (tok_embeddings,
layers.{i}.attention.{wq,wk,wv,wo}, layers.{i}.feed_forward.{w1,w2,w3},
layers.{i}.{attention_norm,ffn_norm}, norm, output), so the reference's
checkpoints load and quantize_model() swaps the same 113 nn.Linear modules for
QuantizedLinear.  forward(tokens, start_pos) has the reference's semantics
(llama/model.py:419-456), including the fp16/fp32 boundaries of RMSNorm
(:61, :74-75), RoPE on (even, odd) pairs as complex numbers (:126-152) and the
fp32 softmax (:274).

Additions:
  * ModelArgs.use_scaled_rope: the llama3 RoPE frequency scaling (factor 32,
    low/high frequency factors 1/4, original context 8192), which the reference
    lacks; off by default so logits match the reference.
  * Llama.decode_step(tokens, pos): one token per sequence at the position held
    in the int64 device tensor `pos`; the KV-cache write, the RoPE row and the
    attention mask all index through it.  Attention runs over the whole cache
    with positions > pos masked to -inf, which gives the reference's softmax
    over [0, pos] (masked entries contribute exact zeros).
  * The grouped-query attention reads the cache without the materialised
    repeat_kv copy (llama/model.py:155-164, 265-266): queries are grouped per
    KV head instead.
  * Tensor parallelism (llama/tp.py) sets n_local_heads / n_local_kv_heads and
    a process group; row-parallel outputs are all-reduced, vocab shards of the
    logits all-gathered.
  * Llama.enable_fused_decode(): decode_step through llama.fused (RMSNorm, RoPE,
    KV-cache writes, SwiGLU and residual adds folded into the INT4 GEMVs, one
    attention kernel per block).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn.functional as F
from torch import nn

from .generation import Generation


@dataclass
class ModelArgs:  # Llama 3.2-1B, llama/model.py:15-30
    dim: int = 2048
    n_layers: int = 16
    n_heads: int = 32
    n_kv_heads: int = 8
    vocab_size: int = 128256
    multiple_of: int = 1024
    ffn_dim_multiplier: float = 1.5
    norm_eps: float = 1e-5
    rope_theta: float = 500000
    max_batch_size: int = 4
    max_seq_len: int = 256
    kv_caching: bool = True
    use_scaled_rope: bool = False


class RMSNorm(torch.nn.Module):
    """Root-mean-square norm with the reference's fp16 / fp32 boundaries (llama/model.py:32-75): the
    statistics and the scaling in fp32, the result cast back to the input dtype, then the weight."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        inv_rms = torch.rsqrt(xf.square().mean(-1, keepdim=True) + self.eps)
        return (xf * inv_rms).type_as(x) * self.weight


def apply_llama3_scaling(freqs: torch.Tensor, factor: float = 32.0, low_freq_factor: float = 1.0,
                         high_freq_factor: float = 4.0, old_context_len: int = 8192) -> torch.Tensor:
    """Llama 3.x RoPE frequency scaling: long wavelengths divided by `factor`, short ones kept,
    a linear blend in between (the published llama3 rope_scaling rule)."""
    low_freq_wavelen = old_context_len / low_freq_factor
    high_freq_wavelen = old_context_len / high_freq_factor
    out = []
    for f in freqs.tolist():
        wavelen = 2 * math.pi / f
        if wavelen < high_freq_wavelen:
            out.append(f)
        elif wavelen > low_freq_wavelen:
            out.append(f / factor)
        else:
            smooth = (old_context_len / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor)
            out.append((1 - smooth) * f / factor + smooth * f)
    return torch.tensor(out, dtype=freqs.dtype, device=freqs.device)


def rope_frequencies(head_dim: int, theta: float, use_scaled: bool = False) -> torch.Tensor:
    """Per-pair angular frequencies theta^(-2i / head_dim), i < head_dim / 2, in fp32 (computed as the
    reciprocal of the power, the reference's rounding: llama/model.py:78-98)."""
    exponents = torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim
    freqs = 1.0 / (theta ** exponents)
    return apply_llama3_scaling(freqs) if use_scaled else freqs


def precompute_freqs_cis(dim: int, end: int, theta: float = 10000.0, use_scaled: bool = False):
    """Unit complex rotations e^{i t f} (complex64 [end, dim/2]) for positions t < end."""
    angles = torch.outer(torch.arange(end), rope_frequencies(dim, theta, use_scaled)).float()
    return torch.polar(torch.ones_like(angles), angles)


def _rotate(x: torch.Tensor, rot: torch.Tensor) -> torch.Tensor:
    """x [b, s, heads, d] as d/2 complex (even, odd) pairs in fp32, times rot [s, d/2]."""
    pairs = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
    rotated = pairs * rot[None, :, None, :]
    return torch.view_as_real(rotated).flatten(3).type_as(x)


def apply_rotary_emb(xq: torch.Tensor, xk: torch.Tensor, freqs_cis: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """RoPE on queries and keys: pairs rotated as complex numbers in fp32, cast back
    (llama/model.py:126-152)."""
    if freqs_cis.shape != (xq.shape[1], xq.shape[-1] // 2):
        raise ValueError(f"rotations {tuple(freqs_cis.shape)} do not match {tuple(xq.shape)}")
    return _rotate(xq, freqs_cis), _rotate(xk, freqs_cis)


def ffn_hidden_dim(dim: int, multiple_of: int, ffn_dim_multiplier: Optional[float]) -> int:
    """SwiGLU width: 2/3 of 4*dim, times the multiplier, rounded up to multiple_of (8192 for
    Llama-3.2-1B; llama/model.py:296-308)."""
    hidden = int(2 * (4 * dim) / 3)
    if ffn_dim_multiplier is not None:
        hidden = int(ffn_dim_multiplier * hidden)
    return -(-hidden // multiple_of) * multiple_of


class Attention(nn.Module):
    def __init__(self, args: ModelArgs):
        super().__init__()
        self.n_kv_heads = args.n_heads if args.n_kv_heads is None else args.n_kv_heads
        self.n_local_heads = args.n_heads
        self.n_local_kv_heads = self.n_kv_heads
        self.n_rep = self.n_local_heads // self.n_local_kv_heads
        self.head_dim = args.dim // args.n_heads
        self.wq = nn.Linear(args.dim, args.n_heads * self.head_dim, bias=False)
        self.wk = nn.Linear(args.dim, self.n_kv_heads * self.head_dim, bias=False)
        self.wv = nn.Linear(args.dim, self.n_kv_heads * self.head_dim, bias=False)
        self.wo = nn.Linear(args.n_heads * self.head_dim, args.dim, bias=False)
        self.kv_caching = args.kv_caching
        self.max_batch_size = args.max_batch_size
        self.max_seq_len = args.max_seq_len
        self.cache_k: Optional[torch.Tensor] = None
        self.cache_v: Optional[torch.Tensor] = None
        self.tp_group = None  # set by llama.tp.shard_model

    def _ensure_cache(self, like: torch.Tensor):
        shape = (self.max_batch_size, self.max_seq_len, self.n_local_kv_heads, self.head_dim)
        if self.cache_k is None or self.cache_k.device != like.device or self.cache_k.dtype != like.dtype \
                or tuple(self.cache_k.shape) != shape:
            # ordinary tensors even when first reached under inference_mode, so later
            # in-place cache writes work in any grad mode
            with torch.inference_mode(False):
                self.cache_k = torch.zeros(shape, dtype=like.dtype, device=like.device)
                self.cache_v = torch.zeros(shape, dtype=like.dtype, device=like.device)

    def _reduce(self, out: torch.Tensor) -> torch.Tensor:
        if self.tp_group is not None:
            import torch.distributed as dist

            dist.all_reduce(out, group=self.tp_group)
        return out

    def forward(self, x: torch.Tensor, start_pos: int, freqs_cis: torch.Tensor, mask: Optional[torch.Tensor]):
        """The reference's attention (llama/model.py:222-277) with a Python start_pos."""
        bsz, seqlen, _ = x.shape
        xq, xk, xv = self.wq(x), self.wk(x), self.wv(x)
        xq = xq.view(bsz, seqlen, self.n_local_heads, self.head_dim)
        xk = xk.view(bsz, seqlen, self.n_local_kv_heads, self.head_dim)
        xv = xv.view(bsz, seqlen, self.n_local_kv_heads, self.head_dim)
        xq, xk = apply_rotary_emb(xq, xk, freqs_cis=freqs_cis)
        if self.kv_caching:
            self._ensure_cache(xq)
            self.cache_k[:bsz, start_pos: start_pos + seqlen] = xk
            self.cache_v[:bsz, start_pos: start_pos + seqlen] = xv
            keys = self.cache_k[:bsz, : start_pos + seqlen]
            values = self.cache_v[:bsz, : start_pos + seqlen]
        else:
            keys, values = xk, xv
        output = self._attend(xq, keys, values, mask)
        return self._reduce(self.wo(output.view(bsz, seqlen, -1)))

    def _attend(self, xq, keys, values, bias):
        """softmax(q k^T / sqrt(d) + bias) v with grouped KV heads.
        xq [b, s, H, d]; keys/values [b, L, Hkv, d]; bias broadcastable to [s, L] or None."""
        b, s, H, d = xq.shape
        Hkv = keys.shape[2]
        rep = H // Hkv
        q = xq.view(b, s, Hkv, rep, d).permute(0, 2, 3, 1, 4).reshape(b, Hkv, rep * s, d)  # [b, Hkv, rep*s, d]
        k = keys.permute(0, 2, 3, 1)  # [b, Hkv, d, L]
        v = values.transpose(1, 2)  # [b, Hkv, L, d]
        scores = torch.matmul(q, k) / math.sqrt(self.head_dim)  # fp16, as the reference (:271)
        scores = scores.view(b, Hkv, rep, s, -1)
        if bias is not None:
            scores = scores + bias
        scores = F.softmax(scores.float(), dim=-1).type_as(xq)  # (:274)
        out = torch.matmul(scores.view(b, Hkv, rep * s, -1), v)  # [b, Hkv, rep*s, d]
        return out.view(b, Hkv, rep, s, d).permute(0, 3, 1, 2, 4).reshape(b, s, H * d).contiguous()

    def decode(self, x: torch.Tensor, pos: torch.Tensor, freqs_row: torch.Tensor, bias: torch.Tensor):
        """One new token per sequence at device position `pos` (int64 [1])."""
        bsz = x.shape[0]
        xq, xk, xv = self.wq(x), self.wk(x), self.wv(x)
        xq = xq.view(bsz, 1, self.n_local_heads, self.head_dim)
        xk = xk.view(bsz, 1, self.n_local_kv_heads, self.head_dim)
        xv = xv.view(bsz, 1, self.n_local_kv_heads, self.head_dim)
        xq, xk = apply_rotary_emb(xq, xk, freqs_cis=freqs_row)
        self._ensure_cache(xq)
        self.cache_k[:bsz].index_copy_(1, pos, xk)
        self.cache_v[:bsz].index_copy_(1, pos, xv)
        output = self._attend(xq, self.cache_k[:bsz], self.cache_v[:bsz], bias)
        return self._reduce(self.wo(output))


class FeedForward(nn.Module):
    def __init__(self, dim: int, hidden_dim: int, multiple_of: int, ffn_dim_multiplier: Optional[float]):
        super().__init__()
        hidden_dim = ffn_hidden_dim(hidden_dim // 4, multiple_of, ffn_dim_multiplier)
        self.w1 = nn.Linear(dim, hidden_dim, bias=False)
        self.w2 = nn.Linear(hidden_dim, dim, bias=False)
        self.w3 = nn.Linear(dim, hidden_dim, bias=False)
        self.tp_group = None

    def forward(self, x):
        out = self.w2(F.silu(self.w1(x)) * self.w3(x))
        if self.tp_group is not None:
            import torch.distributed as dist

            dist.all_reduce(out, group=self.tp_group)
        return out


class TransformerBlock(nn.Module):
    def __init__(self, layer_id: int, args: ModelArgs):
        super().__init__()
        self.n_heads = args.n_heads
        self.dim = args.dim
        self.head_dim = args.dim // args.n_heads
        self.attention = Attention(args)
        self.feed_forward = FeedForward(dim=args.dim, hidden_dim=4 * args.dim, multiple_of=args.multiple_of,
                                        ffn_dim_multiplier=args.ffn_dim_multiplier)
        self.layer_id = layer_id
        self.attention_norm = RMSNorm(args.dim, eps=args.norm_eps)
        self.ffn_norm = RMSNorm(args.dim, eps=args.norm_eps)

    def forward(self, x, start_pos: int, freqs_cis, mask):
        h = x + self.attention(self.attention_norm(x), start_pos, freqs_cis, mask)
        return h + self.feed_forward(self.ffn_norm(h))

    def decode(self, x, pos, freqs_row, bias):
        h = x + self.attention.decode(self.attention_norm(x), pos, freqs_row, bias)
        return h + self.feed_forward(self.ffn_norm(h))


class Llama(Generation):
    def __init__(self, params: ModelArgs):
        super().__init__()
        self.params = params
        self.vocab_size = params.vocab_size
        self.n_layers = params.n_layers
        self.tok_embeddings = nn.Embedding(params.vocab_size, params.dim)
        self.layers = torch.nn.ModuleList()
        for layer_id in range(params.n_layers):
            self.layers.append(TransformerBlock(layer_id, params))
        self.norm = RMSNorm(params.dim, eps=params.norm_eps)
        self.output = nn.Linear(params.dim, params.vocab_size, bias=False)
        self.freqs_cis = precompute_freqs_cis(params.dim // params.n_heads, params.max_seq_len * 2,
                                              params.rope_theta, params.use_scaled_rope)
        self.tp_group = None  # vocab-sharded lm_head when set (llama.tp)
        self.tp_world = 1

    def _logits(self, h: torch.Tensor) -> torch.Tensor:
        out = self.output(h)
        if self.tp_group is not None:
            import torch.distributed as dist

            parts = [torch.empty_like(out) for _ in range(self.tp_world)]
            dist.all_gather(parts, out.contiguous(), group=self.tp_group)
            out = torch.cat(parts, dim=-1)
        return out.float()

    def forward(self, tokens: torch.Tensor, start_pos: int):
        """Logits [b, s, vocab] fp32 for tokens [b, s] at Python position start_pos (llama/model.py:419-456)."""
        _bsz, seqlen = tokens.shape
        h = self.tok_embeddings(tokens)
        self.freqs_cis = self.freqs_cis.to(h.device)
        freqs_cis = self.freqs_cis[start_pos: start_pos + seqlen]
        mask = None
        if seqlen > 1:
            mask = torch.full((seqlen, seqlen), float("-inf"), device=tokens.device)
            mask = torch.triu(mask, diagonal=1)
            if start_pos > 0:
                mask = torch.cat([torch.zeros(seqlen, start_pos, device=tokens.device), mask], dim=1)
        for layer in self.layers:
            h = layer(h, start_pos, freqs_cis, mask)
        h = self.norm(h)
        return self._logits(h)

    def decode_step(self, tokens: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """Logits [b, 1, vocab] fp32 for tokens [b, 1] at the device position pos (int64 [1]).

        Every operation is a device operation with static shapes, so the step can be
        captured once in a CUDA graph and replayed for any position.  After
        enable_fused_decode() the step runs as fused kernels (llama.fused)."""
        if getattr(self, "_fused", None) is not None:
            return self._fused.decode_step(tokens, pos)
        h = self.tok_embeddings(tokens)
        self.freqs_cis = self.freqs_cis.to(h.device)
        freqs_row = self.freqs_cis.index_select(0, pos)  # [1, head_dim/2]
        L = self.params.max_seq_len
        idx = torch.arange(L, device=h.device)
        bias = torch.zeros(L, dtype=h.dtype, device=h.device).masked_fill(idx > pos, float("-inf"))
        for layer in self.layers:
            h = layer.decode(h, pos, freqs_row, bias)
        h = self.norm(h)
        return self._logits(h)

    def enable_fused_decode(self, enabled: bool = True, nvlink_allreduce: bool = True, program: bool = False,
                            fused_allreduce: bool = True):
        """Run decode_step as the fused INT4 kernels of llama.fused (five launches per block, or with
        program=True the whole step as one persistent launch, llama.program, on a single GPU).
        Needs a quantized fp16 model on a CUDA device; shares this model's KV caches.  Under tensor
        parallelism the row-parallel sums go over NVLink peer memory (llama.comm) inside the GEMV's
        launch (fused_allreduce) or in a kernel of their own, or through NCCL."""
        if enabled:
            from .fused import FusedDecoder

            self._fused = FusedDecoder(self, nvlink_allreduce=nvlink_allreduce, program=program,
                                       fused_allreduce=fused_allreduce)
        else:
            self._fused = None
        return self

    def reset_cache(self):
        for layer in self.layers:
            layer.attention.cache_k = None
            layer.attention.cache_v = None
