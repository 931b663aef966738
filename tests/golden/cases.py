"""Seeded input generators shared by make_golden.py and the tests.

Every case is regenerated from its seed with torch's CPU generator, so the
committed fixtures only need the outputs (and, for large cases, hashes).
Weights follow the reference's random-weight recipe, N(0, 0.02) in fp16
(int4_gemv_bench.py:67, dequant_traffic.py:159); activations are N(0, 1) fp16.
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch

# name, N (out_features), K (in_features), M (rows of x), group_size, weight kind, seed
GEMV_CASES = [
    ("tiny", 16, 128, 1, 128, "normal", 11),
    ("odd_rows", 33, 256, 3, 128, "normal", 12),
    ("g32", 64, 512, 5, 32, "normal", 13),
    ("g64", 48, 384, 2, 64, "normal", 14),
    ("g256", 40, 1024, 4, 256, "normal", 15),
    ("m16", 80, 1024, 16, 128, "normal", 16),
    ("edge_rows", 24, 256, 4, 128, "edge", 17),
    ("big_x", 64, 512, 2, 128, "normal_big_x", 18),
    ("kv_m1", 512, 2048, 1, 128, "normal", 19),
    ("q_m8", 2048, 2048, 8, 128, "normal", 20),
    ("down_m2", 2048, 8192, 2, 128, "normal", 21),
    ("config0", 8192, 2048, 1, 128, "config0", 0),
]

# cases small enough to store every array in full
FULL_CASES = {"tiny", "odd_rows", "g32", "g64", "g256", "m16", "edge_rows", "big_x"}

# check_impl.py:86-103 quantizer shapes
QUANT_CASES = [
    ("check_shapes_g32", 128, 256, 32, 1.0, 31),  # check_impl.py:86-93
    ("roundtrip_g128", 256, 512, 128, 0.1, 32),  # check_impl.py:95-103
    ("huge_g128", 16, 256, 128, 3000.0, 33),  # large magnitudes, W16 still finite
    ("edge_g64", 32, 256, 64, "edge", 34),  # the edge rows of _edge_weights
]


def sha256(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _edge_weights(N: int, K: int, gen: torch.Generator) -> torch.Tensor:
    """Rows that exercise the quantizer's corner cases, one kind per row (cycled)."""
    w = torch.empty(N, K)
    for n in range(N):
        kind = n % 8
        if kind == 0:  # all zero: scale 0 -> 1, zero point -0.0
            w[n] = 0.0
        elif kind == 1:  # constant positive: scale 0 -> 1
            w[n] = 0.375
        elif kind == 2:  # non-negative with exact zeros: zero point from -(+0)
            w[n] = torch.rand(K, generator=gen)
            w[n, ::7] = 0.0
        elif kind == 3:  # min 0, max 15 in each group -> scale 1, exact .5 ties round half to even
            base = torch.arange(K, dtype=torch.float32) % 31 * 0.5
            base[::64] = 0.0
            base[1::64] = 15.0
            w[n] = base
        elif kind == 4:  # large magnitudes (outputs stay finite in fp16)
            w[n] = torch.randn(K, generator=gen) * 300.0
        elif kind == 5:  # tiny magnitudes: fp16-subnormal scales
            w[n] = torch.randn(K, generator=gen) * 2e-6
        elif kind == 6:  # all negative
            w[n] = -torch.rand(K, generator=gen) - 0.01
        else:  # one outlier per group
            w[n] = torch.randn(K, generator=gen) * 0.02
            w[n, 5::128] = 3.0
    return w.half()


def make_gemv_inputs(case) -> tuple[torch.Tensor, torch.Tensor]:
    """-> (W fp16 [N, K], x fp16 [M, K]) on the CPU."""
    name, N, K, M, group, kind, seed = case
    gen = torch.Generator().manual_seed(seed)
    if kind == "config0":
        # seed 0: x = randn(1, 2048), then W = randn(8192, 2048) * 0.02, both to fp16
        x = torch.randn(M, K, generator=gen).half()
        w = (torch.randn(N, K, generator=gen) * 0.02).half()
        return w, x
    if kind == "edge":
        w = _edge_weights(N, K, gen)
    else:
        w = (torch.randn(N, K, generator=gen) * 0.02).half()
    x = torch.randn(M, K, generator=gen)
    if kind == "normal_big_x":
        x = x * 100.0
    return w, x.half()


def make_quant_input(case) -> torch.Tensor:
    name, N, K, group, mult, seed = case
    gen = torch.Generator().manual_seed(seed)
    if mult == "edge":
        return _edge_weights(N, K, gen)
    return (torch.randn(N, K, generator=gen) * mult).half()


# ---------------------------------------------------------------------------
# Tiny Llama for model-level golden vectors (same architecture, small sizes;
# every K is a multiple of 128 so the INT4 kernels take it).
# ---------------------------------------------------------------------------
TINY_MODEL = dict(dim=256, n_layers=2, n_heads=8, n_kv_heads=2, vocab_size=1000, multiple_of=64,
                  ffn_dim_multiplier=1.5, norm_eps=1e-5, rope_theta=500000.0, max_batch_size=2, max_seq_len=24)
# the same shape family with 8 KV heads and K shards of whole 128-groups at 2, 4 and 8 ranks
TP_MODEL = dict(dim=1024, n_layers=2, n_heads=16, n_kv_heads=8, vocab_size=1024, multiple_of=1024,
                ffn_dim_multiplier=1.5, norm_eps=1e-5, rope_theta=500000.0, max_batch_size=2, max_seq_len=24)
TINY_PROMPT_LEN = 8
TINY_DECODE_STEPS = 6
TINY_SEED = 77


def tiny_state_dict(args: dict, seed: int = TINY_SEED) -> dict:
    """Seeded fp16 weights keyed like the reference's Llama state dict."""
    gen = torch.Generator().manual_seed(seed)
    dim, L = args["dim"], args["n_layers"]
    hd = dim // args["n_heads"]
    kv = args["n_kv_heads"] * hd
    hidden = int(2 * 4 * dim / 3)
    hidden = int(args["ffn_dim_multiplier"] * hidden)
    hidden = args["multiple_of"] * ((hidden + args["multiple_of"] - 1) // args["multiple_of"])

    def randn(*shape, std):
        return (torch.randn(*shape, generator=gen) * std).half()

    sd = {"tok_embeddings.weight": randn(args["vocab_size"], dim, std=1.0)}
    for i in range(L):
        p = f"layers.{i}."
        sd[p + "attention.wq.weight"] = randn(dim, dim, std=0.05)
        sd[p + "attention.wk.weight"] = randn(kv, dim, std=0.05)
        sd[p + "attention.wv.weight"] = randn(kv, dim, std=0.05)
        sd[p + "attention.wo.weight"] = randn(dim, dim, std=0.05)
        sd[p + "feed_forward.w1.weight"] = randn(hidden, dim, std=0.05)
        sd[p + "feed_forward.w2.weight"] = randn(dim, hidden, std=0.05)
        sd[p + "feed_forward.w3.weight"] = randn(hidden, dim, std=0.05)
        sd[p + "attention_norm.weight"] = (1.0 + 0.1 * torch.randn(dim, generator=gen)).half()
        sd[p + "ffn_norm.weight"] = (1.0 + 0.1 * torch.randn(dim, generator=gen)).half()
    sd["norm.weight"] = (1.0 + 0.1 * torch.randn(dim, generator=gen)).half()
    sd["output.weight"] = randn(args["vocab_size"], dim, std=0.05)
    return sd


def tiny_prompt(args: dict, seed: int = TINY_SEED + 1) -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(0, args["vocab_size"], (args["max_batch_size"], TINY_PROMPT_LEN), generator=gen)
