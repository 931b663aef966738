"""Tensor parallelism for the INT4 decode model (new here: the reference has none).

Column-parallel (output features split, no communication):
    wq, wk, wv   by heads   (rows of packed / scale / zero_point are head-major,
                             llama/model.py:245-247)
    w1, w3       by hidden features
    output       by vocabulary entries -> logits all-gathered
Row-parallel (input features split, outputs all-reduced):
    wo           by heads   (its input is the concatenated head outputs)
    w2           by hidden features
Every K shard is a whole number of quantization groups, so a shard of an INT4
layer is an INT4 layer of the same format: packed[:, k0/2 : k1/2] and
scale / zero_point[:, k0/g : k1/g].  Embeddings and norms are replicated.

The collectives are torch.distributed calls on the given process group (NCCL
over NVLink on GPUs, gloo on CPUs); they are captured into the decode CUDA graph
like every other launch.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from .quantize import QuantizedLinear


def _span(total: int, rank: int, world: int, what: str, multiple: int = 1):
    if total % world or (total // world) % multiple:
        raise ValueError(f"{what}: {total} does not split into {world} shards of a multiple of {multiple}")
    size = total // world
    return rank * size, (rank + 1) * size


def shard_int4_rows(packed, scale, zero, rank: int, world: int):
    """Output-feature shard [N/world rows] of INT4 buffers."""
    r0, r1 = _span(packed.shape[0], rank, world, "out_features")
    return packed[r0:r1].contiguous(), scale[r0:r1].contiguous(), zero[r0:r1].contiguous()


def shard_int4_cols(packed, scale, zero, rank: int, world: int, group_size: int):
    """Input-feature shard [K/world columns] of INT4 buffers; K/world must hold whole groups
    (and stay a multiple of 128 for the fused kernels)."""
    K = packed.shape[1] * 2
    k0, k1 = _span(K, rank, world, "in_features", multiple=max(group_size, 128))
    return (packed[:, k0 // 2:k1 // 2].contiguous(), scale[:, k0 // group_size:k1 // group_size].contiguous(),
            zero[:, k0 // group_size:k1 // group_size].contiguous())


def _shard_linear(lin: nn.Module, rank: int, world: int, dim: int) -> nn.Module:
    """dim 0: output features (column-parallel), dim 1: input features (row-parallel)."""
    if isinstance(lin, QuantizedLinear):
        if lin.bias is not None:
            raise ValueError("tensor-parallel INT4 layers take no bias")
        if dim == 0:
            p, s, z = shard_int4_rows(lin.packed_weight, lin.scale, lin.zero_point, rank, world)
            out = QuantizedLinear(lin.in_features, lin.out_features // world, lin.group_size)
        else:
            p, s, z = shard_int4_cols(lin.packed_weight, lin.scale, lin.zero_point, rank, world, lin.group_size)
            out = QuantizedLinear(lin.in_features // world, lin.out_features, lin.group_size)
        out = out.to(lin.packed_weight.device)
        out.packed_weight.copy_(p)
        out.scale.copy_(s)
        out.zero_point.copy_(z)
        return out
    if isinstance(lin, nn.Linear):
        w = lin.weight.data
        if dim == 0:
            r0, r1 = _span(w.shape[0], rank, world, "out_features")
            w = w[r0:r1]
        else:
            k0, k1 = _span(w.shape[1], rank, world, "in_features")
            w = w[:, k0:k1]
        out = nn.Linear(w.shape[1], w.shape[0], bias=False, device=w.device, dtype=w.dtype)
        out.weight.data.copy_(w)
        return out
    raise TypeError(f"cannot shard {type(lin).__name__}")


def shard_model(model: nn.Module, group=None) -> nn.Module:
    """Shard a (quantized or fp) Llama in place for this rank of `group` (default: WORLD)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if world == 1:
        return model
    for layer in model.layers:
        att, ff = layer.attention, layer.feed_forward
        if att.n_local_heads % world or att.n_local_kv_heads % world:
            raise ValueError(f"{att.n_local_heads} query / {att.n_local_kv_heads} KV heads do not split {world} ways")
        att.wq = _shard_linear(att.wq, rank, world, 0)
        att.wk = _shard_linear(att.wk, rank, world, 0)
        att.wv = _shard_linear(att.wv, rank, world, 0)
        att.wo = _shard_linear(att.wo, rank, world, 1)
        att.n_local_heads //= world
        att.n_local_kv_heads //= world
        att.cache_k = att.cache_v = None
        att.tp_group = group if group is not None else dist.group.WORLD
        ff.w1 = _shard_linear(ff.w1, rank, world, 0)
        ff.w3 = _shard_linear(ff.w3, rank, world, 0)
        ff.w2 = _shard_linear(ff.w2, rank, world, 1)
        ff.tp_group = att.tp_group
    model.output = _shard_linear(model.output, rank, world, 0)
    model.tp_group = group if group is not None else dist.group.WORLD
    model.tp_world = world
    return model
