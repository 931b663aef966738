"""Convert a compressed-tensors W4A16_ASYM checkpoint (GPTQ / AWQ "pack-quantized")
into this repository's INT4 format, the format QuantizedLinear and the B200 kernels
take.  Restates the reference's convert_ct.py (convert_ct.py:43-122) with the same
outputs.

compressed-tensors "pack-quantized":
  weight_packed      int32 [N, K/8]   8 nibbles per int32 along K, element 0 in bits 0-3
  weight_zero_point  int32 [N/8, G]   8 nibbles per int32 along N
  weight_scale       fp16  [N, G]
  nibble = signed int4 + 8 and W = (q_signed - zp_signed) * scale, so with q = nibble
  and zp = nibble, W = (q - zp) * scale: the repository format (llama/quantize.py:44-75).

The repository packs two nibbles per uint8 with the even k in the low nibble.  Those
are the bytes of the little-endian int32 words, so the packed weight converts by
reinterpreting its storage, with no per-nibble work.  The zero points are unpacked
from their N-direction nibbles.  HF's q_proj / k_proj rows are permuted for its
rotate_half RoPE; unpermute_rows restores the interleaved (Meta) order that
llama/model.py's RoPE expects, for packed rows, scales and zero points alike.

Writes, as the reference does:
  <out>/<name>_int4.pt   {"int4": {meta linear name: (packed uint8, scale fp16, zero fp16)},
                          "group_size": 128, "source": ckpt}
  <out>/<name>_fake.pth  Meta-key fp16 state dict, every Linear dequantized

    python llama-efficient-inference_b200/convert_ct.py --name gptq --ckpt <dir with model.safetensors>
"""
from __future__ import annotations

import argparse
import os
import re
import sys

import torch

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
if PKG_DIR not in sys.path:
    sys.path.insert(0, PKG_DIR)

MAP = {"self_attn.q_proj": "attention.wq", "self_attn.k_proj": "attention.wk", "self_attn.v_proj": "attention.wv",
       "self_attn.o_proj": "attention.wo", "mlp.gate_proj": "feed_forward.w1", "mlp.up_proj": "feed_forward.w3",
       "mlp.down_proj": "feed_forward.w2"}
GROUP = 128


def unpack_int32(x: torch.Tensor, axis: int) -> torch.Tensor:
    """int32 tensor with 8 nibbles per element along `axis` (element 0 in the low bits) -> uint8 nibbles."""
    shifts = torch.arange(0, 32, 4, dtype=torch.int32, device=x.device)
    if axis == 1:
        n = (x.unsqueeze(-1) >> shifts) & 0xF  # [N, K/8, 8]
        return n.reshape(x.shape[0], -1).to(torch.uint8)
    n = (x.unsqueeze(1) >> shifts.view(1, 8, 1)) & 0xF  # [N/8, 8, G]
    return n.reshape(-1, x.shape[1]).to(torch.uint8)


def packed_from_int32(packed: torch.Tensor, k: int) -> torch.Tensor:
    """weight_packed int32 [N, K/8] -> packed uint8 [N, K/2] (byte j = q[2j] | q[2j+1] << 4)."""
    if packed.dtype != torch.int32 or k % 8:
        raise ValueError(f"expected int32 words of 8 nibbles and K % 8 == 0, got {packed.dtype}, K={k}")
    if sys.byteorder != "little":
        q = unpack_int32(packed, 1)[:, :k]
        return (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous()
    return packed.contiguous().view(torch.uint8)[:, : k // 2].contiguous()


def unpermute_rows(t: torch.Tensor, heads: int) -> torch.Tensor:
    """HF rotate_half row order -> interleaved (even, odd) pairs per head."""
    rows = t.shape[0]
    return t.view(heads, 2, rows // heads // 2, *t.shape[1:]).transpose(1, 2).reshape(rows, *t.shape[1:])


def permute_rows(t: torch.Tensor, heads: int) -> torch.Tensor:
    """The inverse of unpermute_rows (HF's permutation of Meta q_proj / k_proj rows)."""
    rows = t.shape[0]
    return t.view(heads, rows // heads // 2, 2, *t.shape[1:]).transpose(1, 2).reshape(rows, *t.shape[1:])


def dequant(packed: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor, group: int = GROUP) -> torch.Tensor:
    """QuantizedLinear.dequantize_packed (v1) on any device: fp32 (q - zp) * scale, then fp16."""
    n = packed.shape[0]
    q = torch.stack([packed & 0xF, packed >> 4], dim=-1).reshape(n, -1)
    k = q.shape[1]
    w = (q.float().reshape(n, k // group, group) - zero.float().unsqueeze(-1)) * scale.float().unsqueeze(-1)
    return w.reshape(n, k).half()


def convert_linear(packed_i32: torch.Tensor, zp_i32: torch.Tensor, scale: torch.Tensor, shape,
                   heads: int | None = None):
    """One compressed-tensors Linear -> (packed uint8 [N, K/2], scale fp16 [N, G], zero fp16 [N, G])."""
    n, k = (int(v) for v in shape)
    packed = packed_from_int32(packed_i32, k)
    zero = unpack_int32(zp_i32, 0)[:n]
    if packed.shape != (n, k // 2) or zero.shape != scale.shape:
        raise ValueError(f"unexpected shapes: packed {tuple(packed.shape)}, zero {tuple(zero.shape)}, "
                         f"scale {tuple(scale.shape)} for [{n}, {k}]")
    if heads is not None:
        packed, zero, scale = unpermute_rows(packed, heads), unpermute_rows(zero, heads), unpermute_rows(scale, heads)
    return packed.contiguous(), scale.half().contiguous(), zero.half().contiguous()


def convert(tensors, n_heads: int, n_kv_heads: int):
    """{safetensors key: tensor} of a compressed-tensors Llama -> (int4 dict, fp16 Meta state dict)."""
    layers = sorted({int(m.group(1)) for key in tensors for m in [re.match(r"model\.layers\.(\d+)\.", key)] if m})
    int4, fake = {}, {}
    for i in layers:
        for hf, meta in MAP.items():
            pre = f"model.layers.{i}.{hf}."
            heads = {"self_attn.q_proj": n_heads, "self_attn.k_proj": n_kv_heads}.get(hf)
            p, s, z = convert_linear(tensors[pre + "weight_packed"], tensors[pre + "weight_zero_point"],
                                     tensors[pre + "weight_scale"], tensors[pre + "weight_shape"].tolist(), heads)
            name = f"layers.{i}.{meta}"
            int4[name] = (p.cpu(), s.cpu(), z.cpu())
            fake[name + ".weight"] = dequant(p, s, z).cpu()
        fake[f"layers.{i}.attention_norm.weight"] = tensors[f"model.layers.{i}.input_layernorm.weight"].cpu()
        fake[f"layers.{i}.ffn_norm.weight"] = tensors[f"model.layers.{i}.post_attention_layernorm.weight"].cpu()
    fake["norm.weight"] = tensors["model.norm.weight"].cpu()
    emb = tensors["model.embed_tokens.weight"].cpu()
    fake["tok_embeddings.weight"] = emb
    fake["output.weight"] = tensors["lm_head.weight"].cpu() if "lm_head.weight" in tensors else emb
    return int4, fake


def load_int4(model, int4: dict) -> None:
    """Copy converted INT4 buffers into the QuantizedLinear modules of a quantize_model()-ed Llama."""
    for name, (p, s, z) in int4.items():
        mod = model.get_submodule(name)
        mod.packed_weight.copy_(p)
        mod.scale.copy_(s)
        mod.zero_point.copy_(z)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--name", required=True)
    ap.add_argument("--ckpt", required=True, help="directory holding model.safetensors")
    ap.add_argument("--out", default=".")
    ap.add_argument("--n-heads", type=int, default=32)
    ap.add_argument("--n-kv-heads", type=int, default=8)
    a = ap.parse_args()
    from safetensors import safe_open

    with safe_open(os.path.join(a.ckpt, "model.safetensors"), "pt", device="cpu") as f:
        tensors = {k: f.get_tensor(k) for k in f.keys()}
    int4, fake = convert(tensors, a.n_heads, a.n_kv_heads)
    tied = "lm_head.weight" not in tensors
    print(f"converted {len(int4)} Linear; lm_head {'tied to embed_tokens' if tied else 'from lm_head.weight'} (FP16)")
    os.makedirs(a.out, exist_ok=True)
    torch.save({"int4": int4, "group_size": GROUP, "source": a.ckpt}, os.path.join(a.out, f"{a.name}_int4.pt"))
    torch.save(fake, os.path.join(a.out, f"{a.name}_fake.pth"))
    print(f"saved {a.out}/{a.name}_int4.pt and {a.name}_fake.pth")


if __name__ == "__main__":
    main()
