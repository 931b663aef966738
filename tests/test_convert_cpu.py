"""compressed-tensors W4A16_ASYM ("pack-quantized") -> repository INT4 format
(llama-efficient-inference_b200/convert_ct.py, restating the reference's convert_ct.py),
on the CPU: the converted buffers are bit-identical to the oracle's quantization of the
same weights, q_proj / k_proj rows return to the interleaved RoPE order, and the
dequantized weights equal compressed-tensors' own decompression formula."""
import numpy as np
import pytest
import torch

from oracle import oracle


def to_ct(packed: np.ndarray, scale: np.ndarray, zero: np.ndarray):
    """Repository INT4 buffers -> compressed-tensors tensors (the inverse of the conversion)."""
    n, half_k = packed.shape
    w_packed = torch.from_numpy(np.ascontiguousarray(packed)).view(torch.int32)  # [N, K/8], little-endian words
    z = torch.from_numpy(zero.astype(np.float32)).to(torch.int32)  # integers 0..15
    g = z.shape[1]
    z8 = z.view(n // 8, 8, g)
    zp = torch.zeros(n // 8, g, dtype=torch.int32)
    for j in range(8):
        zp |= z8[:, j, :] << (4 * j)
    return w_packed, zp, torch.from_numpy(scale), torch.tensor([n, 2 * half_k])


def quantized(n, k, seed):
    w = (np.random.default_rng(seed).standard_normal((n, k)) * 0.02).astype(np.float16)
    return oracle.quantize(w, 128)


def test_unpack_int32_nibble_order():
    import convert_ct

    x = torch.tensor([[0x76543210]], dtype=torch.int32)
    assert convert_ct.unpack_int32(x, 1).tolist() == [[0, 1, 2, 3, 4, 5, 6, 7]]
    assert convert_ct.unpack_int32(x, 0).view(-1).tolist() == [0, 1, 2, 3, 4, 5, 6, 7]


@pytest.mark.parametrize("heads", [None, 4])
def test_convert_linear_is_bit_exact(heads):
    import convert_ct

    packed, scale, zero = quantized(64, 512, 1 + (heads or 0))
    if heads is None:
        ct = to_ct(packed, scale, zero)
    else:  # an HF checkpoint holds q_proj / k_proj rows in rotate_half order
        perm = lambda a: convert_ct.permute_rows(torch.from_numpy(a), heads).numpy()
        ct = to_ct(perm(packed), perm(scale), perm(zero))
    p, s, z = convert_ct.convert_linear(*ct, heads=heads)
    assert np.array_equal(p.numpy(), packed)
    assert np.array_equal(s.numpy().view(np.uint16), scale.view(np.uint16))
    assert np.array_equal(z.numpy().astype(np.float32), zero.astype(np.float32))


def test_permute_rows_inverts():
    import convert_ct

    t = torch.arange(64 * 3).view(64, 3)
    assert torch.equal(convert_ct.unpermute_rows(convert_ct.permute_rows(t, 4), 4), t)


def test_dequant_matches_compressed_tensors_formula_and_oracle():
    import convert_ct

    packed, scale, zero = quantized(32, 256, 7)
    ours = convert_ct.dequant(torch.from_numpy(packed), torch.from_numpy(scale), torch.from_numpy(zero))
    assert np.array_equal(ours.numpy().view(np.uint16), oracle.dequantize(packed, scale, zero, 128).view(np.uint16))
    # compressed-tensors: signed int4 = nibble - 8, W = (q_s - zp_s) * scale in fp32, stored fp16
    w_packed, zp, sc, shape = to_ct(packed, scale, zero)
    q_s = convert_ct.unpack_int32(w_packed, 1).float() - 8
    zp_s = convert_ct.unpack_int32(zp, 0).float() - 8
    ct = ((q_s.view(32, 2, 128) - zp_s.unsqueeze(-1)) * sc.float().unsqueeze(-1)).view(32, 256).half()
    assert torch.equal(ct.view(torch.int16), ours.view(torch.int16))


def test_convert_checkpoint_and_load():
    import convert_ct
    from llama.quantize import QuantizedLinear

    dim, kv, ffn, heads, kv_heads = 256, 64, 512, 4, 1
    shapes = {"self_attn.q_proj": (dim, dim), "self_attn.k_proj": (kv, dim), "self_attn.v_proj": (kv, dim),
              "self_attn.o_proj": (dim, dim), "mlp.gate_proj": (ffn, dim), "mlp.up_proj": (ffn, dim),
              "mlp.down_proj": (dim, ffn)}
    tensors, want = {}, {}
    for i, (hf, (n, k)) in enumerate(shapes.items()):
        packed, scale, zero = quantized(n, k, 100 + i)
        want[convert_ct.MAP[hf]] = (packed, scale, zero)
        h = {"self_attn.q_proj": heads, "self_attn.k_proj": kv_heads}.get(hf)
        src = (packed, scale, zero) if h is None else tuple(
            convert_ct.permute_rows(torch.from_numpy(a), h).numpy() for a in (packed, scale, zero))
        w_packed, zp, sc, shape = to_ct(*src)
        pre = f"model.layers.0.{hf}."
        tensors.update({pre + "weight_packed": w_packed, pre + "weight_zero_point": zp, pre + "weight_scale": sc,
                        pre + "weight_shape": shape})
    ones = torch.ones(dim, dtype=torch.float16)
    tensors.update({"model.layers.0.input_layernorm.weight": ones, "model.layers.0.post_attention_layernorm.weight": ones,
                    "model.norm.weight": ones, "model.embed_tokens.weight": torch.zeros(100, dim, dtype=torch.float16)})
    int4, fake = convert_ct.convert(tensors, heads, kv_heads)
    assert set(int4) == {f"layers.0.{m}" for m in convert_ct.MAP.values()}
    assert "output.weight" in fake and fake["output.weight"] is fake["tok_embeddings.weight"]  # tied
    for meta, (packed, scale, zero) in want.items():
        p, s, z = int4[f"layers.0.{meta}"]
        assert np.array_equal(p.numpy(), packed)
        assert np.array_equal(fake[f"layers.0.{meta}.weight"].numpy().view(np.uint16),
                              oracle.dequantize(packed, scale, zero, 128).view(np.uint16))
    # into QuantizedLinear modules
    mods = torch.nn.Module()
    mods.add_module("wq", QuantizedLinear(dim, dim, 128))
    convert_ct.load_int4(mods, {"wq": int4["layers.0.attention.wq"]})
    assert torch.equal(mods.wq.packed_weight, int4["layers.0.attention.wq"][0])
