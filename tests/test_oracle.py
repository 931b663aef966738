"""The CPU oracle against the reference's own outputs (tests/golden/).

Pins: bit-exact quantize_tensor (llama/quantize.py:44-75) and
dequantize_packed (:78-104) on every golden case, and the v1 forward
(:143-147) within the fp16 output rounding.  Also the reference's own
quantizer checks (check_impl.py:86-103).
"""
import numpy as np
import pytest
import torch

import cases
from oracle import oracle


def bits(a):
    return np.ascontiguousarray(a).view(np.uint16 if a.dtype.itemsize == 2 else np.uint8)


@pytest.mark.parametrize("case", cases.QUANT_CASES, ids=[c[0] for c in cases.QUANT_CASES])
def test_quantize_matches_reference_bits(case, golden):
    meta, arr = golden
    name, N, K, group = case[:4]
    w = cases.make_quant_input(case).numpy()
    assert np.array_equal(bits(w), bits(arr[f"quant/{name}/w"])), "input generator drifted"
    packed, scale, zero = oracle.quantize(w, group)
    assert np.array_equal(packed, arr[f"quant/{name}/packed"])
    assert np.array_equal(bits(scale), bits(arr[f"quant/{name}/scale"]))
    assert np.array_equal(bits(zero), bits(arr[f"quant/{name}/zero"]))  # includes the sign of zero
    w16 = oracle.dequantize(packed, scale, zero, group)
    assert np.array_equal(bits(w16), bits(arr[f"quant/{name}/w16"]))


def test_quantize_shapes_and_dtypes():
    """check_impl.py:86-93: gs=32, out=128, in=256."""
    w = (np.random.default_rng(0).standard_normal((128, 256)) ).astype(np.float16)
    packed, scale, zero = oracle.quantize(w, 32)
    assert packed.shape == (128, 128) and packed.dtype == np.uint8
    assert scale.shape == (128, 8) and zero.shape == (128, 8)
    assert scale.dtype == np.float16 and zero.dtype == np.float16


def test_roundtrip_error_bounded():
    """check_impl.py:95-103: 0 < rel_err < 0.2 for W ~ N(0, 0.1), gs=128."""
    w = (np.random.default_rng(1).standard_normal((256, 512)) * 0.1).astype(np.float16)
    packed, scale, zero = oracle.quantize(w, 128)
    w16 = oracle.dequantize(packed, scale, zero, 128)
    rel = np.abs(w.astype(np.float32) - w16.astype(np.float32)).max() / (np.abs(w).max() + 1e-8)
    assert 0 < rel < 0.2


def test_quantize_input_dtypes_agree():
    """weight.float() makes fp16 / fp32 / bf16 inputs of the same values quantize identically."""
    w16 = (np.random.default_rng(2).standard_normal((8, 256)) * 0.02).astype(np.float16)
    ref = oracle.quantize(w16, 128)
    got32 = oracle.quantize(w16.astype(np.float32), 128)
    wt = torch.from_numpy(w16.astype(np.float32)).to(torch.bfloat16)
    gotbf = oracle.quantize(wt.view(torch.int16).numpy().view(np.uint16), 128, dtype="bf16")
    refbf = oracle.quantize(wt.float().numpy(), 128)
    for a, b in zip(ref, got32):
        assert np.array_equal(bits(a), bits(b))
    for a, b in zip(refbf, gotbf):
        assert np.array_equal(bits(a), bits(b))


@pytest.mark.parametrize("case", cases.GEMV_CASES, ids=[c[0] for c in cases.GEMV_CASES])
def test_linear_matches_reference(case, golden):
    meta, arr = golden
    name, N, K, M, group = case[:5]
    info = meta["gemv"][name]
    w, x = cases.make_gemv_inputs(case)
    w, x = w.numpy(), x.numpy()
    assert cases.sha256(w) == info["sha256"]["w"] and cases.sha256(x) == info["sha256"]["x"], "input generator drifted"
    packed, scale, zero = oracle.quantize(w, group)
    assert cases.sha256(packed) == info["sha256"]["packed"]
    assert cases.sha256(scale) == info["sha256"]["scale"]
    assert cases.sha256(zero) == info["sha256"]["zero"]
    w16 = oracle.dequantize(packed, scale, zero, group)
    assert cases.sha256(w16) == info["sha256"]["w16"]
    y, y32 = oracle.linear(x, packed, scale, zero, group)
    y_ref = arr[f"gemv/{name}/y"]
    tol = oracle.tolerance(y_ref)
    assert np.abs(y.astype(np.float32) - y_ref.astype(np.float32)).max() <= tol
    # the oracle's sums are the exact sums: they match the reference's fp32 matmul to fp32 rounding
    y32_ref = arr[f"gemv/{name}/y32"]
    assert np.abs(y32 - y32_ref).max() <= 1e-5 * max(1.0, float(np.abs(y32_ref).max()))


def test_planted_nibble_swap_is_caught(golden):
    """A packing mistake (even/odd nibbles swapped) must fail the tolerance check."""
    meta, arr = golden
    case = next(c for c in cases.GEMV_CASES if c[0] == "m16")
    w, x = cases.make_gemv_inputs(case)
    packed, scale, zero = oracle.quantize(w.numpy(), 128)
    swapped = ((packed >> 4) | (packed << 4)).astype(np.uint8)
    y_bad, _ = oracle.linear(x.numpy(), swapped, scale, zero, 128)
    y_ref = arr["gemv/m16/y"]
    assert np.abs(y_bad.astype(np.float32) - y_ref.astype(np.float32)).max() > oracle.tolerance(y_ref)


def test_planted_zero_point_offset_is_caught(golden):
    """Dequantizing with zero + 1 must fail the tolerance check."""
    meta, arr = golden
    case = next(c for c in cases.GEMV_CASES if c[0] == "g64")
    w, x = cases.make_gemv_inputs(case)
    packed, scale, zero = oracle.quantize(w.numpy(), 64)
    y_bad, _ = oracle.linear(x.numpy(), packed, scale, (zero.astype(np.float32) + 1).astype(np.float16), 64)
    y_ref = arr["gemv/g64/y"]
    assert np.abs(y_bad.astype(np.float32) - y_ref.astype(np.float32)).max() > oracle.tolerance(y_ref)
