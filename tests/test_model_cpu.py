"""The model code (llama/model.py) against the reference's llama/model.py, on the CPU.

The golden logits come from the reference's own model (tiny Llama config, seeded
fp16 weights, `.cuda()` stubbed) run by tests/golden/make_golden.py.  Here our
model runs the same weights unquantized in fp16 on the CPU (nn.Linear), through
the reference-style forward(tokens, start_pos) and through the graph-friendly
decode_step(tokens, pos) whose position is a tensor.
"""
import numpy as np
import pytest
import torch

import cases

TOL = 1e-3  # relative to max|logits|; measured exact (0.0) on this CPU, slack for other BLAS builds


@pytest.fixture(scope="module")
def model():
    from llama.model import Llama, ModelArgs

    args = ModelArgs(**cases.TINY_MODEL)
    torch.set_default_dtype(torch.float16)
    try:
        m = Llama(args)
    finally:
        torch.set_default_dtype(torch.float32)
    m.load_state_dict(cases.tiny_state_dict(cases.TINY_MODEL), strict=True)
    return m.eval()


def close(a: torch.Tensor, ref: np.ndarray, tol=TOL):
    a = a.float().numpy()
    err = np.abs(a - ref).max()
    assert err <= tol * np.abs(ref).max(), f"max|d logits| = {err:.3e} vs max|ref| = {np.abs(ref).max():.3e}"


def test_state_dict_keys_match_reference(model):
    assert set(model.state_dict()) == set(cases.tiny_state_dict(cases.TINY_MODEL))


@torch.inference_mode()
def test_forward_matches_reference_model(model, golden):
    meta, arr = golden
    model.reset_cache()
    prompt = torch.from_numpy(arr["model/prompt"])
    logits = model(prompt, 0)
    close(logits, arr["model/fp16/prefill_logits"])
    nxt = logits[:, -1].argmax(-1, keepdim=True)
    toks = [nxt]
    ref_dec = arr["model/fp16/decode_logits"]
    for i in range(cases.TINY_DECODE_STEPS):
        lg = model(nxt, prompt.shape[1] + i)
        close(lg, ref_dec[:, i:i + 1])
        nxt = lg[:, -1].argmax(-1, keepdim=True)
        toks.append(nxt)
    assert np.array_equal(torch.cat(toks, 1).numpy(), arr["model/fp16/tokens"])


@torch.inference_mode()
def test_decode_step_with_tensor_position(model, golden):
    meta, arr = golden
    model.reset_cache()
    prompt = torch.from_numpy(arr["model/prompt"])
    nxt = model(prompt, 0)[:, -1].argmax(-1, keepdim=True)
    pos = torch.tensor([prompt.shape[1]], dtype=torch.long)
    ref_dec = arr["model/fp16/decode_logits"]
    toks = [nxt]
    for i in range(cases.TINY_DECODE_STEPS):
        lg = model.decode_step(nxt, pos)
        close(lg, ref_dec[:, i:i + 1])
        nxt = lg[:, -1].argmax(-1, keepdim=True)
        toks.append(nxt)
        pos += 1
    assert np.array_equal(torch.cat(toks, 1).numpy(), arr["model/fp16/tokens"])


def test_llama3_rope_scaling_rule():
    """Scaled frequencies: short wavelengths kept, long ones / 32, smooth blend in between."""
    import math

    from llama.model import apply_llama3_scaling

    freqs = 1.0 / (500000.0 ** (torch.arange(0, 64, 2).float() / 64))
    scaled = apply_llama3_scaling(freqs)
    for f, s in zip(freqs.tolist(), scaled.tolist()):
        wl = 2 * math.pi / f
        if wl < 8192 / 4:
            assert s == pytest.approx(f)
        elif wl > 8192:
            assert s == pytest.approx(f / 32)
        else:
            assert f / 32 <= s <= f


class _IdTokenizer:
    """Token ids as text: encode('3 9 4') -> [bos, 3, 9, 4]; decode joins ids with spaces."""
    bos_id, eos_id, pad_id = 1, 2, -1

    def encode(self, text, bos, eos):
        return ([self.bos_id] if bos else []) + [int(t) for t in text.split()] + ([self.eos_id] if eos else [])

    def decode(self, ids):
        return " ".join(str(i) for i in ids)


def test_generate_greedy_matches_eager_loop(model):
    """Generation.generate (greedy, with and without the KV cache, prompts of different lengths) gives the
    tokens of the reference-style eager loop for each prompt on its own."""
    from llama.generation import eager_tokens

    tok = _IdTokenizer()
    prompts = ["5 17 33 8", "40 41 42 43 44 45"]
    steps = 4
    for kv in (True, False):
        for m in model.layers:
            m.attention.cache_k = m.attention.cache_v = None
        out = model.generate(tok, prompts, max_gen_len=steps, temperature=0.0, top_p=0.9, kv_caching=kv,
                             device="cpu")
        for p, o in zip(prompts, out):
            model.reset_cache()
            ids = torch.tensor([tok.encode(p, bos=True, eos=False)])
            ref = eager_tokens(model, ids, steps - 1)[0].tolist()
            if tok.eos_id in ref:
                ref = ref[:ref.index(tok.eos_id)]
            assert o["generation"] == tok.decode(ref), (kv, p, o, ref)


def test_sample_top_p_keeps_the_nucleus():
    """sample_top_p draws only tokens inside the smallest set whose mass reaches p."""
    from llama.generation import sample_top_p

    torch.manual_seed(0)
    probs = torch.tensor([[0.05, 0.5, 0.1, 0.3, 0.05]]).repeat(2000, 1)
    drawn = sample_top_p(probs, 0.75).view(-1)
    assert set(drawn.tolist()) == {1, 3}  # 0.5 + 0.3 reaches 0.75; 0.1 starts above it


def test_int4_operators_trace_with_fake_tensors():
    """li4::int4_linear and li4::int4_gemm are registered PyTorch operators whose fake kernels give the
    output shape without running anything (what torch.compile traces through)."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    from llama.quantize import QuantizedLinear

    QuantizedLinear(256, 64)  # constructing a layer registers the operators
    with FakeTensorMode():
        x = torch.empty(2, 3, 256, dtype=torch.float16)
        p = torch.empty(64, 128, dtype=torch.uint8)
        s = torch.empty(64, 2, dtype=torch.float16)
        assert torch.ops.li4.int4_linear(x, p, s, s, 128).shape == (2, 3, 64)
        xm = torch.empty(40, 256, dtype=torch.float16)
        assert torch.ops.li4.int4_gemm(xm, p, s, s, 128).shape == (40, 64)
