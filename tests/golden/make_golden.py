"""Generate the golden fixtures from the reference's own code.

Run in a container where the reference checkout exists (read-only is fine):

    python tests/golden/make_golden.py --reference PATH_TO_REFERENCE_CHECKOUT

It loads llama/quantize.py by file path (as the reference's own
dequant_traffic.py:47-53 does, so no tokenizer or CUDA is needed), runs
quantize_tensor / dequantize_packed / dequantize_packed_v2 and the v1
forward (dequantize + fp16 F.linear on the CPU) on the seeded inputs of
cases.py, and writes tests/golden/golden.npz plus golden.json (hashes and
metadata).  The tests never read the reference checkout.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402


def load_reference_quantize(ref_root: str):
    path = os.path.join(ref_root, "llama", "quantize.py")
    spec = importlib.util.spec_from_file_location("reference_llama_quantize", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def load_reference_model(ref_root: str):
    """llama/model.py by path under a package stub (no tokenizer import), .cuda() as identity."""
    import types

    pkg = types.ModuleType("llama")
    pkg.__path__ = [os.path.join(ref_root, "llama")]
    sys.modules["llama"] = pkg
    importlib.import_module("llama.generation")
    return importlib.import_module("llama.model")


@torch.inference_mode()
def run_reference_model(model, prompt, steps):
    """Prefill logits, then greedy decode steps as the reference's bench.py:154-161 does."""
    logits = [model(prompt, 0)]
    nxt = logits[0][:, -1].argmax(-1, keepdim=True)
    toks = [nxt]
    for i in range(steps):
        lg = model(nxt, prompt.shape[1] + i)
        logits.append(lg)
        nxt = lg[:, -1].argmax(-1, keepdim=True)
        toks.append(nxt)
    return logits, torch.cat(toks, 1)


def model_golden(ref_root, ref_quantize, arrays, meta):
    rm = load_reference_model(ref_root)
    saved_cuda = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *a, **k: self  # Attention.__init__ allocates its cache with .cuda()
    try:
        args = rm.ModelArgs(**cases.TINY_MODEL)
        sd = cases.tiny_state_dict(cases.TINY_MODEL)
        prompt = cases.tiny_prompt(cases.TINY_MODEL)
        torch.set_default_dtype(torch.float16)
        model = rm.Llama(args)
        torch.set_default_dtype(torch.float32)
        model.load_state_dict(sd, strict=True)
        model.eval()
        for tag in ("fp16", "int4"):
            if tag == "int4":
                ref_quantize.quantize_model(model, 128)  # DEQUANT_IMPL "v1": dequantize + F.linear
            for layer in model.layers:  # fresh caches for each run
                layer.attention.cache_k.zero_()
                layer.attention.cache_v.zero_()
            logits, toks = run_reference_model(model, prompt, cases.TINY_DECODE_STEPS)
            arrays[f"model/{tag}/prefill_logits"] = logits[0].numpy()
            arrays[f"model/{tag}/decode_logits"] = torch.cat(logits[1:], 1).numpy()
            arrays[f"model/{tag}/tokens"] = toks.numpy()
            print(f"tiny model {tag}: greedy tokens {toks.tolist()}")
        arrays["model/prompt"] = prompt.numpy()
        meta["model"] = {"args": cases.TINY_MODEL, "steps": cases.TINY_DECODE_STEPS,
                         "note": "reference llama/model.py on the CPU, fp16 weights; int4 = quantize_model + v1"}
    finally:
        torch.Tensor.cuda = saved_cuda
        torch.set_default_dtype(torch.float32)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout (the directory holding llama/)")
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref = load_reference_quantize(a.reference)
    QL = ref.QuantizedLinear

    arrays: dict[str, np.ndarray] = {}
    meta = {"torch": torch.__version__, "reference": "llama/quantize.py", "gemv": {}, "quant": {}}

    for case in cases.QUANT_CASES:
        name, N, K, group, mult, seed = case
        w = cases.make_quant_input(case)
        p, s, z = QL.quantize_tensor(w, group)
        w16 = QL.dequantize_packed(p, s, z, group)
        w16_v2 = QL.dequantize_packed_v2(p, s, z, group)
        assert torch.equal(w16.view(torch.int16), w16_v2.view(torch.int16))
        rel = ((w.float() - w16.float()).abs().max() / (w.abs().max() + 1e-8)).item()
        for key, t in (("w", w), ("packed", p), ("scale", s), ("zero", z), ("w16", w16)):
            arrays[f"quant/{name}/{key}"] = t.numpy()
        meta["quant"][name] = {"N": N, "K": K, "group": group, "roundtrip_rel_err": rel}

    for case in cases.GEMV_CASES:
        name, N, K, M, group, kind, seed = case
        w, x = cases.make_gemv_inputs(case)
        p, s, z = QL.quantize_tensor(w, group)
        w16 = QL.dequantize_packed(p, s, z, group)
        assert torch.equal(w16.view(torch.int16), QL.dequantize_packed_v2(p, s, z, group).view(torch.int16))
        y = F.linear(x, w16)  # the reference's v1 forward, fp16 on the CPU (llama/quantize.py:143-146)
        y32 = F.linear(x.float(), w16.float())
        info = {
            "N": N, "K": K, "M": M, "group": group, "kind": kind, "seed": seed,
            "sha256": {k: cases.sha256(t.numpy()) for k, t in
                       (("w", w), ("x", x), ("packed", p), ("scale", s), ("zero", z), ("w16", w16))},
            "max_abs_y": float(y.float().abs().max()),
            "ref_fp16_vs_fp32_max_err": float((y.float() - y32).abs().max()),
        }
        meta["gemv"][name] = info
        arrays[f"gemv/{name}/y"] = y.numpy()
        arrays[f"gemv/{name}/y32"] = y32.numpy()
        if name in cases.FULL_CASES:
            for key, t in (("packed", p), ("scale", s), ("zero", z), ("w16", w16)):
                arrays[f"gemv/{name}/{key}"] = t.numpy()
        print(f"{name:>10} N={N:>5} K={K:>5} M={M:>2} g={group:>3} max|y|={info['max_abs_y']:.3f} "
              f"fp16-vs-fp32 {info['ref_fp16_vs_fp32_max_err']:.2e}")

    model_golden(a.reference, ref, arrays, meta)

    np.savez_compressed(os.path.join(a.out, "golden.npz"), **arrays)
    with open(os.path.join(a.out, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", os.path.join(a.out, "golden.npz"))


if __name__ == "__main__":
    main()
