"""Stage the unmodified reference package next to this file, for the comparator legs of bench.py.

    python baseline/stage_reference.py /path/to/llama-efficient-inference

The reference is a plain source tree (no setup.py or pyproject.toml), so
`pip install --target baseline/_ref` refuses it.  This copies its `llama/`
package, byte for byte and unchanged, to baseline/_ref/llama/ -- the location
a `pip install --target baseline/_ref` would have used.  baseline/_ref/ is
git-ignored: the reference's sources never enter this repository's history,
but the copy travels with the working tree to the GPU machine, where bench.py
imports from it (by file path, as the reference's own int4_linear_fn does):

  * llama/int4_gemv.py  -- the reference's Triton kernel, timed on the same
    B200 as the bar the CUDA kernels have to beat (bench.py `reference_gpu`);
  * llama/quantize.py   -- the reference's own CPU path (v1 dequantize + fp16
    F.linear), timed on the host cores (`cpu_baseline.reference_torch`);
  * llama/model.py      -- the reference model, one CPU decode step timed with
    its `.cuda()` KV-cache allocation stubbed to stay on the host.

Nothing on the product path reads baseline/_ref.
"""
import argparse
import hashlib
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
DEST = os.path.join(HERE, "_ref", "llama")
FILES = ("__init__.py", "config.py", "generation.py", "int4_gemv.py", "model.py", "quantize.py", "tokenizer.py")


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("reference", help="root of the reference checkout (the directory holding llama/)")
    a = ap.parse_args()
    src = os.path.join(a.reference, "llama")
    if not os.path.isdir(src):
        print(f"no llama/ package under {a.reference}", file=sys.stderr)
        return 1
    os.makedirs(DEST, exist_ok=True)
    for name in FILES:
        shutil.copyfile(os.path.join(src, name), os.path.join(DEST, name))
        with open(os.path.join(DEST, name), "rb") as f:
            print(f"{hashlib.sha256(f.read()).hexdigest()[:16]}  baseline/_ref/llama/{name}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
