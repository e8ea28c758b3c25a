"""Copies the reference's tiny-checkpoint golden fixtures into tests/golden/tiny.

Source: decider-engine tests/fixtures/tiny (a synthetic 2-layer checkpoint,
seed 4242, with PyTorch/Transformers FP32 reference outputs generated upstream)
and tests/request.json. The copies are byte-for-byte; run this script with
the reference checkout given as the argument or in DECIDER_REFERENCE:

    python tests/golden/make_golden.py /path/to/decider-engine
"""
import os
import shutil
import sys

FILES = [
    "strands_decider_config.json",
    "tokenizer.json",
    "head.safetensors",
    "raw-reference.json",
    "reference.json",
    "base/config.json",
    "base/model.safetensors",
    "lora/adapter_config.json",
    "lora/adapter_model.safetensors",
]


def main(ref: str) -> None:
    here = os.path.dirname(os.path.abspath(__file__))
    src = os.path.join(ref, "tests", "fixtures", "tiny")
    dst = os.path.join(here, "tiny")
    for f in FILES:
        os.makedirs(os.path.dirname(os.path.join(dst, f)), exist_ok=True)
        shutil.copyfile(os.path.join(src, f), os.path.join(dst, f))
    shutil.copyfile(os.path.join(ref, "tests", "request.json"), os.path.join(here, "request.json"))


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DECIDER_REFERENCE")
    if not ref:
        sys.exit("usage: make_golden.py <decider-engine checkout> (or set DECIDER_REFERENCE)")
    main(ref)
