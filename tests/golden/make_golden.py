"""Regenerate tests/golden/native/ from the reference's own test fixtures.

The reference (QwenDecisionCore.jl) pins its whole forward with a tiny
Qwen3.5 checkpoint and PyTorch-computed logits under
test/fixtures/native/ (loaded by test/runtests.jl:16-31 and
test/backbone.jl:1-34).  Those files are data, not code: this script copies
them byte for byte so the parity tests can run where the reference tree is
absent, and records each file's SHA-256 in MANIFEST.json.

    python tests/golden/make_golden.py REFERENCE_ROOT

`cuda_reference.json` (21 cases x 3 rows, lengths 1-256) sits beside the
pinned `reference.json` in the reference but no reference test loads it; it
is copied as an extra, unpinned check.
"""
import hashlib
import json
import os
import shutil
import sys

FILES = ("config.json", "model.safetensors", "readout.safetensors",
         "reference.json", "cuda_reference.json")


def main(argv):
    if len(argv) != 2:
        raise SystemExit("usage: make_golden.py REFERENCE_ROOT (the QwenDecisionCore.jl checkout)")
    root = argv[1]
    src = os.path.join(root, "test", "fixtures", "native")
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "native")
    os.makedirs(dst, exist_ok=True)
    manifest = {}
    for name in FILES:
        shutil.copyfile(os.path.join(src, name), os.path.join(dst, name))
        with open(os.path.join(dst, name), "rb") as f:
            manifest[name] = hashlib.sha256(f.read()).hexdigest()
    manifest["_source"] = "QwenDecisionCore.jl v0.1.0 test/fixtures/native"
    with open(os.path.join(dst, "MANIFEST.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print("wrote", dst)


if __name__ == "__main__":
    main(sys.argv)
