"""Regenerates the golden fixtures under tests/golden/ from the reference.

The reference (Hale-Token) ships two tiny random-weight models with golden
logits computed by its independent NumPy float64 model
(scripts/reference/make_fixtures.py; checked by tests/litmus.rs:15-59 and
tests/tiered_cache.rs:26-102 of the reference). This script copies those data
files verbatim -- config.json, model.safetensors, expected.json -- and records
their SHA-256 in MANIFEST.json, so the tests can run where the reference is
not mounted (the GPU box).

Usage: python tests/golden/make_golden.py REFERENCE_ROOT
(REFERENCE_ROOT: the reference crate's checkout; also read from the
HALE_REFERENCE_ROOT environment variable)
"""
import hashlib
import json
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURES = ("tiny-qwen3-moe", "tiny-mixtral")
FILES = ("config.json", "model.safetensors", "expected.json")


def main(ref_root):
    manifest = {"source": "reference tests/fixtures/<name>/", "files": {}}
    for name in FIXTURES:
        src = os.path.join(ref_root, "tests", "fixtures", name)
        dst = os.path.join(HERE, name)
        os.makedirs(dst, exist_ok=True)
        for f in FILES:
            shutil.copyfile(os.path.join(src, f), os.path.join(dst, f))
            with open(os.path.join(dst, f), "rb") as fh:
                manifest["files"][f"{name}/{f}"] = hashlib.sha256(fh.read()).hexdigest()
    with open(os.path.join(HERE, "MANIFEST.json"), "w") as fh:
        json.dump(manifest, fh, indent=1, sort_keys=True)
        fh.write("\n")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HALE_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py REFERENCE_ROOT")
    main(root)
