"""TEST INFRASTRUCTURE ONLY -- stages the reference's own optimizer as the timed CPU baseline.

    python oracle/stage_ref.py [--reference <HybridAgent checkout>]

Copies ``hybrid_rl/__init__.py`` and ``hybrid_rl/optimizer.py`` of the reference checkout,
byte for byte, into ``oracle/_ref/hybrid_rl/`` and writes ``oracle/_ref/STAGED.json`` with the
SHA-256 of every staged file.  Those two files are the whole ``ZeroOneAdamW`` path: the
optimizer imports only ``torch`` and ``torch.distributed`` (optimizer.py:8-9) and the package
``__init__`` is a docstring.  ``oracle/_ref/`` is git-ignored (it is the reference's code,
not this project's) but travels with the working tree to the GPU machines, where
``bench.py --impl reference`` and the CPU-baseline leg import the staged
``hybrid_rl.optimizer.ZeroOneAdamW`` unmodified.  Where it was never staged they time
``oracle/torch_ops.py`` (the same op sequence) and say so (kind "port").
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
FILES = ("hybrid_rl/__init__.py", "hybrid_rl/optimizer.py")


def _default_reference() -> str:
    """The reference checkout: $HYBRIDAGENT_REFERENCE, else the path BASELINE.json records."""
    if os.environ.get("HYBRIDAGENT_REFERENCE"):
        return os.environ["HYBRIDAGENT_REFERENCE"]
    try:
        with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as fh:
            return json.load(fh)["reference_path"]
    except (OSError, KeyError, ValueError):
        return ""


DEFAULT_REFERENCE = _default_reference()


def sha256(path: str) -> str:
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def stage(reference: str = DEFAULT_REFERENCE) -> bool:
    """Stages the files if the checkout exists; returns whether oracle/_ref holds them."""
    if not reference or not all(os.path.exists(os.path.join(reference, f)) for f in FILES):
        return staged() is not None
    record = {"source": "HybridAgent hybrid_rl (unmodified)", "files": {}}
    for f in FILES:
        src, dst = os.path.join(reference, f), os.path.join(OUT, f)
        os.makedirs(os.path.dirname(dst), exist_ok=True)
        shutil.copyfile(src, dst)
        record["files"][f] = sha256(dst)
        if record["files"][f] != sha256(src):
            raise RuntimeError(f"staged copy of {f} differs from its source")
    with open(os.path.join(OUT, "STAGED.json"), "w") as fh:
        json.dump(record, fh, indent=1)
    return True


def staged() -> dict | None:
    """The STAGED.json record if every staged file is present and unchanged, else None."""
    try:
        with open(os.path.join(OUT, "STAGED.json")) as fh:
            record = json.load(fh)
    except (OSError, ValueError):
        return None
    for f, digest in record.get("files", {}).items():
        p = os.path.join(OUT, f)
        if not os.path.exists(p) or sha256(p) != digest:
            return None
    return record if set(record.get("files", {})) == set(FILES) else None


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=DEFAULT_REFERENCE)
    a = ap.parse_args()
    print("staged" if stage(a.reference) else "reference checkout not found; nothing staged")
