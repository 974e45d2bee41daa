"""Pack textsift's kernel-conformance fixtures into tests/golden/conformance.npz.

Source: tests/native/conformance/fixtures/<op>/{meta.json, uniform.bin,
_uniform_*.bin, <input>.bin, _output_initial.bin, expected.bin} of
teamchong/textsift (dumped from browser WebGPU by
tests/conformance/dump-fixtures.spec.ts).  The reference checkout is only
present where the fixtures are generated; the GPU hosts read the npz.

Run: python tests/golden/make_golden.py path/to/textsift
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "conformance.npz")


def main(ref_root: str) -> None:
    fx = os.path.join(ref_root, "tests", "native", "conformance", "fixtures")
    arrays: dict[str, np.ndarray] = {}
    metas = {}
    for op in sorted(os.listdir(fx)):
        d = os.path.join(fx, op)
        if not os.path.isdir(d):
            continue
        metas[op] = json.load(open(os.path.join(d, "meta.json")))
        for f in sorted(os.listdir(d)):
            if f.endswith(".bin"):
                arrays[f"{op}/{f[:-4]}"] = np.fromfile(os.path.join(d, f), dtype=np.uint8)
    arrays["__meta__"] = np.frombuffer(json.dumps(metas, sort_keys=True).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT}: {len(metas)} ops, {len(arrays) - 1} arrays")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py path/to/textsift")
    main(sys.argv[1])
