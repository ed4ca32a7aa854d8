"""Regenerate tests/golden/golden.npz from the reference's own compiled kernels.

    make -C oracle ref            # needs the reference sources
    python tests/golden/make_golden.py

Each case's inputs are redrawn from its seed (cases.py); the reference
(oracle/_ref/libnnc_ref.so: the reference's nn_ops kernels, its
model_attn_span, and ref_shim.cpp's restatement of its dispatch) computes the
outputs, which are stored with a digest of the inputs.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

import oracle as O  # noqa: E402
from oracle import scenarios as S  # noqa: E402
from golden import cases as G  # noqa: E402


def main() -> int:
    if O.ref() is None:
        print("oracle/_ref/libnnc_ref.so is missing: run `make -C oracle ref` first", file=sys.stderr)
        return 1
    out = {}
    for name, case in G.all_cases().items():
        if case.kv_type == O.KV_F16:
            continue
        outs, _ = S.run_checker(case, "ref")
        out[name + ".in_sha"] = np.array(G.inputs_digest(case))
        for s in range(case.n_seqs):
            for li in range(len(case.layers)):
                out[f"{name}.out.{s}.{li}"] = outs[s][li].astype(np.float32)
    for name in G.UNIT_CASES:
        out[f"unit.{name}"] = G.run_unit(name, "ref").astype(np.float32)
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")
    return 0


if __name__ == "__main__":
    sys.exit(main())
