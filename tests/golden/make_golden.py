"""Regenerate tests/golden/*.npz from the CPU oracle.

Each block case is first cross-checked against the independent numpy restatement
(tests/numpy_ref.py): identical routing and outputs within the parity tolerance.
Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle"), os.path.dirname(HERE)]

import numpy as np  # noqa: E402

import oracle as O  # noqa: E402
import golden_cases as G  # noqa: E402
import numpy_ref as R  # noqa: E402
import mlx_rs_b200.synth as S  # noqa: E402
from parity import assert_close, metrics  # noqa: E402


def main():
    cases = G.make_all(O)
    for name, d in cases.items():
        if name.startswith("block_"):
            bw = G.block_from_dict(d)
            rout, ridx, rw = R.block_forward(bw, d["x"])
            assert np.array_equal(ridx, d["idx"]), name
            assert metrics(d["weights"], S.f32_to_bf16_bits(rw.astype(np.float32)))["max_ulp"] <= 1.0, name
            assert_close(d["out"], S.f32_to_bf16_bits(rout.astype(np.float32)), name)
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, **d)
        print(f"{path}: {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
