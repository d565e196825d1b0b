"""Generates tests/golden/head_ref_p5.npz from the reference's own binary64 head.

Run from the repository root where the reference checkout is available:
    make -C oracle REF=<reference checkout>     # builds oracle/_ref/libref_head.so
    python tests/golden/make_head_golden.py

Runs head_reference (src/head_reference.cpp:434-441) on
synthetic_head_weights(3) and head_test_features("random", 1) at the T01
640x640 profile and records, for the P5 level (4 Cross-Scan directions x 25
tokens): the Mamba block's FP32 parameters, its input tokens, the block
output with the residual ("p5.residual") and its scale, the downsampled map
that the level expands and the merged level output ("p5.merge").  The tests
(tests/test_block_oracle_ref.py on the CPU, tests/test_head_golden_gpu.py on
the GPU) read only this file.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
sys.path.insert(0, ROOT)

from oracle import ref_head as rh  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "head_ref_p5.npz")
WEIGHT_SEED, KIND, FEATURE_SEED, PROFILE, LEVEL = 3, "random", 1, "t01", "p5"


def main() -> None:
    assert rh.available(), "build oracle/_ref/libref_head.so first: make -C oracle REF=<reference checkout>"
    rh.run_head(WEIGHT_SEED, KIND, FEATURE_SEED, PROFILE)
    arrays = {f"w.{k}": v for k, v in rh.block_params(LEVEL).items()}
    arrays["tokens"] = rh.tensor(LEVEL + ".tokens")
    arrays["residual"], arrays["residual_sigma"] = rh.tensor(LEVEL + ".residual", want_sigma=True)
    arrays["downsample"] = rh.tensor(LEVEL + ".downsample")
    arrays["merge"], arrays["merge_sigma"] = rh.tensor(LEVEL + ".merge", want_sigma=True)
    arrays["meta"] = np.array([WEIGHT_SEED, FEATURE_SEED], np.int64)
    np.savez_compressed(OUT, **arrays)
    print("wrote", OUT, {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    main()
