"""Regenerates tests/golden/block_local_L256_h3.npz from the reference tree.

The reference vendors Laya's ``block_local`` kernel golden at
``tests/data/kernels/block_local_L256/`` (tensors q, k, v, reference, kernel,
each [1, 16, 256, 64] fp32; block 128, Block3, seed 256; meta.json).  The GPU
box has no copy of the reference, so three heads (0, 7, 15; heads are
independent) are committed here, with the golden's meta fields that the tests
assert on.  Run from the repository root:

    python tests/golden/make_golden.py /path/to/raya
"""
import json
import os
import sys

import numpy as np
from safetensors.numpy import load_file

HEADS = [0, 7, 15]


def main(ref_root: str) -> None:
    src = os.path.join(ref_root, "tests", "data", "kernels", "block_local_L256")
    meta = json.load(open(os.path.join(src, "meta.json")))
    t = load_file(os.path.join(src, "tensors.safetensors"))
    out = {name: np.ascontiguousarray(t[name][0, HEADS]) for name in ("q", "k", "v", "reference", "kernel")}
    keep = {key: meta[key] for key in ("pattern", "scale", "block", "heads", "length", "head_dim",
                                       "tolerance", "max_abs_diff", "input_seed", "note")}
    keep["heads_kept"] = HEADS
    here = os.path.dirname(os.path.abspath(__file__))
    np.savez(os.path.join(here, "block_local_L256_h3.npz"), meta=json.dumps(keep), **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <root of the raya source tree>")
    main(sys.argv[1])
