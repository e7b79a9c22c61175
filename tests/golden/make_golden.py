"""Regenerates the golden fixtures of the reference's own device kernels
(src/kernels/darknet_kernels.hip, compiled for the host by oracle/build_oracle.py and run
through oracle/ref_emulate.cpp) on the gputest cases of tests/golden/cases.py:

  reference_gputest.json  SHA-256 of every output whose comparison class is exact/value
                          (bit patterns; -0.0 folded to +0.0 for the value class)
  reference_gputest.npz   the outputs whose class is tol (compared with a tolerance)

It needs the reference tree, so it runs in the development container:

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import cases  # noqa: E402

JSON_OUT = os.path.join(HERE, "reference_gputest.json")
NPZ_OUT = os.path.join(HERE, "reference_gputest.npz")


def digest(a: np.ndarray, value_class: bool) -> str:
    a = np.ascontiguousarray(a)
    if value_class and a.dtype == np.float32:
        a = a + np.float32(0.0)  # -0.0 + 0.0 == +0.0
    return hashlib.sha256(a.tobytes()).hexdigest()


def main():
    from oracle.oracle import Oracle, RefEmulation

    d = cases.inputs()
    ref = cases.run_reference_all(RefEmulation(), Oracle(), d)
    digests, arrays = {}, {}
    for k, v in sorted(ref.items()):
        cls = cases.comparison_class(k)
        if cls == "tol":
            arrays[k] = v
        else:
            digests[k] = {"class": cls, "dtype": str(v.dtype), "n": int(v.size), "sha256": digest(v, cls == "value")}
    with open(JSON_OUT, "w") as f:
        json.dump(digests, f, indent=1, sort_keys=True)
    np.savez_compressed(NPZ_OUT, **arrays)
    print(JSON_OUT, len(digests), "digests;", NPZ_OUT, os.path.getsize(NPZ_OUT), "bytes,", len(arrays), "arrays")


if __name__ == "__main__":
    main()
