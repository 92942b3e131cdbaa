"""Writes tests/golden/packers.npz: seeded fp32 weights (edge blocks
included) and their Q4_K / Q6_K bytes from tinygiant_b200.quants.

A regression fixture for the host packers that make the synthetic weights.
When it was written, the same bytes came from the packers' earlier C++ form,
and gguf-py's independent decoders read the layouts back
(tests/test_abi_cpu.py::test_packers_match_gguf_decoders).

    python tests/golden/make_packers.py
"""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from tinygiant_b200 import quants as Q  # noqa: E402


def weights():
    rng = np.random.default_rng([20261202, 5])
    w = (rng.standard_normal((24, 512)) * 0.02).astype(np.float32)
    w[0, :256] = 0.0                                  # all-zero block
    w[1, 256:] = np.abs(w[1, 256:])                   # all-positive block
    w[2, :32] = 1.0                                   # constant sub-block
    w[3, 16:48] = -2.5                                # constant straddling two sub-blocks
    w[4, :256] = -0.0                                 # negative zeros
    w[5, :64] = np.float32(1e-38)                     # subnormal-scale values
    w[6, 3] = np.float32(65504 * 70)                  # beyond the fp16 range
    w[7] = rng.integers(-3, 4, 512).astype(np.float32)   # ties in magnitude
    w[8, ::2] = -0.0
    w[9] *= 1e4
    w[10] *= 1e-6
    return w


def main():
    w = weights()
    np.savez_compressed(Path(__file__).with_name("packers.npz"), w=w, q4k=Q.pack_q4k(w), q6k=Q.pack_q6k(w))


if __name__ == "__main__":
    main()
