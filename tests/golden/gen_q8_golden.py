"""Generate tests/golden/q8_0_golden.npz: float blocks and their Q8_0 encoding by gguf-py.

gguf-py's Q8_0 quantizer (gguf.quants.Q8_0.quantize_blocks) documents bit-exactness with ggml's
reference quantize_row_q8_0 (ggml-quants.c), the activation quantizer of the reference's Q8_0
mul_mat. The fixture pins the oracle's (and the GPU's) activation quantization.
Run from the repository root: python tests/golden/gen_q8_golden.py
"""
import os

import gguf
import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    rng = np.random.default_rng(7)
    x = rng.standard_normal((64, 32)).astype(np.float32) * rng.choice([1e-4, 0.02, 1.0, 30.0], (64, 1)).astype(np.float32)
    x[0] = 0.0                                   # d = 0
    x[1] = np.arange(32, dtype=np.float32) - 15.5   # ties at .5 after scaling
    x[2] = np.float32(127.0) * np.sign(rng.standard_normal(32)).astype(np.float32)
    x[3, 5] = -1e-30                             # tiny / denormal-range values
    blocks = gguf.quants.quantize(x, gguf.GGMLQuantizationType.Q8_0)
    out = os.path.join(ROOT, "tests", "golden", "q8_0_golden.npz")
    np.savez_compressed(out, x=x, blocks=np.asarray(blocks, np.uint8))
    print("wrote", out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
