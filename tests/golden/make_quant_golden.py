"""Generate tests/golden/quant_pin.npz from the reference's own weight quantizers.

Imports quantize_q8_0 / quantize_q4_0 from the reference converter
(scripts/convert_to_gguf.py:90-146 of the reference tree, found at
$KD_REFERENCE_DIR or the sibling directory "reference" of this repository) and
stores, for seeded weights and hand-made edge blocks, the inputs and the exact
bytes it writes.  tests/test_oracle.py checks the oracle's restatement against
them; the committed .npz is what the tests read, so they run without the tree.

    python tests/golden/make_quant_golden.py
"""
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def reference_converter():
    ref = os.environ.get("KD_REFERENCE_DIR") or os.path.join(os.path.dirname(ROOT), "reference")
    path = os.path.join(ref, "scripts", "convert_to_gguf.py")
    if not os.path.isfile(path):
        raise SystemExit(f"{path} not found; cannot regenerate the quantizer pins")
    spec = importlib.util.spec_from_file_location("kd_ref_convert_to_gguf", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def edge_rows():
    """Blocks that exercise the rounding and sign rules: all zero, a single value, exact .5 ratios
    (round-half-even in q8_0), a negative extreme (q4_0's signed scale), ties of |max| with both signs."""
    z = np.zeros(32, np.float32)
    one = z.copy(); one[5] = 3.0
    half = (np.arange(32, dtype=np.float32) - 16) * np.float32(127.0 / 32.0)
    half[0] = 127.0                          # d = 1: x / d = k + 0.5 on the odd k/2 entries below
    half[1:9] = np.array([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5, -127.5], np.float32)
    neg = np.linspace(-4, 1, 32).astype(np.float32)
    tie = np.linspace(-2, 2, 32).astype(np.float32)
    tiny = (np.arange(32, dtype=np.float32) - 10) * np.float32(1e-8)
    return np.stack([np.concatenate([z, one]), np.concatenate([half, neg]), np.concatenate([tie, tiny])])


def main():
    conv = reference_converter()
    rng = np.random.default_rng(20260101)
    out = {}
    cases = {
        "rand": (rng.standard_normal((8, 256)) * 0.02).astype(np.float32),
        "heavy": (rng.standard_t(3, (4, 128))).astype(np.float32),
        "edge": edge_rows(),
    }
    for name, w in cases.items():
        out[f"{name}_w"] = w
        out[f"{name}_q8_0"] = np.frombuffer(conv.quantize_q8_0(w), np.uint8).reshape(w.shape[0], -1).copy()
        out[f"{name}_q4_0"] = np.frombuffer(conv.quantize_q4_0(w), np.uint8).reshape(w.shape[0], -1).copy()
    dst = os.path.join(HERE, "quant_pin.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst, os.path.getsize(dst), "bytes")


if __name__ == "__main__":
    sys.exit(main())
