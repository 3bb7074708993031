"""Generate tests/golden/ref_pin.npz from the reference's own code.

Runs oracle/_ref/kd_ref_pin -- the reference's src/rng.hpp (PhiloxRNG) and
src/rope.hpp (get_freqs, compute_text_rope, compute_visual_rope) compiled from
the reference sources by oracle/ref_pin/Makefile -- and stores its outputs.
Needs the reference tree (oracle/build_oracle.py's default location, or
$KD_REFERENCE_DIR); the committed .npz is what the tests read, so they run
without it.

    python tests/golden/make_golden.py
"""
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.build_oracle import build_ref_pin  # noqa: E402

LAYOUT = [  # name, number of float32 values, in the order pin_main.cpp writes them
    ("philox_s42_off0", 4096),
    ("philox_s42_off1", 4096),
    ("philox_s1234567890abcdef_off0", 1000),
    ("freqs_16", 16),
    ("freqs_24", 24),
    ("text_rope_7x128", 7 * 128),
    ("visual_rope_3x4x5_s111", 60 * 128),
    ("visual_rope_3x4x5_s122", 60 * 128),
    ("visual_rope_5x16x16_s122_rows", 6 * 128),
    ("visual_rope_31x32x32_s111_rows", 4 * 128),
    ("visual_rope_3x4x5_a162424_s122", 60 * 64),
]
ROWS_5x16x16 = [0, 1, 17, 255, 256, 1279]
ROWS_31x32x32 = [0, 1023, 1024, 31743]


def main():
    pin = build_ref_pin(verbose=True)
    if pin is None:
        raise SystemExit("reference tree not found; cannot regenerate the pin vectors")
    raw = subprocess.run([pin], check=True, stdout=subprocess.PIPE).stdout
    vals = np.frombuffer(raw, dtype="<f4")
    assert vals.size == sum(n for _, n in LAYOUT), (vals.size, sum(n for _, n in LAYOUT))
    out, off = {}, 0
    for name, n in LAYOUT:
        out[name] = vals[off:off + n].copy()
        off += n
    out["rows_5x16x16"] = np.array(ROWS_5x16x16, dtype=np.int64)
    out["rows_31x32x32"] = np.array(ROWS_31x32x32, dtype=np.int64)
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_pin.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst, os.path.getsize(dst), "bytes")


if __name__ == "__main__":
    main()
