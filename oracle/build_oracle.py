"""Build the CPU oracle (test infrastructure, never the product).

- oracle/_build/libkd_oracle.so : the C restatement in oracle/kd_oracle.c
- oracle/_ref/kd_ref_pin        : the reference's own RoPE/Philox code, compiled
                                  from the reference sources by oracle/ref_pin/Makefile
                                  (only where the reference tree exists).
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "libkd_oracle.so")
PIN = os.path.join(HERE, "_ref", "kd_ref_pin")
# The reference checkout: $KD_REFERENCE_DIR, else a sibling directory of this repository named
# "reference" (the layout in which the pin recipe is run); absent on machines without it.
REF_SIBLING = os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_oracle(force=False, verbose=False):
    src = os.path.join(HERE, "kd_oracle.c")
    hdr = os.path.join(HERE, "kd_oracle.h")
    if force or _stale(LIB, [src, hdr, __file__]):
        os.makedirs(os.path.dirname(LIB), exist_ok=True)
        cc = shutil.which("gcc") or "cc"
        cmd = [cc, "-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared",
               "-std=c11", "-Wall", "-Wno-unknown-pragmas", "-o", LIB + ".tmp", src, "-lm"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        os.replace(LIB + ".tmp", LIB)
    return LIB


def build_ref_pin(ref=None, verbose=False):
    """Compile oracle/_ref/kd_ref_pin when the reference tree is present; returns its path or None."""
    ref = ref or os.environ.get("KD_REFERENCE_DIR") or REF_SIBLING
    if not os.path.isfile(os.path.join(ref, "src", "rope.hpp")):
        return PIN if os.path.exists(PIN) else None
    subprocess.run(["make", "-s", "-C", os.path.join(HERE, "ref_pin"), f"REF={ref}"], check=True,
                   stdout=None if verbose else subprocess.DEVNULL)
    return PIN


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv, verbose=True))
    print(build_ref_pin(verbose=True))
