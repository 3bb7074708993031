"""Shared helpers for the parity tests: seeded inputs, oracle runs and the north-star gates.

Gates: cosine >= 0.99995, max-abs error <= 2e-2 x output RMS,
softmax LSE within 1e-3 -- evaluated against the fp64 oracle on the same rounded operands.
Against the ggml-faithful oracle (f16 value accumulator for f16 V) cosine and LSE are
gated the same way, and the max-abs error may exceed the fp64 gate by no more than the
faithful oracle's own deviation from fp64 (triangle inequality).
"""
import numpy as np

import oracle

COS_MIN = 0.99995
MAXABS_REL = 2e-2
LSE_TOL = 1e-3


def seeded(shape, seed, offset):
    return oracle.philox_randn(seed, int(np.prod(shape)), offset).reshape(shape)


def lse_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    inf_g, inf_r = np.isneginf(got), np.isneginf(ref)
    assert np.array_equal(inf_g, inf_r), "fully-masked rows differ"
    fin = ~inf_r
    return float(np.max(np.abs(got[fin] - ref[fin]))) if fin.any() else 0.0


HALF_ULP_REL = {"bf16": 2.0 ** -8, "f16": 2.0 ** -11}


def assert_gates(got, exact, ggml=None, lse=None, lse_ref=None, label="", out_type=None):
    """out_type 'bf16' / 'f16': the output is stored in that format, so each element may also
    carry the format's rounding (half an ulp, <= |x| * 2^-8 for bf16, 2^-11 for f16) on top of
    the 2e-2 x RMS computation gate."""
    m = oracle.parity_metrics(got, exact)
    assert np.all(np.isfinite(got)), f"{label}: non-finite output"
    assert m["cos"] >= COS_MIN, f"{label}: cosine {m['cos']:.7f} vs fp64 oracle"
    if out_type is None:
        assert m["maxabs_over_rms"] <= MAXABS_REL, f"{label}: max-abs/RMS {m['maxabs_over_rms']:.3e} vs fp64 oracle"
    else:
        g = np.asarray(got, np.float64)
        r = np.asarray(exact, np.float64)
        excess = np.abs(g - r) - np.abs(r) * HALF_ULP_REL[out_type]
        worst = float(np.max(excess)) / (m["rms"] + 1e-300)
        assert worst <= MAXABS_REL, f"{label}: max-abs/RMS beyond {out_type} rounding {worst:.3e} vs fp64 oracle"
        m["maxabs_beyond_rounding_over_rms"] = worst
    out = {"exact": m}
    if ggml is not None:
        mg = oracle.parity_metrics(got, ggml)
        own = oracle.parity_metrics(ggml, exact)["maxabs"]
        assert mg["cos"] >= COS_MIN, f"{label}: cosine {mg['cos']:.7f} vs ggml-faithful oracle"
        assert mg["maxabs"] <= own + MAXABS_REL * m["rms"], \
            f"{label}: max-abs {mg['maxabs']:.3e} vs ggml-faithful oracle exceeds its own error {own:.3e} + gate"
        out["ggml"] = mg
    if lse is not None:
        e = lse_err(lse, lse_ref)
        assert e <= LSE_TOL, f"{label}: LSE error {e:.3e}"
        out["lse_err"] = e
    return out
