"""Error of a kernel output beyond its own storage rounding — TEST INFRASTRUCTURE ONLY.

The attention tolerances (max-abs 2e-3 for bf16 / fp16 caches, 5e-3 for fp8 caches, against
an fp32 recomputation) bound the kernel's arithmetic.  The output tensor itself is bf16 or
fp16, whose grid spacing exceeds 2e-3 once |x| >= 0.5 (bf16 keeps 8 significant bits, so an
output in [0.5, 1) is rounded by up to 2**-9 = 1.95e-3).  A correctly computed output can
therefore sit up to half a unit in the last place (ulp) of its format away from the fp32
value with no arithmetic error at all.

``excess(got, want, bits)`` returns, per element, ``|got - want|`` minus half an ulp of the
output format at the larger of the two magnitudes: the part of the error that the output's
rounding cannot explain.  The parity tests require ``excess <= tolerance`` and report the
plain max-abs error beside it.
"""

from __future__ import annotations

import numpy as np

SIGNIFICANT_BITS = {"bfloat16": 8, "float16": 11, "float32": 24}


def half_ulp(mag: np.ndarray, bits: int) -> np.ndarray:
    """Half the spacing of a float format with ``bits`` significant bits at magnitude ``mag``
    (normal range): 2**(floor(log2 mag) - bits)."""
    mag = np.asarray(mag, np.float64)
    e = np.floor(np.log2(np.maximum(mag, np.finfo(np.float64).tiny)))
    return np.where(mag > 0, np.exp2(e - bits), 0.0)


def excess(got, want, bits: int = 8) -> np.ndarray:
    """``|got - want|`` beyond half an ulp of the output format (``bits`` significant bits:
    8 for bf16, 11 for fp16)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    mag = np.maximum(np.abs(got), np.abs(want))
    return np.abs(got - want) - half_ulp(mag, bits)


def report(got, want, bits: int = 8) -> dict:
    """Max-abs error and max excess over the output rounding, for messages and logs."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return {"max_abs": float(np.abs(got - want).max()) if got.size else 0.0,
            "max_excess": float(excess(got, want, bits).max()) if got.size else 0.0}
