"""Route selection from held-out measurement reports (drop-in for projection_policy.py).

Pure CPU logic over the reference's report format: a report of kind
"streaming-projection" or "half-projection" promotes its custom configuration for
a shape only when every held-out case of that shape selected the same
configuration, came from at least two input seeds, passed the bitwise and
numerics checks, kept the A/A control within 1 % and showed a gain whose 95 %
interval lies above max(1 %, |A/A|). Otherwise the fastest vendor method that
was measured in every case is chosen. Compressed-projection reports never
promote a custom route here (projection_policy.py:9-62).
"""

from __future__ import annotations

import re
import statistics

VENDORS = ("torch_mm", "torch_mv", "cublas_mm", "cublas_mv", "cublas_packed_mm", "cublas_packed_mv")
_HALF_VENDORS = ("cublas_compute32", "cublas_packed_compute32", "torch_mm_out_fp32")
_HALF_CONFIG = re.compile(r"t(?:32|64|128|256)_v(?:2|8)")
_FP32_CONFIG = re.compile(r"(?:(?:tiny|warp)_t(?:32|64|128|256)_v(?:1|4)|(?:lossless|fp28)_t(?:32|64|128|256))")
_COMPRESSED_KINDS = ("compressed-projection", "compressed-projection-tuning", "compressed-projection-validation")


def _case_passes(case, half):
    checks = (case.get("bitwise_layout_check") and case.get("numerics_passed") and case.get("noise_gated_win")) \
        if half else (case.get("bitwise_round_trip") and case.get("accepted_custom_win"))
    if not checks:
        return False
    aa = case.get("aa_time_saved_pct", float("inf"))
    return abs(aa) <= 1 and case["candidate_gain_ci95_pct"][0] > max(1, abs(aa))


def choose(profile, shape, force_vendor=False, *, output_dtype=None):
    """Decision dict: backend ("custom" | "vendor"), config, reason,
    custom_win_validated, accepted_10pct_target."""
    kind = profile.get("kind")
    if kind in _COMPRESSED_KINDS:
        return compressed_vendor_fallback(profile, shape, output_dtype or "fp32")
    half = kind == "half-projection"
    if kind not in ("streaming-projection", "half-projection") or profile.get("status") != "complete" \
            or (half and profile.get("mode") != "validate"):
        raise ValueError("Use a completed held-out streaming validation report")
    cases = [case for case in profile["cases"] if tuple(case["shape_mnk"]) == tuple(shape)]
    if not cases:
        return {"backend": "vendor", "config": "cublas_compute32" if half else "torch_mm",
                "reason": "Shape has no held-out validation", "custom_win_validated": False,
                "accepted_10pct_target": False}
    selected = {case["selected"] for case in cases}
    if len(selected) != 1:
        raise ValueError("Validation changed the selected kernel between cases")
    config = selected.pop()
    if not (_HALF_CONFIG if half else _FP32_CONFIG).fullmatch(config):
        raise ValueError("Unrecognized custom configuration")
    seeds = {case["seed"] for case in cases}
    if len(seeds) >= 2 and all(_case_passes(case, half) for case in cases) and not force_vendor:
        return {"backend": "custom", "config": ("half_" + config) if half else config,
                "reason": "All held-out A/A and positive-gain checks passed", "custom_win_validated": True,
                "accepted_10pct_target": all(case["candidate_gain_ci95_pct"][0] > 10 for case in cases)}
    allowed = _HALF_VENDORS if half else VENDORS
    measured = [name for name in allowed if all(name in case["methods"] for case in cases)]
    vendor = min(measured, key=lambda name: statistics.median(case["methods"][name]["median_us"] for case in cases))
    return {"backend": "vendor", "config": vendor, "reason": "Custom candidate did not pass every held-out noise gate",
            "custom_win_validated": False, "accepted_10pct_target": False}


def compressed_vendor_fallback(profile, shape, output_dtype):
    """The vendor route for compressed-projection reports, with the reason."""
    if output_dtype not in ("bf16", "fp32"):
        raise ValueError("Compressed BF16 projections support BF16 or FP32 output")
    recorded = profile.get("bindings", {}).get("output_dtype", profile.get("output_dtype", output_dtype))
    if recorded != output_dtype:
        reason = "Profile output contract differs; use the current vendor for the requested output"
    elif any(tuple(case.get("shape_mnk", ())) == tuple(shape) and case.get("time_saved_pct") is not None
             and case["time_saved_pct"] < 0 for case in profile.get("cases", ())):
        reason = "Compressed kernel regressed on this shape; skip packing and use the current vendor"
    else:
        reason = "Custom dispatch requires the complete audited three-process held-out cohort"
    return {"backend": "vendor", "config": "torch_mm" if output_dtype == "bf16" else "torch_mm_out_fp32",
            "reason": reason, "requires_packing": False, "custom_win_validated": False,
            "accepted_10pct_target": False, "dispatch_overhead_validated": False}
