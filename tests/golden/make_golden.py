"""Generate golden fixtures for the oracle by running the reference's own code.

Run where the reference tree is available, with its path in KLAB_REFERENCE; the
GPU box and CI only read the committed fixture files:

    KLAB_REFERENCE=<reference checkout> python tests/golden/make_golden.py

What runs here is the reference's Python, unmodified:
  * compressed_bf16.pack_bits / unpack_bits, bf16_reference.decode_bf16
  * projection_accuracy.round_bf16_bits / check_outputs
  * mtile_bf16.tile_for_m
  * int8_weights.quantize_weights / Int8Weights.dequantize,
    fp4.quantize_weights / FP4Weights.dequantize,
    lossless_weights.pack_weights, packed_fp32.pack_weights,
    projection_policy.choose (decisions on synthetic held-out reports)
The quantizers and packers refuse non-CUDA tensors, and this container has no GPU.
They run on CPU tensors here through a shim: a Tensor subclass whose .device
reports "cuda" (so the device check passes) and a module-level torch proxy that
drops device= arguments of the factory calls. Every tensor operation is still
the reference's own torch call, on CPU, where float32 division, rounding and the
float8 conversion are the same IEEE operations as on the GPU. `kernel_lab` is
replaced by an empty module because its import creates cache directories in the
(read-only) reference tree; none of the functions used here touches it.
"""

from __future__ import annotations

import hashlib
import importlib.util
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REFERENCE = Path(os.environ["KLAB_REFERENCE"]) if os.environ.get("KLAB_REFERENCE") else None


def _load(name: str):
    spec = importlib.util.spec_from_file_location(name, REFERENCE / f"{name}.py")
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


class _CudaLooking(torch.Tensor):
    """CPU tensor that reports device type 'cuda' to the reference's input checks."""

    @property
    def device(self):  # noqa: D401 - property mirrors torch.Tensor.device
        return torch.device("cuda")


class _TorchProxy(types.ModuleType):
    """torch, except that factory functions ignore device= (everything stays on CPU)."""

    def __init__(self):
        super().__init__("torch_proxy")

    def __getattr__(self, name):
        value = getattr(torch, name)
        if name in ("tensor", "empty", "zeros", "ones", "arange", "full"):
            def factory(*args, _fn=value, **kwargs):
                kwargs.pop("device", None)
                return _fn(*args, **kwargs)
            return factory
        return value


def _plain(t):
    return t.as_subclass(torch.Tensor).detach().cpu().numpy()


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def codec_fixtures(cb, br):
    out = {}
    cases = {}
    cases["all_patterns"] = np.arange(65536, dtype=np.uint16).reshape(1024, 64)
    mixed = np.full((3, 129), 0xBF80, dtype=np.uint16)
    mixed[0, 64:128] = np.arange(64, dtype=np.uint16) << 7
    mixed[1, 0] = 0x7FC1
    mixed[2, 128] = 0x8000
    cases["mixed_tail"] = mixed
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((48, 320), dtype=np.float32) * np.float32(0.02))
    bits = ((w.view(np.uint32).astype(np.uint64) + 0x7FFF + ((w.view(np.uint32) >> 16) & 1)) >> 16).astype(np.uint16)
    bits[3, 5] = 0x0000
    bits[7, 64:128] = (np.arange(64, dtype=np.uint16) << 7)  # forces a raw block
    bits[9, 10] = 0x8001
    cases["normal_ragged"] = bits
    cases["coded_only"] = np.full((1, 64), 0x3F80, dtype=np.uint16)
    cases["raw_only"] = (np.arange(64, dtype=np.uint16) << 7).reshape(1, 64)
    for name, case in cases.items():
        packed = cb.pack_bits(case)
        decoded = br.decode_bf16(packed.payload.tobytes(), packed.metadata, packed.n, packed.k)
        assert np.array_equal(decoded, case) and np.array_equal(cb.unpack_bits(packed), case)
        out[f"{name}__bits"] = case
        out[f"{name}__metadata"] = packed.metadata
        out[f"{name}__payload_sha256"] = np.array(_sha(packed.payload))
        out[f"{name}__storage_bytes"] = np.array(packed.storage_bytes)
        out[f"{name}__source_sha256"] = np.array(packed.source_sha256)
        if packed.payload.nbytes <= 64 * 1024:
            out[f"{name}__payload"] = packed.payload
    return out


def rounding_fixtures(pa):
    values = np.array([0.0, -0.0, 1.0, 1.00390625, 1.00390625 - 1e-12, 1.00390625 + 1e-12, -1.00390625,
                       2.0 ** -133, -(2.0 ** -133), 2.0 ** -135, -(2.0 ** -134), 2.0 ** 128, -(2.0 ** 128),
                       3.3895313892515355e38, 3.4e38, 1e-40, -7.5e-39, 0.1, -0.3, 123.456, 65504.0,
                       1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8])
    rng = np.random.default_rng(5)
    values = np.concatenate([values, rng.standard_normal(2000) * np.exp2(rng.integers(-140, 120, 2000))])
    bits = pa.round_bf16_bits(values)
    checks = []
    ref = rng.standard_normal(64)
    for dtype, delta in (("fp32", 0.0), ("fp32", 2e-4), ("bf16", 0.0)):
        actual = ref + delta
        if dtype == "bf16":
            actual = (pa.round_bf16_bits(actual).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        report = pa.check_outputs(ref, actual, output_dtype=dtype)
        checks.append([report["passed"], report["violations"]])
    return {"round__values": values, "round__bits": bits, "check__ref": ref,
            "check__results": np.array(checks, dtype=np.int64)}


def quant_fixtures(i8, fp4, lw):
    out = {}
    for proxy_target in (i8, fp4, lw):
        proxy_target.torch = _TorchProxy()
    rng = np.random.default_rng(21)
    w = (rng.standard_normal((24, 256), dtype=np.float32) * np.float32(0.02))
    w[0, :64] = 0.0                                  # an all-zero group
    w[1, 3] = 1e-40                                  # subnormal
    w[2, :16] = np.float32(0.75) * w[2, 0]           # repeated values
    out["w"] = w
    q = i8.quantize_weights(torch.from_numpy(w.copy()).as_subclass(_CudaLooking))
    out["int8__codes"] = _plain(q.codes)
    out["int8__scales"] = _plain(q.scales)
    deq = i8.Int8Weights(torch.from_numpy(out["int8__codes"]), torch.from_numpy(out["int8__scales"]))
    out["int8__dequant"] = deq.dequantize().numpy()
    q = fp4.quantize_weights(torch.from_numpy(w.copy()).as_subclass(_CudaLooking))
    out["fp4__packed"] = _plain(q.packed)
    out["fp4__scales"] = _plain(q.scales)
    out["fp4__global"] = _plain(q.global_scale)
    deq = fp4.FP4Weights(torch.from_numpy(out["fp4__packed"]), torch.from_numpy(out["fp4__scales"]),
                         torch.from_numpy(out["fp4__global"]))
    out["fp4__dequant"] = deq.dequantize().numpy()
    # Values placed exactly on E2M1 ties relative to a scale of 1 (global 1/448/6 * ...).
    ties = np.zeros((2, 32), dtype=np.float32)
    ties[0, :16] = np.array([6, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5, -0.75, -1.75, -3.5, -5, 0.5, 1, 3, 4],
                            dtype=np.float32)
    ties[1, :16] = -ties[0, :16]
    ties[:, 16:] = ties[:, :16] * np.float32(0.5)
    out["ties"] = ties
    q = fp4.quantize_weights(torch.from_numpy(ties.copy()).as_subclass(_CudaLooking))
    out["ties__packed"] = _plain(q.packed)
    out["ties__scales"] = _plain(q.scales)
    out["ties__global"] = _plain(q.global_scale)
    zero = np.zeros((5, 64), dtype=np.float32)
    out["zero__int8_scales"] = _plain(i8.quantize_weights(torch.from_numpy(zero).as_subclass(_CudaLooking)).scales)
    zq = fp4.quantize_weights(torch.from_numpy(zero[:, :16].copy()).as_subclass(_CudaLooking))
    out["zero__fp4_packed"] = _plain(zq.packed)
    out["zero__fp4_global"] = _plain(zq.global_scale)
    lq = lw.pack_weights(torch.from_numpy(w.copy()).as_subclass(_CudaLooking))
    out["lossless__mantissa"] = _plain(lq.mantissa)
    out["lossless__exponents"] = _plain(lq.exponents)
    out["lossless__metadata"] = _plain(lq.metadata)
    return out


def lossless_cases():
    """FP32 matrices that exercise both block kinds of the lossless formats."""
    rng = np.random.default_rng(31)
    cases = {}
    w = rng.standard_normal((16, 192), dtype=np.float32) * np.float32(0.02)
    w[0, :64] = np.float32(1.5)                                 # one exponent: delta 0 everywhere
    w[1, 64:128] = np.float32(2.0) ** np.arange(-8, 8, 0.25, dtype=np.float32)[:64]  # deltas up to 15
    w[2, :4] = [np.float32(np.inf), -np.float32(np.inf), np.float32(np.nan), -0.0]  # wide: exponent 255 and 0
    w[3, 100] = np.float32(1e-40)                               # subnormal: exponent 0, wide block
    w[4, 130] = np.float32(3e38)                                # huge
    w[5, :] = 0.0                                               # all zero (narrow, base 0)
    w[6, :64] = -np.float32(7.25)
    cases["mixed"] = w
    cases["normal"] = rng.standard_normal((8, 512), dtype=np.float32)
    wide = rng.standard_normal((4, 128), dtype=np.float32) * np.exp2(rng.integers(-60, 60, (4, 128))).astype(np.float32)
    cases["wide"] = wide.astype(np.float32)
    return cases


def lossless_fixtures(lw, pf):
    """lossless_weights.pack_weights and packed_fp32.pack_weights, run as written."""
    out = {}
    for module in (lw, pf):
        module.torch = _TorchProxy()
    for name, w in lossless_cases().items():
        out[f"{name}__w"] = w
        lq = lw.pack_weights(torch.from_numpy(w.copy()).as_subclass(_CudaLooking))
        out[f"{name}__lf32_mantissa"] = _plain(lq.mantissa)
        out[f"{name}__lf32_exponents"] = _plain(lq.exponents)
        out[f"{name}__lf32_metadata"] = _plain(lq.metadata)
        pq = pf.pack_weights(torch.from_numpy(w.copy()).as_subclass(_CudaLooking))
        out[f"{name}__fp28_payload"] = _plain(pq.payload)
        out[f"{name}__fp28_metadata"] = _plain(pq.metadata)
    return out


def policy_reports():
    """Synthetic held-out reports in the reference's format: every branch of choose()."""
    def case(seed, selected="warp_t128_v4", gain=(12.0, 15.0), aa=0.4, ok=True, half=False, shape=(1, 4096, 4096)):
        c = {"shape_mnk": list(shape), "seed": seed, "selected": selected, "candidate_gain_ci95_pct": list(gain),
             "aa_time_saved_pct": aa,
             "methods": {"torch_mm": {"median_us": 30.0 + seed}, "cublas_mv": {"median_us": 25.0 + seed},
                         "cublas_compute32": {"median_us": 28.0}, "torch_mm_out_fp32": {"median_us": 27.0}}}
        if half:
            c.update(bitwise_layout_check=ok, numerics_passed=ok, noise_gated_win=ok)
        else:
            c.update(bitwise_round_trip=ok, accepted_custom_win=ok)
        return c

    base = {"kind": "streaming-projection", "status": "complete"}
    reports = {
        "custom_pass": dict(base, cases=[case(1), case(2)]),
        "custom_small_gain": dict(base, cases=[case(1, gain=(3.0, 5.0)), case(2, gain=(4.0, 6.0))]),
        "one_seed": dict(base, cases=[case(1), case(1)]),
        "noisy_aa": dict(base, cases=[case(1, aa=2.5), case(2)]),
        "failed_check": dict(base, cases=[case(1, ok=False), case(2)]),
        "lossless": dict(base, cases=[case(1, selected="lossless_t128"), case(2, selected="lossless_t128")]),
        "other_shape": dict(base, cases=[case(1, shape=(2, 64, 64))]),
        "half_pass": {"kind": "half-projection", "status": "complete", "mode": "validate", "dtype": "bf16",
                      "cases": [case(1, "t128_v8", half=True), case(2, "t128_v8", half=True)]},
        "compressed": {"kind": "compressed-projection", "output_dtype": "bf16",
                       "cases": [{"shape_mnk": [1, 4096, 4096], "time_saved_pct": -3.0}]},
        "compressed_ok": {"kind": "compressed-projection-validation", "output_dtype": "fp32", "cases": []},
    }
    return reports


def policy_fixtures(pp):
    out = {"reports": policy_reports(), "decisions": {}}
    for name, report in out["reports"].items():
        for force in (False, True):
            try:
                decision = pp.choose(report, (1, 4096, 4096), force_vendor=force,
                                     output_dtype="bf16" if name == "compressed" else None)
            except ValueError as exc:
                decision = {"error": str(exc)}
            out["decisions"][f"{name}__force{int(force)}"] = decision
    for name, report in (("bad_selected", {"kind": "streaming-projection", "status": "complete",
                                           "cases": [{"shape_mnk": [1, 4096, 4096], "seed": 1, "selected": "a"},
                                                     {"shape_mnk": [1, 4096, 4096], "seed": 2, "selected": "b"}]}),
                         ("bad_config", {"kind": "streaming-projection", "status": "complete",
                                         "cases": [{"shape_mnk": [1, 4096, 4096], "seed": 1, "selected": "zz"}]}),
                         ("incomplete", {"kind": "streaming-projection", "status": "running", "cases": []})):
        out["reports"][name] = report
        try:
            decision = pp.choose(report, (1, 4096, 4096))
        except ValueError as exc:
            decision = {"error": str(exc)}
        out["decisions"][f"{name}__force0"] = decision
    return out


def main():
    if REFERENCE is None or not REFERENCE.is_dir():
        raise SystemExit(f"set KLAB_REFERENCE to the reference tree (got {REFERENCE})")
    sys.path.insert(0, str(REFERENCE))
    sys.modules["kernel_lab"] = types.ModuleType("kernel_lab")
    cb = _load("compressed_bf16")
    br = _load("bf16_reference")
    pa = _load("projection_accuracy")
    mt = _load("mtile_bf16")
    i8 = _load("int8_weights")
    fp4 = _load("fp4")
    lw = _load("lossless_weights")
    pf = _load("packed_fp32")
    pp = _load("projection_policy")

    fixtures = {}
    fixtures.update(codec_fixtures(cb, br))
    fixtures.update(rounding_fixtures(pa))
    ms = np.array([1, 2, 3, 4, 5, 7, 8, 9, 15, 16, 17, 64, 65535])
    fixtures["tile__m"] = ms
    fixtures["tile__tile"] = np.array([mt.tile_for_m(int(m)) for m in ms])
    fixtures["tile__kernel_count"] = np.array(len(mt.kernel_names()))
    np.savez_compressed(HERE / "reference_codec.npz", **fixtures)
    np.savez_compressed(HERE / "reference_quant.npz", **quant_fixtures(i8, fp4, lw))
    np.savez_compressed(HERE / "reference_lossless.npz", **lossless_fixtures(lw, pf))
    import json

    (HERE / "reference_policy.json").write_text(json.dumps(policy_fixtures(pp), indent=1, sort_keys=True) + "\n")
    for name in ("reference_codec.npz", "reference_quant.npz", "reference_lossless.npz", "reference_policy.json"):
        print(name, (HERE / name).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
