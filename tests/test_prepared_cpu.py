"""Prepared-plan host logic without a GPU: the route policy reproduces the
reference projection_policy.choose decisions recorded in
tests/golden/reference_policy.json, and the prepared operators' Fake kernels
keep the reference schemas and logical checks."""

import json
from pathlib import Path

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "reference_policy.json").read_text())


@pytest.mark.parametrize("key", sorted(GOLDEN["decisions"]))
def test_policy_matches_reference_decisions(key):
    from klab_b200 import projection_policy as pp

    name, force = key.rsplit("__force", 1)
    report = GOLDEN["reports"][name]
    expected = GOLDEN["decisions"][key]
    try:
        got = pp.choose(report, (1, 4096, 4096), force_vendor=bool(int(force)),
                        output_dtype="bf16" if name == "compressed" else None)
    except ValueError as exc:
        got = {"error": str(exc)}
    assert got == expected


def test_prepared_op_schemas():
    import klab_b200.native_prepared  # noqa: F401
    import klab_b200.prepared_kernels  # noqa: F401

    schemas = {
        "prepared_bf16::raw_r2": "prepared_bf16::raw_r2(Tensor x, Tensor w, SymInt m, SymInt n, SymInt k, "
                                 "SymInt threads, SymInt vector, str output_dtype) -> Tensor",
        "klab_native_v1::raw": "klab_native_v1::raw(Tensor x, Tensor w, int plan, int m, int n, int k, "
                               "int threads, int vector, str output_dtype) -> Tensor",
        "klab_native_v1::_retire_plan": "klab_native_v1::_retire_plan(int plan) -> ()",
        "klab_native_v1::plan_info": "klab_native_v1::plan_info(int plan) -> str",
    }
    for name, schema in schemas.items():
        ns, op = name.split("::")
        got = str(getattr(getattr(torch.ops, ns), op).default._schema)
        assert got.replace("SymInt", "int") == schema.replace("SymInt", "int"), got


def test_prepared_fakes_check_contracts():
    import klab_b200.native_prepared  # noqa: F401
    import klab_b200.prepared_kernels  # noqa: F401

    with FakeTensorMode():
        x = torch.empty(2, 256, dtype=torch.bfloat16)
        w = torch.empty(64, 256, dtype=torch.bfloat16)
        y = torch.ops.prepared_bf16.raw_r2(x, w, 2, 64, 256, 128, 8, "fp32")
        assert y.shape == (2, 64) and y.dtype == torch.float32
        payload = torch.empty(64 * 4 * 96, dtype=torch.uint8)
        meta = torch.empty(64 * 4, dtype=torch.int32)
        y = torch.ops.prepared_bf16.coded_r2(x, payload, meta, 2, 64, 256, 128, 8, "bf16")
        assert y.dtype == torch.bfloat16
        y = torch.ops.klab_native_v1.coded(x, payload, meta, 7, 2, 64, 256, 128, 8, "bf16")
        assert y.shape == (2, 64)
        with pytest.raises(ValueError):
            torch.ops.prepared_bf16.raw_r2(x, w, 2, 64, 256, 96, 8, "fp32")          # threads
        with pytest.raises(ValueError):
            torch.ops.prepared_bf16.raw_r2(x, w, 3, 64, 256, 128, 8, "fp32")         # prepared M
        with pytest.raises(ValueError):
            torch.ops.prepared_bf16.coded_r2(x, payload[:10], meta, 2, 64, 256, 128, 8, "bf16")
        with pytest.raises(ValueError):
            torch.ops.klab_native_v1.raw(x, w, 1, 2, 64, 256, 128, 8, "fp16")       # output dtype


def test_register_plan_validates_image_before_device():
    import hashlib

    import klab_b200.native_prepared  # noqa: F401

    ops = torch.ops.klab_native_v1
    image = torch.frombuffer(bytearray(b"image"), dtype=torch.uint8)
    digest = hashlib.sha256(b"image").hexdigest()
    with pytest.raises(ValueError, match="SHA-256"):
        ops._register_plan(image, 0, 1, 64, 256, 128, 8, "raw", "bf16", "XYZ")
    with pytest.raises(ValueError, match="does not match"):
        ops._register_plan(image, 0, 1, 64, 256, 128, 8, "raw", "bf16", "0" * 64)
    with pytest.raises(ValueError, match="kind"):
        ops._register_plan(image, 0, 1, 64, 256, 128, 8, "half", "bf16", digest)
    with pytest.raises(ValueError):
        ops._register_plan(image, 0, 1, 64, 250, 128, 8, "raw", "bf16", digest)   # K % vector
    if not torch.cuda.is_available():
        with pytest.raises(ValueError, match="not available"):
            ops._register_plan(image, 0, 1, 64, 256, 128, 8, "raw", "bf16", digest)
    with pytest.raises(ValueError, match="Unknown"):
        ops.plan_info(123456)
