"""Frozen cuBLASLt plan records checked without a GPU (the reference's
cublaslt_baseline.validate_frozen contract, cublaslt_baseline.py:117-165): a record
restores only into exactly the context it was frozen in, with a 64-byte algorithm."""

import base64
import copy

import pytest

from klab_b200.lt_baseline import CONTEXT_FIELDS, FORMAT, validate_frozen

CONTEXT = {"library_version": 120804, "device_uuid": "GPU-0000", "input_dtype": "bf16", "output_dtype": "bf16",
           "shape_mnk": [1, 4096, 4096]}
RECORD = {"format": FORMAT, **CONTEXT, "compute_type": 68, "workspace_bytes": 1 << 20,
          "algorithm_b64": base64.b64encode(bytes(range(64))).decode()}


def test_valid_record_returns_the_algorithm():
    assert validate_frozen(RECORD, CONTEXT) == bytes(range(64))
    ctx = dict(CONTEXT, shape_mnk=(1, 4096, 4096))   # tuple and list compare equal
    assert validate_frozen(RECORD, ctx) == bytes(range(64))


@pytest.mark.parametrize("field", CONTEXT_FIELDS)
def test_any_context_difference_is_rejected(field):
    other = {"library_version": 120900, "device_uuid": "GPU-1111", "input_dtype": "fp16", "output_dtype": "fp32",
             "shape_mnk": [2, 4096, 4096]}[field]
    with pytest.raises(ValueError, match=field):
        validate_frozen(RECORD, dict(CONTEXT, **{field: other}))


@pytest.mark.parametrize("change", [
    {"format": "cublaslt-plan-v1"}, {"compute_type": 77}, {"workspace_bytes": 1 << 40}, {"workspace_bytes": -1},
    {"algorithm_b64": "not base64!"}, {"algorithm_b64": base64.b64encode(b"x" * 63).decode()},
    {"shape_mnk": [0, 4096, 4096]}, {"shape_mnk": [1, 4096]}, {"input_dtype": "fp32", "output_dtype": "bf16"},
])
def test_malformed_records_are_rejected(change):
    bad = copy.deepcopy(RECORD)
    bad.update(change)
    with pytest.raises(ValueError):
        validate_frozen(bad, CONTEXT)


def test_missing_fields_are_rejected():
    for field in ("algorithm_b64", "device_uuid", "compute_type"):
        bad = {k: v for k, v in RECORD.items() if k != field}
        with pytest.raises(ValueError):
            validate_frozen(bad, CONTEXT)
