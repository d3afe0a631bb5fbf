"""Shape-specific prepared projections chosen once, outside the hot path
(drop-in for dynamic_projection.py:150-164 prepare_projection / PreparedProjection).

prepare_projection(w, tokens, profile, output_dtype):
* BF16 weights with BF16 output (or a compressed-projection report) ->
  prepared_bf16.PreparedBF16Projection;
* otherwise a PreparedProjection with FP32 output: without a report, the B200
  prepared plan for the weight dtype (FP32 weights: the FP32 projection; FP16/BF16:
  the half projection); with a held-out report (a dict or a JSON path in the
  reference's format), projection_policy.choose picks the route: lossless_* and
  fp28_* pack the weights losslessly, the other custom configurations use the
  plain plan, vendor configurations run through vendor_call (the operator
  kernel_lab::dynamic_vendor). kernel_lab::dynamic_tiny exposes the fixed-K FP32
  projection as an operator. The reference additionally
  checks its report against the hashes of its own source files and the GPU's
  UUID; those describe its validation runs and are not carried over.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from . import _native
from . import lossless_weights
from . import packed_fp32
from .kernel_lab import default_lab
from .prepared import PreparedPlan
from .projection_policy import choose
from .vendor import vendor_call

_WFMT = {torch.float32: _native.W_F32, torch.float16: _native.W_F16, torch.bfloat16: _native.W_BF16}


@torch.library.custom_op("kernel_lab::dynamic_vendor", mutates_args=(), device_types="cuda")
def dynamic_vendor(x: torch.Tensor, w: torch.Tensor, config: str) -> torch.Tensor:
    """x . W^T (FP32) through the vendor route `config` (dynamic_projection.py:47-55)."""
    return vendor_call(x, w, config)


@dynamic_vendor.register_fake
def _dynamic_vendor_fake(x, w, config):
    return x.new_empty((x.shape[0], w.shape[1] if "packed" in config else w.shape[0]), dtype=torch.float32)


@torch.library.custom_op("kernel_lab::dynamic_tiny", mutates_args=(), device_types="cuda")
def dynamic_tiny(x: torch.Tensor, w: torch.Tensor, threads: int, vector: int) -> torch.Tensor:
    """KernelLab.tiny_matmul as an operator (dynamic_projection.py:58-63): FP32 x . W^T for
    K in {64, ..., 1024}; threads / vector are validated launch hints."""
    with torch.cuda.device(x.device):
        return default_lab().tiny_matmul(x, w, threads, vector)


@dynamic_tiny.register_fake
def _dynamic_tiny_fake(x, w, threads, vector):
    return x.new_empty((x.shape[0], w.shape[0]))


def _load_profile(profile):
    if profile is None or isinstance(profile, dict):
        return profile
    return json.loads(Path(profile).read_text())


class PreparedProjection:
    def __init__(self, w, tokens=1, profile=None):
        if torch.cuda.is_current_stream_capturing():
            raise ValueError("Prepare weights before CUDA graph capture")
        if not isinstance(w, torch.Tensor) or w.device.type != "cuda" or not w.is_contiguous() or w.requires_grad \
                or w.dtype not in _WFMT:
            raise ValueError("Expected contiguous inference-only FP32, FP16, or BF16 CUDA weights")
        if w.ndim != 2 or min(w.shape) <= 0 or tokens <= 0:
            raise ValueError("Expected nonempty w[N,K] and positive tokens")
        self.dtype = w.dtype
        self.m, self.n, self.k = tokens, *w.shape
        data = _load_profile(profile)
        if data is not None:
            dtype_name = {torch.float32: "fp32", torch.float16: "fp16", torch.bfloat16: "bf16"}[w.dtype]
            if (w.dtype == torch.float32 and data.get("kind") != "streaming-projection") or \
                    (w.dtype != torch.float32 and (data.get("kind") != "half-projection"
                                                   or data.get("dtype") != dtype_name)):
                raise ValueError("Validation precision contract does not match the supplied weight dtype")
            self.plan = choose(data, (tokens, self.n, self.k))
        else:
            self.plan = {"backend": "custom", "config": "b200_stream_gemv", "reason": "No report: B200 prepared plan",
                         "custom_win_validated": False, "accepted_10pct_target": False}
        self.strategy = self.plan["config"]
        self.packed, self.w, self.native = None, w, None
        if self.plan["backend"] == "vendor":
            self.w = w.T.contiguous() if "packed" in self.strategy else w
            # vendor handles and workspaces exist before any later graph capture
            vendor_call(torch.zeros(tokens, self.k, device=w.device, dtype=w.dtype), self.w, self._vendor_config())
            return
        if self.strategy.startswith("lossless_") and w.dtype == torch.float32:
            self.packed = lossless_weights.pack_weights(w)
        elif self.strategy.startswith("fp28_") and w.dtype == torch.float32:
            self.packed = packed_fp32.pack_weights(w)
        else:
            self.native = PreparedPlan(_WFMT[w.dtype], w.dtype, torch.float32, tokens, self.n, self.k, w.device)
        self.linear(torch.zeros(tokens, self.k, device=w.device, dtype=w.dtype))

    def linear(self, x, out=None):
        if x.device != self.w.device or x.dtype != self.dtype or not x.is_contiguous() or x.requires_grad:
            raise ValueError("Expected contiguous inference-only input matching the prepared weight dtype/device")
        if x.ndim != 2 or tuple(x.shape) != (self.m, self.k):
            raise ValueError("Input shape differs; prepare a plan for this token count")
        if self.plan["backend"] == "vendor":
            config = self._vendor_config()
            return vendor_call(x, self.w, config, out) if out is not None else dynamic_vendor(x, self.w, config)
        if isinstance(self.packed, lossless_weights.LosslessWeights):
            return lossless_weights.fused_linear(x, self.packed, out=out)
        if isinstance(self.packed, packed_fp32.PackedFP32Weights):
            return packed_fp32.fused_linear(x, self.packed, out=out)
        return self.native.launch(x, self.w, out=out)

    def _vendor_config(self):
        """The report's vendor route when it names one of vendor_call's, else torch.mm."""
        from .vendor import CONFIGS

        return self.strategy if self.strategy in CONFIGS else ("torch_mm" if self.dtype == torch.float32
                                                                else "torch_mm_out_fp32")

    __call__ = linear


def prepare_projection(w, tokens=1, profile=None, *, output_dtype=torch.float32):
    """Weights must stay immutable; select (and pack) once, then call with x[tokens, K]."""
    if w.dtype == torch.bfloat16:
        data = _load_profile(profile)
        compressed = data is not None and data.get("kind") in (
            "compressed-projection", "compressed-projection-tuning", "compressed-projection-validation")
        if compressed or (output_dtype == torch.bfloat16 and profile is None):
            from .prepared_bf16 import PreparedBF16Projection

            return PreparedBF16Projection(w, tokens, data, output_dtype=output_dtype)
    if output_dtype != torch.float32:
        raise ValueError("Legacy projection profiles require FP32 output")
    return PreparedProjection(w, tokens, profile)
