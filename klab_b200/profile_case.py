"""A few launches of one benchmark projection case through the public API, for a
profiler to capture (e.g. `ncu -k regex:stream_gemv -s 2 -c 1 python -m
klab_b200.profile_case --shape c2`). Seeded synthetic weights and activations
with the configs' shapes and distributions; nothing is timed or checked here.

Shapes: c1 (BF16 4096x4096, M=1), gate (BF16 14336x4096, M=1), c2 / c2m4 / c2m16
(INT8 per row 14336x4096, M=1/4/16), c3 / c3m8 (E2M1 + FP16 scale per 32,
8192x8192, M=1/8), c4 (lossless-coded BF16 4096x4096, M=1); attn (decode
attention with the KV append, 32 query / 8 kv heads of 64, 4095 cached tokens of
a 4096-token cache).
"""

from __future__ import annotations

import argparse

import torch

from . import compressed_bf16 as cb
from . import fp4, int8_weights

SHAPES = ("c1", "gate", "c2", "c2m4", "c2m16", "c3", "c3m8", "c4", "attn")


def case(shape, device="cuda"):
    """A zero-argument callable running one projection of the named case."""
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(1)

    def normal(shape_, std=1.0):
        return torch.randn(shape_, generator=g, device=dev).mul_(std)

    if shape in ("c1", "gate"):
        n, k = (4096, 4096) if shape == "c1" else (14336, 4096)
        w = normal((n, k), 0.02).to(torch.bfloat16)
        x = normal((1, k)).to(torch.bfloat16)
        return lambda: cb.raw_linear(x, w, threads=128, vector=8, output_dtype="bf16")
    if shape == "c4":
        w = normal((4096, 4096), 0.02).to(torch.bfloat16)
        packed = cb.upload(cb.pack_bits(w.view(torch.int16).cpu().numpy().view("uint16")), dev)
        x = normal((1, 4096)).to(torch.bfloat16)
        return lambda: cb.fused_linear(x, packed, threads=128, vector=8, output_dtype="bf16")
    if shape in ("c3", "c3m8"):
        q = fp4.quantize_weights_f16(normal((8192, 8192), 0.02))
        x = normal((1 if shape == "c3" else 8, 8192)).to(torch.bfloat16)
        return lambda: q.linear(x, output_dtype=torch.bfloat16)
    if shape in ("c2", "c2m4", "c2m16"):
        q = int8_weights.quantize_weights_per_row(normal((14336, 4096), 0.02))
        x = normal(({"c2": 1, "c2m4": 4, "c2m16": 16}[shape], 4096)).to(torch.bfloat16)
        return lambda: int8_weights.fused_linear(x, q.codes, q.scales, output_dtype=torch.bfloat16)
    if shape == "attn":
        from .decode_attn import decode_attention

        kc, vc = normal((8, 4096, 64)).to(torch.bfloat16), normal((8, 4096, 64)).to(torch.bfloat16)
        q, kn, vn = (normal((n,)).to(torch.bfloat16) for n in (32 * 64, 8 * 64, 8 * 64))
        return lambda: decode_attention(q, kn, vn, kc, vc, 4095)
    raise ValueError(f"unknown shape {shape!r}; expected one of {SHAPES}")


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--shape", choices=SHAPES, default="c2")
    parser.add_argument("--iters", type=int, default=4)
    args = parser.parse_args(argv)
    fn = case(args.shape)
    for _ in range(args.iters):
        fn()
    torch.cuda.synchronize()
    print("ok", args.shape)


if __name__ == "__main__":
    main()
